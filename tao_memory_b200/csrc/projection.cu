// Model-side neighbour of the operator: the split of a fused Q/K/V projection into
// the five operands and the RMS normalisation of the exact-local q and k (reference
// examples/common.py:6-20: projected = x W^T reshaped [.., 3, H, D] -> raw_q, raw_k,
// v; q = rms_norm(raw_q), k = rms_norm(raw_k) over the width), forward and backward,
// one warp per (token, head).  The projection GEMM itself is the caller's (cuBLAS).
// HBM-bound: 3 H D bf16 read and 5 H D written per token forward.
#include <cuda_runtime.h>

#include "../../include/tao_b200.h"
#include "common.cuh"

void tao_set_last_error(const char* msg);

namespace tao {
namespace {

// Lane l holds channels [l * D/32, (l+1) * D/32) of a head row (D/32 = 2 or 4).
template <int D>
struct Slice {
  static constexpr int N = D / 32;
  float x[N];
  TAO_DEVI void load(const bf16* row, int lane) {
    if constexpr (N == 2) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(row + 2 * lane);
      x[0] = lo_f(w);
      x[1] = hi_f(w);
    } else {
      const uint2 w = *reinterpret_cast<const uint2*>(row + 4 * lane);
      x[0] = lo_f(w.x);
      x[1] = hi_f(w.x);
      x[2] = lo_f(w.y);
      x[3] = hi_f(w.y);
    }
  }
  TAO_DEVI void store(bf16* row, int lane) const {
    if constexpr (N == 2) {
      *reinterpret_cast<uint32_t*>(row + 2 * lane) = pack2(x[0], x[1]);
    } else {
      *reinterpret_cast<uint2*>(row + 4 * lane) = make_uint2(pack2(x[0], x[1]), pack2(x[2], x[3]));
    }
  }
  static TAO_DEVI uint32_t pack2(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  TAO_DEVI float sumsq() const {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) s += x[i] * x[i];
    return warp_sum(s);
  }
};

template <int D>
__global__ void __launch_bounds__(256) qkv_split_norm_kernel(const bf16* __restrict__ proj, long long rows, int H,
                                                             float eps, bf16* q, bf16* k, bf16* v, bf16* raw_q,
                                                             bf16* raw_k) {
  const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= rows * H) return;
  const long long r = w / H;
  const int h = (int)(w % H);
  const bf16* src = proj + r * 3 * H * D + (long long)h * D;
  const long long dst = (r * H + h) * D;
  Slice<D> rq, rk, vv;
  rq.load(src, lane);
  rk.load(src + (long long)H * D, lane);
  vv.load(src + 2LL * H * D, lane);
  rq.store(raw_q + dst, lane);
  rk.store(raw_k + dst, lane);
  vv.store(v + dst, lane);
  const float sq = rsqrtf(rq.sumsq() / D + eps), sk = rsqrtf(rk.sumsq() / D + eps);
#pragma unroll
  for (int i = 0; i < Slice<D>::N; ++i) {
    rq.x[i] *= sq;
    rk.x[i] *= sk;
  }
  rq.store(q + dst, lane);
  rk.store(k + dst, lane);
}

// d_proj = [d_raw_q + bf16(dx_q), d_raw_k + bf16(dx_k), dv] with the RMS-norm adjoint
// dx = r dy - x r^3 (sum_j x_j dy_j) / D, r = (sum x^2 / D + eps)^(-1/2), in fp32.
template <int D>
__global__ void __launch_bounds__(256) qkv_split_norm_bwd_kernel(const bf16* __restrict__ raw_q,
                                                                 const bf16* __restrict__ raw_k,
                                                                 const bf16* __restrict__ dq,
                                                                 const bf16* __restrict__ dk,
                                                                 const bf16* __restrict__ dv,
                                                                 const bf16* __restrict__ d_raw_q,
                                                                 const bf16* __restrict__ d_raw_k, long long rows,
                                                                 int H, float eps, bf16* d_proj) {
  const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= rows * H) return;
  const long long r = w / H;
  const int h = (int)(w % H);
  const long long src = (r * H + h) * D;
  bf16* dst = d_proj + r * 3 * H * D + (long long)h * D;
  const bf16* xs[2] = {raw_q + src, raw_k + src};
  const bf16* dys[2] = {dq + src, dk + src};
  const bf16* dds[2] = {d_raw_q + src, d_raw_k + src};
#pragma unroll
  for (int part = 0; part < 2; ++part) {
    Slice<D> x, dy, dd;
    x.load(xs[part], lane);
    dy.load(dys[part], lane);
    dd.load(dds[part], lane);
    const float rs = rsqrtf(x.sumsq() / D + eps);
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < Slice<D>::N; ++i) dot += x.x[i] * dy.x[i];
    dot = warp_sum(dot);
    const float c = rs * rs * rs * dot / D;
#pragma unroll
    for (int i = 0; i < Slice<D>::N; ++i) dd.x[i] = dd.x[i] + rb(rs * dy.x[i] - x.x[i] * c);
    dd.store(dst + (long long)part * H * D, lane);
  }
  Slice<D> g;
  g.load(dv + src, lane);
  g.store(dst + 2LL * H * D, lane);
}

int pfail(int code, const char* msg) {
  tao_set_last_error(msg);
  return code;
}

}  // namespace
}  // namespace tao

extern "C" {

int tao_qkv_split_norm(const void* projected, long long rows, int heads, int width, float eps, void* q, void* k,
                       void* v, void* raw_q, void* raw_k, void* stream) {
  using namespace tao;
  if (!projected || !q || !k || !v || !raw_q || !raw_k) return pfail(TAO_ERR_ARG, "null pointer");
  if (width != 64 && width != 128) return pfail(TAO_ERR_ARG, "head width must be 64 or 128");
  if (rows <= 0 || heads <= 0) return pfail(TAO_ERR_ARG, "rows and heads must be positive");
  const long long warps = rows * heads;
  const unsigned grid = (unsigned)((warps + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto P = [](const void* p) { return static_cast<const bf16*>(p); };
  auto W = [](void* p) { return static_cast<bf16*>(p); };
  if (width == 64)
    qkv_split_norm_kernel<64><<<grid, 256, 0, s>>>(P(projected), rows, heads, eps, W(q), W(k), W(v), W(raw_q),
                                                   W(raw_k));
  else
    qkv_split_norm_kernel<128><<<grid, 256, 0, s>>>(P(projected), rows, heads, eps, W(q), W(k), W(v), W(raw_q),
                                                    W(raw_k));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TAO_OK : pfail(TAO_ERR_CUDA, cudaGetErrorString(e));
}

int tao_qkv_split_norm_backward(const void* raw_q, const void* raw_k, const void* dq, const void* dk,
                                const void* dv, const void* d_raw_q, const void* d_raw_k, long long rows, int heads,
                                int width, float eps, void* d_projected, void* stream) {
  using namespace tao;
  if (!raw_q || !raw_k || !dq || !dk || !dv || !d_raw_q || !d_raw_k || !d_projected)
    return pfail(TAO_ERR_ARG, "null pointer");
  if (width != 64 && width != 128) return pfail(TAO_ERR_ARG, "head width must be 64 or 128");
  if (rows <= 0 || heads <= 0) return pfail(TAO_ERR_ARG, "rows and heads must be positive");
  const long long warps = rows * heads;
  const unsigned grid = (unsigned)((warps + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto P = [](const void* p) { return static_cast<const bf16*>(p); };
  if (width == 64)
    qkv_split_norm_bwd_kernel<64><<<grid, 256, 0, s>>>(P(raw_q), P(raw_k), P(dq), P(dk), P(dv), P(d_raw_q),
                                                       P(d_raw_k), rows, heads, eps, static_cast<bf16*>(d_projected));
  else
    qkv_split_norm_bwd_kernel<128><<<grid, 256, 0, s>>>(P(raw_q), P(raw_k), P(dq), P(dk), P(dv), P(d_raw_q),
                                                        P(d_raw_k), rows, heads, eps,
                                                        static_cast<bf16*>(d_projected));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TAO_OK : pfail(TAO_ERR_CUDA, cudaGetErrorString(e));
}

}  // extern "C"
