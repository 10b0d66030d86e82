// Sufficient statistics of the association fine writers on the tensor cores.
//
// Reference: association_statistics (association_writer.py:11-18), called by the
// seal of a 256-token block when TaoConfig.fine_writer is "regularized_association"
// or "feature_mass_association" (tao_stream.py:62-65, 72-74):
//   u = bf16(softmax over channels of k[t])   (fp32 softmax, one rounding)
//   G = u^T u,  X = u^T v                       (fp32 products and sums)
//   mass = sum_t u[t]                           (fp32, feature-mass writer only)
// u and v are bf16 values, so every product is exact in fp32 and the bf16 tensor-
// core MMA with fp32 accumulation computes the same sums as the reference's fp32
// matmul, up to summation order.
//
// One CTA (128 threads) per (block, head): the 256x D key and value tiles are
// staged in shared memory, u replaces the keys in place, then warp w computes rows
// [w*D/4, (w+1)*D/4) of G and of X with mma.sync.
#pragma once
#include "common.cuh"
#include "window_attention.cuh"

namespace tao {

template <int D>
__global__ void __launch_bounds__(128) writer_stats_kernel(const bf16* __restrict__ k, const bf16* __restrict__ v,
                                                           long long token_stride, long long head_stride,
                                                           long long block_stride, int heads, float* gram,
                                                           float* cross, float* mass) {
  using namespace wa;
  constexpr int NT = 256, CH = D / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sU = smem_u32(smem);   // [256][D] keys, then u
  const uint32_t sV = sU + NT * D * 2;  // [256][D]
  const int blk = blockIdx.x / heads, h = blockIdx.x % heads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bf16* kb = k + blk * block_stride + h * head_stride;
  const bf16* vb = v + blk * block_stride + h * head_stride;
  for (int idx = tid; idx < NT * CH; idx += 128) {
    const int r = idx / CH, c = idx % CH;
    cp_async16(sU + swz(r, c * 8, D), kb + r * token_stride + c * 8, true);
    cp_async16(sV + swz(r, c * 8, D), vb + r * token_stride + c * 8, true);
  }
  cp_commit();
  cp_wait<0>();
  __syncthreads();
  // u = bf16(softmax_d(k[t])): two tokens per thread
  for (int t = tid; t < NT; t += 128) {
    float x[D];
#pragma unroll
    for (int c = 0; c < CH; ++c) unpack8(*reinterpret_cast<const uint4*>(smem + swz(t, c * 8, D)), x + c * 8);
    float m = x[0];
#pragma unroll
    for (int d = 1; d < D; ++d) m = fmaxf(m, x[d]);
    float sum = 0.f;
#pragma unroll
    for (int d = 0; d < D; ++d) {
      x[d] = expf(x[d] - m);
      sum += x[d];
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      uint4 o;
      o.x = pack_bf16(__fdiv_rn(x[c * 8 + 0], sum), __fdiv_rn(x[c * 8 + 1], sum));
      o.y = pack_bf16(__fdiv_rn(x[c * 8 + 2], sum), __fdiv_rn(x[c * 8 + 3], sum));
      o.z = pack_bf16(__fdiv_rn(x[c * 8 + 4], sum), __fdiv_rn(x[c * 8 + 5], sum));
      o.w = pack_bf16(__fdiv_rn(x[c * 8 + 6], sum), __fdiv_rn(x[c * 8 + 7], sum));
      *reinterpret_cast<uint4*>(smem + swz(t, c * 8, D)) = o;
    }
  }
  __syncthreads();
  // feature mass (feature-mass writer, tao_stream.py:62-65): sum_t u[t][d] in fp32
  if (mass != nullptr) {
    for (int d = tid; d < D; d += 128) {
      float m = 0.f;
      for (int t = 0; t < NT; ++t) m += bf(*reinterpret_cast<const bf16*>(smem + swz(t, d, D)));
      mass[((long long)blk * heads + h) * D + d] = m;
    }
  }
  // G[d][e] = sum_t u[t][d] u[t][e], X[d][e] = sum_t u[t][d] v[t][e]
  constexpr int MT = D / 64;  // m-tiles of 16 rows per warp
  constexpr int NTL = D / 8;
  const int g = lane >> 2, c4 = lane & 3;
  for (int which = 0; which < 2; ++which) {
    const uint32_t sB = which == 0 ? sU : sV;
    float acc[MT][NTL][4];
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int j = 0; j < NTL; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.f;
    for (int kt = 0; kt < NT / 16; ++kt) {
      uint32_t a[MT][4];
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        const int d0 = warp * (D / 4) + i * 16;
        const int r = kt * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
        const int c = d0 + ((lane >> 3) & 1) * 8;
        ldsm_x4_t(sU + swz(r, c, D), a[i][0], a[i][1], a[i][2], a[i][3]);
      }
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = np * 16 + (lane >> 4) * 8;
        ldsm_x4_t(sB + swz(r, c, D), b0, b1, b2, b3);
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          mma16816(acc[i][2 * np], a[i], b0, b1);
          mma16816(acc[i][2 * np + 1], a[i], b2, b3);
        }
      }
    }
    float* out = (which == 0 ? gram : cross) + ((long long)blk * heads + h) * D * D;
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      const int d0 = warp * (D / 4) + i * 16;
#pragma unroll
      for (int j = 0; j < NTL; ++j) {
        const int e = j * 8 + c4 * 2;
        *reinterpret_cast<float2*>(out + (long long)(d0 + g) * D + e) = make_float2(acc[i][j][0], acc[i][j][1]);
        *reinterpret_cast<float2*>(out + (long long)(d0 + g + 8) * D + e) = make_float2(acc[i][j][2], acc[i][j][3]);
      }
    }
  }
}

}  // namespace tao
