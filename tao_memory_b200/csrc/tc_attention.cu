// Host side of the tcgen05 windowed attention: TMA tensor maps and the launch,
// plus the dispatcher that picks it or the mma.sync kernel.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/tao_b200.h"
#include "tc_attention.cuh"
#include "tc_attention_bwd.cuh"
#include "window_attention.cuh"

void tao_set_last_error(const char* msg);

namespace {

int g_attention_variant = 1;  // 1: tcgen05 where the shape allows it, 0: mma.sync only

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q{};
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// [rows][cols] bf16 row-major, boxes of 128 rows x 64 columns (128 B), 128B swizzle.
bool row_map(CUtensorMap* map, const void* base, unsigned long long rows, unsigned long long cols) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [rows][cols] fp32 row-major, boxes of 32 rows x 32 columns (128 B), 128B swizzle.
bool f32_map(CUtensorMap* map, const void* base, unsigned long long rows, unsigned long long cols) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename F>
bool smem_attr(F* fn, size_t bytes) {
  return bytes <= 48 * 1024 ||
         cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess;
}

bool aligned(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace tao {

// Windowed causal attention over contiguous [B][T][H][D] operands (training and
// tao_window_attention).  Returns TAO_OK or a status (message recorded).
int launch_window_attention(const bf16* q, const bf16* k, const bf16* v, bf16* out, float* lse, int B,
                            int T, int H, int D, int* err, cudaStream_t s) {
  const bool tc = g_attention_variant == 1 && (D == 64 || D == 128) && aligned(q) && aligned(k) && aligned(v);
  if (tc) {
    CUtensorMap mq, mk, mv;
    const unsigned long long rows = (unsigned long long)B * T, cols = (unsigned long long)H * D;
    if (!row_map(&mq, q, rows, cols) || !row_map(&mk, k, rows, cols) || !row_map(&mv, v, rows, cols)) {
      tao_set_last_error("cuTensorMapEncodeTiled failed");
      return TAO_ERR_CUDA;
    }
    const dim3 grid((T + tc::kTcBM - 1) / tc::kTcBM, B * H);
    if (D == 64) {
      if (!smem_attr(tc_window_attention_kernel<64>, tc::TcAttnCfg<64>::SMEM)) {
        tao_set_last_error("smem attribute");
        return TAO_ERR_CUDA;
      }
      tc_window_attention_kernel<64><<<grid, tc::kTcThreads, tc::TcAttnCfg<64>::SMEM, s>>>(mq, mk, mv, out, lse, T, H,
                                                                                          err, tc::TcRing{});
    } else {
      if (!smem_attr(tc_window_attention_kernel<128>, tc::TcAttnCfg<128>::SMEM)) {
        tao_set_last_error("smem attribute");
        return TAO_ERR_CUDA;
      }
      tc_window_attention_kernel<128><<<grid, tc::kTcThreads, tc::TcAttnCfg<128>::SMEM, s>>>(mq, mk, mv, out, lse, T,
                                                                                            H, err, tc::TcRing{});
    }
    return TAO_OK;
  }
  WinAttnParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.out = out;
  p.lse = lse;
  p.q_batch_stride = p.k_batch_stride = p.o_batch_stride = (long long)T * H * D;
  p.q_row_stride = p.k_row_stride = p.o_row_stride = (long long)H * D;
  p.k_head_stride = D;
  p.heads = H;
  p.nq = T;
  p.qpos0 = 0;
  p.kstart = -1;
  const dim3 grid((T + 63) / 64, B * H);
  if (D == 64) {
    const size_t smem = (size_t)(64 + 4 * 64) * 64 * 2;
    if (!smem_attr(window_attention_kernel<64>, smem)) {
      tao_set_last_error("smem attribute");
      return TAO_ERR_CUDA;
    }
    window_attention_kernel<64><<<grid, 128, smem, s>>>(p);
  } else {
    const size_t smem = (size_t)(64 + 4 * 64) * 128 * 2;
    if (!smem_attr(window_attention_kernel<128>, smem)) {
      tao_set_last_error("smem attribute");
      return TAO_ERR_CUDA;
    }
    window_attention_kernel<128><<<grid, 128, smem, s>>>(p);
  }
  return TAO_OK;
}

int attention_variant() { return g_attention_variant; }

// Attention of a streaming chunk (w queries of each of R states, at their cursors)
// over each state's ring on the tensor cores: q and out [R][w][H][D].  Returns
// TAO_ERR_ARG (nothing launched) for widths other than 64 and 128.
int launch_ring_attention(TaoState* const* states, const bf16* q, bf16* out, int R, int w, int H, int D, int* err,
                          cudaStream_t s) {
  const CUtensorMap none{};
  const dim3 grid((w + tc::kTcBM - 1) / tc::kTcBM, R * H);
  const tc::TcRing ring{states, q, w};
  if (D == 64) {
    if (!smem_attr(tc_window_attention_kernel<64, true>, tc::TcAttnCfg<64>::SMEM)) {
      tao_set_last_error("smem attribute");
      return TAO_ERR_CUDA;
    }
    tc_window_attention_kernel<64, true><<<grid, tc::kTcThreads, tc::TcAttnCfg<64>::SMEM, s>>>(none, none, none, out,
                                                                                               nullptr, 0, H, err, ring);
  } else if (D == 128) {
    if (!smem_attr(tc_window_attention_kernel<128, true>, tc::TcAttnCfg<128>::SMEM)) {
      tao_set_last_error("smem attribute");
      return TAO_ERR_CUDA;
    }
    tc_window_attention_kernel<128, true><<<grid, tc::kTcThreads, tc::TcAttnCfg<128>::SMEM, s>>>(
        none, none, none, out, nullptr, 0, H, err, ring);
  } else {
    tao_set_last_error("ring attention on the tensor cores takes widths 64 and 128");
    return TAO_ERR_ARG;
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    tao_set_last_error(cudaGetErrorString(e));
    return TAO_ERR_CUDA;
  }
  return TAO_OK;
}

// Windowed attention backward on the tensor cores (widths 64 and 128): dK, dV and dQ
// of contiguous [B][T][H][D] operands.  dq_acc is fp32 scratch of the same shape.  At
// width 128 each key block runs as two CTAs, one per half of the gradient channels.
int launch_attention_backward_tc(const bf16* q, const bf16* k, const bf16* v, const bf16* dout, const float* lse,
                                 const float* rowdot, bf16* dq, bf16* dk, bf16* dv, float* dq_acc, int B, int T,
                                 int H, int D, int* err, cudaStream_t s) {
  if (D != 64 && D != 128) {
    tao_set_last_error("attention backward on the tensor cores takes widths 64 and 128");
    return TAO_ERR_ARG;
  }
  for (const void* p : {(const void*)q, (const void*)k, (const void*)v, (const void*)dout, (const void*)dq_acc})
    if (!aligned(p)) {
      tao_set_last_error("attention backward operands must be 16-byte aligned");
      return TAO_ERR_ARG;
    }
  CUtensorMap mq, mk, mv, mo, mdq;
  const unsigned long long rows = (unsigned long long)B * T, cols = (unsigned long long)H * D;
  if (!row_map(&mq, q, rows, cols) || !row_map(&mk, k, rows, cols) || !row_map(&mv, v, rows, cols) ||
      !row_map(&mo, dout, rows, cols) || !f32_map(&mdq, dq_acc, rows, cols)) {
    tao_set_last_error("cuTensorMapEncodeTiled failed");
    return TAO_ERR_CUDA;
  }
  const bool attr = D == 64 ? smem_attr(tc_attention_bwd_kernel<64>, tb::Cfg<64>::SMEM)
                            : smem_attr(tc_attention_bwd_kernel<128>, tb::Cfg<128>::SMEM);
  if (!attr) {
    tao_set_last_error("smem attribute");
    return TAO_ERR_CUDA;
  }
  const long long n = (long long)B * T * H * D;
  if (cudaMemsetAsync(dq_acc, 0, (size_t)n * sizeof(float), s) != cudaSuccess) {
    tao_set_last_error("dq accumulator memset failed");
    return TAO_ERR_CUDA;
  }
  TcBwdArgs a{lse, rowdot, dk, dv, T, H, err};
  const dim3 grid((T + tb::kBN - 1) / tb::kBN, B * H, D / 64);
  if (D == 64)
    tc_attention_bwd_kernel<64><<<grid, tb::kThreads, tb::Cfg<64>::SMEM, s>>>(mq, mk, mv, mo, mdq, a);
  else
    tc_attention_bwd_kernel<128><<<grid, tb::kThreads, tb::Cfg<128>::SMEM, s>>>(mq, mk, mv, mo, mdq, a);
  const long long n8 = n / 8;
  dq_convert_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, s>>>(dq_acc, dq, n8, D == 64 ? 0.125f
                                                                                        : 0.08838834764831845f);
  return TAO_OK;
}

}  // namespace tao

extern "C" int tao_attention_variant(int variant) {
  if (variant < 0 || variant > 1) {
    tao_set_last_error("attention variant must be 0 or 1");
    return TAO_ERR_ARG;
  }
  g_attention_variant = variant;
  return TAO_OK;
}
