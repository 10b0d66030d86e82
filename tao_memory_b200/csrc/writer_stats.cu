// extern "C" entry of the association-writer statistics kernel.
#include <cuda_runtime.h>

#include "../../include/tao_b200.h"
#include "writer_stats.cuh"

void tao_set_last_error(const char* msg);

extern "C" int tao_writer_stats(const void* k, const void* v, long long token_stride, long long head_stride,
                                long long block_stride, int blocks, int heads, int width, float* gram,
                                float* cross, float* mass, void* stream) {
  if (!k || !v || !gram || !cross || blocks <= 0 || heads <= 0 || token_stride <= 0) {
    tao_set_last_error("bad writer statistics arguments");
    return TAO_ERR_ARG;
  }
  if (width != 64 && width != 128) {
    tao_set_last_error("head width must be 64 or 128");
    return TAO_ERR_ARG;
  }
  if (((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15) || (token_stride * 2) % 16 ||
      (head_stride * 2) % 16 || (block_stride * 2) % 16 || ((reinterpret_cast<uintptr_t>(gram) |
                                                              reinterpret_cast<uintptr_t>(cross) |
                                                              reinterpret_cast<uintptr_t>(mass)) & 7)) {
    tao_set_last_error("writer statistics operands must be 16-byte aligned rows");
    return TAO_ERR_ARG;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)2 * 256 * width * 2;
  cudaError_t e;
  if (width == 64) {
    e = cudaFuncSetAttribute(tao::writer_stats_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      tao::writer_stats_kernel<64><<<blocks * heads, 128, smem, s>>>(
          static_cast<const tao::bf16*>(k), static_cast<const tao::bf16*>(v), token_stride, head_stride,
          block_stride, heads, gram, cross, mass);
  } else {
    e = cudaFuncSetAttribute(tao::writer_stats_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      tao::writer_stats_kernel<128><<<blocks * heads, 128, smem, s>>>(
          static_cast<const tao::bf16*>(k), static_cast<const tao::bf16*>(v), token_stride, head_stride,
          block_stride, heads, gram, cross, mass);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    tao_set_last_error(cudaGetErrorString(e));
    return TAO_ERR_CUDA;
  }
  return TAO_OK;
}
