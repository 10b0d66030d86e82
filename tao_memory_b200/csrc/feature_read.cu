// extern "C" entry points of the training feature-mass read (tcgen05 kernels in
// feature_read.cuh).
#include <cuda_runtime.h>

#include "../../include/tao_b200.h"
#include "feature_read.cuh"

void tao_set_last_error(const char* msg);

namespace {

int ffail(int code, const char* msg) {
  tao_set_last_error(msg);
  return code;
}

int visible_max(int T) {
  const int tiles = (T + 255) / 256;
  return tiles > 3 ? tiles - 3 : 0;
}

template <int D>
int feature_launch(const tao::FeatArgs& a, bool back, cudaStream_t s) {
  using namespace tao;
  const int vmax = visible_max(a.T);
  if (vmax > 256) return ffail(TAO_ERR_CAPACITY, "feature read: more than 256 visible fines");
  if (a.mmax > 64) return ffail(TAO_ERR_CAPACITY, "feature read: more than 64 selected fines per query");
  const size_t smem = FeatSmem<D>(vmax, a.mmax, back).total;
  if (smem > 227 * 1024) return ffail(TAO_ERR_CAPACITY, "feature read: sequence too long for shared memory");
  const dim3 grid((a.T + kFeatQ - 1) / kFeatQ, a.B * a.H);
  cudaError_t e;
  if (back) {
    e = cudaFuncSetAttribute(feature_read_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) feature_read_bwd_kernel<D><<<grid, kFeatQ, smem, s>>>(a);
  } else {
    e = cudaFuncSetAttribute(feature_read_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) feature_read_fwd_kernel<D><<<grid, kFeatQ, smem, s>>>(a);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TAO_OK : ffail(TAO_ERR_CUDA, cudaGetErrorString(e));
}

int feature_entry(const void* grad, const void* raw_q, const void* fine_z, const void* fine_c, const int16_t* sel,
                  int batch, int tokens, int heads, int width, int mmax, void* out, float* dz, float* dc, int* err,
                  bool back, void* stream) {
  if (!raw_q || !fine_z || !fine_c || !sel || !out || !err || (back && (!grad || !dz || !dc)))
    return ffail(TAO_ERR_ARG, "null pointer");
  if (width != 64 && width != 128) return ffail(TAO_ERR_ARG, "head width must be 64 or 128");
  if (batch <= 0 || tokens <= 768 || heads <= 0 || mmax <= 0)
    return ffail(TAO_ERR_ARG, "feature read: bad shape (tokens must exceed 768)");
  tao::FeatArgs a{};
  a.raw_q = static_cast<const tao::bf16*>(raw_q);
  a.z = static_cast<const tao::bf16*>(fine_z);
  a.C = static_cast<const tao::bf16*>(fine_c);
  a.g = static_cast<const tao::bf16*>(grad);
  a.sel = sel;
  a.out = static_cast<tao::bf16*>(out);
  a.dz = dz;
  a.dc = dc;
  a.B = batch;
  a.T = tokens;
  a.H = heads;
  a.S = tokens / 256 - 1;
  a.mmax = mmax;
  a.err = err;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return width == 64 ? feature_launch<64>(a, back, s) : feature_launch<128>(a, back, s);
}

}  // namespace

extern "C" {

int tao_feature_read_forward(const void* raw_q, const void* fine_z, const void* fine_c, const int16_t* sel,
                             int batch, int tokens, int heads, int width, int mmax, void* out, int* err,
                             void* stream) {
  return feature_entry(nullptr, raw_q, fine_z, fine_c, sel, batch, tokens, heads, width, mmax, out, nullptr,
                       nullptr, err, false, stream);
}

int tao_feature_read_backward(const void* grad, const void* raw_q, const void* fine_z, const void* fine_c,
                              const int16_t* sel, int batch, int tokens, int heads, int width, int mmax,
                              void* d_raw_q, float* dz, float* dc, int* err, void* stream) {
  return feature_entry(grad, raw_q, fine_z, fine_c, sel, batch, tokens, heads, width, mmax, d_raw_q, dz, dc, err,
                       true, stream);
}

}  // extern "C"
