// tao_stream_decode_noalloc: one decode step for a batch of requests that
// allocates nothing.
//
// Who needs it: a caller that may not call cudaMalloc -- for example a serving
// loop whose device memory is owned by another runtime's pool, or a
// latency-critical loop where cudaMalloc/cudaFree could synchronise the device.
// tao_stream_step needs a caller-provided workspace; this variant keeps its
// scratch (route slots, split partials, the error word) in the file-scope device
// array below instead, so the caller passes only inputs, outputs and states.
//
// Limits and sharing:
// * the scratch holds kScratchBytes (4 MiB); a batch whose decode scratch
//   (tao_stream_workspace_bytes for the same shapes, with the route-budget-sized
//   split) is larger is rejected with TAO_ERR_CAPACITY;
// * every GPU that loads the library holds one such array until the process exits;
// * every call on a device shares the array and it keeps the last call's contents;
//   the error word is cleared at the start of each call, every other region is
//   written before it is read.  Calls that overlap on the GPU (other streams, other
//   host threads) race on the array: serialise them;
// * the first call on each device looks the array's device address up
//   (cudaGetSymbolAddress with that device current); make that first call before
//   any stream capture.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/tao_b200.h"
#include "stream_kernels.cuh"

void tao_set_last_error(const char* msg);

namespace {

constexpr size_t kScratchBytes = size_t(4) << 20;
constexpr int kMaxDevices = 64;

// Host code must not use this name as an address: on the host it is a stand-in
// symbol.  The device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

int na_fail(int code, const char* msg) {
  tao_set_last_error(msg);
  return code;
}

size_t na_align(size_t x) { return (x + 255) & ~size_t(255); }

int na_budget(int count, const TaoPolicy& p) {
  if (count <= 0) return 0;
  long long sq = (long long)p.budget_root_scale * count;
  long long lo = 0, hi = 1;
  while (hi * hi <= sq) hi <<= 1;
  while (lo < hi) {
    long long mid = (lo + hi + 1) / 2;
    if (mid * mid <= sq) lo = mid; else hi = mid - 1;
  }
  if (lo * lo < sq) ++lo;
  long long b = lo + p.budget_offset;
  return (int)(b < count ? b : count);
}

// Device address of the scratch array for the current device (set up once).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return na_fail(TAO_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return na_fail(TAO_ERR_ARG, "device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || !p) {
      char buf[256];
      snprintf(buf, sizeof(buf), "cudaGetSymbolAddress(decode scratch): %s", cudaGetErrorString(e));
      return na_fail(TAO_ERR_CUDA, buf);
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return TAO_OK;
}

template <typename F>
bool na_smem(F* fn, size_t bytes) {
  return bytes <= 48 * 1024 ||
         cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess;
}

template <int D>
int na_launch(const tao::StepArgs& a, cudaStream_t s) {
  using namespace tao;
  using Cfg = DecodeCfg<D>;
  const size_t prep_smem = (size_t)D * 4 + (size_t)a.pmax * 4 + (size_t)(8 * a.pmax + 8) * 8 + (size_t)a.pmax * 8;
  const size_t main_smem = (size_t)Cfg::FPC * D * D * 2 + (size_t)Cfg::FPC * D * 4;
  const size_t fin_smem = (size_t)2 * kFine * D * 2 + (size_t)2 * D * 4;
  if (!na_smem(prep_kernel<D>, prep_smem) || !na_smem(decode_main_kernel<D>, main_smem) ||
      !na_smem(finalize_kernel<D>, fin_smem))
    return na_fail(TAO_ERR_CUDA, "shared-memory attribute rejected");
  prep_kernel<D><<<dim3(a.R * a.H, a.nslot), 256, prep_smem, s>>>(a);
  decode_main_kernel<D><<<dim3(a.R * a.H, a.kblocks + a.msplit), 128, main_smem, s>>>(a);
  finalize_kernel<D><<<a.R * a.H, 256, fin_smem, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return na_fail(TAO_ERR_CUDA, cudaGetErrorString(e));
  return TAO_OK;
}

}  // namespace

extern "C" int tao_stream_decode_noalloc(void* const* states, int n_states, const int64_t* host_pos,
                                         const int32_t* host_cap, const TaoPolicy* policy, int heads,
                                         int width, const void* q, const void* k, const void* v,
                                         const void* raw_q, const void* raw_k, const void* fusion_a,
                                         const void* fusion_b, float alpha, void* out, void* stream) {
  if (!states || n_states <= 0 || !host_pos || !host_cap || !policy)
    return na_fail(TAO_ERR_ARG, "null state, cursor, capacity or policy array");
  if (width != 64 && width != 128) return na_fail(TAO_ERR_ARG, "head width must be 64 or 128");
  if (heads <= 0) return na_fail(TAO_ERR_ARG, "heads must be positive");
  if (policy->fine_tokens != 256 || policy->local_keep != 512 || policy->coarse_group != 8)
    return na_fail(TAO_ERR_ARG, "kernels are specialised for fine_tokens=256, local_keep=512, coarse_group=8");
  if (policy->route_period <= 0 || policy->layer_stagger < 0 || policy->budget_root_scale <= 0 ||
      policy->budget_offset < 0 || policy->route_cap <= 0)
    return na_fail(TAO_ERR_ARG, "invalid routing policy");
  if (policy->fine_read != 0)
    return na_fail(TAO_ERR_ARG, "the feature-mass read (policy.fine_read = 1) is served by tao_stream_step");
  if (policy->coarse != 0)
    return na_fail(TAO_ERR_ARG, "the coarse value branch (policy.coarse = 1) is served by tao_stream_step");
  for (const void* p : {q, k, v, raw_q, raw_k, fusion_a, fusion_b, (const void*)out})
    if (!p) return na_fail(TAO_ERR_ARG, "null tensor pointer");
  for (const void* p : {q, k, v, raw_q, raw_k, (const void*)out})
    if (reinterpret_cast<uintptr_t>(p) & 15) return na_fail(TAO_ERR_ARG, "token tensors must be 16-byte aligned");

  int pmax = 1, mbound = 1;
  for (int r = 0; r < n_states; ++r) {
    const long long pos = host_pos[r];
    if (pos < 0) return na_fail(TAO_ERR_POSITION, "negative position");
    const long long start = pos < 768 ? 0 : 256LL * ((pos - 512) / 256);
    const int S = pos >= 768 ? (int)((pos - 768) / 256) + 1 : 0;
    const bool seal = (pos + 1 - start) == 768;
    const int cap = host_cap[r];
    if (cap <= 0 || cap % 8) return na_fail(TAO_ERR_ARG, "fine capacity must be a positive multiple of 8");
    if (S + (seal ? 1 : 0) > cap) return na_fail(TAO_ERR_CAPACITY, "fine bank capacity too small");
    if (cap / 8 + 1 > pmax) pmax = cap / 8 + 1;
    const int mb = na_budget(cap, *policy);
    if (mb > mbound) mbound = mb;
  }
  const int route_cap = policy->route_cap;
  if (mbound > route_cap) mbound = route_cap;
  const size_t prep_smem = (size_t)width * 4 + (size_t)pmax * 4 + (size_t)(8 * pmax + 8) * 8 + (size_t)pmax * 8;
  if (prep_smem > 200 * 1024) return na_fail(TAO_ERR_CAPACITY, "fine capacity too large for the route kernel");

  // scratch carve-out (same regions as the workspace of tao_stream_step, tokens = 1)
  const int fpc = width == 64 ? 4 : 1, kblocks = width == 64 ? 6 : 12, nslot = 2;
  const int msplit = (mbound + fpc - 1) / fpc;
  const size_t R = n_states, H = heads, D = width;
  size_t off = 0;
  const size_t o_err = off;         off = na_align(off + 256);
  const size_t o_ids = off;         off = na_align(off + R * H * nslot * route_cap * 4);
  const size_t o_pages = off;       off = na_align(off + R * H * nslot * route_cap * 4);
  const size_t o_n = off;           off = na_align(off + R * nslot * 2 * 4);
  const size_t o_local = off;       off = na_align(off + R * H * kblocks * (D + 2) * 4);
  const size_t o_fine = off;        off = na_align(off + R * H * msplit * (D + 1) * 4);
  if (off > kScratchBytes) {
    char buf[256];
    snprintf(buf, sizeof(buf), "decode scratch of %zu bytes exceeds the static %zu-byte array; "
             "use tao_stream_step with a workspace", off, kScratchBytes);
    return na_fail(TAO_ERR_CAPACITY, buf);
  }

  void* base = nullptr;
  int rc = scratch_address(&base);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(base);
  cudaError_t e = cudaMemsetAsync(ws + o_err, 0, 256, s);  // error word starts at zero
  if (e != cudaSuccess) return na_fail(TAO_ERR_CUDA, cudaGetErrorString(e));

  tao::StepArgs a{};
  a.states = reinterpret_cast<TaoState* const*>(states);
  a.R = n_states;
  a.w = 1;
  a.H = heads;
  a.pol = {policy->route_period, policy->layer_stagger, policy->budget_root_scale, policy->budget_offset};
  a.q = static_cast<const tao::bf16*>(q);
  a.k = static_cast<const tao::bf16*>(k);
  a.v = static_cast<const tao::bf16*>(v);
  a.raw_q = static_cast<const tao::bf16*>(raw_q);
  a.raw_k = static_cast<const tao::bf16*>(raw_k);
  a.fa = static_cast<const tao::bf16*>(fusion_a);
  a.fb = static_cast<const tao::bf16*>(fusion_b);
  a.gain = __bfloat162float(__float2bfloat16_rn(2.0f * alpha));
  a.out = static_cast<tao::bf16*>(out);
  a.err = reinterpret_cast<int*>(ws + o_err);
  a.nslot = nslot;
  a.route_cap = route_cap;
  a.slot_ids = reinterpret_cast<int32_t*>(ws + o_ids);
  a.slot_pages = reinterpret_cast<int32_t*>(ws + o_pages);
  a.slot_n = reinterpret_cast<int32_t*>(ws + o_n);
  a.kblocks = kblocks;
  a.msplit = msplit;
  a.local_part = reinterpret_cast<float*>(ws + o_local);
  a.local_out = nullptr;
  a.fine_part = reinterpret_cast<float*>(ws + o_fine);
  a.pmax = pmax;
  return width == 64 ? na_launch<64>(a, s) : na_launch<128>(a, s);
}

// Device error word of the allocation-free decode on the current device: the
// kernels of tao_stream_decode_noalloc record a route overflow or a wait timeout
// there (the word a workspace caller reads with tao_stream_check).  Synchronises
// `stream`, returns the word in *flags and clears it.
extern "C" int tao_stream_decode_noalloc_check(int* flags, void* stream) {
  void* base = nullptr;
  int rc = scratch_address(&base);
  if (rc) return rc;
  int host = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&host, base, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && host) e = cudaMemsetAsync(base, 0, sizeof(int), s);
  if (e != cudaSuccess) return na_fail(TAO_ERR_CUDA, cudaGetErrorString(e));
  if (flags) *flags = host;
  if (host) {
    char buf[128];
    snprintf(buf, sizeof(buf), "device error flags 0x%x", host);
    return na_fail(TAO_ERR_DEVICE, buf);
  }
  return TAO_OK;
}
