// extern "C" entry points of libtao_b200.so (declared in include/tao_b200.h).
//
// Host side: argument validation with the reference's error cases
// (operator.py:77-78, tao_stream.py:931-932), workspace carving, grid sizing and
// kernel launches on the caller's stream.  No allocation happens here: state
// buffers and the workspace are owned by the caller.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/tao_b200.h"
#include "decode_fused.cuh"
#include "stream_kernels.cuh"
#include "tc_writer.cuh"
#include "window_attention.cuh"

namespace tao {
int launch_window_attention(const bf16* q, const bf16* k, const bf16* v, bf16* out, float* lse, int B,
                            int T, int H, int D, int* err, cudaStream_t s);
int launch_ring_attention(TaoState* const* states, const bf16* q, bf16* out, int R, int w, int H, int D, int* err,
                          cudaStream_t s);
int attention_variant();
}  // namespace tao

namespace {

thread_local std::string g_last_error;
// Events recorded around the main kernel of the next step, training forward or
// training backward (whichever takes them first, from any host thread: torch runs
// the backward on its own thread); cleared when taken.
std::mutex g_prof_mutex;
cudaEvent_t g_prof_start = nullptr, g_prof_stop = nullptr;
// Decode kernel choice: 1 = persistent fused kernel, one stage per CTA (default),
// 3 = the same with two stages (fewer resident CTAs: measured slower), 0 =
// warp-specialised persistent, 2 = one warp per 8 KB item.
int g_decode_variant = 1;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TAO_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return TAO_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// --- host mirrors of the device schedule (common.cuh) ---------------------
int h_budget(int count, const TaoPolicy& p) {
  if (count <= 0) return 0;
  long long sq = (long long)p.budget_root_scale * count;
  long long r = 0;
  {
    long long lo = 0, hi = 1;
    while (hi * hi <= sq) hi <<= 1;
    while (lo < hi) {
      long long mid = (lo + hi + 1) / 2;
      if (mid * mid <= sq) lo = mid; else hi = mid - 1;
    }
    r = lo;
  }
  if (r * r < sq) ++r;
  long long b = r + p.budget_offset;
  return (int)(b < count ? b : count);
}
int h_sealed_at(long long pos) { return pos >= 768 ? (int)((pos - 768) / 256) + 1 : 0; }
long long h_window_start(long long pos) { return pos < 768 ? 0 : 256LL * ((pos - 512) / 256); }

int fpc_for(int width) { return width == 64 ? 4 : 1; }
// selected fines per fine item of the decode kernel of the current variant
int fused_fpc(int width) {
  if (g_decode_variant == 2) return 1;
  if (g_decode_variant == 4 && width == 64) return 2;
  return fpc_for(width);
}
int kblocks_for(int width) { return width == 64 ? 6 : 12; }

struct Layout {
  size_t err, slot_ids, slot_pages, slot_n, local_part, local_out, fine_part, coarse_out, total;
  int nslot, msplit, kblocks;
};

// Route slots: slot 0 = routes stored in the state, then one per refresh anchor
// of the chunk (at most ceil(w / period) periodic turns plus position 768).
int nslot_for(int w, int period) {
  int n = 1 + (w + period - 1) / period + 1;
  return n < 1 + w ? n : 1 + w;
}

// feature: the feature-mass read, which serves w == 1 through the prefill kernels
// (window attention output + one fine partial per query).
Layout make_layout(int R, int w, int H, int D, int route_cap, int msplit_decode, int period,
                   bool feature = false, bool coarse = false) {
  Layout L{};
  L.nslot = nslot_for(w, period);
  L.kblocks = kblocks_for(D);
  L.msplit = (w == 1 && !feature) ? msplit_decode : 1;
  size_t off = 0;
  L.err = off;
  off = align256(off + 256);
  L.slot_ids = off;
  off = align256(off + (size_t)R * H * L.nslot * route_cap * 4);
  L.slot_pages = off;
  off = align256(off + (size_t)R * H * L.nslot * route_cap * 4);
  L.slot_n = off;
  off = align256(off + (size_t)R * L.nslot * 2 * 4);
  L.local_part = off;
  // decode partials: room for the warp kernel's 768/(2048/D) local items per (r, h)
  if (w == 1) off = align256(off + (size_t)R * H * (768 / (2048 / D)) * (D + 2) * 4);
  L.local_out = off;
  if (w > 1 || feature) off = align256(off + (size_t)R * w * H * D * 2);
  L.fine_part = off;
  off = align256(off + (size_t)R * w * H * L.msplit * (D + 1) * 4);
  L.coarse_out = off;   // coarse value branch: bf16 coarse read of every query
  if (coarse) off = align256(off + (size_t)R * w * H * D * 2);
  L.total = off;
  return L;
}

float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

}  // namespace

// Lets other translation units of the library report a message through
// tao_last_error() on the calling host thread.
void tao_set_last_error(const char* msg) { g_last_error = msg; }

// Hands the pending profiling events (tao_stream_profile_next) to another
// translation unit's launcher and clears them.
void tao_take_profile_events(cudaEvent_t* start, cudaEvent_t* stop) {
  std::lock_guard<std::mutex> lock(g_prof_mutex);
  *start = g_prof_start;
  *stop = g_prof_stop;
  g_prof_start = g_prof_stop = nullptr;
}

namespace {

// Opt in to more than the default dynamic shared memory when a launch needs most of
// the default 48 KB (static shared memory of the kernel counts against it too).
template <typename F>
int set_smem(F* fn, size_t bytes) {
  if (bytes > 40 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return fail(TAO_ERR_CUDA, "smem attribute: %s", cudaGetErrorString(e));
  }
  return TAO_OK;
}

template <int D>
int launch_step(tao::StepArgs a, const Layout& L, cudaStream_t s) {
  using namespace tao;
  int rc;
  // prep: append + routing
  const size_t prep_smem = (size_t)D * 4 + (size_t)a.pmax * 4 + (size_t)(8 * a.pmax + 8) * 8 + (size_t)a.pmax * 8;
  if ((rc = set_smem(prep_kernel<D>, prep_smem))) return rc;
  prep_kernel<D><<<dim3(a.R * a.H, L.nslot), 256, prep_smem, s>>>(a);
  if ((rc = check_launch("prep_kernel"))) return rc;
  cudaEvent_t prof0, prof1;
  tao_take_profile_events(&prof0, &prof1);
  if (prof0) cudaEventRecord(prof0, s);
  if (a.w == 1 && !a.feature) {
    using Cfg = DecodeCfg<D>;
    const size_t main_smem = (size_t)Cfg::FPC * D * D * 2 + (size_t)Cfg::FPC * D * 4;
    if ((rc = set_smem(decode_main_kernel<D>, main_smem))) return rc;
    decode_main_kernel<D><<<dim3(a.R * a.H, a.kblocks + a.msplit), 128, main_smem, s>>>(a);
    if ((rc = check_launch("decode_main_kernel"))) return rc;
  } else {
    WinAttnParams p{};
    p.q = a.q;
    p.out = a.local_out;
    p.q_batch_stride = (long long)a.w * a.H * D;
    p.q_row_stride = (long long)a.H * D;
    p.o_batch_stride = p.q_batch_stride;
    p.o_row_stride = p.q_row_stride;
    p.k_row_stride = D;
    p.k_head_stride = (long long)kWindow * D;
    p.heads = a.H;
    p.nq = a.w;
    p.ring = 1;
    p.states = a.states;
    if (attention_variant() == 1) {
      // tcgen05 / TMEM over each state's ring (cp.async tiles in the TMA layout)
      if ((rc = launch_ring_attention(a.states, a.q, a.local_out, a.R, a.w, a.H, D, a.err, s))) return rc;
    } else {
      const size_t attn_smem = (size_t)(64 + 4 * 64) * D * 2;
      if ((rc = set_smem(window_attention_kernel<D>, attn_smem))) return rc;
      window_attention_kernel<D><<<dim3((a.w + 63) / 64, a.R * a.H), 128, attn_smem, s>>>(p);
      if ((rc = check_launch("window_attention_kernel"))) return rc;
    }
    const size_t pf_smem = (size_t)2 * D * D * 2 + (size_t)(2 * 16 * D + 2 * D) * 4;
    if ((rc = set_smem(prefill_fine_kernel<D>, pf_smem))) return rc;
    prefill_fine_kernel<D><<<dim3(a.R * a.H, (a.w + 15) / 16), 128, pf_smem, s>>>(a);
    if ((rc = check_launch("prefill_fine_kernel"))) return rc;
  }
  if (prof1) cudaEventRecord(prof1, s);
  if (a.coarse) {
    // coarse value read: tiles of qt queries (a power of two, at most QTMAX)
    using CC = CoarseCfg<D>;
    int qt = 1;
    while (qt < a.w && qt < CC::QTMAX) qt *= 2;
    const size_t cs = CC::smem(qt);
    if ((rc = set_smem(coarse_read_kernel<D>, cs))) return rc;
    coarse_read_kernel<D><<<dim3(a.R * a.H, (a.w + qt - 1) / qt), 256, cs, s>>>(a, qt);
    if ((rc = check_launch("coarse_read_kernel"))) return rc;
  }
  const size_t fin_smem = (size_t)2 * kFine * D * 2 + (size_t)2 * D * 4;
  if ((rc = set_smem(finalize_kernel<D>, fin_smem))) return rc;
  finalize_kernel<D><<<a.R * a.H, 256, fin_smem, s>>>(a);
  return check_launch("finalize_kernel");
}

// Graph mode (tao_decode_graph_mode): every decode step launches the route and seal
// kernels, which decide on the device from the cursor whether this token refreshes
// or seals, so one captured launch sequence serves every token.
thread_local int g_graph_mode = 0;

constexpr int kMaxDevices = 64;

// Streaming multiprocessors of a device, queried once per device.
int device_sm_count(int dev) {
  static std::atomic<int> sms_of[kMaxDevices];
  int sms = sms_of[dev].load(std::memory_order_relaxed);
  if (sms <= 0) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    sms_of[dev].store(sms, std::memory_order_relaxed);
  }
  return sms;
}

// Persistent fused decode kernel with NS stages per CTA: as many CTAs as are resident
// at once, each walking the same number of items (give or take one) by the grid stride.
// Slot-major item tables of the fused kernel from each request's bound on its selected
// fines (mb[r]): a request gets KB local items and ceil(mb[r] / FPC) fine items per
// head, so short requests in a mixed batch launch no empty fine items.  Past the
// tables' limits (or without bounds) every request gets KB + ms items (nslots = 0).
template <int D, int IB>
void fused_tables(tao::FusedArgs& f, const int* mb) {
  using Cfg = tao::FusedCfg<D, IB>;
  const int R = f.s.R, H = f.s.H;
  f.nslots = 0;
  if (!mb || R > tao::kFusedMaxReq) return;
  int per[tao::kFusedMaxReq], order[tao::kFusedMaxReq];
  int most = 0;
  for (int r = 0; r < R; ++r) {
    int fi = (mb[r] + Cfg::FPC - 1) / Cfg::FPC;
    if (fi > f.ms) fi = f.ms;  // within the partial buffers' stride
    per[r] = Cfg::KB + fi;
    if (per[r] > most) most = per[r];
    order[r] = r;
  }
  if (most > tao::kFusedMaxSlots) return;
  bool uniform = true;  // every request at the full count: the plain item order
  for (int r = 0; r < R; ++r) uniform = uniform && per[r] == Cfg::KB + f.ms;
  if (uniform) return;
  for (int i = 1; i < R; ++i) {  // stable: most items first
    const int x = order[i];
    int j = i;
    while (j > 0 && per[order[j - 1]] < per[x]) {
      order[j] = order[j - 1];
      --j;
    }
    order[j] = x;
  }
  int base = 0, active = R;
  for (int sl = 0; sl < most; ++sl) {
    while (active > 0 && per[order[active - 1]] <= sl) --active;
    f.slot_base[sl] = base;
    base += active * H;
  }
  f.slot_base[most] = base;
  for (int r = 0; r < R; ++r) {
    f.rorder[r] = (int16_t)order[r];
    f.per_r[r] = (int16_t)per[r];
  }
  f.nslots = most;
}

template <int D, int NS, int IB>
int launch_fused(tao::FusedArgs f, int sms, int dev, cudaStream_t s, const int* mb) {
  using namespace tao;
  const size_t smem = (size_t)NS * FusedCfg<D, IB>::STAGE;
  fused_tables<D, IB>(f, mb);
  const int total = f.nslots ? f.slot_base[f.nslots] : f.s.R * f.s.H * (FusedCfg<D, IB>::KB + f.ms);
  int rc;
  if ((rc = set_smem(decode_fused_kernel<D, NS, IB>, smem))) return rc;
  // resident CTAs per SM: one occupancy query per (device, width, stages), kept for the process
  static std::atomic<int> per_sm_of[kMaxDevices];
  int per_sm = per_sm_of[dev].load(std::memory_order_relaxed);
  if (per_sm <= 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_fused_kernel<D, NS, IB>, 128, smem) != cudaSuccess ||
        per_sm <= 0)
      per_sm = 1;
    per_sm_of[dev].store(per_sm, std::memory_order_relaxed);
  }
  const int resident = per_sm * sms;
  const int rounds = (total + resident - 1) / resident;
  decode_fused_kernel<D, NS, IB><<<(total + rounds - 1) / rounds, 128, smem, s>>>(f);
  return TAO_OK;
}

// Operands of a host-staged decode step (tao_decode_step_host): the route kernel copies
// `vecs` 16-byte vectors from page-locked host memory `in` to the device stage and reads
// raw_q from host memory itself.
struct HostStage {
  const uint4* in;
  uint4* stage;
  int vecs;
  const tao::bf16* raw_q;
  int* host_done;  // device address of the page-locked completion word (or null)
};

template <int D>
int launch_decode(const tao::StepArgs& a, int ms, bool refresh, bool seal, cudaStream_t s,
                  const HostStage* hs = nullptr, const int* mb = nullptr) {
  using namespace tao;
  int rc;
  if (refresh || hs) {  // a host-staged step always launches it: it brings the operands in
    StepArgs ar = a;
    if (hs) {
      ar.h_in = hs->in;
      ar.h_stage = hs->stage;
      ar.h_vecs = hs->vecs;
      ar.raw_q = hs->raw_q;
    }
    const size_t smem = (size_t)D * 4 + (size_t)a.pmax * 4 + (size_t)(8 * a.pmax + 8) * 8 + (size_t)a.pmax * 8;
    if ((rc = set_smem(decode_route_kernel<D>, smem))) return rc;
    decode_route_kernel<D><<<a.R * a.H, 1024, smem, s>>>(ar);
    if ((rc = check_launch("decode_route_kernel"))) return rc;
  }
  FusedArgs f{};
  f.s = a;
  f.ms = ms;
  const int total = a.R * a.H * (FusedCfg<D>::KB + ms);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(TAO_ERR_CUDA, "no current CUDA device (or device index above %d)", kMaxDevices - 1);
  const int sms = device_sm_count(dev);
  cudaEvent_t prof0, prof1;
  tao_take_profile_events(&prof0, &prof1);
  if (prof0) cudaEventRecord(prof0, s);
  if (g_decode_variant == 2) {
    const int wt = a.R * a.H * (WarpCfg<D>::LI + ms);
    decode_warp_kernel<D><<<(wt + 7) / 8, 256, 0, s>>>(f);
  } else if (g_decode_variant == 0) {
    if (a.R > kWsMaxReq) return fail(TAO_ERR_ARG, "decode variant 0 takes at most %d requests per call", kWsMaxReq);
    const size_t smem = (size_t)kWsStages * WsLayout<D>::STAGE;
    if ((rc = set_smem(decode_ws_kernel<D>, smem))) return rc;
    int grid = total < sms ? total : sms;
    const int need = (total + kWsMaxItems - 1) / kWsMaxItems;
    if (grid < need) grid = need;
    decode_ws_kernel<D><<<grid, 288, smem, s>>>(f);
  } else if (g_decode_variant == 3) {
    if ((rc = launch_fused<D, 2, 32768>(f, sms, dev, s, mb))) return rc;   // two 32 KB stages per CTA
  } else if (D == 64 && g_decode_variant == 4) {
    // two 16 KB stages per CTA: items of 64 keys or 2 fines
    if constexpr (D == 64) {
      if ((rc = launch_fused<D, 2, 16384>(f, sms, dev, s, mb))) return rc;
    }
  } else {
    if ((rc = launch_fused<D, 1, 32768>(f, sms, dev, s, mb))) return rc;   // one 32 KB stage per CTA
  }
  if (prof1) cudaEventRecord(prof1, s);
  if ((rc = check_launch("decode_fused_kernel"))) return rc;
  if (seal) {
    // the block writer on the tensor cores (C = p^T v by tcgen05.mma into TMEM)
    const size_t ss = TcWriterCfg<D>::SMEM;
    if ((rc = set_smem(tc_seal_kernel<D>, ss))) return rc;
    tc_seal_kernel<D><<<a.R * a.H, 128, ss, s>>>(a);
    if ((rc = check_launch("tc_seal_kernel"))) return rc;
  }
  return TAO_OK;
}

}  // namespace

namespace {

int decode_step_impl(void* const* states, int n_states, const int64_t* host_pos, const int32_t* host_layer,
                     const int32_t* host_cap, const TaoPolicy* policy, int heads, int width, const void* q,
                     const void* k, const void* v, const void* raw_q, const void* raw_k, const void* fusion_a,
                     const void* fusion_b, float alpha, void* out, void* workspace, size_t workspace_bytes,
                     void* stream, const HostStage* hs) {
  if (!states || n_states <= 0 || !host_pos || !host_cap || !host_layer || !policy)
    return fail(TAO_ERR_ARG, "null state, cursor, layer, capacity or policy array");
  if (policy->coarse && hs)
    return fail(TAO_ERR_ARG, "the coarse value branch decodes through tao_decode_step (device operands)");
  if (hs && hs->host_done && (g_decode_variant == 0 || g_decode_variant == 2))
    return fail(TAO_ERR_ARG, "a completion word needs the fused decode kernel (variant 1, 3 or 4)");
  if (policy->coarse)   // the coarse value branch decodes through the stream-step kernels
    return tao_stream_step(states, n_states, host_pos, host_cap, policy, 1, heads, width, q, k, v, raw_q, raw_k,
                           fusion_a, fusion_b, alpha, out, workspace, workspace_bytes, stream);
  if (width != 64 && width != 128) return fail(TAO_ERR_ARG, "head width must be 64 or 128, got %d", width);
  if (heads <= 0) return fail(TAO_ERR_ARG, "heads must be positive");
  if (policy->fine_tokens != 256 || policy->local_keep != 512 || policy->coarse_group != 8)
    return fail(TAO_ERR_ARG, "kernels are specialised for fine_tokens=256, local_keep=512, coarse_group=8");
  if (policy->route_period <= 0 || policy->layer_stagger < 0 || policy->budget_root_scale <= 0 ||
      policy->budget_offset < 0 || policy->route_cap <= 0)
    return fail(TAO_ERR_ARG, "invalid routing policy");
  if (policy->fine_read != 0 && policy->fine_read != 1)
    return fail(TAO_ERR_ARG, "policy.fine_read must be 0 or 1, got %d", policy->fine_read);
  if (policy->fine_read == 1 && (g_decode_variant == 0 || g_decode_variant == 2))
    return fail(TAO_ERR_ARG, "the feature-mass read runs in the fused decode kernel (variant 1, 3 or 4)");
  for (const void* p : {q, k, v, raw_q, raw_k, fusion_a, fusion_b, (const void*)out, (const void*)workspace})
    if (!p) return fail(TAO_ERR_ARG, "null tensor pointer");
  for (const void* p : {q, k, v, raw_q, raw_k, (const void*)out})
    if (!aligned16(p)) return fail(TAO_ERR_ARG, "token tensors must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return fail(TAO_ERR_ARG, "workspace must be 256-byte aligned");
  int pmax = 1, mbound = 1;
  bool refresh = false, seal = false;
  // per-request bound on the selected fines the fused kernel reads: the budget of the
  // fines sealed now (routes refreshed this step or earlier never select more); a
  // step that may be captured and replayed at later positions bounds by capacity
  int mb_req[tao::kFusedMaxReq];
  for (int r = 0; r < n_states; ++r) {
    const long long pos = host_pos[r];
    if (pos < 0) return fail(TAO_ERR_POSITION, "negative position");
    const long long start = h_window_start(pos);
    const int S = h_sealed_at(pos);
    const bool sl = (pos + 1 - start) == 768;
    const int cap = host_cap[r];
    if (cap <= 0 || cap % 8) return fail(TAO_ERR_ARG, "fine capacity must be a positive multiple of 8");
    if (S + (sl ? 1 : 0) > cap) return fail(TAO_ERR_CAPACITY, "fine bank capacity %d too small for %d fines", cap, S + 1);
    seal |= sl;
    const long long first_turn = 768 + (long long)policy->layer_stagger * host_layer[r];
    refresh |= S > 0 && (pos == 768 || (pos >= first_turn && (pos - first_turn) % policy->route_period == 0));
    if (cap / 8 + 1 > pmax) pmax = cap / 8 + 1;
    const int mb = h_budget(cap, *policy);
    if (mb > mbound) mbound = mb;
    if (r < tao::kFusedMaxReq) {
      const int m = g_graph_mode ? mb : h_budget(S, *policy);
      mb_req[r] = m < policy->route_cap ? m : policy->route_cap;
    }
  }
  const int route_cap = policy->route_cap;
  if (mbound > route_cap) mbound = route_cap;
  if (policy->fine_read == 1 && mbound > tao::kRouteCapMax)
    return fail(TAO_ERR_CAPACITY, "feature-mass decode holds at most %d selected fines", tao::kRouteCapMax);
  // fine partials per (r, h): one per selected fine (warp kernel) or per group of fpc
  const int fpc = fused_fpc(width);
  const int ms = (mbound + fpc - 1) / fpc;
  const Layout L = make_layout(n_states, 1, heads, width, route_cap, ms, policy->route_period);
  if (workspace_bytes < L.total) return fail(TAO_ERR_ARG, "workspace too small: %zu < %zu", workspace_bytes, L.total);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
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
  a.gain = bf16_round(2.0f * alpha);
  a.out = static_cast<tao::bf16*>(out);
  a.err = reinterpret_cast<int*>(ws + L.err);
  a.nslot = L.nslot;
  a.route_cap = route_cap;
  a.kblocks = L.kblocks;
  a.msplit = ms;
  a.local_part = reinterpret_cast<float*>(ws + L.local_part);
  a.fine_part = reinterpret_cast<float*>(ws + L.fine_part);
  a.pmax = pmax;
  a.feature = policy->fine_read;
  if (hs && hs->host_done) {
    a.done = reinterpret_cast<int*>(ws + L.err) + 4;  // inside the error word's 256-byte block
    a.host_done = hs->host_done;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (g_graph_mode) refresh = seal = true;
  const int* mbp = n_states <= tao::kFusedMaxReq ? mb_req : nullptr;
  return width == 64 ? launch_decode<64>(a, ms, refresh, seal, s, hs, mbp)
                     : launch_decode<128>(a, ms, refresh, seal, s, hs, mbp);
}

}  // namespace

extern "C" {

int tao_decode_step(void* const* states, int n_states, const int64_t* host_pos,
                    const int32_t* host_layer, const int32_t* host_cap, const TaoPolicy* policy,
                    int heads, int width, const void* q, const void* k, const void* v,
                    const void* raw_q, const void* raw_k, const void* fusion_a,
                    const void* fusion_b, float alpha, void* out, void* workspace,
                    size_t workspace_bytes, void* stream) {
  return decode_step_impl(states, n_states, host_pos, host_layer, host_cap, policy, heads, width, q, k, v, raw_q,
                          raw_k, fusion_a, fusion_b, alpha, out, workspace, workspace_bytes, stream, nullptr);
}

int tao_decode_step_host(void* const* states, int n_states, const int64_t* host_pos, const int32_t* host_layer,
                         const int32_t* host_cap, const TaoPolicy* policy, int heads, int width,
                         const void* host_in, void* stage, void* host_out, void* host_done,
                         const void* fusion_a, const void* fusion_b, float alpha, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (!host_in || !stage || !host_out) return fail(TAO_ERR_ARG, "null host operand, stage or host output");
  if (n_states <= 0 || heads <= 0 || (width != 64 && width != 128))
    return fail(TAO_ERR_ARG, "invalid request count, heads or width");
  void* in_dev = nullptr;
  void* out_dev = nullptr;
  void* done_dev = nullptr;
  int rc;
  if ((rc = tao_host_device_pointer(host_in, &in_dev))) return rc;
  if ((rc = tao_host_device_pointer(host_out, &out_dev))) return rc;
  if (host_done && (rc = tao_host_device_pointer(host_done, &done_dev))) return rc;
  if (reinterpret_cast<uintptr_t>(done_dev) & 3) return fail(TAO_ERR_ARG, "completion word must be 4-byte aligned");
  const size_t row = (size_t)n_states * heads * width;  // elements of one operand
  if (!aligned16(in_dev) || !aligned16(stage) || !aligned16(out_dev))
    return fail(TAO_ERR_ARG, "host operands, stage and host output must be 16-byte aligned");
  const tao::bf16* st = static_cast<const tao::bf16*>(stage);
  HostStage hs{static_cast<const uint4*>(in_dev), static_cast<uint4*>(stage), (int)(5 * row * 2 / 16),
               static_cast<const tao::bf16*>(in_dev) + 3 * row, static_cast<int*>(done_dev)};
  return decode_step_impl(states, n_states, host_pos, host_layer, host_cap, policy, heads, width, st, st + row,
                          st + 2 * row, st + 3 * row, st + 4 * row, fusion_a, fusion_b, alpha, out_dev, workspace,
                          workspace_bytes, stream, &hs);
}

int tao_decode_graph_mode(int on) {
  g_graph_mode = on ? 1 : 0;
  return TAO_OK;
}

const char* tao_last_error(void) { return g_last_error.c_str(); }

int tao_version(void) { return 1; }

size_t tao_state_sizeof(void) { return sizeof(TaoState); }

size_t tao_stream_workspace_bytes(int n_states, int tokens, int heads, int width, int route_cap,
                                  const TaoPolicy* policy) {
  if (n_states <= 0 || tokens <= 0 || heads <= 0 || (width != 64 && width != 128) ||
      route_cap <= 0 || !policy || policy->route_period <= 0)
    return 0;
  // one fine partial per selected fine covers every decode kernel variant
  return make_layout(n_states, tokens, heads, width, route_cap, route_cap, policy->route_period,
                     policy->fine_read != 0, policy->coarse != 0).total;
}

int tao_stream_step(void* const* states, int n_states, const int64_t* host_pos,
                    const int32_t* host_cap, const TaoPolicy* policy, int tokens, int heads,
                    int width, const void* q, const void* k, const void* v, const void* raw_q,
                    const void* raw_k, const void* fusion_a, const void* fusion_b, float alpha,
                    void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!states || n_states <= 0 || !host_pos || !host_cap || !policy)
    return fail(TAO_ERR_ARG, "null state, cursor, capacity or policy array");
  if (width != 64 && width != 128)
    return fail(TAO_ERR_ARG, "head width must be 64 or 128, got %d", width);
  if (heads <= 0) return fail(TAO_ERR_ARG, "heads must be positive");
  if (tokens <= 0 || tokens > 256)
    return fail(TAO_ERR_ARG, "tokens per call must be in [1, 256], got %d", tokens);
  if (policy->fine_tokens != 256 || policy->local_keep != 512 || policy->coarse_group != 8)
    return fail(TAO_ERR_ARG, "kernels are specialised for fine_tokens=256, local_keep=512, coarse_group=8");
  if (policy->route_period <= 0 || policy->layer_stagger < 0 || policy->budget_root_scale <= 0 ||
      policy->budget_offset < 0)
    return fail(TAO_ERR_ARG, "invalid routing policy");
  if (policy->fine_read != 0 && policy->fine_read != 1)
    return fail(TAO_ERR_ARG, "policy.fine_read must be 0 or 1, got %d", policy->fine_read);
  if (policy->coarse != 0 && policy->coarse != 1)
    return fail(TAO_ERR_ARG, "policy.coarse must be 0 or 1, got %d", policy->coarse);
  if (policy->coarse && policy->fine_read)
    return fail(TAO_ERR_ARG, "the coarse value branch is served with the normalised fine read (fine_read 0)");
  const void* ptrs[] = {q, k, v, raw_q, raw_k, fusion_a, fusion_b, out, workspace};
  for (const void* p : ptrs)
    if (!p) return fail(TAO_ERR_ARG, "null tensor pointer");
  for (const void* p : {q, k, v, raw_q, raw_k, (const void*)out})
    if (!aligned16(p)) return fail(TAO_ERR_ARG, "token tensors must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(TAO_ERR_ARG, "workspace must be 256-byte aligned");

  int route_cap = -1, pmax = 1, mbound = 1;
  for (int r = 0; r < n_states; ++r) {
    const long long pos = host_pos[r];
    if (pos < 0) return fail(TAO_ERR_POSITION, "negative position");
    const long long start = h_window_start(pos);
    if (pos + tokens - start > 768)
      return fail(TAO_ERR_SEAL, "chunk crosses a fine seal boundary");
    const int S = h_sealed_at(pos);
    const bool seal = (pos + tokens - start) == 768;
    const int cap = host_cap[r];
    if (cap <= 0 || cap % 8) return fail(TAO_ERR_ARG, "fine capacity must be a positive multiple of 8");
    if (S + (seal ? 1 : 0) > cap)
      return fail(TAO_ERR_CAPACITY, "fine bank capacity %d too small for %d fines", cap, S + 1);
    const int pm = cap / 8 + 1;
    if (pm > pmax) pmax = pm;
    const int mb = h_budget(cap, *policy);
    if (mb > mbound) mbound = mb;
  }
  route_cap = policy->route_cap;
  if (route_cap <= 0) return fail(TAO_ERR_ARG, "policy.route_cap must be positive");
  if (mbound > route_cap) mbound = route_cap;
  const size_t prep_smem = (size_t)width * 4 + (size_t)pmax * 4 + (size_t)(8 * pmax + 8) * 8 + (size_t)pmax * 8;
  if (prep_smem > 200 * 1024) return fail(TAO_ERR_CAPACITY, "fine capacity too large for the route kernel");

  const int fpc = fpc_for(width);
  const Layout L = make_layout(n_states, tokens, heads, width, route_cap, (mbound + fpc - 1) / fpc,
                               policy->route_period, policy->fine_read != 0, policy->coarse != 0);
  if (workspace_bytes < L.total)
    return fail(TAO_ERR_ARG, "workspace too small: %zu < %zu", workspace_bytes, L.total);

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  tao::StepArgs a{};
  a.states = reinterpret_cast<TaoState* const*>(states);
  a.R = n_states;
  a.w = tokens;
  a.H = heads;
  a.pol = {policy->route_period, policy->layer_stagger, policy->budget_root_scale, policy->budget_offset};
  a.q = static_cast<const tao::bf16*>(q);
  a.k = static_cast<const tao::bf16*>(k);
  a.v = static_cast<const tao::bf16*>(v);
  a.raw_q = static_cast<const tao::bf16*>(raw_q);
  a.raw_k = static_cast<const tao::bf16*>(raw_k);
  a.fa = static_cast<const tao::bf16*>(fusion_a);
  a.fb = static_cast<const tao::bf16*>(fusion_b);
  a.gain = bf16_round(2.0f * alpha);
  a.out = static_cast<tao::bf16*>(out);
  a.err = reinterpret_cast<int*>(ws + L.err);
  a.nslot = L.nslot;
  a.route_cap = route_cap;
  a.slot_ids = reinterpret_cast<int32_t*>(ws + L.slot_ids);
  a.slot_pages = reinterpret_cast<int32_t*>(ws + L.slot_pages);
  a.slot_n = reinterpret_cast<int32_t*>(ws + L.slot_n);
  a.kblocks = L.kblocks;
  a.msplit = L.msplit;
  a.local_part = reinterpret_cast<float*>(ws + L.local_part);
  a.local_out = reinterpret_cast<tao::bf16*>(ws + L.local_out);
  a.fine_part = reinterpret_cast<float*>(ws + L.fine_part);
  a.pmax = pmax;
  a.feature = policy->fine_read;
  a.coarse = policy->coarse;
  a.coarse_out = reinterpret_cast<tao::bf16*>(ws + L.coarse_out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return width == 64 ? launch_step<64>(a, L, s) : launch_step<128>(a, L, s);
}

int tao_event_create(void** event) {
  if (!event) return fail(TAO_ERR_ARG, "null event slot");
  cudaEvent_t e;
  cudaError_t err = cudaEventCreate(&e);
  if (err != cudaSuccess) return fail(TAO_ERR_CUDA, "event create: %s", cudaGetErrorString(err));
  *event = e;
  return TAO_OK;
}

int tao_event_destroy(void* event) {
  if (event) cudaEventDestroy(static_cast<cudaEvent_t>(event));
  return TAO_OK;
}

int tao_event_record(void* event, void* stream) {
  cudaError_t err = cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return fail(TAO_ERR_CUDA, "event record: %s", cudaGetErrorString(err));
  return TAO_OK;
}

int tao_event_elapsed(void* start, void* stop, float* ms) {
  cudaError_t err = cudaEventSynchronize(static_cast<cudaEvent_t>(stop));
  if (err == cudaSuccess)
    err = cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(stop));
  if (err != cudaSuccess) return fail(TAO_ERR_CUDA, "event elapsed: %s", cudaGetErrorString(err));
  return TAO_OK;
}

int tao_stream_profile_next(void* start, void* stop) {
  std::lock_guard<std::mutex> lock(g_prof_mutex);
  g_prof_start = static_cast<cudaEvent_t>(start);
  g_prof_stop = static_cast<cudaEvent_t>(stop);
  return TAO_OK;
}

int tao_decode_variant(int variant) {
  if (variant < 0 || variant > 4) return fail(TAO_ERR_ARG, "decode variant must be 0, 1, 2, 3 or 4");
  g_decode_variant = variant;
  return TAO_OK;
}

int tao_stream_check(void* workspace, int* flags, void* stream) {
  if (!workspace) return fail(TAO_ERR_ARG, "null workspace");
  int host = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&host, workspace, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && host) e = cudaMemsetAsync(workspace, 0, sizeof(int), s);
  if (e != cudaSuccess) return fail(TAO_ERR_CUDA, "check: %s", cudaGetErrorString(e));
  if (flags) *flags = host;
  if (host) return fail(TAO_ERR_DEVICE, "device error flags 0x%x", host);
  return TAO_OK;
}

}  // extern "C"

namespace {

template <int D>
__global__ void ring_copy_kernel(tao::bf16* ring, tao::bf16* flat, int H, long long first, int count,
                                 int to_flat) {
  // flat [count][H][D] <-> ring [H][768][D]
  const long long n = (long long)count * H * (D / 8);
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(idx % (D / 8));
    const int h = (int)((idx / (D / 8)) % H);
    const long long t = idx / ((long long)(D / 8) * H);
    uint4* rp = reinterpret_cast<uint4*>(ring + ((long long)h * tao::kWindow + (first + t) % tao::kWindow) * D) + c;
    uint4* fp = reinterpret_cast<uint4*>(flat + (t * H + h) * D) + c;
    if (to_flat) *fp = *rp; else *rp = *fp;
  }
}

int ring_copy(void* ring, void* flat, int heads, int width, long long first, int count, int to_flat,
              void* stream) {
  if (!ring || !flat || heads <= 0 || count < 0 || count > 768 || first < 0)
    return fail(TAO_ERR_ARG, "bad ring copy arguments");
  if (width != 64 && width != 128) return fail(TAO_ERR_ARG, "head width must be 64 or 128");
  if (count == 0) return TAO_OK;
  const long long n = (long long)count * heads * (width / 8);
  const int blocks = (int)((n + 255) / 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (width == 64)
    ring_copy_kernel<64><<<blocks, 256, 0, s>>>((tao::bf16*)ring, (tao::bf16*)flat, heads, first, count, to_flat);
  else
    ring_copy_kernel<128><<<blocks, 256, 0, s>>>((tao::bf16*)ring, (tao::bf16*)flat, heads, first, count, to_flat);
  return check_launch("ring_copy_kernel");
}

}  // namespace

extern "C" {

int tao_ring_gather(const void* ring, int heads, int width, int64_t first_position, int count,
                    void* out, void* stream) {
  return ring_copy(const_cast<void*>(ring), out, heads, width, first_position, count, 1, stream);
}

int tao_ring_scatter(void* ring, int heads, int width, int64_t first_position, int count,
                     const void* in, void* stream) {
  return ring_copy(ring, const_cast<void*>(in), heads, width, first_position, count, 0, stream);
}

namespace {
int memo_rebuild(void* state, int heads, int width, int sealed, int weights_only, void* stream) {
  if (!state || heads <= 0 || sealed < 0) return fail(TAO_ERR_ARG, "bad memo rebuild arguments");
  if (width != 64 && width != 128) return fail(TAO_ERR_ARG, "head width must be 64 or 128");
  if (sealed == 0) return TAO_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (width == 64)
    tao::memo_rebuild_kernel<64><<<heads, 256, 0, s>>>(static_cast<TaoState*>(state), sealed, weights_only);
  else
    tao::memo_rebuild_kernel<128><<<heads, 256, 0, s>>>(static_cast<TaoState*>(state), sealed, weights_only);
  return check_launch("memo_rebuild_kernel");
}
}  // namespace

int tao_state_rebuild_memo(void* state, int heads, int width, int sealed, void* stream) {
  return memo_rebuild(state, heads, width, sealed, 0, stream);
}

int tao_state_refresh_page_weights(void* state, int heads, int width, int sealed, void* stream) {
  return memo_rebuild(state, heads, width, sealed, 1, stream);
}

int tao_window_attention(const void* q, const void* k, const void* v, void* out, float* lse,
                         int batch, int tokens, int heads, int width, void* stream) {
  if (!q || !k || !v || !out || batch <= 0 || tokens <= 0 || heads <= 0)
    return fail(TAO_ERR_ARG, "bad window attention arguments");
  if (width != 64 && width != 128) return fail(TAO_ERR_ARG, "head width must be 64 or 128");
  for (const void* p : {q, k, v, (const void*)out})
    if (!aligned16(p)) return fail(TAO_ERR_ARG, "tensors must be 16-byte aligned");
  int rc = tao::launch_window_attention(static_cast<const tao::bf16*>(q), static_cast<const tao::bf16*>(k),
                                         static_cast<const tao::bf16*>(v), static_cast<tao::bf16*>(out), lse,
                                         batch, tokens, heads, width, nullptr, static_cast<cudaStream_t>(stream));
  if (rc) return rc;
  return check_launch("window_attention_kernel");
}

}  // extern "C"
