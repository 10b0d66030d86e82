// Streaming prefill/decode kernels for the TaoMemory operator on sm_100a.
//
// One call of tao_stream_step advances R requests by w tokens (w == 1: decode).
// Everything that depends on the cursor (sealed fines, pages, refresh anchors,
// seal point) is derived on the device from TaoState.position, so one captured
// CUDA graph of a decode step replays correctly across seals and refreshes.
//
//   prep      : append k/v/raw_k to the ring; copy the current route ids to
//               slot 0; route each refresh anchor of the chunk into slot j
//               (tao_stream.py:196-227, 310-357)
//   main      : decode: split-K local attention + split-M selected fine read
//               (query_fresh_fine.py:8-49), HBM-bound, bulk copies into smem
//   prefill   : window attention (tensor cores) + fine read per 16-query tile
//   coarse    : coarse value branch only: every query reads the matrices of all
//               completed pages (tao_stream.py:299-305)
//   finalize  : combine partials, fine = bf16(bf16(num)/bf16(den)), pointwise
//               fusion (fusion_pointwise.py:10-92), commit routes, seal the
//               oldest block when the window reaches 768 (tao_stream.py:56-77,
//               435-512), refresh the page memo (tao_stream.py:399-416), close a
//               coarse page (tao_stream.py:486-500), advance
#pragma once
#include "../../include/tao_b200.h"
#include "common.cuh"

namespace tao {

struct StepArgs {
  TaoState* const* states;  // device array [R]
  int R, w, H;
  Policy pol;
  const bf16 *q, *k, *v, *raw_q, *raw_k;  // [R][w][H][D]
  const bf16 *fa, *fb;                    // [H][D][3]
  float gain;                             // bf16(2 alpha) as float
  bf16* out;                              // [R][w][H][D]
  // workspace carve-out
  int* err;
  int nslot, route_cap;
  int32_t* slot_ids;    // [R][H][nslot][route_cap]
  int32_t* slot_pages;  // [R][H][nslot][route_cap]
  int32_t* slot_n;      // [R][nslot][2]  (M, K)
  int kblocks;          // decode: key blocks per (r,h)
  int msplit;           // fine partials per query
  float* local_part;    // decode: [R][H][kblocks][D+2]
  bf16* local_out;      // prefill: [R][w][H][D]
  float* fine_part;     // [R][w][H][msplit][D+1]
  int pmax;             // max pages over the batch (smem sizing)
  int feature;          // 1: feature-mass read of the selected fines (TaoPolicy.fine_read)
  int coarse;           // 1: coarse value branch (TaoPolicy.coarse)
  bf16* coarse_out;     // coarse branch: [R][w][H][D] coarse read of the chunk's queries
  // host-staged decode (tao_decode_step_host): the route kernel first copies h_vecs
  // 16-byte vectors of the step's operands from page-locked host memory into the stage
  const uint4* h_in;
  uint4* h_stage;
  int h_vecs;
  // completion word of a host-staged step (null: none): once every output row of the
  // step is in host memory the fused kernel stores the step's sequence number (kept in
  // done[1]; done[0] counts the (request, head) rows finished) into *host_done
  int* done;
  int* host_done;
};

// Position-derived plan of one chunk (constant history inside a chunk).
struct Plan {
  long long t0;
  int S, completed, pending, P;
  long long start;
  bool seal;
};
TAO_DEVI Plan make_plan(const TaoState& st, int w) {
  Plan pl;
  pl.t0 = st.position;
  pl.S = sealed_at(pl.t0);
  pl.completed = pl.S / kGroup;
  pl.pending = pl.S % kGroup;
  pl.P = pl.completed + (pl.pending > 0);
  pl.start = window_start(pl.t0);
  pl.seal = (pl.t0 + w - pl.start) == kWindow;
  return pl;
}
// Route slot of the query at absolute position t: number of refresh anchors in
// [t0, t] (0 = the routes stored in the state).
TAO_DEVI int slot_of(long long t0, long long t, int layer, const Policy& pol) {
  int n = 0;
  for (long long x = t0; x <= t; ++x) n += is_refresh(x, layer, pol);
  return n;
}

// Bounded wait taken by thread 0 and broadcast, so that every thread of the
// CTA leaves together on a timeout (no divergent exit before a barrier).
TAO_DEVI bool wait_uniform(uint64_t* bar, uint32_t phase, int* err, int* flag) {
  if (threadIdx.x == 0) *flag = mbar_wait(bar, phase, err) ? 1 : 0;
  __syncthreads();
  const bool ok = *flag != 0;
  if (ok) {
    while (!mbar_try_wait(bar, phase)) {
    }  // already complete: one poll
  }
  return ok;
}

template <int D>
TAO_DEVI const bf16* ring_head(const void* ring, int h) {
  return reinterpret_cast<const bf16*>(ring) + (long long)h * kWindow * D;
}

// ---------------------------------------------------------------------------
// prep
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) prep_kernel(StepArgs a) {
  const int r = blockIdx.x / a.H, h = blockIdx.x % a.H;
  TaoState& st = *a.states[r];
  const Plan pl = make_plan(st, a.w);
  const int tid = threadIdx.x;
  const long long base = ((long long)r * a.H + h) * a.nslot;

  if (blockIdx.y == 0) {
    // append the chunk's k, v, raw_k (16-byte vectors)
    constexpr int CH = D / 8;
    bf16* kr = reinterpret_cast<bf16*>(st.k_ring) + (long long)h * kWindow * D;
    bf16* vr = reinterpret_cast<bf16*>(st.v_ring) + (long long)h * kWindow * D;
    bf16* rr = reinterpret_cast<bf16*>(st.rk_ring) + (long long)h * kWindow * D;
    for (int idx = tid; idx < a.w * CH; idx += blockDim.x) {
      int i = idx / CH, c = idx % CH;
      long long src = (((long long)r * a.w + i) * a.H + h) * D + c * 8;
      long long dst = ((pl.t0 + i) % kWindow) * D + c * 8;
      *reinterpret_cast<uint4*>(kr + dst) = *reinterpret_cast<const uint4*>(a.k + src);
      *reinterpret_cast<uint4*>(vr + dst) = *reinterpret_cast<const uint4*>(a.v + src);
      *reinterpret_cast<uint4*>(rr + dst) = *reinterpret_cast<const uint4*>(a.raw_k + src);
    }
    // slot 0: routes currently stored in the state (a state holding more routes
    // than this call's slots is flagged and read with no fines, never copied past
    // the slot)
    int n = st.n_route, kc = st.n_chosen;
    if (n > a.route_cap || kc > a.route_cap || n > st.route_cap || kc > st.route_cap) {
      if (tid == 0) atomicOr(a.err, kErrRouteCap);
      n = kc = 0;
    }
    for (int m = tid; m < n; m += blockDim.x)
      a.slot_ids[base * a.route_cap + m] = st.route_ids[(long long)h * st.route_cap + m];
    for (int m = tid; m < kc; m += blockDim.x)
      a.slot_pages[base * a.route_cap + m] = st.route_pages[(long long)h * st.route_cap + m];
    if (h == 0 && tid == 0) {
      a.slot_n[((long long)r * a.nslot) * 2] = n;
      a.slot_n[((long long)r * a.nslot) * 2 + 1] = kc;
    }
    return;
  }

  // ---- refresh anchor number (blockIdx.y - 1) of this chunk
  if (pl.S == 0) return;
  const int want = blockIdx.y - 1;
  long long anchor = -1;
  {
    int seen = 0;
    for (int i = 0; i < a.w; ++i) {
      if (is_refresh(pl.t0 + i, st.layer_index, a.pol)) {
        if (seen == want) { anchor = pl.t0 + i; break; }
        ++seen;
      }
    }
  }
  if (anchor < 0) return;
  const int slot = want + 1;
  const int ai = (int)(anchor - pl.t0);

  extern __shared__ __align__(128) uint8_t dsm[];
  float* hq = reinterpret_cast<float*>(dsm);                   // [D]
  float* pm = hq + D;                                          // page mass [pmax]
  float* cm = pm + a.pmax;                                     // candidate mass [8*pmax+8]
  int* cand_id = reinterpret_cast<int*>(cm + 8 * a.pmax + 8);  // [8*pmax+8]
  int* chosen = cand_id + 8 * a.pmax + 8;                      // [pmax]
  int* sorted = chosen + a.pmax;                               // [pmax]

  const int warp = tid >> 5, lane = tid & 31, nwarp = blockDim.x >> 5;
  const bf16* pz = reinterpret_cast<const bf16*>(st.page_z) + (long long)h * (st.cap_fines / kGroup + 1) * D;
  const bf16* pw = reinterpret_cast<const bf16*>(st.page_w) + (long long)h * (st.cap_fines / kGroup + 1) * D;
  const bf16* fz = reinterpret_cast<const bf16*>(st.fine_z) + (long long)h * st.cap_fines * D;

  // h = bf16(softmax_d(raw_q[anchor]))
  if (warp == 0) {
    const bf16* x = a.raw_q + (((long long)r * a.w + ai) * a.H + h) * D;
    float vals[D / 32];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
      vals[j] = bf(x[lane + 32 * j]);
      mx = fmaxf(mx, vals[j]);
    }
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
      vals[j] = expf(vals[j] - mx);
      s += vals[j];
    }
    s = warp_sum(s);
#pragma unroll
    for (int j = 0; j < D / 32; ++j) hq[lane + 32 * j] = rb(__fdiv_rn(vals[j], s));
  }
  __syncthreads();

  const Counts cnt = routed_counts(pl.completed, pl.pending, a.pol);
  const int K = cnt.coarse, U = cnt.eligible, M = cnt.selected;
  if (M > a.route_cap || pl.P > a.pmax) {
    if (tid == 0) atomicOr(a.err, kErrRouteCap);
    if (h == 0 && tid == 0) {
      a.slot_n[((long long)r * a.nslot + slot) * 2] = 0;
      a.slot_n[((long long)r * a.nslot + slot) * 2 + 1] = 0;
    }
    return;
  }

  // page masses over completed pages: bf16(sum_d bf16(h*pw))
  if (K > 0) {
    for (int p = warp; p < pl.completed; p += nwarp) {
      float s = 0.f;
      for (int d = lane; d < D; d += 32) s += rb(__fmul_rn(hq[d], bf(pw[(long long)p * D + d])));
      s = warp_sum(s);
      if (lane == 0) pm[p] = rb(s);
    }
    __syncthreads();
    // stable top-K (ties -> lower page), then ascending page order
    for (int p = tid; p < pl.completed; p += blockDim.x) {
      float v = pm[p];
      int rank = 0;
      for (int q = 0; q < pl.completed; ++q) {
        float u = pm[q];
        rank += (u > v) || (u == v && q < p);
      }
      if (rank < K) chosen[rank] = p;
    }
    __syncthreads();
    for (int j = tid; j < K; j += blockDim.x) {
      int pg = chosen[j], pos = 0;
      for (int i = 0; i < K; ++i) pos += chosen[i] < pg;
      sorted[pos] = pg;
    }
    __syncthreads();
    for (int j = tid; j < K; j += blockDim.x) chosen[j] = sorted[j];
    __syncthreads();
  }
  // candidate list: 8 fines of each chosen page, then the pending fines
  for (int u = tid; u < U; u += blockDim.x) {
    cand_id[u] = (u < kGroup * K) ? chosen[u / kGroup] * kGroup + (u % kGroup)
                                  : pl.completed * kGroup + (u - kGroup * K);
  }
  __syncthreads();
  // candidate mass: bf16(sum_d bf16(bf16(h*pw[page]) * bf16(exp(bf16(z - pz[page])))))
  for (int u = warp; u < U; u += nwarp) {
    int id = cand_id[u], page = id / kGroup;
    float s = 0.f;
    for (int d = lane; d < D; d += 32) {
      float hv = rb(__fmul_rn(hq[d], bf(pw[(long long)page * D + d])));
      float w = rb(expf(rb(__fsub_rn(bf(fz[(long long)id * D + d]), bf(pz[(long long)page * D + d])))));
      s += rb(__fmul_rn(hv, w));
    }
    s = warp_sum(s);
    if (lane == 0) cm[u] = rb(s);
  }
  __syncthreads();
  int32_t* ids = a.slot_ids + (base + slot) * a.route_cap;
  int32_t* pgs = a.slot_pages + (base + slot) * a.route_cap;
  for (int u = tid; u < U; u += blockDim.x) {
    float v = cm[u];
    int rank = 0;
    for (int q = 0; q < U; ++q) {
      float x = cm[q];
      rank += (x > v) || (x == v && q < u);
    }
    if (rank < M) ids[rank] = cand_id[u];
  }
  for (int j = tid; j < K; j += blockDim.x) pgs[j] = chosen[j];
  if (h == 0 && tid == 0) {
    a.slot_n[((long long)r * a.nslot + slot) * 2] = M;
    a.slot_n[((long long)r * a.nslot + slot) * 2 + 1] = K;
  }
}

// ---------------------------------------------------------------------------
// decode main: blockIdx.y < kblocks -> local attention key block,
//              else -> selected-fine group (FPC fines)
// ---------------------------------------------------------------------------
template <int D>
struct DecodeCfg {
  static constexpr int SLOTS = (D == 64) ? 128 : 64;  // keys per local block (32 KB K+V)
  static constexpr int FPC = (D == 64) ? 4 : 1;       // fines per CTA (32 KB of C)
  static constexpr int KBLOCKS = kWindow / SLOTS;
};

template <int D>
__global__ void __launch_bounds__(128) decode_main_kernel(StepArgs a) {
  using Cfg = DecodeCfg<D>;
  const int r = blockIdx.x / a.H, h = blockIdx.x % a.H;
  const TaoState& st = *a.states[r];
  const Plan pl = make_plan(st, 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ int wflag;
  __shared__ float qv[D];
  __shared__ float red[128 + 8];

  if (blockIdx.y < a.kblocks) {
    // ------------------------------------------------ local attention block
    const int kb = blockIdx.y;
    const long long t = pl.t0;
    const int tm = (int)(t % kWindow);
    float* part = a.local_part + (((long long)r * a.H + h) * a.kblocks + kb) * (D + 2);
    // valid slots: position p(s) = t - ((tm - s) mod 768) >= start
    const int s0 = kb * Cfg::SLOTS;
    auto slot_pos = [&](int s) -> long long { return t - (long long)((tm - s + kWindow) % kWindow); };
    bool any = false;
    {
      // the window is contiguous in position; a block has a valid slot iff
      // one of its slots maps into [start, t]
      long long count = t - pl.start + 1;  // keys in window
      // slot s is valid iff (tm - s) mod 768 < count
      int d0 = (tm - s0 + kWindow) % kWindow;             // distance of first slot
      int d1 = (tm - (s0 + Cfg::SLOTS - 1) + kWindow) % kWindow;
      // distances over the block form at most two decreasing runs; test ends
      any = (d0 < count) || (d1 < count) || (tm >= s0 && tm < s0 + Cfg::SLOTS);
    }
    if (!any) {
      if (tid == 0) { part[D] = -INFINITY; part[D + 1] = 0.f; }
      return;
    }
    bf16* sk = reinterpret_cast<bf16*>(dsm);
    bf16* sv = sk + Cfg::SLOTS * D;
    if (tid == 0) {
      mbar_init(&bar, 1);
      fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
      const uint32_t bytes = Cfg::SLOTS * D * 2;
      mbar_expect_tx(&bar, 2 * bytes);
      bulk_g2s(sk, ring_head<D>(st.k_ring, h) + (long long)s0 * D, bytes, &bar);
      bulk_g2s(sv, ring_head<D>(st.v_ring, h) + (long long)s0 * D, bytes, &bar);
    }
    const float sl = 1.4426950408889634f / sqrtf((float)D);
    const bf16* qrow = a.q + ((long long)r * a.H + h) * D;
    for (int d = tid; d < D; d += 128) qv[d] = bf(qrow[d]) * sl;
    __syncthreads();
    if (!wait_uniform(&bar, 0, a.err, &wflag)) return;
    // scores: D=64 -> one key per thread; D=128 -> two threads per key
    constexpr int TPK = 128 / Cfg::SLOTS;  // threads per key (1 or 2)
    const int key = tid / TPK, part_id = tid % TPK;
    float sc = 0.f;
    {
      const bf16* kr = sk + key * D;
      constexpr int NCH = D / 8 / TPK;
#pragma unroll
      for (int i = 0; i < NCH; ++i) {
        int c = part_id * NCH + ((i + key) % NCH);  // rotate chunks: conflict-free
        uint4 u = *reinterpret_cast<const uint4*>(kr + c * 8);
        float f[8];
        unpack8(u, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) sc += f[e] * qv[c * 8 + e];
      }
      if (TPK == 2) sc += __shfl_xor_sync(0xffffffffu, sc, 1);
    }
    const long long kp = slot_pos(s0 + key);
    if (kp < pl.start || kp > t) sc = -INFINITY;
    // block max / sum over keys
    float mx = warp_max(sc);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float pkey = (sc == -INFINITY) ? 0.f : exp2f(sc - mx);
    float ls = warp_sum(part_id == 0 ? pkey : 0.f);
    __syncthreads();
    if (lane == 0) red[warp] = ls;
    // stash p per key for the P*V pass
    float* pk = red + 8;  // [SLOTS] (<=128)
    if (part_id == 0) pk[key] = pkey;
    __syncthreads();
    const float lsum = red[0] + red[1] + red[2] + red[3];
    // acc[e] = sum_j p_j v_j[e]: thread -> (e chunk, key group)
    constexpr int ECH = D / 8;                 // 8 or 16 chunks
    constexpr int KG = 128 / ECH;              // 16 or 8 key groups
    constexpr int KPG = Cfg::SLOTS / KG;       // 8 keys per group
    const int ec = tid % ECH, kg = tid / ECH;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < KPG; ++i) {
      int j = kg * KPG + i;
      float pj = pk[j];
      uint4 u = *reinterpret_cast<const uint4*>(sv + j * D + ec * 8);
      float f[8];
      unpack8(u, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += pj * f[e];
    }
    // reduce over key groups through shared memory (reuse the K buffer)
    __syncthreads();
    float* rs = reinterpret_cast<float*>(dsm);  // [KG][D]
#pragma unroll
    for (int e = 0; e < 8; ++e) rs[kg * D + ec * 8 + e] = acc[e];
    __syncthreads();
    for (int d = tid; d < D; d += 128) {
      float s = 0.f;
      for (int g2 = 0; g2 < KG; ++g2) s += rs[g2 * D + d];
      part[d] = s;
    }
    if (tid == 0) { part[D] = mx; part[D + 1] = lsum; }
    return;
  }

  // -------------------------------------------------- selected fine group
  if (pl.S == 0) return;
  const int ms = blockIdx.y - a.kblocks;
  const int slot = is_refresh(pl.t0, st.layer_index, a.pol) ? 1 : 0;
  const long long sbase = ((long long)r * a.H + h) * a.nslot + slot;
  const int M = a.slot_n[((long long)r * a.nslot + slot) * 2];
  const int m0 = ms * Cfg::FPC;
  if (m0 >= M) return;
  const int nf = min(Cfg::FPC, M - m0);
  const int32_t* ids = a.slot_ids + sbase * a.route_cap + m0;
  const long long pstride = (long long)(st.cap_fines / kGroup + 1) * D;
  const bf16* fc = reinterpret_cast<const bf16*>(st.fine_c) + (long long)h * st.cap_fines * D * D;
  const bf16* fz = reinterpret_cast<const bf16*>(st.fine_z) + (long long)h * st.cap_fines * D;
  const bf16* pz = reinterpret_cast<const bf16*>(st.page_z) + h * pstride;
  const bf16* pw = reinterpret_cast<const bf16*>(st.page_w) + h * pstride;
  bf16* sc_ = reinterpret_cast<bf16*>(dsm);                          // [FPC][D][D]
  float* ch = reinterpret_cast<float*>(dsm + Cfg::FPC * D * D * 2);   // [FPC][D]
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint32_t bytes = D * D * 2;
    mbar_expect_tx(&bar, nf * bytes);
    for (int i = 0; i < nf; ++i) bulk_g2s(sc_ + i * D * D, fc + (long long)ids[i] * D * D, bytes, &bar);
  }
  // h = bf16(softmax(raw_q)), one warp
  if (warp == 0) {
    const bf16* x = a.raw_q + ((long long)r * a.H + h) * D;
    float vals[D / 32];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) { vals[j] = bf(x[lane + 32 * j]); mx = fmaxf(mx, vals[j]); }
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) { vals[j] = expf(vals[j] - mx); s += vals[j]; }
    s = warp_sum(s);
#pragma unroll
    for (int j = 0; j < D / 32; ++j) qv[lane + 32 * j] = rb(__fdiv_rn(vals[j], s));
  }
  __syncthreads();
  // channels: ch = bf16(bf16(h*pw[page]) * bf16(exp(bf16(z - pz[page])))); den part
  float den = 0.f;
  for (int i = warp; i < nf; i += 4) {
    int id = ids[i], page = id / kGroup;
    float s = 0.f;
    for (int d = lane; d < D; d += 32) {
      float hv = rb(__fmul_rn(qv[d], bf(pw[(long long)page * D + d])));
      float w = rb(expf(rb(__fsub_rn(bf(fz[(long long)id * D + d]), bf(pz[(long long)page * D + d])))));
      float c = rb(__fmul_rn(hv, w));
      ch[i * D + d] = c;
      s += c;
    }
    s = warp_sum(s);
    if (lane == 0) red[i] = rb(s);
  }
  __syncthreads();
  if (tid == 0) for (int i = 0; i < nf; ++i) den += red[i];
  if (!wait_uniform(&bar, 0, a.err, &wflag)) return;
  // acc[e] = sum_i sum_d ch[i][d] * C_i[d][e]
  constexpr int ECH = D / 8;
  constexpr int RG = 128 / ECH;   // row groups: 16 (D64) or 8 (D128)
  constexpr int RPG = D / RG;     // rows per group: 4 or 16
  const int ec = tid % ECH, rg = tid / ECH;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int i = 0; i < nf; ++i) {
    const bf16* cm = sc_ + i * D * D;
#pragma unroll
    for (int j = 0; j < RPG; ++j) {
      int d = rg * RPG + j;
      float c = ch[i * D + d];
      uint4 u = *reinterpret_cast<const uint4*>(cm + d * D + ec * 8);
      float f[8];
      unpack8(u, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += c * f[e];
    }
  }
  __syncthreads();
  float* rs = reinterpret_cast<float*>(dsm);  // reuse C buffer: [RG][D]
#pragma unroll
  for (int e = 0; e < 8; ++e) rs[rg * D + ec * 8 + e] = acc[e];
  __syncthreads();
  float* part = a.fine_part + (((long long)r * a.H + h) * a.msplit + ms) * (D + 1);
  for (int d = tid; d < D; d += 128) {
    float s = 0.f;
    for (int g2 = 0; g2 < RG; ++g2) s += rs[g2 * D + d];
    part[d] = s;
  }
  if (tid == 0) part[D] = den;
}

// ---------------------------------------------------------------------------
// prefill fine read: one CTA per (r,h, 16-query tile); C streamed through a
// double-buffered shared-memory pipeline (bulk copies).
// a.feature == 0: normalised association read (query_fresh_fine.py:8-49),
//   channel = bf16(bf16(h*page_w) * bf16(exp(bf16(z - page_z)))), partial numerator
//   and denominator per query.
// a.feature == 1: feature-mass read (association_writer.py:43-53 through
//   tao_stream.py:362-367): mass_m = sum_d h_d exp(z_m,d) (fp32), channel =
//   bf16(h * mass_m / sum_m mass_m), numerator only (no denominator).  Also serves
//   w == 1 for that writer.
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(128) prefill_fine_kernel(StepArgs a) {
  constexpr int QT = 16;
  const int r = blockIdx.x / a.H, h = blockIdx.x % a.H;
  const TaoState& st = *a.states[r];
  const Plan pl = make_plan(st, a.w);
  if (pl.S == 0) return;
  const int i0 = blockIdx.y * QT;
  const int nq = min(QT, a.w - i0);
  if (nq <= 0) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int wflag;
  bf16* cbuf = reinterpret_cast<bf16*>(dsm);                      // [2][D][D]
  float* hq = reinterpret_cast<float*>(dsm + 2 * D * D * 2);       // [QT][D]
  float* ch = hq + QT * D;                                         // [QT][D]
  float* wv = ch + QT * D;                                         // [D]
  float* pwv = wv + D;                                             // [D]
  __shared__ float den_s[QT];
  __shared__ float tot_s[QT];  // feature read: total feature mass of each query
  __shared__ int seg_s[QT];

  const long long pstride = (long long)(st.cap_fines / kGroup + 1) * D;
  const bf16* fc = reinterpret_cast<const bf16*>(st.fine_c) + (long long)h * st.cap_fines * D * D;
  const bf16* fz = reinterpret_cast<const bf16*>(st.fine_z) + (long long)h * st.cap_fines * D;
  const bf16* pz = reinterpret_cast<const bf16*>(st.page_z) + h * pstride;
  const bf16* pw = reinterpret_cast<const bf16*>(st.page_w) + h * pstride;

  if (tid < QT) {
    den_s[tid] = 0.f;
    seg_s[tid] = (tid < nq) ? slot_of(pl.t0, pl.t0 + i0 + tid, st.layer_index, a.pol) : -1;
  }
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  // h for each query of the tile (one warp per query, round robin)
  for (int qi = warp; qi < nq; qi += 4) {
    const bf16* x = a.raw_q + (((long long)r * a.w + i0 + qi) * a.H + h) * D;
    float vals[D / 32];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) { vals[j] = bf(x[lane + 32 * j]); mx = fmaxf(mx, vals[j]); }
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) { vals[j] = expf(vals[j] - mx); s += vals[j]; }
    s = warp_sum(s);
#pragma unroll
    for (int j = 0; j < D / 32; ++j) hq[qi * D + lane + 32 * j] = rb(__fdiv_rn(vals[j], s));
  }
  __syncthreads();

  // accumulator mapping: thread -> (query qa, 8-column chunk) ; D=64: 16q x 8ch = 128
  constexpr int ECH = D / 8;
  constexpr int QPT = (QT * ECH) / 128;  // queries per thread: 1 (D64) or 2 (D128)
  float acc[QPT][8];
#pragma unroll
  for (int u = 0; u < QPT; ++u)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[u][e] = 0.f;
  const int ec = tid % ECH;
  const int qbase = (tid / ECH) * QPT;

  uint32_t phase[2] = {0, 0};
  const int first_seg = seg_s[0], last_seg = seg_s[nq - 1];
  for (int seg = first_seg; seg <= last_seg; ++seg) {
    const long long sbase = ((long long)r * a.H + h) * a.nslot + seg;
    const int M = a.slot_n[((long long)r * a.nslot + seg) * 2];
    const int32_t* ids = a.slot_ids + sbase * a.route_cap;
    __syncthreads();
    if (tid == 0 && M > 0) {
      mbar_expect_tx(&bars[0], D * D * 2);
      bulk_g2s(cbuf, fc + (long long)ids[0] * D * D, D * D * 2, &bars[0]);
    }
    if (a.feature) {
      // total feature mass over the segment's selected fines, while C_0 is in flight
      for (int qi = warp; qi < nq; qi += 4) {
        if (seg_s[qi] != seg) continue;
        float tot = 0.f;
        for (int m = 0; m < M; ++m) {
          const bf16* zr = fz + (long long)ids[m] * D;
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < D / 32; ++j)
            s += __fmul_rn(hq[qi * D + lane + 32 * j], expf(bf(zr[lane + 32 * j])));
          tot += warp_sum(s);
        }
        if (lane == 0) tot_s[qi] = tot;
      }
    }
    for (int m = 0; m < M; ++m) {
      const int buf = m & 1;
      if (tid == 0 && m + 1 < M) {
        mbar_expect_tx(&bars[buf ^ 1], D * D * 2);
        bulk_g2s(cbuf + (buf ^ 1) * D * D, fc + (long long)ids[m + 1] * D * D, D * D * 2, &bars[buf ^ 1]);
      }
      const int id = ids[m], page = id / kGroup;
      if (!a.feature) {
        for (int d = tid; d < D; d += 128) {
          wv[d] = rb(expf(rb(__fsub_rn(bf(fz[(long long)id * D + d]), bf(pz[(long long)page * D + d])))));
          pwv[d] = bf(pw[(long long)page * D + d]);
        }
      }
      __syncthreads();
      // channels for the tile's queries in this segment
      for (int qi = warp; qi < nq; qi += 4) {
        if (seg_s[qi] != seg) continue;
        if (a.feature) {
          // same per-fine mass as above (same order), then bf16(h * mass / total)
          const bf16* zr = fz + (long long)id * D;
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < D / 32; ++j)
            s += __fmul_rn(hq[qi * D + lane + 32 * j], expf(bf(zr[lane + 32 * j])));
          const float mix = __fdiv_rn(warp_sum(s), tot_s[qi]);
#pragma unroll
          for (int j = 0; j < D / 32; ++j)
            ch[qi * D + lane + 32 * j] = rb(__fmul_rn(mix, hq[qi * D + lane + 32 * j]));
          continue;
        }
        float s = 0.f;
        for (int d = lane; d < D; d += 32) {
          float hv = rb(__fmul_rn(hq[qi * D + d], pwv[d]));
          float c = rb(__fmul_rn(hv, wv[d]));
          ch[qi * D + d] = c;
          s += c;
        }
        s = warp_sum(s);
        if (lane == 0) den_s[qi] += rb(s);
      }
      __syncthreads();
      if (!wait_uniform(&bars[buf], phase[buf], a.err, &wflag)) return;
      phase[buf] ^= 1;
      const bf16* cm = cbuf + buf * D * D;
#pragma unroll
      for (int u = 0; u < QPT; ++u) {
        const int qi = qbase + u;
        if (qi >= nq || seg_s[qi] != seg) continue;
        for (int d = 0; d < D; ++d) {
          float c = ch[qi * D + d];
          uint4 v4 = *reinterpret_cast<const uint4*>(cm + d * D + ec * 8);
          float f[8];
          unpack8(v4, f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[u][e] += c * f[e];
        }
      }
      __syncthreads();  // buffer `buf` is refilled at m + 2
    }
  }
#pragma unroll
  for (int u = 0; u < QPT; ++u) {
    const int qi = qbase + u;
    if (qi >= nq) continue;
    float* part = a.fine_part + ((((long long)r * a.w + i0 + qi) * a.H + h) * a.msplit) * (D + 1);
#pragma unroll
    for (int e = 0; e < 8; ++e) part[ec * 8 + e] = acc[u][e];
    if (ec == 0) part[D] = den_s[qi];
  }
}

// ---------------------------------------------------------------------------
// page memo: page_z[p] = bf16 logsumexp composite over the fines of page p,
// page_w = bf16(softmax over pages per channel)
// ---------------------------------------------------------------------------
template <int D>
TAO_DEVI float page_lse(const bf16* fz, int first, int n, int d) {
  // torch.logsumexp on bf16 (amax, sub, exp, sum, log, add -- each rounded)
  float mx = -INFINITY;
  for (int i = 0; i < n; ++i) mx = fmaxf(mx, bf(fz[(long long)(first + i) * D + d]));
  float m0 = (fabsf(mx) == INFINITY) ? 0.f : mx;
  float s = 0.f;
  for (int i = 0; i < n; ++i) s += rb(expf(rb(__fsub_rn(bf(fz[(long long)(first + i) * D + d]), m0))));
  s = rb(s);
  return rb(__fadd_rn(rb(logf(s)), m0));
}

template <int D>
TAO_DEVI void refresh_memo(const TaoState& st, int h, int S, int p_from) {
  const int P = S / kGroup + (S % kGroup > 0);
  const long long pstride = (long long)(st.cap_fines / kGroup + 1) * D;
  const bf16* fz = reinterpret_cast<const bf16*>(st.fine_z) + (long long)h * st.cap_fines * D;
  bf16* pz = reinterpret_cast<bf16*>(st.page_z) + h * pstride;
  bf16* pw = reinterpret_cast<bf16*>(st.page_w) + h * pstride;
  for (int idx = threadIdx.x; idx < (P - p_from) * D; idx += blockDim.x) {
    int p = p_from + idx / D, d = idx % D;
    int n = min(kGroup, S - p * kGroup);
    pz[(long long)p * D + d] = tobf(page_lse<D>(fz, p * kGroup, n, d));
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float mx = -INFINITY;
    for (int p = 0; p < P; ++p) mx = fmaxf(mx, bf(pz[(long long)p * D + d]));
    float s = 0.f;
    for (int p = 0; p < P; ++p) s += expf(bf(pz[(long long)p * D + d]) - mx);
    for (int p = 0; p < P; ++p) pw[(long long)p * D + d] = tobf(__fdiv_rn(expf(bf(pz[(long long)p * D + d]) - mx), s));
  }
}

// ---------------------------------------------------------------------------
// coarse value branch (TaoPolicy.coarse): page matrices and their read
// ---------------------------------------------------------------------------
// Coarse matrix of completed page p of head h (tao_stream.py:486-500):
// w_s[d] = bf16(exp(bf16(z_s[d] - page_z[p][d]))) for the page's 8 fines, then
// C_page[d][e] = bf16(sum_s w_s[d] * C_s[d][e]) (fp32 sum in fine order, one rounding).
// page_z[p] must be final (written by refresh_memo before a barrier).
template <int D>
TAO_DEVI void build_page_c(const TaoState& st, int h, int p) {
  __shared__ float wts[kGroup * 128];
  const long long pstride = (long long)(st.cap_fines / kGroup + 1) * D;
  const bf16* fz = reinterpret_cast<const bf16*>(st.fine_z) + ((long long)h * st.cap_fines + p * kGroup) * D;
  const bf16* pz = reinterpret_cast<const bf16*>(st.page_z) + h * pstride + (long long)p * D;
  const bf16* fc = reinterpret_cast<const bf16*>(st.fine_c) + ((long long)h * st.cap_fines + p * kGroup) * D * D;
  bf16* pc = reinterpret_cast<bf16*>(st.page_c) + (h * pstride + (long long)p * D) * D;
  for (int idx = threadIdx.x; idx < kGroup * D; idx += blockDim.x) {
    const int sf = idx / D, d = idx % D;
    wts[idx] = rb(expf(rb(__fsub_rn(bf(fz[(long long)sf * D + d]), bf(pz[d])))));
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < D * D / 8; idx += blockDim.x) {
    const int d = idx / (D / 8), e0 = (idx % (D / 8)) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int sf = 0; sf < kGroup; ++sf) {
      const float w = wts[sf * D + d];
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(fc + ((long long)sf * D + d) * D + e0), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(acc[e], __fmul_rn(w, f[e]));
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) ow[e] = bf16x2(acc[2 * e], acc[2 * e + 1]);
    *reinterpret_cast<uint4*>(pc + (long long)d * D + e0) = o;
  }
  __syncthreads();
}

// coarse_w[p][d] = bf16(softmax over the completed pages p < completed of page_z[p][d])
// (tao_stream.py:299: F.softmax(page_z[:, :, :len(pages)], dim=2)).
template <int D>
TAO_DEVI void refresh_coarse_w(const TaoState& st, int h, int completed) {
  const long long pstride = (long long)(st.cap_fines / kGroup + 1) * D;
  const bf16* pz = reinterpret_cast<const bf16*>(st.page_z) + h * pstride;
  bf16* cw = reinterpret_cast<bf16*>(st.coarse_w) + h * pstride;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float mx = -INFINITY;
    for (int p = 0; p < completed; ++p) mx = fmaxf(mx, bf(pz[(long long)p * D + d]));
    float sum = 0.f;
    for (int p = 0; p < completed; ++p) sum += expf(bf(pz[(long long)p * D + d]) - mx);
    for (int p = 0; p < completed; ++p)
      cw[(long long)p * D + d] = tobf(__fdiv_rn(expf(bf(pz[(long long)p * D + d]) - mx), sum));
  }
}

template <int D>
struct CoarseCfg {
  static constexpr int EPT = 16;           // output channels per thread
  static constexpr int EG = D / EPT;       // threads per query row (4 or 8)
  static constexpr int QTMAX = 256 / EG;   // queries per CTA at most (64 or 32)
  static constexpr size_t smem(int qt) { return (size_t)2 * D * D * 2 + (size_t)qt * D * 4 + (size_t)256 * EPT * 4; }
};

// Coarse value read of a chunk's queries (tao_stream.py:299-305):
// coarse[q][e] = bf16(sum_p sum_d bf16(h[q][d] * coarse_w[p][d]) * C_p[d][e]) over the
// completed pages p, with h = bf16(softmax_d(raw_q[q])).  CTA = (request, head) x a
// tile of qt queries (qt a power of two <= QTMAX); the page matrices stream through a
// two-stage shared-memory buffer filled by bulk copies (one per page, mbarrier
// completion, bounded waits).  Thread = (query, 16 output channels, one slice of the
// d range); slices are summed in order through shared memory.
// The history of a chunk is fixed (it seals only after its last query), so the pages
// read are those complete at the chunk's first position.
template <int D>
__global__ void __launch_bounds__(256) coarse_read_kernel(StepArgs a, int qt) {
  using Cfg = CoarseCfg<D>;
  constexpr int EPT = Cfg::EPT, EG = Cfg::EG;
  const int r = blockIdx.x / a.H, h = blockIdx.x % a.H;
  const TaoState& st = *a.states[r];
  const Plan pl = make_plan(st, a.w);
  const int Pc = pl.completed;
  const int q0 = blockIdx.y * qt, nq = min(qt, a.w - q0);
  if (nq <= 0 || Pc == 0) return;
  if (!st.page_c || !st.coarse_w) {   // a state without coarse buffers: reported, nothing read
    if (threadIdx.x == 0) atomicOr(a.err, kErrState);
    return;
  }
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int slices = 256 / (qt * EG);
  const int sl = tid % slices, eg = (tid / slices) % EG, qi = tid / (slices * EG);
  const int dlen = D / slices, d0 = sl * dlen;
  extern __shared__ __align__(128) uint8_t dsm[];
  bf16* cS = reinterpret_cast<bf16*>(dsm);                                // [2][D][D]
  float* hS = reinterpret_cast<float*>(dsm + (size_t)2 * D * D * 2);      // [qt][D]
  float* red = hS + qt * D;                                               // [256][EPT]
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int okflag;
  const long long pstride = (long long)(st.cap_fines / kGroup + 1) * D;
  const bf16* pcb = reinterpret_cast<const bf16*>(st.page_c) + h * pstride * D;
  const bf16* cwb = reinterpret_cast<const bf16*>(st.coarse_w) + h * pstride;
  constexpr uint32_t kPageBytes = D * D * 2;
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    mbar_expect_tx(&bars[0], kPageBytes);
    bulk_g2s(cS, pcb, kPageBytes, &bars[0]);
  }
  // h = bf16(softmax_d(raw_q)) of the tile's queries, one warp per query
  for (int i = warp; i < nq; i += 8) {
    const bf16* x = a.raw_q + (((long long)r * a.w + q0 + i) * a.H + h) * D;
    float vals[D / 32];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
      vals[j] = bf(x[lane + 32 * j]);
      mx = fmaxf(mx, vals[j]);
    }
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
      vals[j] = expf(vals[j] - mx);
      sum += vals[j];
    }
    sum = warp_sum(sum);
#pragma unroll
    for (int j = 0; j < D / 32; ++j) hS[i * D + lane + 32 * j] = rb(__fdiv_rn(vals[j], sum));
  }
  float acc[EPT];
#pragma unroll
  for (int e = 0; e < EPT; ++e) acc[e] = 0.f;
  const bool live = qi < nq;
  uint32_t phase[2] = {0, 0};
  for (int p = 0; p < Pc; ++p) {
    const int buf = p & 1;
    if (tid == 0 && p + 1 < Pc) {   // buffer buf ^ 1 was released by the barrier ending p - 1
      mbar_expect_tx(&bars[buf ^ 1], kPageBytes);
      bulk_g2s(cS + (buf ^ 1) * D * D, pcb + (long long)(p + 1) * D * D, kPageBytes, &bars[buf ^ 1]);
    }
    if (!wait_uniform(&bars[buf], phase[buf], a.err, &okflag)) {
      // give the copy still in flight its bounded wait before the CTA leaves
      if (tid == 0 && p + 1 < Pc) mbar_wait(&bars[buf ^ 1], phase[buf ^ 1], a.err);
      return;
    }
    phase[buf] ^= 1;
    if (live) {
      const bf16* cp = cS + buf * D * D;
      for (int d = d0; d < d0 + dlen; ++d) {
        const float av = rb(__fmul_rn(hS[qi * D + d], bf(cwb[(long long)p * D + d])));
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(cp + d * D + eg * EPT), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(acc[e], __fmul_rn(av, f[e]));
        unpack8(*reinterpret_cast<const uint4*>(cp + d * D + eg * EPT + 8), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[8 + e] = __fadd_rn(acc[8 + e], __fmul_rn(av, f[e]));
      }
    }
    __syncthreads();  // buffer `buf` is refilled at p + 2
  }
#pragma unroll
  for (int e = 0; e < EPT; ++e) red[tid * EPT + e] = acc[e];
  __syncthreads();
  if (live && sl == 0) {
    float sum[EPT];
#pragma unroll
    for (int e = 0; e < EPT; ++e) sum[e] = 0.f;
    for (int k = 0; k < slices; ++k)
#pragma unroll
      for (int e = 0; e < EPT; ++e) sum[e] = __fadd_rn(sum[e], red[(tid + k) * EPT + e]);
    bf16* o = a.coarse_out + (((long long)r * a.w + q0 + qi) * a.H + h) * D + eg * EPT;
#pragma unroll
    for (int e = 0; e < EPT; e += 2) *reinterpret_cast<uint32_t*>(o + e) = bf16x2(sum[e], sum[e + 1]);
  }
}

// Softmax writer for one 256-token block of head h (tao_stream.py:66-76).
template <int D>
TAO_DEVI void seal_block(const TaoState& st, int h, long long block_pos, int S, uint8_t* smem) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int s0 = (int)(block_pos % kWindow);
  const bf16* rk = ring_head<D>(st.rk_ring, h) + (long long)s0 * D;
  const bf16* vv = ring_head<D>(st.v_ring, h) + (long long)s0 * D;
  bf16* prob = reinterpret_cast<bf16*>(smem);            // [256][D]: raw keys, then probabilities
  bf16* vs = prob + kFine * D;                           // [256][D]
  float* mx = reinterpret_cast<float*>(vs + kFine * D);  // [D]
  float* zp = mx + D;                                    // [D] partition
  for (int idx = tid; idx < kFine * D / 8; idx += nt) {
    reinterpret_cast<uint4*>(vs)[idx] = reinterpret_cast<const uint4*>(vv)[idx];
    reinterpret_cast<uint4*>(prob)[idx] = reinterpret_cast<const uint4*>(rk)[idx];
  }
  __syncthreads();
  // per channel: max over tokens, partition = bf16(sum_t bf16(exp(bf16(k - max)))) in token order
  for (int d = tid; d < D; d += nt) {
    float m = -INFINITY;
    for (int t = 0; t < kFine; ++t) m = fmaxf(m, bf(prob[t * D + d]));
    mx[d] = m;
    float s = 0.f;
    for (int t = 0; t < kFine; ++t) s += rb(expf(rb(__fsub_rn(bf(prob[t * D + d]), m))));
    zp[d] = rb(s);
  }
  __syncthreads();
  for (int idx = tid; idx < kFine * D; idx += nt) {
    const int d = idx % D;
    const float e = rb(expf(rb(__fsub_rn(bf(prob[idx]), mx[d]))));
    prob[idx] = tobf(__fdiv_rn(e, zp[d]));
  }
  bf16* zout = reinterpret_cast<bf16*>(st.fine_z) + ((long long)h * st.cap_fines + S) * D;
  for (int d = tid; d < D; d += nt) zout[d] = tobf(__fadd_rn(mx[d], rb(logf(zp[d]))));
  __syncthreads();
  // C[d][e] = sum_t prob[t][d] * v[t][e]
  bf16* cout = reinterpret_cast<bf16*>(st.fine_c) + ((long long)h * st.cap_fines + S) * D * D;
  for (int idx = tid; idx < D * D / 4; idx += nt) {
    int d = idx / (D / 4), e0 = (idx % (D / 4)) * 4;
    float c0 = 0, c1 = 0, c2 = 0, c3 = 0;
    for (int t = 0; t < kFine; ++t) {
      float pr = bf(prob[t * D + d]);
      const __nv_bfloat162* vp = reinterpret_cast<const __nv_bfloat162*>(vs + t * D + e0);
      float2 a0 = __bfloat1622float2(vp[0]), a1 = __bfloat1622float2(vp[1]);
      c0 += pr * a0.x; c1 += pr * a0.y; c2 += pr * a1.x; c3 += pr * a1.y;
    }
    cout[(long long)d * D + e0] = tobf(c0);
    cout[(long long)d * D + e0 + 1] = tobf(c1);
    cout[(long long)d * D + e0 + 2] = tobf(c2);
    cout[(long long)d * D + e0 + 3] = tobf(c3);
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// finalize
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) finalize_kernel(StepArgs a) {
  const int r = blockIdx.x / a.H, h = blockIdx.x % a.H;
  TaoState& st = *a.states[r];
  const Plan pl = make_plan(st, a.w);
  const int tid = threadIdx.x;
  const bool hist = pl.S > 0;
  extern __shared__ __align__(128) uint8_t dsm[];
  using Cfg = DecodeCfg<D>;
  __shared__ int seg_s[kFine];
  if (tid == 0) {
    int n = 0;
    for (int i = 0; i < a.w; ++i) {
      n += is_refresh(pl.t0 + i, st.layer_index, a.pol);
      seg_s[i] = n;
    }
  }
  __syncthreads();

  // ---- outputs
  for (int idx = tid; idx < a.w * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    const long long row = ((long long)r * a.w + i) * a.H + h;
    float local;
    if (a.w == 1 && !a.feature) {
      const float* part = a.local_part + ((long long)r * a.H + h) * a.kblocks * (D + 2);
      float M = -INFINITY;
      for (int b = 0; b < a.kblocks; ++b) M = fmaxf(M, part[b * (D + 2) + D]);
      float L = 0.f, O = 0.f;
      for (int b = 0; b < a.kblocks; ++b) {
        float mb = part[b * (D + 2) + D];
        if (mb == -INFINITY) continue;
        float sc = exp2f(mb - M);
        L += sc * part[b * (D + 2) + D + 1];
        O += sc * part[b * (D + 2) + d];
      }
      local = rb(O / L);
    } else {
      local = bf(a.local_out[row * D + d]);
    }
    float outv = local;
    if (hist) {
      const int seg = seg_s[i];
      const int M = a.slot_n[((long long)r * a.nslot + seg) * 2];
      const int nparts = (a.w == 1 && !a.feature) ? (M + Cfg::FPC - 1) / Cfg::FPC : 1;
      const float* part = a.fine_part + row * a.msplit * (D + 1);
      float acc = 0.f, den = 0.f;
      for (int s = 0; s < nparts; ++s) {
        acc += part[s * (D + 1) + d];
        den += part[s * (D + 1) + D];
      }
      // feature-mass read: bf16 of the fp32 sum, no denominator (association_writer.py:53)
      const float fine = a.feature ? rb(acc) : rb(__fdiv_rn(rb(acc), rb(den)));
      // pointwise fusion, reference cast chain (fusion_pointwise.py:19-92); the
      // coarse term is present once a page is complete in the coarse value branch,
      // and the local bias is then bf16(log 2) (two history terms)
      const bool coarse_on = a.coarse && pl.completed > 0;
      const float q = bf(a.raw_q[row * D + d]);
      const bf16* fa = a.fa + ((long long)h * D + d) * 3;
      const bf16* fb = a.fb + ((long long)h * D + d) * 3;
      float s0 = rb(__fadd_rn(rb(__fmul_rn(bf(fa[0]), q)), bf(fb[0])));
      s0 = rb(__fadd_rn(s0, coarse_on ? kLocalBiasTwo : 0.f));  // local bias log(#history terms)
      const float s1 = coarse_on ? rb(__fadd_rn(rb(__fmul_rn(bf(fa[1]), q)), bf(fb[1]))) : -INFINITY;
      const float s2 = rb(__fadd_rn(rb(__fmul_rn(bf(fa[2]), q)), bf(fb[2])));
      const float mx = fmaxf(fmaxf(s0, s1), s2);
      const float e0 = expf(s0 - mx), e1 = coarse_on ? expf(s1 - mx) : 0.f, e2 = expf(s2 - mx);
      const float sum = (e0 + e1) + e2;
      const float rho0 = rb(__fdiv_rn(e0, sum)), rho2 = rb(__fdiv_rn(e2, sum));
      const float cval = coarse_on ? bf(a.coarse_out[row * D + d]) : 0.f;
      const float rho1 = coarse_on ? rb(__fdiv_rn(e1, sum)) : 0.f;
      const float lt = rb(__fmul_rn(rho0, rb(__fmul_rn(2.f, local))));
      const float ct = rb(__fmul_rn(rho1, rb(__fmul_rn(a.gain, cval))));
      const float ft = rb(__fmul_rn(rho2, rb(__fmul_rn(a.gain, fine))));
      outv = rb(__fadd_rn(rb(__fadd_rn(lt, ct)), ft));
    }
    a.out[row * D + d] = tobf(outv);
  }

  // ---- commit the last route slot of this chunk into the state
  if (hist) {
    const int last = seg_s[a.w - 1];
    if (last > 0) {
      const long long sbase = ((long long)r * a.H + h) * a.nslot + last;
      const int M = a.slot_n[((long long)r * a.nslot + last) * 2];
      const int K = a.slot_n[((long long)r * a.nslot + last) * 2 + 1];
      for (int m = tid; m < M; m += blockDim.x)
        st.route_ids[(long long)h * st.route_cap + m] = a.slot_ids[sbase * a.route_cap + m];
      for (int m = tid; m < K; m += blockDim.x)
        st.route_pages[(long long)h * st.route_cap + m] = a.slot_pages[sbase * a.route_cap + m];
    }
  }

  // ---- seal the oldest block once the window holds 768 tokens
  if (pl.seal) {
    __syncthreads();
    seal_block<D>(st, h, pl.start, pl.S, dsm);
    const int p_from = pl.S / kGroup;  // only the page that received the fine changes
    refresh_memo<D>(st, h, pl.S + 1, p_from);
    if (a.coarse && (pl.S + 1) % kGroup == 0 && st.page_c && st.coarse_w) {
      // the page closed: its coarse matrix and the softmax over completed pages
      __syncthreads();
      build_page_c<D>(st, h, p_from);
      refresh_coarse_w<D>(st, h, p_from + 1);
    }
  }

  // ---- last CTA of this request advances the cursor
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    int old = atomicAdd(&st.arrive, 1);
    if (old == a.H - 1) {
      const int last = hist ? seg_s[a.w - 1] : 0;
      if (last > 0) {
        st.n_route = a.slot_n[((long long)r * a.nslot + last) * 2];
        st.n_chosen = a.slot_n[((long long)r * a.nslot + last) * 2 + 1];
        st.route_refreshes += last;
      }
      if (pl.seal) st.seal_events += 1;
      st.position = pl.t0 + a.w;
      st.arrive = 0;
      __threadfence();
    }
  }
}

// Rebuild page_z / page_w of a state from its fine_z (after import); with
// weights_only, page_z stays as written and only page_w is recomputed.
template <int D>
__global__ void __launch_bounds__(256) memo_rebuild_kernel(TaoState* st, int S, int weights_only) {
  refresh_memo<D>(*st, blockIdx.x, S, weights_only ? S / kGroup + (S % kGroup > 0) : 0);
  if (st->coarse_w && S >= kGroup) {   // coarse value branch: softmax over the completed pages
    __syncthreads();
    refresh_coarse_w<D>(*st, blockIdx.x, S / kGroup);
  }
}

}  // namespace tao
