// Fused single-kernel decode step (one token for each of R requests).
//
// Work items per (request r, head h): KB local-attention key blocks and MS groups
// of selected fines (query_fresh_fine.py:8-49), one CTA per item with its bulk
// copies issued first and the load-independent work (query scaling, h softmax,
// channel weights) done while they are in flight.  Each item writes a partial; the CTA
// that completes the last item of (r, h) combines the partials, applies the
// pointwise fusion (fusion_pointwise.py:10-92) and writes the output; the CTA
// that completes the last head of request r advances its cursor.  Arrival
// counters are TaoState.counters[h] and TaoState.arrive, reset by their last user.
//
// Routing (refresh tokens) and sealing (window full) run as separate small
// kernels that the host launches only on the steps that need them.
//
// Feature-mass read (StepArgs.feature, the feature-read writers): a fine item first
// forms every selected fine's mass sum_d h_d exp(z_m,d) of its (r, h) (the z rows are
// a few KB, L2-resident) and their total, then its own fines' channels
// bf16(h * mass_m / total); its partial has no denominator and the combine rounds
// the sum (association_writer.py:43-53).
#pragma once
#include "stream_kernels.cuh"

namespace tao {

// Feature-mass read: the host refuses batches whose route budget could exceed this.
constexpr int kRouteCapMax = 256;

// Per-request item counts of the fused kernel (requests with fewer selected fines get
// fewer fine items instead of empty ones), for up to kFusedMaxReq requests and
// kFusedMaxSlots items per head; larger batches give every request KB + ms items.
constexpr int kFusedMaxReq = 64;
constexpr int kFusedMaxSlots = 12 + kRouteCapMax;

struct FusedArgs {
  StepArgs s;        // states, shapes, inputs, outputs, policy, partial buffers
  int ms;            // fine items per (r, h) allotted in the partial buffers (their stride)
  // Item order, slot-major: slot s holds one item per head of every request with more
  // than s items per head, requests with more items first.  nslots = 0: every request
  // has KB + ms items per head and item i is (request, head) i % (R H), slot i / (R H).
  int nslots;
  int slot_base[kFusedMaxSlots + 1];  // first item of each slot; slot_base[nslots] = items
  int16_t rorder[kFusedMaxReq];       // requests by items per head, most first
  int16_t per_r[kFusedMaxReq];        // items per head of each request
};

// Item geometry: an item's copies fill one IB-byte stage, either the K and V rows of
// SLOTS ring slots or the C matrices of FPC selected fines.  IB = 32 KB: 128 keys or 4
// fines at width 64, 64 keys or 1 fine at width 128; IB = 16 KB (width 64 only): 64
// keys or 2 fines.
template <int D, int IB = 32768>
struct FusedCfg {
  static constexpr int STAGE = IB;              // bytes per pipeline stage
  static constexpr int SLOTS = IB / (4 * D);    // keys per local block
  static constexpr int FPC = IB / (2 * D * D);  // fines per selected-fine group
  static constexpr int KB = kWindow / SLOTS;    // local blocks per (r, h)
  static_assert(FPC >= 1 && FPC <= 4 && SLOTS >= 64 && SLOTS <= 128, "item geometry");
};

// Item i -> (rh, slot): slots of one (r, h) are spread over the grid.
struct Item {
  int r, h, slot;
};
TAO_DEVI Item item_of(int i, int R, int H) {
  const int rh = i % (R * H);
  return {rh / H, rh % H, i / (R * H)};
}

// Item i of a fused launch.
TAO_DEVI Item fused_item(const FusedArgs& f, int i) {
  if (f.nslots == 0) {
    const int rh = i % (f.s.R * f.s.H);
    return {rh / f.s.H, rh % f.s.H, i / (f.s.R * f.s.H)};
  }
  int lo = 0, hi = f.nslots - 1;  // the last slot starting at or before i
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (f.slot_base[mid] <= i) lo = mid;
    else hi = mid - 1;
  }
  const int j = i - f.slot_base[lo];
  return {f.rorder[j / f.s.H], j % f.s.H, lo};
}

template <int D>
TAO_DEVI bool local_block_live(long long t, long long start, int s0, int slots) {
  const int tm = (int)(t % kWindow);
  if (tm >= s0 && tm < s0 + slots) return true;
  const long long count = t - start + 1;
  const int dist = (tm - (s0 + slots - 1) + kWindow) % kWindow;  // nearest slot of the block
  return dist < count;
}

// Source addresses of one item's bulk copies (resolved ahead of the copy so a CTA
// can issue its next item the moment its stage is free).
template <int D, int IB = 32768>
struct ItemCopy {
  static constexpr int N = FusedCfg<D, IB>::FPC > 2 ? FusedCfg<D, IB>::FPC : 2;
  const void* src[N];
  int id[FusedCfg<D, IB>::FPC];  // selected-fine items: the fine ids (their channel rows are read by id)
  uint32_t bytes;            // per copy
  int n;                     // copies (0: nothing to load)
};

template <int D, int IB>
TAO_DEVI ItemCopy<D, IB> resolve_item(const FusedArgs& f, const Item& it) {
  using Cfg = FusedCfg<D, IB>;
  ItemCopy<D, IB> c;
  c.n = 0;
  c.bytes = 0;
#pragma unroll
  for (int i = 0; i < Cfg::FPC; ++i) c.id[i] = 0;
  const TaoState& st = *f.s.states[it.r];
  const long long t = st.position;
  if (it.slot < Cfg::KB) {
    const int s0 = it.slot * Cfg::SLOTS;
    if (!local_block_live<D>(t, window_start(t), s0, Cfg::SLOTS)) return c;
    c.bytes = Cfg::SLOTS * D * 2;
    c.n = 2;
    c.src[0] = ring_head<D>(st.k_ring, it.h) + (long long)s0 * D;
    c.src[1] = ring_head<D>(st.v_ring, it.h) + (long long)s0 * D;
    return c;
  }
  if (t < kWindow) return c;
  const int m0 = (it.slot - Cfg::KB) * Cfg::FPC;
  const int M = st.n_route;
  if (m0 >= M) return c;
  const int nf = min(Cfg::FPC, M - m0);
  const int32_t* ids = st.route_ids + (long long)it.h * st.route_cap + m0;
  const bf16* fc = reinterpret_cast<const bf16*>(st.fine_c) + (long long)it.h * st.cap_fines * D * D;
  int id[Cfg::FPC];  // all ids first
#pragma unroll
  for (int i = 0; i < Cfg::FPC; ++i) id[i] = i < nf ? ids[i] : 0;
#pragma unroll
  for (int i = 0; i < Cfg::FPC; ++i) {
    c.src[i] = fc + (long long)id[i] * D * D;
    c.id[i] = id[i];
  }
  c.bytes = D * D * 2;
  c.n = nf;
  return c;
}

// Issue the bulk copies of a resolved item into `stage`; returns the bytes armed.
template <int D, int IB>
TAO_DEVI uint32_t issue_copy(const ItemCopy<D, IB>& c, uint8_t* stage, uint64_t* bar) {
  if (c.n == 0) return 0;
  mbar_expect_tx(bar, c.n * c.bytes);
#pragma unroll
  for (int i = 0; i < ItemCopy<D, IB>::N; ++i)
    if (i < c.n) bulk_g2s(stage + i * c.bytes, c.src[i], c.bytes, bar);
  return c.n * c.bytes;
}

// h = bf16(softmax_d(raw_q)) of request r, head h (one warp), into hq[D].
// vals[j] holds channel lane + 32 j (loaded by the caller ahead of other work).
template <int D>
TAO_DEVI void softmax_vals(float (&vals)[D / 32], float* hq, int lane) {
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < D / 32; ++j) mx = fmaxf(mx, vals[j]);
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

template <int D>
TAO_DEVI void softmax_row(const bf16* x, float* hq, int lane) {
  float vals[D / 32];
#pragma unroll
  for (int j = 0; j < D / 32; ++j) vals[j] = bf(x[lane + 32 * j]);
  softmax_vals<D>(vals, hq, lane);
}

// After a wait that gave up: thread 0 gives every other stage's copy still in flight
// its own bounded wait, so no bulk copy outlives the CTA's shared memory.
template <int NS>
TAO_DEVI void drain_stages(uint64_t* bars, const uint32_t* armed, const uint32_t* phases, int cur, int* err) {
  if (threadIdx.x != 0) return;
#pragma unroll
  for (int x = 0; x < NS; ++x)
    if (x != cur && armed[x]) mbar_wait(&bars[x], phases[x], err);
}

// Persistent form: the grid holds as many CTAs as fit on the GPU at once and each
// walks the items i = blockIdx.x, + gridDim.x, ...  While an item's copy is in
// flight, thread 0 resolves the next item's sources; the next copy is issued as
// soon as the item's compute has released the stage (before its arrival atomic),
// so a CTA's next load overlaps its own arrival and combine.  The combine reads
// the partials from L2 and leaves the stage to the copy in flight.
//
// NS pipeline stages per CTA (the dynamic shared memory holds NS * STAGE bytes): the
// CTA's items rotate through them, item j in stage j % NS, so with NS = 2 the copy of
// the CTA's next item is already in flight while the current one computes; an item's
// successor in its stage (i + NS * gridDim.x) is issued as soon as the item has
// released the stage.  Registers are capped for 6 resident CTAs per SM (the shared
// memory's limit with one 32 KB stage).
template <int D, int NS, int IB>
__global__ void __launch_bounds__(128, 6) decode_fused_kernel(const __grid_constant__ FusedArgs f) {
  using Cfg = FusedCfg<D, IB>;
  const StepArgs& a = f.s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  extern __shared__ __align__(128) uint8_t dsm_all[];
  __shared__ __align__(8) uint64_t bars[NS];
  __shared__ uint32_t armed_s[NS];
  __shared__ int flag;
  __shared__ float qv[D];
  __shared__ float red[128 + 8];
  __shared__ float chs[Cfg::FPC * D];
  __shared__ float mass_s[kRouteCapMax];  // feature read: mass of every selected fine
  __shared__ int last_rh;
  __shared__ int ids_s[NS][Cfg::FPC];     // fine ids of the item in each stage
  const int total = f.nslots ? f.slot_base[f.nslots] : a.R * a.H * (Cfg::KB + f.ms);
  constexpr int kArriver = (D < 128) ? D : 0;  // a thread with no channel in the combine (D = 64)
  ItemCopy<D, IB> next_copy{};
  if (tid == 0) {
#pragma unroll
    for (int x = 0; x < NS; ++x) mbar_init(&bars[x], 1);
    fence_mbar_init();
    ItemCopy<D, IB> c[NS] = {};  // every stage's sources first, so their loads overlap
#pragma unroll
    for (int x = 0; x < NS; ++x)
      if (blockIdx.x + x * gridDim.x < total) c[x] = resolve_item<D, IB>(f, fused_item(f, blockIdx.x + x * gridDim.x));
#pragma unroll
    for (int x = 0; x < NS; ++x) {
#pragma unroll
      for (int y = 0; y < Cfg::FPC; ++y) ids_s[x][y] = c[x].id[y];
      armed_s[x] = issue_copy<D, IB>(c[x], dsm_all + x * Cfg::STAGE, &bars[x]);
    }
  }
  uint32_t phases[NS];
#pragma unroll
  for (int x = 0; x < NS; ++x) phases[x] = 0;
  int sidx = 0;   // stage of the current item
  for (int i = blockIdx.x; i < total; i += gridDim.x, sidx = (sidx + 1 == NS) ? 0 : sidx + 1) {
    const Item it = fused_item(f, i);
    TaoState& st = *a.states[it.r];
    const long long t = st.position;
    const int n_route = st.n_route;
    const int nxt = i + NS * gridDim.x;   // the next item of this stage
    uint8_t* const dsm = dsm_all + sidx * Cfg::STAGE;
    uint64_t& bar = bars[sidx];
    uint32_t phase = 0;
#pragma unroll
    for (int x = 0; x < NS; ++x)
      if (x == sidx) phase = phases[x];
    __syncthreads();
    const uint32_t armed = armed_s[sidx];
    if (tid == 0 && nxt < total) next_copy = resolve_item<D, IB>(f, fused_item(f, nxt));  // overlaps the copy
    const long long src = ((long long)it.r * a.H + it.h) * D;
    // The combine's per-channel operands (raw_q, fusion_a terms 0 and 2, fusion_b terms
    // 0 and 2 of channel d = tid), loaded now so that their latency is off the
    // combine's path; only the CTA that completes the last item of (r, h) uses them.
    uint32_t fin[3] = {0u, 0u, 0u};
    if (tid < D && t >= kWindow) {
      const bf16* fa = a.fa + ((long long)it.h * D + tid) * 3;
      const bf16* fb = a.fb + ((long long)it.h * D + tid) * 3;
      fin[0] = *reinterpret_cast<const uint16_t*>(a.raw_q + src + tid);
      fin[1] = *reinterpret_cast<const uint16_t*>(fa) | ((uint32_t)*reinterpret_cast<const uint16_t*>(fa + 2) << 16);
      fin[2] = *reinterpret_cast<const uint16_t*>(fb) | ((uint32_t)*reinterpret_cast<const uint16_t*>(fb + 2) << 16);
    }
    if (it.slot < Cfg::KB) {
      // ------------------------------------------------ local attention block
      const int s0 = it.slot * Cfg::SLOTS;
      const float sl = 1.4426950408889634f / sqrtf((float)D);
      for (int d = tid; d < D; d += 128) qv[d] = bf(a.q[src + d]) * sl;
      __syncthreads();
      float* part = a.local_part + (((long long)it.r * a.H + it.h) * Cfg::KB + it.slot) * (D + 2);
      if (!armed) {
        if (tid == 0) { part[D] = -INFINITY; part[D + 1] = 0.f; }
      } else {
        if (!wait_uniform(&bar, phase, a.err, &flag)) {
          drain_stages<NS>(bars, armed_s, phases, sidx, a.err);
          return;
        }
        bf16* sk = reinterpret_cast<bf16*>(dsm);
        bf16* sv = sk + Cfg::SLOTS * D;
        const int tm = (int)(t % kWindow);
        if (tm >= s0 && tm < s0 + Cfg::SLOTS) {
          // this block owns the current token's slot: append to the ring, patch smem
          for (int d = tid; d < D / 8; d += 128) {
            const uint4 kk = reinterpret_cast<const uint4*>(a.k + src)[d];
            const uint4 vv = reinterpret_cast<const uint4*>(a.v + src)[d];
            const uint4 rr = reinterpret_cast<const uint4*>(a.raw_k + src)[d];
            reinterpret_cast<uint4*>(sk + (tm - s0) * D)[d] = kk;
            reinterpret_cast<uint4*>(sv + (tm - s0) * D)[d] = vv;
            reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(st.k_ring) + ((long long)it.h * kWindow + tm) * D)[d] = kk;
            reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(st.v_ring) + ((long long)it.h * kWindow + tm) * D)[d] = vv;
            reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(st.rk_ring) + ((long long)it.h * kWindow + tm) * D)[d] = rr;
          }
          __syncthreads();
        }
        constexpr int TPK = 128 / Cfg::SLOTS;
        const int key = tid / TPK, pid = tid % TPK;
        float sc = 0.f;
        {
          const bf16* kr = sk + key * D;
          constexpr int NCH = D / 8 / TPK;
#pragma unroll
          for (int x = 0; x < NCH; ++x) {
            const int c = pid * NCH + ((x + key) % NCH);
            float fv[8];
            unpack8(*reinterpret_cast<const uint4*>(kr + c * 8), fv);
#pragma unroll
            for (int e = 0; e < 8; ++e) sc += fv[e] * qv[c * 8 + e];
          }
          if (TPK == 2) sc += __shfl_xor_sync(0xffffffffu, sc, 1);
        }
        const long long kp = t - (long long)((tm - (s0 + key) + kWindow) % kWindow);
        if (kp < window_start(t) || kp > t) sc = -INFINITY;
        float mx = warp_max(sc);
        if (lane == 0) red[warp] = mx;
        __syncthreads();
        mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
        const float pk = (sc == -INFINITY) ? 0.f : exp2f(sc - mx);
        const float ls = warp_sum(pid == 0 ? pk : 0.f);
        if (pid == 0) red[8 + key] = pk;
        __syncthreads();
        if (lane == 0) red[4 + warp] = ls;
        constexpr int ECH = D / 8, KG = 128 / ECH, KPG = Cfg::SLOTS / KG;
        const int ec = tid % ECH, kg = tid / ECH;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int x = 0; x < KPG; ++x) {
          const int kk = kg * KPG + x;
          const float pj = red[8 + kk];
          float fv[8];
          unpack8(*reinterpret_cast<const uint4*>(sv + kk * D + ec * 8), fv);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += pj * fv[e];
        }
        // reduce over key groups in the (now free) K half of the stage
        float* rs = reinterpret_cast<float*>(dsm);
        __syncthreads();
#pragma unroll
        for (int e = 0; e < 8; ++e) rs[kg * D + ec * 8 + e] = acc[e];
        __syncthreads();
        for (int d = tid; d < D; d += 128) {
          float sum = 0.f;
          for (int g2 = 0; g2 < KG; ++g2) sum += rs[g2 * D + d];
          part[d] = sum;
        }
        if (tid == 0) { part[D] = mx; part[D + 1] = red[4] + red[5] + red[6] + red[7]; }
      }
    } else if (t >= kWindow) {
      // -------------------------------------------------- selected fine group
      const int m0 = (it.slot - Cfg::KB) * Cfg::FPC;
      const int nf = min(Cfg::FPC, st.n_route - m0);
      if (nf > 0) {
        const long long pstride = (long long)(st.cap_fines / kGroup + 1) * D;
        const bf16* fz = reinterpret_cast<const bf16*>(st.fine_z) + (long long)it.h * st.cap_fines * D;
        const bf16* pz = reinterpret_cast<const bf16*>(st.page_z) + it.h * pstride;
        const bf16* pw = reinterpret_cast<const bf16*>(st.page_w) + it.h * pstride;
        // The channels do not depend on the matrices in flight: compute them first.
        // Warp x reads the z, page z and page weight rows of fine x (its id came with
        // the copy) while warp 0 also reads raw_q, so the loads overlap.
        static_assert(Cfg::FPC <= 4, "one fine per warp");
        const bool mine = !a.feature && warp < nf;
        float hraw[D / 32], wv[D / 32], pwv[D / 32];
        if (warp == 0) {
#pragma unroll
          for (int j = 0; j < D / 32; ++j) hraw[j] = bf(a.raw_q[src + lane + 32 * j]);
        }
        if (mine) {
          const int id = ids_s[sidx][warp], page = id / kGroup;
#pragma unroll
          for (int j = 0; j < D / 32; ++j) {
            const int d = lane + 32 * j;
            const float zz = bf(fz[(long long)id * D + d]), pp = bf(pz[(long long)page * D + d]);
            pwv[j] = bf(pw[(long long)page * D + d]);
            wv[j] = rb(expf(rb(__fsub_rn(zz, pp))));
          }
        }
        if (warp == 0) softmax_vals<D>(hraw, qv, lane);
        __syncthreads();
        if (a.feature) {
          // masses of all n_route selected fines (each item forms the same total)
          const int32_t* all = st.route_ids + (long long)it.h * st.route_cap;
          const int nm = min(n_route, kRouteCapMax);
          for (int m = warp; m < nm; m += 4) {
            const bf16* zr = fz + (long long)all[m] * D;
            float sm = 0.f;
#pragma unroll
            for (int j = 0; j < D / 32; ++j) sm += __fmul_rn(qv[lane + 32 * j], expf(bf(zr[lane + 32 * j])));
            sm = warp_sum(sm);
            if (lane == 0) mass_s[m] = sm;
          }
          __syncthreads();
          float tot = 0.f;
          for (int m = 0; m < nm; ++m) tot += mass_s[m];
          for (int idx = tid; idx < nf * D; idx += 128) {
            const int x = idx / D, d = idx % D;
            chs[x * D + d] = rb(__fmul_rn(__fdiv_rn(mass_s[m0 + x], tot), qv[d]));
          }
          if (tid < nf) red[tid] = 0.f;
        }
        if (mine) {
          float sum = 0.f;
#pragma unroll
          for (int j = 0; j < D / 32; ++j) {
            const int d = lane + 32 * j;
            const float c = rb(__fmul_rn(rb(__fmul_rn(qv[d], pwv[j])), wv[j]));
            chs[warp * D + d] = c;
            sum += c;
          }
          sum = warp_sum(sum);
          if (lane == 0) red[warp] = rb(sum);
        }
        if (!wait_uniform(&bar, phase, a.err, &flag)) {
          drain_stages<NS>(bars, armed_s, phases, sidx, a.err);
          return;
        }
        constexpr int ECH = D / 8, RG = 128 / ECH, RPG = D / RG;
        const int ec = tid % ECH, rg = tid / ECH;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const bf16* sc_ = reinterpret_cast<const bf16*>(dsm);
        for (int x = 0; x < nf; ++x) {
#pragma unroll
          for (int y = 0; y < RPG; ++y) {
            const int d = rg * RPG + y;
            const float c = chs[x * D + d];
            float fv[8];
            unpack8(*reinterpret_cast<const uint4*>(sc_ + x * D * D + d * D + ec * 8), fv);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] += c * fv[e];
          }
        }
        __syncthreads();
        float* rs = reinterpret_cast<float*>(dsm);
#pragma unroll
        for (int e = 0; e < 8; ++e) rs[rg * D + ec * 8 + e] = acc[e];
        __syncthreads();
        float* part = a.fine_part + (((long long)it.r * a.H + it.h) * f.ms + (it.slot - Cfg::KB)) * (D + 1);
        for (int d = tid; d < D; d += 128) {
          float sum = 0.f;
          for (int g2 = 0; g2 < RG; ++g2) sum += rs[g2 * D + d];
          part[d] = sum;
        }
        if (tid == 0) {
          float den = 0.f;
          for (int x = 0; x < nf; ++x) den += red[x];
          part[D] = den;
        }
      }
    }
    if (armed) {
#pragma unroll
      for (int x = 0; x < NS; ++x)
        if (x == sidx) phases[x] ^= 1u;
    }
    // ---- the stage is free: issue the next item, then arrive; the CTA completing
    // the last item of (r, h) finalises it.  Every thread orders its shared-memory
    // writes of this item (generic proxy) before the next bulk copy (async proxy).
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
#pragma unroll
      for (int y = 0; y < Cfg::FPC; ++y) ids_s[sidx][y] = next_copy.id[y];
      armed_s[sidx] = (nxt < total) ? issue_copy<D, IB>(next_copy, dsm, &bar) : 0u;
    }
    if (tid == 32) {  // warp 1 arrives while warp 0 issues the copy
      const int per = f.nslots ? f.per_r[it.r] : Cfg::KB + f.ms;  // items of (r, h)
      last_rh = (atomic_add_release(&st.counters[it.h], 1) == per - 1) ? 1 : 0;
      if (last_rh) {
        st.counters[it.h] = 0;
        fence_acquire();
      }
    }
    __syncthreads();
    if (!last_rh) continue;
    // Every item of (r, h) is complete, so every item of this head has read the
    // cursor: arrive for the request now (its last head moves the cursor at the end);
    // with D = 64 the arriving thread has no channel, so its round trip overlaps
    // the combine.
    int arrived = 0;
    if (tid == kArriver) arrived = atomic_add_release(&st.arrive, 1);
    const bool hist = t >= kWindow;
    const int nparts = hist ? (n_route + Cfg::FPC - 1) / Cfg::FPC : 0;
    if (tid == 0 && nparts > (f.nslots ? f.per_r[it.r] : Cfg::KB + f.ms) - Cfg::KB)
      atomicOr(a.err, kErrRouteCap);  // more routes than the launch gave fine items
    if (tid < D) {  // D <= 128: one channel per thread; partials straight from L2
      const int d = tid;
      const float* lg = a.local_part + ((long long)it.r * a.H + it.h) * Cfg::KB * (D + 2);
      const float* fg = a.fine_part + ((long long)it.r * a.H + it.h) * f.ms * (D + 1);
      // the first 16 fine partials go out with the local ones: one round trip to L2
      float va[16], vd[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        va[u] = u < nparts ? __ldcg(fg + u * (D + 1) + d) : 0.f;
        vd[u] = u < nparts ? __ldcg(fg + u * (D + 1) + D) : 0.f;
      }
      float lm[Cfg::KB], ll[Cfg::KB], lo[Cfg::KB];
#pragma unroll
      for (int b2 = 0; b2 < Cfg::KB; ++b2) {
        lm[b2] = __ldcg(lg + b2 * (D + 2) + D);
        ll[b2] = __ldcg(lg + b2 * (D + 2) + D + 1);
        lo[b2] = __ldcg(lg + b2 * (D + 2) + d);
      }
      float Mx = -INFINITY;
#pragma unroll
      for (int b2 = 0; b2 < Cfg::KB; ++b2) Mx = fmaxf(Mx, lm[b2]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int b2 = 0; b2 < Cfg::KB; ++b2) {
        if (lm[b2] == -INFINITY) continue;
        const float scl = exp2f(lm[b2] - Mx);
        L += scl * ll[b2];
        O += scl * lo[b2];
      }
      const float local = rb(O / L);
      float outv = local;
      if (hist) {
        float acc = 0.f, den = 0.f;
        for (int p0 = 0; p0 < nparts; p0 += 16) {  // 16 partials' loads in flight, then summed in order
          if (p0 > 0) {
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const int p2 = p0 + u;
              va[u] = p2 < nparts ? __ldcg(fg + p2 * (D + 1) + d) : 0.f;
              vd[u] = p2 < nparts ? __ldcg(fg + p2 * (D + 1) + D) : 0.f;
            }
          }
#pragma unroll
          for (int u = 0; u < 16; ++u)
            if (p0 + u < nparts) {
              acc += va[u];
              den += vd[u];
            }
        }
        const float fine = a.feature ? rb(acc) : rb(__fdiv_rn(rb(acc), rb(den)));
        const float qq = lo_f(fin[0]);
        const float s0 = rb(__fadd_rn(rb(__fmul_rn(lo_f(fin[1]), qq)), lo_f(fin[2])));  // + 0 (middle term) is exact
        const float s2 = rb(__fadd_rn(rb(__fmul_rn(hi_f(fin[1]), qq)), hi_f(fin[2])));
        const float mx = fmaxf(s0, s2);
        const float e0 = expf(s0 - mx), e2 = expf(s2 - mx);
        const float rho0 = rb(__fdiv_rn(e0, e0 + e2)), rho2 = rb(__fdiv_rn(e2, e0 + e2));
        const float lt = rb(__fmul_rn(rho0, __fmul_rn(2.f, local)));  // bf16(2 * local) = 2 * local
        const float ft = rb(__fmul_rn(rho2, rb(__fmul_rn(a.gain, fine))));
        outv = rb(__fadd_rn(__fadd_rn(lt, 0.f), ft));  // lt + 0 (middle term) is exact: no rounding
      }
      a.out[src + d] = tobf(outv);
    }
    if (a.host_done) {  // host-staged step: publish it once every row is in host memory
      __syncthreads();  // this CTA's row is written (the fence below is cumulative)
      if (tid == 0) {
        __threadfence_system();
        if (atomicAdd(a.done, 1) == a.R * a.H - 1) {
          __threadfence_system();
          a.done[0] = 0;
          const int seq = a.done[1] + 1;
          a.done[1] = seq;
          *reinterpret_cast<volatile int*>(a.host_done) = seq;
        }
      }
    }
    if (tid == kArriver && arrived == a.H - 1) {  // the request's last head: advance its cursor
      fence_acquire();
      st.arrive = 0;
      st.position = t + 1;
    }
  }
}

// ---------------------------------------------------------------------------
// Warp-specialised persistent variant: each CTA owns up to kWsMaxItems items.
//  * start: request descriptors -> shared memory; the 32 producer lanes build
//    every item's metadata in parallel (route ids included)
//  * warp 8 lane 0 streams each item into a ring of NS stages: the big tile
//    (K|V rows or selected matrices) plus the small rows the item needs (q or
//    raw_q, fine z / page z / page weight rows, the new token's k / v / raw k),
//    all as bulk copies on the stage's full mbarrier
//  * warps 0-3 and 4-7 consume alternate items from shared memory only, release
//    the stage (empty mbarrier) and follow the same arrival / combine protocol
// ---------------------------------------------------------------------------
constexpr int kWsStages = 6;
constexpr int kWsMaxItems = 64;
constexpr int kWsMaxReq = 64;

struct ReqCache {
  const bf16 *k, *v, *rk, *fc, *fz, *pz, *pw;
  const int32_t* ids;
  int32_t* counters;
  TaoState* st;
  long long t;
  int n_route, cap, route_cap, pages;
};

template <int D>
struct WsMeta {
  int r, h, slot, nf, armed, own;
  int ids[FusedCfg<D>::FPC];
};

template <int D>
struct WsLayout {
  static constexpr int MAIN = 32768;                 // K|V tile or selected matrices
  static constexpr int ROW = D * 2;                  // one bf16 row
  static constexpr int AUX = ROW * (1 + 3 + 3 * FusedCfg<D>::FPC);
  static constexpr int STAGE = MAIN + ((AUX + 127) / 128) * 128;
};

TAO_DEVI void group_sync(int g) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(128) : "memory");
}

TAO_DEVI bool group_wait(uint64_t* bar, uint32_t phase, int* err, int* flag, int g, int gtid) {
  if (gtid == 0) *flag = mbar_wait(bar, phase, err) ? 1 : 0;
  group_sync(g);
  const bool ok = *flag != 0;
  if (ok) {
    while (!mbar_try_wait(bar, phase)) {
    }
  }
  return ok;
}

template <int D>
struct WsGroupScratch {
  float qv[D];
  float red[128 + 8];
  float chs[FusedCfg<D>::FPC * D];
  int flag;
  int last;
};

template <int D>
__global__ void __launch_bounds__(288) decode_ws_kernel(FusedArgs f) {
  using Cfg = FusedCfg<D>;
  using LY = WsLayout<D>;
  constexpr int NS = kWsStages;
  const StepArgs& a = f.s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ __align__(8) uint64_t full[NS], empty[NS];
  __shared__ ReqCache rq[kWsMaxReq];
  __shared__ WsMeta<D> meta[kWsMaxItems];
  __shared__ WsGroupScratch<D> gs[2];
  const int per = Cfg::KB + f.ms;
  const int total = a.R * a.H * per;
  const int G = gridDim.x;
  const int nitems = (total - (int)blockIdx.x + G - 1) / G;
  if (tid == 0) {
    for (int x = 0; x < NS; ++x) {
      mbar_init(&full[x], 1);
      mbar_init(&empty[x], 1);
    }
    fence_mbar_init();
  }
  for (int r = tid; r < a.R; r += blockDim.x) {
    TaoState* st = a.states[r];
    ReqCache c;
    c.k = reinterpret_cast<const bf16*>(st->k_ring);
    c.v = reinterpret_cast<const bf16*>(st->v_ring);
    c.rk = reinterpret_cast<const bf16*>(st->rk_ring);
    c.fc = reinterpret_cast<const bf16*>(st->fine_c);
    c.fz = reinterpret_cast<const bf16*>(st->fine_z);
    c.pz = reinterpret_cast<const bf16*>(st->page_z);
    c.pw = reinterpret_cast<const bf16*>(st->page_w);
    c.ids = st->route_ids;
    c.counters = st->counters;
    c.st = st;
    c.t = st->position;
    c.n_route = st->n_route;
    c.cap = st->cap_fines;
    c.route_cap = st->route_cap;
    c.pages = st->cap_fines / kGroup + 1;
    rq[r] = c;
  }
  __syncthreads();

  if (warp == 8) {
    // ---------------------------------------------------------- producer
    for (int j = lane; j < nitems; j += 32) {
      const Item it = item_of(blockIdx.x + j * G, a.R, a.H);
      const ReqCache& c = rq[it.r];
      WsMeta<D> m;
      m.r = it.r; m.h = it.h; m.slot = it.slot; m.nf = 0; m.own = 0; m.armed = 0;
      if (it.slot < Cfg::KB) {
        const int s0 = it.slot * Cfg::SLOTS;
        const int tm = (int)(c.t % kWindow);
        m.armed = local_block_live<D>(c.t, window_start(c.t), s0, Cfg::SLOTS) ? 1 : 0;
        m.own = (tm >= s0 && tm < s0 + Cfg::SLOTS) ? 1 : 0;
      } else if (c.t >= kWindow) {
        const int m0 = (it.slot - Cfg::KB) * Cfg::FPC;
        m.nf = max(0, min(Cfg::FPC, c.n_route - m0));
        for (int x = 0; x < m.nf; ++x) m.ids[x] = c.ids[(long long)it.h * c.route_cap + m0 + x];
        m.armed = m.nf > 0;
      }
      meta[j] = m;
    }
    __syncwarp();
    if (lane != 0) return;
    for (int j = 0; j < nitems; ++j) {
      const int sj = j % NS, use = j / NS;
      if (use > 0 && !mbar_wait(&empty[sj], (use - 1) & 1, a.err)) return;
      const WsMeta<D>& m = meta[j];
      if (!m.armed) {
        mbar_arrive(&full[sj]);
        continue;
      }
      const ReqCache& c = rq[m.r];
      uint8_t* stage = dsm + (size_t)sj * LY::STAGE;
      uint8_t* aux = stage + LY::MAIN;
      const long long src = ((long long)m.r * a.H + m.h) * D;
      if (m.slot < Cfg::KB) {
        const uint32_t bytes = Cfg::SLOTS * D * 2;
        const long long hoff = (long long)m.h * kWindow * D + (long long)m.slot * Cfg::SLOTS * D;
        mbar_expect_tx(&full[sj], 2 * bytes + LY::ROW * (m.own ? 4 : 1));
        bulk_g2s(stage, c.k + hoff, bytes, &full[sj]);
        bulk_g2s(stage + bytes, c.v + hoff, bytes, &full[sj]);
        bulk_g2s(aux, a.q + src, LY::ROW, &full[sj]);
        if (m.own) {
          bulk_g2s(aux + LY::ROW, a.k + src, LY::ROW, &full[sj]);
          bulk_g2s(aux + 2 * LY::ROW, a.v + src, LY::ROW, &full[sj]);
          bulk_g2s(aux + 3 * LY::ROW, a.raw_k + src, LY::ROW, &full[sj]);
        }
      } else {
        const uint32_t mbytes = D * D * 2;
        mbar_expect_tx(&full[sj], m.nf * (mbytes + 3 * LY::ROW) + LY::ROW);
        const long long zb = (long long)m.h * c.cap * D;
        const long long pb = (long long)m.h * c.pages * D;
        bulk_g2s(aux, a.raw_q + src, LY::ROW, &full[sj]);
        for (int x = 0; x < m.nf; ++x) {
          const int id = m.ids[x], page = id / kGroup;
          bulk_g2s(stage + x * mbytes, c.fc + ((long long)m.h * c.cap + id) * D * D, mbytes, &full[sj]);
          uint8_t* rows = aux + LY::ROW * (1 + 3 * x);
          bulk_g2s(rows, c.fz + zb + (long long)id * D, LY::ROW, &full[sj]);
          bulk_g2s(rows + LY::ROW, c.pz + pb + (long long)page * D, LY::ROW, &full[sj]);
          bulk_g2s(rows + 2 * LY::ROW, c.pw + pb + (long long)page * D, LY::ROW, &full[sj]);
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int g = warp >> 2, gtid = tid & 127, gwarp = warp & 3;
  WsGroupScratch<D>& sc = gs[g];
  for (int j = g; j < nitems; j += 2) {
    const int sj = j % NS, use = j / NS;
    if (!group_wait(&full[sj], use & 1, a.err, &sc.flag, g, gtid)) return;
    const WsMeta<D>& m = meta[j];
    const ReqCache& c = rq[m.r];
    uint8_t* stage = dsm + (size_t)sj * LY::STAGE;
    const bf16* aux = reinterpret_cast<const bf16*>(stage + LY::MAIN);
    const long long t = c.t;
    const long long src = ((long long)m.r * a.H + m.h) * D;
    if (m.slot < Cfg::KB) {
      // ---------------------------------------------- local attention block
      float* part = a.local_part + (((long long)m.r * a.H + m.h) * Cfg::KB + m.slot) * (D + 2);
      if (!m.armed) {
        if (gtid == 0) { part[D] = -INFINITY; part[D + 1] = 0.f; }
      } else {
        const int s0 = m.slot * Cfg::SLOTS;
        const float sl = 1.4426950408889634f / sqrtf((float)D);
        for (int d = gtid; d < D; d += 128) sc.qv[d] = bf(aux[d]) * sl;
        bf16* sk = reinterpret_cast<bf16*>(stage);
        bf16* sv = sk + Cfg::SLOTS * D;
        const int tm = (int)(t % kWindow);
        if (m.own) {
          // append the current token to the ring and patch the staged rows
          const long long off = ((long long)m.h * kWindow + tm) * D;
          for (int d = gtid; d < D / 8; d += 128) {
            const uint4 kk = reinterpret_cast<const uint4*>(aux + D)[d];
            const uint4 vv = reinterpret_cast<const uint4*>(aux + 2 * D)[d];
            const uint4 rr = reinterpret_cast<const uint4*>(aux + 3 * D)[d];
            reinterpret_cast<uint4*>(sk + (tm - s0) * D)[d] = kk;
            reinterpret_cast<uint4*>(sv + (tm - s0) * D)[d] = vv;
            reinterpret_cast<uint4*>(const_cast<bf16*>(c.k) + off)[d] = kk;
            reinterpret_cast<uint4*>(const_cast<bf16*>(c.v) + off)[d] = vv;
            reinterpret_cast<uint4*>(const_cast<bf16*>(c.rk) + off)[d] = rr;
          }
        }
        group_sync(g);
        constexpr int TPK = 128 / Cfg::SLOTS;
        const int key = gtid / TPK, pid = gtid % TPK;
        float scv = 0.f;
        {
          const bf16* kr = sk + key * D;
          constexpr int NCH = D / 8 / TPK;
#pragma unroll
          for (int x = 0; x < NCH; ++x) {
            const int ch = pid * NCH + ((x + key) % NCH);
            float fv[8];
            unpack8(*reinterpret_cast<const uint4*>(kr + ch * 8), fv);
#pragma unroll
            for (int e = 0; e < 8; ++e) scv += fv[e] * sc.qv[ch * 8 + e];
          }
          if (TPK == 2) scv += __shfl_xor_sync(0xffffffffu, scv, 1);
        }
        const long long kp = t - (long long)((tm - (s0 + key) + kWindow) % kWindow);
        if (kp < window_start(t) || kp > t) scv = -INFINITY;
        float mx = warp_max(scv);
        if (lane == 0) sc.red[gwarp] = mx;
        group_sync(g);
        mx = fmaxf(fmaxf(sc.red[0], sc.red[1]), fmaxf(sc.red[2], sc.red[3]));
        const float pk = (scv == -INFINITY) ? 0.f : exp2f(scv - mx);
        const float ls = warp_sum(pid == 0 ? pk : 0.f);
        if (pid == 0) sc.red[8 + key] = pk;
        group_sync(g);
        if (lane == 0) sc.red[4 + gwarp] = ls;
        constexpr int ECH = D / 8, KG = 128 / ECH, KPG = Cfg::SLOTS / KG;
        const int ec = gtid % ECH, kg = gtid / ECH;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int x = 0; x < KPG; ++x) {
          const int kk = kg * KPG + x;
          const float pj = sc.red[8 + kk];
          float fv[8];
          unpack8(*reinterpret_cast<const uint4*>(sv + kk * D + ec * 8), fv);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += pj * fv[e];
        }
        float* rs = reinterpret_cast<float*>(stage);
        group_sync(g);
#pragma unroll
        for (int e = 0; e < 8; ++e) rs[kg * D + ec * 8 + e] = acc[e];
        group_sync(g);
        for (int d = gtid; d < D; d += 128) {
          float sum = 0.f;
          for (int g2 = 0; g2 < KG; ++g2) sum += rs[g2 * D + d];
          part[d] = sum;
        }
        if (gtid == 0) { part[D] = mx; part[D + 1] = sc.red[4] + sc.red[5] + sc.red[6] + sc.red[7]; }
      }
    } else if (m.armed) {
      // ------------------------------------------------ selected fine group
      const int nf = m.nf;
      if (gwarp == 0) softmax_row<D>(aux, sc.qv, lane);
      group_sync(g);
      for (int x = gwarp; x < nf; x += 4) {
        const bf16* rows = aux + D * (1 + 3 * x);
        float sum = 0.f;
        for (int d = lane; d < D; d += 32) {
          const float hv = rb(__fmul_rn(sc.qv[d], bf(rows[2 * D + d])));
          const float w = rb(expf(rb(__fsub_rn(bf(rows[d]), bf(rows[D + d])))));
          const float cc = rb(__fmul_rn(hv, w));
          sc.chs[x * D + d] = cc;
          sum += cc;
        }
        sum = warp_sum(sum);
        if (lane == 0) sc.red[x] = rb(sum);
      }
      group_sync(g);
      constexpr int ECH = D / 8, RG = 128 / ECH, RPG = D / RG;
      const int ec = gtid % ECH, rg = gtid / ECH;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      const bf16* cm = reinterpret_cast<const bf16*>(stage);
      for (int x = 0; x < nf; ++x) {
#pragma unroll
        for (int y = 0; y < RPG; ++y) {
          const int d = rg * RPG + y;
          const float cc = sc.chs[x * D + d];
          float fv[8];
          unpack8(*reinterpret_cast<const uint4*>(cm + x * D * D + d * D + ec * 8), fv);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += cc * fv[e];
        }
      }
      group_sync(g);
      float* rs = reinterpret_cast<float*>(stage);
#pragma unroll
      for (int e = 0; e < 8; ++e) rs[rg * D + ec * 8 + e] = acc[e];
      group_sync(g);
      float* part = a.fine_part + (((long long)m.r * a.H + m.h) * f.ms + (m.slot - Cfg::KB)) * (D + 1);
      for (int d = gtid; d < D; d += 128) {
        float sum = 0.f;
        for (int g2 = 0; g2 < RG; ++g2) sum += rs[g2 * D + d];
        part[d] = sum;
      }
      if (gtid == 0) {
        float den = 0.f;
        for (int x = 0; x < nf; ++x) den += sc.red[x];
        part[D] = den;
      }
    }
    // ---- release the stage, then arrival
    group_sync(g);
    if (gtid == 0) {
      mbar_arrive(&empty[sj]);
      __threadfence();
      sc.last = (atomicAdd(&c.counters[m.h], 1) == per - 1) ? 1 : 0;
      if (sc.last) c.counters[m.h] = 0;
      __threadfence();
    }
    group_sync(g);
    if (!sc.last) continue;
    const bool hist = t >= kWindow;
    const int M = c.n_route;
    const int nparts = (M + Cfg::FPC - 1) / Cfg::FPC;
    const float* lp = a.local_part + ((long long)m.r * a.H + m.h) * Cfg::KB * (D + 2);
    const float* fp = a.fine_part + ((long long)m.r * a.H + m.h) * f.ms * (D + 1);
    for (int d = gtid; d < D; d += 128) {
      float Mx = -INFINITY;
      for (int b2 = 0; b2 < Cfg::KB; ++b2) Mx = fmaxf(Mx, __ldcg(lp + b2 * (D + 2) + D));
      float L = 0.f, O = 0.f;
      for (int b2 = 0; b2 < Cfg::KB; ++b2) {
        const float mb = __ldcg(lp + b2 * (D + 2) + D);
        if (mb == -INFINITY) continue;
        const float scl = exp2f(mb - Mx);
        L += scl * __ldcg(lp + b2 * (D + 2) + D + 1);
        O += scl * __ldcg(lp + b2 * (D + 2) + d);
      }
      const float local = rb(O / L);
      float outv = local;
      if (hist) {
        float acc = 0.f, den = 0.f;
        for (int p2 = 0; p2 < nparts; ++p2) {
          acc += __ldcg(fp + p2 * (D + 1) + d);
          den += __ldcg(fp + p2 * (D + 1) + D);
        }
        const float fine = rb(__fdiv_rn(rb(acc), rb(den)));
        const float qq = bf(a.raw_q[src + d]);
        const bf16* fa = a.fa + ((long long)m.h * D + d) * 3;
        const bf16* fb = a.fb + ((long long)m.h * D + d) * 3;
        const float s0 = rb(__fadd_rn(rb(__fadd_rn(rb(__fmul_rn(bf(fa[0]), qq)), bf(fb[0]))), 0.f));
        const float s2 = rb(__fadd_rn(rb(__fmul_rn(bf(fa[2]), qq)), bf(fb[2])));
        const float mx = fmaxf(s0, s2);
        const float e0 = expf(s0 - mx), e2 = expf(s2 - mx);
        const float rho0 = rb(__fdiv_rn(e0, e0 + e2)), rho2 = rb(__fdiv_rn(e2, e0 + e2));
        const float lt = rb(__fmul_rn(rho0, rb(__fmul_rn(2.f, local))));
        const float ft = rb(__fmul_rn(rho2, rb(__fmul_rn(a.gain, fine))));
        outv = rb(__fadd_rn(rb(__fadd_rn(lt, 0.f)), ft));
      }
      a.out[src + d] = tobf(outv);
    }
    group_sync(g);
    if (gtid == 0) {
      __threadfence();
      if (atomicAdd(&c.st->arrive, 1) == a.H - 1) {
        c.st->arrive = 0;
        c.st->position = t + 1;
        __threadfence();
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Warp-granular variant: one warp per 8 KB work item, no block barriers.
//   local item  : KPW consecutive ring slots (32 keys for D64, 16 for D128): 4 KB
//                 of K and 4 KB of V read with 16-byte vector loads into registers
//   fine item   : one selected fine matrix in 4 KB slices, two slices in flight
//                 (8 KB for D64, 32 KB for D128)
// Lane l of a 512-byte warp load holds row (l / CPR) and 16-byte chunk (l % CPR)
// of that slice (CPR = D/8 chunks per row).  Partials go to the workspace; the
// warp completing the last item of (r, h) combines and fuses; the warp completing
// the last head of request r advances its cursor.
// ---------------------------------------------------------------------------
template <int D>
struct WarpCfg {
  static constexpr int CPR = D / 8;              // 16-byte chunks per row
  static constexpr int RPL = 32 / CPR;           // rows per 512-byte warp load
  static constexpr int KPW = 4096 / (D * 2);     // rows per 4 KB slice (keys per local item)
  static constexpr int LI = kWindow / KPW;       // local items per (r, h): 24 (D64) / 48 (D128)
  static constexpr int LOADS = KPW / RPL;        // 512-byte warp loads per 4 KB slice (8)
  static constexpr int FCH = D / KPW;            // 4 KB slices of a fine matrix: 2 / 8
};

template <int D>
__global__ void __launch_bounds__(256) decode_warp_kernel(FusedArgs f) {
  using W = WarpCfg<D>;
  const StepArgs& a = f.s;
  const int lane = threadIdx.x & 31;
  const int per = W::LI + f.ms;
  const int total = a.R * a.H * per;
  const int wi = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (wi >= total) return;
  const Item it = item_of(wi, a.R, a.H);
  TaoState& st = *a.states[it.r];
  const long long t = st.position;
  const long long src = ((long long)it.r * a.H + it.h) * D;
  const int row = lane / W::CPR, chunk = lane % W::CPR;
  if (it.slot < W::LI) {
    // ---------------------------------------------------- local attention item
    const int s0 = it.slot * W::KPW;
    const int tm = (int)(t % kWindow);
    const long long start = window_start(t);
    float* part = a.local_part + (((long long)it.r * a.H + it.h) * W::LI + it.slot) * (D + 2);
    const bf16* kr = ring_head<D>(st.k_ring, it.h) + (long long)s0 * D;
    const bf16* vr = ring_head<D>(st.v_ring, it.h) + (long long)s0 * D;
    if (!local_block_live<D>(t, start, s0, W::KPW)) {
      if (lane == 0) { part[D] = -INFINITY; part[D + 1] = 0.f; }
    } else {
      uint4 kv[W::LOADS], vv[W::LOADS];
#pragma unroll
      for (int x = 0; x < W::LOADS; ++x) {
        kv[x] = __ldcs(reinterpret_cast<const uint4*>(kr + (x * W::RPL + row) * D) + chunk);
        vv[x] = __ldcs(reinterpret_cast<const uint4*>(vr + (x * W::RPL + row) * D) + chunk);
      }
      const uint4 qc = *(reinterpret_cast<const uint4*>(a.q + src) + chunk);
      // the current token: use (and append) the new k / v
      const bool own = tm >= s0 && tm < s0 + W::KPW;
      if (own) {
        const uint4 nk = *(reinterpret_cast<const uint4*>(a.k + src) + chunk);
        const uint4 nv = *(reinterpret_cast<const uint4*>(a.v + src) + chunk);
        const int x0 = (tm - s0) / W::RPL, r0 = (tm - s0) % W::RPL;
#pragma unroll
        for (int x = 0; x < W::LOADS; ++x)
          if (x == x0 && row == r0) { kv[x] = nk; vv[x] = nv; }
        if (row == 0) {
          const uint4 nr = *(reinterpret_cast<const uint4*>(a.raw_k + src) + chunk);
          const long long off = ((long long)it.h * kWindow + tm) * D;
          reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(st.k_ring) + off)[chunk] = nk;
          reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(st.v_ring) + off)[chunk] = nv;
          reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(st.rk_ring) + off)[chunk] = nr;
        }
      }
      float qf[8];
      unpack8(qc, qf);
      const float sl = 1.4426950408889634f / sqrtf((float)D);
      float sc[W::LOADS];
      float mx = -INFINITY;
#pragma unroll
      for (int x = 0; x < W::LOADS; ++x) {
        float kf[8];
        unpack8(kv[x], kf);
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) dot += kf[e] * qf[e];
#pragma unroll
        for (int o = W::CPR / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const int key = s0 + x * W::RPL + row;
        const long long kp = t - (long long)((tm - key + kWindow) % kWindow);
        sc[x] = (kp < start || kp > t) ? -INFINITY : dot * sl;
        mx = fmaxf(mx, sc[x]);
      }
      mx = warp_max(mx);
      float lsum = 0.f, acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int x = 0; x < W::LOADS; ++x) {
        const float p = (sc[x] == -INFINITY) ? 0.f : exp2f(sc[x] - mx);
        lsum += (chunk == 0) ? p : 0.f;
        float vf[8];
        unpack8(vv[x], vf);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += p * vf[e];
      }
      lsum = warp_sum(lsum);
#pragma unroll
      for (int o = 16; o >= W::CPR; o >>= 1)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
      if (row == 0) {
#pragma unroll
        for (int e = 0; e < 8; ++e) part[chunk * 8 + e] = acc[e];
      }
      if (lane == 0) { part[D] = mx; part[D + 1] = lsum; }
    }
  } else if (t >= kWindow) {
    // ---------------------------------------------------- selected fine item
    const int m = it.slot - W::LI;
    if (m < st.n_route) {
      const int id = st.route_ids[(long long)it.h * st.route_cap + m];
      const int page = id / kGroup;
      const bf16* cmat = reinterpret_cast<const bf16*>(st.fine_c) + ((long long)it.h * st.cap_fines + id) * D * D;
      constexpr int CHUNKS = W::FCH;
      uint4 cv[2][W::LOADS];
#pragma unroll
      for (int x = 0; x < W::LOADS; ++x)
        cv[0][x] = __ldcs(reinterpret_cast<const uint4*>(cmat + (x * W::RPL + row) * D) + chunk);
      if (CHUNKS > 1) {
#pragma unroll
        for (int x = 0; x < W::LOADS; ++x)
          cv[1][x] = __ldcs(reinterpret_cast<const uint4*>(cmat + (W::KPW + x * W::RPL + row) * D) + chunk);
      }
      // channels: ch[d] = bf16(bf16(h*pw) * bf16(exp(bf16(z - pz)))) for d = lane + 32 j
      const long long pstride = (long long)(st.cap_fines / kGroup + 1) * D;
      const bf16* fz = reinterpret_cast<const bf16*>(st.fine_z) + ((long long)it.h * st.cap_fines + id) * D;
      const bf16* pz = reinterpret_cast<const bf16*>(st.page_z) + it.h * pstride + (long long)page * D;
      const bf16* pw = reinterpret_cast<const bf16*>(st.page_w) + it.h * pstride + (long long)page * D;
      float hq[D / 32];
      {
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < D / 32; ++j) { hq[j] = bf(a.raw_q[src + lane + 32 * j]); mx = fmaxf(mx, hq[j]); }
        mx = warp_max(mx);
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < D / 32; ++j) { hq[j] = expf(hq[j] - mx); s += hq[j]; }
        s = warp_sum(s);
#pragma unroll
        for (int j = 0; j < D / 32; ++j) hq[j] = rb(__fdiv_rn(hq[j], s));
      }
      float ch[D / 32], den = 0.f;
#pragma unroll
      for (int j = 0; j < D / 32; ++j) {
        const int d = lane + 32 * j;
        const float hv = rb(__fmul_rn(hq[j], bf(pw[d])));
        const float w = rb(expf(rb(__fsub_rn(bf(fz[d]), bf(pz[d])))));
        ch[j] = rb(__fmul_rn(hv, w));
        den += ch[j];
      }
      den = warp_sum(den);
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int c = 0; c < CHUNKS; ++c) {
        const int cb = c & 1;
#pragma unroll
        for (int x = 0; x < W::LOADS; ++x) {
          // matrix row of this lane; rows of one load never cross a 32-row boundary
          const int d = c * W::KPW + x * W::RPL + row;
          constexpr int JJ = 0;
          const float chd = __shfl_sync(0xffffffffu, ch[((c * W::KPW + x * W::RPL) >> 5) + JJ], d & 31);
          float cf[8];
          unpack8(cv[cb][x], cf);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += chd * cf[e];
        }
        if (c + 2 < CHUNKS) {
#pragma unroll
          for (int x = 0; x < W::LOADS; ++x)
            cv[cb][x] = __ldcs(reinterpret_cast<const uint4*>(cmat + ((c + 2) * W::KPW + x * W::RPL + row) * D) + chunk);
        }
      }
#pragma unroll
      for (int o = 16; o >= W::CPR; o >>= 1)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
      float* part = a.fine_part + (((long long)it.r * a.H + it.h) * f.ms + m) * (D + 1);
      if (row == 0) {
#pragma unroll
        for (int e = 0; e < 8; ++e) part[chunk * 8 + e] = acc[e];
      }
      if (lane == 0) part[D] = rb(den);
    }
  }
  // ---- arrival; the warp completing (r, h) combines and fuses
  __syncwarp();
  int last = 0;
  if (lane == 0) {
    __threadfence();
    last = (atomicAdd(&st.counters[it.h], 1) == per - 1) ? 1 : 0;
    if (last) st.counters[it.h] = 0;
    __threadfence();
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  const bool hist = t >= kWindow;
  const int M = st.n_route;
  const float* lp = a.local_part + ((long long)it.r * a.H + it.h) * W::LI * (D + 2);
  const float* fp = a.fine_part + ((long long)it.r * a.H + it.h) * f.ms * (D + 1);
  float Mx = -INFINITY;
  for (int b2 = lane; b2 < W::LI; b2 += 32) Mx = fmaxf(Mx, __ldcg(lp + b2 * (D + 2) + D));
  Mx = warp_max(Mx);
  float sc2[W::LI / 32 + 1];
  float L = 0.f;
#pragma unroll
  for (int x = 0; x < W::LI / 32 + 1; ++x) {
    const int b2 = lane + 32 * x;
    float v = 0.f;
    if (b2 < W::LI) {
      const float mb = __ldcg(lp + b2 * (D + 2) + D);
      v = (mb == -INFINITY) ? 0.f : exp2f(mb - Mx);
      L += v * __ldcg(lp + b2 * (D + 2) + D + 1);
    }
    sc2[x] = v;
  }
  L = warp_sum(L);
  float den = 0.f;
  if (hist) {
    for (int m2 = lane; m2 < M; m2 += 32) den += __ldcg(fp + m2 * (D + 1) + D);
    den = warp_sum(den);
  }
#pragma unroll
  for (int j = 0; j < D / 32; ++j) {
    const int d = lane + 32 * j;
    float O = 0.f;
    for (int b2 = 0; b2 < W::LI; ++b2) {
      const float w = __shfl_sync(0xffffffffu, sc2[b2 >> 5], b2 & 31);
      if (w != 0.f) O += w * __ldcg(lp + b2 * (D + 2) + d);
    }
    const float local = rb(O / L);
    float outv = local;
    if (hist) {
      float acc = 0.f;
      for (int m2 = 0; m2 < M; ++m2) acc += __ldcg(fp + m2 * (D + 1) + d);
      const float fine = rb(__fdiv_rn(rb(acc), rb(den)));
      const float qq = bf(a.raw_q[src + d]);
      const bf16* fa = a.fa + ((long long)it.h * D + d) * 3;
      const bf16* fb = a.fb + ((long long)it.h * D + d) * 3;
      const float s0 = rb(__fadd_rn(rb(__fadd_rn(rb(__fmul_rn(bf(fa[0]), qq)), bf(fb[0]))), 0.f));
      const float s2 = rb(__fadd_rn(rb(__fmul_rn(bf(fa[2]), qq)), bf(fb[2])));
      const float mx = fmaxf(s0, s2);
      const float e0 = expf(s0 - mx), e2 = expf(s2 - mx);
      const float rho0 = rb(__fdiv_rn(e0, e0 + e2)), rho2 = rb(__fdiv_rn(e2, e0 + e2));
      const float lt = rb(__fmul_rn(rho0, rb(__fmul_rn(2.f, local))));
      const float ft = rb(__fmul_rn(rho2, rb(__fmul_rn(a.gain, fine))));
      outv = rb(__fadd_rn(rb(__fadd_rn(lt, 0.f)), ft));
    }
    a.out[src + d] = tobf(outv);
  }
  __syncwarp();
  if (lane == 0) {
    __threadfence();
    if (atomicAdd(&st.arrive, 1) == a.H - 1) {
      st.arrive = 0;
      st.position = t + 1;
      __threadfence();
    }
  }
}

// Routing on refresh tokens: writes the state's route arrays directly.
template <int D>
// 1024 threads: the page and candidate loops are latency chains of row loads (cold
// after other work evicted them), so more warps cut the serial iterations per warp.
__global__ void __launch_bounds__(1024) decode_route_kernel(StepArgs a) {
  // host-staged step: bring the step's operands in first (one vector per thread,
  // spread over the CTAs); this launch reads raw_q from host memory itself
  for (long long g = (long long)threadIdx.x * gridDim.x + blockIdx.x; g < a.h_vecs;
       g += (long long)gridDim.x * blockDim.x)
    a.h_stage[g] = a.h_in[g];
  const int r = blockIdx.x / a.H, h = blockIdx.x % a.H;
  TaoState& st = *a.states[r];
  const long long t = st.position;
  const int S = sealed_at(t);
  if (S == 0 || !is_refresh(t, st.layer_index, a.pol)) return;
  const int completed = S / kGroup, pending = S % kGroup;
  const int P = completed + (pending > 0);
  extern __shared__ __align__(128) uint8_t dsm[];
  float* hq = reinterpret_cast<float*>(dsm);
  float* pm = hq + D;
  float* cm = pm + a.pmax;
  int* cand_id = reinterpret_cast<int*>(cm + 8 * a.pmax + 8);
  int* chosen = cand_id + 8 * a.pmax + 8;
  int* sorted = chosen + a.pmax;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarp = blockDim.x >> 5;
  const long long pstride = (long long)(st.cap_fines / kGroup + 1) * D;
  const bf16* pz = reinterpret_cast<const bf16*>(st.page_z) + h * pstride;
  const bf16* pw = reinterpret_cast<const bf16*>(st.page_w) + h * pstride;
  const bf16* fz = reinterpret_cast<const bf16*>(st.fine_z) + (long long)h * st.cap_fines * D;
  if (warp == 0) softmax_row<D>(a.raw_q + ((long long)r * a.H + h) * D, hq, lane);
  __syncthreads();
  const Counts cnt = routed_counts(completed, pending, a.pol);
  const int K = cnt.coarse, U = cnt.eligible, M = cnt.selected;
  if (M > st.route_cap || P > a.pmax) {
    if (tid == 0) atomicOr(a.err, kErrRouteCap);
    return;
  }
  if (K > 0) {
    for (int p = warp; p < completed; p += nwarp) {
      float s = 0.f;
      for (int d = lane; d < D; d += 32) s += rb(__fmul_rn(hq[d], bf(pw[(long long)p * D + d])));
      s = warp_sum(s);
      if (lane == 0) pm[p] = rb(s);
    }
    __syncthreads();
    for (int p = tid; p < completed; p += blockDim.x) {
      const float v = pm[p];
      int rank = 0;
      for (int q = 0; q < completed; ++q) {
        const float u = pm[q];
        rank += (u > v) || (u == v && q < p);
      }
      if (rank < K) chosen[rank] = p;
    }
    __syncthreads();
    for (int j = tid; j < K; j += blockDim.x) {
      int pg = chosen[j], pos = 0;
      for (int x = 0; x < K; ++x) pos += chosen[x] < pg;
      sorted[pos] = pg;
    }
    __syncthreads();
  }
  for (int u = tid; u < U; u += blockDim.x)
    cand_id[u] = (u < kGroup * K) ? sorted[u / kGroup] * kGroup + (u % kGroup)
                                  : completed * kGroup + (u - kGroup * K);
  __syncthreads();
  for (int u = warp; u < U; u += nwarp) {
    const int id = cand_id[u], page = id / kGroup;
    float s = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float hv = rb(__fmul_rn(hq[d], bf(pw[(long long)page * D + d])));
      const float w = rb(expf(rb(__fsub_rn(bf(fz[(long long)id * D + d]), bf(pz[(long long)page * D + d])))));
      s += rb(__fmul_rn(hv, w));
    }
    s = warp_sum(s);
    if (lane == 0) cm[u] = rb(s);
  }
  __syncthreads();
  int32_t* ids = st.route_ids + (long long)h * st.route_cap;
  int32_t* pgs = st.route_pages + (long long)h * st.route_cap;
  for (int u = tid; u < U; u += blockDim.x) {
    const float v = cm[u];
    int rank = 0;
    for (int q = 0; q < U; ++q) {
      const float x = cm[q];
      rank += (x > v) || (x == v && q < u);
    }
    if (rank < M) ids[rank] = cand_id[u];
  }
  for (int j = tid; j < K; j += blockDim.x) pgs[j] = sorted[j];
  if (h == 0 && tid == 0) {
    st.n_route = M;
    st.n_chosen = K;
    st.route_refreshes += 1;
  }
}

}  // namespace tao
