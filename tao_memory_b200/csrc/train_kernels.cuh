// Training forward kernels of tao_attention on sm_100a.
//
// Reference: tao_stream.py:80-123 (writer over all blocks), 530-593 (page
// summaries), 596-665 (per-tile routing and selected read), operator.py:21-39
// (fusion).  Every query routes (route_interval = 1): tile t of 256 queries sees
// the first max(0, t - 2) sealed fines.
#pragma once
#include "tcgen05.cuh"
#include "common.cuh"
#include "window_attention.cuh"

namespace tao {

struct TrainDims {
  int B, T, H, S;   // S = T/256 - 1 sealed blocks (0 when T <= 768)
  long long row;    // token stride in elements (H * D)
};

// both values rounded to bf16 (one cvt.rn.bf16x2.f32)
TAO_DEVI void rb2(float& x, float& y) {
  const uint32_t u = wa::pack_bf16(x, y);
  x = lo_f(u);
  y = hi_f(u);
}
// bf16 pair of two values that are already bf16-representable (no rounding)
TAO_DEVI uint32_t pack_exact(float x, float y) {
  return (__float_as_uint(x) >> 16) | (__float_as_uint(y) & 0xffff0000u);
}

// Per-channel max and partition of a staged [256][D] key block, with the token
// range split over NTHREADS / D thread groups (partials combined in `scratch`,
// 2 * NTHREADS floats): m = max_t k, Z = bf16(sum_t bf16(exp(bf16(k - m)))).
// Tokens go two at a time (one packed conversion per rounding point, the sum
// still in token order); eset(t, d, e) receives every e = bf16(exp(bf16(k - m))).
template <int D, int NTHREADS, typename KAt, typename ESet>
TAO_DEVI void channel_stats(KAt kat, float* mx, float* zp, float* scratch, ESet eset) {
  constexpr int G = NTHREADS / D, TPG = 256 / G;
  const int tid = threadIdx.x, d = tid % D, grp = tid / D;
  float m = -INFINITY;
  for (int t = grp * TPG; t < (grp + 1) * TPG; ++t) m = fmaxf(m, kat(t, d));
  scratch[grp * D + d] = m;
  __syncthreads();
  m = -INFINITY;
#pragma unroll
  for (int x = 0; x < G; ++x) m = fmaxf(m, scratch[x * D + d]);
  float sum = 0.f;
  for (int t = grp * TPG; t < (grp + 1) * TPG; t += 2) {
    float e0 = __fsub_rn(kat(t, d), m), e1 = __fsub_rn(kat(t + 1, d), m);
    rb2(e0, e1);
    e0 = expf(e0);
    e1 = expf(e1);
    rb2(e0, e1);
    eset(t, d, e0);
    eset(t + 1, d, e1);
    sum += e0;
    sum += e1;
  }
  scratch[NTHREADS + grp * D + d] = sum;
  __syncthreads();
  if (grp == 0) {
    float z = 0.f;
#pragma unroll
    for (int x = 0; x < G; ++x) z += scratch[NTHREADS + x * D + d];
    mx[d] = m;
    zp[d] = rb(z);
  }
  __syncthreads();
}
template <int D, int NTHREADS, typename KAt>
TAO_DEVI void channel_stats(KAt kat, float* mx, float* zp, float* scratch) {
  channel_stats<D, NTHREADS>(kat, mx, zp, scratch, [](int, int, float) {});
}

// ---------------------------------------------------------------------------
// Writer: one CTA per (b, h, block s).  z[b][h][s][d] and C[b][h][s][d][e] with
// the reference's rounding points; C = p^T v on the tensor cores.
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(128) writer_kernel(const bf16* __restrict__ raw_k,
                                                     const bf16* __restrict__ v, bf16* z_out,
                                                     bf16* c_out, TrainDims dm, int write_c) {
  using namespace wa;
  constexpr int NT = 256, CH = D / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sP = smem_u32(smem);        // [256][D] raw keys, then probabilities
  const uint32_t sV = sP + NT * D * 2;       // [256][D]
  float* mx = reinterpret_cast<float*>(smem + 2 * NT * D * 2);
  float* zp = mx + D;
  const int s = blockIdx.x % dm.S, h = (blockIdx.x / dm.S) % dm.H, b = blockIdx.x / (dm.S * dm.H);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bf16* kb = raw_k + ((long long)b * dm.T + (long long)s * NT) * dm.row + (long long)h * D;
  const bf16* vb = v + ((long long)b * dm.T + (long long)s * NT) * dm.row + (long long)h * D;
  for (int idx = tid; idx < NT * CH; idx += 128) {
    int r = idx / CH, c = idx % CH;
    cp_async16(sP + swz(r, c * 8, D), kb + (long long)r * dm.row + c * 8, true);
    cp_async16(sV + swz(r, c * 8, D), vb + (long long)r * dm.row + c * 8, true);
  }
  cp_commit();
  cp_wait<0>();
  __syncthreads();
  auto at = [&](int r, int d) -> bf16& {
    return *reinterpret_cast<bf16*>(smem + swz(r, d, D));
  };
  // per channel: max, partition = bf16(sum_t bf16(exp(bf16(k - max))))
  __shared__ float stat_scratch[2 * 128];
  // e replaces the key in shared memory (it is exact in bf16); p = bf16(e / Z)
  channel_stats<D, 128>([&](int t, int d) { return bf(at(t, d)); }, mx, zp, stat_scratch,
                        [&](int t, int d, float e) { at(t, d) = tobf(e); });
  for (int idx = tid; idx < NT * D / 2; idx += 128) {  // two channels at a time
    const int t = idx / (D / 2), d = (idx % (D / 2)) * 2;
    uint32_t* cell = reinterpret_cast<uint32_t*>(smem + swz(t, d, D));
    const uint32_t e2 = *cell;
    *cell = wa::pack_bf16(__fdiv_rn(lo_f(e2), zp[d]), __fdiv_rn(hi_f(e2), zp[d + 1]));
  }
  bf16* zo = z_out + (((long long)b * dm.H + h) * dm.S + s) * D;
  for (int d = tid; d < D; d += 128) zo[d] = tobf(__fadd_rn(mx[d], rb(logf(zp[d]))));
  if (!write_c) return;  // the caller supplies C (another fine writer)
  __syncthreads();
  // C[d][e] = sum_t p[t][d] v[t][e]: warp w owns rows d in [w*D/4, (w+1)*D/4)
  constexpr int MT = D / 64;  // m-tiles of 16 rows per warp: 1 (D64) or 2 (D128)
  constexpr int NTL = D / 8;  // n-tiles of 8 columns
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
      ldsm_x4_t(sP + swz(r, c, D), a[i][0], a[i][1], a[i][2], a[i][3]);
    }
#pragma unroll
    for (int np = 0; np < D / 16; ++np) {
      uint32_t b0, b1, b2, b3;
      const int r = kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int c = np * 16 + (lane >> 4) * 8;
      ldsm_x4_t(sV + swz(r, c, D), b0, b1, b2, b3);
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        mma16816(acc[i][2 * np], a[i], b0, b1);
        mma16816(acc[i][2 * np + 1], a[i], b2, b3);
      }
    }
  }
  bf16* co = c_out + (((long long)b * dm.H + h) * dm.S + s) * (long long)D * D;
  const int g = lane >> 2, c4 = lane & 3;
#pragma unroll
  for (int i = 0; i < MT; ++i) {
    const int d0 = warp * (D / 4) + i * 16;
#pragma unroll
    for (int j = 0; j < NTL; ++j) {
      const int e = j * 8 + c4 * 2;
      *reinterpret_cast<__nv_bfloat162*>(co + (long long)(d0 + g) * D + e) =
          __floats2bfloat162_rn(acc[i][j][0], acc[i][j][1]);
      *reinterpret_cast<__nv_bfloat162*>(co + (long long)(d0 + g + 8) * D + e) =
          __floats2bfloat162_rn(acc[i][j][2], acc[i][j][3]);
    }
  }
}

// ---------------------------------------------------------------------------
// Page prefix table: pzpre[b][h][p][n-1][d] = bf16 logsumexp composite over the
// first n fines of page p (n = 1..8), the page log-partition a tile sees for a
// pending page of n fines (n = 8: a completed page).  tao_stream.py:530-593.
// ---------------------------------------------------------------------------
template <int D>
__global__ void page_prefix_kernel(const bf16* __restrict__ z, bf16* pzpre, TrainDims dm, int pages) {
  const long long total = (long long)dm.B * dm.H * pages * D;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(idx % D);
    const int p = (int)((idx / D) % pages);
    const long long bh = idx / ((long long)D * pages);
    const bf16* zb = z + (bh * dm.S + (long long)p * kGroup) * D + d;
    const int avail = min(kGroup, dm.S - p * kGroup);
    for (int n = 1; n <= kGroup; ++n) {
      float out = 0.f;
      if (n <= avail) {
        float mx = -INFINITY;
        for (int i = 0; i < n; ++i) mx = fmaxf(mx, bf(zb[(long long)i * D]));
        const float m0 = (fabsf(mx) == INFINITY) ? 0.f : mx;
        float s = 0.f;
        for (int i = 0; i < n; ++i) s += rb(expf(rb(__fsub_rn(bf(zb[(long long)i * D]), m0))));
        out = rb(__fadd_rn(rb(logf(rb(s))), m0));
      }
      pzpre[((bh * pages + p) * kGroup + (n - 1)) * D + d] = tobf(out);
    }
  }
}

// ---------------------------------------------------------------------------
// Training read: one CTA (256 threads) per (tile of 256 queries, b, h).
//  1. page table of the tile: completed pages + the pending prefix; page weights
//     pw = bf16(softmax over pages); segment weights sw[s] = bf16(exp(bf16(z-pz)))
//  2. thread q routes query q: h = bf16(softmax(raw_q)), page mass top-K (stable),
//     candidate scores bf16(sum_d bf16(bf16(h*pw)*sw)), top-M (stable) kept as an
//     insertion list; den = bf16(sum of the selected scores)
//  3. for every fine s selected by some query of the tile: A_s[q] = a_{q,s}
//     (zero rows for queries that did not select s), acc += A_s . C_s on the
//     tensor cores (C_s double-buffered through cp.async)
//  4. epilogue: num = bf16(acc), fine = bf16(num/den), pointwise fusion -> out.
// Tiles without history (t < 3) copy the local output.
// ---------------------------------------------------------------------------
struct ReadArgs {
  const bf16 *raw_q, *local, *fa, *fb;  // [B,T,H,D] x2, [H,D,3] x2
  const float* gain;                     // [H] bf16(2*alpha_h) as float
  const bf16 *z, *C, *pzpre;             // [B,H,S,D], [B,H,S,D,D], [B,H,pages,8,D]
  bf16* out;                             // [B,T,H,D]
  bf16* num_out;                         // [B,T,H,D]   (saved for backward)
  float* den_out;                        // [B,T,H]
  int16_t* sel_out;                      // [B,T,H,mmax] selected fine ids (-1 pad)
  TrainDims dm;
  int pages, mmax, umax;
  int* err;
  int external_fusion;                   // 1: out = fine (the caller fuses), no pointwise gate here
  int route_only;                        // 1: routing into sel_out only (the caller reads the fines)
  int tc;                                // 1 (width 64): the selected read on tcgen05 (TMEM accumulators)
};

template <int D>
struct ReadSmem {
  static constexpr int NBUF = (D == 64) ? 2 : 1;
  static size_t bytes(int P, int V, int mmax) {
    size_t s = 0;
    s += 256 * D * 2;              // h
    s += 256 * D * 2;              // A tile
    s += NBUF * D * D * 2;         // C buffers
    s += 2 * (size_t)P * D * 4;    // pw, pz
    s += (size_t)V * D * 2 + 16;   // segment weights
    s += 256 * (size_t)(mmax + 1) * 4;  // top scores
    s += 256 * (size_t)(mmax + 1) * 4;  // top ids
    s += 256 * 4 + (size_t)(V + 8) * 4 * 2 + 256;   // den, use flags + list, misc
    s += (size_t)(V + 31) / 32 * 256 * 4;          // selection bits [word][query]
    return s + 1024;                               // slack to align the window to 1024 bytes

  }
};

// Epilogue of the selected read for channels e, e + 1 of one query (operator.py:21-39,
// index-only preset): fine = bf16(bf16(num) / den), the pointwise gate with raw_q q2
// and the local output l2 (bf16 pairs), or with external fusion fine alone; every
// rounding point rounds the pair with one conversion; bf16(x + 0) and bf16(2 * local)
// are exact and not re-rounded (x + 0 is kept: it turns -0 into +0).
TAO_DEVI void read_epilogue_pair(const ReadArgs& a, long long base, int e, float n0, float n1, float den,
                                 uint32_t q2, uint32_t l2, const float* fab0, const float* fab1, float gain) {
  const float qv[2] = {lo_f(q2), hi_f(q2)}, loc[2] = {lo_f(l2), hi_f(l2)};
  float nums[2] = {n0, n1};
  rb2(nums[0], nums[1]);
  float fine[2], s0[2], s2[2], rho0[2], rho2[2], lt[2], fg[2], res[2];
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    const float* fa = fab0 + (e + x) * 3;
    fine[x] = __fdiv_rn(nums[x], den);
    s0[x] = __fmul_rn(fa[0], qv[x]);
    s2[x] = __fmul_rn(fa[2], qv[x]);
  }
  rb2(fine[0], fine[1]);
  if (a.external_fusion) {   // the caller applies the pointwise gate: out = fine
    *reinterpret_cast<uint32_t*>(a.out + base + e) = pack_exact(fine[0], fine[1]);
    *reinterpret_cast<uint32_t*>(a.num_out + base + e) = pack_exact(nums[0], nums[1]);
    return;
  }
  rb2(s0[0], s0[1]);
  rb2(s2[0], s2[1]);
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    const float* fb = fab1 + (e + x) * 3;
    s0[x] = __fadd_rn(s0[x], fb[0]);
    s2[x] = __fadd_rn(s2[x], fb[2]);
    fg[x] = __fmul_rn(gain, fine[x]);
  }
  rb2(s0[0], s0[1]);
  rb2(s2[0], s2[1]);
  rb2(fg[0], fg[1]);
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    const float mx = fmaxf(s0[x], s2[x]);
    // the larger term is exp(0) = 1 exactly: one exponential per element
    const float eo = expf(fminf(s0[x], s2[x]) - mx);
    const float e0 = s0[x] >= s2[x] ? 1.f : eo, e2 = s0[x] >= s2[x] ? eo : 1.f;
    rho0[x] = __fdiv_rn(e0, e0 + e2);
    rho2[x] = __fdiv_rn(e2, e0 + e2);
  }
  rb2(rho0[0], rho0[1]);
  rb2(rho2[0], rho2[1]);
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    lt[x] = __fmul_rn(rho0[x], __fmul_rn(2.f, loc[x]));
    res[x] = __fmul_rn(rho2[x], fg[x]);
  }
  rb2(lt[0], lt[1]);
  rb2(res[0], res[1]);
#pragma unroll
  for (int x = 0; x < 2; ++x) res[x] = __fadd_rn(__fadd_rn(lt[x], 0.f), res[x]);
  rb2(res[0], res[1]);
  *reinterpret_cast<uint32_t*>(a.out + base + e) = pack_exact(res[0], res[1]);
  *reinterpret_cast<uint32_t*>(a.num_out + base + e) = pack_exact(nums[0], nums[1]);
}

// TC: the selected read on tcgen05 (a separate instantiation, so that each kernel
// carries the code of one contraction path only).
template <int D, bool TC = false>
__global__ void __launch_bounds__(256, 2) train_read_kernel(ReadArgs a) {
  using namespace wa;
  constexpr int NBUF = ReadSmem<D>::NBUF;
  // grid (B*H, tiles), tiles heaviest first: the longest CTAs are dispatched first
  const int tile = gridDim.y - 1 - blockIdx.y, b = blockIdx.x / a.dm.H, h = blockIdx.x % a.dm.H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = tile * 256;
  const int nq = min(256, a.dm.T - q0);
  const int V = max(0, tile - 2);
  const long long row = a.dm.row;
  const long long hoff = (long long)h * D;

  if (V == 0) {  // no history: output = local (operator.py:39); external fusion: fine = 0
    if (a.route_only) return;
    for (int idx = tid; idx < nq * (D / 8); idx += 256) {
      const int q = idx / (D / 8), c = idx % (D / 8);
      const long long off = ((long long)b * a.dm.T + q0 + q) * row + hoff + c * 8;
      *reinterpret_cast<uint4*>(a.out + off) =
          a.external_fusion ? make_uint4(0, 0, 0, 0) : *reinterpret_cast<const uint4*>(a.local + off);
    }
    return;
  }
  const int completed = V / kGroup, pending = V % kGroup, P = completed + (pending > 0);
  const Policy pol{24, 2, 2, 2};
  const Counts cnt = routed_counts(completed, pending, pol);
  const int K = cnt.coarse, M = cnt.selected;
  if (M > a.mmax || completed > 64) {
    if (tid == 0) atomicOr(a.err, kErrRouteCap);
    return;
  }

  extern __shared__ __align__(128) uint8_t smem_raw[];
  // 1024-byte aligned window: the A and C tiles are 128B-swizzled tensor-core operands
  uint8_t* const smem = smem_raw + (((smem_u32(smem_raw) + 1023u) & ~1023u) - smem_u32(smem_raw));
  uint8_t* ptr = smem;
  const uint32_t sH = smem_u32(ptr);   ptr += 256 * D * 2;
  const uint32_t sA = smem_u32(ptr);   ptr += 256 * D * 2;
  const uint32_t sC = smem_u32(ptr);   ptr += NBUF * D * D * 2;
  float* pzS = reinterpret_cast<float*>(ptr);  ptr += (size_t)P * D * 4;
  bf16* pw2S = reinterpret_cast<bf16*>(ptr);   ptr += (size_t)P * D * 2;   // page weights (bf16 values)
  ptr += (size_t)P * D * 2;                                                // (keeps the old footprint)
  bf16* swS = reinterpret_cast<bf16*>(ptr);    ptr += ((size_t)V * D * 2 + 15) / 16 * 16;
  float* topS = reinterpret_cast<float*>(ptr); ptr += 256 * (size_t)(a.mmax + 1) * 4;
  int* topI = reinterpret_cast<int*>(ptr);     ptr += 256 * (size_t)(a.mmax + 1) * 4;
  float* denS = reinterpret_cast<float*>(ptr); ptr += 256 * 4;
  uint32_t* selB = reinterpret_cast<uint32_t*>(ptr); ptr += (size_t)(V + 31) / 32 * 256 * 4;
  int* useS = reinterpret_cast<int*>(ptr);
  const int TS = a.mmax + 1;  // row stride of the top lists (odd-ish: fewer bank conflicts)

  // ---- 1. page table, page weights, segment weights
  const bf16* pzb = a.pzpre + ((long long)b * a.dm.H + h) * a.pages * kGroup * D;
  for (int idx = tid; idx < P * D; idx += 256) {
    const int p = idx / D, d = idx % D;
    const int n = (p < completed) ? kGroup : pending;
    pzS[idx] = bf(__ldg(pzb + ((long long)p * kGroup + (n - 1)) * D + d));
  }
  for (int i = tid; i < V; i += 256) useS[i] = 0;
  __syncthreads();
  for (int d = tid; d < D; d += 256) {
    float mx = -INFINITY;
    for (int p = 0; p < P; ++p) mx = fmaxf(mx, pzS[p * D + d]);
    float sum = 0.f;
    for (int p = 0; p < P; ++p) sum += expf(pzS[p * D + d] - mx);
    for (int p = 0; p < P; ++p) pw2S[p * D + d] = tobf(__fdiv_rn(expf(pzS[p * D + d] - mx), sum));
  }
  const bf16* zb = a.z + ((long long)b * a.dm.H + h) * a.dm.S * D;
#pragma unroll 4
  for (int idx = tid; idx < V * D; idx += 256) {
    const int s = idx / D, d = idx % D;
    swS[idx] = tobf(expf(rb(__fsub_rn(bf(__ldg(zb + (long long)s * D + d)), pzS[(s / kGroup) * D + d]))));
  }
  // ---- h = bf16(softmax(raw_q)) per query, stored swizzled
  const int q = tid;
  const bool live = q < nq;
  const bf16* rq = a.raw_q + ((long long)b * a.dm.T + q0 + q) * row + hoff;
  if (live) {
    // the query row, read once into registers (width 64; width 128 re-reads it)
    uint4 rqv[D == 64 ? D / 8 : 1];
    if constexpr (D == 64) {
#pragma unroll
      for (int c = 0; c < D / 8; ++c) rqv[c] = *reinterpret_cast<const uint4*>(rq + c * 8);
    }
    auto rq_chunk = [&](int c) -> uint4 {
      if constexpr (D == 64) return rqv[c];
      else return *reinterpret_cast<const uint4*>(rq + c * 8);
    };
    float mx = -INFINITY;
    for (int c = 0; c < D / 8; ++c) {
      float f[8];
      unpack8(rq_chunk(c), f);
      for (int e = 0; e < 8; ++e) mx = fmaxf(mx, f[e]);
    }
    float sum = 0.f;
    for (int c = 0; c < D / 8; ++c) {
      float f[8];
      unpack8(rq_chunk(c), f);
      for (int e = 0; e < 8; ++e) sum += expf(f[e] - mx);
    }
    for (int c = 0; c < D / 8; ++c) {
      float f[8];
      unpack8(rq_chunk(c), f);
      __nv_bfloat162 o[4];
      for (int e = 0; e < 4; ++e)
        o[e] = __floats2bfloat162_rn(__fdiv_rn(expf(f[2 * e] - mx), sum), __fdiv_rn(expf(f[2 * e + 1] - mx), sum));
      *reinterpret_cast<uint4*>(smem + swz(q, c * 8, D)) = *reinterpret_cast<uint4*>(o);
    }
  }
  __syncthreads();

  // ---- 2. routing of query q (thread q).  Products are formed two at a time as
  // bf16 pairs (bit-identical to rounding each fp32 product) and summed in fp32
  // in channel order.
  float* tS = topS + q * TS;
  int* tI = topI + q * TS;
  int nt = 0;
  const uint32_t* pw2 = reinterpret_cast<const uint32_t*>(pw2S);  // [P][D/2]
  const uint32_t* sw2 = reinterpret_cast<const uint32_t*>(swS);   // [V][D/2]
  auto hchunk = [&](int c) -> uint4 { return *reinterpret_cast<const uint4*>(smem + swz(q, c * 8, D)); };
  // hv = bf16(h * pw[page]) as D/2 pairs
  auto page_hv = [&](int page, uint32_t* hv) {
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      const uint4 hc = hchunk(c);
      const uint4 pc = *reinterpret_cast<const uint4*>(pw2 + page * (D / 2) + c * 4);
      hv[c * 4 + 0] = hmul2u(hc.x, pc.x);
      hv[c * 4 + 1] = hmul2u(hc.y, pc.y);
      hv[c * 4 + 2] = hmul2u(hc.z, pc.z);
      hv[c * 4 + 3] = hmul2u(hc.w, pc.w);
    }
  };
  if (live) {
    // page scores once, then the K best pages (ties: lower page first)
    float ps[64];
    for (int p = 0; p < completed; ++p) {
      float m = 0.f;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        const uint4 hc = hchunk(c);
        const uint4 pc = *reinterpret_cast<const uint4*>(pw2 + p * (D / 2) + c * 4);
        const uint32_t pr[4] = {hmul2u(hc.x, pc.x), hmul2u(hc.y, pc.y), hmul2u(hc.z, pc.z), hmul2u(hc.w, pc.w)};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          m += lo_f(pr[u]);
          m += hi_f(pr[u]);
        }
      }
      ps[p] = rb(m);
    }
    uint64_t chosen = 0;
    for (int k = 0; k < K; ++k) {
      float best = -INFINITY;
      int bp = 0;
      for (int p = 0; p < completed; ++p) {
        if ((chosen >> p) & 1ull) continue;
        if (ps[p] > best) { best = ps[p]; bp = p; }
      }
      chosen |= 1ull << bp;
    }
    float thr = -INFINITY;  // score of the M-th entry once the list is full
    auto consider = [&](int id, float sc) {
      if (nt == M && sc <= thr) return;   // equal scores keep the older id: rejected
      int pos = 0;
      while (pos < nt && tS[pos] >= sc) ++pos;   // stable: equal scores keep the older id first
      if (pos >= M) return;
      const int last = (nt < M) ? nt : M - 1;
      for (int j = last; j > pos; --j) { tS[j] = tS[j - 1]; tI[j] = tI[j - 1]; }
      tS[pos] = sc;
      tI[pos] = id;
      if (nt < M) ++nt;
      if (nt == M) thr = tS[M - 1];
    };
    // candidate fines of a page: score = bf16(sum_d bf16(hv * w_fine))
    auto page_candidates = [&](int page, int first, int count) {
      uint32_t hv[D / 2];
      page_hv(page, hv);
      for (int j = 0; j < count; ++j) {
        const int id = first + j;
        float sc = 0.f;
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
          const uint4 wc = *reinterpret_cast<const uint4*>(sw2 + id * (D / 2) + c * 4);
          const uint32_t pr[4] = {hmul2u(hv[c * 4], wc.x), hmul2u(hv[c * 4 + 1], wc.y), hmul2u(hv[c * 4 + 2], wc.z),
                                  hmul2u(hv[c * 4 + 3], wc.w)};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            sc += lo_f(pr[u]);
            sc += hi_f(pr[u]);
          }
        }
        consider(id, rb(sc));
      }
    };
    for (int p = 0; p < completed; ++p)
      if ((chosen >> p) & 1ull) page_candidates(p, p * kGroup, kGroup);
    if (pending > 0) page_candidates(completed, completed * kGroup, pending);
    float den = 0.f;
    for (int m = 0; m < nt; ++m) {
      den += tS[m];
      useS[tI[m]] = 1;
    }
    denS[q] = rb(den);
    for (int w = 0; w < (V + 31) / 32; ++w) selB[w * 256 + q] = 0u;
    for (int m = 0; m < nt; ++m) selB[(tI[m] >> 5) * 256 + q] |= 1u << (tI[m] & 31);
    int16_t* so = a.sel_out + (((long long)b * a.dm.T + q0 + q) * a.dm.H + h) * a.mmax;
    for (int m = 0; m < a.mmax; ++m) so[m] = (int16_t)(m < nt ? tI[m] : -1);
    a.den_out[((long long)b * a.dm.T + q0 + q) * a.dm.H + h] = denS[q];
  }
  __syncthreads();
  int* list = useS + V;  // compacted list of fines selected by some query of the tile
  __shared__ int nused;
  if (tid == 0) {
    int n = 0;
    for (int s2 = 0; s2 < V; ++s2)
      if (useS[s2]) list[n++] = s2;
    nused = n;
  }
  __syncthreads();
  if (a.route_only) return;  // the caller reads the selected fines itself
  __shared__ float fabS[2][D * 3];   // the epilogue's fusion parameters of this head

  if constexpr (TC) {
    {
      // ---- 3'. the selected read on the 5th-generation tensor cores.  Per listed fine i:
      // each thread writes its query's row of A_i = bf16(hv * w) (zero when the query
      // did not select the fine) into TMEM (tcgen05.st: lane = row, a 32-bit column =
      // two channels), then one thread issues NUM[rows 0-127] += A_i[0:128] C_i and
      // NUM[rows 128-255] += A_i[128:256] C_i as tcgen05.mma with A read from TMEM
      // (M = 128, N = 64, K = 64; C_i [d][e] from shared memory, 128B-swizzled, read
      // MN-major) into two TMEM accumulators, and commits to the mbarrier of A buffer
      // i % 2.  A has two TMEM buffers and C four shared-memory buffers: while MMA i runs
      // the threads form A_{i+1} and C_{i+2} is in flight; a buffer is reused only after
      // the MMA that read it has committed (bounded waits).
      // TMEM: accumulators at columns 0 and D, A buffers (both row halves, D/2 columns
      // each) at 2D and 3D: 256 columns at width 64, 512 at width 128.  Width 128 keeps
      // three C buffers (one in the C region, two in the A tile) and loads one fine
      // ahead instead of two.
      using namespace tc;
      constexpr int TCOLS = D == 64 ? 256 : 512;
      constexpr int NCR = NBUF;        // C buffers in the C region
      constexpr int NC = NCR + 2;      // ring of C buffers (two more in the A tile)
      constexpr int PF = NC - 2;       // fines loaded ahead
      constexpr uint32_t CLBO = D == 64 ? 8192 : 16384;  // MN-major C: 64-column atoms 16 KB apart
      __shared__ __align__(8) uint64_t tbar[2];
      __shared__ uint32_t tslot;
      __shared__ int tok;
      if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tslot)),
                     "r"(TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
      }
      if (tid == 0) {
        mbar_init(&tbar[0], 1);
        mbar_init(&tbar[1], 1);
        fence_mbar_init();
      }
      fence_before();
      __syncthreads();
      fence_after();
      const uint32_t tacc = tslot;
      const bf16* cbt = a.C + ((long long)b * a.dm.H + h) * a.dm.S * (long long)D * D;
      // C buffers 0 .. NCR-1 in the C region, two more in the (now unused) A tile; a C
      // tile [d][e] in 64-column 128B-swizzled atoms (the layout of a TMA box)
      auto cbuf = [&](int k) -> uint32_t { return k < NCR ? sC + k * D * D * 2 : sA + (k - NCR) * D * D * 2; };
      auto load_ct = [&](int s2, int k) {
        const bf16* src = cbt + (long long)s2 * D * D;
        for (int idx = tid; idx < D * D / 8; idx += 256) {
          const int r = idx / (D / 8), c = idx % (D / 8);
          const uint32_t off = (uint32_t)((c >> 3) * 16384 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
          cp_async16(cbuf(k) + off, src + r * D + c * 8, true);
        }
        cp_commit();
      };
      constexpr uint32_t I = idesc_bf16(128, D, 0, 1);
      const int nu = nused;
      const uint32_t arow = (uint32_t)((warp & 3) * 32) << 16;   // this warp's TMEM lanes
      const int half = warp >> 2;                                  // rows 0-127 or 128-255
      bool ok = true;
      int issued = 0;   // MMA groups committed
#pragma unroll
      for (int p0 = 0; p0 < PF; ++p0)
        if (nu > p0) load_ct(list[p0], p0);
      for (int i = 0; i < nu; ++i) {
        const int s2 = list[i], ab = i & 1;
        if (i >= 2) {   // MMA i-2 read A buffer ab and C buffer (i-2) % 4
          if (tid == 0) tok = mbar_wait(&tbar[ab], (uint32_t)(((i >> 1) - 1) & 1), a.err) ? 1 : 0;
          __syncthreads();
          fence_after();
          if (!tok) {
            ok = false;
            break;
          }
        }
        if (i + PF < nu) load_ct(list[i + PF], (i + PF) % NC);
        const bool sel = live && ((selB[(s2 >> 5) * 256 + q] >> (s2 & 31)) & 1u);
        const uint32_t tA = tacc + 2 * D + ab * D + half * (D / 2) + arow;
        if constexpr (D == 64) {
          uint32_t arow_v[32];
          if (sel) {
            uint32_t hv[D / 2];
            page_hv(s2 / kGroup, hv);
#pragma unroll
            for (int c = 0; c < D / 2; ++c) arow_v[c] = hmul2u(hv[c], sw2[s2 * (D / 2) + c]);
          } else {
#pragma unroll
            for (int c = 0; c < D / 2; ++c) arow_v[c] = 0u;
          }
          tmem_st32u(tA, arow_v);
        } else {
          // the row in 64-channel pieces: bf16(bf16(h * page w) * fine w)
          const int page = s2 / kGroup;
#pragma unroll
          for (int j = 0; j < D / 64; ++j) {
            uint32_t arow_v[32];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const int cc = j * 8 + c;
              if (sel) {
                const uint4 hc = hchunk(cc);
                const uint4 pc = *reinterpret_cast<const uint4*>(pw2 + page * (D / 2) + cc * 4);
                const uint4 wc = *reinterpret_cast<const uint4*>(sw2 + s2 * (D / 2) + cc * 4);
                arow_v[c * 4 + 0] = hmul2u(hmul2u(hc.x, pc.x), wc.x);
                arow_v[c * 4 + 1] = hmul2u(hmul2u(hc.y, pc.y), wc.y);
                arow_v[c * 4 + 2] = hmul2u(hmul2u(hc.z, pc.z), wc.z);
                arow_v[c * 4 + 3] = hmul2u(hmul2u(hc.w, pc.w), wc.w);
              } else {
                arow_v[c * 4 + 0] = arow_v[c * 4 + 1] = arow_v[c * 4 + 2] = arow_v[c * 4 + 3] = 0u;
              }
            }
            tmem_st32u(tA + j * 32, arow_v);
          }
        }
        // C_i complete: at most the PF later loads stay in flight
        if constexpr (PF == 2) {
          if (i + 2 < nu) cp_wait<2>();
          else if (i + 1 < nu) cp_wait<1>();
          else cp_wait<0>();
        } else {
          if (i + 1 < nu) cp_wait<1>();
          else cp_wait<0>();
        }
        fence_proxy_async();
        fence_before();
        __syncthreads();
        if (tid == 0) {
          fence_after();
          const uint32_t cB = cbuf(i % NC);
          const uint32_t tAb = tacc + 2 * D + ab * D;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t accf = (i > 0 || k > 0) ? 1u : 0u;
            mma_ts(tacc, tAb + k * 8, sdesc(cB + k * 2048, CLBO, 1024), I, accf);
            mma_ts(tacc + D, tAb + D / 2 + k * 8, sdesc(cB + k * 2048, CLBO, 1024), I, accf);
          }
          commit(&tbar[ab]);
        }
        issued = i + 1;
      }
      // the last committed group covers every earlier MMA (also after a failed wait:
      // nothing is left in flight when the TMEM is freed)
      if (issued > 0) {
        const int last = issued - 1;
        if (tid == 0) tok = mbar_wait(&tbar[last & 1], (uint32_t)((last >> 1) & 1), a.err) ? 1 : 0;
        __syncthreads();
        fence_after();
        ok = ok && tok != 0;
      }
      // epilogue: raw_q and local rows staged (coalesced) into the h and A tiles
      for (int idx = tid; idx < nq * (D / 8); idx += 256) {
        const int r = idx / (D / 8), c = idx % (D / 8);
        const long long off = ((long long)b * a.dm.T + q0 + r) * row + hoff + c * 8;
        cp_async16(sH + swz(r, c * 8, D), a.raw_q + off, true);
        cp_async16(sA + swz(r, c * 8, D), a.local + off, true);
      }
      cp_commit();
      for (int idx = tid; idx < D * 3; idx += 256) {
        fabS[0][idx] = bf(a.fa[(long long)h * D * 3 + idx]);
        fabS[1][idx] = bf(a.fb[(long long)h * D * 3 + idx]);
      }
      cp_wait<0>();
      __syncthreads();
      if (ok) {
        // thread t holds query row t: warps 0-3 read accumulator 0 (rows 0-127), warps
        // 4-7 accumulator 1 (rows 128-255), each its 32 TMEM lanes
        const float gain = a.gain[h];
        const int r = tid;
        const uint32_t tl = tacc + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(warp >> 2) * D;
        const long long base = ((long long)b * a.dm.T + q0 + r) * row + hoff;
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          float v[32];
          if (nu > 0) {
            tmem_ld32(tl + c0, v);
          } else {
#pragma unroll
            for (int x = 0; x < 32; ++x) v[x] = 0.f;
          }
          if (r < nq) {
            const float den = denS[r];
#pragma unroll
            for (int x = 0; x < 32; x += 2) {
              const int e = c0 + x;
              const uint32_t q2 = *reinterpret_cast<const uint32_t*>(smem + swz(r, e, D));
              const uint32_t l2 = *reinterpret_cast<const uint32_t*>(smem + 256 * D * 2 + swz(r, e, D));
              read_epilogue_pair(a, base, e, v[x], v[x + 1], den, q2, l2, fabS[0], fabS[1], gain);
            }
          }
        }
      }
      fence_before();
      __syncthreads();
      if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tacc), "r"(TCOLS));
      return;
    }
  } else {
  // ---- 3. dense per-fine GEMMs on the tensor cores
  constexpr int NTL = D / 8;
  float acc[2][NTL][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < NTL; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.f;
  const bf16* cb = a.C + ((long long)b * a.dm.H + h) * a.dm.S * (long long)D * D;
  auto load_c = [&](int s2, int buf) {
    const bf16* src = cb + (long long)s2 * D * D;
    for (int idx = tid; idx < D * D / 8; idx += 256) {
      const int r = idx / (D / 8), c = idx % (D / 8);
      cp_async16(sC + buf * D * D * 2 + swz(r, c * 8, D), src + r * D + c * 8, true);
    }
    cp_commit();
  };
  const int nu = nused;
  if (nu > 0) load_c(list[0], 0);
  for (int i = 0; i < nu; ++i) {
    const int s2 = list[i];
    const int buf = (NBUF == 2) ? (i & 1) : 0;
    if (NBUF == 2 && i + 1 < nu) load_c(list[i + 1], buf ^ 1);
    // A_s row q: bf16(hv * w_s) where query q selected fine s2, else zero
    const bool sel = live && ((selB[(s2 >> 5) * 256 + q] >> (s2 & 31)) & 1u);
    if (sel) {
      uint32_t hv[D / 2];
      page_hv(s2 / kGroup, hv);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        const uint4 wc = *reinterpret_cast<const uint4*>(sw2 + s2 * (D / 2) + c * 4);
        const uint4 o = make_uint4(hmul2u(hv[c * 4], wc.x), hmul2u(hv[c * 4 + 1], wc.y),
                                   hmul2u(hv[c * 4 + 2], wc.z), hmul2u(hv[c * 4 + 3], wc.w));
        *reinterpret_cast<uint4*>(smem + 256 * D * 2 + swz(q, c * 8, D)) = o;
      }
    } else {
      for (int c = 0; c < D / 8; ++c)
        *reinterpret_cast<uint4*>(smem + 256 * D * 2 + swz(q, c * 8, D)) = make_uint4(0, 0, 0, 0);
    }
    if (NBUF == 2 && i + 1 < nu) cp_wait<1>(); else cp_wait<0>();
    __syncthreads();
#pragma unroll
    for (int kt = 0; kt < D / 16; ++kt) {
      uint32_t af[2][4];
#pragma unroll
      for (int mi = 0; mi < 2; ++mi) {
        const int r = warp * 32 + mi * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kt * 16 + (lane >> 4) * 8;
        ldsm_x4(sA + swz(r, c, D), af[mi][0], af[mi][1], af[mi][2], af[mi][3]);
      }
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = np * 16 + (lane >> 4) * 8;
        ldsm_x4_t(sC + buf * D * D * 2 + swz(r, c, D), b0, b1, b2, b3);
#pragma unroll
        for (int mi = 0; mi < 2; ++mi) {
          mma16816(acc[mi][2 * np], af[mi], b0, b1);
          mma16816(acc[mi][2 * np + 1], af[mi], b2, b3);
        }
      }
    }
    __syncthreads();
    if (NBUF == 1 && i + 1 < nu) load_c(list[i + 1], 0);
  }

  // ---- 4. epilogue: num, fine, fusion (operator.py:21-39, index-only preset).
  // The tile's raw_q and local rows are staged (coalesced) into the h and A
  // buffers, free now, and the fusion parameters of this head into shared memory.
  for (int idx = tid; idx < nq * (D / 8); idx += 256) {
    const int r = idx / (D / 8), c = idx % (D / 8);
    const long long off = ((long long)b * a.dm.T + q0 + r) * row + hoff + c * 8;
    cp_async16(sH + swz(r, c * 8, D), a.raw_q + off, true);
    cp_async16(sA + swz(r, c * 8, D), a.local + off, true);
  }
  cp_commit();
  for (int idx = tid; idx < D * 3; idx += 256) {
    fabS[0][idx] = bf(a.fa[(long long)h * D * 3 + idx]);
    fabS[1][idx] = bf(a.fb[(long long)h * D * 3 + idx]);
  }
  cp_wait<0>();
  __syncthreads();
  const float gain = a.gain[h];
  const int g = lane >> 2, c4 = lane & 3;
#pragma unroll
  for (int mi = 0; mi < 2; ++mi) {
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = warp * 32 + mi * 16 + g + hr * 8;
      if (r >= nq) continue;
      const float den = denS[r];
      const long long base = ((long long)b * a.dm.T + q0 + r) * row + hoff;
#pragma unroll
      for (int j = 0; j < NTL; ++j) {
        // channels e, e + 1: every rounding point rounds the pair with one conversion;
        // bf16(x + 0) and bf16(2 * local) are exact and not re-rounded (x + 0 is kept:
        // it turns -0 into +0)
        const int e = j * 8 + c4 * 2;
        const uint32_t q2 = *reinterpret_cast<const uint32_t*>(smem + swz(r, e, D));
        const uint32_t l2 = *reinterpret_cast<const uint32_t*>(smem + 256 * D * 2 + swz(r, e, D));
        read_epilogue_pair(a, base, e, acc[mi][j][hr * 2], acc[mi][j][hr * 2 + 1], den, q2, l2, fabS[0], fabS[1],
                           gain);
      }
    }
  }
  }  // the mma.sync path
}

}  // namespace tao
