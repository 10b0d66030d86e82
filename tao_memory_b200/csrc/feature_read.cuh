// Feature-mass read of training and its backward on the 5th-generation tensor cores
// (sm_100a): the read of the feature-read fine writers (feature-mass and
// structured-Gram), reference _read_training_group (tao_stream.py:600-601, 658-661)
// with feature_read_coefficients (association_writer.py:43-53) and
// selected_fine_numerator / _SelectedContraction (indirect_fine.py:65-133).
//
// One CTA of 128 threads per (batch, head, block of 128 queries); thread i owns
// query q0 + i.  Per query: h = bf16(fp32 softmax(raw_q)), for each selected fine m
// mass_m = sum_d h_d exp(z_m,d) (fp32), w_m = mass_m / sum_j mass_j and the
// coefficients a_m,d = bf16(w_m h_d).  The contraction out = sum_m a_m . C_m runs
// fine by fine over the block: for each fine s selected by some query of the block,
// the block's coefficient rows for s (zero for queries that did not select it) form
// the A operand A_s [128 queries x D] and
//   forward:   OUT += A_s C_s                      (M = 128, N = D, K = D)
//   backward:  dA_s = G C_s^T                      (M = 128, N = D, K = D)
//              dC_s = A_s^T G                      (M = D padded to 128, N = D, K = 128)
// each as tcgen05.mma issued by one thread into TMEM accumulators, operands in shared
// memory with 128-byte swizzle: A_s and G K-major (query rows of 128 B per 64-channel
// atom), C_s stored [d][e] (read MN-major for the forward, K-major for dA), A_s^T and
// G read MN-major for dC.  At width 64 the dC instruction's rows 64-127 take the G
// tile (placed right after A_s) as a stand-in and land in TMEM lanes nobody reads.
// Waits on the tensor core are bounded; a timeout records kErrWaitTimeout, drains the
// MMA in flight (bounded) and frees the TMEM.
#pragma once
#include "common.cuh"
#include "tcgen05.cuh"
#include "window_attention.cuh"

namespace tao {

constexpr int kFeatQ = 128;  // queries per CTA

// Byte offset of (row r, column c) in a tile of `rows` rows whose columns come in
// 64-column atoms of rows x 128 B, 16-byte chunks XOR-swizzled by r % 8 (the
// canonical 128B-swizzled operand layout).
TAO_DEVI uint32_t sw_off(int r, int c, int rows) {
  return (uint32_t)(c >> 6) * (uint32_t)rows * 128u + (uint32_t)r * 128u +
         ((uint32_t)(((c & 63) >> 3) ^ (r & 7)) << 4) + ((uint32_t)(c & 7) << 1);
}

// Shared-memory plan of one CTA (bytes); `back` adds the backward's buffers.
template <int D>
struct FeatSmem {
  static constexpr int HS = D + 2;                  // padded bf16 row of h (conflict-free)
  static constexpr uint32_t ATILE = kFeatQ * D * 2;   // A_s or G: 128 rows x D
  static constexpr uint32_t CTILE = D * D * 2;        // C_s
  size_t a, g, c, h, e, w, id, dmix, dz, bar, total;
  __host__ __device__ FeatSmem(int V, int mmax, bool back) {
    size_t off = 0;
    a = off;  off += ATILE;                 // 1024-aligned (the window is aligned)
    g = off;  off += back ? ATILE : 0;      // right after A_s: the dC stand-in rows at width 64
    c = off;  off += CTILE;
    h = off;  off += (size_t)kFeatQ * HS * 2;
    e = off;  off += (size_t)V * D * 4;   // exp(z) of the visible fines
    w = off;  off += (size_t)kFeatQ * mmax * 4;
    id = off; off += ((size_t)kFeatQ * mmax * 2 + 15) / 16 * 16;
    dmix = off; off += back ? (size_t)kFeatQ * mmax * 4 : 0;
    dz = off; off += back ? (size_t)V * D * 4 : 0;
    bar = off; off += 64 + 256 * 4;       // mbarrier, TMEM slot, used-fine bits, list (<= 256 fines)
    total = off + 1024;                   // slack to align the window to 1024 bytes
  }
};

struct FeatArgs {
  const bf16 *raw_q, *z, *C, *g;  // [B,T,H,D], [B,H,S,D], [B,H,S,D,D], grad [B,T,H,D] (backward)
  const int16_t* sel;             // [B,T,H,mmax], -1 pads
  bf16* out;                      // forward: [B,T,H,D]; backward: d_raw_q [B,T,H,D]
  float *dz, *dc;                 // backward accumulators [B,H,S,D], [B,H,S,D,D]
  int B, T, H, S, mmax;
  int* err;
};

// Per-CTA prologue shared by the forward and the backward: h, exp(z), the selected
// fines' weights and the list of fines some query of the block selected.  Returns the
// number of listed fines (in `list`, ascending).
template <int D>
TAO_DEVI int feat_prologue(const FeatArgs& a, int b, int hh, int q0, int V, uint8_t* sm, const FeatSmem<D>& L) {
  const int tid = threadIdx.x, q = q0 + tid;
  const bool live = q < a.T;
  bf16* sH = reinterpret_cast<bf16*>(sm + L.h);
  float* sE = reinterpret_cast<float*>(sm + L.e);
  float* sW = reinterpret_cast<float*>(sm + L.w);
  int16_t* sId = reinterpret_cast<int16_t*>(sm + L.id);
  uint32_t* used = reinterpret_cast<uint32_t*>(sm + L.bar + 32);   // V <= 256: 8 words
  int* list = reinterpret_cast<int*>(sm + L.bar + 64);
  if (tid < 8) used[tid] = 0u;
  // h = bf16(softmax over channels of raw_q in fp32)
  {
    float x[D];
    if (live) {
      const uint4* src = reinterpret_cast<const uint4*>(a.raw_q + (((long long)b * a.T + q) * a.H + hh) * D);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) unpack8(__ldg(src + c), x + 8 * c);
    } else {
#pragma unroll
      for (int d = 0; d < D; ++d) x[d] = 0.f;
    }
    float mx = -INFINITY;
#pragma unroll
    for (int d = 0; d < D; ++d) mx = fmaxf(mx, x[d]);
    float sum = 0.f;
#pragma unroll
    for (int d = 0; d < D; ++d) {
      x[d] = expf(x[d] - mx);
      sum += x[d];
    }
#pragma unroll
    for (int d = 0; d < D; d += 2) {
      const float h0 = live ? __fdiv_rn(x[d], sum) : 0.f, h1 = live ? __fdiv_rn(x[d + 1], sum) : 0.f;
      *reinterpret_cast<uint32_t*>(sH + tid * FeatSmem<D>::HS + d) = wa::pack_bf16(h0, h1);
    }
  }
  const bf16* zb = a.z + ((long long)b * a.H + hh) * a.S * D;
  for (int idx = tid; idx < V * D; idx += kFeatQ) sE[idx] = expf(bf(__ldg(zb + idx)));
  __syncthreads();
  // selected fines of this query: mass_m = sum_d h_d exp(z_m,d), w_m = mass_m / total
  if (live) {
    const int16_t* so = a.sel + (((long long)b * a.T + q) * a.H + hh) * a.mmax;
    const bf16* hr = sH + tid * FeatSmem<D>::HS;
    float total = 0.f;
    int m = 0;
    for (; m < a.mmax; ++m) {
      const int s = so[m];
      if (s < 0 || s >= V) break;
      const float* er = sE + s * D;
      float mass = 0.f;
      for (int d = 0; d < D; ++d) mass += bf(hr[d]) * er[d];
      sW[tid * a.mmax + m] = mass;
      sId[tid * a.mmax + m] = (int16_t)s;
      total += mass;
      atomicOr(&used[s >> 5], 1u << (s & 31));
    }
    for (int j = 0; j < m; ++j) sW[tid * a.mmax + j] = __fdiv_rn(sW[tid * a.mmax + j], total);
    for (int j = m; j < a.mmax; ++j) sId[tid * a.mmax + j] = -1;
  } else {
    for (int j = 0; j < a.mmax; ++j) sId[tid * a.mmax + j] = -1;
  }
  __syncthreads();
  __shared__ int n_used;
  if (tid == 0) {
    int n = 0;
    for (int s = 0; s < V; ++s)
      if ((used[s >> 5] >> (s & 31)) & 1u) list[n++] = s;
    n_used = n;
  }
  __syncthreads();
  return n_used;
}

// Row `tid` of A_s (the query's coefficients for fine s, zero when it did not select
// s) in the K-major swizzled layout; returns the query's slot m of s (-1: none).
template <int D>
TAO_DEVI int feat_form_a(const FeatArgs& a, int s, uint8_t* sm, const FeatSmem<D>& L) {
  const int tid = threadIdx.x;
  const float* sW = reinterpret_cast<const float*>(sm + L.w);
  const int16_t* sId = reinterpret_cast<const int16_t*>(sm + L.id);
  const bf16* hr = reinterpret_cast<const bf16*>(sm + L.h) + tid * FeatSmem<D>::HS;
  int slot = -1;
  for (int m = 0; m < a.mmax; ++m) {
    const int id = sId[tid * a.mmax + m];
    if (id < 0) break;
    if (id == s) slot = m;
  }
  const float wv = slot >= 0 ? sW[tid * a.mmax + slot] : 0.f;
#pragma unroll
  for (int c = 0; c < D / 8; ++c) {
    const uint32_t* h2 = reinterpret_cast<const uint32_t*>(hr + 8 * c);
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) op[e] = wa::pack_bf16(__fmul_rn(wv, lo_f(h2[e])), __fmul_rn(wv, hi_f(h2[e])));
    *reinterpret_cast<uint4*>(sm + L.a + sw_off(tid, 8 * c, kFeatQ)) = o;
  }
  return slot;
}

// C_s into the swizzled [d][e] tile (cp.async; the caller waits).
template <int D>
TAO_DEVI void feat_load_c(const FeatArgs& a, int b, int hh, int s, uint8_t* sm, const FeatSmem<D>& L) {
  const bf16* cs = a.C + (((long long)b * a.H + hh) * a.S + s) * (long long)D * D;
  for (int idx = threadIdx.x; idx < D * D / 8; idx += kFeatQ) {
    const int d = idx / (D / 8), c = idx % (D / 8);
    wa::cp_async16(smem_u32(sm + L.c + sw_off(d, 8 * c, D)), cs + d * D + 8 * c, true);
  }
}

// The window of dynamic shared memory aligned to 1024 bytes (128B-swizzled operands).
TAO_DEVI uint8_t* feat_window(uint8_t* raw) {
  const uint32_t r = smem_u32(raw);
  return raw + (((r + 1023u) & ~1023u) - r);
}

template <int D>
TAO_DEVI uint32_t feat_tmem_alloc(uint8_t* sm, const FeatSmem<D>& L, uint32_t cols) {
  uint32_t* slot = reinterpret_cast<uint32_t*>(sm + L.bar + 8);
  if (threadIdx.x < 32) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 0) {
    mbar_init(reinterpret_cast<uint64_t*>(sm + L.bar), 1);
    fence_mbar_init();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  return *slot;
}

// Every thread waits (bounded) for the MMAs committed to the barrier; false after a
// timeout (the error word is set).
template <int D>
TAO_DEVI bool feat_wait(uint8_t* sm, const FeatSmem<D>& L, uint32_t phase, const FeatArgs& a) {
  int* ok = reinterpret_cast<int*>(sm + L.bar + 12);
  if (threadIdx.x == 0) *ok = mbar_wait(reinterpret_cast<uint64_t*>(sm + L.bar), phase, a.err) ? 1 : 0;
  __syncthreads();
  tc::fence_after();
  return *ok != 0;
}

template <int D>
TAO_DEVI void feat_tmem_free(uint8_t* sm, const FeatSmem<D>& L, uint32_t tbase, uint32_t cols, bool ok,
                             uint32_t phase, const FeatArgs& a) {
  if (!ok && threadIdx.x == 0)   // give the MMA still in flight its bounded wait first
    mbar_wait(reinterpret_cast<uint64_t*>(sm + L.bar), phase, a.err);
  tc::fence_before();
  __syncthreads();
  if (threadIdx.x < 32)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(cols));
}

// Forward: grid (ceil(T / 128), B * H), 128 threads.
template <int D>
__global__ void __launch_bounds__(kFeatQ) feature_read_fwd_kernel(FeatArgs a) {
  using namespace tc;
  extern __shared__ uint8_t sm_raw[];
  const int b = blockIdx.y / a.H, hh = blockIdx.y % a.H, q0 = blockIdx.x * kFeatQ;
  const int tid = threadIdx.x, warp = tid >> 5, q = q0 + tid;
  const int V = max(0, q0 / 256 - 2);
  bf16* orow = a.out + (((long long)b * a.T + q) * a.H + hh) * D;
  if (V == 0) {   // the first three tiles read no fine
    if (q < a.T)
#pragma unroll
      for (int c = 0; c < D / 8; ++c) reinterpret_cast<uint4*>(orow)[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  uint8_t* sm = feat_window(sm_raw);
  const FeatSmem<D> L(V, a.mmax, false);
  const int n = feat_prologue<D>(a, b, hh, q0, V, sm, L);
  const int* list = reinterpret_cast<const int*>(sm + L.bar + 64);
  const uint32_t tbase = feat_tmem_alloc<D>(sm, L, D);
  const uint32_t aA = smem_u32(sm + L.a), aC = smem_u32(sm + L.c);
  constexpr uint32_t I = idesc_bf16(128, D, 0, 1);   // A K-major, B (C_s, rows = d) MN-major
  uint32_t phase = 0;
  bool ok = true;
  for (int i = 0; i < n && ok; ++i) {
    const int s = list[i];
    feat_load_c<D>(a, b, hh, s, sm, L);
    wa::cp_commit();
    feat_form_a<D>(a, s, sm, L);
    wa::cp_wait<0>();
    fence_proxy_async();
    fence_before();
    __syncthreads();
    fence_after();
    if (tid == 0) {
#pragma unroll
      for (int k = 0; k < D / 16; ++k)
        mma(tbase, sdesc(aA + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024), sdesc(aC + k * 2048, D * 128, 1024), I,
            (i > 0 || k > 0) ? 1u : 0u);
      commit(reinterpret_cast<uint64_t*>(sm + L.bar));
    }
    ok = feat_wait<D>(sm, L, phase, a);
    phase ^= 1u;
  }
  if (ok) {
    // thread tid holds query row tid of the accumulator in TMEM lane tid (tcgen05.ld
    // is warp-collective: lanes of queries past T load too and store nothing)
#pragma unroll
    for (int c0 = 0; c0 < D; c0 += 32) {
      float v[32];
      if (n > 0) {
        tmem_ld32(tbase + ((uint32_t)(warp * 32) << 16) + c0, v);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0.f;
      }
      if (q < a.T) {
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 o;
          o.x = wa::pack_bf16(v[e], v[e + 1]);
          o.y = wa::pack_bf16(v[e + 2], v[e + 3]);
          o.z = wa::pack_bf16(v[e + 4], v[e + 5]);
          o.w = wa::pack_bf16(v[e + 6], v[e + 7]);
          *reinterpret_cast<uint4*>(orow + c0 + e) = o;
        }
      }
    }
  }
  feat_tmem_free<D>(sm, L, tbase, D, ok, phase ^ 1u, a);
}

// Backward: grid (ceil(T / 128), B * H), 128 threads.  Per listed fine s: dA_s and
// dC_s on the tensor cores; from dA each selecting query takes d mix_m = sum_d
// bf16(dA) h_d and d query += bf16(dA) w_m; dC_s is added to a.dc.  Then per query
// d mass_m = d mix_m / total - sum_j d mix_j mass_j / total^2, d query += d mass_m
// exp(z_m), the z terms bf16(d mass_m h_d exp(z_m,d)) are summed per fine in shared
// memory and added to a.dz, and d raw_q = bf16(softmax backward of bf16(d query)).
template <int D>
__global__ void __launch_bounds__(kFeatQ) feature_read_bwd_kernel(FeatArgs a) {
  using namespace tc;
  extern __shared__ uint8_t sm_raw[];
  const int b = blockIdx.y / a.H, hh = blockIdx.y % a.H, q0 = blockIdx.x * kFeatQ;
  const int tid = threadIdx.x, warp = tid >> 5, q = q0 + tid;
  const bool live = q < a.T;
  const int V = max(0, q0 / 256 - 2);
  const long long row = (((long long)b * a.T + q) * a.H + hh) * D;
  if (V == 0) {   // no fine read: no gradient
    if (live)
#pragma unroll
      for (int c = 0; c < D / 8; ++c) reinterpret_cast<uint4*>(a.out + row)[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  uint8_t* sm = feat_window(sm_raw);
  const FeatSmem<D> L(V, a.mmax, true);
  // G: the query rows of the gradient, K-major swizzled (zero rows past T)
#pragma unroll
  for (int c = 0; c < D / 8; ++c)
    wa::cp_async16(smem_u32(sm + L.g + sw_off(tid, 8 * c, kFeatQ)), live ? a.g + row + 8 * c : a.g, live);
  wa::cp_commit();
  float* sDmix = reinterpret_cast<float*>(sm + L.dmix);
  float* sDz = reinterpret_cast<float*>(sm + L.dz);
  for (int j = 0; j < a.mmax; ++j) sDmix[tid * a.mmax + j] = 0.f;
  for (int idx = tid; idx < V * D; idx += kFeatQ) sDz[idx] = 0.f;
  const int n = feat_prologue<D>(a, b, hh, q0, V, sm, L);
  const int* list = reinterpret_cast<const int*>(sm + L.bar + 64);
  const float* sW = reinterpret_cast<const float*>(sm + L.w);
  const float* sE = reinterpret_cast<const float*>(sm + L.e);
  const int16_t* sId = reinterpret_cast<const int16_t*>(sm + L.id);
  const bf16* hr = reinterpret_cast<const bf16*>(sm + L.h) + tid * FeatSmem<D>::HS;
  const uint32_t tbase = feat_tmem_alloc<D>(sm, L, 2 * D);
  const uint32_t aA = smem_u32(sm + L.a), aG = smem_u32(sm + L.g), aC = smem_u32(sm + L.c);
  constexpr uint32_t IA = idesc_bf16(128, D, 0, 0);   // dA = G C^T: both K-major
  constexpr uint32_t IC = idesc_bf16(128, D, 1, 1);   // dC = A^T G: both read MN-major
  float dq[D];
#pragma unroll
  for (int d = 0; d < D; ++d) dq[d] = 0.f;
  uint32_t phase = 0;
  bool ok = true;
  float* dcb = a.dc + ((long long)b * a.H + hh) * a.S * (long long)D * D;
  for (int i = 0; i < n && ok; ++i) {
    const int s = list[i];
    feat_load_c<D>(a, b, hh, s, sm, L);
    wa::cp_commit();
    const int slot = feat_form_a<D>(a, s, sm, L);
    wa::cp_wait<0>();
    fence_proxy_async();
    fence_before();
    __syncthreads();
    fence_after();
    if (tid == 0) {
#pragma unroll
      for (int k = 0; k < D / 16; ++k)
        mma(tbase, sdesc(aG + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024),
            sdesc(aC + (k >> 2) * (D * 128) + (k & 3) * 32, 16, 1024), IA, k > 0 ? 1u : 0u);
#pragma unroll
      for (int k = 0; k < kFeatQ / 16; ++k)
        mma(tbase + D, sdesc(aA + k * 2048, 16384, 1024), sdesc(aG + k * 2048, 16384, 1024), IC, k > 0 ? 1u : 0u);
      commit(reinterpret_cast<uint64_t*>(sm + L.bar));
    }
    ok = feat_wait<D>(sm, L, phase, a);
    phase ^= 1u;
    if (!ok) break;
    // dA row of this query (TMEM lane tid)
    const float wv = slot >= 0 ? sW[tid * a.mmax + slot] : 0.f;
    float dmix = 0.f;
#pragma unroll
    for (int c0 = 0; c0 < D; c0 += 32) {
      float v[32];
      tmem_ld32(tbase + ((uint32_t)(warp * 32) << 16) + c0, v);
      if (slot >= 0) {
        const uint32_t* h2 = reinterpret_cast<const uint32_t*>(hr + c0);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float a0 = rb(v[e]), a1 = rb(v[e + 1]);
          dmix += a0 * lo_f(h2[e / 2]) + a1 * hi_f(h2[e / 2]);
          dq[c0 + e] += a0 * wv;
          dq[c0 + e + 1] += a1 * wv;
        }
      }
    }
    if (slot >= 0) sDmix[tid * a.mmax + slot] = dmix;
    // dC row d = tid (TMEM lane tid of the second accumulator), added to the fine's dC
    if (warp < D / 32) {
      float* dst = dcb + (long long)s * D * D + (long long)tid * D;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        float v[32];
        tmem_ld32(tbase + ((uint32_t)(warp * 32) << 16) + D + c0, v);
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          atomicAdd(reinterpret_cast<float4*>(dst + c0 + e), make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]));
      }
    }
    fence_before();
    __syncthreads();
  }
  if (ok) {
    // the mixture and mass adjoints of this query; the z terms summed per fine
    if (live) {
      float mass[64];   // mmax <= 64 (checked by the host)
      float total = 0.f;
      int mq = 0;
      for (; mq < a.mmax; ++mq) {
        const int s = sId[tid * a.mmax + mq];
        if (s < 0) break;
        const float* er = sE + s * D;
        float m_ = 0.f;
        for (int d = 0; d < D; ++d) m_ += bf(hr[d]) * er[d];
        mass[mq] = m_;
        total += m_;
      }
      float dtot = 0.f;
      for (int m = 0; m < mq; ++m) dtot += __fdiv_rn(-sDmix[tid * a.mmax + m] * mass[m], __fmul_rn(total, total));
      for (int m = 0; m < mq; ++m) {
        const int s = sId[tid * a.mmax + m];
        const float dmass = __fdiv_rn(sDmix[tid * a.mmax + m], total) + dtot;
        const float* er = sE + s * D;
        float* dzr = sDz + s * D;
#pragma unroll
        for (int d = 0; d < D; ++d) dq[d] += dmass * er[d];
        for (int j = 0; j < D; ++j) {
          const int d = (j + tid) & (D - 1);   // rotated: the queries of one fine hit other banks
          atomicAdd(dzr + d, rb(__fmul_rn(__fmul_rn(dmass, bf(hr[d])), er[d])));
        }
      }
    }
    __syncthreads();
    float* dzg = a.dz + ((long long)b * a.H + hh) * a.S * D;
    for (int idx = tid; idx < V * D; idx += kFeatQ)
      if (sDz[idx] != 0.f) atomicAdd(dzg + idx, sDz[idx]);
    // d raw_q: softmax backward of bf16(d query) against the fp32 softmax of raw_q
    if (live) {
      const uint4* src = reinterpret_cast<const uint4*>(a.raw_q + row);
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        float x[8];
        unpack8(__ldg(src + c), x);
#pragma unroll
        for (int e = 0; e < 8; ++e) mx = fmaxf(mx, x[e]);
      }
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        float x[8];
        unpack8(__ldg(src + c), x);
#pragma unroll
        for (int e = 0; e < 8; ++e) sum += expf(x[e] - mx);
      }
      float dot = 0.f;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        float x[8];
        unpack8(__ldg(src + c), x);
#pragma unroll
        for (int e = 0; e < 8; ++e) dot += __fdiv_rn(expf(x[e] - mx), sum) * rb(dq[8 * c + e]);
      }
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        float x[8];
        unpack8(__ldg(src + c), x);
        uint4 o;
        uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const float y0 = __fdiv_rn(expf(x[e] - mx), sum), y1 = __fdiv_rn(expf(x[e + 1] - mx), sum);
          op[e / 2] = wa::pack_bf16(y0 * (rb(dq[8 * c + e]) - dot), y1 * (rb(dq[8 * c + e + 1]) - dot));
        }
        reinterpret_cast<uint4*>(a.out + row)[c] = o;
      }
    }
  }
  feat_tmem_free<D>(sm, L, tbase, 2 * D, ok, phase ^ 1u, a);
}

}  // namespace tao
