// Windowed causal attention backward on the 5th-generation tensor cores (sm_100a).
//
// Gradients of the local attention of tao_stream.py:760-787 (SDPA semantics of
// flash_attention.py:16-37): query t reads keys [ws(t), t], ws(t) =
// max(0, 256*floor(t/256) - 512), scale 1/8.  With P = exp(s/8 - lse[t]) and
// dS = P (dP - rowdot[t]), dP = dO V^T, rowdot[t] = sum_d dO[t]·O[t]:
//   dV = P^T dO,  dK = dS^T Q / 8,  dQ = dS K / 8.
// P and dS are rounded to bf16 before the products, as the mma.sync kernels do.
//
// One CTA per (128-key block, batch, head), width 64; 288 threads:
//   warps 0-7  elementwise: warp w owns key rows 32(w%4).. (its TMEM lane
//              quadrant) and query columns 64(w/4)..+63 of each query block
//   warp 8     TMA copies and MMA issue (one lane issues, the warp walks)
// TMEM (512 columns): S^T 0-127 and dP^T 128-255 (fp32, lanes = keys), dV 256-319,
// dK 320-383 (fp32, accumulated over the query blocks), dQ 384-447 (fp32, lanes =
// queries).  P^T and dS^T (bf16) go to shared memory, so the S^T / dP^T columns are
// free as soon as the elementwise warps have loaded them.
// Per query block i (128 queries):
//   S^T = K Q_i^T, dP^T = V dO_i^T                          (SS, N=128)   -> sfull
//   elementwise: load S^T, dP^T -> sfree (the issuer starts block i+1's S^T, dP^T);
//   P^T, dS^T in registers; then (block i-1's products done: ofull) read out dQ_{i-1}
//   -> dqfree, and write P^T, dS^T to shared memory          -> pfull
//   dV += P^T dO_i, dK += dS^T Q_i (A K-major from shared memory), dQ_i = dS K (A =
//   dS^T read MN-major)                                      -> ofull
//   dQ rows: each warp stages its 32x32 fp32 dQ box in shared memory and adds it to
//   an fp32 accumulator with one TMA reduce-add
// dQ of a query block collects the contributions of up to six key blocks; the
// accumulator is zeroed before the launch and converted to bf16 afterwards.
#pragma once
#include "tc_attention.cuh"

namespace tao {
namespace tb {

constexpr int kBN = 128;                 // keys per CTA
constexpr int kBQ = 128;                 // queries per block
constexpr int kD = 64;
constexpr int kTile = 128 * kD * 2;      // 16 KB
constexpr int kThreads = 288;
// K, V, Q[2], dO[2], dS^T (two 16 KB atoms), dQ staging (4 KB per elementwise
// warp), P^T (two 16 KB atoms), lse/rowdot [2][2][128] fp32, barriers
constexpr int kOffK = 0, kOffV = kTile, kOffQ = 2 * kTile, kOffO = 4 * kTile, kOffDS = 6 * kTile;
constexpr int kOffDQ = 8 * kTile;
constexpr int kOffPT = kOffDQ + 8 * 4096;  // P^T: two 64-query tiles like dS^T
constexpr int kOffStat = kOffPT + 2 * kTile;
constexpr int kOffBar = kOffStat + 2 * 2 * 128 * 4;
constexpr int kSmem = kOffBar + 128;
constexpr int kTmemCols = 512;

// Layout by width.  Width 64: the layout above.  Width 128: each CTA computes half of
// the gradient channels (blockIdx.z; S^T and dP^T are full-width contractions, so the
// two halves each form them), K, V, Q[2], dO[2] are full-width tiles of two 64-channel
// atoms, P^T lives in TMEM (columns 448-511, bf16 pairs, the A operand of the dV
// product) instead of shared memory, and each warp stages its dQ box in its own rows
// of the dS^T buffer (free between the block's products and the next dS^T).
template <int D>
struct Cfg {
  static constexpr int TILE = 128 * D * 2;  // K, V, Q, dO tiles
  static constexpr int NA = D / 64;         // 64-channel atoms per tile
  static constexpr bool PT_TMEM = D == 128;
  static constexpr int OFF_K = 0, OFF_V = TILE, OFF_Q = 2 * TILE, OFF_O = 4 * TILE, OFF_DS = 6 * TILE;
  static constexpr int OFF_DQ = PT_TMEM ? OFF_DS : OFF_DS + 2 * kTile;
  static constexpr int OFF_PT = OFF_DQ + 8 * 4096;  // width 64 only
  static constexpr int OFF_STAT = PT_TMEM ? OFF_DS + 2 * kTile : OFF_PT + 2 * kTile;
  static constexpr int OFF_BAR = OFF_STAT + 2 * 2 * 128 * 4;
  static constexpr int SMEM = OFF_BAR + 128;
};
static_assert(Cfg<64>::SMEM == kSmem, "width-64 layout");
static_assert(Cfg<128>::SMEM <= 232448, "width-128 layout exceeds shared memory");

// Bulk tensor reduce-add of a shared-memory box into global memory (TMA).
TAO_DEVI void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map),
      "r"(x), "r"(y), "r"(smem_u32(src))
      : "memory");
}
TAO_DEVI void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
TAO_DEVI void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
TAO_DEVI void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
TAO_DEVI uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&t);
}
// TMEM column of the bf16 pair holding query column `c` (even) of a 128-query
// block: each half of the block is packed into the first half of the fp32
// columns it was read from (0-63 -> 0-31, 64-127 -> 64-95).
TAO_DEVI constexpr uint32_t pair_col(int c) { return c < 64 ? c / 2 : 64 + (c - 64) / 2; }

}  // namespace tb

struct TcBwdArgs {
  const float* lse;     // [B][H][T] natural log
  const float* rowdot;  // [B][H][T]
  bf16* dk;             // [B][T][H][64]
  bf16* dv;
  int T, H;
  int* err;
};

template <int D>
__global__ void __launch_bounds__(tb::kThreads, 1) tc_attention_bwd_kernel(
    const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
    const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
    const __grid_constant__ CUtensorMap tdq, TcBwdArgs a) {
  using namespace tc;
  using namespace tb;
  using C = tb::Cfg<D>;
  constexpr int TILE = C::TILE, NA = C::NA;
  constexpr int kOffK = C::OFF_K, kOffV = C::OFF_V, kOffQ = C::OFF_Q, kOffO = C::OFF_O, kOffDS = C::OFF_DS;
  constexpr int kOffDQ = C::OFF_DQ, kOffPT = C::OFF_PT;
  constexpr float kScale = D == 64 ? 0.125f : 0.08838834764831845f;  // 1 / sqrt(D)
  extern __shared__ __align__(1024) uint8_t sm[];
  if (smem_u32(sm) & 1023u) {
    if (threadIdx.x == 0 && a.err) atomicOr(a.err, kErrState);
    return;
  }
  float* const lseS = reinterpret_cast<float*>(sm + C::OFF_STAT);  // [2][128] lse * log2(e)
  float* const rdS = lseS + 2 * 128;                                // [2][128]
  uint64_t* const bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* const kvbar = bars;
  uint64_t* const qbar = bars + 1;     // [2] Q_i and dO_i
  uint64_t* const statbar = bars + 3;  // [2] lse / rowdot of block i
  uint64_t* const sfull = bars + 5;
  uint64_t* const pfull = bars + 6;
  uint64_t* const ofull = bars + 7;
  uint64_t* const dqfree = bars + 8;
  uint64_t* const sfree = bars + 9;
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(bars + 11);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = a.T, H = a.H;
  const int b = blockIdx.y / H, h = blockIdx.y % H;
  const int k0 = blockIdx.x * kBN;
  int qend = (k0 / kFine + 3) * kFine;  // queries whose window reaches this key block
  if (qend > T) qend = T;
  const int nq = (qend - k0 + kBQ - 1) / kBQ;
  const int half = D == 128 ? (int)blockIdx.z : 0;  // gradient channels 64 half .. + 63
  const int row0 = b * T, col = h * D, ccol = col + 64 * half;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(kvbar, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qbar[i], 1);
      mbar_init(&statbar[i], 32);
    }
    mbar_init(sfull, 1);
    mbar_init(pfull, 256);
    mbar_init(ofull, 1);
    mbar_init(dqfree, 256);
    mbar_init(sfree, 256);
    *abort_flag = 0;
    fence_mbar_init();
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tS = tbase, tDP = tbase + 128, tDV = tbase + 256, tDK = tbase + 320, tDQ = tbase + 384;
  const uint32_t tPT = tbase + 448;  // width 128: P^T (bf16 pairs)
  const float* lse_g = a.lse + ((long long)b * H + h) * T;
  const float* rd_g = a.rowdot + ((long long)b * H + h) * T;

  if (warp == 8) {
    // ================= issuer =================
    const bool leader = lane == 0;
    constexpr uint32_t I_S = idesc_bf16(128, 128, 0, 0);   // K-major A and B
    constexpr uint32_t I_KV = idesc_bf16(128, 64, 0, 1);   // A K-major, B MN-major
    constexpr uint32_t I_Q = idesc_bf16(128, 64, 1, 1);    // A and B MN-major
    int q_armed[2] = {0, 0}, q_done[2] = {0, 0};
    int s_issued = 0, o_issued = 0;
    bool kv_pending = true;
    auto load_q = [&](int i) {
      const int st = i & 1;
      if (leader) {
        mbar_expect_tx(&qbar[st], 2 * TILE);
#pragma unroll
        for (int at = 0; at < NA; ++at) {
          tma_2d(sm + kOffQ + st * TILE + at * kTile, &tq, col + 64 * at, row0 + k0 + i * kBQ, &qbar[st]);
          tma_2d(sm + kOffO + st * TILE + at * kTile, &tdo, col + 64 * at, row0 + k0 + i * kBQ, &qbar[st]);
        }
      }
      ++q_armed[st];
    };
    // lse (scaled to log2) and rowdot of query block i: fetched into registers
    // early, published into stat buffer i&1 once that buffer is free
    float pl[4], pr[4];
    auto fetch_stats = [&](int i) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int q = k0 + i * kBQ + lane * 4 + u;
        pl[u] = q < T ? lse_g[q] * 1.4426950408889634f : 0.f;
        pr[u] = q < T ? rd_g[q] : 0.f;
      }
    };
    auto publish_stats = [&](int i) {
      const int st = i & 1;
      *reinterpret_cast<float4*>(lseS + st * 128 + lane * 4) = make_float4(pl[0], pl[1], pl[2], pl[3]);
      *reinterpret_cast<float4*>(rdS + st * 128 + lane * 4) = make_float4(pr[0], pr[1], pr[2], pr[3]);
      mbar_arrive(&statbar[st]);
    };
    if (leader) {
      mbar_expect_tx(kvbar, 2 * TILE);
#pragma unroll
      for (int at = 0; at < NA; ++at) {
        tma_2d(sm + kOffK + at * kTile, &tk, col + 64 * at, row0 + k0, kvbar);
        tma_2d(sm + kOffV + at * kTile, &tv, col + 64 * at, row0 + k0, kvbar);
      }
    }
    for (int i = 0; i < 2 && i < nq; ++i) load_q(i);
    fetch_stats(0);
    publish_stats(0);
    if (nq > 1) fetch_stats(1);
    bool fine = warp_wait(kvbar, 0, a.err, abort_flag);
    if (fine) kv_pending = false;
    const uint32_t aK = smem_u32(sm + kOffK), aV = smem_u32(sm + kOffV), aDS = smem_u32(sm + kOffDS);
    const uint32_t aPT = smem_u32(sm + kOffPT);
    // S^T, dP^T of block i (its Q and dO stage must have landed)
    auto issue_s = [&](int i) -> bool {
      const int st = i & 1;
      if (!warp_wait(&qbar[st], q_done[st] & 1, a.err, abort_flag)) return false;
      ++q_done[st];
      fence_after();
      const uint32_t aQ = smem_u32(sm + kOffQ + st * TILE), aO = smem_u32(sm + kOffO + st * TILE);
      if (leader) {  // full-width contractions: 64-channel atoms 16 KB apart, 4 K-steps each
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          mma(tS, sdesc(aK + (k >> 2) * kTile + (k & 3) * 32, 16, 1024),
              sdesc(aQ + (k >> 2) * kTile + (k & 3) * 32, 16, 1024), I_S, k > 0);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          mma(tDP, sdesc(aV + (k >> 2) * kTile + (k & 3) * 32, 16, 1024),
              sdesc(aO + (k >> 2) * kTile + (k & 3) * 32, 16, 1024), I_S, k > 0);
        commit(sfull);
      }
      __syncwarp();
      ++s_issued;
      return true;
    };
    if (fine) fine = issue_s(0);
    for (int i = 0; fine && i < nq; ++i) {
      const int st = i & 1;
      // S^T(i), dP^T(i) loaded by the elementwise warps: their columns are free
      if (!(fine = warp_wait(sfree, i & 1, a.err, abort_flag))) break;
      if (i + 1 < nq) {
        publish_stats(i + 1);  // stat buffer (i+1)&1 was last read by block i-1
        if (i + 2 < nq) fetch_stats(i + 2);
        if (!(fine = issue_s(i + 1))) break;
      }
      // P^T(i), dS^T(i) in shared memory; dQ columns read out (block i-1)
      if (!(fine = warp_wait(pfull, i & 1, a.err, abort_flag))) break;
      if (i > 0 && !(fine = warp_wait(dqfree, (i - 1) & 1, a.err, abort_flag))) break;
      fence_after();
      // this CTA's gradient channels: the `half` atom of Q, dO and K
      const uint32_t aQ = smem_u32(sm + kOffQ + st * TILE) + half * kTile;
      const uint32_t aO = smem_u32(sm + kOffO + st * TILE) + half * kTile;
      const uint32_t aKh = aK + half * kTile;
      if (leader) {
#pragma unroll
        for (int k = 0; k < kBQ / 16; ++k) {  // A = P^T (keys x queries), 16 queries per step
          if constexpr (C::PT_TMEM)
            mma_ts(tDV, tPT + k * 8, sdesc(aO + k * 2048, 8192, 1024), I_KV, (i > 0 || k > 0) ? 1u : 0u);
          else
            mma(tDV, sdesc(aPT + (k >> 2) * kTile + (k & 3) * 32, 16, 1024), sdesc(aO + k * 2048, 8192, 1024),
                I_KV, (i > 0 || k > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int k = 0; k < kBQ / 16; ++k)
          mma(tDK, sdesc(aDS + (k >> 2) * kTile + (k & 3) * 32, 16, 1024), sdesc(aQ + k * 2048, 8192, 1024),
              I_KV, (i > 0 || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k)
          mma(tDQ, sdesc(aDS + k * 2048, kTile, 1024), sdesc(aKh + k * 2048, 8192, 1024), I_Q, k > 0);
        commit(ofull);
      }
      __syncwarp();
      ++o_issued;
      // stage i&1 is free once block i's products are done: refill it with block i+2
      if (i + 2 < nq) {
        if (!(fine = warp_wait(ofull, i & 1, a.err, abort_flag))) break;
        load_q(i + 2);
      }
    }
    if (!fine) {
      // drain (bounded): copies and MMAs of this CTA still in flight
      *abort_flag = 1;
      if (kv_pending) mbar_wait(kvbar, 0, nullptr);
      for (int st = 0; st < 2; ++st)
        if (q_armed[st] > q_done[st]) mbar_wait(&qbar[st], q_done[st] & 1, nullptr);
      if (s_issued) mbar_wait(sfull, (s_issued - 1) & 1, nullptr);
      if (o_issued) mbar_wait(ofull, (o_issued - 1) & 1, nullptr);
    }
    __syncwarp();
  } else {
    // ================= elementwise =================
    const int qd = warp & 3, ch = warp >> 2;
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const int kr = qd * 32 + lane;  // key row of this thread
    const int key = k0 + kr;
    const float sl = 1.4426950408889634f * kScale;  // log2(e) / sqrt(D)
    uint8_t* const dsrow = sm + kOffDS + ch * kTile + kr * 128;
    uint8_t* const ptrow = sm + kOffPT + ch * kTile + kr * 128;
    uint8_t* const stage = sm + kOffDQ + warp * 4096;
    // dQ rows of block j (its products complete) -> fp32 accumulator
    auto dq_out = [&](int j) {
      const int qj = k0 + j * kBQ;
      float v[32];
      tmem_ld32(tDQ + lane_off + ch * 32, v);
      fence_before();
      mbar_arrive(dqfree);  // the dQ columns are free once read
      // stage rows (query qj + 32qd + lane, channels 32ch..+31) as a 128B-swizzled
      // 32x32 fp32 box; rows past T hold exact zeros (their P and dS are zero)
      if (lane == 0) bulk_wait_read0();  // the previous box has been read out
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<float4*>(stage + lane * 128 + ((c ^ (lane & 7)) << 4)) =
            make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_2d(&tdq, stage, ccol + ch * 32, row0 + qj + qd * 32);
        bulk_commit();
        // width 128: the box sits in this warp's dS^T rows, written next
        if constexpr (C::PT_TMEM) bulk_wait_read0();
      }
      if constexpr (C::PT_TMEM) __syncwarp();
    };
    bool ok = true;
    for (int i = 0; i < nq; ++i) {
      const int q0 = k0 + i * kBQ;
      const int sb = i & 1;
      if (!(ok = warp_wait(&statbar[sb], (i >> 1) & 1, a.err, abort_flag))) break;
      if (!(ok = warp_wait(sfull, i & 1, a.err, abort_flag))) break;
      fence_after();
      // this thread's 64 columns of S^T and dP^T, then the columns are released
      float s[64], dp[64];
      tmem_ld32(tS + lane_off + ch * 64, s);
      tmem_ld32(tS + lane_off + ch * 64 + 32, s + 32);
      tmem_ld32(tDP + lane_off + ch * 64, dp);
      tmem_ld32(tDP + lane_off + ch * 64 + 32, dp + 32);
      fence_before();
      mbar_arrive(sfree);
      const bool masked = (i == 0) || (q0 + kBQ > T);
      uint32_t pp[32], dd[32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int c0 = ch * 64 + c * 32;  // first query column of this chunk
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          // lse / rowdot of four query columns: one broadcast vector load each
          const float4 l4 = *reinterpret_cast<const float4*>(lseS + sb * 128 + c0 + e);
          const float4 r4 = *reinterpret_cast<const float4*>(rdS + sb * 128 + c0 + e);
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, rv[4] = {r4.x, r4.y, r4.z, r4.w};
          float pv[4], dv[4];
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            float p = ex2(fmaf(s[c * 32 + e + x], sl, -lv[x]));
            if (masked) {
              const int q = q0 + c0 + e + x;
              if (key > q || q >= T) p = 0.f;
            }
            pv[x] = p;
            dv[x] = p * (dp[c * 32 + e + x] - rv[x]);
          }
          pp[c * 16 + e / 2] = pack2(pv[0], pv[1]);
          pp[c * 16 + e / 2 + 1] = pack2(pv[2], pv[3]);
          dd[c * 16 + e / 2] = pack2(dv[0], dv[1]);
          dd[c * 16 + e / 2 + 1] = pack2(dv[2], dv[3]);
        }
      }
      // block i-1's products are done: its dQ is read out and the P^T / dS^T
      // buffers may be overwritten
      if (i > 0) {
        if (!(ok = warp_wait(ofull, (i - 1) & 1, a.err, abort_flag))) break;
        fence_after();
        dq_out(i - 1);
      }
      // P^T and dS^T rows (queries contiguous, 128B swizzle by key row), for the
      // dV / dK products (K-major A) and the dQ product (dS^T read MN-major)
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int chunk = (c * 4 + u) ^ (kr & 7);
          const int o = c * 16 + 4 * u;
          *reinterpret_cast<uint4*>(dsrow + chunk * 16) = make_uint4(dd[o], dd[o + 1], dd[o + 2], dd[o + 3]);
          if constexpr (!C::PT_TMEM)
            *reinterpret_cast<uint4*>(ptrow + chunk * 16) = make_uint4(pp[o], pp[o + 1], pp[o + 2], pp[o + 3]);
        }
      if constexpr (C::PT_TMEM) {
        tmem_st32u(tPT + lane_off + ch * 32, pp);  // this thread's 64 query columns as 32 pairs
        fence_before();
      }
      fence_proxy_async();
      mbar_arrive(pfull);
    }
    if (ok && nq > 0) {  // the last block's dQ
      if ((ok = warp_wait(ofull, (nq - 1) & 1, a.err, abort_flag))) {
        fence_after();
        dq_out(nq - 1);
      }
    }
    if (lane == 0) bulk_wait0();  // dQ reductions complete before the CTA ends
    __syncwarp();
    if (ok) {
      // dV, dK rows of this CTA's keys (all query blocks accumulated)
      float dvv[32], dkk[32];
      tmem_ld32(tDV + lane_off + ch * 32, dvv);
      tmem_ld32(tDK + lane_off + ch * 32, dkk);
      if (key < T) {
        const long long off = ((long long)(row0 + key) * H + h) * D + 64 * half + ch * 32;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 pv, pk;
          pv.x = pack2(dvv[8 * u], dvv[8 * u + 1]);
          pv.y = pack2(dvv[8 * u + 2], dvv[8 * u + 3]);
          pv.z = pack2(dvv[8 * u + 4], dvv[8 * u + 5]);
          pv.w = pack2(dvv[8 * u + 6], dvv[8 * u + 7]);
          pk.x = pack2(dkk[8 * u] * kScale, dkk[8 * u + 1] * kScale);
          pk.y = pack2(dkk[8 * u + 2] * kScale, dkk[8 * u + 3] * kScale);
          pk.z = pack2(dkk[8 * u + 4] * kScale, dkk[8 * u + 5] * kScale);
          pk.w = pack2(dkk[8 * u + 6] * kScale, dkk[8 * u + 7] * kScale);
          *reinterpret_cast<uint4*>(a.dv + off + 8 * u) = pv;
          *reinterpret_cast<uint4*>(a.dk + off + 8 * u) = pk;
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTmemCols));
  }
}

// dq = bf16(dq_acc * scale) (scale = 1 / sqrt(D)), eight elements per thread.
__global__ void dq_convert_kernel(const float* __restrict__ acc, bf16* __restrict__ dq, long long n8, float scale) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const float4 x = reinterpret_cast<const float4*>(acc)[2 * i];
  const float4 y = reinterpret_cast<const float4*>(acc)[2 * i + 1];
  uint4 o;
  o.x = tb::pack2(x.x * scale, x.y * scale);
  o.y = tb::pack2(x.z * scale, x.w * scale);
  o.z = tb::pack2(y.x * scale, y.y * scale);
  o.w = tb::pack2(y.z * scale, y.w * scale);
  reinterpret_cast<uint4*>(dq)[i] = o;
}

}  // namespace tao
