// Windowed causal attention forward on the 5th-generation tensor cores (sm_100a).
//
// Same semantics as window_attention_kernel (tao_stream.py:760-787 through
// flash_attention.py:16-37): query t of [B][T][H][D] bf16 operands (D = 64 or 128)
// reads keys [max(0, 256*floor(t/256) - 512), t] with scale 1/sqrt(D).
//
// One CTA (one warpgroup, 128 threads) owns 128 queries of one (batch, head):
//   * Q, K and V tiles arrive by TMA (cp.async.bulk.tensor, 128B swizzle) into
//     1024-byte-aligned shared memory; K and V have two stages each
//   * S = Q K^T: tcgen05.mma kind::f16, M=128 N=128 K=D, fp32 accumulator in TMEM
//   * each thread owns one query row: tcgen05.ld of its S row, window mask,
//     online softmax in registers, P (bf16 pairs) written back to TMEM with
//     tcgen05.st (shared memory bandwidth is left to the MMA operands)
//   * O += P V: tcgen05.mma M=128 N=D K=128, A = P read from TMEM, V an MN-major
//     shared-memory operand; O
//     stays in TMEM for the whole CTA and is rescaled there only when a row
//     maximum grows by more than 2^8 (p = 2^(s - stale max) stays <= 256)
//   * S of the next key block is computed while the softmax of this one runs
// Every mbarrier wait is bounded; on a timeout the CTA records the error, frees
// its TMEM and returns.
#pragma once
#include <cuda.h>

#include "../../include/tao_b200.h"
#include "common.cuh"
#include "tcgen05.cuh"

namespace tao {
namespace tc {

constexpr int kTcBM = 128, kTcBN = 128, kTcD = 64;
constexpr int kTcAtom = kTcBM * 64 * 2;    // 16 KB: 128 rows x 128 B (64 channels)
constexpr int kTcTile = kTcBM * kTcD * 2;  // one operand tile at width 64
constexpr int kTcThreads = 160;            // warps 0-3: softmax rows, warp 4: TMA + MMA issue
// Per width: Q, K[2], V[2] tiles of D/64 atoms each, then 9 mbarriers, the TMEM
// address slot and the abort flag; TMEM columns S fp32 0-127, O fp32 128..128+D-1,
// P bf16 pairs after O (width 64: 256 columns, two CTAs per SM; width 128: 320 of a
// 512-column allocation, one CTA per SM).
template <int D>
struct TcAttnCfg {
  static constexpr int TILE = kTcBM * D * 2;
  static constexpr int SMEM = 5 * TILE + 128;
  static constexpr int TMEM_COLS = D == 64 ? 256 : 512;
  static constexpr int CTAS = D == 64 ? 2 : 1;
};
constexpr int kTcSmem = TcAttnCfg<64>::SMEM;
constexpr int kTcTmemCols = 256;
// O is rescaled only when a row maximum grows by more than this (log2 units):
// until then scores are exponentiated against the stale maximum (p <= 2^8).
constexpr float kTcRescale = 8.f;

// Streaming prefill form (RING): the chunk's queries q [B][w][H][D] at positions
// states[b]->position + i read the state's ring of keys and values ([H][768][D], row =
// position % 768), written for the chunk before the launch; the output goes to
// [B][w][H][D].  A 128-key block of a window is 128 consecutive ring rows (windows
// start at multiples of 256), so its tiles are loaded by cp.async into the same
// 128B-swizzled layout a TMA box has, 16 bytes per lane, each lane arriving on the
// tile's mbarrier when its copies land.
struct TcRing {
  TaoState* const* states;
  const bf16* q;
  int w;
};

// Byte offset of channel chunk c (8 bf16) of tile row r in a 128B-swizzled tile of
// 64-channel atoms: the layout of a TMA box of 64 columns x 128 rows per atom.
TAO_DEVI uint32_t sw128_off(int r, int c) {
  return (uint32_t)((c >> 3) * kTcAtom + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}
// One lane's share of a 128-row tile: rows[r * D .. + D) -> dst (rows >= nrows zero),
// then an arrival on `bar` once this lane's copies have landed.
template <int D>
TAO_DEVI void cp_tile(uint8_t* dst, const bf16* rows, long long row_stride, int nrows, uint64_t* bar, int lane) {
  constexpr int CH = D / 8;
  for (int idx = lane; idx < kTcBM * CH; idx += 32) {
    const int r = idx / CH, c = idx % CH;
    const bool ok = r < nrows;
    const bf16* src = rows + (long long)(ok ? r : 0) * row_stride + c * 8;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst + sw128_off(r, c))), "l"(src),
                 "r"(ok ? 16 : 0)
                 : "memory");
  }
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait that also gives up as soon as another thread of the CTA raised
// the abort flag (so one timeout ends every wait of the CTA promptly).
TAO_DEVI bool wait_or_abort(uint64_t* bar, uint32_t phase, int* err, volatile int* abort) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (mbar_try_wait(bar, phase)) return true;
    if ((i & 31u) == 31u && *abort) return false;
  }
  *abort = 1;
  if (err) atomicOr(err, kErrWaitTimeout);
  return false;
}
// Warp-uniform outcome of wait_or_abort (tcgen05.ld/st need the whole warp).
TAO_DEVI bool warp_wait(uint64_t* bar, uint32_t phase, int* err, volatile int* abort) {
  return __all_sync(0xffffffffu, wait_or_abort(bar, phase, err, abort));
}

}  // namespace tc


// Roles and hand-offs of one CTA (all by mbarrier; no CTA-wide barrier in the loop):
//   issuer (warp 4, one lane): TMA copies of Q, K(j), V(j); S(j) = Q K(j)^T into
//     TMEM -> sfull; O += P(j) V(j) -> ofull.  K stage j&1 is refilled with K(j+2)
//     once the softmax warps have read S(j) (sfree); V stage (j+1)&1 with V(j+1)
//     once O(j-1) is complete.
//   softmax (warps 0-3, one query row per thread): sfull(j) -> tcgen05.ld S row ->
//     sfree -> mask, row max -> ofull(j-1) -> rescale the O row in TMEM if its
//     maximum moved by more than 2^8 -> P(j) (bf16 pairs) to TMEM -> pfull.
//
// RING: the streaming prefill form (see TcRing); the tensor maps are unused, lse is
// not written and T is ignored.
template <int D, bool RING = false>
__global__ void __launch_bounds__(tc::kTcThreads, tc::TcAttnCfg<D>::CTAS) tc_window_attention_kernel(
    const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
    const __grid_constant__ CUtensorMap tv, bf16* __restrict__ out, float* __restrict__ lse, int T,
    int H, int* err, tc::TcRing ring) {
  using namespace tc;
  constexpr int TILE = TcAttnCfg<D>::TILE, NA = D / 64;
  // 128B-swizzled tiles need 1024-byte alignment; the kernel uses no static
  // shared memory, so the dynamic window starts aligned (checked, never assumed).
  extern __shared__ __align__(1024) uint8_t sm[];
  if (smem_u32(sm) & 1023u) {
    if (threadIdx.x == 0 && err) atomicOr(err, kErrState);
    return;
  }
  uint8_t* const sQ = sm;
  uint8_t* const sK = sm + TILE;      // [2] stages
  uint8_t* const sV = sm + 3 * TILE;  // [2] stages
  uint64_t* const bars = reinterpret_cast<uint64_t*>(sm + 5 * TILE);
  uint64_t* const qbar = bars;
  uint64_t* const kfull = bars + 1;  // [2]
  uint64_t* const vfull = bars + 3;  // [2]
  uint64_t* const sfull = bars + 5;
  uint64_t* const sfree = bars + 6;
  uint64_t* const pfull = bars + 7;
  uint64_t* const ofull = bars + 8;
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(bars + 10);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.y / H, h = blockIdx.y % H;
  const int q0 = blockIdx.x * kTcBM;  // the 128 queries share one 256-token tile
  // absolute position of query row 0, rows that exist, the bound on key positions
  long long qa0 = q0, tlimit = T;
  int nrow = T - q0;
  const bf16* kring = nullptr;
  const bf16* vring = nullptr;
  if constexpr (RING) {
    const TaoState& st = *ring.states[b];
    qa0 = st.position + q0;
    nrow = ring.w - q0;
    tlimit = 0x7fffffffffffffffll;
    kring = reinterpret_cast<const bf16*>(st.k_ring) + (long long)h * kWindow * D;
    vring = reinterpret_cast<const bf16*>(st.v_ring) + (long long)h * kWindow * D;
  }
  long long kstart = (qa0 / kFine) * kFine - kKeep;
  if (kstart < 0) kstart = 0;
  const long long kend = min(qa0 + kTcBM, qa0 + nrow);
  const int nblk = (int)((kend - kstart + kTcBN - 1) / kTcBN);
  const int row0 = b * T;
  const int col = h * D;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TcAttnCfg<D>::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    constexpr int LOADERS = RING ? 32 : 1;  // cp.async: every issuer lane arrives
    mbar_init(qbar, LOADERS);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kfull[i], LOADERS);
      mbar_init(&vfull[i], LOADERS);
    }
    mbar_init(sfull, 1);
    mbar_init(sfree, kTcBM);
    mbar_init(pfull, kTcBM);
    mbar_init(ofull, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tS = tbase, tO = tbase + 128, tP = tbase + 128 + D;

  if (warp == 4) {
    // ================= issuer (the whole warp walks the schedule; lane 0 issues) =====
    constexpr uint32_t IS = idesc_bf16(128, 128, 0, 0), IO = idesc_bf16(128, D, 0, 1);
    const bool leader = lane == 0;
    int k_armed[2] = {0, 0}, k_done[2] = {0, 0}, v_armed[2] = {0, 0}, v_done[2] = {0, 0};
    int s_issued = 0, o_issued = 0;
    auto load_k = [&](int j) {
      const int st = j & 1;
      if constexpr (RING) {
        cp_tile<D>(sK + st * TILE, kring + ((kstart + (long long)j * kTcBN) % kWindow) * D, D, kTcBN, &kfull[st],
                   lane);
      } else if (leader) {
        mbar_expect_tx(&kfull[st], TILE);
#pragma unroll
        for (int at = 0; at < NA; ++at)
          tma_2d(sK + st * TILE + at * kTcAtom, &tk, col + 64 * at, row0 + kstart + j * kTcBN, &kfull[st]);
      }
      ++k_armed[st];
    };
    auto load_v = [&](int j) {
      const int st = j & 1;
      if constexpr (RING) {
        cp_tile<D>(sV + st * TILE, vring + ((kstart + (long long)j * kTcBN) % kWindow) * D, D, kTcBN, &vfull[st],
                   lane);
      } else if (leader) {
        mbar_expect_tx(&vfull[st], TILE);
#pragma unroll
        for (int at = 0; at < NA; ++at)
          tma_2d(sV + st * TILE + at * kTcAtom, &tv, col + 64 * at, row0 + kstart + j * kTcBN, &vfull[st]);
      }
      ++v_armed[st];
    };
    auto issue_s = [&](int j) -> bool {
      const int st = j & 1;
      if (!warp_wait(&kfull[st], k_done[st] & 1, err, abort_flag)) return false;
      ++k_done[st];
      if constexpr (RING) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // cp.async -> MMA
      fence_after();
      if (leader) {
        const uint32_t kaddr = smem_u32(sK + st * TILE), qaddr = smem_u32(sQ);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)   // 64-channel atoms of 16 KB, 4 K-steps each
          mma(tS, sdesc(qaddr + (k >> 2) * kTcAtom + (k & 3) * 32, 16, 1024),
              sdesc(kaddr + (k >> 2) * kTcAtom + (k & 3) * 32, 16, 1024), IS, k > 0);
        commit(sfull);
      }
      __syncwarp();
      ++s_issued;
      return true;
    };
    if constexpr (RING) {
      cp_tile<D>(sQ, ring.q + (((long long)b * ring.w + q0) * H + h) * D, (long long)H * D, min(nrow, kTcBM), qbar,
                 lane);
    } else if (leader) {
      mbar_expect_tx(qbar, TILE);
#pragma unroll
      for (int at = 0; at < NA; ++at) tma_2d(sQ + at * kTcAtom, &tq, col + 64 * at, row0 + q0, qbar);
    }
    for (int j = 0; j < 2 && j < nblk; ++j) {
      load_k(j);
      load_v(j);
    }
    bool fine = warp_wait(qbar, 0, err, abort_flag);
    if constexpr (RING) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // cp.async -> MMA
    fine = fine && issue_s(0);
    for (int j = 0; fine && j < nblk; ++j) {
      // S(j) has been read: the S columns and K stage j&1 are free
      if (!(fine = warp_wait(sfree, j & 1, err, abort_flag))) break;
      fence_after();
      if (j + 2 < nblk) load_k(j + 2);
      if (j + 1 < nblk && !(fine = issue_s(j + 1))) break;
      // O(j-1) complete: V stage (j+1)&1 is free
      if (j >= 1 && j + 1 < nblk) {
        if (!(fine = warp_wait(ofull, (j - 1) & 1, err, abort_flag))) break;
        load_v(j + 1);
      }
      // P(j) written (and the O rows rescaled): O += P(j) V(j)
      if (!(fine = warp_wait(pfull, j & 1, err, abort_flag))) break;
      const int st = j & 1;
      if (!(fine = warp_wait(&vfull[st], v_done[st] & 1, err, abort_flag))) break;
      ++v_done[st];
      if constexpr (RING) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // cp.async -> MMA
      fence_after();
      if (leader) {
        const uint32_t vaddr = smem_u32(sV + st * TILE);
#pragma unroll
        for (int k = 0; k < kTcBN / 16; ++k)  // A = P(j) from TMEM, 16 keys = 8 columns per step;
          // V MN-major: 64-channel atoms 16 KB apart (LBO)
          mma_ts(tO, tP + k * 8, sdesc(vaddr + k * 2048, kTcAtom, 1024), IO, (j > 0 || k > 0) ? 1u : 0u);
        commit(ofull);
      }
      __syncwarp();
      ++o_issued;
    }
    if (!fine) {
      // drain (bounded): copies and MMAs of this CTA still in flight
      *abort_flag = 1;
      mbar_wait(qbar, 0, nullptr);
      for (int st = 0; st < 2; ++st) {
        if (k_armed[st] > k_done[st]) mbar_wait(&kfull[st], k_done[st] & 1, nullptr);
        if (v_armed[st] > v_done[st]) mbar_wait(&vfull[st], v_done[st] & 1, nullptr);
      }
      if (s_issued) mbar_wait(sfull, (s_issued - 1) & 1, nullptr);
      if (o_issued) mbar_wait(ofull, (o_issued - 1) & 1, nullptr);
    }
    __syncwarp();
  } else {
    // ================= softmax rows =================
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const long long qpos = qa0 + tid;
    const float sl = 1.4426950408889634f / sqrtf((float)D);  // log2(e) / sqrt(D)
    float mu = -INFINITY;  // exponent base of P and O (scaled log2 units)
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      if (!(ok = warp_wait(sfull, j & 1, err, abort_flag))) break;
      fence_after();
      float sc[kTcBN];
#pragma unroll
      for (int c = 0; c < kTcBN / 32; ++c) tmem_ld32(tS + lane_off + c * 32, sc + c * 32);
      fence_before();
      mbar_arrive(sfree);
      const long long kb0 = kstart + (long long)j * kTcBN;
      if (kb0 + kTcBN - 1 > qa0 || kb0 + kTcBN > tlimit) {  // block reaches the diagonal or the end
#pragma unroll
        for (int c = 0; c < kTcBN; ++c) {
          const long long kp = kb0 + c;
          if (kp > qpos || kp >= tlimit) sc[c] = -INFINITY;
        }
      }
      float m4[4];  // four independent chains, then a tree
#pragma unroll
      for (int c = 0; c < 4; ++c) m4[c] = sc[c];
#pragma unroll
      for (int c = 4; c < kTcBN; ++c) m4[c & 3] = fmaxf(m4[c & 3], sc[c]);
      const float mnew = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * sl;
      float alpha = 1.f;
      const bool rescale = mnew > mu + kTcRescale;  // false for fully masked rows
      if (rescale) {
        alpha = ex2(mu - mnew);  // 0 when mu = -inf
        mu = mnew;
      }
      const float nb = (mu == -INFINITY) ? 0.f : -mu;
      // O(j-1) complete: the P buffer is free and the O row may be rescaled
      if (j > 0) {
        if (!(ok = warp_wait(ofull, (j - 1) & 1, err, abort_flag))) break;
        fence_after();
      }
      float r4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float pk[32];  // 64 keys as 32 bf16 pairs (bit patterns), low half = lower key
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float p0 = ex2(fmaf(sc[half * 64 + 2 * e], sl, nb));
          const float p1 = ex2(fmaf(sc[half * 64 + 2 * e + 1], sl, nb));
          r4[e & 3] += p0 + p1;
          __nv_bfloat162 t2 = __floats2bfloat162_rn(p0, p1);
          pk[e] = __uint_as_float(*reinterpret_cast<uint32_t*>(&t2));
        }
        tmem_st32(tP + lane_off + half * 32, pk);
      }
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {  // after the exponentials: sc[] is dead
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float ov[32];
          tmem_ld32(tO + lane_off + c * 32, ov);
#pragma unroll
          for (int d = 0; d < 32; ++d) ov[d] *= alpha;
          tmem_st32(tO + lane_off + c * 32, ov);
        }
      }
      l = l * alpha + ((r4[0] + r4[1]) + (r4[2] + r4[3]));
      fence_before();
      mbar_arrive(pfull);
    }
    // ---- epilogue: O complete -> normalise -> bf16 rows; lse in natural log
    if (ok && warp_wait(ofull, (nblk - 1) & 1, err, abort_flag)) {
      fence_after();
      float ov[D];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) tmem_ld32(tO + lane_off + c * 32, ov + c * 32);
      if (tid < nrow) {
        const float inv = 1.f / l;
        bf16* orow = RING ? out + (((long long)b * ring.w + q0 + tid) * H + h) * D
                          : out + ((long long)(row0 + qpos) * H + h) * D;
#pragma unroll
        for (int c8 = 0; c8 < D / 8; ++c8) {
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 t2 =
                __floats2bfloat162_rn(ov[c8 * 8 + 2 * e] * inv, ov[c8 * 8 + 2 * e + 1] * inv);
            pk[e] = *reinterpret_cast<uint32_t*>(&t2);
          }
          *reinterpret_cast<uint4*>(orow + c8 * 8) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
        if (!RING && lse) lse[((long long)b * H + h) * T + qpos] = (mu + log2f(l)) * 0.6931471805599453f;
      }
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(TcAttnCfg<D>::TMEM_COLS));
  }
}

}  // namespace tao
