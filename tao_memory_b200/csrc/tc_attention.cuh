// Windowed causal attention forward on the 5th-generation tensor cores (sm_100a).
//
// Same semantics as window_attention_kernel (tao_stream.py:760-787 through
// flash_attention.py:16-37): query t of [B][T][H][64] bf16 operands reads keys
// [max(0, 256*floor(t/256) - 512), t] with scale 1/8.
//
// One CTA (one warpgroup, 128 threads) owns 128 queries of one (batch, head):
//   * Q, K and V tiles arrive by TMA (cp.async.bulk.tensor, 128B swizzle) into
//     1024-byte-aligned shared memory; K/V are double-buffered per 128-key block
//   * S = Q K^T: tcgen05.mma kind::f16, M=128 N=128 K=64, fp32 accumulator in TMEM
//   * each thread owns one query row: tcgen05.ld of its S row, scale + window mask,
//     online softmax in registers, P (bf16) written to shared memory in the
//     K-major swizzled layout the tensor core reads
//   * O_blk = P V: tcgen05.mma M=128 N=64 K=128 with V as an MN-major operand,
//     read back and accumulated in registers with the softmax rescale
// Every mbarrier wait is bounded; on a timeout the CTA records the error, frees
// its TMEM and returns.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace tao {
namespace tc {

// Shared-memory matrix descriptor, 128B swizzle (SM100 layout type 2, version 1).
TAO_DEVI uint64_t sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// Instruction descriptor, kind::f16: bf16 x bf16 -> fp32.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn_major << 15) |
         ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
TAO_DEVI void mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}
TAO_DEVI void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
TAO_DEVI void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
TAO_DEVI void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
TAO_DEVI void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
TAO_DEVI void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

TAO_DEVI void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// CTA-wide bounded wait: thread 0 polls (bounded), the verdict is broadcast by
// the barrier, and every thread then observes the completed phase itself (one
// poll succeeds at once) so the copied bytes are visible to it.
TAO_DEVI bool wait_all(uint64_t* bar, uint32_t phase, int* err) {
  int got = 1;
  if (threadIdx.x == 0) got = mbar_wait(bar, phase, err) ? 1 : 0;
  if (!__syncthreads_and(got)) return false;
  return mbar_wait(bar, phase, err);
}

constexpr int kTcBM = 128, kTcBN = 128, kTcD = 64;
constexpr int kTcTile = kTcBM * kTcD * 2;  // 16 KB: 128 rows x 128 B
// Q, K[2], V[2], P[2] tiles, then 5 mbarriers and the TMEM address slot.
constexpr int kTcSmem = 7 * kTcTile + 64;
constexpr int kTcTmemCols = 256;           // S: columns 0-127, O block: 128-191

}  // namespace tc

__global__ void __launch_bounds__(128) tc_window_attention_kernel(
    const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
    const __grid_constant__ CUtensorMap tv, bf16* __restrict__ out, float* __restrict__ lse, int T,
    int H, int* err) {
  using namespace tc;
  // 128B-swizzled tiles need 1024-byte alignment; the kernel uses no static
  // shared memory, so the dynamic window starts aligned (checked, never assumed).
  extern __shared__ __align__(1024) uint8_t sm[];
  if (smem_u32(sm) & 1023u) {
    if (threadIdx.x == 0 && err) atomicOr(err, kErrState);
    return;
  }
  uint8_t* sQ = sm;
  uint8_t* sK[2] = {sm + kTcTile, sm + 2 * kTcTile};
  uint8_t* sV[2] = {sm + 3 * kTcTile, sm + 4 * kTcTile};
  uint8_t* sP = sm + 5 * kTcTile;  // two K-major tiles: keys 0-63 and 64-127
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + 7 * kTcTile);
  uint64_t* qbar = bars;
  uint64_t* kvbar = bars + 1;  // [2]
  uint64_t* sbar = bars + 3;
  uint64_t* obar = bars + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int b = blockIdx.y / H, h = blockIdx.y % H;
  const int q0 = blockIdx.x * kTcBM;  // the 128 queries share one 256-token tile
  int kstart = (q0 / kFine) * kFine - kKeep;
  if (kstart < 0) kstart = 0;
  const int kend = min(q0 + kTcBM, T);
  const int nblk = (kend - kstart + kTcBN - 1) / kTcBN;
  const int row0 = b * T;
  const int col = h * kTcD;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTcTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(bars + i, 1);
    fence_mbar_init();
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tS = tbase, tO = tbase + 128;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;

  // Outstanding-completion bookkeeping (uniform across the CTA) for the drain.
  int kv_armed[2] = {0, 0}, kv_done[2] = {0, 0}, s_done = 0, o_done = 0;
  bool s_pending = false, o_pending = false;
  if (tid == 0) {
    mbar_expect_tx(qbar, kTcTile);
    tma_2d(sQ, &tq, col, row0 + q0, qbar);
  }
  for (int j = 0; j < 2 && j < nblk; ++j) {
    if (tid == 0) {
      mbar_expect_tx(&kvbar[j], 2 * kTcTile);
      tma_2d(sK[j], &tk, col, row0 + kstart + j * kTcBN, &kvbar[j]);
      tma_2d(sV[j], &tv, col, row0 + kstart + j * kTcBN, &kvbar[j]);
    }
    kv_armed[j] = 1;
  }
  const int qpos = q0 + tid;
  float o[kTcD];
#pragma unroll
  for (int d = 0; d < kTcD; ++d) o[d] = 0.f;
  float m = -INFINITY, l = 0.f;
  const float sl = 1.4426950408889634f * 0.125f;  // log2(e) / sqrt(64)
  constexpr uint32_t IS = idesc_bf16(128, 128, 0, 0), IO = idesc_bf16(128, 64, 0, 1);
  bool ok = wait_all(qbar, 0, err);
  for (int j = 0; ok && j < nblk; ++j) {
    const int s = j & 1;
    ok = wait_all(&kvbar[s], kv_done[s] & 1, err);
    if (!ok) break;
    ++kv_done[s];
    // ---- S = Q K^T (M=128 queries, N=128 keys, K=64 channels)
    if (tid == 0) {
      fence_after();
#pragma unroll
      for (int k = 0; k < kTcD / 16; ++k)
        mma(tS, sdesc(smem_u32(sQ) + k * 32, 16, 1024), sdesc(smem_u32(sK[s]) + k * 32, 16, 1024), IS, k > 0);
      commit(sbar);
    }
    s_pending = true;
    ok = wait_all(sbar, s_done & 1, err);
    if (!ok) break;
    ++s_done;
    s_pending = false;
    fence_after();
    // ---- this thread's score row: scale, window mask, online softmax, P -> smem
    const int kb0 = kstart + j * kTcBN;
    float sc[kTcBN];
#pragma unroll
    for (int c = 0; c < kTcBN / 32; ++c) tmem_ld32(tS + lane_off + c * 32, sc + c * 32);
    float mx = m;
#pragma unroll
    for (int c = 0; c < kTcBN; ++c) {
      const int kp = kb0 + c;
      sc[c] = (kp <= qpos && kp < T) ? sc[c] * sl : -INFINITY;
      mx = fmaxf(mx, sc[c]);
    }
    const float base = (mx == -INFINITY) ? 0.f : mx;
    const float alpha = (m == -INFINITY) ? 0.f : exp2f(m - base);
    float rs = 0.f;
#pragma unroll
    for (int c8 = 0; c8 < kTcBN / 8; ++c8) {
      uint32_t pk[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p0 = exp2f(sc[c8 * 8 + 2 * e] - base), p1 = exp2f(sc[c8 * 8 + 2 * e + 1] - base);
        rs += p0 + p1;
        __nv_bfloat162 t2 = __floats2bfloat162_rn(p0, p1);
        pk[e] = *reinterpret_cast<uint32_t*>(&t2);
      }
      const int sub = c8 >> 3, chunk = c8 & 7;
      uint8_t* dst = sP + sub * kTcTile + tid * 128 + ((chunk ^ (tid & 7)) << 4);
      *reinterpret_cast<uint4*>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
    l = l * alpha + rs;
    m = mx;
    fence_proxy_async();  // generic-proxy P stores -> visible to the tensor core
    fence_before();
    __syncthreads();
    // ---- O_blk = P V (M=128 queries, N=64 channels, K=128 keys; V is MN-major)
    if (tid == 0) {
      fence_after();
#pragma unroll
      for (int k = 0; k < kTcBN / 16; ++k) {
        const uint64_t ad = sdesc(smem_u32(sP) + (k >> 2) * kTcTile + (k & 3) * 32, 16, 1024);
        const uint64_t bd = sdesc(smem_u32(sV[s]) + k * 2048, 8192, 1024);
        mma(tO, ad, bd, IO, k > 0);
      }
      commit(obar);
    }
    o_pending = true;
    ok = wait_all(obar, o_done & 1, err);
    if (!ok) break;
    ++o_done;
    o_pending = false;
    fence_after();
    float ob[kTcD];
#pragma unroll
    for (int c = 0; c < kTcD / 32; ++c) tmem_ld32(tO + lane_off + c * 32, ob + c * 32);
#pragma unroll
    for (int d = 0; d < kTcD; ++d) o[d] = o[d] * alpha + ob[d];
    fence_before();
    __syncthreads();  // every thread has read S and O: TMEM and stage s are free
    if (j + 2 < nblk) {
      if (tid == 0) {
        fence_after();
        mbar_expect_tx(&kvbar[s], 2 * kTcTile);
        tma_2d(sK[s], &tk, col, row0 + kstart + (j + 2) * kTcBN, &kvbar[s]);
        tma_2d(sV[s], &tv, col, row0 + kstart + (j + 2) * kTcBN, &kvbar[s]);
      }
      ++kv_armed[s];
    }
  }
  if (!ok) {
    // drain: wait (bounded) for this CTA's copies and MMAs still in flight
    if (tid == 0) {
      mbar_wait(qbar, 0, nullptr);
      for (int s = 0; s < 2; ++s)
        if (kv_armed[s] > kv_done[s]) mbar_wait(&kvbar[s], kv_done[s] & 1, nullptr);
      if (s_pending) mbar_wait(sbar, s_done & 1, nullptr);
      if (o_pending) mbar_wait(obar, o_done & 1, nullptr);
    }
  } else if (qpos < T) {
    const float inv = 1.f / l;
    bf16* orow = out + ((long long)(row0 + qpos) * H + h) * kTcD;
#pragma unroll
    for (int c8 = 0; c8 < kTcD / 8; ++c8) {
      uint32_t pk[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        __nv_bfloat162 t2 = __floats2bfloat162_rn(o[c8 * 8 + 2 * e] * inv, o[c8 * 8 + 2 * e + 1] * inv);
        pk[e] = *reinterpret_cast<uint32_t*>(&t2);
      }
      *reinterpret_cast<uint4*>(orow + c8 * 8) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
    if (lse) lse[((long long)b * H + h) * T + qpos] = (m + log2f(l)) * 0.6931471805599453f;
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTcTmemCols));
  }
}

}  // namespace tao
