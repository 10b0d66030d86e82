// Training fine writer on the 5th-generation tensor cores (sm_100a).
//
// One CTA of 128 threads per (batch, head, sealed 256-token block).  Reference: the
// softmax writer of _seal_training_all (tao_stream.py:80-123, one block as in
// tao_stream.py:66-76): per channel m = max_t k, e = bf16(exp(bf16(k - m))),
// Z = bf16(sum_t e), p = bf16(e / Z), z = bf16(m + bf16(log Z)); C = bf16(p^T v) with
// fp32 accumulation.
//
// The block's raw keys and values are copied into shared memory in the layout of the
// tensor core's MN-major operands with 128-byte swizzle: 64-channel atoms of 256 token
// rows x 128 B (16-byte chunks XOR-ed with row % 8), 1024-byte aligned.  p replaces the
// keys in place, then one thread issues C = p^T v as 16 tcgen05.mma (M = 128, N = D,
// K = 16 tokens each; A = p^T and B = v both MN-major) into a TMEM accumulator, and
// commits to an mbarrier.  At width 64 the instruction's rows 64-127 take the value
// atom as a stand-in A operand; they land in TMEM lanes 64-127, which nobody reads.
// Thread d of the epilogue reads row d of C from TMEM lane d (tcgen05.ld) and writes
// it as bf16.  The wait on the MMA is bounded; on a timeout the CTA records the error,
// frees its TMEM and returns.
#pragma once
#include "stream_kernels.cuh"
#include "tcgen05.cuh"
#include "train_kernels.cuh"

namespace tao {

template <int D>
struct TcWriterCfg {
  static constexpr int NA = D / 64;                      // 64-channel atoms per operand
  static constexpr uint32_t ATOM = 256 * 128;            // 256 token rows x 128 B
  static constexpr uint32_t TILE = NA * ATOM;            // keys / probabilities, or values
  // two tiles, the channel statistics, their scratch, the mbarrier and TMEM slot, and
  // the slack to align the dynamic window to 1024 bytes
  static constexpr size_t SMEM = 2 * (size_t)TILE + 2 * D * 4 + 2 * 128 * 4 + 64 + 1024;
  static constexpr uint32_t TMEM_COLS = D;               // fp32 accumulator, N = D columns
};

// Byte offset of (token t, channel d) in an operand tile of TcWriterCfg<D>.
template <int D>
TAO_DEVI uint32_t tw_off(int t, int d) {
  return (uint32_t)(d >> 6) * TcWriterCfg<D>::ATOM + (uint32_t)t * 128u +
         ((uint32_t)(((d & 63) >> 3) ^ (t & 7)) << 4) + ((uint32_t)(d & 7) << 1);
}

// One 256-token block: the softmax writer's z (z_out[D]) and, when write_c, C
// (c_out[D][D]) from keys and values with rows `row` elements apart.  128 threads;
// `sm_raw` is the kernel's dynamic shared memory (TcWriterCfg<D>::SMEM bytes).
// Returns false when the wait on the MMA gave up (the error word is set).
template <int D>
TAO_DEVI bool tc_block_writer(const bf16* __restrict__ kb, const bf16* __restrict__ vb, long long row,
                              bf16* zo, bf16* co, int write_c, int* err, uint8_t* sm_raw) {
  using namespace tc;
  using Cfg = TcWriterCfg<D>;
  constexpr int NT = 256, CH = D / 8;
  const uint32_t raw = smem_u32(sm_raw);
  uint8_t* const sm = sm_raw + (((raw + 1023u) & ~1023u) - raw);   // 1024-byte aligned window
  uint8_t* const sP = sm;                  // keys, then probabilities (A operand)
  uint8_t* const sV = sm + Cfg::TILE;      // values (B operand)
  float* const mx = reinterpret_cast<float*>(sm + 2 * Cfg::TILE);
  float* const zp = mx + D;
  float* const scratch = zp + D;                                        // [2 * 128]
  uint64_t* const bar = reinterpret_cast<uint64_t*>(scratch + 2 * 128);
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  int* const okflag = reinterpret_cast<int*>(tmem_slot + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  for (int idx = tid; idx < NT * CH; idx += 128) {
    const int r = idx / CH, c = idx % CH;
    wa::cp_async16(smem_u32(sP + tw_off<D>(r, c * 8)), kb + (long long)r * row + c * 8, true);
    wa::cp_async16(smem_u32(sV + tw_off<D>(r, c * 8)), vb + (long long)r * row + c * 8, true);
  }
  wa::cp_commit();
  if (write_c && warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(Cfg::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  wa::cp_wait<0>();
  __syncthreads();

  auto at = [&](int t, int d) -> bf16& { return *reinterpret_cast<bf16*>(sP + tw_off<D>(t, d)); };
  // e replaces the key in shared memory (exact in bf16); then p = bf16(e / Z) in place
  channel_stats<D, 128>([&](int t, int d) { return bf(at(t, d)); }, mx, zp, scratch,
                        [&](int t, int d, float e) { at(t, d) = tobf(e); });
  for (int idx = tid; idx < NT * D / 2; idx += 128) {  // two channels at a time
    const int t = idx / (D / 2), d = (idx % (D / 2)) * 2;
    uint32_t* cell = reinterpret_cast<uint32_t*>(sP + tw_off<D>(t, d));
    const uint32_t e2 = *cell;
    *cell = wa::pack_bf16(__fdiv_rn(lo_f(e2), zp[d]), __fdiv_rn(hi_f(e2), zp[d + 1]));
  }
  for (int d = tid; d < D; d += 128) zo[d] = tobf(__fadd_rn(mx[d], rb(logf(zp[d]))));
  if (!write_c) return true;  // the caller supplies C (another fine writer); no TMEM was taken

  // C = p^T v: the generic-proxy writes of p become visible to the tensor core
  fence_proxy_async();
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tbase = *tmem_slot;
  if (tid == 0) {
    constexpr uint32_t I = idesc_bf16(128, D, 1, 1);   // A and B MN-major
    const uint32_t aP = smem_u32(sP), aV = smem_u32(sV);
    // M = 128: atom 1 of A is the next tile (the values at width 64: rows 64-127 unused)
    for (int k = 0; k < NT / 16; ++k)
      mma(tbase, sdesc(aP + k * 2048, Cfg::ATOM, 1024), sdesc(aV + k * 2048, Cfg::ATOM, 1024), I, k > 0);
    commit(bar);
  }
  // every thread waits (bounded) for the accumulator; a timeout skips the epilogue
  if (tid == 0) *okflag = mbar_wait(bar, 0, err) ? 1 : 0;
  __syncthreads();
  fence_after();
  const bool ok = *okflag != 0;
  if (ok && warp < D / 32) {
    // warp w reads TMEM lanes 32w..32w+31: thread d holds row d of C
    bf16* crow = co + (long long)tid * D;
#pragma unroll
    for (int c0 = 0; c0 < D; c0 += 32) {
      float vals[32];
      tmem_ld32(tbase + ((uint32_t)(warp * 32) << 16) + c0, vals);
#pragma unroll
      for (int e = 0; e < 32; e += 8) {
        uint4 o;
        o.x = wa::pack_bf16(vals[e], vals[e + 1]);
        o.y = wa::pack_bf16(vals[e + 2], vals[e + 3]);
        o.z = wa::pack_bf16(vals[e + 4], vals[e + 5]);
        o.w = wa::pack_bf16(vals[e + 6], vals[e + 7]);
        *reinterpret_cast<uint4*>(crow + c0 + e) = o;
      }
    }
  } else if (!ok && tid == 0) {
    // give the MMA still in flight its bounded wait before the TMEM goes back
    mbar_wait(bar, 0, err);
  }
  fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(Cfg::TMEM_COLS));
  return ok;
}

template <int D>
__global__ void __launch_bounds__(128) tc_writer_kernel(const bf16* __restrict__ raw_k,
                                                        const bf16* __restrict__ v, bf16* z_out, bf16* c_out,
                                                        TrainDims dm, int write_c, int* err) {
  extern __shared__ uint8_t sm_raw[];
  const int s = blockIdx.x % dm.S, h = (blockIdx.x / dm.S) % dm.H, b = blockIdx.x / (dm.S * dm.H);
  const long long first = ((long long)b * dm.T + (long long)s * 256) * dm.row + (long long)h * D;
  tc_block_writer<D>(raw_k + first, v + first, dm.row, z_out + (((long long)b * dm.H + h) * dm.S + s) * D,
                     c_out + (((long long)b * dm.H + h) * dm.S + s) * (long long)D * D, write_c, err, sm_raw);
}

// Decode seal (the window of a request reached 768 tokens on the token just served):
// the oldest 256-token block of head h is sealed as fine S with the same block writer
// (its keys and values are 256 consecutive ring slots), then the page memo of the page
// receiving it is refreshed (tao_stream.py:435-512, 399-416).  One CTA of 128 threads
// per (request, head); CTAs of requests that do not seal return at once.
template <int D>
__global__ void __launch_bounds__(128) tc_seal_kernel(StepArgs a) {
  extern __shared__ uint8_t sm_raw[];
  const int r = blockIdx.x / a.H, h = blockIdx.x % a.H;
  TaoState& st = *a.states[r];
  const long long t = st.position - 1;  // the token just served
  const long long start = window_start(t);
  if (t + 1 - start != kWindow) return;
  const int S = sealed_at(t);
  const long long slot0 = (long long)h * kWindow + start % kWindow;
  bf16* zo = reinterpret_cast<bf16*>(st.fine_z) + ((long long)h * st.cap_fines + S) * D;
  bf16* co = reinterpret_cast<bf16*>(st.fine_c) + ((long long)h * st.cap_fines + S) * (long long)D * D;
  if (!tc_block_writer<D>(reinterpret_cast<const bf16*>(st.rk_ring) + slot0 * D,
                          reinterpret_cast<const bf16*>(st.v_ring) + slot0 * D, D, zo, co, 1, a.err, sm_raw))
    return;
  __syncthreads();
  refresh_memo<D>(st, h, S + 1, S / kGroup);
  if (h == 0 && threadIdx.x == 0) st.seal_events += 1;
}

}  // namespace tao
