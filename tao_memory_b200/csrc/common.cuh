// Shared device helpers for the TaoMemory sm_100a kernels.
//
// Rounding helpers: every `rb()` marks a bf16 rounding point of the reference
// (a `.to(bfloat16)` or a bf16 tensor op).  Products and sums that feed such a
// point use __fmul_rn/__fadd_rn so the compiler can never contract them into an
// FMA across the rounding point.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>

#define TAO_DEVI __device__ __forceinline__

namespace tao {

typedef __nv_bfloat16 bf16;

constexpr int kFine = 256;        // tokens per sealed fine block (TaoConfig.fine_tokens)
constexpr int kKeep = 512;        // exact tokens kept after a seal (TaoConfig.local_keep)
constexpr int kWindow = 768;      // serve limit = ring capacity in tokens
constexpr int kGroup = 8;         // fines per coarse page (TaoConfig.coarse_group)
// bf16(log 2): the fusion's local bias with two history terms (coarse and fine)
constexpr float kLocalBiasTwo = 0.69140625f;

// Device error word bits (workspace[0]); read back by tao_stream_check.
constexpr int kErrWaitTimeout = 1;
constexpr int kErrRouteCap = 2;
constexpr int kErrState = 4;

TAO_DEVI float rb(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
TAO_DEVI float bf(bf16 x) { return __bfloat162float(x); }
TAO_DEVI bf16 tobf(float x) { return __float2bfloat16_rn(x); }

TAO_DEVI float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
TAO_DEVI float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Products of two bf16 pairs rounded to bf16, lane by lane.  The product of two
// bf16 values is exact in fp32, so this equals rb(a * b) for each lane.
TAO_DEVI uint32_t hmul2u(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
// Low / high bf16 of a pair as fp32.
// Two floats rounded to bf16 (nearest even) and packed, lo in the low half.
TAO_DEVI uint32_t bf16x2(float lo, float hi) {
  __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&t);
}
TAO_DEVI float lo_f(uint32_t x) { return __uint_as_float(x << 16); }
TAO_DEVI float hi_f(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }

// Unpack 8 bf16 (one 16-byte vector) into fp32.
TAO_DEVI void unpack8(const uint4& u, float* f) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(p[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// ---------------------------------------------------------------------------
// mbarrier + bulk (TMA, non-tensor) copies global -> shared.
// Every wait is bounded; a timeout sets kErrWaitTimeout and returns false.
// ---------------------------------------------------------------------------
TAO_DEVI uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

TAO_DEVI void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
TAO_DEVI void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
TAO_DEVI void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
TAO_DEVI void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned).
TAO_DEVI void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
TAO_DEVI bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// Bounded wait: ~2^22 polls (each try_wait may itself suspend briefly), far
// beyond any legitimate copy latency.
TAO_DEVI bool mbar_wait(uint64_t* bar, uint32_t phase, int* err) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (mbar_try_wait(bar, phase)) return true;
  }
  if (err) atomicOr(err, kErrWaitTimeout);
  return false;
}

// Arrival counters: a release-ordered add (the CTA's earlier writes, ordered by a
// preceding barrier, become visible first) and an acquire fence for the winner.
TAO_DEVI int atomic_add_release(int* p, int v) {
  int old;
  asm volatile("atom.add.release.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
TAO_DEVI void fence_acquire() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Integer schedule (reference tao_stream.py:29-37, config.py:54-60,
// tao_stream.py:196-227, 914-917, 959-967).
// ---------------------------------------------------------------------------
struct Policy {
  int route_period;   // 24
  int layer_stagger;  // 2
  int root_scale;     // 2
  int offset;         // 2
};

TAO_DEVI long long isqrt_ll(long long n) {
  long long r = (long long)sqrt((double)n);
  while (r * r > n) --r;
  while ((r + 1) * (r + 1) <= n) ++r;
  return r;
}
TAO_DEVI int budget(int count, const Policy& p) {
  if (count <= 0) return 0;
  long long sq = (long long)p.root_scale * count;
  long long r = isqrt_ll(sq);
  if (r * r < sq) ++r;
  long long b = r + p.offset;
  return (int)(b < count ? b : count);
}
struct Counts {
  int coarse, eligible, selected;
};
TAO_DEVI Counts routed_counts(int completed, int pending, const Policy& p) {
  int cb = budget(kGroup * completed, p);
  int coarse = (2 * cb + kGroup - 1) / kGroup;
  coarse = coarse < completed ? coarse : completed;
  int eligible = kGroup * coarse + pending;
  int b = budget(kGroup * completed + pending, p);
  return {coarse, eligible, eligible < b ? eligible : b};
}
// Sealed fines before the token at `pos` is processed.
TAO_DEVI int sealed_at(long long pos) {
  return pos >= kWindow ? (int)((pos - kWindow) / kFine) + 1 : 0;
}
// First absolute position of the exact local window when `pos` is served.
TAO_DEVI long long window_start(long long pos) {
  return pos < kWindow ? 0 : (long long)kFine * ((pos - kKeep) / kFine);
}
TAO_DEVI bool is_refresh(long long pos, int layer, const Policy& p) {
  long long first_turn = kWindow + (long long)p.layer_stagger * layer;
  return pos == kWindow || (pos >= first_turn && (pos - first_turn) % p.route_period == 0);
}

}  // namespace tao
