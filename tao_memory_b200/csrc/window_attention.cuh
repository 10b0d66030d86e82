// Exact windowed causal attention over [tokens][heads][width] bf16 operands.
//
// Semantics (reference flash_attention.py:16-37 as called by tao_stream.py:760-787
// and StreamCache.process tao_stream.py:933-934): query at absolute position t
// reads keys [window_start, t] with scale 1/sqrt(D); window_start is 0 before the
// first seal and 256*floor(t/256) - 512 afterwards.  One CTA owns 64 queries of
// one (batch, head); keys stream through double-buffered shared memory in blocks
// of 64; scores and P*V run on the tensor cores (bf16 in, fp32 accumulate) with
// an online softmax in registers.
#pragma once
#include "../../include/tao_b200.h"
#include "common.cuh"

namespace tao {

struct WinAttnParams {
  const bf16* q;      // query rows: q + qoff(b) + i * q_row_stride + h * D
  const bf16* k;      // key rows: contiguous (row = position) or ring (row = position % 768)
  const bf16* v;
  bf16* out;
  float* lse;         // optional [B][H][nq] natural log-sum-exp of scaled scores
  long long q_batch_stride, q_row_stride;   // in elements
  long long k_batch_stride, k_row_stride, k_head_stride;
  long long o_batch_stride, o_row_stride;
  int heads;
  int nq;             // queries per (b,h)
  long long qpos0;    // absolute position of query row 0
  long long kstart;   // first visible key position (< 0: derive per 256-tile)
  int ring;           // 1: key row = position % 768
  TaoState* const* states;  // optional: per-batch ring pointers and cursor (prefill)
};

namespace wa {

TAO_DEVI uint32_t swz(int row, int col, int width) {
  // byte offset of element (row, col) in a [rows][width] bf16 tile, 16-byte
  // chunks XOR-swizzled by row % 8 (conflict-free ldmatrix)
  return row * width * 2 + ((((col >> 3) ^ (row & 7))) << 4) + ((col & 7) << 1);
}

TAO_DEVI void cp_async16(uint32_t dst, const void* src, bool valid) {
  int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz)
               : "memory");
}
TAO_DEVI void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
TAO_DEVI void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

TAO_DEVI void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
TAO_DEVI void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
TAO_DEVI void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
TAO_DEVI uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&t);
}

}  // namespace wa

template <int D>
__global__ void __launch_bounds__(128) window_attention_kernel(WinAttnParams p) {
  using namespace wa;
  constexpr int BM = 64, BN = 64, CH = D / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK = sQ + BM * D * 2;
  const uint32_t sV = sK + 2 * BN * D * 2;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y, b = bh / p.heads, h = bh % p.heads;
  const int i0 = blockIdx.x * BM;
  const int nq = min(BM, p.nq - i0);
  if (nq <= 0) return;
  long long qbase_pos = p.qpos0;
  long long kstart = p.kstart;
  const bf16* kbase = p.k + b * p.k_batch_stride;
  const bf16* vbase = p.v + b * p.k_batch_stride;
  if (p.states) {
    const TaoState& st = *p.states[b];
    qbase_pos = st.position;
    kstart = window_start(st.position);
    kbase = reinterpret_cast<const bf16*>(st.k_ring);
    vbase = reinterpret_cast<const bf16*>(st.v_ring);
  }
  const long long qpos0 = qbase_pos + i0;
  if (kstart < 0) {
    long long tile = qpos0 / kFine;
    kstart = tile * kFine - kKeep;
    if (kstart < 0) kstart = 0;
  }
  const long long kend = qpos0 + nq;  // exclusive

  const bf16* qb = p.q + b * p.q_batch_stride + (long long)h * D;
  const bf16* kb = kbase + (long long)h * p.k_head_stride;
  const bf16* vb = vbase + (long long)h * p.k_head_stride;

  auto krow = [&](long long pos) -> long long {
    return (p.ring ? (pos % kWindow) : pos) * p.k_row_stride;
  };

  // ---- load Q tile (rows >= nq zero-filled)
  for (int idx = tid; idx < BM * CH; idx += 128) {
    int r = idx / CH, c = idx % CH;
    bool ok = r < nq;
    const bf16* src = qb + (long long)(i0 + (ok ? r : 0)) * p.q_row_stride + c * 8;
    cp_async16(sQ + swz(r, c * 8, D), src, ok);
  }
  auto load_kv = [&](long long k0, int buf) {
    for (int idx = tid; idx < BN * CH; idx += 128) {
      int r = idx / CH, c = idx % CH;
      long long pos = k0 + r;
      bool ok = pos < kend;
      long long off = krow(ok ? pos : k0) + c * 8;
      cp_async16(sK + buf * BN * D * 2 + swz(r, c * 8, D), kb + off, ok);
      cp_async16(sV + buf * BN * D * 2 + swz(r, c * 8, D), vb + off, ok);
    }
  };
  load_kv(kstart, 0);
  cp_commit();

  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  uint32_t qf[D / 16][4];
  const float sl = 1.4426950408889634f / sqrtf((float)D);  // log2(e)/sqrt(D)
  const int g = lane >> 2, c4 = lane & 3;
  const long long qrow0 = qpos0 + warp * 16 + g;  // absolute position of this thread's row g
  const int nblocks = (int)((kend - kstart + BN - 1) / BN);

  for (int blk = 0; blk < nblocks; ++blk) {
    const long long k0 = kstart + (long long)blk * BN;
    if (blk + 1 < nblocks) {
      load_kv(k0 + BN, (blk + 1) & 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (blk == 0) {
#pragma unroll
      for (int kt = 0; kt < D / 16; ++kt) {
        int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        int c = kt * 16 + (lane >> 4) * 8;
        ldsm_x4(sQ + swz(r, c, D), qf[kt][0], qf[kt][1], qf[kt][2], qf[kt][3]);
      }
    }
    const uint32_t kbuf = sK + (blk & 1) * BN * D * 2;
    const uint32_t vbuf = sV + (blk & 1) * BN * D * 2;
    float s[BN / 8][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int np = 0; np < BN / 16; ++np) {
#pragma unroll
      for (int kt = 0; kt < D / 16; ++kt) {
        uint32_t b0, b1, b2, b3;
        int r = np * 16 + (lane & 7) + (lane >> 4) * 8;
        int c = kt * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(kbuf + swz(r, c, D), b0, b1, b2, b3);
        mma16816(s[2 * np], qf[kt], b0, b1);
        mma16816(s[2 * np + 1], qf[kt], b2, b3);
      }
    }
    // mask + online softmax (rows g and g+8 of this warp's 16)
    float mnew[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      long long qp = qrow0 + hr * 8;
      float mx = mrow[hr];
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          long long kp = k0 + j * 8 + c4 * 2 + e;
          float val = s[j][hr * 2 + e] * sl;
          if (kp >= kend || kp > qp) val = -INFINITY;
          s[j][hr * 2 + e] = val;
          mx = fmaxf(mx, val);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mnew[hr] = mx;
    }
    float alpha_r[2], base[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      base[hr] = (mnew[hr] == -INFINITY) ? 0.f : mnew[hr];
      alpha_r[hr] = (mrow[hr] == -INFINITY) ? 0.f : exp2f(mrow[hr] - base[hr]);
      mrow[hr] = mnew[hr];
    }
    float lsum[2] = {0.f, 0.f};
    uint32_t pa[BN / 16][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
      float p0 = exp2f(s[j][0] - base[0]), p1 = exp2f(s[j][1] - base[0]);
      float p2 = exp2f(s[j][2] - base[1]), p3 = exp2f(s[j][3] - base[1]);
      lsum[0] += p0 + p1;
      lsum[1] += p2 + p3;
      int kt = j >> 1;
      if ((j & 1) == 0) {
        pa[kt][0] = pack_bf16(p0, p1);
        pa[kt][1] = pack_bf16(p2, p3);
      } else {
        pa[kt][2] = pack_bf16(p0, p1);
        pa[kt][3] = pack_bf16(p2, p3);
      }
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      lsum[hr] += __shfl_xor_sync(0xffffffffu, lsum[hr], 1);
      lsum[hr] += __shfl_xor_sync(0xffffffffu, lsum[hr], 2);
      lrow[hr] = lrow[hr] * alpha_r[hr] + lsum[hr];
    }
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      o[j][0] *= alpha_r[0];
      o[j][1] *= alpha_r[0];
      o[j][2] *= alpha_r[1];
      o[j][3] *= alpha_r[1];
    }
#pragma unroll
    for (int kt = 0; kt < BN / 16; ++kt) {
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t b0, b1, b2, b3;
        int r = kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        int c = dp * 16 + (lane >> 4) * 8;
        ldsm_x4_t(vbuf + swz(r, c, D), b0, b1, b2, b3);
        mma16816(o[2 * dp], pa[kt], b0, b1);
        mma16816(o[2 * dp + 1], pa[kt], b2, b3);
      }
    }
    __syncthreads();  // buffer (blk&1) is refilled two iterations later
  }

  // ---- epilogue
  bf16* ob = p.out + b * p.o_batch_stride + (long long)h * D;
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    int r = warp * 16 + g + hr * 8;
    if (r >= nq) continue;
    float inv = 1.f / lrow[hr];
    bf16* orow = ob + (long long)(i0 + r) * p.o_row_stride;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      __nv_bfloat162 t = __floats2bfloat162_rn(o[j][hr * 2] * inv, o[j][hr * 2 + 1] * inv);
      *reinterpret_cast<__nv_bfloat162*>(orow + j * 8 + c4 * 2) = t;
    }
    if (p.lse && c4 == 0) {
      p.lse[((long long)b * p.heads + h) * p.nq + i0 + r] =
          (mrow[hr] + log2f(lrow[hr])) * 0.6931471805599453f;
    }
  }
}

}  // namespace tao
