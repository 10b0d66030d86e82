// Training backward kernels of tao_attention on sm_100a.
//
// Reference: the torch autograd of operator._fuse_training (operator.py:21-39),
// of the SDPA local attention (flash_attention.py:16-37 via tao_stream.py:760-787),
// _SelectedRead.backward (selected_read.py:175-187) and of the writer and page
// summaries (tao_stream.py:80-123, 530-593).  Rounding points follow those ops.
#pragma once
#include "tcgen05.cuh"
#include "common.cuh"
#include "window_attention.cuh"
#include "train_kernels.cuh"

namespace tao {

struct BwdArgs {
  const bf16 *g, *raw_q, *local, *num, *fa, *fb, *q, *k, *v, *raw_k;
  const float *den, *gain, *lse;
  const bf16 *z, *C, *pzpre;
  const int16_t* sel;
  bf16 *d_local, *gn, *d_rq_f;   // [B,T,H,D]
  float *gd, *dv_row;            // [B,T,H], [B,H,T] (row dot of dO and O for attention)
  float *d_fa, *d_fb;            // fp32 [H,D,3] accumulators
  bf16 *dq, *dk, *dv, *d_raw_q, *d_raw_k;
  float *dC, *dz;                // fp32 [B,H,S,D,D] (reduced), [B,H,S,D] accumulators
  bf16* dcp;                     // per-(tile, fine) dC partials [B,H,npairs,D,D]
  float* dq_acc;                 // fp32 [B,T,H,D] dQ accumulator (tensor-core path) or null
  int caller_c;                  // 1: fine C came from the caller; writer backward: z path only
  int external_fusion;           // 1: g is d(fine), d_local comes from the caller (split_bwd_kernel)
  int route_only;                // 1: only the local attention's gradients (the caller reads the fines)
  int npairs;                    // sum over tiles of visible fines
  TrainDims dm;
  int pages, mmax;
  int* err;
};

// Rows (tokens) of one warp in the fusion backward and the external-fusion split.
constexpr int kFusionRowsPerWarp = 16;

// ---------------------------------------------------------------------------
// External fusion (the caller applied the pointwise gate to the local and fine
// outputs and returns their gradients): g holds d(fine), d_local holds the
// caller's d(local).  This kernel takes the place of fusion_bwd_kernel: it forms
// the gradients of fine = bf16(bf16(num) / den) (torch's division backward, each
// op rounded: d num = bf16(d fine / den), d den = -sum_d bf16(d fine * bf16(fine / den)))
// for rows with history, the attention row dot sum_d d(local) * local, and no
// raw_q or fusion-parameter gradient (the caller's gate owns those).
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) split_bwd_kernel(BwdArgs a) {
  constexpr int NP = D / 64;
  const int tile = blockIdx.x, b = blockIdx.y / a.dm.H, h = blockIdx.y % a.dm.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = tile * 8 * kFusionRowsPerWarp + warp * kFusionRowsPerWarp;
  const int rows = min(kFusionRowsPerWarp, a.dm.T - t0);
  for (int rr = 0; rr < rows; ++rr) {
    const int t = t0 + rr;
    const long long base = ((long long)b * a.dm.T + t) * a.dm.row + (long long)h * D + 2 * lane;
    const bool present = t >= kWindow && !a.route_only;
    const float den = present ? a.den[((long long)b * a.dm.T + t) * a.dm.H + h] : 1.f;
    float rowdot = 0.f, dden = 0.f;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const uint32_t dl2 = *reinterpret_cast<const uint32_t*>(a.d_local + base + 64 * p);
      const uint32_t l2 = __ldg(reinterpret_cast<const unsigned int*>(a.local + base + 64 * p));
      rowdot += lo_f(dl2) * lo_f(l2) + hi_f(dl2) * hi_f(l2);
      float dn[2] = {0.f, 0.f};
      if (present) {
        const uint32_t g2 = __ldg(reinterpret_cast<const unsigned int*>(a.g + base + 64 * p));
        const uint32_t n2 = __ldg(reinterpret_cast<const unsigned int*>(a.num + base + 64 * p));
        const float dfine[2] = {lo_f(g2), hi_f(g2)}, nums[2] = {lo_f(n2), hi_f(n2)};
        float fine[2], t2[2], dd[2];
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          fine[x] = __fdiv_rn(nums[x], den);
          dn[x] = __fdiv_rn(dfine[x], den);
        }
        rb2(fine[0], fine[1]);
        rb2(dn[0], dn[1]);
#pragma unroll
        for (int x = 0; x < 2; ++x) t2[x] = __fdiv_rn(fine[x], den);
        rb2(t2[0], t2[1]);
#pragma unroll
        for (int x = 0; x < 2; ++x) dd[x] = __fmul_rn(dfine[x], t2[x]);
        rb2(dd[0], dd[1]);
        dden += -dd[0] + -dd[1];
      }
      *reinterpret_cast<uint32_t*>(a.gn + base + 64 * p) = pack_exact(dn[0], dn[1]);
      *reinterpret_cast<uint32_t*>(a.d_rq_f + base + 64 * p) = 0u;
    }
    rowdot = warp_sum(rowdot);
    dden = warp_sum(dden);
    if (lane == 0) {
      a.gd[((long long)b * a.dm.T + t) * a.dm.H + h] = rb(dden);
      a.dv_row[((long long)b * a.dm.H + h) * a.dm.T + t] = rowdot;
    }
  }
}

// ---------------------------------------------------------------------------
// Fusion backward: one warp per (token, head) row, each lane a pair of adjacent
// channels (64p + 2*lane, +1), so every bf16 rounding point rounds both with one
// packed conversion; each warp takes kFusionRowsPerWarp consecutive tokens (the
// next row's inputs are loaded while the current one is processed), a CTA 8 warps.
// ---------------------------------------------------------------------------

template <int D>
__global__ void __launch_bounds__(256) fusion_bwd_kernel(BwdArgs a) {
  constexpr int NP = D / 64;
  const int tile = blockIdx.x, b = blockIdx.y / a.dm.H, h = blockIdx.y % a.dm.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float gain = a.gain[h];
  float acc_fa[NP][2][3], acc_fb[NP][2][3], fa[NP][2][3], fb[NP][2][3];
#pragma unroll
  for (int p = 0; p < NP; ++p)
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
      for (int x = 0; x < 3; ++x) {
        const long long i = ((long long)h * D + 64 * p + 2 * lane + k) * 3 + x;
        acc_fa[p][k][x] = acc_fb[p][k][x] = 0.f;
        fa[p][k][x] = bf(a.fa[i]);
        fb[p][k][x] = bf(a.fb[i]);
      }
  const int t0 = tile * 8 * kFusionRowsPerWarp + warp * kFusionRowsPerWarp;
  const int rows = min(kFusionRowsPerWarp, a.dm.T - t0);
  // row inputs (read-only in this kernel): g, local, raw_q, num pairs and den
  uint32_t cg[NP], cl[NP], cq[NP], cn[NP];
  float cden = 1.f;
  auto load_row = [&](int t, uint32_t (&g2)[NP], uint32_t (&l2)[NP], uint32_t (&q2)[NP], uint32_t (&n2)[NP],
                      float& den) {
    const long long base = ((long long)b * a.dm.T + t) * a.dm.row + (long long)h * D + 2 * lane;
    const bool present = t >= kWindow;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      g2[p] = __ldg(reinterpret_cast<const unsigned int*>(a.g + base + 64 * p));
      l2[p] = __ldg(reinterpret_cast<const unsigned int*>(a.local + base + 64 * p));
      q2[p] = present ? __ldg(reinterpret_cast<const unsigned int*>(a.raw_q + base + 64 * p)) : 0u;
      n2[p] = present ? __ldg(reinterpret_cast<const unsigned int*>(a.num + base + 64 * p)) : 0u;
    }
    den = present ? __ldg(a.den + ((long long)b * a.dm.T + t) * a.dm.H + h) : 1.f;
  };
  if (rows > 0) load_row(t0, cg, cl, cq, cn, cden);
  for (int rr = 0; rr < rows; ++rr) {
    const int t = t0 + rr;
    uint32_t ng[NP], nl[NP], nq[NP], nn[NP];
    float nden = 1.f;
    if (rr + 1 < rows) load_row(t + 1, ng, nl, nq, nn, nden);
    const long long base = ((long long)b * a.dm.T + t) * a.dm.row + (long long)h * D + 2 * lane;
    const bool present = t >= kWindow;
    const float den = cden;
    float rowdot = 0.f, dden = 0.f;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const float gv[2] = {lo_f(cg[p]), hi_f(cg[p])}, loc[2] = {lo_f(cl[p]), hi_f(cl[p])};
      float dloc[2] = {gv[0], gv[1]}, dnum[2] = {0.f, 0.f}, drq[2] = {0.f, 0.f};
      if (present) {
        // the channel pair as float2: every rounded product / sum is a packed
        // fp32x2 instruction (each lane IEEE round-to-nearest), divisions stay scalar
        const float2 qv = make_float2(lo_f(cq[p]), hi_f(cq[p]));
        const float2 gv2 = make_float2(gv[0], gv[1]), lc2 = make_float2(loc[0], loc[1]);
        const float2 fa0w = make_float2(fa[p][0][0], fa[p][1][0]), fa2w = make_float2(fa[p][0][2], fa[p][1][2]);
        const float2 fb0w = make_float2(fb[p][0][0], fb[p][1][0]), fb2w = make_float2(fb[p][0][2], fb[p][1][2]);
        const float2 gain2 = make_float2(gain, gain), two = make_float2(2.f, 2.f);
        float2 fine = make_float2(__fdiv_rn(lo_f(cn[p]), den), __fdiv_rn(hi_f(cn[p]), den));
        rb2(fine.x, fine.y);
        float2 s0 = __fmul2_rn(fa0w, qv), s2 = __fmul2_rn(fa2w, qv);
        rb2(s0.x, s0.y);
        rb2(s2.x, s2.y);
        s0 = __fadd2_rn(s0, fb0w);  // base0; + 0 (the absent middle term) is exact
        s2 = __fadd2_rn(s2, fb2w);
        rb2(s0.x, s0.y);
        rb2(s2.x, s2.y);
        float2 rho0, rho2;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const float a0 = k ? s0.y : s0.x, a2 = k ? s2.y : s2.x;
          const float mx = fmaxf(a0, a2);
          // the larger term is exp(0) = 1 exactly: one exponential per element
          const float eo = expf(fminf(a0, a2) - mx);
          const float e0 = a0 >= a2 ? 1.f : eo, e2 = a0 >= a2 ? eo : 1.f;
          (k ? rho0.y : rho0.x) = __fdiv_rn(e0, e0 + e2);
          (k ? rho2.y : rho2.x) = __fdiv_rn(e2, e0 + e2);
        }
        rb2(rho0.x, rho0.y);
        rb2(rho2.x, rho2.y);
        float2 fg = __fmul2_rn(gain2, fine);
        float2 drho0 = __fmul2_rn(gv2, __fmul2_rn(two, lc2));  // bf16(2 * local) = 2 * local
        float2 t1 = __fmul2_rn(gv2, rho0);
        float2 dfine = __fmul2_rn(gv2, rho2);
        rb2(fg.x, fg.y);
        rb2(drho0.x, drho0.y);
        rb2(t1.x, t1.y);
        rb2(dfine.x, dfine.y);
        float2 drho2 = __fmul2_rn(gv2, fg);
        const float2 dl = __fmul2_rn(two, t1);  // exact
        dloc[0] = dl.x;
        dloc[1] = dl.y;
        dfine = __fmul2_rn(dfine, gain2);
        rb2(drho2.x, drho2.y);
        rb2(dfine.x, dfine.y);
        const float2 dot = __ffma2_rn(drho0, rho0, __fmul2_rn(drho2, rho2));
        float2 ds0 = __fmul2_rn(rho0, __fadd2_rn(drho0, make_float2(-dot.x, -dot.y)));
        float2 ds2 = __fmul2_rn(rho2, __fadd2_rn(drho2, make_float2(-dot.x, -dot.y)));
        rb2(ds0.x, ds0.y);
        rb2(ds2.x, ds2.y);
        acc_fb[p][0][0] += ds0.x;
        acc_fb[p][1][0] += ds0.y;
        acc_fb[p][0][2] += ds2.x;
        acc_fb[p][1][2] += ds2.y;
        float2 fa0 = __fmul2_rn(ds0, qv), fa2 = __fmul2_rn(ds2, qv);
        float2 x0 = __fmul2_rn(ds0, fa0w), x1 = __fmul2_rn(ds2, fa2w);
        float2 dn = make_float2(__fdiv_rn(dfine.x, den), __fdiv_rn(dfine.y, den));
        float2 t2 = make_float2(__fdiv_rn(fine.x, den), __fdiv_rn(fine.y, den));
        rb2(fa0.x, fa0.y);
        rb2(fa2.x, fa2.y);
        rb2(x0.x, x0.y);
        rb2(x1.x, x1.y);
        rb2(dn.x, dn.y);
        rb2(t2.x, t2.y);
        acc_fa[p][0][0] += fa0.x;
        acc_fa[p][1][0] += fa0.y;
        acc_fa[p][0][2] += fa2.x;
        acc_fa[p][1][2] += fa2.y;
        float2 rq = __fadd2_rn(x0, x1);
        float2 dd = __fmul2_rn(dfine, t2);
        rb2(rq.x, rq.y);
        rb2(dd.x, dd.y);
        drq[0] = rq.x;
        drq[1] = rq.y;
        dnum[0] = dn.x;
        dnum[1] = dn.y;
        dden += -dd.x + -dd.y;
      }
      *reinterpret_cast<uint32_t*>(a.d_local + base + 64 * p) = pack_exact(dloc[0], dloc[1]);
      *reinterpret_cast<uint32_t*>(a.gn + base + 64 * p) = pack_exact(dnum[0], dnum[1]);
      *reinterpret_cast<uint32_t*>(a.d_rq_f + base + 64 * p) = pack_exact(drq[0], drq[1]);
      rowdot += dloc[0] * loc[0] + dloc[1] * loc[1];
    }
    rowdot = warp_sum(rowdot);
    dden = warp_sum(dden);
    if (lane == 0) {
      a.gd[((long long)b * a.dm.T + t) * a.dm.H + h] = rb(dden);
      a.dv_row[((long long)b * a.dm.H + h) * a.dm.T + t] = rowdot;
    }
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      cg[p] = ng[p];
      cl[p] = nl[p];
      cq[p] = nq[p];
      cn[p] = nn[p];
    }
    cden = nden;
  }
  // block reduction of the fusion parameter gradients, one atomic per value per CTA
  __shared__ float red[8][D][6];
#pragma unroll
  for (int p = 0; p < NP; ++p)
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
      for (int x = 0; x < 3; ++x) {
        red[warp][64 * p + 2 * lane + k][x] = acc_fa[p][k][x];
        red[warp][64 * p + 2 * lane + k][3 + x] = acc_fb[p][k][x];
      }
  __syncthreads();
  for (int idx = threadIdx.x; idx < D * 6; idx += 256) {
    const int d = idx / 6, x = idx % 6;
    float s = 0.f;
    for (int w = 0; w < 8; ++w) s += red[w][d][x];
    if (s != 0.f) {
      float* dst = (x < 3) ? a.d_fa : a.d_fb;
      atomicAdd(dst + ((long long)h * D + d) * 3 + (x % 3), s);
    }
  }
}

// ---------------------------------------------------------------------------
// Windowed attention backward.  Query t sees keys [ws(t), t], ws(t) =
// max(0, 256*floor(t/256) - 512).  P = exp(s*scale - lse[t]); dS = P (dP - rowdot).
// ---------------------------------------------------------------------------
TAO_DEVI long long win_lo(long long t) {
  long long s = (t / kFine) * kFine - kKeep;
  return s < 0 ? 0 : s;
}

// dK, dV: one CTA per (64-key block, b, h); warps own 16 keys; loop over the
// query blocks that can see the keys.
template <int D>
__global__ void __launch_bounds__(128) attn_bwd_kv_kernel(BwdArgs a) {
  using namespace wa;
  constexpr int BN = 64, CH = D / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem), sV = sK + BN * D * 2;
  const uint32_t sQ = sV + BN * D * 2, sO = sQ + 2 * 64 * D * 2;  // double-buffered Q, dO
  float* lseS = reinterpret_cast<float*>(smem + 2 * BN * D * 2 + 4 * 64 * D * 2);  // [2][64]
  float* rdS = lseS + 128;                                                          // [2][64]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.y / a.dm.H, h = blockIdx.y % a.dm.H;
  const long long k0 = (long long)blockIdx.x * BN;
  const int T = a.dm.T;
  const long long row = a.dm.row;
  const bf16* qb = a.q + (long long)b * T * row + (long long)h * D;
  const bf16* kb = a.k + (long long)b * T * row + (long long)h * D;
  const bf16* vb = a.v + (long long)b * T * row + (long long)h * D;
  const bf16* ob = a.d_local + (long long)b * T * row + (long long)h * D;
  const float* lse = a.lse + ((long long)b * a.dm.H + h) * T;
  const float* rd = a.dv_row + ((long long)b * a.dm.H + h) * T;
  for (int idx = tid; idx < BN * CH; idx += 128) {
    const int r = idx / CH, c = idx % CH;
    const bool ok = k0 + r < T;
    const long long off = (ok ? k0 + r : k0) * row + c * 8;
    cp_async16(sK + swz(r, c * 8, D), kb + off, ok);
    cp_async16(sV + swz(r, c * 8, D), vb + off, ok);
  }
  long long qend = (k0 / kFine + 3) * kFine;
  if (qend > T) qend = T;
  const int nqb = (int)((qend - k0 + 63) / 64);
  auto load_q = [&](int qb_i, int buf) {
    const long long q0 = k0 + (long long)qb_i * 64;
    for (int idx = tid; idx < 64 * CH; idx += 128) {
      const int r = idx / CH, c = idx % CH;
      const bool ok = q0 + r < T;
      const long long off = (ok ? q0 + r : q0) * row + c * 8;
      cp_async16(sQ + buf * 64 * D * 2 + swz(r, c * 8, D), qb + off, ok);
      cp_async16(sO + buf * 64 * D * 2 + swz(r, c * 8, D), ob + off, ok);
    }
    for (int r = tid; r < 64; r += 128) {
      const bool ok = q0 + r < T;
      lseS[buf * 64 + r] = ok ? lse[q0 + r] * 1.4426950408889634f : 0.f;
      rdS[buf * 64 + r] = ok ? rd[q0 + r] : 0.f;
    }
  };
  load_q(0, 0);
  cp_commit();
  const float scale = 1.f / sqrtf((float)D), sl = 1.4426950408889634f * scale;
  const int g = lane >> 2, c4 = lane & 3;
  float dk[D / 8][4], dvv[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j)
#pragma unroll
    for (int x = 0; x < 4; ++x) dk[j][x] = dvv[j][x] = 0.f;
  uint32_t kf[D / 16][4], vf[D / 16][4];
  for (int qi = 0; qi < nqb; ++qi) {
    const int buf = qi & 1;
    if (qi + 1 < nqb) {
      load_q(qi + 1, buf ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (qi == 0) {
#pragma unroll
      for (int kt = 0; kt < D / 16; ++kt) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kt * 16 + (lane >> 4) * 8;
        ldsm_x4(sK + swz(r, c, D), kf[kt][0], kf[kt][1], kf[kt][2], kf[kt][3]);
        ldsm_x4(sV + swz(r, c, D), vf[kt][0], vf[kt][1], vf[kt][2], vf[kt][3]);
      }
    }
    const long long q0 = k0 + (long long)qi * 64;
    const uint32_t qbuf = sQ + buf * 64 * D * 2, obuf = sO + buf * 64 * D * 2;
    float st[8][4], dp[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int x = 0; x < 4; ++x) st[j][x] = dp[j][x] = 0.f;
#pragma unroll
    for (int np = 0; np < 4; ++np) {
#pragma unroll
      for (int kt = 0; kt < D / 16; ++kt) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = kt * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(qbuf + swz(r, c, D), b0, b1, b2, b3);
        mma16816(st[2 * np], kf[kt], b0, b1);
        mma16816(st[2 * np + 1], kf[kt], b2, b3);
        ldsm_x4(obuf + swz(r, c, D), b0, b1, b2, b3);
        mma16816(dp[2 * np], vf[kt], b0, b1);
        mma16816(dp[2 * np + 1], vf[kt], b2, b3);
      }
    }
    // P^T and dS^T (rows: keys, cols: queries)
    uint32_t pa[4][4], da[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float pv[4], dsv[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        const long long kp = k0 + warp * 16 + g + (x >> 1) * 8;
        const int ql = j * 8 + c4 * 2 + (x & 1);
        const long long qp = q0 + ql;
        const bool ok = qp < T && kp <= qp && kp >= win_lo(qp) && kp < T;
        const float p = ok ? exp2f(st[j][x] * sl - lseS[buf * 64 + ql]) : 0.f;
        pv[x] = p;
        dsv[x] = p * (dp[j][x] - rdS[buf * 64 + ql]);
      }
      const int kt = j >> 1;
      if ((j & 1) == 0) {
        pa[kt][0] = pack_bf16(pv[0], pv[1]);
        pa[kt][1] = pack_bf16(pv[2], pv[3]);
        da[kt][0] = pack_bf16(dsv[0], dsv[1]);
        da[kt][1] = pack_bf16(dsv[2], dsv[3]);
      } else {
        pa[kt][2] = pack_bf16(pv[0], pv[1]);
        pa[kt][3] = pack_bf16(pv[2], pv[3]);
        da[kt][2] = pack_bf16(dsv[0], dsv[1]);
        da[kt][3] = pack_bf16(dsv[2], dsv[3]);
      }
    }
    // dV += P^T dO ; dK += dS^T Q   (B operands from [query][d] tiles, transposed loads)
#pragma unroll
    for (int kt = 0; kt < 4; ++kt) {
#pragma unroll
      for (int dpi = 0; dpi < D / 16; ++dpi) {
        uint32_t b0, b1, b2, b3;
        const int r = kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dpi * 16 + (lane >> 4) * 8;
        ldsm_x4_t(obuf + swz(r, c, D), b0, b1, b2, b3);
        mma16816(dvv[2 * dpi], pa[kt], b0, b1);
        mma16816(dvv[2 * dpi + 1], pa[kt], b2, b3);
        ldsm_x4_t(qbuf + swz(r, c, D), b0, b1, b2, b3);
        mma16816(dk[2 * dpi], da[kt], b0, b1);
        mma16816(dk[2 * dpi + 1], da[kt], b2, b3);
      }
    }
    __syncthreads();
  }
  bf16* dkb = a.dk + (long long)b * T * row + (long long)h * D;
  bf16* dvb = a.dv + (long long)b * T * row + (long long)h * D;
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const long long kp = k0 + warp * 16 + g + hr * 8;
    if (kp >= T) continue;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const int e = j * 8 + c4 * 2;
      *reinterpret_cast<__nv_bfloat162*>(dkb + kp * row + e) =
          __floats2bfloat162_rn(dk[j][hr * 2] * scale, dk[j][hr * 2 + 1] * scale);
      *reinterpret_cast<__nv_bfloat162*>(dvb + kp * row + e) =
          __floats2bfloat162_rn(dvv[j][hr * 2], dvv[j][hr * 2 + 1]);
    }
  }
}

// dQ: one CTA per (64-query block, b, h); loop over the key blocks in the window.
template <int D>
__global__ void __launch_bounds__(128) attn_bwd_q_kernel(BwdArgs a) {
  using namespace wa;
  constexpr int BN = 64, CH = D / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem), sO = sQ + 64 * D * 2;
  const uint32_t sK = sO + 64 * D * 2, sV = sK + 2 * BN * D * 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.y / a.dm.H, h = blockIdx.y % a.dm.H;
  const int T = a.dm.T;
  const long long row = a.dm.row;
  const long long q0 = (long long)blockIdx.x * 64;
  const int nq = (int)min(64LL, T - q0);
  const bf16* qb = a.q + (long long)b * T * row + (long long)h * D;
  const bf16* kb = a.k + (long long)b * T * row + (long long)h * D;
  const bf16* vb = a.v + (long long)b * T * row + (long long)h * D;
  const bf16* ob = a.d_local + (long long)b * T * row + (long long)h * D;
  const float* lse = a.lse + ((long long)b * a.dm.H + h) * T;
  const float* rd = a.dv_row + ((long long)b * a.dm.H + h) * T;
  for (int idx = tid; idx < 64 * CH; idx += 128) {
    const int r = idx / CH, c = idx % CH;
    const bool ok = r < nq;
    const long long off = (q0 + (ok ? r : 0)) * row + c * 8;
    cp_async16(sQ + swz(r, c * 8, D), qb + off, ok);
    cp_async16(sO + swz(r, c * 8, D), ob + off, ok);
  }
  const long long kstart = win_lo(q0), kend = q0 + nq;
  auto load_kv = [&](long long kk, int buf) {
    for (int idx = tid; idx < BN * CH; idx += 128) {
      const int r = idx / CH, c = idx % CH;
      const bool ok = kk + r < kend;
      const long long off = (ok ? kk + r : kk) * row + c * 8;
      cp_async16(sK + buf * BN * D * 2 + swz(r, c * 8, D), kb + off, ok);
      cp_async16(sV + buf * BN * D * 2 + swz(r, c * 8, D), vb + off, ok);
    }
  };
  load_kv(kstart, 0);
  cp_commit();
  const int g = lane >> 2, c4 = lane & 3;
  const float scale = 1.f / sqrtf((float)D), sl = 1.4426950408889634f * scale;
  float lrow[2], rrow[2];
  long long qrow[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int r = warp * 16 + g + hr * 8;
    qrow[hr] = q0 + r;
    lrow[hr] = r < nq ? lse[q0 + r] * 1.4426950408889634f : 0.f;
    rrow[hr] = r < nq ? rd[q0 + r] : 0.f;
  }
  float dq[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) dq[j][0] = dq[j][1] = dq[j][2] = dq[j][3] = 0.f;
  uint32_t qf[D / 16][4], of[D / 16][4];
  const int nblk = (int)((kend - kstart + BN - 1) / BN);
  for (int blk = 0; blk < nblk; ++blk) {
    const long long kk = kstart + (long long)blk * BN;
    if (blk + 1 < nblk) {
      load_kv(kk + BN, (blk + 1) & 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (blk == 0) {
#pragma unroll
      for (int kt = 0; kt < D / 16; ++kt) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kt * 16 + (lane >> 4) * 8;
        ldsm_x4(sQ + swz(r, c, D), qf[kt][0], qf[kt][1], qf[kt][2], qf[kt][3]);
        ldsm_x4(sO + swz(r, c, D), of[kt][0], of[kt][1], of[kt][2], of[kt][3]);
      }
    }
    const uint32_t kbuf = sK + (blk & 1) * BN * D * 2, vbuf = sV + (blk & 1) * BN * D * 2;
    float s[8][4], dp[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int x = 0; x < 4; ++x) s[j][x] = dp[j][x] = 0.f;
#pragma unroll
    for (int np = 0; np < 4; ++np) {
#pragma unroll
      for (int kt = 0; kt < D / 16; ++kt) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = kt * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(kbuf + swz(r, c, D), b0, b1, b2, b3);
        mma16816(s[2 * np], qf[kt], b0, b1);
        mma16816(s[2 * np + 1], qf[kt], b2, b3);
        ldsm_x4(vbuf + swz(r, c, D), b0, b1, b2, b3);
        mma16816(dp[2 * np], of[kt], b0, b1);
        mma16816(dp[2 * np + 1], of[kt], b2, b3);
      }
    }
    uint32_t da[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float dsv[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        const int hr = x >> 1;
        const long long kp = kk + j * 8 + c4 * 2 + (x & 1);
        const bool ok = kp < kend && kp <= qrow[hr] && qrow[hr] < T;
        const float p = ok ? exp2f(s[j][x] * sl - lrow[hr]) : 0.f;
        dsv[x] = p * (dp[j][x] - rrow[hr]);
      }
      const int kt = j >> 1;
      if ((j & 1) == 0) {
        da[kt][0] = pack_bf16(dsv[0], dsv[1]);
        da[kt][1] = pack_bf16(dsv[2], dsv[3]);
      } else {
        da[kt][2] = pack_bf16(dsv[0], dsv[1]);
        da[kt][3] = pack_bf16(dsv[2], dsv[3]);
      }
    }
#pragma unroll
    for (int kt = 0; kt < 4; ++kt) {
#pragma unroll
      for (int dpi = 0; dpi < D / 16; ++dpi) {
        uint32_t b0, b1, b2, b3;
        const int r = kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dpi * 16 + (lane >> 4) * 8;
        ldsm_x4_t(kbuf + swz(r, c, D), b0, b1, b2, b3);
        mma16816(dq[2 * dpi], da[kt], b0, b1);
        mma16816(dq[2 * dpi + 1], da[kt], b2, b3);
      }
    }
    __syncthreads();
  }
  bf16* dqb = a.dq + (long long)b * T * row + (long long)h * D;
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int r = warp * 16 + g + hr * 8;
    if (r >= nq) continue;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const int e = j * 8 + c4 * 2;
      *reinterpret_cast<__nv_bfloat162*>(dqb + (q0 + r) * row + e) =
          __floats2bfloat162_rn(dq[j][hr * 2] * scale, dq[j][hr * 2 + 1] * scale);
    }
  }
}

// ---------------------------------------------------------------------------
// Selected-read backward: one CTA (NT threads, 16 * MI query rows per warp) per
// (tile part, b, h).
// Fines are visited page by page; for fine s only the queries that selected it
// take part: they are compacted into a row list (ldmatrix gathers their rows by
// address, so nothing is copied) and
//   dA   = bf16(bf16(gn . C_s^T) + gd)                  (tensor cores)
//   dhv += bf16(dA * w_s)   -> per page: dh += bf16(dhv*pw), dpw += bf16(dhv*h)
//   dw_s = sum_q bf16(dA * hv)                          -> dz, d page_z via exp
//   dC_s = A_s^T . gn (bf16 per tile)                   (tensor cores)
// run over ceil(selected/16) row blocks instead of all NQ rows.  dhv lives in
// shared memory (fp32, rows XOR-swizzled by 16-byte chunk); C_{s+1} is fetched
// while fine s is processed (D = 64).  Then the softmax backward of h (-> d raw_q)
// and of the page weights, and the logsumexp backward of the tile's page
// log-partitions (-> dz).
// ---------------------------------------------------------------------------
template <int D>
struct ReadBwdSmem {
  static constexpr int NQ = (D == 64) ? 256 : 128;  // queries per CTA
  static constexpr int NT = (D == 64) ? NQ : 2 * NQ;  // threads per CTA (2 * NQ: fewer registers per thread)
  static constexpr int CB = (D == 64) ? 2 : 1;      // C_s buffers (2: next fine prefetched)
  static size_t bytes(int P, int V, int /*mmax*/) {
    const size_t words = (size_t)(V + 31) / 32;
    return 1024 + 3 * (size_t)NQ * D * 2 + (size_t)CB * D * D * 2 + (size_t)NQ * (D + 2) * 4 + 4 * (size_t)P * D * 4 +
           (size_t)P * D * 2 + (size_t)D * 2 + words * NQ * 4 + NQ * 4 + NQ + (size_t)(NT / 32) * D * 4 +
           (size_t)(V + 8) * 4 * 2 + 64;
  }
};

// float offset of the channel pair (r, d..d+1) in a [rows][D] fp32 tile whose
// 16-byte chunks are XOR-swizzled by r % 8
template <int D>
TAO_DEVI int dhv_off(int r, int d) {
  return r * D + ((((d >> 2) ^ (r & 7))) << 2) + (d & 3);
}

// TC: dA and dC on tcgen05 over the tile's dense query rows (a separate instantiation:
// each kernel carries one contraction path).  The gn, A and C tiles are then laid out
// as 64-channel 128B-swizzled atoms (the layout of a TMA box; at width 64 the same as
// the ldmatrix swizzle of the mma.sync path).  Width 128 (128 queries, two threads per
// query): each thread forms and consumes one 64-channel half of its query's rows.
template <int D, bool TC = false>
__global__ void __launch_bounds__(ReadBwdSmem<D>::NT, 1) read_bwd_kernel(BwdArgs a) {
  using namespace wa;
  constexpr int NQ = ReadBwdSmem<D>::NQ, NT = ReadBwdSmem<D>::NT, CB = ReadBwdSmem<D>::CB, QS = 256 / NQ;
  constexpr int NW = NT / 32, MI = NQ / (16 * NW);  // warp w owns query rows 16*MI*w .. + 16*MI - 1
  // grid (B*H*QS, tiles), tiles heaviest first: the longest CTAs are dispatched first
  const int tile = gridDim.y - 1 - blockIdx.y, bh = blockIdx.x / QS, b = bh / a.dm.H, h = bh % a.dm.H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = tile * 256 + (blockIdx.x % QS) * NQ, nq = max(0, min(NQ, a.dm.T - q0));
  const int V = max(0, tile - 2);
  const long long row = a.dm.row, hoff = (long long)h * D;
  if (V == 0) {
    for (int idx = tid; idx < nq * (D / 8); idx += NT) {
      const int q = idx / (D / 8), c = idx % (D / 8);
      const long long off = ((long long)b * a.dm.T + q0 + q) * row + hoff + c * 8;
      *reinterpret_cast<uint4*>(a.d_raw_q + off) = *reinterpret_cast<const uint4*>(a.d_rq_f + off);
    }
    return;
  }
  const int completed = V / kGroup, pending = V % kGroup, P = completed + (pending > 0);
  const int M = a.mmax, VW = (V + 31) / 32;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // 1024-byte aligned window: the tiles are 128B-swizzled tensor-core operands
  uint8_t* const smem = smem_raw + (((smem_u32(smem_raw) + 1023u) & ~1023u) - smem_u32(smem_raw));
  uint8_t* ptr = smem;
  const uint32_t sH = smem_u32(ptr);  ptr += NQ * D * 2;
  const uint32_t sG = smem_u32(ptr);  ptr += NQ * D * 2;
  const uint32_t sA = smem_u32(ptr);  ptr += NQ * D * 2;   // A_s rows of the selecting queries, compacted
  const uint32_t sC = smem_u32(ptr);  ptr += CB * D * D * 2;
  uint8_t* hB = smem;
  uint8_t* aB = smem + 2 * NQ * D * 2;
  float* dhvS = reinterpret_cast<float*>(ptr);  ptr += (size_t)NQ * (D + 2) * 4;  // dhv of the current page
  // dhv cell of (row, channel pair): swizzled rows for the fragment accesses of the
  // mma.sync path; padded rows (D + 2 floats) for the row-per-thread accesses of the
  // tcgen05 path (two 64-bit wavefronts per warp)
  auto dho = [](int r, int d) -> int { return TC ? r * (D + 2) + d : dhv_off<D>(r, d); };
  // byte offset of chunk c8 (8 channels) of row r in an operand tile of `rows` rows
  auto opnd = [](int r, int c8, int rows) -> uint32_t {
    if constexpr (TC)
      return (uint32_t)((c8 >> 3) * rows * 128 + r * 128 + (((c8 & 7) ^ (r & 7)) << 4));
    else
      return (uint32_t)swz(r, c8 * 8, D);
  };
  float* pwS = reinterpret_cast<float*>(ptr);   ptr += (size_t)P * D * 4;
  float* pzS = reinterpret_cast<float*>(ptr);   ptr += (size_t)P * D * 4;
  float* dpwS = reinterpret_cast<float*>(ptr);  ptr += (size_t)P * D * 4;
  float* dpzS = reinterpret_cast<float*>(ptr);  ptr += (size_t)P * D * 4;
  bf16* pw2S = reinterpret_cast<bf16*>(ptr);    ptr += (size_t)P * D * 2;  // page weights as bf16
  bf16* wS = reinterpret_cast<bf16*>(ptr);      ptr += D * 2;              // w_s of the current fine
  uint32_t* selB = reinterpret_cast<uint32_t*>(ptr); ptr += (size_t)VW * NQ * 4;  // [word][query] bits
  float* gdS = reinterpret_cast<float*>(ptr);   ptr += NQ * 4;
  uint8_t* rowS = ptr;                          ptr += NQ;   // compacted row -> query
  float* dwS = reinterpret_cast<float*>(ptr);   ptr += (size_t)NW * D * 4;  // per-warp dw partials
  int* useS = reinterpret_cast<int*>(ptr);
  int* list = useS + V;
  __shared__ int cntS[NW];
  __shared__ unsigned balS[NW];   // the selecting queries of each warp for the current fine

  // ---- tables (as in the forward)
  const bf16* pzb = a.pzpre + ((long long)b * a.dm.H + h) * a.pages * kGroup * D;
  for (int idx = tid; idx < P * D; idx += NT) {
    const int pg = idx / D, d = idx % D;
    const int n = (pg < completed) ? kGroup : pending;
    pzS[idx] = bf(__ldg(pzb + ((long long)pg * kGroup + (n - 1)) * D + d));
    dpwS[idx] = 0.f;
    dpzS[idx] = 0.f;
  }
  for (int i = tid; i < V; i += NT) useS[i] = 0;
  for (int i = tid; i < NQ * (D + 2); i += NT) dhvS[i] = 0.f;
  __syncthreads();
  for (int d = tid; d < D; d += NT) {
    float mx = -INFINITY;
    for (int pg = 0; pg < P; ++pg) mx = fmaxf(mx, pzS[pg * D + d]);
    float sum = 0.f;
    for (int pg = 0; pg < P; ++pg) sum += expf(pzS[pg * D + d] - mx);
    for (int pg = 0; pg < P; ++pg) {
      pwS[pg * D + d] = rb(__fdiv_rn(expf(pzS[pg * D + d] - mx), sum));
      pw2S[pg * D + d] = tobf(pwS[pg * D + d]);
    }
  }
  const bf16* zb = a.z + ((long long)b * a.dm.H + h) * a.dm.S * D;
  // ---- per query: h (swizzled); gn (swizzled), gd and the selection bits (with
  // 2 * NQ threads the second NQ load these while the first NQ compute h)
  const int q = tid % NQ;
  const bool first = tid < NQ;
  const bool live = q < nq;
  const long long qbase = ((long long)b * a.dm.T + q0 + q) * row + hoff;
  // every global read of this kernel is of data it does not write: read-only
  // loads (ld.global.nc), issued before the shared-memory stores that use them
  if (first) {
    uint4 rv[D / 8];
    if (live) {
      const uint4* rq = reinterpret_cast<const uint4*>(a.raw_q + qbase);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) rv[c] = __ldg(rq + c);
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        float f[8];
        unpack8(rv[c], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) mx = fmaxf(mx, f[e]);
      }
      // exponentials kept from the sum for the output when they fit in registers (width 64)
      constexpr int KEEP = (D == 64) ? D : 1;
      float ex[KEEP];
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        float f[8];
        unpack8(rv[c], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float x = expf(f[e] - mx);
          if (D == 64) ex[(c * 8 + e) % KEEP] = x;
          sum += x;
        }
      }
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        float f[8];
        unpack8(rv[c], f);
        __nv_bfloat162 o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x0 = (D == 64) ? ex[(c * 8 + 2 * e) % KEEP] : expf(f[2 * e] - mx);
          const float x1 = (D == 64) ? ex[(c * 8 + 2 * e + 1) % KEEP] : expf(f[2 * e + 1] - mx);
          o[e] = __floats2bfloat162_rn(__fdiv_rn(x0, sum), __fdiv_rn(x1, sum));
        }
        rv[c] = *reinterpret_cast<uint4*>(o);
      }
    } else {
#pragma unroll
      for (int c = 0; c < D / 8; ++c) rv[c] = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int c = 0; c < D / 8; ++c) *reinterpret_cast<uint4*>(hB + swz(q, c * 8, D)) = rv[c];
  }
  if (NT == NQ || !first) {
    for (int w = 0; w < VW; ++w) selB[w * NQ + q] = 0u;
    uint4 gv[D / 8];
    float gdv = 0.f;
    if (live) {
      const uint4* gq = reinterpret_cast<const uint4*>(a.gn + qbase);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) gv[c] = __ldg(gq + c);
      gdv = __ldg(a.gd + ((long long)b * a.dm.T + q0 + q) * a.dm.H + h);
    } else {
#pragma unroll
      for (int c = 0; c < D / 8; ++c) gv[c] = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int c = 0; c < D / 8; ++c) *reinterpret_cast<uint4*>(hB + NQ * D * 2 + opnd(q, c, NQ)) = gv[c];
    gdS[q] = gdv;
    if (live) {
      const short* so = reinterpret_cast<const short*>(a.sel) + (((long long)b * a.dm.T + q0 + q) * a.dm.H + h) * a.mmax;
      for (int m0 = 0; m0 < M; m0 += 8) {
        int sv[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) sv[m] = (m0 + m < M) ? (int)__ldg(so + m0 + m) : -1;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int s = sv[m];
          if (s >= 0 && s < V) {
            selB[(s >> 5) * NQ + q] |= 1u << (s & 31);
            useS[s] = 1;
          }
        }
      }
    }
  }
  __syncthreads();
  __shared__ int nused;
  if (tid == 0) {
    int n = 0;
    for (int sf = 0; sf < V; ++sf)
      if (useS[sf]) list[n++] = sf;
    nused = n;
  }
  __syncthreads();
  if (QS == 1 && nused < V) {
    // dC partials of fines no query of this tile selected are zero (the reduction
    // reads every pair; the buffer is not cleared beforehand)
    for (int sf = 0; sf < V; ++sf) {
      if (useS[sf]) continue;
      const long long pair = (long long)(tile - 3) * (tile - 2) / 2 + sf;
      bf16* dcb = a.dcp + (((long long)b * a.dm.H + h) * a.npairs + pair) * (long long)D * D;
      for (int idx = tid * 8; idx < D * D; idx += NT * 8) *reinterpret_cast<uint4*>(dcb + idx) = make_uint4(0, 0, 0, 0);
    }
  }

  constexpr int NTL = D / 8;
  const int g = lane >> 2, c4 = lane & 3;
  float dh[MI][NTL][4];  // rows 16 * (MI * warp + mi) + g (+ 8)
#pragma unroll
  for (int mi = 0; mi < MI; ++mi)
#pragma unroll
    for (int j = 0; j < NTL; ++j)
#pragma unroll
      for (int x = 0; x < 4; ++x) dh[mi][j][x] = 0.f;
  const bf16* cb = a.C + ((long long)b * a.dm.H + h) * a.dm.S * (long long)D * D;
  int cur_page = -1;
  const uint32_t* pw2 = reinterpret_cast<const uint32_t*>(pw2S);
  const uint32_t* w2 = reinterpret_cast<const uint32_t*>(wS);
  auto pair_at = [&](const uint8_t* base, int r, int d) -> uint32_t {  // bf16 pair (d even) of row r
    return *reinterpret_cast<const uint32_t*>(base + swz(r, d, D));
  };
  auto fetch_c = [&](int sf, int buf) {
    for (int idx = tid; idx < D * D / 8; idx += NT) {
      const int r = idx / (D / 8), c = idx % (D / 8);
      cp_async16(sC + buf * D * D * 2 + opnd(r, c, D), cb + (long long)sf * D * D + r * D + c * 8, true);
    }
  };
  auto flush_page = [&](int pg) {
    // dh += bf16(bf16(dhv)*pw[pg]) ; dpw[pg] += sum_q bf16(bf16(dhv)*h) ; dhv = 0
    float part[NTL][2];
#pragma unroll
    for (int j = 0; j < NTL; ++j) part[j][0] = part[j][1] = 0.f;
#pragma unroll
    for (int rr = 0; rr < 2 * MI; ++rr) {
      const int mi = rr >> 1, xp = rr & 1;
      const int r = (warp * MI + mi) * 16 + g + xp * 8;
      float2 acc[NTL];
      uint32_t hp[NTL];
#pragma unroll
      for (int j = 0; j < NTL; ++j) {  // all loads before the stores that clear the cells
        const int d = j * 8 + c4 * 2;
        acc[j] = *reinterpret_cast<const float2*>(dhvS + dho(r, d));
        hp[j] = pair_at(hB, r, d);
      }
#pragma unroll
      for (int j = 0; j < NTL; ++j)
        *reinterpret_cast<float2*>(dhvS + dho(r, j * 8 + c4 * 2)) = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < NTL; ++j) {
        const int d = j * 8 + c4 * 2;
        const uint32_t v2 = wa::pack_bf16(acc[j].x, acc[j].y);
        const uint32_t pp = hmul2u(v2, pw2[(pg * D + d) / 2]);
        const uint32_t hh = hmul2u(v2, hp[j]);
        dh[mi][j][2 * xp] += lo_f(pp);
        dh[mi][j][2 * xp + 1] += hi_f(pp);
        part[j][0] += lo_f(hh);
        part[j][1] += hi_f(hh);
      }
    }
#pragma unroll
    for (int j = 0; j < NTL; ++j)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        float v = part[j][x];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        if (g == 0) atomicAdd(&dpwS[pg * D + j * 8 + c4 * 2 + x], v);
      }
  };
  const int nu = nused;
  float znext = (nu > 0 && tid < D) ? bf(__ldg(zb + (long long)list[0] * D + tid)) : 0.f;  // z of the next fine
  if (CB == 2 && nu > 0) {
    fetch_c(list[0], 0);
    cp_commit();
  }
  // tcgen05 path: TMEM columns 0-127 hold dA of query rows 0-127 / 128-255, columns
  // 128-191 dC_s (lanes 0-63 = rows d); one mbarrier for the MMA group of a fine
  __shared__ __align__(8) uint64_t tbar;
  __shared__ uint32_t tslot;
  __shared__ int tok;
  uint32_t tbase = 0, tphase = 0;
  bool tc_ok = true;
  if constexpr (TC) {
    if (warp == 0) {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tslot)),
                   "r"(256));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
      mbar_init(&tbar, 1);
      fence_mbar_init();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    tbase = tslot;
  }
  for (int i = 0; i < nu; ++i) {
    const int sf = list[i], pg = sf / kGroup;
    const int buf = (CB == 2) ? (i & 1) : 0;
    // ---- phase 1: page change, w_s, C prefetch, selection ballot
    if (pg != cur_page) {
      if (cur_page >= 0) flush_page(cur_page);
      cur_page = pg;
    }
    if (tid < D) {  // D <= NT: one channel per thread
      const float zc = znext;
      if (i + 1 < nu) znext = bf(__ldg(zb + (long long)list[i + 1] * D + tid));
      wS[tid] = tobf(expf(rb(__fsub_rn(zc, pzS[pg * D + tid]))));
    }
    if (CB == 2) {
      if (i + 1 < nu) fetch_c(list[i + 1], buf ^ 1);
    } else {
      fetch_c(sf, 0);
    }
    cp_commit();
    const bool sel = first && ((selB[(sf >> 5) * NQ + q] >> (sf & 31)) & 1u);
    const unsigned ballot = __ballot_sync(0xffffffffu, sel);
    if (lane == 0) {
      cntS[warp] = __popc(ballot);
      balS[warp] = ballot;
    }
    __syncthreads();
    if constexpr (TC) {
      // ---- phase 2': A_s over the dense query rows (row q = query q, zero unless it
      // selected fine sf), K-major 128B-swizzled like the h and gn tiles
      // this thread's channels: all 64 at width 64, half tid / NQ of 128 at width 128
      constexpr int DH = 64;
      const int dch = (D == 64) ? 0 : (tid / NQ) * 64;
      const bool selq = live && ((selB[(sf >> 5) * NQ + q] >> (sf & 31)) & 1u);
      uint32_t hvw[DH / 2];  // hv = bf16(h * pw[pg]) of this query's channels, kept for the dA epilogue
      {
#pragma unroll
        for (int cc = 0; cc < DH / 8; ++cc) {
          const int c = dch / 8 + cc;
          uint4 o = make_uint4(0, 0, 0, 0);
          if (selq) {
            const uint4 hc = *reinterpret_cast<const uint4*>(hB + swz(q, c * 8, D));
            const uint4 pc = *reinterpret_cast<const uint4*>(pw2 + (pg * D + c * 8) / 2);
            const uint4 wc = *reinterpret_cast<const uint4*>(w2 + c * 4);
            hvw[cc * 4] = hmul2u(hc.x, pc.x);
            hvw[cc * 4 + 1] = hmul2u(hc.y, pc.y);
            hvw[cc * 4 + 2] = hmul2u(hc.z, pc.z);
            hvw[cc * 4 + 3] = hmul2u(hc.w, pc.w);
            o = make_uint4(hmul2u(hvw[cc * 4], wc.x), hmul2u(hvw[cc * 4 + 1], wc.y), hmul2u(hvw[cc * 4 + 2], wc.z),
                           hmul2u(hvw[cc * 4 + 3], wc.w));
          } else {
            hvw[cc * 4] = hvw[cc * 4 + 1] = hvw[cc * 4 + 2] = hvw[cc * 4 + 3] = 0u;
          }
          *reinterpret_cast<uint4*>(aB + opnd(q, c, NQ)) = o;
        }
      }
      if (CB == 2) cp_wait<1>();
      else cp_wait<0>();
      tc::fence_proxy_async();
      tc::fence_before();
      __syncthreads();
      // ---- phase 3': dA = gn . C_s^T (M = 128 x 2 query halves, N = 64, K = 64; gn and
      // C_s K-major) and dC_s = A_s^T . gn (M = 128 over d, K = 256 queries, both read
      // MN-major; rows 64-127 of that instruction take the next 32 KB of shared memory
      // as a stand-in and land in TMEM lanes nobody reads); bounded wait
      const uint32_t cbuf = sC + buf * D * D * 2;
      if (tid == 0) {
        tc::fence_after();
        if (tc_ok) {
          constexpr uint32_t IA = tc::idesc_bf16(128, D, 0, 0), IC = tc::idesc_bf16(128, D, 1, 1);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {  // K = e in 64-channel atoms: gn atoms NQ rows, C atoms D rows
            const uint32_t ga = sG + (k >> 2) * NQ * 128 + (k & 3) * 32, ca = cbuf + (k >> 2) * D * 128 + (k & 3) * 32;
            tc::mma(tbase, tc::sdesc(ga, 16, 1024), tc::sdesc(ca, 16, 1024), IA, k > 0 ? 1u : 0u);
            if constexpr (NQ == 256)   // query rows 128-255
              tc::mma(tbase + 64, tc::sdesc(ga + 16384, 16, 1024), tc::sdesc(ca, 16, 1024), IA, k > 0 ? 1u : 0u);
          }
#pragma unroll
          for (int k = 0; k < NQ / 16; ++k)
            tc::mma(tbase + 128, tc::sdesc(sA + k * 2048, NQ * 128, 1024), tc::sdesc(sG + k * 2048, NQ * 128, 1024),
                    IC, k > 0 ? 1u : 0u);
          tc::commit(&tbar);
          tok = mbar_wait(&tbar, tphase, a.err) ? 1 : 0;
        } else {
          tok = 0;
        }
      }
      __syncthreads();
      tc::fence_after();
      const bool okf = tok != 0;
      if (tc_ok && !okf) {
        tc_ok = false;   // the group stays in flight: drained (bounded) before the TMEM is freed
      } else if (okf) {
        tphase ^= 1u;
      }
      // dC_s of this tile: TMEM lanes 0-(D-1) (warps 0 .. D/32-1), the reference's per-tile bf16
      const long long pair = (long long)(tile - 3) * (tile - 2) / 2 + sf;
      bf16* dcb = a.dcp + (((long long)b * a.dm.H + h) * a.npairs + pair) * (long long)D * D;
      // width 64: warps 0-1, all 64 columns; width 128: every warp, lanes 32 (w % 4) and
      // columns 64 (w / 4) .. + 63 (the adds of the two half tiles spread over 8 warps)
      constexpr int DCW = 64;  // columns per warp
      const int drow = (D == 64) ? tid : (warp & 3) * 32 + lane;
      const int dcol0 = (D == 64) ? 0 : (warp >> 2) * 64;
      if (D == 128 || warp < D / 32) {
#pragma unroll
        for (int cc = 0; cc < DCW; cc += 32) {
          const int c0 = dcol0 + cc;
          float v[32];
          if (okf) {
            tc::tmem_ld32(tbase + 128 + ((uint32_t)((warp & 3) * 32) << 16) + c0, v);
          } else {
#pragma unroll
            for (int x = 0; x < 32; ++x) v[x] = 0.f;
          }
          if constexpr (QS == 1) {
#pragma unroll
            for (int x = 0; x < 32; x += 8) {
              uint4 o;
              o.x = wa::pack_bf16(v[x], v[x + 1]);
              o.y = wa::pack_bf16(v[x + 2], v[x + 3]);
              o.z = wa::pack_bf16(v[x + 4], v[x + 5]);
              o.w = wa::pack_bf16(v[x + 6], v[x + 7]);
              *reinterpret_cast<uint4*>(dcb + (long long)drow * D + c0 + x) = o;
            }
          } else {  // half tiles: both halves add into the zero-initialised partial
#pragma unroll
            for (int x = 0; x < 32; x += 8)  // eight bf16 adds per vector reduction
              asm volatile("red.global.add.noftz.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(
                               dcb + (long long)drow * D + c0 + x),
                           "r"(wa::pack_bf16(v[x], v[x + 1])), "r"(wa::pack_bf16(v[x + 2], v[x + 3])),
                           "r"(wa::pack_bf16(v[x + 4], v[x + 5])), "r"(wa::pack_bf16(v[x + 6], v[x + 7]))
                           : "memory");
          }
        }
      }
      // dA of this thread's query row (TMEM lane q % 128 of accumulator q / 128):
      // dA = bf16(bf16(gn . C^T) + gd); dhv += bf16(dA * w_s); the products
      // bf16(dA * hv) go channel-major ([d][query], conflict-free) to the (now free) A
      // tile for the column sums of dw_s
      {
        const float gdv = gdS[q];
        bf16* phT = reinterpret_cast<bf16*>(aB) + q;
#pragma unroll
        for (int c0 = 0; c0 < DH; c0 += 32) {
          float v[32];
          if (okf) {  // accumulator of this query half (width 64) or this channel half (width 128)
            tc::tmem_ld32(tbase + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(tid / 128) * 64 + c0, v);
          } else {
#pragma unroll
            for (int x = 0; x < 32; ++x) v[x] = 0.f;
          }
          if (selq) {
#pragma unroll
            for (int x = 0; x < 32; x += 2) {
              const int d = dch + c0 + x;
              const uint32_t dav = wa::pack_bf16(__fadd_rn(rb(v[x]), gdv), __fadd_rn(rb(v[x + 1]), gdv));
              const uint32_t pw_ = hmul2u(dav, w2[d / 2]);
              const uint32_t ph = hmul2u(dav, hvw[(c0 + x) / 2]);
              float2* cell = reinterpret_cast<float2*>(dhvS + dho(q, d));
              float2 acc = *cell;
              acc.x += lo_f(pw_);
              acc.y += hi_f(pw_);
              *cell = acc;
              phT[(long long)d * NQ] = __ushort_as_bfloat16((unsigned short)(ph & 0xffffu));
              phT[(long long)(d + 1) * NQ] = __ushort_as_bfloat16((unsigned short)(ph >> 16));
            }
          }
        }
      }
      __syncthreads();
      // dw_s partials: the NW groups of 32 queries (one warp's), summed over the groups in
      // phase 4; only the selecting queries' products are read (the others hold A values)
      constexpr int NPART = NQ / 32;  // groups of 32 queries: the first NQ threads' warps
      for (int idx = tid; idx < NPART * D; idx += NT) {
        const int part = idx % NPART, d = idx / NPART;
        const unsigned m = balS[part];
        const uint4* col = reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(aB) + (long long)d * NQ +
                                                          part * 32);
        float sum = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float f[8];
          unpack8(col[c], f);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if ((m >> (c * 8 + e)) & 1u) sum += f[e];
        }
        dwS[part * D + d] = sum;
      }
    } else {
    // ---- phase 2: compacted row list and A_s = bf16(bf16(h * pw) * w_s) of the selecting queries
    int before = 0, ns = 0;
#pragma unroll
    for (int w = 0; w < NQ / 32; ++w) {  // only the first NQ threads vote
      const int c = cntS[w];
      before += (w < warp) ? c : 0;
      ns += c;
    }
    const int npad = (ns + 15) & ~15;
    if (sel) {
      const int pos = before + __popc(ballot & ((1u << lane) - 1u));
      rowS[pos] = (uint8_t)q;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        const uint4 hc = *reinterpret_cast<const uint4*>(hB + swz(q, c * 8, D));
        const uint4 pc = *reinterpret_cast<const uint4*>(pw2 + (pg * D + c * 8) / 2);
        const uint4 wc = *reinterpret_cast<const uint4*>(w2 + c * 4);
        *reinterpret_cast<uint4*>(aB + swz(pos, c * 8, D)) =
            make_uint4(hmul2u(hmul2u(hc.x, pc.x), wc.x), hmul2u(hmul2u(hc.y, pc.y), wc.y),
                       hmul2u(hmul2u(hc.z, pc.z), wc.z), hmul2u(hmul2u(hc.w, pc.w), wc.w));
      }
    }
    if (tid >= ns && tid < npad) {  // padding rows: A = 0, any valid query row for gn
      rowS[tid] = 0;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) *reinterpret_cast<uint4*>(aB + swz(tid, c * 8, D)) = make_uint4(0, 0, 0, 0);
    }
    if (CB == 2) cp_wait<1>();
    else cp_wait<0>();
    __syncthreads();
    // ---- phase 3a: dA = gn . C_s^T over the compacted rows, 16 per block; elementwise
    const uint32_t cbuf = sC + buf * D * D * 2;
    uint32_t wv[NTL], pv[NTL];  // w_s and pw[pg] pairs of this lane's channels
#pragma unroll
    for (int j = 0; j < NTL; ++j) {
      wv[j] = w2[(j * 8 + c4 * 2) / 2];
      pv[j] = pw2[(pg * D + j * 8 + c4 * 2) / 2];
    }
    float wpart[NTL][2];
#pragma unroll
    for (int j = 0; j < NTL; ++j) wpart[j][0] = wpart[j][1] = 0.f;
    for (int mt = warp; mt < npad / 16; mt += NW) {
      float da[NTL][4];
#pragma unroll
      for (int j = 0; j < NTL; ++j) da[j][0] = da[j][1] = da[j][2] = da[j][3] = 0.f;
      const int arow = rowS[mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8];
#pragma unroll
      for (int kt = 0; kt < D / 16; ++kt) {
        uint32_t af[4];
        ldsm_x4(sG + swz(arow, kt * 16 + (lane >> 4) * 8, D), af[0], af[1], af[2], af[3]);
#pragma unroll
        for (int np = 0; np < D / 16; ++np) {
          uint32_t b0, b1, b2, b3;
          const int r = np * 16 + (lane & 7) + (lane >> 4) * 8;
          const int c = kt * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(cbuf + swz(r, c, D), b0, b1, b2, b3);
          mma16816(da[2 * np], af, b0, b1);
          mma16816(da[2 * np + 1], af, b2, b3);
        }
      }
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int ci = mt * 16 + g + hr * 8;
        if (ci >= ns) continue;
        const int r = rowS[ci];
        const float gdv = gdS[r];
        float2 acc[NTL];
        uint32_t hp[NTL];
#pragma unroll
        for (int j = 0; j < NTL; ++j) {  // all loads before the stores
          const int d = j * 8 + c4 * 2;
          acc[j] = *reinterpret_cast<const float2*>(dhvS + dho(r, d));
          hp[j] = pair_at(hB, r, d);
        }
#pragma unroll
        for (int j = 0; j < NTL; ++j) {
          // dA = bf16(bf16(gn . C^T) + gd), a pair of channels
          const uint32_t dav = wa::pack_bf16(__fadd_rn(rb(da[j][2 * hr]), gdv), __fadd_rn(rb(da[j][2 * hr + 1]), gdv));
          const uint32_t pw_ = hmul2u(dav, wv[j]);
          const uint32_t ph = hmul2u(dav, hmul2u(hp[j], pv[j]));  // hv = bf16(h * pw)
          acc[j].x += lo_f(pw_);
          acc[j].y += hi_f(pw_);
          wpart[j][0] += lo_f(ph);
          wpart[j][1] += hi_f(ph);
        }
#pragma unroll
        for (int j = 0; j < NTL; ++j) *reinterpret_cast<float2*>(dhvS + dho(r, j * 8 + c4 * 2)) = acc[j];
      }
    }
#pragma unroll
    for (int j = 0; j < NTL; ++j)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        float v = wpart[j][x];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        if (g == 0) dwS[warp * D + j * 8 + c4 * 2 + x] = v;  // summed over warps after the barrier
      }
    // ---- phase 3b: dC_s = A_s^T . gn over the compacted rows : output [d][e];
    // warps tile (m-tiles of d rows) x (n ranges)
    {
      constexpr int MTILES = D / 16;
      constexpr int WPM = NW >= MTILES ? NW / MTILES : 1;   // warps per m-tile
      constexpr int MPW = NW >= MTILES ? 1 : MTILES / NW;   // m-tiles per warp
      constexpr int NPW = (D / 8) / WPM;                    // n-tiles per warp
      // this tile's bf16 partial of dC_s (the reference rounds dC per tile as well)
      const long long pair = (long long)(tile - 3) * (tile - 2) / 2 + sf;
      bf16* dcb = a.dcp + (((long long)b * a.dm.H + h) * a.npairs + pair) * (long long)D * D;
      for (int mm = 0; mm < MPW; ++mm) {
        const int mt = (NW >= MTILES) ? warp / WPM : warp * MPW + mm;
        const int n0 = (NW >= MTILES) ? (warp % WPM) * NPW : 0;
        float dc[NPW][4];
#pragma unroll
        for (int j = 0; j < NPW; ++j) dc[j][0] = dc[j][1] = dc[j][2] = dc[j][3] = 0.f;
        for (int kt = 0; kt < npad / 16; ++kt) {
          uint32_t af[4];
          const int r = kt * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
          const int c = mt * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4_t(sA + swz(r, c, D), af[0], af[1], af[2], af[3]);
          const int grow = rowS[kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8];
#pragma unroll
          for (int np = 0; np < NPW / 2; ++np) {
            uint32_t b0, b1, b2, b3;
            const int cc = (n0 + 2 * np) * 8 + (lane >> 4) * 8;
            ldsm_x4_t(sG + swz(grow, cc, D), b0, b1, b2, b3);
            mma16816(dc[2 * np], af, b0, b1);
            mma16816(dc[2 * np + 1], af, b2, b3);
          }
        }
#pragma unroll
        for (int j = 0; j < NPW; ++j) {
          const int e = (n0 + j) * 8 + c4 * 2;
          const int d0 = mt * 16 + g;
          if (QS == 1) {
            *reinterpret_cast<__nv_bfloat162*>(dcb + (long long)d0 * D + e) = __floats2bfloat162_rn(dc[j][0], dc[j][1]);
            *reinterpret_cast<__nv_bfloat162*>(dcb + (long long)(d0 + 8) * D + e) = __floats2bfloat162_rn(dc[j][2], dc[j][3]);
          } else {  // half tiles: both halves add into the zero-initialised partial
            atomicAdd(reinterpret_cast<__nv_bfloat162*>(dcb + (long long)d0 * D + e), __floats2bfloat162_rn(dc[j][0], dc[j][1]));
            atomicAdd(reinterpret_cast<__nv_bfloat162*>(dcb + (long long)(d0 + 8) * D + e), __floats2bfloat162_rn(dc[j][2], dc[j][3]));
          }
        }
      }
    }
    }  // the mma.sync path
    __syncthreads();
    // ---- phase 4: dw_s -> d(z - pz) = bf16(bf16(dw) * w) : dz[s] += ., d page_z[pg] -= .
    for (int d = tid; d < D; d += NT) {
      float dw = 0.f;
      constexpr int NDW = TC ? NQ / 32 : NW;  // dw partial groups written in phase 3 (3')
#pragma unroll
      for (int w = 0; w < NDW; ++w) dw += dwS[w * D + d];
      const float ddiff = rb(__fmul_rn(rb(dw), bf(wS[d])));
      atomicAdd(a.dz + (((long long)b * a.dm.H + h) * a.dm.S + sf) * D + d, ddiff);
      dpzS[pg * D + d] -= ddiff;
    }
  }
  if constexpr (TC) {
    if (!tc_ok && tid == 0) mbar_wait(&tbar, tphase, a.err);   // the group still in flight
    tc::fence_before();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(256));
  }
  if (cur_page >= 0) flush_page(cur_page);
  __syncthreads();
  // ---- softmax backward of h -> d raw_q = bf16(fusion part + this part)
#pragma unroll
  for (int rr = 0; rr < 2 * MI; ++rr) {
    const int mi = rr >> 1, hr = rr & 1;
    const int r = (warp * MI + mi) * 16 + g + hr * 8;
    // h of this row as channel pairs, bf16(dh) with one packed conversion per pair
    uint32_t hp[NTL];
    float dr[NTL][2];
#pragma unroll
    for (int j = 0; j < NTL; ++j) {
      hp[j] = pair_at(hB, r, j * 8 + c4 * 2);
      dr[j][0] = dh[mi][j][hr * 2];
      dr[j][1] = dh[mi][j][hr * 2 + 1];
      rb2(dr[j][0], dr[j][1]);
    }
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NTL; ++j) {
      dot += lo_f(hp[j]) * dr[j][0];
      dot += hi_f(hp[j]) * dr[j][1];
    }
    dot += __shfl_xor_sync(0xffffffffu, dot, 1);
    dot += __shfl_xor_sync(0xffffffffu, dot, 2);
    if (r >= nq) continue;
    const long long base = ((long long)b * a.dm.T + q0 + r) * row + hoff;
    __nv_bfloat162 fpart[NTL];
#pragma unroll
    for (int j = 0; j < NTL; ++j)
      fpart[j] = __ldg(reinterpret_cast<const __nv_bfloat162*>(a.d_rq_f + base + j * 8 + c4 * 2));
#pragma unroll
    for (int j = 0; j < NTL; ++j) {
      const float2 fp = __bfloat1622float2(fpart[j]);
      float x0 = lo_f(hp[j]) * (dr[j][0] - dot), x1 = hi_f(hp[j]) * (dr[j][1] - dot);
      rb2(x0, x1);  // d raw_q of this part, then bf16(fusion part + this part)
      *reinterpret_cast<uint32_t*>(a.d_raw_q + base + j * 8 + c4 * 2) = wa::pack_bf16(fp.x + x0, fp.y + x1);
    }
  }
  // ---- page weights softmax backward, then logsumexp backward of page_z -> dz
  for (int d = tid; d < D; d += NT) {
    float dot = 0.f;
    for (int pg = 0; pg < P; ++pg) dot += pwS[pg * D + d] * rb(dpwS[pg * D + d]);
    for (int pg = 0; pg < P; ++pg)
      dpzS[pg * D + d] += rb(pwS[pg * D + d] * (rb(dpwS[pg * D + d]) - dot));
  }
  __syncthreads();
#pragma unroll 4
  for (int idx = tid; idx < V * D / 2; idx += NT) {  // channel pairs: packed rounding, one 8-byte atomic
    const int sf = idx / (D / 2), d = (idx % (D / 2)) * 2, pg = sf / kGroup;
    const float2 zz = __bfloat1622float2(__ldg(reinterpret_cast<const __nv_bfloat162*>(zb + (long long)sf * D + d)));
    float w0 = __fsub_rn(zz.x, pzS[pg * D + d]), w1 = __fsub_rn(zz.y, pzS[pg * D + d + 1]);
    rb2(w0, w1);
    w0 = expf(w0);
    w1 = expf(w1);
    rb2(w0, w1);
    float g0 = dpzS[pg * D + d], g1 = dpzS[pg * D + d + 1];
    rb2(g0, g1);
    g0 = __fmul_rn(g0, w0);
    g1 = __fmul_rn(g1, w1);
    rb2(g0, g1);
    atomicAdd(reinterpret_cast<float2*>(a.dz + (((long long)b * a.dm.H + h) * a.dm.S + sf) * D + d),
              make_float2(g0, g1));
  }
}

// ---------------------------------------------------------------------------
// dC[b][h][s] = sum over the tiles t >= s + 3 of their bf16 partials (fp32 sum).
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) dc_reduce_kernel(BwdArgs a, int tiles) {
  const int s = blockIdx.x % a.dm.S, bh = blockIdx.x / a.dm.S;
  const bf16* base = a.dcp + (long long)bh * a.npairs * D * D;
  float* out = a.dC + ((long long)bh * a.dm.S + s) * D * D;
  for (int x = threadIdx.x * 8; x < D * D; x += 256 * 8) {  // 8 elements (16 bytes) per load
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int t = s + 3; t < tiles; ++t) {
      const long long pair = (long long)(t - 3) * (t - 2) / 2 + s;
      float v[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(base + pair * D * D + x)), v);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += v[e];
    }
    *reinterpret_cast<float4*>(out + x) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(out + x + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

// ---------------------------------------------------------------------------
// Writer backward: one CTA (256 threads) per (b, h, block s).
//   p = bf16(e / Z), e = bf16(exp(bf16(k - m))) are formed once into shared memory
//   (p over the raw keys, e in its own tile for width 64), then
//   dv += P . dC and dprob = V . dC^T run as two separate tensor-core passes so the
//   width-64 kernel fits two CTAs per SM.
// ---------------------------------------------------------------------------
template <int D>
struct WriterBwdSmem {
  static constexpr bool kStoreE = (D == 64);
  static constexpr size_t bytes() {
    return (size_t)(kStoreE ? 3 : 2) * 256 * D * 2 + (size_t)D * D * 2 + (size_t)256 * (D / 32) * 4 +
           (size_t)6 * D * 4;
  }
};

template <int D>
__global__ void __launch_bounds__(256, (D == 64) ? 2 : 1) writer_bwd_kernel(BwdArgs a) {
  using namespace wa;
  constexpr int NT = 256, CH = D / 8, NTL = D / 8, TW = D / 32;
  constexpr bool kStoreE = WriterBwdSmem<D>::kStoreE;
  const int s = blockIdx.x % a.dm.S, h = (blockIdx.x / a.dm.S) % a.dm.H, b = blockIdx.x / (a.dm.S * a.dm.H);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ptr = smem;
  const uint32_t sK = smem_u32(ptr);   // raw keys, then probabilities p
  uint8_t* kB = ptr;                   ptr += NT * D * 2;
  const uint32_t sV = smem_u32(ptr);   ptr += NT * D * 2;
  uint8_t* eB = ptr;                   ptr += kStoreE ? NT * D * 2 : 0;
  const uint32_t sD = smem_u32(ptr);
  uint8_t* dB = ptr;                   ptr += D * D * 2;
  uint32_t* tieS = reinterpret_cast<uint32_t*>(ptr);  ptr += NT * TW * 4;   // k == max, one bit per (t, d)
  float* mx = reinterpret_cast<float*>(ptr);
  float* zp = mx + D;
  float* dzS = zp + D;
  float* dZp = dzS + D;   // sum_t of the partition term from prob
  float* dmS = dZp + D;   // sum_t d_x
  float* dZ = dmS + D;
  const long long row = a.dm.row;
  const long long tok0 = (long long)b * a.dm.T + (long long)s * NT;
  const bf16* kb = a.raw_k + tok0 * row + (long long)h * D;
  const bf16* vb = a.v + tok0 * row + (long long)h * D;
  const float* dcb = a.dC + (((long long)b * a.dm.H + h) * a.dm.S + s) * (long long)D * D;
  for (int idx = tid; idx < NT * CH; idx += 256) {
    const int r = idx / CH, c = idx % CH;
    cp_async16(sK + swz(r, c * 8, D), kb + (long long)r * row + c * 8, true);
    cp_async16(sV + swz(r, c * 8, D), vb + (long long)r * row + c * 8, true);
  }
  cp_commit();
  {
    // dC (fp32) -> bf16 tile; all read-only loads issued before the stores.  A
    // caller-supplied C (another fine writer) takes its dC elsewhere: z path only.
    constexpr int NV = D * D / 4 / 256;
    float4 cv[NV];
#pragma unroll
    for (int it = 0; it < NV; ++it)
      cv[it] = a.caller_c ? make_float4(0.f, 0.f, 0.f, 0.f)
                          : __ldg(reinterpret_cast<const float4*>(dcb) + tid + it * 256);
#pragma unroll
    for (int it = 0; it < NV; ++it) {
      const int e0 = (tid + it * 256) * 4, r = e0 / D, c = e0 % D;
      *reinterpret_cast<uint2*>(dB + swz(r, c, D)) =
          make_uint2(wa::pack_bf16(cv[it].x, cv[it].y), wa::pack_bf16(cv[it].z, cv[it].w));
    }
  }
  for (int d = tid; d < D; d += 256) {
    dzS[d] = rb(__ldg(a.dz + (((long long)b * a.dm.H + h) * a.dm.S + s) * D + d));
    dZp[d] = 0.f;
    dmS[d] = 0.f;
  }
  cp_wait<0>();
  __syncthreads();
  auto at = [&](uint8_t* base, int t, int d) -> bf16& { return *reinterpret_cast<bf16*>(base + swz(t, d, D)); };
  __shared__ float stat_scratch[(8 * D > 512) ? 8 * D : 512];  // also per-warp [8][D] partials
  channel_stats<D, 256>([&](int t, int d) { return bf(at(kB, t, d)); }, mx, zp, stat_scratch);
  // ties of the max (thread t: its token row)
  {
    const int t = tid;
#pragma unroll
    for (int w = 0; w < TW; ++w) {
      uint32_t bits = 0;
      for (int j = 0; j < 32; ++j) bits |= (uint32_t)(bf(at(kB, t, w * 32 + j)) == mx[w * 32 + j]) << j;
      tieS[t * TW + w] = bits;
    }
  }
  __syncthreads();
  // e and p, once per element, two adjacent channels at a time (one packed
  // conversion per rounding point)
  for (int idx = tid; idx < NT * D / 2; idx += 256) {
    const int t = idx / (D / 2), d = (idx % (D / 2)) * 2;
    const uint32_t k2 = *reinterpret_cast<const uint32_t*>(kB + swz(t, d, D));
    float e0 = __fsub_rn(lo_f(k2), mx[d]), e1 = __fsub_rn(hi_f(k2), mx[d + 1]);
    rb2(e0, e1);
    e0 = expf(e0);
    e1 = expf(e1);
    rb2(e0, e1);
    if (kStoreE) *reinterpret_cast<uint32_t*>(eB + swz(t, d, D)) = pack_exact(e0, e1);
    *reinterpret_cast<uint32_t*>(kB + swz(t, d, D)) = wa::pack_bf16(__fdiv_rn(e0, zp[d]), __fdiv_rn(e1, zp[d + 1]));
  }
  __syncthreads();
  const int g = lane >> 2, c4 = lane & 3;
  bf16* dvb = a.dv + tok0 * row + (long long)h * D;
  // ---- pass 1: dv_w = P . dC (rows: this warp's 32 tokens) ; dv += dv_w
  {
    float dvw[2][NTL][4];
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
      for (int j = 0; j < NTL; ++j)
#pragma unroll
        for (int x = 0; x < 4; ++x) dvw[mi][j][x] = 0.f;
#pragma unroll
    for (int kt = 0; kt < D / 16; ++kt) {
      uint32_t ap[2][4];
#pragma unroll
      for (int mi = 0; mi < 2; ++mi) {
        const int r = warp * 32 + mi * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kt * 16 + (lane >> 4) * 8;
        ldsm_x4(sK + swz(r, c, D), ap[mi][0], ap[mi][1], ap[mi][2], ap[mi][3]);
      }
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t b0, b1, b2, b3;  // B = dC (k = d, n = e): transposed loads
        const int r = kt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = np * 16 + (lane >> 4) * 8;
        ldsm_x4_t(sD + swz(r, c, D), b0, b1, b2, b3);
#pragma unroll
        for (int mi = 0; mi < 2; ++mi) {
          mma16816(dvw[mi][2 * np], ap[mi], b0, b1);
          mma16816(dvw[mi][2 * np + 1], ap[mi], b2, b3);
        }
      }
    }
#pragma unroll
    for (int mi = 0; mi < 2; ++mi) {
      // dv += dv_w: this CTA's own rows; the 2 x NTL loads go out before the stores
      __nv_bfloat162 old[2][NTL];
#pragma unroll
      for (int hr = 0; hr < 2; ++hr)
#pragma unroll
        for (int j = 0; j < NTL; ++j)
          old[hr][j] = *reinterpret_cast<const __nv_bfloat162*>(
              dvb + (long long)(warp * 32 + mi * 16 + g + hr * 8) * row + j * 8 + c4 * 2);
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int t = warp * 32 + mi * 16 + g + hr * 8;
#pragma unroll
        for (int j = 0; j < NTL; ++j) {
          const float2 o = __bfloat1622float2(old[hr][j]);
          float w0 = dvw[mi][j][hr * 2], w1 = dvw[mi][j][hr * 2 + 1];
          rb2(w0, w1);
          *reinterpret_cast<uint32_t*>(dvb + (long long)t * row + j * 8 + c4 * 2) = wa::pack_bf16(o.x + w0, o.y + w1);
        }
      }
    }
  }
  // ---- pass 2: dprob = V . dC^T
  float dp[2][NTL][4];
#pragma unroll
  for (int mi = 0; mi < 2; ++mi)
#pragma unroll
    for (int j = 0; j < NTL; ++j)
#pragma unroll
      for (int x = 0; x < 4; ++x) dp[mi][j][x] = 0.f;
#pragma unroll
  for (int kt = 0; kt < D / 16; ++kt) {
    uint32_t av[2][4];
#pragma unroll
    for (int mi = 0; mi < 2; ++mi) {
      const int r = warp * 32 + mi * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int c = kt * 16 + (lane >> 4) * 8;
      ldsm_x4(sV + swz(r, c, D), av[mi][0], av[mi][1], av[mi][2], av[mi][3]);
    }
#pragma unroll
    for (int np = 0; np < D / 16; ++np) {
      uint32_t b0, b1, b2, b3;  // B = dC^T (k = e, n = d): rows of dC, non-transposed
      const int r = np * 16 + (lane & 7) + (lane >> 4) * 8;
      const int c = kt * 16 + ((lane >> 3) & 1) * 8;
      ldsm_x4(sD + swz(r, c, D), b0, b1, b2, b3);
#pragma unroll
      for (int mi = 0; mi < 2; ++mi) {
        mma16816(dp[mi][2 * np], av[mi], b0, b1);
        mma16816(dp[mi][2 * np + 1], av[mi], b2, b3);
      }
    }
  }
  // partition term of the probability gradient: sum_t -bf16(dprob) * bf16(p / Z)
  float zpart[NTL][2];
#pragma unroll
  for (int j = 0; j < NTL; ++j) zpart[j][0] = zpart[j][1] = 0.f;
#pragma unroll
  for (int mi = 0; mi < 2; ++mi)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int t = warp * 32 + mi * 16 + g + hr * 8;
#pragma unroll
      for (int j = 0; j < NTL; ++j) {
        const int d = j * 8 + c4 * 2;
        const uint32_t p2 = *reinterpret_cast<const uint32_t*>(kB + swz(t, d, D));
        float a0 = dp[mi][j][hr * 2], a1 = dp[mi][j][hr * 2 + 1];
        float q0 = __fdiv_rn(lo_f(p2), zp[d]), q1 = __fdiv_rn(hi_f(p2), zp[d + 1]);
        rb2(a0, a1);
        rb2(q0, q1);
        float m0 = -__fmul_rn(a0, q0), m1 = -__fmul_rn(a1, q1);
        rb2(m0, m1);
        zpart[j][0] += m0;
        zpart[j][1] += m1;
      }
    }
#pragma unroll
  for (int j = 0; j < NTL; ++j)
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      float v = zpart[j][x];
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      if (g == 0) stat_scratch[warp * D + j * 8 + c4 * 2 + x] = v;  // per-warp partial
    }
  __syncthreads();
  for (int d = tid; d < D; d += 256) {
    float zsum = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) zsum += stat_scratch[w * D + d];
    dZp[d] = zsum;
    const float dlog = rb(__fdiv_rn(dzS[d], zp[d]));   // z = max + log(partition)
    dZ[d] = rb(rb(zsum) + dlog);
  }
  __syncthreads();
  // d_e = bf16(bf16(dprob / Z) + dZ) ; d_x = bf16(d_e * e) -> d raw_k ; sum_t d_x
  bf16* dkb = a.d_raw_k + tok0 * row + (long long)h * D;
  float mpart[NTL][2];
#pragma unroll
  for (int j = 0; j < NTL; ++j) mpart[j][0] = mpart[j][1] = 0.f;
#pragma unroll
  for (int mi = 0; mi < 2; ++mi)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int t = warp * 32 + mi * 16 + g + hr * 8;
      uint32_t kp[NTL];  // e pairs (width 64) or raw key pairs, loaded before the stores below
#pragma unroll
      for (int j = 0; j < NTL; ++j)
        kp[j] = kStoreE ? *reinterpret_cast<const uint32_t*>(eB + swz(t, j * 8 + c4 * 2, D))
                        : __ldg(reinterpret_cast<const unsigned int*>(kb + (long long)t * row + j * 8 + c4 * 2));
#pragma unroll
      for (int j = 0; j < NTL; ++j) {
        const int d = j * 8 + c4 * 2;
        float ev[2];
        if (kStoreE) {
          ev[0] = lo_f(kp[j]);
          ev[1] = hi_f(kp[j]);
        } else {
          ev[0] = __fsub_rn(lo_f(kp[j]), mx[d]);
          ev[1] = __fsub_rn(hi_f(kp[j]), mx[d + 1]);
          rb2(ev[0], ev[1]);
          ev[0] = expf(ev[0]);
          ev[1] = expf(ev[1]);
          rb2(ev[0], ev[1]);
        }
        float a0 = dp[mi][j][hr * 2], a1 = dp[mi][j][hr * 2 + 1];
        rb2(a0, a1);
        float q0 = __fdiv_rn(a0, zp[d]), q1 = __fdiv_rn(a1, zp[d + 1]);
        rb2(q0, q1);
        float de0 = __fadd_rn(q0, dZ[d]), de1 = __fadd_rn(q1, dZ[d + 1]);
        rb2(de0, de1);
        float dx0 = __fmul_rn(de0, ev[0]), dx1 = __fmul_rn(de1, ev[1]);
        rb2(dx0, dx1);
        mpart[j][0] += dx0;
        mpart[j][1] += dx1;
        *reinterpret_cast<uint32_t*>(dkb + (long long)t * row + d) = pack_exact(dx0, dx1);
      }
    }
#pragma unroll
  for (int j = 0; j < NTL; ++j)
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      float v = mpart[j][x];
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      if (g == 0) stat_scratch[warp * D + j * 8 + c4 * 2 + x] = v;  // per-warp partial
    }
  __syncthreads();
  for (int d = tid; d < D; d += 256) {
    float msum = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) msum += stat_scratch[w * D + d];
    dmS[d] = msum;
  }
  __syncthreads();
  // max: dm = dz - sum_t d_x, shared evenly by the tokens that attain the max
  {
    constexpr int G = 256 / D, TPG = NT / G;
    const int d = tid % D, grp = tid / D;
    const uint32_t bit = 1u << (d & 31);
    int cnt = 0;
    for (int t = grp * TPG; t < (grp + 1) * TPG; ++t) cnt += (tieS[t * TW + d / 32] & bit) != 0;
    stat_scratch[grp * D + d] = (float)cnt;
    __syncthreads();
    int count = 0;
#pragma unroll
    for (int x = 0; x < G; ++x) count += (int)stat_scratch[x * D + d];
    const float dm = rb(dzS[d] - rb(dmS[d]));
    const float share = rb(dm / count);
    for (int t = grp * TPG; t < (grp + 1) * TPG; ++t)
      if (tieS[t * TW + d / 32] & bit) {
        bf16* p = dkb + (long long)t * row + d;
        *p = tobf(bf(*p) + share);
      }
  }
}

}  // namespace tao
