// extern "C" training entry points (tao_attention forward / backward).
#include <cuda_runtime.h>

#include <cstdio>

#include "../../include/tao_b200.h"
#include "tc_writer.cuh"
#include "train_backward.cuh"

void tao_set_last_error(const char* msg);
void tao_take_profile_events(cudaEvent_t* start, cudaEvent_t* stop);
namespace tao {
int launch_window_attention(const bf16* q, const bf16* k, const bf16* v, bf16* out, float* lse, int B,
                            int T, int H, int D, int* err, cudaStream_t s);
int launch_attention_backward_tc(const bf16* q, const bf16* k, const bf16* v, const bf16* dout, const float* lse,
                                 const float* rowdot, bf16* dq, bf16* dk, bf16* dv, float* dq_acc, int B, int T,
                                 int H, int D, int* err, cudaStream_t s);
int attention_variant();
}  // namespace tao

namespace {

int tfail(int code, const char* msg) {
  tao_set_last_error(msg);
  return code;
}

int t_budget(int count) {
  if (count <= 0) return 0;
  long long sq = 2LL * count, r = 0;
  while ((r + 1) * (r + 1) <= sq) ++r;
  if (r * r < sq) ++r;
  return (int)(r + 2 < count ? r + 2 : count);
}
int t_selected(int completed, int pending) {
  const int cb = t_budget(8 * completed);
  int coarse = (2 * cb + 7) / 8;
  if (coarse > completed) coarse = completed;
  const int eligible = 8 * coarse + pending;
  const int b = t_budget(8 * completed + pending);
  return eligible < b ? eligible : b;
}

struct Geometry {
  int tiles, S, pages, vmax, pmax, mmax;
};
Geometry geometry(int T) {
  Geometry g{};
  g.tiles = (T + 255) / 256;
  g.S = T > 768 ? T / 256 - 1 : 0;
  g.pages = g.S > 0 ? (g.S + 7) / 8 : 0;
  g.vmax = g.tiles > 3 ? g.tiles - 3 : 0;
  g.pmax = g.vmax / 8 + 1;
  g.mmax = 1;
  for (int v = 1; v <= g.vmax; ++v) {
    const int m = t_selected(v / 8, v % 8);
    if (m > g.mmax) g.mmax = m;
  }
  return g;
}

template <typename F>
bool tsmem(F* fn, size_t bytes) {
  return bytes <= 48 * 1024 ||
         cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess;
}

template <int D>
int train_forward(const tao::bf16* q, const tao::bf16* k, const tao::bf16* v, const tao::bf16* rq,
                  const tao::bf16* rk, const tao::bf16* fa, const tao::bf16* fb, const float* gain, int B,
                  int T, int H, tao::bf16* out, const TaoTrainBuffers& tb, cudaStream_t s) {
  using namespace tao;
  const Geometry g = geometry(T);
  TrainDims dm{B, T, H, g.S, (long long)H * D};
  // 1. exact local window attention
  cudaEvent_t ev0, ev1;
  tao_take_profile_events(&ev0, &ev1);
  if (ev0) cudaEventRecord(ev0, s);
  if (int rc = launch_window_attention(q, k, v, static_cast<bf16*>(tb.local), tb.lse, B, T, H, D, tb.err, s))
    return rc;
  if (ev1) cudaEventRecord(ev1, s);
  const bool route_only = (tb.flags & TAO_TRAIN_ROUTE_ONLY) != 0;  // z and page prefixes from the caller
  if (g.S > 0 && !route_only) {
    // 2. writer over all sealed blocks (tcgen05 by default, mma.sync with attention
    // variant 0), 3. page prefix table
    const int write_c = (tb.flags & TAO_TRAIN_CALLER_FINE_C) ? 0 : 1;
    if (attention_variant() == 1) {
      const size_t wsmem = TcWriterCfg<D>::SMEM;
      if (!tsmem(tc_writer_kernel<D>, wsmem)) return tfail(TAO_ERR_CUDA, "smem attribute");
      tc_writer_kernel<D><<<B * H * g.S, 128, wsmem, s>>>(rk, v, static_cast<bf16*>(tb.fine_z),
                                                          static_cast<bf16*>(tb.fine_c), dm, write_c, tb.err);
    } else {
      const size_t wsmem = (size_t)2 * 256 * D * 2 + 2 * D * 4;
      if (!tsmem(writer_kernel<D>, wsmem)) return tfail(TAO_ERR_CUDA, "smem attribute");
      writer_kernel<D><<<B * H * g.S, 128, wsmem, s>>>(rk, v, static_cast<bf16*>(tb.fine_z),
                                                        static_cast<bf16*>(tb.fine_c), dm, write_c);
    }
    const long long n = (long long)B * H * g.pages * D;
    page_prefix_kernel<D><<<(int)((n + 255) / 256), 256, 0, s>>>(
        static_cast<const bf16*>(tb.fine_z), static_cast<bf16*>(tb.page_prefix), dm, g.pages);
  }
  // 4. routing + selected read + fusion
  ReadArgs a{};
  a.raw_q = rq;
  a.local = static_cast<const bf16*>(tb.local);
  a.fa = fa;
  a.fb = fb;
  a.gain = gain;
  a.z = static_cast<const bf16*>(tb.fine_z);
  a.C = static_cast<const bf16*>(tb.fine_c);
  a.pzpre = static_cast<const bf16*>(tb.page_prefix);
  a.out = out;
  a.num_out = static_cast<bf16*>(tb.num);
  a.den_out = tb.den;
  a.sel_out = tb.sel;
  a.dm = dm;
  a.pages = g.pages;
  a.mmax = g.mmax;
  a.err = tb.err;
  a.external_fusion = (tb.flags & TAO_TRAIN_EXTERNAL_FUSION) ? 1 : 0;
  a.route_only = route_only ? 1 : 0;
  a.tc = attention_variant() == 1 ? 1 : 0;   // the selected read on tcgen05
  const size_t rsmem = ReadSmem<D>::bytes(g.pmax, g.vmax, g.mmax);
  if (rsmem > 227 * 1024) return tfail(TAO_ERR_CAPACITY, "sequence too long for the training read kernel");
  bool launched = false;
  if (a.tc) {
    if (!tsmem(train_read_kernel<D, true>, rsmem)) return tfail(TAO_ERR_CUDA, "smem attribute");
    train_read_kernel<D, true><<<dim3(B * H, g.tiles), 256, rsmem, s>>>(a);
    launched = true;
  }
  if (!launched) {
    if (!tsmem(train_read_kernel<D>, rsmem)) return tfail(TAO_ERR_CUDA, "smem attribute");
    train_read_kernel<D><<<dim3(B * H, g.tiles), 256, rsmem, s>>>(a);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return tfail(TAO_ERR_CUDA, cudaGetErrorString(e));
  return TAO_OK;
}

template <int D>
int train_backward(const tao::BwdArgs& a0, cudaStream_t s) {
  using namespace tao;
  BwdArgs a = a0;
  const Geometry g = geometry(a.dm.T);
  const int B = a.dm.B, H = a.dm.H, T = a.dm.T;
  cudaEvent_t ev0, ev1;  // profiling hook: around the selected-read backward
  tao_take_profile_events(&ev0, &ev1);
  // d raw_k of the tokens past the last sealed block gets no writer gradient: zero
  // those rows here (the writer backward writes all the others)
  const long long tail0 = (long long)g.S * kFine;
  if (tail0 < T) {
    const size_t row_bytes = (size_t)H * D * 2;
    if (cudaMemset2DAsync(a.d_raw_k + tail0 * H * D, (size_t)T * row_bytes, 0, (size_t)(T - tail0) * row_bytes, B,
                          s) != cudaSuccess)
      return tfail(TAO_ERR_CUDA, "d_raw_k tail memset");
  }
  // width 128 splits a tile's queries over two CTAs that add into the same dC partial
  if (!a.route_only && ReadBwdSmem<D>::NQ < 256 && a.npairs > 0 &&
      cudaMemsetAsync(a.dcp, 0, (size_t)B * H * a.npairs * D * D * 2, s) != cudaSuccess)
    return tfail(TAO_ERR_CUDA, "dc_partial memset");
  if (a.route_only) {
    // the caller differentiates the writer and the read: no raw_q / raw_k gradient here
    const size_t bytes = (size_t)B * T * H * D * 2;
    if (cudaMemsetAsync(a.d_raw_q, 0, bytes, s) != cudaSuccess || cudaMemsetAsync(a.d_raw_k, 0, bytes, s) != cudaSuccess)
      return tfail(TAO_ERR_CUDA, "route-only gradient memset");
  }
  const dim3 fgrid((T + 8 * kFusionRowsPerWarp - 1) / (8 * kFusionRowsPerWarp), B * H);
  if (a.external_fusion || a.route_only)
    split_bwd_kernel<D><<<fgrid, 256, 0, s>>>(a);
  else
    fusion_bwd_kernel<D><<<fgrid, 256, 0, s>>>(a);
  if (a.dq_acc && attention_variant() == 1) {
    if (int rc = launch_attention_backward_tc(a.q, a.k, a.v, a.d_local, a.lse, a.dv_row, a.dq, a.dk, a.dv,
                                              a.dq_acc, B, T, H, D, a.err, s))
      return rc;
  } else {
    const size_t asmem = (size_t)(2 * 64 + 4 * 64) * D * 2 + 256 * 4;
    if (!tsmem(attn_bwd_kv_kernel<D>, asmem) || !tsmem(attn_bwd_q_kernel<D>, asmem))
      return tfail(TAO_ERR_CUDA, "smem attribute");
    attn_bwd_kv_kernel<D><<<dim3((T + 63) / 64, B * H), 128, asmem, s>>>(a);
    attn_bwd_q_kernel<D><<<dim3((T + 63) / 64, B * H), 128, asmem, s>>>(a);
  }
  if (a.route_only) {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TAO_OK : tfail(TAO_ERR_CUDA, cudaGetErrorString(e));
  }
  const size_t rsmem = ReadBwdSmem<D>::bytes(g.pmax, g.vmax, g.mmax);
  if (rsmem > 227 * 1024) return tfail(TAO_ERR_CAPACITY, "sequence too long for the read backward kernel");
  const bool tc_bwd = attention_variant() == 1;   // dA / dC on tcgen05
  if (tc_bwd) {
    if (!tsmem(read_bwd_kernel<D, true>, rsmem)) return tfail(TAO_ERR_CUDA, "smem attribute");
  } else if (!tsmem(read_bwd_kernel<D>, rsmem)) {
    return tfail(TAO_ERR_CUDA, "smem attribute");
  }
  constexpr int NQ = ReadBwdSmem<D>::NQ;
  if (ev0) cudaEventRecord(ev0, s);
  if (tc_bwd)
    read_bwd_kernel<D, true><<<dim3(B * H * (256 / NQ), g.tiles), ReadBwdSmem<D>::NT, rsmem, s>>>(a);
  else
    read_bwd_kernel<D><<<dim3(B * H * (256 / NQ), g.tiles), ReadBwdSmem<D>::NT, rsmem, s>>>(a);
  if (ev1) cudaEventRecord(ev1, s);
  if (g.S > 0) {
    dc_reduce_kernel<D><<<B * H * g.S, 256, 0, s>>>(a, g.tiles);
    const size_t wsmem = WriterBwdSmem<D>::bytes();
    if (!tsmem(writer_bwd_kernel<D>, wsmem)) return tfail(TAO_ERR_CUDA, "smem attribute");
    writer_bwd_kernel<D><<<B * H * g.S, 256, wsmem, s>>>(a);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return tfail(TAO_ERR_CUDA, cudaGetErrorString(e));
  return TAO_OK;
}

}  // namespace

extern "C" {

int tao_train_backward(const void* grad_out, const void* q, const void* k, const void* v,
                       const void* raw_q, const void* raw_k, const void* fusion_a,
                       const void* fusion_b, const float* gain, int batch, int tokens, int heads,
                       int width, const void* out, const TaoTrainBuffers* saved,
                       const TaoTrainGrads* grads, void* stream) {
  (void)out;
  if (!grad_out || !q || !k || !v || !raw_q || !raw_k || !fusion_a || !fusion_b || !gain || !saved || !grads)
    return tfail(TAO_ERR_ARG, "null pointer");
  if (width != 64 && width != 128) return tfail(TAO_ERR_ARG, "head width must be 64 or 128");
  if (batch <= 0 || tokens <= 0 || heads <= 0) return tfail(TAO_ERR_ARG, "bad shape");
  const Geometry g = geometry(tokens);
  if (saved->mmax != g.mmax) return tfail(TAO_ERR_ARG, "saved.mmax does not match tao_train_geometry");
  using tao::bf16;
  tao::BwdArgs a{};
  auto C = [](const void* p) { return static_cast<const bf16*>(p); };
  auto W = [](void* p) { return static_cast<bf16*>(p); };
  a.g = C(grad_out); a.raw_q = C(raw_q); a.local = C(saved->local); a.num = C(saved->num);
  a.fa = C(fusion_a); a.fb = C(fusion_b); a.q = C(q); a.k = C(k); a.v = C(v); a.raw_k = C(raw_k);
  a.den = saved->den; a.gain = gain; a.lse = saved->lse;
  a.z = C(saved->fine_z); a.C = C(saved->fine_c); a.pzpre = C(saved->page_prefix); a.sel = saved->sel;
  a.d_local = W(grads->d_local); a.gn = W(grads->gn); a.d_rq_f = W(grads->d_rq_f);
  a.gd = grads->gd; a.dv_row = grads->row_dot; a.d_fa = grads->d_fusion_a; a.d_fb = grads->d_fusion_b;
  a.dq = W(grads->dq); a.dk = W(grads->dk); a.dv = W(grads->dv); a.d_raw_q = W(grads->d_raw_q);
  a.d_raw_k = W(grads->d_raw_k); a.dC = grads->dC; a.dz = grads->dz;
  a.dcp = W(grads->dc_partial);
  a.dq_acc = grads->dq_acc;
  a.npairs = g.vmax * (g.vmax + 1) / 2;
  a.dm = tao::TrainDims{batch, tokens, heads, g.S, (long long)heads * width};
  a.pages = g.pages;
  a.mmax = g.mmax;
  a.err = saved->err;
  a.caller_c = (saved->flags & TAO_TRAIN_CALLER_FINE_C) ? 1 : 0;
  a.external_fusion = (saved->flags & TAO_TRAIN_EXTERNAL_FUSION) ? 1 : 0;
  a.route_only = (saved->flags & TAO_TRAIN_ROUTE_ONLY) ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return width == 64 ? train_backward<64>(a, s) : train_backward<128>(a, s);
}

int tao_train_pairs(int tokens) {
  const Geometry g = geometry(tokens);
  return g.vmax * (g.vmax + 1) / 2;
}

int tao_train_geometry(int tokens, int* sealed, int* pages, int* mmax) {
  if (tokens <= 0) return tfail(TAO_ERR_ARG, "tokens must be positive");
  const Geometry g = geometry(tokens);
  if (sealed) *sealed = g.S;
  if (pages) *pages = g.pages;
  if (mmax) *mmax = g.mmax;
  return TAO_OK;
}

int tao_train_forward(const void* q, const void* k, const void* v, const void* raw_q, const void* raw_k,
                      const void* fusion_a, const void* fusion_b, const float* gain, int batch,
                      int tokens, int heads, int width, void* out, const TaoTrainBuffers* buffers,
                      void* stream) {
  if (!q || !k || !v || !raw_q || !raw_k || !fusion_a || !fusion_b || !gain || !out || !buffers)
    return tfail(TAO_ERR_ARG, "null pointer");
  if (width != 64 && width != 128) return tfail(TAO_ERR_ARG, "head width must be 64 or 128");
  if (batch <= 0 || tokens <= 0 || heads <= 0) return tfail(TAO_ERR_ARG, "bad shape");
  const TaoTrainBuffers& tb = *buffers;
  if (!tb.local || !tb.lse || !tb.num || !tb.den || !tb.sel || !tb.err)
    return tfail(TAO_ERR_ARG, "null training buffer");
  if (tokens > 768 && (!tb.fine_z || !tb.fine_c || !tb.page_prefix))
    return tfail(TAO_ERR_ARG, "null fine buffers");
  if (tb.mmax != geometry(tokens).mmax) return tfail(TAO_ERR_ARG, "buffers.mmax does not match tao_train_geometry");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  using tao::bf16;
  auto B = [](const void* p) { return static_cast<const bf16*>(p); };
  return width == 64
             ? train_forward<64>(B(q), B(k), B(v), B(raw_q), B(raw_k), B(fusion_a), B(fusion_b), gain, batch,
                                 tokens, heads, static_cast<bf16*>(out), tb, s)
             : train_forward<128>(B(q), B(k), B(v), B(raw_q), B(raw_k), B(fusion_a), B(fusion_b), gain, batch,
                                  tokens, heads, static_cast<bf16*>(out), tb, s);
}

}  // extern "C"
