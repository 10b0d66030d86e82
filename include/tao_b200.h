/* C ABI of the B200-native TaoMemory attention operator (libtao_b200.so).
 *
 * Plain pointers, sizes and a CUDA stream passed as `void*`; no framework types.
 * All tensors are device memory, bf16 (`uint16_t` storage), contiguous, in the
 * layouts stated per entry point.  Every function returns TAO_OK or an error
 * code; tao_last_error() gives the message of the last failing call on the
 * calling host thread.
 *
 * Reference interfaces replaced (LaurenceLong/tao-memory, tao_attention/):
 *   tao_stream_step       -> StreamCache.process + fusion (tao_stream.py:919-979,
 *                            operator.py:70-127), batched over requests; the
 *                            decode form is operator.py:130-137
 *   tao_state_init        -> StreamCache.__init__ / reset (tao_stream.py:795-851)
 *   tao_window_attention  -> flash_attention.flash_attn_func (flash_attention.py:16-37)
 *                            in the windowed form of tao_stream.py:760-787
 *   tao_train_forward     -> operator.tao_attention forward (operator.py:42-54)
 *   tao_train_backward    -> its autograd backward (selected_read.py:175-187 and
 *                            the torch autograd around it)
 */
#ifndef TAO_B200_H
#define TAO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TAO_OK 0
#define TAO_ERR_ARG 1        /* shape / width / alignment / capacity argument      */
#define TAO_ERR_POSITION 2   /* position does not match the request's cursor       */
#define TAO_ERR_SEAL 3       /* chunk crosses a fine seal boundary                 */
#define TAO_ERR_CAPACITY 4   /* fine bank or route capacity too small              */
#define TAO_ERR_CUDA 5       /* CUDA launch / runtime error                        */
#define TAO_ERR_DEVICE 6     /* a kernel reported an error (bounded wait expired)  */
#define TAO_ERR_TIMEOUT 7    /* a host wait (tao_host_wait) expired                */

/* Geometry of the preset (TaoConfig, config.py:7-19).  fine_tokens, local_keep and
 * coarse_group must be 256, 512 and 8; the schedule fields are free.  route_cap is
 * the length of the route-id arrays of every state passed to one call.  fine_read
 * selects the read of the selected fines: 0 = normalised association read
 * (softmax and regularised-association writers, query_fresh_fine.py:8-49),
 * 1 = feature-mass read (feature-mass writer, association_writer.py:43-53 via
 * tao_stream.py:362-367); tao_decode_step serves fine_read 1 with its default
 * decode kernel (variant 1) for up to 256 selected fines, tao_stream_decode_noalloc
 * refuses it.  coarse = 1 selects the coarse value branch (TaoConfig
 * coarse_index_only=False, the historical default): every completed page carries a
 * coarse matrix C_page = bf16(sum_s bf16(exp(bf16(z_s - page_z))) * C_s) built when the
 * page closes (tao_stream.py:486-500), every query reads all completed pages'
 * matrices (tao_stream.py:299-305) and the pointwise fusion gains its coarse term;
 * it needs fine_read 0 and states with page_c / coarse_w buffers; decode steps then
 * run through the tao_stream_step kernels. */
typedef struct TaoPolicy {
  int32_t fine_tokens;
  int32_t local_keep;
  int32_t coarse_group;
  int32_t route_period;
  int32_t layer_stagger;
  int32_t budget_root_scale;
  int32_t budget_offset;
  int32_t route_cap;
  int32_t fine_read;
  int32_t coarse;
} TaoPolicy;

/* Device-resident descriptor of one request's one-layer state.  The host writes
 * it (pointers, capacities, cursor) and the kernels update `position`, `n_route`,
 * `n_chosen`, the counters and the buffers it points to.
 *
 * Buffers (H heads, D width, all bf16 unless noted):
 *   k_ring, v_ring, rk_ring : [H][768][D]  exact local window, slot = position % 768
 *   fine_c                  : [H][cap_fines][D][D]
 *   fine_z                  : [H][cap_fines][D]
 *   page_z, page_w          : [H][cap_fines/8 + 1][D]  page log-partition and its
 *                             softmax over pages (the page-normalisation memo)
 *   route_ids               : int32 [H][route_cap]   selected fines, rank order
 *   route_pages             : int32 [H][route_cap]   pages kept by the page top-K
 *   counters                : int32 [H], zero-initialised; per-head arrival counters
 *                             of the fused decode kernel (reset by their last user)
 *   page_c                  : [H][cap_fines/8 + 1][D][D]  coarse matrix of each
 *                             completed page (coarse value branch only, else NULL)
 *   coarse_w                : [H][cap_fines/8 + 1][D]  softmax over the completed
 *                             pages of page_z (coarse value branch only, else NULL)
 */
typedef struct TaoState {
  void* k_ring;
  void* v_ring;
  void* rk_ring;
  void* fine_c;
  void* fine_z;
  void* page_z;
  void* page_w;
  int32_t* route_ids;
  int32_t* route_pages;
  int32_t* counters;
  int64_t position;
  int32_t n_route;
  int32_t n_chosen;
  int32_t cap_fines;
  int32_t route_cap;
  int32_t layer_index;
  int32_t heads;
  int32_t width;
  int32_t arrive;        /* internal: per-step arrival counter, keep 0 */
  int32_t route_refreshes;
  int32_t seal_events;
  void* page_c;
  void* coarse_w;
} TaoState;

const char* tao_last_error(void);
int tao_version(void);
size_t tao_state_sizeof(void);

/* Bytes of workspace tao_stream_step needs for n_states requests of `tokens`
 * new tokens each (tokens == 1 for decode). */
size_t tao_stream_workspace_bytes(int n_states, int tokens, int heads, int width,
                                  int route_cap, const TaoPolicy* policy);

/* Advance n_states requests by `tokens` new tokens each.
 *   states      : device array of n_states pointers to device TaoState
 *   host_pos    : host array of the n_states cursors (validated: chunk must not
 *                 cross a seal boundary; fine capacity must suffice)
 *   host_cap    : host array of the n_states fine capacities
 *   q,k,v,raw_q,raw_k,out : [n_states][tokens][H][D]
 *   fusion_a, fusion_b    : [H][D][3]
 *   alpha                 : history scale (gain = bf16(2 * alpha))
 *   workspace             : tao_stream_workspace_bytes(...) bytes, 256-byte aligned
 * Reference: StreamCache.process + pointwise fusion (tao_stream.py:919-979,
 * operator.py:79-99). */
int tao_stream_step(void* const* states, int n_states, const int64_t* host_pos,
                    const int32_t* host_cap, const TaoPolicy* policy, int tokens,
                    int heads, int width, const void* q, const void* k, const void* v,
                    const void* raw_q, const void* raw_k, const void* fusion_a,
                    const void* fusion_b, float alpha, void* out, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Fast decode step: one token for each of n_states requests in one fused kernel
 * (plus a routing kernel on refresh tokens and a seal kernel when a window fills).
 * Same arguments as tao_stream_step with tokens = 1, plus host_layer (the layer
 * index of each state, used to decide on the host whether any request refreshes).
 * Workspace: tao_stream_workspace_bytes(n_states, 1, ...).  Results agree with
 * tao_stream_step up to fp32 summation order (routes identical).  Reference:
 * tao_attention_decode (operator.py:130-137). */
int tao_decode_step(void* const* states, int n_states, const int64_t* host_pos,
                    const int32_t* host_layer, const int32_t* host_cap, const TaoPolicy* policy,
                    int heads, int width, const void* q, const void* k, const void* v,
                    const void* raw_q, const void* raw_k, const void* fusion_a,
                    const void* fusion_b, float alpha, void* out, void* workspace,
                    size_t workspace_bytes, void* stream);

/* tao_decode_step for a caller whose operands arrive in, and whose result leaves
 * through, page-locked host memory:
 *   host_in   : page-locked [5][n_states][1][H][D] bf16 (q, k, v, raw_q, raw_k)
 *   stage     : device [5][n_states][1][H][D] bf16 (the operands' device copy)
 *   host_out  : page-locked [n_states][1][H][D] bf16
 *   host_done : page-locked int32 completion word, or NULL
 * Host buffers need a device mapping (see tao_host_device_pointer); operands, stage
 * and output 16-byte aligned.  The step's routing kernel is always launched: it
 * first copies host_in to stage over the host link (and reads raw_q from host memory
 * itself), and the fused kernel writes each (request, head)'s output row straight
 * into host_out.  With host_done, once every row of the step is in host memory the
 * fused kernel stores the step's sequence number there: the count of steps with a
 * completion word run on this workspace (1 for the first), so a host thread can
 * wait for the result with tao_host_wait instead of synchronising the stream (a
 * seal kernel may still run after it, in stream order).  A completion word needs
 * decode variant 1, 3 or 4.  Results are those of tao_copy_host_to_device_many +
 * tao_decode_step + tao_copy_device_to_host, with two kernels fewer per step.  The
 * coarse value branch is refused (TAO_ERR_ARG).  No counterpart in the reference. */
int tao_decode_step_host(void* const* states, int n_states, const int64_t* host_pos,
                         const int32_t* host_layer, const int32_t* host_cap, const TaoPolicy* policy,
                         int heads, int width, const void* host_in, void* stage, void* host_out,
                         void* host_done, const void* fusion_a, const void* fusion_b, float alpha,
                         void* workspace, size_t workspace_bytes, void* stream);

/* The device address of page-locked host memory (*device), or TAO_ERR_ARG when
 * `host` is not page-locked memory with a device mapping. */
int tao_host_device_pointer(const void* host, void** device);

/* Spin (without the Python interpreter's lock, for ctypes callers) until the int32 at
 * `word` (page-locked host memory written by a kernel) reaches `value` (wrap-around
 * order: word - value >= 0), or `timeout_us` microseconds pass (TAO_ERR_TIMEOUT). */
int tao_host_wait(const void* word, int value, long long timeout_us);

/* cudaGraphLaunch of an instantiated graph (cudaGraphExec_t) on `stream`. */
int tao_graph_launch(void* graph_exec, void* stream);

/* Select the decode kernel of tao_decode_step for this process: 1 = persistent fused
 * kernel with one 32 KB copy stage per CTA (default), 3 = the same with two 32 KB
 * stages per CTA (half the resident CTAs; measured slower), 4 = the same with two
 * 16 KB stages per CTA and half-size items (64 keys or 2 fines; width 64, width 128
 * runs variant 1), 0 = warp-specialised persistent kernel, 2 = one warp per 8 KB work
 * item.  Variants 1 and 3 give identical results; the others agree to fp32
 * summation order. */
int tao_decode_variant(int variant);

/* Graph mode for the calling host thread (on != 0): tao_decode_step then always
 * launches its route and seal kernels, which decide on the device from each state's
 * cursor whether the token refreshes the routes or seals a block.  A step launched
 * in this mode can be captured once into a CUDA graph and replayed for every later
 * token while the fine-bank capacity (grid sizes) is unchanged; nothing is re-captured
 * at a seal.  Reference counterpart: HistoryRegionGraph
 * (history_region_graph.py:10-113), which captures only the history read and
 * re-captures at every seal. */
int tao_decode_graph_mode(int on);

/* Read and clear the device error word of a workspace (synchronises `stream`).
 * Returns TAO_OK or TAO_ERR_DEVICE; *flags receives the raw bits. */
int tao_stream_check(void* workspace, int* flags, void* stream);

/* Host<->device transfer of a decode step's operands by the SMs: a kernel reads
 * (or writes) page-locked, device-mapped host memory directly, 16 bytes per thread,
 * on `stream`.  For the tens of kilobytes of one decode step this costs about one
 * round trip over the host link instead of a copy engine's setup latency.  The host
 * buffer must be page-locked with a device mapping (checked with
 * cudaPointerGetAttributes; otherwise TAO_ERR_ARG and nothing is accessed), the
 * other must be device memory of the calling thread's current device (where the
 * kernel runs), both 16-byte aligned and `bytes` a multiple of 16.  The device
 * range must lie inside one allocation (its extent comes from the driver,
 * cuMemGetAddressRange; otherwise TAO_ERR_ARG); the host range is the caller's to
 * keep in bounds.
 * No counterpart in the reference (its operands are already on the device). */
int tao_copy_host_to_device(void* dst, const void* host_src, size_t bytes, void* stream);
int tao_copy_device_to_host(void* host_dst, const void* src, size_t bytes, void* stream);

/* The same transfer for n (1..8) buffers in one launch: dst[i] <- host_src[i],
 * bytes[i] each, with the checks above on every pair.  A decode step's five
 * operands cross in one launch.  No counterpart in the reference. */
int tao_copy_host_to_device_many(void* const* dst, const void* const* host_src, const size_t* bytes,
                                 int n, void* stream);

/* Decode step (one token for each of n_states requests) that allocates nothing:
 * same arguments and results as tao_stream_step with tokens = 1, but its scratch
 * lives in a static 4 MiB device array inside the library instead of a
 * caller-provided workspace.  For callers that cannot call cudaMalloc (memory
 * owned by another runtime's pool, or loops where an allocation could
 * synchronise the device).  Batches whose decode scratch exceeds 4 MiB return
 * TAO_ERR_CAPACITY.  All calls on a device share that array: calls that overlap
 * on the GPU race, so serialise them; the first call on a device sets the array
 * up and should come before any stream capture.  No counterpart in the reference. */
int tao_stream_decode_noalloc(void* const* states, int n_states, const int64_t* host_pos,
                              const int32_t* host_cap, const TaoPolicy* policy, int heads,
                              int width, const void* q, const void* k, const void* v,
                              const void* raw_q, const void* raw_k, const void* fusion_a,
                              const void* fusion_b, float alpha, void* out, void* stream);

/* The device error word of tao_stream_decode_noalloc on the calling thread's
 * current device (route overflow, expired bounded wait), which lives in the same
 * static array: synchronises `stream`, stores the word in *flags, clears it and
 * returns TAO_ERR_DEVICE when it was set.  Read it after the calls whose result
 * matters, before the next call clears it.  No counterpart in the reference. */
int tao_stream_decode_noalloc_check(int* flags, void* stream);

/* CUDA events for timing (thin wrappers over the runtime, so callers need no
 * other binding).  tao_stream_profile_next(start, stop) makes the next library
 * call that launches one of these (from any host thread) record `start` just
 * before and `stop` just after it, on the stream it launches on: the main
 * kernel(s) of a stream / decode step (the local-attention + fine-read phase),
 * the windowed local-attention kernel of tao_train_forward, or the selected-read
 * backward kernel of tao_train_backward.  No reference counterpart (profiling
 * hook). */
int tao_event_create(void** event);
int tao_event_destroy(void* event);
int tao_event_record(void* event, void* stream);
int tao_event_elapsed(void* start, void* stop, float* ms);
int tao_stream_profile_next(void* start, void* stop);

/* Copy `count` ring slots of one request into a token-ordered [count][H][D] buffer
 * (used by export).  first_position is the absolute position of the first token. */
int tao_ring_gather(const void* ring, int heads, int width, int64_t first_position,
                    int count, void* out, void* stream);
/* Inverse of tao_ring_gather (used by import). */
int tao_ring_scatter(void* ring, int heads, int width, int64_t first_position, int count,
                     const void* in, void* stream);

/* Recompute the page memo (page_z, page_w) of one device state from its fine_z for
 * `sealed` fines (after import).  `state` is the device TaoState.  Reference:
 * LayerState._prepare_q1_page_memo (tao_stream.py:399-416). */
int tao_state_rebuild_memo(void* state, int heads, int width, int sealed, void* stream);

/* Recompute only the page weights page_w = bf16(softmax over pages of page_z) per
 * channel, keeping page_z as the caller wrote it.  The feature-mass writer sets
 * page_z itself (bf16(log of the accumulated feature mass), tao_stream.py:62-65 and
 * 463-500) after each seal and after import.  Reference: the memo refresh of
 * LayerState._prepare_q1_page_memo (tao_stream.py:399-416). */
int tao_state_refresh_page_weights(void* state, int heads, int width, int sealed, void* stream);

/* Windowed causal attention used by training (tao_stream.py:760-787 semantics):
 * query t sees keys [max(0, 256*floor(t/256) - 512), t].  q,k,v,out [B][T][H][D];
 * lse: fp32 [B][H][T] (log-sum-exp of the scaled scores, saved for backward). */
int tao_window_attention(const void* q, const void* k, const void* v, void* out,
                         float* lse, int batch, int tokens, int heads, int width,
                         void* stream);

/* Sufficient statistics of the association fine writers for `blocks` x `heads`
 * 256-token blocks: u = bf16(softmax over channels of k[t]) (fp32 softmax), then
 * gram = u^T u and cross = u^T v, fp32 [blocks][heads][width][width], and when
 * `mass` is not null the feature mass sum_t u[t], fp32 [blocks][heads][width].
 * Token t of (block b, head h) starts at k + b*block_stride + h*head_stride +
 * t*token_stride (elements; rows 16-byte aligned), likewise for v.  Reference:
 * association_statistics (association_writer.py:11-18) at a seal
 * (tao_stream.py:62-65, 72-74). */
int tao_writer_stats(const void* k, const void* v, long long token_stride, long long head_stride,
                     long long block_stride, int blocks, int heads, int width, float* gram,
                     float* cross, float* mass, void* stream);

/* Select the tensor-core form of the windowed attention (tao_window_attention, the
 * training forward and backward, the streaming prefill chunk over the ring) and of
 * the training selected read and its backward, for this process: 1 = tcgen05/TMEM
 * kernels (default, widths 64 and 128; TMA tiles for contiguous operands, cp.async
 * tiles for the ring), 0 = mma.sync kernels everywhere.  Outputs agree to fp32
 * summation order.  No counterpart in the reference (it has one attention path,
 * flash_attention.py:16-37). */
int tao_attention_variant(int variant);

/* ---- training (tao_attention, operator.py:42-54) -------------------------
 * Saved buffers of one forward, allocated by the caller (sizes from
 * tao_train_geometry; S sealed blocks, P pages, mmax selected fines per query):
 *   local [B][T][H][D] bf16, lse fp32 [B][H][T], fine_z [B][H][S][D] bf16,
 *   fine_c [B][H][S][D][D] bf16, page_prefix [B][H][P][8][D] bf16,
 *   num [B][T][H][D] bf16, den fp32 [B][T][H], sel int16 [B][T][H][mmax],
 *   err int32 (device error word). */
typedef struct TaoTrainBuffers {
  void* local;
  float* lse;
  void* fine_z;
  void* fine_c;
  void* page_prefix;
  void* num;
  float* den;
  int16_t* sel;
  int* err;
  int32_t mmax;
  int32_t flags;  /* TAO_TRAIN_CALLER_FINE_C: fine_c holds the caller's fine matrices */
} TaoTrainBuffers;

/* TaoTrainBuffers.flags bit for fine writers other than softmax (reference
 * _seal_training_all, tao_stream.py:80-123): the caller fills fine_c before
 * tao_train_forward (the writer kernel then writes fine_z only, which keeps the
 * softmax writer's z), and tao_train_backward returns dC in grads->dC for the caller
 * to differentiate; the library's writer backward then carries the z path only. */
#define TAO_TRAIN_CALLER_FINE_C 1
/* TaoTrainBuffers.flags bit for callers that apply the pointwise fusion themselves
 * (the coarse value branch fuses three terms, operator.py:21-39): tao_train_forward
 * then writes out = fine = bf16(bf16(num) / den) (zero before position 768) instead
 * of the fused output, and tao_train_backward takes grad_out = d(fine) and the
 * caller's d(local) in grads->d_local (read, not written); it returns no raw_q
 * gradient of the gate and no fusion-parameter gradients (zero). */
#define TAO_TRAIN_EXTERNAL_FUSION 2
/* TaoTrainBuffers.flags bit for the feature-read fine writers (feature-mass and
 * structured-Gram, reference tao_stream.py:87-106, 538-549, 600-601, 658-661): the
 * caller fills fine_z (bf16 log feature mass) and page_prefix (bf16 log of each
 * page's fine-order mass prefix) before tao_train_forward, which then computes the
 * local attention into buffers.local and the routing into buffers.sel only (no
 * writer, no read, `out` untouched); the caller reads the selected fines with
 * tao_feature_read_forward.  tao_train_backward then takes the caller's d(local) in
 * grads->d_local and returns the local attention's dq, dk, dv with zero d_raw_q and
 * d_raw_k (grad_out is not read). */
#define TAO_TRAIN_ROUTE_ONLY 4

/* S = T/256 - 1 sealed blocks (0 for T <= 768), pages = ceil(S/8), and the
 * largest number of selected fines any query of a T-token sequence reads. */
int tao_train_geometry(int tokens, int* sealed, int* pages, int* mmax);

/* Forward of tao_attention for [B][T][H][D] bf16 operands (index-only preset):
 * windowed local attention, softmax writer over all sealed blocks, per-query
 * routing with fresh selection, selected fine read and pointwise fusion.
 * gain: device fp32 [H] = bf16(2 * alpha_h).  Reference: tao_stream.py:668-787,
 * operator.py:21-54. */
int tao_train_forward(const void* q, const void* k, const void* v, const void* raw_q,
                      const void* raw_k, const void* fusion_a, const void* fusion_b,
                      const float* gain, int batch, int tokens, int heads, int width,
                      void* out, const TaoTrainBuffers* buffers, void* stream);

/* Gradient buffers of one backward (caller-allocated):
 *   dq, dk, dv, d_raw_q, d_raw_k : bf16 [B][T][H][D] (written completely)
 *   d_fusion_a, d_fusion_b       : fp32 [H][D][3], zero-filled (accumulated)
 *   d_local, gn, d_rq_f          : bf16 [B][T][H][D] scratch
 *   gd                           : fp32 [B][T][H] scratch
 *   row_dot                      : fp32 [B][H][T] scratch
 *   dC, dz                       : fp32 [B][H][S][D][D], [B][H][S][D]; dz zero-filled
 *   dc_partial                   : bf16 [B][H][tao_train_pairs(T)][D][D] scratch (one dC
 *                                  partial per (tile, visible fine) pair; the library
 *                                  clears what it accumulates into) */
typedef struct TaoTrainGrads {
  void* dq;
  void* dk;
  void* dv;
  void* d_raw_q;
  void* d_raw_k;
  float* d_fusion_a;
  float* d_fusion_b;
  void* d_local;
  void* gn;
  void* d_rq_f;
  float* gd;
  float* row_dot;
  float* dC;
  float* dz;
  void* dc_partial;
  float* dq_acc;  /* fp32 [B][T][H][D] scratch for the tensor-core attention backward
                     (width 64); NULL selects the mma.sync kernels */
} TaoTrainGrads;

/* Number of (256-query tile, visible fine) pairs of a T-token sequence. */
int tao_train_pairs(int tokens);

/* Backward of tao_train_forward: gradients of q, k, v, raw_q, raw_k and the
 * fusion parameters for the upstream gradient grad_out [B][T][H][D] bf16.
 * Reference: autograd of operator._fuse_training, SDPA, _SelectedRead.backward
 * (selected_read.py:175-187), the writer and page summaries. */
int tao_train_backward(const void* grad_out, const void* q, const void* k, const void* v,
                       const void* raw_q, const void* raw_k, const void* fusion_a,
                       const void* fusion_b, const float* gain, int batch, int tokens, int heads,
                       int width, const void* out, const TaoTrainBuffers* saved,
                       const TaoTrainGrads* grads, void* stream);

/* Feature-mass read of training (reference _read_training_group with a feature-read
 * writer, tao_stream.py:600-601, 658-661; feature_read_coefficients and
 * selected_fine_numerator, association_writer.py:43-53, indirect_fine.py:65-133):
 * for query t of head h, h = bf16(fp32 softmax(raw_q)); for each selected fine m
 * (sel[b][t][h][0..mmax), -1 pads, from TAO_TRAIN_ROUTE_ONLY)
 * mass_m = sum_d h_d exp(z_m,d) in fp32, w_m = mass_m / sum_m mass_m,
 * coefficient_m,d = bf16(w_m h_d) and out = bf16(sum_m sum_d coefficient_m,d C_m[d][:])
 * with fp32 accumulation (queries of the first three tiles read nothing: zero).
 * raw_q, out: bf16 [B][T][H][D]; fine_z: bf16 [B][H][S][D]; fine_c: bf16
 * [B][H][S][D][D].  The contraction runs per 128-query block and per selected fine
 * on the tensor cores (tcgen05.mma, TMEM accumulator). */
int tao_feature_read_forward(const void* raw_q, const void* fine_z, const void* fine_c,
                             const int16_t* sel, int batch, int tokens, int heads, int width,
                             int mmax, void* out, int* err, void* stream);

/* Backward of tao_feature_read_forward for grad [B][T][H][D] bf16 (the gradient of
 * out): d_raw_q bf16 [B][T][H][D] (written completely), and accumulated into the
 * caller's zero-filled fp32 buffers dz [B][H][S][D] (sum over queries of
 * bf16(d mass * h * exp(z)), the gradient of the selected z) and dc [B][H][S][D][D]
 * (sum over the selecting queries of coefficient^T grad).  Reference rounding points:
 * d coefficient = bf16(grad . C^T) (indirect_fine.py:185-206), the d z terms rounded
 * to bf16 per (query, fine, channel); the caller rounds dz and dc to bf16. */
int tao_feature_read_backward(const void* grad, const void* raw_q, const void* fine_z,
                              const void* fine_c, const int16_t* sel, int batch, int tokens,
                              int heads, int width, int mmax, void* d_raw_q, float* dz, float* dc,
                              int* err, void* stream);

/* Model-side neighbour (reference examples/common.py:6-20): split a fused Q/K/V
 * projection projected [rows][3][heads][width] bf16 (x W^T of the caller's GEMM) into
 * raw_q, raw_k, v [rows][heads][width] and q = rms_norm(raw_q), k = rms_norm(raw_k)
 * over the width: x * rsqrt(mean(x^2) + eps) in fp32 (torch's rms_norm default eps is
 * the fp32 epsilon 2^-23, its compute type's).  One warp per (row, head). */
int tao_qkv_split_norm(const void* projected, long long rows, int heads, int width, float eps, void* q,
                       void* k, void* v, void* raw_q, void* raw_k, void* stream);

/* Backward of tao_qkv_split_norm: d_projected [rows][3][heads][width] bf16 =
 * [d_raw_q + bf16(dx_q), d_raw_k + bf16(dx_k), dv] with the RMS-norm adjoint
 * dx = r dy - x r^3 sum_j(x_j dy_j) / width in fp32. */
int tao_qkv_split_norm_backward(const void* raw_q, const void* raw_k, const void* dq, const void* dk,
                                const void* dv, const void* d_raw_q, const void* d_raw_k, long long rows,
                                int heads, int width, float eps, void* d_projected, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TAO_B200_H */
