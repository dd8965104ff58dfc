/*
 * dsv2.h - C ABI of the B200 (sm_100a) DeepSeek-V2-Lite decode kernels (libdsv2.so).
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t passed as
 * void*, enqueues its kernels on that stream and returns a status code.  Nothing
 * here allocates device memory, synchronises the stream or reads device values on
 * the host, so every call can be captured in a CUDA graph.  Work buffers are owned
 * by the caller.  Integers are element counts/strides unless the name says bytes.
 *
 * Each function cites the reference (heiheiha798/Flash-DeepSeeek-V2-Lite) Python
 * function whose behaviour it provides; the Python package re-exports those names
 * on top of this ABI.
 */
#ifndef DSV2_H
#define DSV2_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DSV2_API __attribute__((visibility("default")))
#else
#define DSV2_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------------- */
#define DSV2_OK 0
#define DSV2_ERR_INVALID 1     /* bad argument (shape, alignment, null pointer)     */
#define DSV2_ERR_LAUNCH 2      /* CUDA launch/driver error                          */
#define DSV2_ERR_DEVICE 3      /* device error word set (bounded wait gave up, index) */
#define DSV2_ERR_UNSUPPORTED 4 /* shape or dtype class the kernels do not cover      */

/* ---- dtype codes ---------------------------------------------------------- */
#define DSV2_BF16 0
#define DSV2_F16 1 /* activations of dsv2_rmsnorm / dsv2_residual_add; norm weights */
#define DSV2_F32 2

/* ---- linear epilogues ----------------------------------------------------- */
#define DSV2_EPI_STORE_BF16 0 /* y = bf16(acc)                                       */
#define DSV2_EPI_STORE_F32 1  /* y = acc                                             */
#define DSV2_EPI_SWIGLU 2     /* y = bf16(silu(bf16(gate)) * bf16(up)), fp32 math    */
#define DSV2_EPI_SCALE_F32 3  /* y = bf16(acc) * route_scale[route] (fp32 store)     */
#define DSV2_EPI_ARGMAX 4     /* internal to dsv2_lm_head_argmax                     */

/* ---- linear families ------------------------------------------------------ */
#define DSV2_FAMILY_SMALL 0 /* mma.sync weight-streaming GEMV (<= 8 tokens per pass)  */
#define DSV2_FAMILY_BATCH 1 /* tcgen05/TMEM tensor-core GEMM (up to 256 tokens/tile)  */

/* Library version (major*100 + minor). */
DSV2_API int dsv2_version(void);

/* Text of the last host-side error of this thread (static storage). */
DSV2_API const char* dsv2_last_error(void);

/* One-time per-device setup: kernel attributes (large shared memory) and the SM
 * count of the current device.  Must run outside stream capture; the other entry
 * points call it lazily. */
DSV2_API int dsv2_init(void);

/* Programmatic dependent launch: every kernel is enqueued with programmatic stream
 * serialization, so it is scheduled while its predecessor in the stream drains and
 * waits on the device (griddepcontrol.wait) before touching that predecessor's outputs.
 * On by default; DSV2_PDL=0 in the environment or this call turns it off.  Returns the
 * previous setting.  Applies to launches made after the call (a captured graph keeps
 * the setting it was captured with).  No reference counterpart. */
DSV2_API int dsv2_set_programmatic_launch(int enable);

/* Number of kernels this library has enqueued in the process (all devices, all
 * streams), for launch accounting.  No reference counterpart. */
DSV2_API int64_t dsv2_kernel_launches(void);

/* ---- device error word ------------------------------------------------------
 * Kernels never trap: a bounded wait that runs out, or an index check that fails,
 * records a code in the current device's error word (first code wins) and the kernel
 * skips the offending work.  Codes: */
#define DSV2_DEVERR_TIMEOUT 1 /* a bounded wait (mbarrier, progress counter, peer) gave up */
#define DSV2_DEVERR_INDEX 2   /* token id >= vocab, position >= max_len, cache row, tile bound */
#define DSV2_DEVERR_TMEM 3    /* tensor-memory allocation failed */

/* Reads (and optionally clears) the device error word of the current device.
 * Synchronous (cudaMemcpyFromSymbol); call outside the hot loop.  Clearing a nonzero
 * word first waits for the device and also zeroes the row tickets of the array that
 * dsv2_mla_decode_noalloc uses (a launch that gave up can leave them nonzero).
 * Progress counters owned by the caller (dsv2_moe sync, dsv2_mla_decode row_sync)
 * must be zeroed by the caller after a nonzero word: dsv2_reset_progress.
 * Expert-parallel state (peer counters derived from the step count) is not
 * recoverable this way: every rank rebuilds its peer buffers. */
DSV2_API int dsv2_get_device_error(int* code, int clear);

/* Waits for `stream` (cudaStreamSynchronize) and returns DSV2_ERR_DEVICE, with the code
 * in dsv2_last_error(), when the device error word is set; DSV2_OK otherwise.  Does not
 * clear the word.  For hosts that check each step's status through the C ABI.  No
 * reference counterpart (the reference's Triton kernels have no device-side checks). */
DSV2_API int dsv2_stream_check(void* stream);

/* Zeroes `count` int32 progress counters on `stream` (cudaMemsetAsync, capturable): the
 * fused MoE's sync array and the latent attention's row_sync tickets, which every
 * successful launch leaves at zero but a launch that gave up may not.  Call after
 * reading a nonzero device error word, before the next launch that uses them.  No
 * reference counterpart. */
DSV2_API int dsv2_reset_progress(void* counters, int64_t count, void* stream);

/* ---- expert parallelism over NVLink peer memory -------------------------------- */
/* Every rank allocates one peer-visible buffer (dsv2_peer_alloc), exports it
 * (dsv2_peer_export, a 64-byte handle), the handles are exchanged by the host (e.g.
 * torch.distributed all_gather_object), and every rank maps the others' buffers
 * (dsv2_peer_import).  The same layout is used in every buffer (byte offsets):
 *   xg   [world * rows_per_rank, hidden] bf16   the router's inputs of every row
 *   ids  [world * rows_per_rank, 6] int32, w [world * rows_per_rank, 6] fp32
 *   part [rows_per_rank, 8, hidden] fp32         MoE slot outputs of this rank's rows
 *   ctr  two uint64 arrival counters, 128 bytes apart (zeroed by dsv2_peer_alloc)
 * With a table whose world > 1: the router writes its rows' inputs and routing into
 * every rank's buffer and signals (dispatch); the bucketing waits for all ranks'
 * dispatch of the MoE layer; the fused MoE writes each routed slot output into the
 * owner rank's part and signals (combine); the add+RMSNorm that consumes a MoE layer's
 * output waits for every rank's combine.  The expected counts come from *epoch (steps
 * completed; advanced by dsv2_lm_head_argmax) and the MoE layer index, so every rank
 * must run the same sequence of steps.  Waits are bounded (device error word).  The
 * reference runs on one GPU (pack_routed_experts rejects ep_size != 1,
 * moe_batch.py:325-326); no reference counterpart. */
typedef struct dsv2_peer_table {
  int32_t world; /* <= 8; 0 or 1 = single GPU */
  int32_t rank;
  void* base[8]; /* base[q] = rank q's buffer as mapped in this process */
  int64_t xg_offset, ids_offset, w_offset, part_offset, ctr_offset;
  int32_t rows_per_rank;
  int32_t n_moe_layers;
  const int64_t* epoch;
  /* polls before a cross-GPU wait gives up and sets the device error word
   * (DSV2_DEVERR_TIMEOUT); 0 = the default 2^24 (several seconds) */
  int32_t wait_polls;
  /* optional uint64[4] accumulators (NULL = none): [0] nanoseconds the CTAs of the
   * bucketing launches spent waiting for every rank's dispatch, [1] their number of
   * waits, [2] / [3] the same for the combine waits of the add+RMSNorm launches */
  uint64_t* wait_stats;
} dsv2_peer_table;

DSV2_API int dsv2_peer_alloc(size_t bytes, void** ptr);
DSV2_API int dsv2_peer_free(void* ptr);
DSV2_API int dsv2_peer_export(const void* ptr, void* handle /* 64 bytes */);
DSV2_API int dsv2_peer_import(const void* handle, void** ptr);
DSV2_API int dsv2_peer_close(void* ptr);

/* RMSNorm: y[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * w, fp32 math, one rounding to
 * x's dtype.  x_dtype DSV2_BF16 or DSV2_F16 (y has the same dtype); w_dtype DSV2_BF16,
 * DSV2_F16 or DSV2_F32.  cols % 8 == 0, cols <= 4096.
 * Reference: rmsnorm_triton, triton_kernels/rmsnorm.py:60-95 (kernel :8-57). */
DSV2_API int dsv2_rmsnorm(const void* x, int64_t x_row_stride, int x_dtype, const void* w, int w_dtype,
                 void* y, int64_t y_row_stride, int rows, int cols, float eps, void* stream);

/* Fused residual add + RMSNorm (two outputs):
 *   h_out[r] = bf16(h[r] + sum_p delta[r, p]),  y[r] = rmsnorm(h_out[r]) * w.
 * delta_dtype DSV2_BF16: delta rows at delta_row_stride, parts at delta_part_stride;
 * DSV2_F32: same, fp32 (MoE per-slot partials).  n_delta == 0 skips the add.
 * h_out == NULL updates h in place; y == NULL skips the norm.  h rows are contiguous.
 * peers (may be NULL): delta is the expert-parallel part of MoE layer moe_layer; the
 * kernel first waits until every rank has combined into it. 
 * Reference: residual_add_triton (attention_prepost.py:191-223) followed by
 * rmsnorm_triton, as applied per decoder layer in src/run.py:459-493. */
DSV2_API int dsv2_add_rmsnorm(void* h, void* h_out, const void* delta, int delta_dtype, int n_delta,
                     int64_t delta_part_stride, int64_t delta_row_stride, const void* w,
                     int w_dtype, void* y, int rows, int cols, float eps,
                     const dsv2_peer_table* peers, int moe_layer, void* stream);

/* Embedding gather + first input RMSNorm: h[r] = table[ids[r]]; y[r] = rmsnorm(h[r]) * w.
 * ids are int64; an id outside [0, vocab) sets the device error word and reads row 0.
 * Reference: the HF embedding + input_layernorm at the top of the decode step
 * (src/run.py:574-581 through model.forward). */
DSV2_API int dsv2_embed_rmsnorm(const int64_t* ids, const void* table, int64_t vocab, const void* w,
                       int w_dtype, void* h, void* y, int rows, int cols, float eps,
                       void* stream);

/* out = a + b in fp32, rounded once to the inputs' dtype (dtype DSV2_BF16 or DSV2_F16),
 * over n contiguous elements (n % 8 == 0).
 * Reference: residual_add_triton, triton_kernels/attention_prepost.py:191-223. */
DSV2_API int dsv2_residual_add(const void* a, const void* b, void* out, int64_t n, int dtype, void* stream);

/* out = bf16(silu(gate) * up) over n contiguous bf16 elements (n % 8 == 0).
 * Reference: silu_mul_triton, triton_kernels/mlp_elementwise.py:24-45. */
DSV2_API int dsv2_silu_mul(const void* gate, const void* up, void* out, int64_t n, void* stream);

/* Deterministic sum of fp32 partials: out[r, c] = sum_{p < n_parts} part[r*row_stride +
 * p*part_stride + c], added in part order, stored as out_dtype (DSV2_BF16 or DSV2_F32)
 * at out_row_stride.  Strides in elements; cols % 8 == 0; rows <= 65535.
 * Reference: the top-k route reduction _down_reduce_topk6_kernel /
 * _batched_down_reduce_topk6_kernel (moe_small_gemv.py:162-192, :311-348), here over
 * partials already scaled by the route weight (the down GEMM's epilogue). */
DSV2_API int dsv2_sum_partials(const float* part, int n_parts, int64_t part_stride, int64_t row_stride,
                      void* out, int out_dtype, int64_t out_row_stride, int rows, int cols,
                      void* stream);

/* attention_mask[b, s] = (attention_mask_index[s] <= pos_b), position_ids[b] = pos_b,
 * pos_b = cache_position[pos_numel == 1 ? 0 : b] (int64 everywhere).  Either output
 * may be NULL.  Reference: prepare_decode_inputs_triton, attention_prepost.py:152-188. */
DSV2_API int dsv2_prepare_decode_inputs(const int64_t* cache_position, int pos_numel,
                               int64_t* attention_mask, int64_t mask_stride_b,
                               int64_t* position_ids, int64_t position_ids_stride_b,
                               const int64_t* attention_mask_index, int batch, int max_len,
                               void* stream);

/* dst[b, h, pos_b, :] = src[b, h, 0, :] with element strides src_strides = {b, h, d},
 * dst_strides = {b, h, s, d}; elem_size 2 or 4.  A position outside [0, max_len)
 * sets the device error word and skips the row.
 * Reference: copy_single_token_to_cache, attention_prepost.py:113-149. */
DSV2_API int dsv2_copy_token_to_cache(const void* src, const int64_t* src_strides, void* dst,
                             const int64_t* dst_strides, const int64_t* cache_position,
                             int pos_numel, int batch, int heads, int dim, int elem_size,
                             int max_len, void* stream);

/* pos[i] += 1 for i < n (int64): the cache_position.add_(1) that closes each captured
 * decode step (src/run.py:588). */
DSV2_API int dsv2_advance_positions(int64_t* pos, int n, void* stream);

/* ---- linear layers --------------------------------------------------------- */
/* Y[row_y(t), n] = epilogue( sum_k W_g[n, k] * X_g[row_x(t), k] ) for every group g,
 * output feature n < n_rows and token t of the group.
 *   W_g = w + g * w_group_stride, rows at w_row_stride (bf16, 16-byte aligned rows)
 *   X_g = x + g * x_group_stride, rows at x_row_stride
 *   Y_g = y + g * y_group_stride, rows at y_row_stride
 * Dense mode (group_offsets == NULL): every group has n_tokens tokens, row_x = row_y = t.
 * Grouped mode: group g owns routes [group_offsets[g], group_offsets[g+1]) (device
 * memory, read by the kernel); row_x(r) = route_x_row ? route_x_row[r] : r,
 * row_y(r) = route_y_row ? route_y_row[r] : r, and max_routes_per_group bounds every
 * group's route count.  SwiGLU: the up row of feature n is W_g row n + up_offset/w_row_stride.
 * k % 32 == 0 (small family) / k % 64 == 0 (batch family).  The batch family also needs
 * w_group_rows / x_group_rows (rows spanned by one group of W / X, for the TMA bounds)
 * and route_x_row == NULL.
 * Reference: _gemv_contig_kernel / _small_batch_gemv_kernel (attention_decode_small.py:54-137,
 * :857-901), _batched_linear_kernel (attention_decode_batch.py:420-468), the grouped MoE
 * GEMMs (moe_batch.py:151-307, moe_small_gemv.py:52-158). */
typedef struct dsv2_linear_args {
  const void* w;
  int64_t w_row_stride;
  int64_t w_group_stride;
  int64_t up_offset;
  int32_t n_rows;
  int32_t k;
  const void* x;
  int64_t x_row_stride;
  int64_t x_group_stride;
  void* y;
  int64_t y_row_stride;
  int64_t y_group_stride;
  int32_t epilogue;
  int32_t n_groups;
  int32_t n_tokens;
  int32_t max_routes_per_group;
  const int32_t* group_offsets;
  const int32_t* route_x_row;
  const int32_t* route_y_row;
  const float* route_scale;
  int64_t w_group_rows;
  int64_t x_group_rows;
  /* batch family, dense mode, DSV2_EPI_STORE_F32 only: split K over k_splits CTAs
   * (1 <= k_splits <= k/64); split s writes its fp32 partial sum at y + s * y_split_stride,
   * the caller sums the partials (e.g. dsv2_add_rmsnorm with fp32 parts).  0 or 1 = no split. */
  int32_t k_splits;
  int64_t y_split_stride;
  /* batch family, grouped mode: nonzero when group_offsets (and the route arrays) were
   * written by a kernel at least two launches earlier on this stream, e.g. the MoE down
   * GEMM after bucketing -> gate_up.  The kernel then reads them, and starts streaming
   * weights, while the previous kernel is still running.  0 = no such guarantee. */
  int32_t offsets_prior;
  /* grouped mode, optional: an upper bound on the total routes group_offsets[n_groups]
   * (0 = none).  The small family then launches work only for as many groups as can hold
   * a route (at B = 1, 8 of the 66 MoE groups) instead of one CTA set per group. */
  int32_t max_routes;
  /* small family, dense, n_tokens 1, optional (x may then be NULL): the token's row of
   * group g is not read from x but merged from the partials that dsv2_mla_decode left
   * unmerged (its part_count): row = bf16(sum_c a_c o_c[g]) with
   * a_c = 2^(m_c - M) / sum_c 2^(m_c - M) l_c, partial c's o at x_parts + (2c n_groups + g) k
   * and (m, l) at x_parts_ml + (2c n_groups + g) 2, c over
   * [x_parts_count[0], x_parts_count[0] + x_parts_count[1]) (at most 160).  For the
   * un-absorb after a one-row attention: the merge is spread over the GEMV's CTAs instead
   * of one attention CTA.  No reference counterpart. */
  const float* x_parts;       /* o_part */
  const float* x_parts_ml;    /* ml_part */
  const int32_t* x_parts_count;
} dsv2_linear_args;

DSV2_API int dsv2_linear(const dsv2_linear_args* args, int family, void* stream);

/* ---- fused MoE (batch family) ------------------------------------------------ */
/* One layer's routed + shared experts in one persistent tcgen05 launch:
 *   h[r, :]            = bf16(silu(bf16(W_gate[g] x_sorted[r])) * bf16(W_up[g] x_sorted[r]))
 *   y[route_slot[r], :] = bf16(W_down[g] h[r]) * route_weight[r]
 * for every route r of group g (rows [group_offsets[g], group_offsets[g+1]) of x_sorted,
 * as the router's bucketing lays them out).  gate_up: [n_groups, 2*inter, hidden] (gate
 * rows then up rows), down: [n_groups, hidden, inter], bf16.  x_sorted / h: [x_rows,
 * hidden] / [x_rows, inter] bf16; y rows are hidden wide, fp32 (the per-slot partials the
 * next fused add+RMSNorm sums).  sync: int32[n_groups + 2], zero before the first call
 * and left zero by every call (per-group progress counters between the two GEMMs, the
 * exit ticket and the shared item counter).
 * hidden % 64 == 0, inter % 64 == 0, n_groups <= 254.  Calls that share `sync` must not
 * overlap on the GPU.
 * Reference: the grouped gate/up + SwiGLU and down kernels of packed_routed_moe
 * (moe_batch.py:151-307, launched at :425-557). */
typedef struct dsv2_moe_args {
  const void* gate_up;
  const void* down;
  int32_t n_groups;
  int32_t hidden;
  int32_t inter;
  const void* x_sorted;
  void* h;
  int32_t x_rows;
  const int32_t* group_offsets;
  int32_t max_routes_per_group;
  const int32_t* route_slot;
  const float* route_weight;
  float* y;
  int32_t* sync;
  /* world > 1: route slot s (token * 8 + k, global tokens) is written to rank
   * s / (8 * rows_per_rank)'s part instead of y, then every rank is signalled */
  const dsv2_peer_table* peers;
  /* tokens per work item (16..128, multiple of 16); 0 = the largest group's size capped
   * at 128 */
  int32_t tile_tokens;
} dsv2_moe_args;

DSV2_API int dsv2_moe(const dsv2_moe_args* args, void* stream);

/* ---- lm_head + greedy sampling ------------------------------------------------ */
/* next_ids[t] = argmax_v bf16(sum_k w[v, k] * x[t, k]) for every token t (lowest index on
 * ties, like torch.argmax over bf16 logits), without writing the logits: the linear's
 * epilogue keeps one (value, index) key per row block and token in `keys`, a second
 * launch reduces them.  When given, input_ids[t] = next_ids[t] and positions[t] += 1
 * (pos_numel 1: positions[0] += 1), closing a decode step.  w: [vocab, hidden] bf16,
 * x: [n_tokens, hidden] bf16 rows at x_row_stride; hidden % 64 == 0 (batch family) or
 * % 32 == 0 (small).  keys: uint64 work buffer of at least ceil(vocab / 16) * n_tokens
 * entries.  Reference: the greedy step of the decode loop, lm_head + argmax
 * (src/run.py:585-586).  step_counter (may be NULL) is incremented once: the epoch of
 * an expert-parallel peer table. */
DSV2_API int dsv2_lm_head_argmax(const void* w, int vocab, int hidden, const void* x,
                                 int64_t x_row_stride, int n_tokens, uint64_t* keys,
                                 int64_t keys_capacity, int64_t* next_ids, int64_t* input_ids,
                                 int64_t* positions, int pos_numel, int64_t* step_counter,
                                 int family, void* stream);

/* ---- MoE routing ------------------------------------------------------------ */
/* Gate GEMV (fp32 over bf16 activations) + softmax + top-6, then bucketing.
 *   logits[r, e] = sum_k x[r, k] * w[e, k] (+ bias[e]);  p = softmax(logits[r]);
 *   topk_ids / topk_weights = 6 largest p (descending, lowest index first on ties),
 *   weights multiplied by `scaling` (routed_scaling_factor).
 * When group_offsets != NULL the routes of experts [expert_lo, expert_lo + n_local) are
 * bucketed (stable, ascending (token, k) order) into n_local groups followed by two
 * shared-expert groups holding rows [shared_lo, shared_hi) with weight 1:
 *   group_offsets[n_local + 3], route_token / route_slot / route_weight[6*rows + 2*shared rows],
 *   route_slot = token * 8 + k (k = 0..5 routed, 6..7 the two shared-expert halves).
 * gather_out (optional, needs bucketing): [routes, hidden] bf16, row i = x[route_token[i]]
 * (the expert-ordered activations the batch-family MoE GEMMs read with TMA).
 * logits: [rows, n_experts] fp32 work buffer.  topk_ids64 may be NULL.  hidden % 64 == 0,
 * hidden <= 2048, rows <= 4096.
 * Reference: router_softmax_topk6_triton (moe_router.py:63-86) with the fp32 gate linear of
 * src/run.py:257-275, and the bucketing of packed_routed_moe (moe_batch.py:101-148, 425-470). */
typedef struct dsv2_router_args {
  const void* x;
  int64_t x_row_stride;
  const void* w;
  int32_t w_dtype;
  int32_t rows;
  int32_t hidden;
  int32_t n_experts;
  const float* bias;
  float scaling;
  float* logits;
  int64_t* topk_ids64;
  int32_t* topk_ids32;
  float* topk_weights;
  void* gather_out;
  int32_t expert_lo;
  int32_t n_local;
  int32_t shared_lo;
  int32_t shared_hi;
  int32_t* group_offsets;
  int32_t* route_token;
  int32_t* route_slot;
  float* route_weight;
  /* world > 1: also write x / top-6 ids / weights of these rows (global rows
   * row_base ..) into every rank's buffer and signal (no bucketing here then) */
  const dsv2_peer_table* peers;
  int32_t row_base;
  /* optional residual add + RMSNorm that forms the router's input in the same launch
   * (bf16 gate, one rank): h[r] = bf16(h[r] + sum_p delta[r, p]) and
   * x[r] = rmsnorm(h[r]) * norm_w, bit for bit what dsv2_add_rmsnorm(h, NULL, delta, ...,
   * norm_w, ..., y = x) computes; x is then an output (rows at x_row_stride).  delta as in
   * dsv2_add_rmsnorm (DSV2_BF16 rows or DSV2_F32 per-part partials); h == NULL: none. */
  void* h;
  const void* delta;
  int32_t delta_dtype;
  int32_t n_delta;
  int64_t delta_part_stride;
  int64_t delta_row_stride;
  const void* norm_w;
  int32_t norm_w_dtype;
  float eps;
  /* optional int32[2], zeroed once before first use and never by the caller again: the
   * grid barrier that lets the bucketing (and gather) run in the same launch as the gate
   * (bf16 gate, one rank).  NULL: the bucketing is a second launch. */
  int32_t* sync;
} dsv2_router_args;

DSV2_API int dsv2_router(const dsv2_router_args* args, void* stream);

/* Softmax + top-6 over precomputed fp32 logits [rows, n_experts] (n_experts <= 64).
 * Reference: router_softmax_topk6_triton, triton_kernels/moe_router.py:63-86. */
DSV2_API int dsv2_softmax_topk(const float* logits, int rows, int n_experts, float scaling,
                      int64_t* topk_ids64, int32_t* topk_ids32, float* topk_weights,
                      void* stream);

/* Bucketing alone (expert parallel: over every rank's rows); same outputs as
 * dsv2_router.  gather_out (optional): row i = gather_src[route_token[i]] (row stride
 * gather_src_stride, cols columns).  peers (may be NULL): the ids / weights / gather
 * source are the peer buffer's, and the kernel first waits for every rank's dispatch of
 * MoE layer moe_layer.  Reference: moe_batch.py:101-148. */
DSV2_API int dsv2_moe_bucket(const int32_t* topk_ids32, const float* topk_weights, int rows,
                    int expert_lo, int n_local, int shared_lo, int shared_hi,
                    int32_t* group_offsets, int32_t* route_token, int32_t* route_slot,
                    float* route_weight, const void* gather_src, int64_t gather_src_stride,
                    void* gather_out, int cols, const dsv2_peer_table* peers, int moe_layer,
                    void* stream);

/* out[r] = x[route_token[r]] for r < group_offsets[n_groups] (r < max_routes): gathers
 * activations into expert-contiguous rows for the batch family.  cols % 8 == 0. */
DSV2_API int dsv2_gather_rows(const void* x, int64_t x_row_stride, const int32_t* route_token,
                     const int32_t* group_offsets, int n_groups, void* out, int cols,
                     int max_routes, void* stream);

/* ---- multi-head latent attention ----------------------------------------------- */
/* New-token preparation for one layer: from qkva[b] = [q (16 x 192) | c_kv (512) | k_pe (64)]
 *   cache[b, pos_b, 0:512]   = bf16(rmsnorm(c_kv) * kv_norm_w)
 *   cache[b, pos_b, 512:576] = rope(k_pe, pos_b)          (interleaved pairs 2j, 2j+1)
 *   q_pe_out[b, h, :]        = rope(q[b, h, 128:192], pos_b)
 * cos/sin: [rope_rows, rope_stride] fp32, entries 0..31 used (attention scaling folded in).
 * Reference: _build_qkv_rope_kernel + _cache_write_q1_dual_kernel
 * (attention_decode_small.py:140-339) and the kv-a RMSNorm (:581). */
typedef struct dsv2_mla_prep_args {
  const void* qkva;
  int64_t qkva_row_stride;
  const void* kv_norm_w;
  float eps;
  const float* cos_tab;
  const float* sin_tab;
  int64_t rope_stride;
  int32_t rope_rows;
  const int64_t* positions;
  int32_t pos_numel;
  void* cache;
  int64_t cache_b_stride;
  int32_t max_len;
  void* q_pe_out;
  int32_t batch;
  /* qkva element type: DSV2_BF16 (one [B, 3648] matrix) or DSV2_F32 (qkva_parts split-K
   * partial sums at qkva + p * qkva_part_stride, summed and rounded to bf16 here) */
  int32_t qkva_dtype;
  int32_t qkva_parts;
  int64_t qkva_part_stride;
  /* optional [B, 16, 128] bf16 copy of q_nope (the input of the absorbed projection) */
  void* q_nope_out;
  /* optional int32[batch]: the cache row (sequence) of each input row, so that several
   * tokens of one sequence are prepared at once (kernel prefill); NULL = row b is cache
   * row b.  cache_batch = rows of the cache (0 = batch). */
  const int32_t* cache_rows;
  int32_t cache_batch;
} dsv2_mla_prep_args;

DSV2_API int dsv2_mla_prep(const dsv2_mla_prep_args* args, void* stream);

/* Latent attention for q_len = 1:
 *   score[h, s] = softmax_scale * (q_abs[b, h] . cache[b, s, :512] + q_pe[b, h] . cache[b, s, 512:])
 *   o_lat[b, h] = sum_{s <= pos_b} softmax(score)[h, s] * cache[b, s, :512]   (bf16 out)
 * for 16 heads.  o_part (batch * n_splits * 16 * 512 fp32) and ml_part (batch * n_splits *
 * 16 * 2 fp32) are caller work buffers.
 * DSV2_FAMILY_SMALL (one launch): the cache tiles of all rows are spread evenly over at
 * most one CTA per SM; split_len (multiple of 32) = fewest positions per CTA; the buffers
 * hold batch * n_splits partial slots, two per CTA (so at most batch * n_splits / 2
 * CTAs); row_sync is required.
 * DSV2_FAMILY_BATCH (two launches, split + merge): split_len (multiple of 64) positions
 * per CTA, o_part [batch, n_splits, 16, 512] with n_splits >= ceil(max_len / split_len).
 * Reference: _decode_attention_q1_kernel / _batched_decode_attention_q1_kernel
 * (attention_decode_small.py:342-423, attention_decode_batch.py:240-342) over the
 * expanded cache; here over the latent cache. */
typedef struct dsv2_mla_decode_args {
  const void* q_abs;
  const void* q_pe;
  const void* cache;
  int64_t cache_b_stride;
  int32_t max_len;
  const int64_t* positions;
  int32_t pos_numel;
  float softmax_scale;
  int32_t split_len;
  int32_t n_splits;
  float* o_part;
  float* ml_part;
  void* o_lat;
  int32_t batch;
  /* nonzero when q_pe, positions and the cache were written at least two launches earlier
   * on this stream (only q_abs may come from the previous launch, e.g. prep -> absorb ->
   * decode): the kernel then starts loading cache tiles while the previous kernel is still
   * running.  0 = no such guarantee. */
  int32_t inputs_prior;
  /* int32[batch], zero before the first call and left zero by every call: the last CTA
   * of a row cut between CTAs merges the row's partials (DSV2_FAMILY_SMALL: required;
   * DSV2_FAMILY_BATCH: must be NULL). */
  int32_t* row_sync;
  /* DSV2_FAMILY_SMALL: mma.sync kernel (32-position tiles, balanced persistent grid);
   * DSV2_FAMILY_BATCH: tcgen05/TMEM kernel (64-position tiles, split grid + merge). */
  int32_t family;
  /* optional int32[batch] (DSV2_FAMILY_SMALL only): the cache row (sequence) each query
   * row attends to, so that many query tokens of one sequence attend at once (kernel
   * prefill, causal through their positions); NULL = query row b reads cache row b.
   * cache_batch = rows of the cache (0 = batch). */
  const int32_t* cache_rows;
  int32_t cache_batch;
  /* optional int32[2] (DSV2_FAMILY_SMALL, batch 1): leave the row's partials unmerged for
   * the next linear (dsv2_linear_args.x_parts) instead of merging them in one CTA and
   * writing o_lat: CTA c stores its (o, m, l) in partial slot 2c, and the launch stores
   * {first CTA, number of CTAs} holding the row's tiles here.  o_lat is not written, the
   * row tickets are not used.  NULL = merge as usual.  No reference counterpart. */
  int32_t* part_count;
} dsv2_mla_decode_args;

DSV2_API int dsv2_mla_decode(const dsv2_mla_decode_args* args, void* stream);

/* Allocation-free form of dsv2_mla_decode, for callers that cannot call cudaMalloc:
 * an embedding runtime that has already handed all device memory to its own pool,
 * a foreign-language host (through an FFI) with no CUDA allocator of its own, or a
 * latency-critical decode thread where cudaMalloc's implicit device synchronisation
 * is not acceptable.  No counterpart in the reference (its attention wrappers
 * allocate their outputs and workspaces with torch).
 * Runs the DSV2_FAMILY_SMALL kernel; its partials (256 slots, so at most 128 CTAs) and
 * row tickets (batch <= 4096, else DSV2_ERR_INVALID with a message) live in a fixed
 * device array inside libdsv2.so (8.4 MB, held by every GPU that loads the library
 * until the process exits).  The caller still passes every input and
 * the o_lat output, laid out as for dsv2_mla_decode.
 * The first call of any libdsv2 entry point on a device (or dsv2_init) looks up that
 * array's device address (cudaGetSymbolAddress) together with the kernels'
 * shared-memory attributes, under the library's lock; make that first call before any
 * stream capture.  The address is cached per device index for the life of the
 * process: after cudaDeviceReset, reload the library.  Between successful calls
 * nothing needs clearing (every partial the merge reads is written earlier in the same
 * call, and every call leaves the row tickets at zero).  A call that gives up on a
 * bounded wait sets the device error word and may leave tickets nonzero; clearing the
 * word with dsv2_get_device_error(&code, 1) zeroes them.  All calls share the one
 * array, so calls that overlap on the GPU (different streams, or several host threads)
 * race and corrupt each other's results: serialise them. */
DSV2_API int dsv2_mla_decode_noalloc(const void* q_abs, const void* q_pe, const void* cache,
                                     int64_t cache_b_stride, int max_len, const int64_t* positions,
                                     int pos_numel, float softmax_scale, int split_len, void* o_lat,
                                     int batch, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSV2_H */
