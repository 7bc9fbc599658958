/* b200quant.h -- C ABI of libb200quant.so, the B200 (sm_100a) implementation
 * of the GGML block-quant matvec/matmul and MoE FFN hot path of the LocalAI
 * reference engine.
 *
 * Part 1 replaces the reference's native library symbol for symbol
 * (engine/native_quant.cpp:705-768, bound by ctypes in
 * engine/native_quant.py:76-94).  Pointers are caller-owned HOST memory; the
 * call copies inputs to the GPU, runs the kernel, copies the result back and
 * returns when the result is in ``out``.  ``threads`` is accepted for ABI
 * compatibility and ignored.  The reference functions return nothing; here a
 * failure is reported through b200q_last_status()/b200q_last_error(), which
 * the Python wrapper checks after every call.
 *
 * Part 2 is the device-pointer API used by the PyTorch host code: all
 * pointers are device memory, work is enqueued on ``stream`` (a
 * cudaStream_t, NULL = legacy default stream) and the call returns without
 * synchronising.  Status: 0 = ok, negative = error (message in
 * b200q_last_error()).
 *
 * Calls are serialised by one library lock, like the reference's pool mutex
 * (engine/native_quant.cpp:361-363).
 */
#ifndef B200QUANT_H
#define B200QUANT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define B200Q_OK 0
#define B200Q_EINVAL (-1)      /* bad type, size, pointer or alignment */
#define B200Q_ECUDA (-2)       /* CUDA runtime error */
#define B200Q_ETIMEOUT (-3)    /* a device-side wait hit its time limit */
#define B200Q_ENODEV (-4)      /* no usable CUDA device */
#define B200Q_EINDEX (-5)      /* a device-side index check failed */

/* ---- Part 1: drop-in for engine/native_quant.cpp ---------------------- */
/* engine/native_quant.cpp:705-709 */
void localai_q8_0_matvec(const uint8_t *raw, const float *x, float *out, int rows, int cols, int threads);
/* engine/native_quant.cpp:711-717 */
void localai_q4_0_matvec(const uint8_t *raw, const float *x, float *out, int rows, int cols, int threads);
/* engine/native_quant.cpp:719-725 */
void localai_q4k_matvec(const uint8_t *raw, const float *x, float *out, int rows, int cols, int threads);
/* engine/native_quant.cpp:726-732 */
void localai_q5k_matvec(const uint8_t *raw, const float *x, float *out, int rows, int cols, int threads);
/* engine/native_quant.cpp:733-738 */
void localai_q6k_matvec(const uint8_t *raw, const float *x, float *out, int rows, int cols, int threads);
/* engine/native_quant.cpp:744-748; vectors [tokens][cols], out [rows][tokens] */
void localai_q8_0_matmul(const uint8_t *raw, const float *vectors, float *out, int rows, int cols, int tokens,
                         int threads);
/* engine/native_quant.cpp:749-753 */
void localai_q4_0_matmul(const uint8_t *raw, const float *vectors, float *out, int rows, int cols, int tokens,
                         int threads);
/* engine/native_quant.cpp:754-758 */
void localai_q4k_matmul(const uint8_t *raw, const float *vectors, float *out, int rows, int cols, int tokens,
                        int threads);
/* engine/native_quant.cpp:759-763 */
void localai_q5k_matmul(const uint8_t *raw, const float *vectors, float *out, int rows, int cols, int tokens,
                        int threads);
/* engine/native_quant.cpp:764-768 */
void localai_q6k_matmul(const uint8_t *raw, const float *vectors, float *out, int rows, int cols, int tokens,
                        int threads);

/* Batched calls of the five localai_*_matmul functions (the reference's
 * prefill path, decoded_matmul_row, engine/native_quant.cpp:620-703) with at
 * least ``tokens`` tokens (default 32) run on the tcgen05 tensor cores -- bf16
 * operands, f32 accumulation, normwise error ~3e-3 -- when the weights are
 * Q4_K, Q6_K or Q8_0 with a multiple of 128 rows and packed rows of whole
 * 16-byte units (Q4_K: any cols; Q8_0: cols % 256 == 0; Q6_K: cols % 2048 ==
 * 0); every other call runs the f32 GEMV (~1e-6).  0 keeps every call on the
 * GEMV; a negative value only queries.  Returns the previous setting. */
int b200q_matmul_tensor_core_min_tokens(int tokens);

/* Status of the last call made by this process (B200Q_* code) and its
 * message.  Replaces the reference's silent failure / None return
 * (engine/native_quant.py:66-99). */
int b200q_last_status(void);
const char *b200q_last_error(void);

/* Select and initialise the CUDA device used by Part 1 (default 0). */
int b200q_init(int device);

/* Host weight registry.  Registering an immutable host range (e.g. the
 * tensor data of an mmap'd GGUF file, engine/gguf_parser.py:153-156) uploads
 * it once; later Part-1 calls whose ``raw`` lies inside the range use the
 * device copy instead of copying the weights again.  Unregister before the
 * host memory is unmapped (GGUFFile.close, engine/gguf_parser.py:83-86). */
int b200q_register_host(const void *ptr, size_t nbytes);
int b200q_unregister_host(const void *ptr);
int b200q_registry_clear(void);
/* Device address of a registered host byte (NULL if not registered). */
void *b200q_registered_device_ptr(const void *host_ptr);

/* ---- Part 2: device-pointer API --------------------------------------- */
/* Exact f32 dequantization of nblocks GGML blocks (engine/dequant.py:27-167). */
int b200q_dequant_f32_dev(int ggml_type, const void *w, float *out, long long nblocks, void *stream);
/* bf16 dequantization (rounded from the exact f32 values). */
int b200q_dequant_bf16_dev(int ggml_type, const void *w, void *out_bf16, long long nblocks, void *stream);

/* y[t*ys_t + r*ys_r] = sum_c W[r][c] * x[t*cols + c], f32 accumulate.
 * W: raw GGUF bytes of a [rows, cols] matrix (2-byte aligned; the
 * unquantised types F32 = 0 and F16 = 1 need 16-byte alignment and cols a
 * multiple of 8); x: f32 [tokens][cols], 16-byte aligned.  Replaces the math of
 * localai_*_matvec/matmul (engine/native_quant.cpp:126-337, :620-681).
 * Allocates nothing; launched with programmatic dependent launch, so the
 * weight stream may start before the previous kernel of ``stream`` ends
 * (W must not be written by that kernel). */
int b200q_gemv_dev(int ggml_type, const void *w, const float *x, float *y, int rows, int cols, int tokens,
                   long long ys_t, long long ys_r, void *stream);

/* Grouped GEMM on the tcgen05 tensor cores with in-kernel Q4_K dequant
 * (bf16 operands, f32 accumulation; the batched path of
 * engine/native_quant.cpp:620-703 and the expert products of
 * engine/zaya.py:303-306).  Group g owns activation rows
 * [row_off[g], row_off[g+1]) of x_bf16 [x_rows, k] (row_off: device int32
 * [groups+1]) and the weight rows [wg*w_rows_per_group, ...) of the raw Q4_K
 * tensor w (rows of ceil(k/256) super-blocks; k a multiple of 64), where
 * wg = group_w[g] if group_w (device int32 [groups]) is given, else g;
 * n_weight_groups is the number of weight groups w holds (needed with
 * group_w).
 *   up_offset <  0: plain mode, out[row*ld_out + n] = x_row . w_n (times
 *                   row_scale[row] if row_scale != NULL), n < n_feat (multiple
 *                   of 128); out is f32, or bf16 when out_is_bf16 != 0;
 *   up_offset >= 0: gate/up mode over n_feat features (multiple of 64):
 *                   act[row*ld_act + f] = bf16(SiLU(x.w_f) * (x.w_{f+up_offset})),
 *                   SiLU as engine/zaya.py:305.
 * max_ctas limits the persistent grid (0 = one CTA per SM). */
int b200q_gemm_q4k_dev(const void *x_bf16, long long x_rows, int k, const void *w, int groups, int w_rows_per_group,
                       int up_offset, int n_feat, const int *row_off, const int *group_w, int n_weight_groups,
                       void *out, int out_is_bf16, long long ld_out, const float *row_scale, void *act_bf16,
                       long long ld_act, int max_ctas, void *stream);

/* ---- MoE layer stages (engine/zaya.py:274-307, generalised to top-k) ----
 * All buffers are device memory owned by the caller; nothing is allocated. */
/* ZAYA router chain steps (engine/zaya.py:274-307), f32, one row per token:
 * state = x (+ prev * w_eda when both are given), out = rmsnorm(state) * norm_w
 * (x / sqrt(mean(x^2) + eps) * w, engine/model.py:82).  prev/w_eda may be NULL. */
int b200q_zaya_router_prep_dev(const float *x, const float *prev, const float *w_eda, const float *norm_w, int T,
                               int R, float eps, float *state, float *out, void *stream);
/* In place exact GELU: x * (1 + erf(x / sqrt 2)) / 2 (engine/zaya.py:181-186). */
int b200q_gelu_dev(float *x, long long n, void *stream);
/* Copy bf16 rows [offsets[group], offsets[group+1]) of src [*, D] into dst
 * (D a multiple of 8, 16-byte aligned rows; at most max_rows rows): the
 * output rows of ZAYA's skip route are the routed input rows. */
int b200q_copy_rows_range_dev(const void *src_bf16, void *dst_bf16, const int *offsets, int group, int D,
                              int max_rows, void *stream);
/* Dense FFN activation (engine/model.py:161-166): out[t * ld_out + f] =
 * silu(gu[t, f]) * gu[t, F + f] for f32 gu [T, 2F] (gate columns, then up
 * columns), ld_out >= F; silu(g) = g / (1 + exp(-clip(g, -80, 80))). */
int b200q_silu_mul_dev(const float *gate_up, int T, int F, float *out, long long ld_out, void *stream);
/* Grouped decode GEMV (MoE experts at small batch): for every group g with
 * tokens n_g = grp_off[g+1] - grp_off[g] (device array, e.g. the dispatch
 * offsets; every n_g <= max_tokens <= 64), y[grp_off[g] + t, r] =
 * sum_c W_g[r, c] * x[grp_off[g] + t, c] for r < rows, with W_g = the raw
 * GGUF rows at w + g * w_group_stride bytes, x f32 rows of cols values, y
 * rows ys_t floats apart; weight rows w_row_bytes apart (0: packed; a padded
 * stride's tail bytes are not read).  Groups without tokens read no weights.
 * active_groups: how many groups are expected to hold tokens (sizes the
 * grid).  max_tokens may not exceed b200q_gemv_grouped_max_tokens(type, cols)
 * (the quantised activations of one group live in shared memory).  x and y
 * hold x_rows rows; a group whose offsets fall outside them (or exceed
 * max_tokens) is skipped and the device error word set (B200Q_EINDEX).  f32
 * accumulation as b200q_gemv_dev. */
int b200q_gemv_grouped_max_tokens(int ggml_type, int cols);
int b200q_gemv_grouped_dev(int ggml_type, const void *w, long long w_group_stride, long long w_row_bytes,
                           int n_groups, const int *grp_off, const float *x, float *y, long long ys_t, int rows,
                           int cols, int max_tokens, int x_rows, int active_groups, void *stream);
/* out[s, :] = h[token_of[s], :] for s < S (f32 rows of D values, D % 4 == 0);
 * h has h_rows rows: a row whose token is outside [0, h_rows) is left
 * unwritten and the device error word set (B200Q_EINDEX). */
int b200q_moe_gather_f32_dev(const float *h, int h_rows, const int *token_of, int S, int D, float *out, void *stream);
/* out[s, :] = h_bf16[token_of[s], :] for s < S (bf16 rows of D values,
 * D % 8 == 0, both 16-byte aligned); same index contract as
 * b200q_moe_gather_f32_dev. */
int b200q_moe_gather_bf16_dev(const void *h_bf16, int h_rows, const int *token_of, int S, int D, void *out,
                              void *stream);
/* The same rows by token: out[slot_of[t * k + j]] = h_bf16[t] for every pair
 * with a slot (slot_of >= 0; slot_of as b200q_moe_dispatch_dev writes it,
 * [T * k]); each row is read once and stored k times (k <= 32).  A slot at or
 * past S sets the device error word. */
int b200q_moe_scatter_bf16_dev(const void *h_bf16, int T, const int *slot_of, int k, int S, int d_model, void *out,
                               void *stream);
/* Grouped GEMM as b200q_gemm_q4k_dev for Q4_K (12), Q5_K (13), Q6_K (14),
 * Q8_0 (8) or Q4_0 (2) weights.  w_row_bytes is the byte distance between
 * weight rows (0: packed rows of k values); it must be a multiple of 16, so
 * rows whose packed size is not (Q6_K with k not a multiple of 2048, Q8_0
 * with k not a multiple of 256, Q4_0 with k not a multiple of 256) need a
 * padded copy.  Q6_K needs k a multiple of 256 when rows are packed; every
 * type needs k a multiple of 64. */
int b200q_gemm_dev(int ggml_type, const void *x_bf16, long long x_rows, int k, const void *w, long long w_row_bytes,
                   int groups, int w_rows_per_group, int up_offset, int n_feat, const int *row_off,
                   const int *group_w, int n_weight_groups, void *out, int out_is_bf16, long long ld_out,
                   const float *row_scale, void *act_bf16, long long ld_act, int max_ctas, void *stream);
/* logits[t*E + e] = h[t] . wr[e] + bias[e] (f32; bias may be NULL). */
int b200q_moe_router_dev(const float *h, const float *wr, const float *bias, float *logits, int T, int E, int D,
                         void *stream);
/* Softmax over each row of logits (f32, max-subtracted, engine/zaya.py:290),
 * selection on p + sel_bias (sel_bias may be NULL, :295), the k largest with
 * the lower expert index first on ties (:296 for k = 1); w = p[e], divided by
 * the sum of the k selected probabilities when renormalize != 0. */
int b200q_moe_topk_dev(const float *logits, const float *sel_bias, int T, int E, int k, int renormalize, int *ids,
                       float *w, void *stream);
/* Router + top-k in one call (b200q_moe_router_dev followed by
 * b200q_moe_topk_dev).  For few tokens the router's K range is split across
 * CTAs; the partial sums then go to ``workspace`` (f32, at least
 * b200q_moe_route_workspace_bytes(T, E, D) bytes; may be NULL when that is 0,
 * in which case the split is not used) and are added in a fixed order, so the
 * logits may differ from b200q_moe_router_dev's in the last bits but are
 * deterministic for a given (T, E, D) and GPU model.  ``logits`` receives the
 * final logits (bias included) in both cases. */
size_t b200q_moe_route_workspace_bytes(int T, int E, int D);
int b200q_moe_route_dev(const float *h, const float *wr, const float *bias, const float *sel_bias, int T, int E, int D,
                        int k, int renormalize, float *logits, int *ids, float *w, void *workspace,
                        size_t workspace_bytes, void *stream);
/* b200q_moe_route_dev that also writes h_bf16 [T, D] = bf16(h) (8-byte
 * aligned), converted while the router stages h (the rows the tensor-core
 * experts read, gathered by b200q_moe_gather_bf16_dev). */
int b200q_moe_route_bf16_dev(const float *h, const float *wr, const float *bias, const float *sel_bias, int T, int E,
                             int D, int k, int renormalize, float *logits, int *ids, float *w, void *workspace,
                             size_t workspace_bytes, void *h_bf16, void *stream);
/* Scratch rows needed by b200q_moe_dispatch_dev: block_counts and base are
 * int32 [b200q_moe_num_blocks(T) * E]. */
int b200q_moe_num_blocks(int T);
/* Stable counting sort of the T*k routed pairs by expert (slot order inside an
 * expert follows (token, j) order): offsets int32 [E+1], slot_of int32 [T*k],
 * token_of int32 [T*k], slot_w f32 [T*k] (routing weight per slot), and, if
 * xperm_bf16 != NULL, xperm[slot] = bf16(h[token_of[slot]]) (bf16 [T*k, D];
 * h 16-byte and xperm 8-byte aligned, D % 4 == 0).  A pair whose expert id is
 * outside [0, E) gets slot_of = -1 and no slot (offsets[E] < T*k), and the
 * device error word is set (B200Q_EINDEX from b200q_check_device_error). */
int b200q_moe_dispatch_dev(const int *ids, const float *w, int T, int k, int E, const float *h, int D,
                           int *block_counts, int *base, int *offsets, int *slot_of, int *token_of, float *slot_w,
                           void *xperm_bf16, void *stream);
/* Allocation-free variant of b200q_moe_dispatch_dev, with no counterpart in
 * the reference.  For callers that must not allocate device memory (a plugin
 * inside a host framework whose memory pool owns the device budget, or a
 * latency-critical loop that cannot take cudaMalloc's implicit
 * synchronisation): the counting-sort scratch lives in a file-scope device
 * array of 256 KB that every GPU loading the library keeps until exit, so the
 * call needs no block_counts/base buffers and calls no cudaMalloc, cudaFree or
 * allocating library routine.  Limit: b200q_moe_num_blocks(T) * E <= 32768
 * (larger calls return B200Q_EINVAL with a message).  Every call looks up the
 * array's device address on the current device (no allocation); the first
 * call on a device also loads the library's device code there, so make it
 * before any stream capture.  All calls share the array (it keeps the last
 * call's contents; nothing in it must start at zero because each call writes
 * every entry it reads), so calls that overlap on the GPU race.  A bad expert
 * id is handled as in b200q_moe_dispatch_dev; it is recorded in an error word
 * inside the array, which b200q_check_device_error reads and clears. */
int b200q_moe_dispatch_noalloc_dev(const int *ids, const float *w, int T, int k, int E, const float *h, int D,
                                   int *offsets, int *slot_of, int *token_of, float *slot_w, void *xperm_bf16,
                                   void *stream);
/* y[t] = sum_{j<k} w_j * out[slot_of[t*k + j]] in j order (f32 [T, D]), with
 * w_j = slot_w[slot] if slot_w != NULL, else 1 (rows already weighted); the
 * rows of out (T*k of them) are f32, or bf16 when out_is_bf16 != 0.  A slot
 * outside [0, T*k) -- the dispatch writes -1 for a pair whose expert id was
 * out of range -- adds nothing. */
int b200q_moe_combine_dev(const void *out, int out_is_bf16, const int *slot_of, const float *slot_w, int T, int k,
                          int D, float *y, void *stream);

/* Device error word: returns and clears the sticky kernel error of the
 * current device (0 if none), including the error word of
 * b200q_moe_dispatch_noalloc_dev.  Synchronises the device. */
int b200q_check_device_error(void);

/* Tuning knobs of the GEMV: bytes of weights per pipeline stage, stage
 * count, the most rows one consumer group handles per stage (1, 2 or 4),
 * and the most CTAs per SM in the grid (0 = as many as fit); 0 (-1 for the
 * last) keeps the current value. */
void b200q_gemv_tuning(int stage_bytes, int stages, int rows_per_group, int ctas_per_sm);
/* Batch-1 Q4_K GEMV on the integer tensor cores (used by b200q_gemv_dev and
 * the localai_q4k_matvec drop-in when the weights are 16-byte aligned):
 * enable (1) or disable (0; -1 keeps), super-blocks per warp per pipeline
 * stage (1..3, 0 = automatic), stages per warp (0 = as many as fit in half an
 * SM's shared memory) and CTAs of one launch per SM (1 or 2; with 1 the other
 * slot runs the next launch's weight stream); -1 keeps a setting. */
void b200q_gemv_mma_tuning(int enable, int sb_per_warp, int stages, int ctas_per_sm);
/* Tensor-core grouped GEMM (b200q_gemm_q4k_dev, b200q_gemm_dev, the batched
 * localai_*_matmul drop-ins, the MoE and expert-parallel layers): 1 (default)
 * runs every tile on a pair of SMs (tcgen05 cta_group::2, M = 256 weight rows
 * x N = 256 activation rows, each SM loading half of the activation tile);
 * 0 runs one tile per SM (M = 128); -1 keeps the mode.  Results are
 * identical.  Returns the number of SM pairs the last pair launch used. */
int b200q_gemm_pair_mode(int on);

/* Number of kernel launches made by this library since load. */
long long b200q_launch_count(void);

/* ---- Expert-parallel exchange over NVLink peer memory (no reference
 * counterpart: the reference runs the MoE block in one CPU process).  One
 * context per rank (one process per GPU); every rank makes the same calls in
 * the same order with the same epoch (1, 2, ... per layer call), or with
 * epoch 0 in every call: the count exchange then advances a device-side
 * counter that the later calls of the layer call read (no per-call host
 * argument, so a layer call can be captured in a CUDA graph and replayed).
 *   b200q_ep_create        allocate this rank's exchange region (counts inbox,
 *                          flags, receive rows bf16 [max_recv_rows, d_model],
 *                          return rows bf16 [max_send_rows, d_model]);
 *   b200q_ep_handle        its CUDA IPC handle (b200q_ep_handle_bytes bytes),
 *                          to be all-gathered by the caller;
 *   b200q_ep_open          map every other rank's region (handles of all
 *                          ranks, rank order); collective;
 *   b200q_ep_exchange_counts_dev  offsets [world * local_experts + 1] of this
 *                          rank's slots sorted by (owner rank, local expert)
 *                          (b200q_moe_dispatch_dev on virtual expert ids);
 *   b200q_ep_send_rows_dev gather h[token_of[slot]] as bf16 into the owner's
 *                          receive buffer (expert-major; in a group the
 *                          receiver's own rows first, then ranks r+1, ...);
 *   b200q_ep_experts_dev   wait for all ranks' rows, gate/up then down on the
 *                          local experts (weights as for b200q_gemm_dev: type,
 *                          row strides, 0 = packed); the down GEMM stores each output row
 *                          (unweighted, bf16) into its source rank's return
 *                          buffer; then signal every rank.  act: bf16
 *                          [max_recv_rows, d_ff] scratch;
 *   b200q_ep_combine_dev   wait for all ranks' outputs, y[t] = sum_j
 *                          slot_w * ret[slot(t, j)] (f32 [T, d_model]).
 * Waits give up after 5 s (b200q_ep_set_wait_limit_ns changes the limit for
 * later launches; 0 restores 5 s) and set the device error word
 * (b200q_check_device_error reports B200Q_ETIMEOUT).  b200q_ep_destroy must be
 * called on all ranks after a barrier. */
int b200q_ep_create(int world, int rank, int local_experts, int d_model, long long max_send_rows,
                    long long max_recv_rows, void **ep);
size_t b200q_ep_handle_bytes(void);
void b200q_ep_set_wait_limit_ns(unsigned long long ns);
int b200q_ep_handle(void *ep, void *handle);
int b200q_ep_open(void *ep, const void *handles);
int b200q_ep_destroy(void *ep);
void *b200q_ep_recv_rows(void *ep);
void *b200q_ep_return_rows(void *ep);
const int *b200q_ep_group_offsets(void *ep);
int b200q_ep_exchange_counts_dev(void *ep, const int *offsets, unsigned int epoch, void *stream);
int b200q_ep_send_rows_dev(void *ep, const float *h, int T, const int *token_of, const int *offsets, int slots,
                           unsigned int epoch, void *stream);
/* b200q_ep_send_rows_dev from bf16 rows (h_bf16 [T, D], 16-byte aligned, e.g.
 * the copy b200q_moe_route_bf16_dev writes): the rows are copied as they are. */
int b200q_ep_send_rows_bf16_dev(void *ep, const void *h_bf16, int T, const int *token_of, const int *offsets,
                                int slots, unsigned int epoch, void *stream);
int b200q_ep_experts_dev(void *ep, int ggml_type, const void *gate_up, long long gate_up_row_bytes,
                         const void *down, long long down_row_bytes, int d_ff, void *act, unsigned int epoch,
                         int max_ctas, void *stream);
/* The exchange fused into the gate/up GEMM (replaces b200q_ep_send_rows_bf16_dev
 * + b200q_ep_experts_dev after b200q_ep_exchange_counts_dev): one warp of every
 * GEMM CTA stores this rank's routed rows h_bf16[token_of[slot]] into their
 * owners' receive buffers with bulk copies, round by round of the receivers'
 * GEMM row tiles, and each GEMM tile waits only until every rank has stored
 * the rows of its own round, so the NVLink transfer overlaps the tensor-core
 * work.  Same arguments and results as the two calls it replaces
 * (bit-identical).  All CTAs of the launch must be resident together (the
 * grid is sized so); a wait that runs out sets the device error word. */
int b200q_ep_dispatch_experts_dev(void *ep, int ggml_type, const void *gate_up, long long gate_up_row_bytes,
                                  const void *down, long long down_row_bytes, int d_ff, void *act,
                                  const void *h_bf16, int T, const int *token_of, const int *offsets, int slots,
                                  unsigned int epoch, int max_ctas, void *stream);
int b200q_ep_combine_dev(void *ep, const int *slot_of, const float *slot_w, int T, int k, float *y,
                         unsigned int epoch, void *stream);

/* ---- Decode step of the reference's Llama decoder (engine/model.py:174-240)
 * around the quantised GEMVs; every call reads the position / token from
 * device memory, so a whole step can be captured in a CUDA graph.  Their
 * kernels are launched programmatic-dependent: each lets the next kernel of
 * the stream launch at once (a following GEMV starts streaming its weights)
 * and reads nothing before the previous kernel has completed.
 *   b200q_dequant_row_dev   out[i][cols] = row row_idx[i] of a quantised (or
 *                           F16 / F32) matrix, i < n (bit-exact; the token
 *                           embedding lookup)
 *   b200q_add_rmsnorm_dev   per row t < T: x += delta (when not NULL);
 *                           rmsnorm(x) * w written to h (f32) and/or h_bf16
 *   b200q_rope_kv_dev       rows t < T of qkv = [q H*hd | k KV*hd | v KV*hd]
 *                           at positions *pos + t: adjacent-pair RoPE of q and
 *                           k over the first ``rotary`` dims, then k, v stored
 *                           at cache[*pos + t] (cache layout [max_seq][KV][hd]);
 *                           pair j turns at pos * base^(-j / (rotary / 2))
 *   b200q_rope_kv_ex_dev    the same with pair j turning at pos * inv_freq[j]
 *                           when inv_freq is given (device f32 [rotary / 2]:
 *                           RoPE scaling -- llama3 frequency interpolation or
 *                           linear, engine/model.py:200-214 -- is a table
 *                           computed once on the host), and with neox != 0
 *                           the pairs (j, j + rotary/2) of Qwen2/Qwen3
 *                           instead of adjacent ones (engine/model.py:212-221)
 *   b200q_qkv_bias_norm_dev before RoPE: qkv rows += bias (optional,
 *                           [(H + 2 KV) * hd], Qwen2's biased projections),
 *                           then every q / k head RMS-normalised with the
 *                           per-head weights q_norm / k_norm (optional, [hd],
 *                           Qwen3); hd a multiple of 32 up to 256
 *   b200q_attn_prefill_dev  causal attention of T query rows (positions
 *                           *pos + t, q from the rotated qkv rows) over cache
 *                           positions 0 .. *pos + t; out bf16 [T][H*hd]; if
 *                           *pos < 0 or *pos + T > max_seq nothing is written
 *                           and the device error word is set (B200Q_EINDEX)
 *   b200q_attn_decode_dev   out[H*hd] = softmax(q k^T / sqrt(hd)) v over
 *                           positions 0..*pos (GQA: head h uses KV head
 *                           h / (H / KV)); scratch of
 *                           b200q_attn_decode_scratch_floats floats; hd a
 *                           multiple of 4 up to 128, H / KV <= 8, q and the
 *                           caches 16-byte aligned
 *   b200q_attn_decode_ex_dev, b200q_attn_prefill_ex_dev  the same with a
 *                           sliding window (engine/model.py:222): a query at
 *                           position p sees positions max(0, p + 1 - window)
 *                           .. p (window 0: all)
 *   b200q_argmax_dev        *token = argmax(logits) (first index on ties);
 *                           with pos: out_tokens[*pos] = token, ++*pos;
 *                           key: optional zero-initialised 64-bit device word
 *                           for the grid-wide version (cleared again after use) */
int b200q_dequant_row_dev(int ggml_type, const void *raw, long long row_bytes, int cols, const int *row_idx, int rows,
                          int n, float *out, void *stream);
int b200q_add_rmsnorm_dev(float *x, const float *delta, const float *w, int T, int D, float eps, float *h,
                          void *h_bf16, void *stream);
int b200q_rope_kv_dev(float *qkv, int T, int H, int KV, int hd, int rotary, float base, const int *pos,
                      float *k_cache, float *v_cache, int max_seq, void *stream);
int b200q_rope_kv_ex_dev(float *qkv, int T, int H, int KV, int hd, int rotary, float base, const float *inv_freq,
                         int neox, const int *pos, float *k_cache, float *v_cache, int max_seq, void *stream);
int b200q_qkv_bias_norm_dev(float *qkv, int T, int H, int KV, int hd, const float *bias, const float *q_norm,
                            const float *k_norm, float eps, void *stream);
int b200q_attn_prefill_dev(const float *qkv, const float *k_cache, const float *v_cache, const int *pos, int T, int H,
                           int KV, int hd, int max_seq, void *out_bf16, void *stream);
int b200q_attn_prefill_ex_dev(const float *qkv, const float *k_cache, const float *v_cache, const int *pos, int T,
                              int H, int KV, int hd, int max_seq, int window, void *out_bf16, void *stream);
/* b200q_attn_prefill_dev on the tensor cores (tcgen05: bf16 operands, f32
 * accumulation, P in bf16), hd = 128: the rotated queries and the cache rows
 * 0 .. *pos + T - 1 are first copied as bf16 into ``scratch``
 * (b200q_attn_prefill_tc_scratch_bytes bytes, 16-byte aligned), then one CTA
 * per (head, 128 queries) runs the causal softmax attention over 128-key
 * blocks.  Same contract for positions and errors as b200q_attn_prefill_dev;
 * out 16-byte aligned. */
size_t b200q_attn_prefill_tc_scratch_bytes(int T, int H, int KV, int hd, int max_seq);
int b200q_attn_prefill_tc_dev(const float *qkv, const float *k_cache, const float *v_cache, const int *pos, int T,
                              int H, int KV, int hd, int max_seq, void *scratch, size_t scratch_bytes, void *out_bf16,
                              void *stream);
size_t b200q_attn_decode_scratch_floats(int H, int hd, int max_seq);
int b200q_attn_decode_dev(const float *q, const float *k_cache, const float *v_cache, const int *pos, int H, int KV,
                          int hd, int max_seq, float *scratch, float *out, void *stream);
int b200q_attn_decode_ex_dev(const float *q, const float *k_cache, const float *v_cache, const int *pos, int H, int KV,
                             int hd, int max_seq, int window, float *scratch, float *out, void *stream);
int b200q_argmax_dev(const float *logits, int V, int *token, int *pos, int *out_tokens, int max_tokens,
                     unsigned long long *key, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* B200QUANT_H */
