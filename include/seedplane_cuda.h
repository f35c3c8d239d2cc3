/*
 * seedplane_cuda.h -- C ABI of the B200 (sm_100a) Qwen2 decode engine.
 *
 * This is the native boundary that replaces SeedPlane's Vulkan runtime (`qwen_vk`), which the
 * reference drives through a JSON-lines subprocess (seedplane/native.py:25-90 ->
 * native/vulkan_decode/qwen_vk.cpp:810-855). Plain pointers and sizes only; no C++ or torch types.
 *
 * Conventions
 *   - Every entry point returns 0 (SP_OK) or a negative SP_ERR_* code; the message of the last
 *     failure on the calling thread is sp_last_error(). Nothing calls exit() or throws across the
 *     ABI (the reference aborted the process on Vulkan errors, qwen_vk.cpp:52-53).
 *   - "dev" pointers are CUDA device pointers on the engine's device; "host" pointers are host
 *     memory. Token ids and positions are int32, logits fp32.
 *   - Work is queued on the caller's stream (`stream`, a cudaStream_t; NULL = legacy default
 *     stream). No call synchronizes the device except where documented.
 *   - One engine per device. Calls on one engine come from one host thread at a time.
 *     Engines on different devices are independent and may run concurrently.
 */
#ifndef SEEDPLANE_CUDA_H
#define SEEDPLANE_CUDA_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SP_OK               0
#define SP_ERR_INVALID     -1   /* bad argument, shape or layout */
#define SP_ERR_CUDA        -2   /* a CUDA runtime call failed (message names it) */
#define SP_ERR_CAPACITY    -3   /* KV cache / position / node limit exceeded */
#define SP_ERR_UNSUPPORTED -4   /* shape not supported by the kernels */
#define SP_ERR_DEVICE      -5   /* a kernel reported an error status (bounded wait, bad index) */

#define SP_WEIGHTS_F16       0  /* fp16 matrices (seedplane-bundle/2 layout)                    */
#define SP_WEIGHTS_I8_B32    1  /* int8 matrices + one fp16 scale per 32 inputs along K          */

/* Architecture. Mirrors the `arch` block of a seedplane-bundle/2 manifest
 * (seedplane/native_bundle.py:129-131) and Qwen2Engine's config reads (qwen_engine.py:44-53). */
typedef struct sp_config {
    int32_t layers, hidden, heads, kv_heads, head_dim, intermediate, vocab;
    int32_t max_positions;     /* RoPE table length (positions are original position ids)      */
    float   rope_theta, rms_norm_eps;
    int32_t tied_embeddings;   /* 1: LM head = embedding matrix                                 */
    int32_t weight_format;     /* SP_WEIGHTS_*                                                  */
} sp_config;

/* One layer's tensors, device pointers in the bundle-v2 layouts (native_bundle.py:112-120):
 * row-major [out, in]. qkv_w rows are q (heads*head_dim), then k, then v (kv_heads*head_dim each).
 * For SP_WEIGHTS_I8_B32 every matrix is int8 and its `_s` pointer holds fp16 scales
 * [out, in/32]; for SP_WEIGHTS_F16 the `_s` pointers are ignored. */
typedef struct sp_layer_weights {
    const void *qkv_w, *qkv_s;   const float *qkv_b;
    const void *o_w, *o_s;
    const void *gate_w, *gate_s;
    const void *up_w, *up_s;
    const void *down_w, *down_s;
    const float *in_norm, *post_norm;
} sp_layer_weights;

typedef struct sp_weights {
    const void *embed;                 /* [vocab, hidden] fp16, device                          */
    const void *lm_head, *lm_head_s;   /* untied head (fp16, or int8 + scales); NULL when tied  */
    const float *final_norm;           /* [hidden] fp32, device                                 */
    const sp_layer_weights *layers;    /* HOST array of `layers` entries                        */
    const float *rope_host;            /* optional HOST table [max_positions][head_dim/2][2] of
                                          (cos, sin) fp32; NULL = computed in double precision  */
} sp_weights;

typedef struct sp_engine sp_engine;
typedef struct sp_kv sp_kv;

/* Last error message of the calling thread ("" if none). */
const char *sp_last_error(void);
/* Library version string. */
const char *sp_version(void);

/* Create an engine on `device`. The library copies the weights into its own arena in the packed
 * layouts its kernels stream (the caller may free its copies on return) and owns all workspace.
 * Replaces qwen_vk's Engine::init (qwen_vk.cpp:283-342). Synchronizes the device. */
int sp_engine_create(const sp_config *cfg, const sp_weights *w, int device, sp_engine **out);
void sp_engine_destroy(sp_engine *e);
/* Bytes of device memory the engine holds (weights arena + workspace). */
int64_t sp_engine_device_bytes(const sp_engine *e);

/* KV cache of `capacity` slots, fp16 [layers][kv_heads][capacity][head_dim] for K and for V.
 * Replaces KVCache.allocate / Qwen2Engine.new_cache (qwen_engine.py:18-29,82-85). */
int sp_kv_create(sp_engine *e, int32_t capacity, sp_kv **out);
void sp_kv_destroy(sp_kv *kv);
int32_t sp_kv_length(const sp_kv *kv);
int32_t sp_kv_capacity(const sp_kv *kv);
/* Truncate (rollback) the committed length, like `cache.length = n` in the reference's linear
 * verifier (experiments/hive_scaling/benchmark_speculative.py:119,127). */
int sp_kv_set_length(sp_kv *kv, int32_t length);

/* Run `n` tokens through the model at cache slots [len, len+n), exactly Qwen2Engine.forward
 * (qwen_engine.py:105-144): tokens_dev[n] int32, positions_dev[n] int32 RoPE positions (NULL =
 * the slots). Token i attends to slots [0, len+i]. Advances the cache length by n.
 * all_logits = 0: logits_dev NULL or fp32 [vocab] of the last token; argmax_dev NULL or int32 [n],
 *   the greedy token after each input token (lowest index on ties).
 * all_logits = 1: logits_dev fp32 [n][vocab] and argmax_dev [n] for every token.
 * all_logits = 2: the last token only (a prompt whose other tokens only fill the cache): logits_dev
 *   [vocab], argmax_dev[0]; the batched pass runs the LM head for that one token. */
int sp_forward(sp_engine *e, sp_kv *kv, const int32_t *tokens_dev, const int32_t *positions_dev,
               int32_t n, float *logits_dev, int32_t all_logits, int32_t *argmax_dev, void *stream);

/* Greedy decode: feed `token` at position `pos` (slot = current length), then feed back each
 * argmax on the device, for `n_steps` steps without host round trips. out_tokens_dev[n_steps]
 * receives the argmax of every step (out[i] is fed at step i+1). logits_dev: NULL or fp32
 * [vocab] = logits of the last step. Advances the cache length by n_steps. Replaces qwen_vk's
 * per-token Session::step + argmax loop (qwen_vk.cpp:519-565,588-613). */
int sp_decode(sp_engine *e, sp_kv *kv, int32_t token, int32_t pos, int32_t n_steps,
              int32_t *out_tokens_dev, float *logits_dev, void *stream);

/* Greedy decode of B independent requests in one batched pass per step (runtime request batching;
 * the reference has none: README.md:67-68, its HIVE agents report batch_size 1, hive/pool.py:465-466).
 * Request b feeds tokens_host[b] at RoPE position positions_host[b] into its own cache kvs[b] (slot =
 * that cache's length, attention over that cache alone), then each step's argmax is fed back on the
 * device for n_steps steps; the weights are streamed once per step for all B requests.
 * out_tokens_dev[n_steps][B] receives every step's argmaxes (row i = the tokens after step i).
 * 1 <= B <= 64, distinct caches of this engine, each with room for n_steps more slots. Advances every
 * cache's length by n_steps. Replaces, for a batch, B calls of sp_decode (the reference's per-request
 * Session::step loop, qwen_vk.cpp:519-565,588-613). */
int sp_decode_batch(sp_engine *e, sp_kv *const *kvs, int32_t B, const int32_t *tokens_host,
                    const int32_t *positions_host, int32_t n_steps, int32_t *out_tokens_dev, void *stream);

/* The prompts of B independent requests in packed batched passes (runtime request batching; see
 * sp_decode_batch): request b appends lens_host[b] tokens (tokens_dev holds the B prompts one after
 * another) to its own cache kvs[b] at slots len .. len + lens_host[b] - 1, RoPE positions = the slots,
 * every token attending to its own cache up to itself. argmax_dev[B]: the greedy token after each
 * prompt's last token (the LM head runs for those rows only). Whole prompts are packed into passes
 * of at most 512 tokens; a longer prompt runs alone through the chunked pass. 1 <= B <= 256,
 * distinct caches of this engine. Advances every cache's length by its prompt's length. Replaces,
 * for a batch, B prompt calls of sp_forward (Qwen2Engine.forward(prompt), qwen_engine.py:105-144). */
int sp_prefill_batch(sp_engine *e, sp_kv *const *kvs, int32_t B, const int32_t *tokens_dev, const int32_t *lens_host,
                     int32_t *argmax_dev, void *stream);

/* Speculative tree verification (no counterpart kernel in the reference; semantics of
 * seedplane/speculative.py:55-92). n nodes in an ancestor-closed order (parent index < own index;
 * -1 = child of the committed prefix). Node i is written to scratch slot len+i at RoPE position
 * base_pos + depth_i - 1 and attends to the committed slots [0, len) and to its ancestors and
 * itself. The cache length is NOT advanced (see sp_kv_commit).
 * argmax_dev[n]: target argmax after each node. logits_dev: NULL or fp32 [n][vocab]. */
int sp_verify_tree(sp_engine *e, sp_kv *kv, const int32_t *tokens_host, const int32_t *parents_host,
                   int32_t n, int32_t base_pos, float *logits_dev, int32_t *argmax_dev, void *stream);

/* Move the K/V of accepted scratch slots into place: for i < n, slot src_slots_host[i] is copied
 * to slot len+i of every layer, then the length becomes len+n. Replaces the reference's KV
 * rollback by truncation (benchmark_speculative.py:119,127) for tree-shaped drafts. */
int sp_kv_commit(sp_kv *kv, const int32_t *src_slots_host, int32_t n, void *stream);

/* Copy the K/V of n consecutive slots, every layer and kv head, from src slots [src_slot0,
 * src_slot0 + n) to dst slots [dst_slot0, dst_slot0 + n). The caches belong to one engine; they may
 * differ in capacity, or be the same cache with disjoint ranges. Lengths are not changed. Replaces
 * the native session's Engine::copy_slots (native/vulkan_decode/qwen_vk.cpp:440-453): a shard
 * window is seeded with the sink tokens' K/V and, in the approximate reuse mode, the halo's
 * (qwen_vk.cpp:512-542). */
int sp_kv_copy(sp_kv *src, int32_t src_slot0, sp_kv *dst, int32_t dst_slot0, int32_t n, void *stream);

/* Greedy argmax of each row of fp32 logits [rows][ld] (device) over the first `cols` columns:
 * argmax_dev[rows] int32, lowest index on ties (NaN is never selected). For logits produced
 * outside the fused LM head, e.g. all-logits verification. Replaces `Qwen2Engine.sample`
 * (qwen_engine.py:147-148) and argmax.comp:8-22. Uses the engine's scratch: calls on one engine
 * are ordered by their stream (one stream per engine). */
int sp_argmax(sp_engine *e, const float *logits_dev, int32_t rows, int32_t cols, int64_t ld, int32_t *argmax_dev,
              void *stream);

/* Per-row top-k of fp32 logits, k in 1..8: indices and values [rows][k] ordered by larger value,
 * lower index on ties (the greedy argmax's rule), and each row's log-sum-exp, so log-probabilities
 * are val - lse. Replaces the drafter-side `torch.topk` + `log_softmax` a tree drafter needs; the
 * reference has no drafter tree (seedplane/speculative.py:18-43 takes given branches). */
int sp_topk(sp_engine *e, const float *logits_dev, int32_t rows, int32_t cols, int64_t ld, int32_t k,
            int32_t *idx_dev, float *val_dev, float *lse_dev, void *stream);

/* Greedy acceptance of a verified draft tree on the device (replaces the selection loop of
 * seedplane/speculative.py:55-92, verify_greedy, fed by one batched pass instead of per-prefix target
 * calls). node_pred_dev: int32 [n] on the engine's device, the target's argmax after each node (the
 * argmax output of sp_verify_tree); root_pred: its argmax after the committed prefix. tokens /
 * parents (host, parents[i] < i, -1 = child of the prefix); path_ends (host, [n_paths]): the last
 * node of each draft branch in input order. Each branch is walked from its root while the target
 * agrees; the first disagreement emits the target's token and rejects the branch; the chosen
 * branch has the most accepted draft tokens, then the most emitted tokens, then the earliest input
 * position; no paths: the one token root_pred. out_host [2n + 5]: emitted count, accepted count,
 * chosen branch (-1: none), the target's token after a fully accepted branch (else -1), emitted
 * tokens [n + 1], accepted node indices [n]. n <= 64, n_paths <= 1024. Synchronises `stream`. */
int sp_accept_greedy(sp_engine *e, const int32_t *node_pred_dev, int32_t root_pred, const int32_t *tokens_host,
                     const int32_t *parents_host, int32_t n, const int32_t *path_ends_host, int32_t n_paths,
                     int32_t *out_host, void *stream);

/* Stochastic acceptance of a draft tree at `temperature` with a counter-based RNG (seed, counter):
 * recursive rejection sampling (children tried in node order, accept with min(1, p/q), residual
 * max(p - q, 0) after a rejection, a draw from the residual when every child is rejected). The
 * reference has no stochastic verifier (seedplane/speculative.py:46-92 is greedy only); the rule
 * and its fp64 arithmetic are restated bit for bit in the repository's CPU oracle.
 * target_logits / draft_logits: device fp32 [n + 1][ld], row 0 = after the committed prefix,
 * row i + 1 = after node i. tokens / parents (host, parents[i] < i, -1 = root child). out_host
 * [2n + 3]: emitted count, accepted count, emitted tokens [n + 1], accepted node indices [n].
 * Synchronises `stream`. */
int sp_accept_stochastic(sp_engine *e, const float *target_logits_dev, const float *draft_logits_dev, int64_t ld,
                         int32_t vocab, const int32_t *tokens_host, const int32_t *parents_host, int32_t n,
                         double temperature, uint64_t seed, uint64_t counter, int32_t *out_host, void *stream);

/* The batched pass's projection on its own: y[t][n] = alpha * W[n, :] . (x[t] + x[lo_row0 + t]),
 * t < t, n < n, over k inputs, on the tcgen05 multi-column GEMM of the engine's device (no reference
 * counterpart: it is the contraction under sp_forward's prompt chunks and sp_verify_tree, which
 * replace qwen_vk.cpp:417-436's gemm_b.comp batch and speculative.py:55-92's per-prefix target calls;
 * exposed for callers and tests of that contraction). W: row-major fp16 [n, k] (w_lo_dev: optional
 * second fp16 half, W = w + w_lo); x: fp16 rows [x_rows, k], token t's hi half at row t, its lo
 * half at row lo_row0 + t. mode 0: y[t * ldy + n] = ...; 1: y[t * ldy + n] += ...; 2 (SwiGLU): rows
 * 2i, 2i + 1 are gate i, up i, and a = SiLU(gate) * up goes to act_hi[t * ld_act + i] = fp16(a),
 * act_lo[...] = fp16(a - hi). t <= 512; k a multiple of 8; the engine's GEMM workspace is used,
 * so calls on one engine are ordered on one stream. */
int sp_mcol_gemm(sp_engine *e, int32_t mode, const void *w_dev, const void *w_lo_dev, float alpha, int32_t n, int32_t k,
                 const void *x_dev, int32_t x_rows, int32_t lo_row0, int32_t t, float *y_dev, int32_t ldy,
                 void *act_hi_dev, void *act_lo_dev, int32_t ld_act, void *stream);

/* Top-k / top-p filter of one logits row before a draw (replaces the masking steps of
 * seedplane/qwen_engine.py:147-156, Qwen2Engine.sample): z_dev[j] = logits_dev[j] / temperature
 * (fp32); then, if top_k > 0, -inf below the top_k-th largest z (ties at the cut kept); then, if
 * top_p < 1, -inf for every entry whose preceding probability mass in descending order (softmax
 * over the entries still kept) exceeds top_p (a group of equal values at the cut is kept whole).
 * Draw from z_dev with sp_accept_stochastic (n = 0, temperature 1). One launch of one CTA on
 * `stream`, no engine, no allocation. vocab in [1, 524288], temperature > 0, top_k >= 0,
 * top_p in [0, 1], else SP_ERR_INVALID. */
int sp_sample_filter(const float *logits_dev, int32_t vocab, double temperature, int32_t top_k, double top_p,
                     float *z_dev, void *stream);

/* sp_argmax without an engine and without any allocation (no reference counterpart: the
 * reference allocates nothing on this path; this entry point exists for callers that must not
 * allocate device memory, e.g. inside a memory-capped serving process or before an engine
 * exists). Same result as sp_argmax. Runs on `device` and sets the calling thread's current
 * device back to what it was before returning; logits_dev and argmax_dev must be device memory
 * of `device` (else SP_ERR_INVALID). Its scratch is a fixed 33,280-byte __device__ array of the
 * library (one per device), so:
 *   - rows <= 128, else SP_ERR_CAPACITY (nothing is launched);
 *   - it clears the row counters it uses (a memset on `stream`) before each launch;
 *   - calls that overlap in time on one device (different streams or threads) race on the same
 *     scratch: order them on one stream;
 *   - the first call on a device looks the scratch up (cudaGetSymbolAddress): make it before any
 *     stream capture. The address is kept for the life of the device's primary context; a
 *     process that resets the device (cudaDeviceReset) must not call this entry point again. */
int sp_argmax_noalloc(int device, const float *logits_dev, int32_t rows, int32_t cols, int64_t ld,
                      int32_t *argmax_dev, void *stream);

/* Kernel timeline of the last step, when the engine was created with SEEDPLANE_TRACE=1: for each
 * GEMV of the step (4 per layer, then the LM head) and each CTA, kernel-start / dependency-wait /
 * prologue / stream / epilogue stamps and per-unit issue and ready stamps of %globaltimer (ns).
 * host_out NULL: returns the number of 64-bit words; else copies them (synchronizes the device)
 * and returns the count. Returns 0 when tracing is off. With SEEDPLANE_MCOL_TRACE=1 (and no step
 * trace) it returns the last sp_mcol_gemm launch's per-CTA phase stamps instead (16 words per CTA,
 * 148 CTAs). The reference had no GPU timestamps
 * (experiments/v18/RESULTS.md:29-30). */
int64_t sp_trace_read(sp_engine *e, uint64_t *host_out, int64_t capacity);

/* Wait for `stream`, then report (and clear) a device-side error status recorded by a kernel since
 * the last call: SP_ERR_DEVICE with a message, or SP_OK. Kernels never trap; a bad token id, an
 * out-of-table position or an expired bounded wait is recorded here instead. */
int sp_device_status(sp_engine *e, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SEEDPLANE_CUDA_H */
