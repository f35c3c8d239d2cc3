// Kernel parameter blocks and host-side launchers of the decode kernels (kernels.cu).
#pragma once

#include "common.cuh"

namespace sp {

enum Prologue : int { PRO_PLAIN = 0, PRO_NORM = 1, PRO_EMBED_NORM = 2 };
enum Epilogue : int { EPI_QKV = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_LMHEAD = 3 };
enum WeightFmt : int { WF_F16 = 0, WF_I8 = 1 };

// Bytes of one fragment tile: 16 rows x 16 inputs of fp16, stored in mma.m16n8k16 A-fragment
// order (lane l's 16 bytes are its registers a0..a3), so one 16-byte shared load per lane feeds
// one tensor-core MMA.
constexpr int kTileBytes = 512;
constexpr int kMaxPrefetch = 4;

// One weight-streaming GEMV y = W . in(x) with a fused prologue and epilogue.
//   W is fragment-packed: strip s (rows 16s..16s+15) and k-tile t (inputs 16t..16t+15) is the
//   512-byte tile at (s * K/16 + t) * 512. Work is split into units = (strip, k segment of nt
//   tiles); each CTA streams a contiguous range of units through a ring of shared-memory stages
//   with 1-D bulk copies, the 8 warps share a unit's tiles, and units of one strip that end in
//   different CTAs are summed by the last CTA to finish the strip (fixed order, deterministic).
struct GemvParams {
    const uint8_t *w;
    int N, K;
    int fmt;                 // WeightFmt (fp16 only in the fragment kernels)
    int nt;                  // k-tiles per unit
    int ks;                  // units per strip = (K/16) / nt
    int stages;              // ring depth
    int grid;                // CTAs
    // prologue
    const float *xin;
    const float *gain;
    const __half *embed;
    float *x_init;
    float eps;
    int vocab;
    // epilogue
    const float *bias;
    float *out;
    __half *kc, *vc;
    int cap;
    const float *rope;
    int max_pos;
    int nh, nkv, hd;
    // split-K partials (strips x ks x 16) and per-strip arrival counters
    float *partial;
    unsigned *strip_cnt;
    // LM head
    int n_valid;             // rows >= n_valid are zero padding (vocab rounded up to 16)
    float *part_val;
    int *part_idx;
    unsigned *counter;
    DevState *st;
    // L2 prefetch of the weight stream ahead of this kernel (issued before the dependency wait)
    const uint8_t *pf_ptr[kMaxPrefetch];
    unsigned long long pf_bytes[kMaxPrefetch];
    int pf_n;
    int evict_first;         // stream weights with an L2 evict-first hint
    // Optional trace (null = off): per CTA kTraceWords %globaltimer stamps, see kTrace* below.
    unsigned long long *trace;
};

// Trace layout per CTA: [0] kernel start, [1] dependency wait returned, [2] prologue done,
// [3] stream loop done, [4] epilogues done, [8 + i] unit i issued, [8 + kTraceUnits + i] unit i
// ready (i < kTraceUnits).
constexpr int kTraceUnits = 24;
constexpr int kTraceWords = 8 + 2 * kTraceUnits;

constexpr int kAttnCluster = 8;      // CTAs per kv head (one thread-block cluster)

struct AttnParams {
    const float *q;          // [NH*HD] fp32 (RoPE applied)
    const __half *kc, *vc;   // this layer's caches [NKV][cap][HD]
    float *out;              // [NH*HD] fp32
    int nh, nkv, hd, cap;
    float scale;
    DevState *st;
    // Optional trace (null = off): per CTA [0] start, [1] wait returned, [2] positions done,
    // [3] CTA partial written, [4] first cluster barrier passed, [5] merged.
    unsigned long long *trace;
};

struct LaunchCfg {
    cudaStream_t stream;
    bool pdl;                // launch with programmatic stream serialization
};

// ---- tensor-core (tcgen05 + TMEM) weight-streaming GEMV: gemv_tc.cu ------------------------
constexpr int kTcTileBytes = 4096;       // 128 rows x 16 inputs of fp16, canonical K-major layout

struct TcGemvParams {
    const uint8_t *w;        // tiles (strip s, k-tile t) at (s * K/16 + t) * 4096
    int N, K;                // N multiple of 128 (zero padded), K multiple of 16
    int n_valid;             // rows >= n_valid are padding
    int grid, stages;
    int b_full;              // B operand holds all K/16 k-tiles (else the CTA's tiles)
    int b_tiles;             // B operand tiles in shared memory
    int max_contrib;         // CTAs that may share one strip
    int max_items;           // strips a CTA may touch
    // prologue
    const float *xin;
    const float *gain;
    const __half *embed;
    float *x_init;
    float eps;
    int vocab;
    // epilogue
    const float *bias;
    float *out;
    __half *kc, *vc;
    int cap;
    const float *rope;
    int max_pos;
    int nh, nkv, hd;
    float *partial;          // [strips][max_contrib][128]
    unsigned *strip_cnt;     // [strips]
    float *part_val;
    int *part_idx;
    unsigned *counter;
    DevState *st;
    const uint8_t *pf_ptr[kMaxPrefetch];
    unsigned long long pf_bytes[kMaxPrefetch];
    int pf_n;
    unsigned long long *trace;
};

void plan_gemv_tc(TcGemvParams &p, int num_sms, int ring_bytes, int b_budget_bytes);
size_t gemv_tc_smem_bytes(const TcGemvParams &p);
int gemv_tc_max_items();
cudaError_t prepare_gemv_tc(int pro, int epi, const TcGemvParams &p);
cudaError_t launch_gemv_tc(int pro, int epi, const TcGemvParams &p, const LaunchCfg &lc);
// Pack an fp16 N x K matrix (packed row r = source row row_of[r] of a / b as in
// launch_pack_fragments, < 0 = zero) into 128 x 16 canonical K-major tiles.
cudaError_t launch_pack_tc(uint8_t *dst, const __half *a, int rows_a, const __half *b, const int *row_of, int N, int K,
                           cudaStream_t s);

// Plan units / stages / grid for a GEMV of N x K; fills the geometry fields.
void plan_gemv(GemvParams &p, int num_sms, int ring_bytes, int max_unit_bytes);
size_t gemv_smem_bytes(const GemvParams &p);
// Set the dynamic shared-memory limit of the kernel instance (call before any stream capture).
cudaError_t prepare_gemv(int pro, int epi, const GemvParams &p);
cudaError_t launch_gemv(int pro, int epi, const GemvParams &p, const LaunchCfg &lc);
cudaError_t prepare_attention();
cudaError_t launch_attention(const AttnParams &p, const LaunchCfg &lc);

// Host-side launches of small utility kernels.
cudaError_t launch_set_state(DevState *st, const DevState &init, cudaStream_t s);
// dst row (r * dst_mul + dst_add) = src row src_row[r], for r < rows.
cudaError_t launch_gather_rows(uint8_t *dst, const uint8_t *src, const int *src_row, int rows, int row_bytes,
                               int dst_mul, int dst_add, cudaStream_t s);
// Fragment-pack an fp16 matrix of N x K: packed row r is source row row_of[r] of `a` when
// row_of[r] < rows_a, else row row_of[r] - rows_a of `b` (gate/up interleave, RoPE pairing);
// row_of[r] < 0 is a zero row (padding).
cudaError_t launch_pack_fragments(uint8_t *dst, const __half *a, int rows_a, const __half *b, const int *row_of,
                                  int N, int K, cudaStream_t s);
cudaError_t launch_kv_commit(__half *k, __half *v, int layers, int nkv, int cap, int hd, const int *src_slots,
                             int n, int dst0, cudaStream_t s);

// ---- persistent decode step: step.cu -----------------------------------------------------------
// One launch per token runs the whole step on one CTA per SM. The ops of the step (GEMVs with
// fused prologues/epilogues, and attention) are a table in device memory. Every CTA owns whole
// output rows of every GEMV (no split-K) and streams all of its weight units through one ring
// without waiting for data. Vectors pass between ops as LL words (a 64-bit store of a 32-bit
// payload and the 32-bit tag of the writing op and step, polled by the readers); the SwiGLU
// activation passes through a 64-bit counter whose readers wait until it reaches CTAs x
// (epoch + 1), where `epoch` counts finished steps (advanced by the LM head's last CTA).
enum StepOpKind : int { OP_GEMV = 0, OP_ATTN = 1 };
constexpr int PRO_ATTN = 3;              // O-projection prologue: the merged attention output
constexpr int kStepAttnRows = 48;        // attention positions staged per sub-chunk
constexpr int kStepMaxChunks = 64;       // attention chunks per q head
constexpr int kStepPassRows = 64;        // GEMV rows per pass (16 per compute warp)
constexpr int kStepTraceWords = 16;      // per op and CTA: [0..7] %globaltimer: reached, dep met, input
                                         // ready, done, first unit available, rows finished, merge
                                         // start / end; [8..15] clock64 at the op's phase boundaries

struct StepOp {
    const uint8_t *w;        // row-block packed weights (GEMV), see k_pack_rows
    const uint64_t *lin;     // LL input: the residual stream (norm prologues), the merged attention
                             // output (PRO_ATTN), q (attention)
    const uint64_t *lres;    // EPI_RESID: LL residual base; null: the token's embedding row
    uint64_t *lout;          // LL output: q (QKV), the residual stream (EPI_RESID), the merged
                             // attention output (attention)
    uint64_t *lkv;           // QKV / attention: the step's new K/V rows, [nkv][k | v][hd / 2] fp16 pairs
    uint64_t *lpart;         // attention: per (q head, chunk) partials [nh][max_chunks][hd + 2]
    const __half *xin_h, *xin_l;   // PRO_PLAIN input: fp16 hi / lo vectors behind counter `dep`
    __half *out_h, *out_l;   // EPI_SWIGLU output: fp16 hi / lo vectors
    const float *gain;       // RMSNorm gains
    const float *bias;       // QKV bias
    __half *kc, *vc;         // this layer's K/V cache (QKV epilogue, attention)
    int kind;                // StepOpKind
    int pro, epi;
    int N, K, n_valid;       // N even: rows come in pairs
    int grid;                // CTAs owning rows (see gemv_share)
    int pass_rows;           // rows per pass (even, <= kStepPassRows)
    int chunk_w;             // inputs per unit (f16: multiple of 256, i8: of 128; or all of K)
    int lin_k, lres_k;       // ops whose tags lin / lres carry
    int dep, dep_n;          // wait until cnt[dep] >= dep_n * (epoch + 1); dep < 0: none
    int sig;                 // cnt[sig] += 1 per CTA; < 0: none
    int fmt;                 // WeightFmt of w
    int cta_bytes;           // WF_I8: bytes of one CTA's rows (CTA c's units start at c * cta_bytes)
    int ksplit;              // CTAs sharing a row group, each over K / ksplit inputs (WF_I8; 1, 2 or 4)
    int pad_;
    uint64_t *lksp;          // split: CTA h > 0's row partials for CTA 0, LL words [ksplit - 1][N]
};
static_assert(sizeof(StepOp) % 16 == 0, "ops are copied to shared memory in 16-byte words");

// The share of CTA c in a step GEMV of N rows (P = N / 2 row pairs) and K inputs: the grid /
// ksplit row groups own pairs [P g / G, P (g + 1) / G); CTA c works on group g = c / ksplit over
// inputs [K0, K0 + Kc), Kc = K / ksplit, K0 = (c % ksplit) Kc.
struct GemvShare {
    int R0, R, K0, Kc;
};
__host__ __device__ inline GemvShare gemv_share(int N, int K, int grid, int ksplit, int c) {
    const int ks = ksplit > 1 ? ksplit : 1, G = grid / ks, g = c / ks, P = N / 2;
    GemvShare s;
    s.R0 = 2 * (int)((long long)P * g / G);
    s.R = 2 * (int)((long long)P * (g + 1) / G) - s.R0;
    s.Kc = K / ks;
    s.K0 = (c - g * ks) * s.Kc;
    return s;
}

struct StepParams {
    const StepOp *ops;
    int n_ops;
    int stages;              // ring stages
    int stage_bytes;         // bytes per stage (multiple of 1024, <= 64 KB)
    int vec_bytes;           // shared input-vector region (GEMV input halves, attention staging)
    int attn_off;            // attention staging offset in it (after the QKV projection's input)
    int nh, nkv, hd, cap, max_pos, vocab, hidden;
    int max_chunks;          // attention chunks per q head at most (nh * max_chunks <= grid)
    int group_chunks;        // grouped items: chunks per kv head at most (nkv * group_chunks <= grid)
    int part_stride;         // attention partial slots per q head (>= both chunk counts)
    int evict_first;         // ring copies carry an L2 evict-first hint
    int max_inflight;        // ring copies in flight at most (0: stages)
    int l2_ahead;            // bytes of its next units a CTA prefetches into L2 while its ring is full
    float eps, scale;
    const float *rope;
    const __half *embed;
    float *part_val;         // LM head: per-CTA argmax
    int *part_idx;
    unsigned *lm_cnt;
    unsigned long long *cnt; // dependency counters
    unsigned long long *epoch;
    DevState *st;
    unsigned long long *trace;   // [n_ops][grid][kStepTraceWords] or null
};

struct StepLayout {
    int stages = 0, stage_bytes = 0, vec_bytes = 0, attn_off = 0;
    size_t smem = 0;         // dynamic shared memory; stage_bytes == 0: does not fit
};

constexpr int kMaxKsplit = 4;            // CTAs a row group of a split int8 GEMV at most
// fills grid, ksplit, pass_rows, chunk_w from N, K (ksplit > 1 only for int8 ops other than the LM
// head, at most max_ksplit)
void plan_step_gemv(StepOp &o, int num_sms, int stage_bytes, int max_ksplit = 1);
bool step_gemv_supported(const StepOp &o, int stage_bytes);
size_t step_gemv_bytes(const StepOp &o);                           // packed bytes of a planned GEMV
// Pack an fp16 N x K matrix (packed row r = source row row_of[r] of a / b as in
// launch_pack_fragments, < 0 = zero) into the plan's row-block layout.
cudaError_t launch_pack_rows(uint8_t *dst, const __half *a, int rows_a, const __half *b, const int *row_of,
                             const StepOp &plan, cudaStream_t s);
// Blockwise int8 (`a`, `b` int8 [rows][K] with fp16 scales `as`, `bs` [rows][K / 32]); `dst` must
// be zeroed first (padding scales of partial row tiles are not written).
cudaError_t launch_pack_rows_i8(uint8_t *dst, const int8_t *a, const __half *as, int rows_a, const int8_t *b,
                                const __half *bs, const int *row_of, const StepOp &plan, cudaStream_t s);
size_t step_attn_smem_bytes(int hd);
// xmax: the largest GEMV input (multiple of 8); hidden: the QKV projection's input; i8: inputs
// of int8 matrices are digit rows (see digitize4_n in step.cu).
StepLayout step_layout(int hidden, int xmax, int hd, int stages, bool i8);
cudaError_t prepare_step(int hd, size_t smem, bool q8);   // q8: the builds with the int8 unit path
// pdl: programmatic dependent launch after the previous kernel in the stream; the grid must be
// resident at once (one CTA per SM), so the launch is cooperative.
// grouped: the build with grouped attention items (one per kv head and chunk) instead of per-head ones
cudaError_t launch_step(int hd, const StepParams &p, int grid, size_t smem, cudaStream_t s, bool pdl, bool q8,
                        bool grouped);

// ---- batched prompt pass: prefill.cu ------------------------------------------------------------
// T prompt tokens per chunk through all layers at once: the multi-column tcgen05 GEMM (mcol.cu)
// on row-major weight copies with the activation split into fp16 hi / lo halves, and this engine's
// kernels for the norms, RoPE + K/V write and causal attention.
constexpr int kPrefillMin = 8;           // shorter inputs run as step launches
constexpr int kPrefillMaxTokens = 512;   // tokens per chunk (scratch size; a multiple of 128)
constexpr int kPrefillLogitRows = 64;    // logits rows per head GEMM (argmax scratch rows)
constexpr int kPrefillMaxCtas = 148;     // GEMM CTAs at most (one per SM; workspace slots)

// One request of a batched decode step (sp_decode_batch): its own cache (layer-0 K / V bases and
// capacity, layout [layer][kv head][cap][head_dim]) and the slot its token's K / V go to (= the
// cache length before the step). The token attends to slots [0, slot] of that cache.
struct BatchLane {
    __half *k, *v;
    int cap;
    int slot;
};
struct PrefillDims {
    int hidden, inter, heads, kv_heads, head_dim, vocab, max_pos, max_tokens;
    float eps;
};
struct PrefillMat {                      // row-major weights W = alpha * (hi + lo), or alpha * q * sc
    const __half *hi;                    // fp16 checkpoints: the weights (alpha 1, no lo)
    const __half *lo;
    float alpha;
    const int8_t *q;                     // int8 checkpoints: the int8 rows [N][K] (hi, lo null) and their
    const __half *sc;                    // 32-input block scales times 2^k, [ceil(K / 64)][N][2] fp16
                                         // (exact); the GEMM splits q * sc into exact fp16 halves on the chip
};
struct PrefillLayer {
    PrefillMat qkv;                      // [(heads + 2 kv_heads) * head_dim, hidden], RoPE partners adjacent
    PrefillMat o;                        // [hidden, heads * head_dim]
    PrefillMat gate_up;                  // [2 inter, hidden]: rows interleaved, 2i = gate i, 2i + 1 = up i
    PrefillMat down;                     // [hidden, inter]
    const float *qkv_b, *in_norm, *post_norm;
};
// Blockwise int8 rows (q [rows][K], fp16 scales [rows][K / 32]) into the batched pass's int8 form:
// source row r to row r * dst_mul + dst_add (or its RoPE-pair position, pair_hd > 0) of dq [N][K],
// and the scales times 2^k (fp16; exact for k >= 0 below overflow) to dsc [ceil(K / 64)][N][2]
// (zeroed first by the caller).
cudaError_t launch_repack_i8(int8_t *dq, __half *dsc, const int8_t *q, const __half *scales, int rows, int N, int K,
                             int k, int dst_mul, int dst_add, int pair_hd, cudaStream_t s);
// Largest |scale| * 127 of a blockwise-int8 matrix (n fp16 scales), into *out (device float).
cudaError_t launch_int8_absmax(float *out, const __half *scales, long long n, cudaStream_t s);
struct PrefillScratch {
    float *x;                            // [T, hidden] residual stream
    __half *xa;                          // GEMM inputs of norms and attention: hi rows [0, max_tokens), lo
                                         // rows [max_tokens, 2 max_tokens), row stride = the GEMM's K
    __half *xb;                          // the down projection's input (SwiGLU), same layout
    float *y;                            // [T, qkv rows] QKV projection
    float *q;                            // [T, heads * head_dim]
    float *logits;                       // [kPrefillLogitRows, vocab]
    float *part;                         // attention partials per (query, head, key chunk): kAttnPartBytes
};
constexpr size_t kAttnPartBytes = (size_t)64 << 20;
size_t prefill_scratch_bytes(const PrefillDims &d);
PrefillScratch prefill_scratch_at(void *base, const PrefillDims &d);
cudaError_t launch_prefill_embed(const PrefillDims &d, const PrefillScratch &s, const __half *embed,
                                 const int32_t *tok, int T, DevState *st, cudaStream_t stream);
// RMSNorm, QKV GEMM, bias + RoPE + K/V write at slots *slot_base + slot_off .., attention
// (causal, or the tree of ancestor masks `mask` [T], T <= 64), O GEMM (+= x)
cudaError_t launch_prefill_layer_front(const PrefillDims &d, const PrefillLayer &L, const PrefillScratch &s, int T,
                                       const int32_t *pos, const uint64_t *mask, __half *kc, __half *vc, int cap,
                                       const int *slot_base, int slot_off, float scale, const float *rope,
                                       DevState *st, cudaStream_t stream);
// The same front for a batched decode step: token t belongs to request lanes[t] (its cache, slot;
// positions pos[t]) and attends to that cache alone (k_attn_batch)
cudaError_t launch_batch_layer_front(const PrefillDims &d, const PrefillLayer &L, const PrefillScratch &s, int B,
                                     const int32_t *pos, const BatchLane *lanes, int layer, float scale,
                                     const float *rope, DevState *st, cudaStream_t stream);
// after a batched decode step: each request's argmax becomes its next token (pos + 1, slot + 1) and
// is stored at out[b]
cudaError_t launch_batch_advance(BatchLane *lanes, int32_t *tok, int32_t *pos, const int32_t *argmax, int32_t *out,
                                 int B, int max_pos, DevState *st, cudaStream_t stream);
// RMSNorm, gate_up GEMM with SwiGLU, down GEMM (+= x)
cudaError_t launch_prefill_layer_ffn(const PrefillDims &d, const PrefillLayer &L, const PrefillScratch &s, int T,
                                     DevState *st, cudaStream_t stream);
// final RMSNorm of rows [r0, r0 + n) and the head GEMM into out [n, vocab]
cudaError_t launch_prefill_logits(const PrefillDims &d, const PrefillScratch &s, const float *final_norm,
                                  const PrefillMat &head, int r0, int n, float *out, DevState *st, cudaStream_t stream);

// ---- multi-column GEMM of the batched pass: mcol.cu ----------------------------------------------
// Y[t][n] = alpha * W[n, :] . (x_hi[t] + x_lo[t]) on tcgen05 (weights = the M 128 operand, tokens'
// hi / lo rows = the N operand), fused epilogue by mode. x: fp16 rows [x_rows, K], token t's hi row
// at t, its lo row at lo_row0 + t. W: row-major fp16 [N, K], or two halves (w + w_lo).
enum { MC_STORE = 0, MC_RESID = 1, MC_SWIGLU = 2, MC_QKV = 3 };
// MC_QKV epilogue: the rows are the QKV projection's with RoPE partners adjacent (row 2p, 2p + 1 =
// dims d, d + head_dim / 2 of one head, p = head * head_dim / 2 + d); adds the bias (natural order),
// rotates q and k by the token's position (rope table [pos][head_dim / 2][cos, sin]), writes q fp32
// [t][heads * head_dim] and k, v fp16 into the cache at slot *slot_base + slot_off + t.
struct McolQkv {
    const float *bias, *rope;
    const int32_t *pos;          // per-token positions or null (= slot)
    const int *slot_base;
    int slot_off, cap, nh, nkv, hd, max_pos;
    float *q;
    __half *kc, *vc;
    const BatchLane *lanes;      // batched decode: token t writes its K / V into lanes[t]'s cache (layer
    int layer;                   // `layer`), kc / vc / cap / slot_base unused
};
struct McolOp {
    int mode;                    // MC_STORE: y[t ldy + n] = ..; MC_RESID: += ..; MC_SWIGLU: see act_*
    const __half *w, *w_lo;      // w_lo: second weight half or null
    const int8_t *wq;            // or int8 weights [N][K] with block scales wsc (PrefillMat::q, sc)
    const __half *wsc;
    float alpha;
    int N, K;
    const __half *x;
    int x_rows, lo_row0, T;
    float *y;
    int ldy;
    __half *act_h, *act_l;       // MC_SWIGLU: rows 2i = gate i, 2i + 1 = up i; act[t ld_act + i] = hi / lo
    int ld_act;
    int max_ctas;
    DevState *st;
    McolQkv qkv;                 // MC_QKV only
    unsigned long long *trace;   // optional: %globaltimer stamps of the launch's phases per CTA
};
struct McolParams {
    int N, K, T, tn, lo_row0, two_w, cs, stages, tmem_cols;   // cs: CTAs of a cluster splitting a tile
    int i8w;                     // int8 weights: tiles dequantized into fp16 hi / lo on the chip
    const __half *wsc;
    float alpha;
    float *y;
    int ldy;
    __half *act_h, *act_l;
    int ld_act;
    DevState *st;
    McolQkv qkv;
    unsigned long long *trace;   // per-CTA phase stamps (kMcolTraceWords each) or null
};
constexpr int kMcolTraceWords = 16;
size_t mcol_max_smem();
int mcol_tile_tokens(int T);
// pdl: programmatic dependent launch after the previous kernel in the stream
cudaError_t launch_mcol(const McolOp &op, cudaStream_t s, bool pdl);

// Per-row top-k (k <= kTopkMax; larger value first, lower index on ties) and log-sum-exp of fp32
// logits (sample.cu): idx / val [rows][k], lse [rows].
constexpr int kTopkMax = 8;
cudaError_t launch_topk_rows(const float *logits, int rows, int cols, long long ld, int k, int *idx, float *val,
                             float *lse, cudaStream_t s);

// top-k / top-p filter of one logits row (z = logits / T, dropped entries -inf); one CTA
constexpr int kSampleFilterMaxVocab = 1 << 19;      // fixed-point mass sums stay below 2^63
cudaError_t launch_sample_filter(const float *logits, int V, double temperature, int top_k, double top_p, float *z,
                                 cudaStream_t s);
// Stochastic acceptance of a draft tree (sample.cu): target / drafter logits [n + 1][ld] (row 0:
// after the committed prefix, row i + 1: after node i), nodes (token, parent); out [2n + 3]:
// emitted count, accepted count, emitted tokens [n + 1], accepted nodes [n]. rows [nr]: the logits
// rows the walk can visit (row 0 and the rows i + 1 of nodes i with children); slot [n + 1]: a
// row's index in rows (-1 if not listed); fp64 scratch MS [2][nr][2], E [2][nr][V] (the rows' p,
// then q).
cudaError_t launch_accept_stochastic(const float *tlog, const float *dlog, long long ld, int V, const int *tok,
                                     const int *parent, int n, const int *rows, const int *slot, int nr,
                                     double temperature, unsigned long long seed, unsigned long long counter,
                                     double *MS, double *E, int *out, cudaStream_t s);
// Greedy acceptance of a verified tree (one warp): pred [n] = target argmax after each node, ends
// [n_paths] = last node of each draft path in input order; out [2 n + 5]: emitted count, accepted
// count, chosen path, target token after a fully accepted path (else -1), emitted tokens (n + 1
// slots), accepted node indices (n slots).
constexpr int kGreedyMaxPaths = 1024;
cudaError_t launch_accept_greedy(const int *pred, int root_pred, const int *tok, const int *parent, int n,
                                 const int *ends, int n_paths, int *out, cudaStream_t s);

// Row-wise greedy argmax (argmax.cu). A row is split over argmax_ctas(cols) CTAs whose partial
// (max, index) pairs meet in the scratch: val / idx [rows][kArgmaxMaxCtas] and one counter per
// row, which must be zero when the kernel starts and is zero again when it ends.
constexpr int kArgmaxMaxCtas = 32;
struct ArgmaxScratch {
    float *val;
    int *idx;
    unsigned *cnt;
};
int argmax_ctas(int cols);
size_t argmax_scratch_bytes(int rows);
ArgmaxScratch argmax_scratch_at(void *base, int rows);
cudaError_t launch_argmax_rows(const float *logits, int rows, int cols, long long ld, int *out, const ArgmaxScratch &sc,
                               cudaStream_t s);
// The fixed scratch of sp_argmax_noalloc on the current device (a __device__ array, no allocation).
int argmax_noalloc_max_rows();
size_t argmax_noalloc_scratch_bytes();
cudaError_t argmax_noalloc_scratch(void **base);

}  // namespace sp
