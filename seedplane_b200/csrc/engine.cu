// Host side of the C ABI (include/seedplane_cuda.h): weight arena and packing, workspace, the
// per-step kernel chain, CUDA-graph replay of that chain, and the forward / decode / verify /
// commit entry points.
//
// A step is the fixed chain  QKV(l) -> attention(l) -> O(l) -> gate_up(l) -> down(l)  for every
// layer, then the LM head. All per-step values (token, position, slot, tree mask, output
// pointers) live in a device-side DevState that the LM head advances, so one captured graph per
// KV cache serves decode, teacher-forced prefill and tree verification. This replaces qwen_vk's
// pre-recorded one-token command buffer (native/vulkan_decode/qwen_vk.cpp:349-412) and its
// per-token submit + fence wait (qwen_vk.cpp:141-147, 519-565).
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/seedplane_cuda.h"
#include "kernels.cuh"

using namespace sp;

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define SP_CUDA(call)                                                                            \
    do {                                                                                         \
        cudaError_t e_ = (call);                                                                 \
        if (e_ != cudaSuccess) return fail(SP_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Inputs of one batched block that a captured verify graph reads from fixed device memory.
struct VerifyIn {
    int32_t slot0;                          // first cache slot of the block
    int32_t pad_;
    int32_t tok[kSmallNodes];
    int32_t pos[kSmallNodes];
    uint64_t mask[kSmallNodes];             // ancestor-or-self bits of node i
};

// Inputs of a batched decode step (sp_decode_batch) that its captured graph reads from fixed device
// memory; the step's last kernel advances them (each request's argmax becomes its next token).
constexpr int kBatchMax = 64;
struct BatchIn {
    BatchLane lanes[kBatchMax];
    int32_t tok[kBatchMax];
    int32_t pos[kBatchMax];
    int32_t argmax[kBatchMax];
    int32_t out[kBatchMax];
};

// Inputs of one packed pass of several requests' prompts (sp_prefill_batch): every token's lane
// (its request's cache and slot) and position, and the rows of the prompts' last tokens.
constexpr int kPrefillBatchMax = 256;      // requests per sp_prefill_batch call
struct PrefillBatchIn {
    BatchLane lanes[kPrefillMaxTokens];
    int32_t pos[kPrefillMaxTokens];
    int32_t last[kPrefillMaxTokens];
};

struct LayerDev {
    const uint8_t *qkv, *o, *gate_up, *down;       // fragment-packed fp16, contiguous in the stream
    const float *qkv_b, *in_norm, *post_norm;
    size_t off_qkv, off_o, off_gu, off_dn;          // offsets in the weight stream
    PrefillLayer pf{};                              // row-major copies for the batched prompt pass
};

// Stage ring per GEMV CTA. CTAs of consecutive kernels share an SM under programmatic dependent
// launch, so ring + input fragments stay near half of the 227 KB of shared memory.
constexpr int kRingBytes = 96 * 1024;
constexpr int kMaxUnitBytes = 32 * 1024;
constexpr int kTcRingBytes = 64 * 1024;     // 4 stages of 16 KB per tensor-core GEMV CTA
constexpr int kTcBBudget = 64 * 1024;       // B operand (hi/lo activation rows) per CTA
constexpr int kArgmaxChunkRows = 64;        // sp_argmax rows per launch (engine scratch is sized for it)
constexpr int kMaxDevices = 64;             // sp_argmax_noalloc: per-device scratch addresses

}  // namespace

struct sp_kv {
    sp_engine *e;
    int32_t capacity;
    int32_t length;
    __half *k, *v;
};

struct sp_engine {
    sp_config c{};
    int device = 0;
    int num_sms = 0;
    bool pdl = true;
    bool use_graph = true;
    uint8_t *arena = nullptr;
    size_t arena_bytes = 0;
    uint8_t *ws = nullptr;
    size_t ws_bytes = 0;
    size_t ws_clear_bytes = 0;              // prefix of ws holding counters and split-strip state
    // The per-token weight stream: every layer's [qkv | o | gate_up | down], then the LM head, in
    // consumption order and contiguous, so prefetching "D bytes ahead" is one address window.
    const uint8_t *stream = nullptr;
    size_t stream_bytes = 0;
    size_t prefetch_ahead = 0;
    bool evict_first = false;
    const __half *embed = nullptr;          // row-major embedding (token gathers)
    const uint8_t *head = nullptr;          // fragment-packed LM head (tied: a packed copy of embed)
    size_t off_head = 0;
    const float *final_norm = nullptr;
    const float *rope = nullptr;
    std::vector<LayerDev> layers;
    // workspace
    float *x = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr;
    float *partial = nullptr;
    unsigned *strip_cnt = nullptr;
    unsigned *lm_cnt = nullptr;
    float *lm_val = nullptr;
    int *lm_idx = nullptr;
    DevState *st = nullptr;
    ArgmaxScratch am{};                     // sp_argmax: kArgmaxChunkRows rows per launch
    // persistent step kernel (default; SEEDPLANE_STEP=chain selects the kernel-per-op chain)
    bool step_kernel = true;
    StepOp s_qkv{}, s_o{}, s_gu{}, s_down{}, s_head{};     // planned step GEMVs (row blocks)
    StepLayout step_lay{};                  // shared memory of the step kernel
    int step_xmax = 0, step_max_chunks = 0;
    int step_group_chunks = 0, step_group_ctx = 0, step_part_stride = 0;   // grouped attention items
    int step_inflight = 0;                  // ring copies in flight at most (0: all stages)
    int step_l2_ahead = 0;                  // bytes per CTA prefetched into L2 ahead of the ring
    unsigned long long *cnt = nullptr;      // dependency counters [5 * layers]
    unsigned long long *epoch = nullptr;    // finished steps (never reset by set-state)
    int n_cnt = 0;
    // step hand-offs, two of each (layer parity): LL words of the residual stream after O (xo) and
    // after down (xd), q, the new K/V rows, attention partials and output; the SwiGLU activation
    uint64_t *ll_xo = nullptr, *ll_xd = nullptr, *ll_q = nullptr, *ll_kv = nullptr, *ll_part = nullptr,
             *ll_attn = nullptr;
    uint64_t *ll_ksp = nullptr;             // split GEMVs' row partials, per parity: for O, down, QKV,
                                            // gate_up kMaxKsplit - 1 regions of the op's N words
    __half *act_h = nullptr, *act_l = nullptr;
    std::map<sp_kv *, StepOp *> step_ops;   // device op table per cache (its K/V pointers)
    int n_step_ops = 0;
    unsigned long long *step_trace = nullptr;
    unsigned long long *trace = nullptr;    // [kernel of the step][CTA][kTraceWords], SEEDPLANE_TRACE=1
    int trace_kernels = 0;
    // planned GEMV geometry (pointers filled per layer at record time)
    bool tc = true;                         // tcgen05 GEMVs (else the mma.sync fragment GEMVs)
    GemvParams g_qkv{}, g_o{}, g_gu{}, g_down{}, g_head{};
    TcGemvParams t_qkv{}, t_o{}, t_gu{}, t_down{}, t_head{};
    cudaStream_t cap_stream = nullptr;
    std::map<std::pair<sp_kv *, int>, cudaGraphExec_t> graphs;   // step per (cache, grouped attention)
    // batched prompt pass (prefill.cu); off with SEEDPLANE_PREFILL=steps
    bool prefill = false;
    PrefillDims pf_dims{};
    PrefillScratch pf{};
    uint8_t *pf_mem = nullptr;
    size_t pf_bytes = 0;
    PrefillMat head_pf{};                   // row-major LM head for the batched pass (the embedding when tied)
    VerifyIn *vt = nullptr;                 // device copy of the block inputs (tree verify, slot base)
    int32_t *acc_scratch = nullptr;         // stochastic acceptance: tree inputs / outputs
    double *acc_rows = nullptr;             // stochastic acceptance: the visited rows' (max, S) and p / q, fp64
    size_t acc_rows_bytes = 0;
    int32_t *gr_buf = nullptr;              // greedy acceptance: tree, path ends and result
    BatchIn *bt = nullptr;                  // batched decode inputs
    PrefillBatchIn *bp = nullptr;           // packed prompt pass inputs
    int32_t *last_only_buf = nullptr;       // sp_forward(all_logits = 2) through the step path: per-step argmaxes
    int32_t last_only_cap = 0;
    std::map<int, cudaGraphExec_t> bgraphs; // batched decode step per batch size
    int32_t *vt_argmax = nullptr;           // [kSmallNodes] argmax of a captured verify pass
    std::map<std::pair<sp_kv *, int>, cudaGraphExec_t> vgraphs;   // verify pass per (cache, nodes)
    unsigned long long *mc_trace = nullptr;  // SEEDPLANE_MCOL_TRACE: stamps of the last multi-column GEMM
    std::vector<sp_kv *> caches;
};

namespace {

// L2 prefetch window of a kernel that streams [off, off + bytes) of the weight stream: the same
// number of bytes, `prefetch_ahead` further on (wrapping into the next token's first layers).
void set_prefetch(const sp_engine *e, GemvParams &p, size_t off, size_t bytes) {
    p.pf_n = 0;
    p.evict_first = e->evict_first ? 1 : 0;
    if (!e->prefetch_ahead || !e->stream_bytes) return;
    size_t beg = (off + e->prefetch_ahead) % e->stream_bytes;
    size_t left = std::min(bytes, e->stream_bytes);
    while (left && p.pf_n < kMaxPrefetch) {
        const size_t n = std::min(left, e->stream_bytes - beg);
        p.pf_ptr[p.pf_n] = e->stream + beg;
        p.pf_bytes[p.pf_n] = n;
        ++p.pf_n;
        left -= n;
        beg = 0;
    }
}

unsigned long long *trace_slot(sp_engine *e, int k) {
    return e->trace ? e->trace + (size_t)k * e->num_sms * kTraceWords : nullptr;
}

// The same GEMV call on the tensor-core kernel: copy the call-site fields across.
cudaError_t launch_tc_from(sp_engine *e, const TcGemvParams &plan, int pro, int epi, const GemvParams &g,
                           const LaunchCfg &lc) {
    TcGemvParams t = plan;
    t.w = g.w;
    t.xin = g.xin;
    t.gain = g.gain;
    t.embed = g.embed;
    t.x_init = g.x_init;
    t.bias = g.bias;
    t.out = g.out;
    t.kc = g.kc;
    t.vc = g.vc;
    t.cap = g.cap;
    for (int i = 0; i < kMaxPrefetch; ++i) {
        t.pf_ptr[i] = g.pf_ptr[i];
        t.pf_bytes[i] = g.pf_bytes[i];
    }
    t.pf_n = g.pf_n;
    t.trace = g.trace;
    return launch_gemv_tc(pro, epi, t, lc);
}

cudaError_t launch_any_gemv(sp_engine *e, int which, int pro, int epi, const GemvParams &g, const LaunchCfg &lc) {
    if (!e->tc) return launch_gemv(pro, epi, g, lc);
    const TcGemvParams *plans[] = {&e->t_qkv, &e->t_o, &e->t_gu, &e->t_down, &e->t_head};
    return launch_tc_from(e, *plans[which], pro, epi, g, lc);
}

// The step's op table for one cache: per layer QKV, attention, O, gate_up, down (ops 5l .. 5l + 4);
// then the LM head. Layer l uses hand-off buffers of parity l & 1; the residual stream the QKV
// projection and the LM head read is the previous down projection's output. Counter 5l + 3
// counts the gate_up CTAs of layer l (the only counted hand-off).
std::vector<StepOp> build_step_ops(const sp_engine *e, const sp_kv *kv) {
    const sp_config &c = e->c;
    const size_t kv_layer = (size_t)c.kv_heads * kv->capacity * c.head_dim;
    const size_t H = c.hidden, I = c.intermediate, HD = c.head_dim;
    const size_t nq = (size_t)c.heads * HD, nkv = (size_t)c.kv_heads * HD;
    const size_t npart = (size_t)c.heads * e->step_part_stride * (HD + 2);
    std::vector<StepOp> ops;
    // split-GEMV partials, per layer parity: kMaxKsplit - 1 regions of N words for each op kind
    const size_t ksp_o = 0, ksp_down = ksp_o + (kMaxKsplit - 1) * (size_t)e->s_o.N;
    const size_t ksp_qkv = ksp_down + (kMaxKsplit - 1) * (size_t)e->s_down.N;
    const size_t ksp_gu = ksp_qkv + (kMaxKsplit - 1) * (size_t)e->s_qkv.N;
    const size_t ksp_par = ksp_gu + (kMaxKsplit - 1) * (size_t)e->s_gu.N;
    auto gemv = [&](const StepOp &plan, const uint8_t *w, int pro, int epi) {
        StepOp o = plan;
        o.kind = OP_GEMV;
        o.w = w;
        o.pro = pro;
        o.epi = epi;
        o.dep = -1;
        o.sig = -1;
        return o;
    };
    for (int l = 0; l < c.layers; ++l) {
        const LayerDev &L = e->layers[l];
        const int par = l & 1, prev = par ^ 1;
        __half *kc = kv->k + l * kv_layer, *vc = kv->v + l * kv_layer;
        StepOp o = gemv(e->s_qkv, L.qkv, l == 0 ? PRO_EMBED_NORM : PRO_NORM, EPI_QKV);
        if (l > 0) {
            o.lin = e->ll_xd + prev * H;
            o.lin_k = 5 * (l - 1) + 4;
        }
        o.gain = L.in_norm;
        o.bias = L.qkv_b;
        o.lout = e->ll_q + par * nq;
        o.lkv = e->ll_kv + par * nkv;
        o.lksp = e->ll_ksp + par * ksp_par + ksp_qkv;
        o.kc = kc;
        o.vc = vc;
        ops.push_back(o);
        StepOp a{};
        a.kind = OP_ATTN;
        a.kc = kc;
        a.vc = vc;
        a.lin = e->ll_q + par * nq;
        a.lin_k = 5 * l;
        a.lkv = e->ll_kv + par * nkv;
        a.lpart = e->ll_part + par * npart;
        a.lout = e->ll_attn + par * nq;
        a.dep = -1;
        a.sig = -1;
        ops.push_back(a);
        o = gemv(e->s_o, L.o, PRO_ATTN, EPI_RESID);
        o.lin = e->ll_attn + par * nq;
        o.lin_k = 5 * l + 1;
        if (l > 0) {                       // layer 0: the residual base is the token's embedding row
            o.lres = e->ll_xd + prev * H;
            o.lres_k = 5 * (l - 1) + 4;
        }
        o.lout = e->ll_xo + par * H;
        o.lksp = e->ll_ksp + par * ksp_par + ksp_o;
        ops.push_back(o);
        o = gemv(e->s_gu, L.gate_up, PRO_NORM, EPI_SWIGLU);
        o.lin = e->ll_xo + par * H;
        o.lin_k = 5 * l + 2;
        o.gain = L.post_norm;
        o.out_h = e->act_h + par * 2 * I;
        o.out_l = e->act_l + par * 2 * I;
        o.lksp = e->ll_ksp + par * ksp_par + ksp_gu;
        o.sig = 5 * l + 3;
        ops.push_back(o);
        o = gemv(e->s_down, L.down, PRO_PLAIN, EPI_RESID);
        o.xin_h = e->act_h + par * 2 * I;
        o.xin_l = e->act_l + par * 2 * I;
        o.dep = 5 * l + 3;
        o.dep_n = e->s_gu.grid;
        o.lres = e->ll_xo + par * H;
        o.lres_k = 5 * l + 2;
        o.lout = e->ll_xd + par * H;
        o.lksp = e->ll_ksp + par * ksp_par + ksp_down;
        ops.push_back(o);
    }
    StepOp o = gemv(e->s_head, e->head, PRO_NORM, EPI_LMHEAD);
    o.lin = e->ll_xd + ((c.layers - 1) & 1) * H;
    o.lin_k = 5 * (c.layers - 1) + 4;
    o.gain = e->final_norm;
    ops.push_back(o);
    return ops;
}

int ensure_step_ops(sp_engine *e, sp_kv *kv, StepOp **out) {
    auto it = e->step_ops.find(kv);
    if (it != e->step_ops.end()) {
        *out = it->second;
        return SP_OK;
    }
    const std::vector<StepOp> ops = build_step_ops(e, kv);
    for (const StepOp &o : ops)            // a split GEMV's second CTAs store their partials through lksp
        if (o.kind == OP_GEMV && o.ksplit > 1 && o.lksp == nullptr)
            return fail(SP_ERR_UNSUPPORTED, "step op table: a split GEMV (N=%d K=%d) has no partials buffer", o.N, o.K);
    StepOp *d = nullptr;
    SP_CUDA(cudaMalloc(&d, ops.size() * sizeof(StepOp)));
    cudaError_t ce = cudaMemcpy(d, ops.data(), ops.size() * sizeof(StepOp), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
        cudaFree(d);
        return fail(SP_ERR_CUDA, "step op table: %s", cudaGetErrorString(ce));
    }
    e->n_step_ops = (int)ops.size();
    e->step_ops[kv] = d;
    *out = d;
    return SP_OK;
}

// grouped: the step kernel's grouped attention items (one per kv head and chunk)
int record_step(sp_engine *e, sp_kv *kv, cudaStream_t s, bool grouped) {
    const sp_config &c = e->c;
    if (e->step_kernel) {
        StepOp *ops = nullptr;
        int rc = ensure_step_ops(e, kv, &ops);
        if (rc != SP_OK) return rc;
        StepParams p{};
        p.ops = ops;
        p.n_ops = e->n_step_ops;
        p.stages = e->step_lay.stages;
        p.stage_bytes = e->step_lay.stage_bytes;
        p.vec_bytes = e->step_lay.vec_bytes;
        p.attn_off = e->step_lay.attn_off;
        p.nh = c.heads;
        p.nkv = c.kv_heads;
        p.hd = c.head_dim;
        p.cap = kv->capacity;
        p.max_pos = c.max_positions;
        p.vocab = c.vocab;
        p.hidden = c.hidden;
        p.max_chunks = e->step_max_chunks;
        p.group_chunks = e->step_group_chunks;
        p.part_stride = e->step_part_stride;
        p.evict_first = e->evict_first ? 1 : 0;
        p.max_inflight = e->step_inflight;
        p.l2_ahead = e->step_l2_ahead;
        p.eps = c.rms_norm_eps;
        p.scale = 1.0f / sqrtf((float)c.head_dim);
        p.rope = e->rope;
        p.embed = e->embed;
        p.part_val = e->lm_val;
        p.part_idx = e->lm_idx;
        p.lm_cnt = e->lm_cnt;
        p.cnt = e->cnt;
        p.epoch = e->epoch;
        p.st = e->st;
        p.trace = e->step_trace;
        SP_CUDA(launch_step(c.head_dim, p, e->num_sms, e->step_lay.smem, s, e->pdl,
                            e->c.weight_format == SP_WEIGHTS_I8_B32, grouped));
        return SP_OK;
    }
    int kidx = 0;       // GEMV index within the step (trace slot)
    const size_t kv_layer = (size_t)c.kv_heads * kv->capacity * c.head_dim;
    const size_t H = c.hidden, I = c.intermediate, QR = (size_t)(c.heads + 2 * c.kv_heads) * c.head_dim;
    for (int l = 0; l < c.layers; ++l) {
        const LayerDev &L = e->layers[l];
        LaunchCfg lc{s, e->pdl && l > 0};
        GemvParams p = e->g_qkv;
        p.w = L.qkv;
        p.xin = e->x;
        p.gain = L.in_norm;
        p.bias = L.qkv_b;
        p.out = e->q;
        p.kc = kv->k + l * kv_layer;
        p.vc = kv->v + l * kv_layer;
        p.cap = kv->capacity;
        set_prefetch(e, p, L.off_qkv, QR * H * 2);
        p.trace = trace_slot(e, kidx++);
        const int pro = l == 0 ? PRO_EMBED_NORM : PRO_NORM;
        SP_CUDA(launch_any_gemv(e, 0, pro, EPI_QKV, p, lc));
        lc.pdl = e->pdl;

        AttnParams a{};
        a.q = e->q;
        a.kc = kv->k + l * kv_layer;
        a.vc = kv->v + l * kv_layer;
        a.out = e->attn;
        a.nh = c.heads;
        a.nkv = c.kv_heads;
        a.hd = c.head_dim;
        a.cap = kv->capacity;
        a.scale = 1.0f / sqrtf((float)c.head_dim);
        a.st = e->st;
        // the attention kernels of layer 0 and of the middle layer are traced after the GEMV slots
        a.trace = (e->trace && (l == 0 || l == c.layers / 2))
                      ? e->trace + (size_t)(e->trace_kernels + (l == 0 ? 0 : 1)) * e->num_sms * kTraceWords
                      : nullptr;
        SP_CUDA(launch_attention(a, lc));

        p = e->g_o;
        p.w = L.o;
        p.xin = e->attn;
        p.out = e->x;
        set_prefetch(e, p, L.off_o, H * H * 2);
        p.trace = trace_slot(e, kidx++);
        SP_CUDA(launch_any_gemv(e, 1, PRO_PLAIN, EPI_RESID, p, lc));

        p = e->g_gu;
        p.w = L.gate_up;
        p.xin = e->x;
        p.gain = L.post_norm;
        p.out = e->act;
        set_prefetch(e, p, L.off_gu, 2 * I * H * 2);
        p.trace = trace_slot(e, kidx++);
        SP_CUDA(launch_any_gemv(e, 2, PRO_NORM, EPI_SWIGLU, p, lc));

        p = e->g_down;
        p.w = L.down;
        p.xin = e->act;
        p.out = e->x;
        set_prefetch(e, p, L.off_dn, H * I * 2);
        p.trace = trace_slot(e, kidx++);
        SP_CUDA(launch_any_gemv(e, 3, PRO_PLAIN, EPI_RESID, p, lc));
    }
    LaunchCfg lc{s, e->pdl};
    GemvParams p = e->g_head;
    p.xin = e->x;
    p.gain = e->final_norm;
    set_prefetch(e, p, e->off_head, align_up(c.vocab, e->tc ? 128 : 16) * H * 2);
    p.trace = trace_slot(e, kidx++);
    SP_CUDA(launch_any_gemv(e, 4, PRO_NORM, EPI_LMHEAD, p, lc));
    return SP_OK;
}

int get_graph(sp_engine *e, sp_kv *kv, bool grouped, cudaGraphExec_t *out) {
    const auto key = std::make_pair(kv, grouped ? 1 : 0);
    auto it = e->graphs.find(key);
    if (it != e->graphs.end()) {
        *out = it->second;
        return SP_OK;
    }
    cudaGraph_t g = nullptr;
    SP_CUDA(cudaStreamBeginCapture(e->cap_stream, cudaStreamCaptureModeThreadLocal));
    int rc = record_step(e, kv, e->cap_stream, grouped);
    cudaError_t ce = cudaStreamEndCapture(e->cap_stream, &g);
    if (rc != SP_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (ce != cudaSuccess) return fail(SP_ERR_CUDA, "graph capture: %s", cudaGetErrorString(ce));
    cudaGraphExec_t ex = nullptr;
    ce = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return fail(SP_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(ce));
    e->graphs[key] = ex;
    *out = ex;
    return SP_OK;
}

int run_steps(sp_engine *e, sp_kv *kv, const DevState &init, int n, cudaStream_t s) {
    if (e->step_kernel) {
        StepOp *ops = nullptr;                // built outside any stream capture
        int rc = ensure_step_ops(e, kv, &ops);
        if (rc != SP_OK) return rc;
    }
    SP_CUDA(launch_set_state(e->st, init, s));
    // the first step's visible context decides the attention items of the whole block
    const bool grouped = e->step_kernel && (long)init.slot + 1 >= (long)e->step_group_ctx;
    if (e->use_graph) {
        cudaGraphExec_t ex;
        int rc = get_graph(e, kv, grouped, &ex);
        if (rc != SP_OK) return rc;
        for (int i = 0; i < n; ++i) SP_CUDA(cudaGraphLaunch(ex, s));
    } else {
        for (int i = 0; i < n; ++i) {
            int rc = record_step(e, kv, s, grouped);
            if (rc != SP_OK) return rc;
        }
    }
    return SP_OK;
}

DevState base_state() {
    DevState d;
    memset(&d, 0, sizeof(d));
    d.tree_base = 0x7fffffff;
    return d;
}

bool env_flag(const char *name, bool dflt) {
    const char *v = getenv(name);
    if (!v || !*v) return dflt;
    return !(v[0] == '0' || v[0] == 'n' || v[0] == 'N' || v[0] == 'f' || v[0] == 'F');
}

long env_long(const char *name, long dflt) {
    const char *v = getenv(name);
    if (!v || !*v) return dflt;
    return strtol(v, nullptr, 10);
}

}  // namespace

extern "C" {

const char *sp_last_error(void) { return g_err.c_str(); }

const char *sp_version(void) { return "seedplane-b200 0.2 (sm_100a)"; }

int sp_engine_create(const sp_config *cfg, const sp_weights *w, int device, sp_engine **out) {
    if (!cfg || !w || !out) return fail(SP_ERR_INVALID, "null argument");
    *out = nullptr;
    const sp_config c = *cfg;
    if (c.layers <= 0 || c.hidden <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.vocab <= 0 || c.intermediate <= 0)
        return fail(SP_ERR_INVALID, "non-positive dimension in config");
    if (c.hidden % c.heads || c.heads % c.kv_heads || c.head_dim != c.hidden / c.heads)
        return fail(SP_ERR_INVALID, "invalid Qwen2 head configuration");
    if (c.head_dim != 64 && c.head_dim != 128) return fail(SP_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
    if (c.heads / c.kv_heads > 8) return fail(SP_ERR_UNSUPPORTED, "more than 8 q heads per kv head");
    if (c.hidden % 16 || c.intermediate % 16)
        return fail(SP_ERR_UNSUPPORTED, "hidden and intermediate must be multiples of 16");
    if (c.weight_format != SP_WEIGHTS_F16 && c.weight_format != SP_WEIGHTS_I8_B32)
        return fail(SP_ERR_INVALID, "unknown weight format %d", c.weight_format);
    const bool i8 = c.weight_format == SP_WEIGHTS_I8_B32;
    if (c.max_positions <= 0) return fail(SP_ERR_INVALID, "max_positions must be positive");
    if (!w->embed || !w->final_norm || !w->layers) return fail(SP_ERR_INVALID, "missing tensors");
    if (!c.tied_embeddings && !w->lm_head) return fail(SP_ERR_INVALID, "untied model without lm_head");
    for (int l = 0; l < c.layers; ++l) {
        const sp_layer_weights &Lw = w->layers[l];
        if (!Lw.qkv_w || !Lw.qkv_b || !Lw.o_w || !Lw.gate_w || !Lw.up_w || !Lw.down_w || !Lw.in_norm || !Lw.post_norm)
            return fail(SP_ERR_INVALID, "layer %d: missing tensor", l);
        if (i8 && (!Lw.qkv_s || !Lw.o_s || !Lw.gate_s || !Lw.up_s || !Lw.down_s))
            return fail(SP_ERR_INVALID, "layer %d: missing int8 block scales", l);
    }
    if (i8 && !c.tied_embeddings && !w->lm_head_s) return fail(SP_ERR_INVALID, "int8 lm_head without scales");
    if (i8 && (c.hidden % 128 || c.intermediate % 128))
        return fail(SP_ERR_UNSUPPORTED, "int8 weights need hidden and intermediate in multiples of 128");

    SP_CUDA(cudaSetDevice(device));
    sp_engine *e = new sp_engine();
    e->c = c;
    e->device = device;
    e->pdl = env_flag("SEEDPLANE_PDL", true);
    e->use_graph = env_flag("SEEDPLANE_GRAPH", true);
    e->prefetch_ahead = (size_t)std::max(0L, env_long("SEEDPLANE_L2_PREFETCH_MB", 0)) << 20;
    e->evict_first = env_flag("SEEDPLANE_EVICT_FIRST", true);
    {
        const char *g = getenv("SEEDPLANE_GEMV");
        e->tc = !(g && strcmp(g, "hmma") == 0);
        const char *st = getenv("SEEDPLANE_STEP");
        e->step_kernel = e->tc && !(st && strcmp(st, "chain") == 0);
    }
    if (i8 && !e->step_kernel) {
        delete e;
        return fail(SP_ERR_UNSUPPORTED, "int8 blockwise weights run on the step kernel only");
    }
    cudaDeviceGetAttribute(&e->num_sms, cudaDevAttrMultiProcessorCount, device);

    const size_t H = c.hidden, I = c.intermediate, V = c.vocab, HD = c.head_dim;
    // Output rows padded with zero rows to whole strips of the kernel-per-op GEMVs: 128 (tensor
    // core) or 16 (fragment GEMV); the step kernel only needs row pairs.
    const size_t rowpad = e->step_kernel ? 2 : (e->tc ? 128 : 16);
    const size_t VP = align_up(V, rowpad);
    if (e->tc && !e->step_kernel &&
        ((size_t)(c.heads + 2 * c.kv_heads) * c.head_dim % 128 || c.hidden % 128 || (2 * (size_t)c.intermediate) % 128)) {
        delete e;
        return fail(SP_ERR_UNSUPPORTED, "tensor-core GEMV needs qkv rows, hidden and 2*intermediate in multiples of 128");
    }
    const size_t QR = (size_t)(c.heads + 2 * c.kv_heads) * HD;
    const size_t padq = e->step_kernel ? rowpad : 1;
    const size_t QRp = align_up(QR, padq), Hp = align_up(H, padq), GUp = align_up(2 * I, padq);
    if (e->step_kernel) {
        // the input splits first (they depend on the shapes only), then the shared-memory layout
        // (a CTA's share of the largest input sizes its vector region; the stage size bounds the
        // units), then the row-block plans (the packing depends on them)
        const int max_ks = (int)env_long("SEEDPLANE_STEP_KSPLIT", kMaxKsplit);
        auto sbase = [&](size_t N, size_t K, size_t n_valid, int pro, int epi, bool q8, int stage_bytes) {
            StepOp o{};
            o.kind = OP_GEMV;
            o.fmt = q8 ? WF_I8 : WF_F16;
            o.pro = pro;
            o.epi = epi;
            o.N = (int)N;
            o.K = (int)K;
            o.n_valid = (int)n_valid;
            plan_step_gemv(o, e->num_sms, stage_bytes, max_ks);
            return o;
        };
        auto share_k = [&](size_t N, size_t K, int pro, int epi) {
            return K / (size_t)std::max(sbase(N, K, N, pro, epi, i8, 64 * 1024).ksplit, 1);   // any stage size
        };
        e->step_xmax = (int)align_up(std::max({H, share_k(Hp, I, PRO_PLAIN, EPI_RESID),
                                               share_k(Hp, (size_t)c.heads * HD, PRO_ATTN, EPI_RESID)}), 8);
        const int want = (int)env_long("SEEDPLANE_STEP_STAGES", 3);
        e->step_inflight = (int)env_long("SEEDPLANE_STEP_INFLIGHT", 0);
        e->step_l2_ahead = (int)env_long("SEEDPLANE_STEP_L2_KB", 0) * 1024;
        e->step_lay = step_layout((int)H, e->step_xmax, (int)HD, std::max(2, want), i8);
        if (e->step_lay.stage_bytes < 16 * 1024 && want > 2) e->step_lay = step_layout((int)H, e->step_xmax, (int)HD, 2, i8);
        if (e->step_lay.stage_bytes < 16 * 1024) {
            delete e;
            return fail(SP_ERR_UNSUPPORTED, "step kernel: the input vector of %d floats leaves no room for the ring",
                        e->step_xmax);
        }
        const int sb = e->step_lay.stage_bytes;
        e->s_qkv = sbase(QRp, H, QR, PRO_NORM, EPI_QKV, i8, sb);
        e->s_o = sbase(Hp, H, H, PRO_ATTN, EPI_RESID, i8, sb);
        e->s_gu = sbase(GUp, H, 2 * I, PRO_NORM, EPI_SWIGLU, i8, sb);
        e->s_down = sbase(Hp, I, H, PRO_PLAIN, EPI_RESID, i8, sb);
        e->s_head = sbase(VP, H, V, PRO_NORM, EPI_LMHEAD, i8 && !c.tied_embeddings, sb);   // a tied head is the fp16 embedding
        for (const StepOp *o : {&e->s_qkv, &e->s_o, &e->s_gu, &e->s_down, &e->s_head}) {
            // a CTA's input share in the vector region: int8 digits and block scales, or fp16 halves
            const size_t kc = (size_t)o->K / std::max(o->ksplit, 1);
            const size_t in = o->fmt == WF_I8 ? 4 * (kc + 16) + kc / 8 : 4 * (size_t)o->K;
            if (!step_gemv_supported(*o, e->step_lay.stage_bytes) || in > (size_t)e->step_lay.vec_bytes) {
                delete e;
                return fail(SP_ERR_UNSUPPORTED, "step GEMV of N=%d K=%d is not supported", o->N, o->K);
            }
        }
    }
    // ---- arena: [weight stream][embed][small tensors] ------------------------------------------
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes, 256); return o; };
    struct LOff { size_t qkv, o, gu, dn, qkv_b, inn, post, rqkv, ro, rgu, rdn, rqkv_lo, ro_lo, rgu_lo, rdn_lo; };
    std::vector<LOff> lo(c.layers);
    // packed matrix bytes: fp16 sizes are multiples of 512 B (no gaps); int8 ones of 32 B
    auto mbytes = [&](const StepOp &o, size_t N, size_t K) { return e->step_kernel ? step_gemv_bytes(o) : N * K * 2; };
    for (int l = 0; l < c.layers; ++l) {
        lo[l].qkv = take(mbytes(e->s_qkv, QRp, H));
        lo[l].o = take(mbytes(e->s_o, Hp, H));
        lo[l].gu = take(mbytes(e->s_gu, GUp, H));
        lo[l].dn = take(mbytes(e->s_down, Hp, I));
    }
    const size_t o_head = take(mbytes(e->s_head, VP, H));
    const size_t stream_end = off;
    const size_t o_embed = take(V * H * 2);
    const size_t o_fnorm = take(H * 4);
    const size_t o_rope = take((size_t)c.max_positions * (HD / 2) * 2 * 4);
    for (int l = 0; l < c.layers; ++l) {
        lo[l].qkv_b = take(QR * 4);
        lo[l].inn = take(H * 4);
        lo[l].post = take(H * 4);
    }
    // row-major copies for the batched prompt pass: the fp16 weights, or for int8 checkpoints the
    // int8 rows and their block scales times a power of two (the GEMM dequantizes them on the chip
    // into exact fp16 hi / lo halves): 1 + 1/16 bytes a weight
    e->prefill = !(getenv("SEEDPLANE_PREFILL") && strcmp(getenv("SEEDPLANE_PREFILL"), "steps") == 0);
    size_t o_head_rm = 0, o_head_rm_lo = 0;
    auto kb64 = [](size_t K) { return (K + 63) / 64; };
    if (e->prefill) {
        const size_t AQ = (size_t)c.heads * HD;
        for (int l = 0; l < c.layers; ++l) {
            lo[l].rqkv = take(QR * H * (i8 ? 1 : 2));
            lo[l].ro = take(H * AQ * (i8 ? 1 : 2));
            lo[l].rgu = take(2 * I * H * (i8 ? 1 : 2));
            lo[l].rdn = take(H * I * (i8 ? 1 : 2));
            if (i8) {                                   // scales [ceil(K / 64)][N][2] fp16
                lo[l].rqkv_lo = take(kb64(H) * QR * 4);
                lo[l].ro_lo = take(kb64(AQ) * H * 4);
                lo[l].rgu_lo = take(kb64(H) * 2 * I * 4);
                lo[l].rdn_lo = take(kb64(I) * H * 4);
            }
        }
        if (!c.tied_embeddings) {
            o_head_rm = take(V * H * (i8 ? 1 : 2));
            if (i8) o_head_rm_lo = take(kb64(H) * V * 4);
        }
    }
    e->arena_bytes = off;
    cudaError_t ce = cudaMalloc(&e->arena, e->arena_bytes);
    if (ce != cudaSuccess) {
        delete e;
        return fail(SP_ERR_CUDA, "weight arena of %zu bytes: %s", off, cudaGetErrorString(ce));
    }
    uint8_t *A = e->arena;
    cudaStream_t s = nullptr;
    int *d_idx = nullptr;
    float *d_absmax = nullptr;
    auto bail = [&](int code) {
        cudaFree(d_idx);
        cudaFree(d_absmax);
        if (s) cudaStreamDestroy(s);
        sp_engine_destroy(e);
        return code;
    };
#define SP_TRY(call)                                                                                 \
    do {                                                                                             \
        cudaError_t e_ = (call);                                                                     \
        if (e_ != cudaSuccess) return bail(fail(SP_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_))); \
    } while (0)
    SP_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    // ---- pack ------------------------------------------------------------------------------
    // Row maps (packed row -> source row): QKV rows are reordered so the two rows of a RoPE pair
    // (d, d + head_dim/2) of a head are adjacent; gate and up rows are interleaved (gate_i, up_i).
    // (padded rows map to -1 = zero row)
    const size_t n_iota = std::max(std::max(VP, GUp), std::max(QRp, Hp));
    std::vector<int> idx(QRp + GUp + n_iota, -1);
    int *h_perm = idx.data(), *h_gu = idx.data() + QRp, *h_iota = idx.data() + QRp + GUp;
    for (size_t r = 0; r < QR; ++r) {
        const size_t hh = r / HD, j = r % HD;
        h_perm[r] = (int)(hh * HD + (j / 2) + (j % 2) * (HD / 2));
    }
    for (size_t i = 0; i < I; ++i) {
        h_gu[2 * i] = (int)i;
        h_gu[2 * i + 1] = (int)(I + i);
    }
    for (size_t i = 0; i < n_iota; ++i) h_iota[i] = i < H ? (int)i : -1;
    std::vector<int> head_rows(VP);
    for (size_t i = 0; i < VP; ++i) head_rows[i] = i < V ? (int)i : -1;
    idx.insert(idx.end(), head_rows.begin(), head_rows.end());
    for (size_t i = 0; i < I; ++i) idx.push_back((int)i);
    SP_TRY(cudaMalloc(&d_idx, idx.size() * 4));
    SP_TRY(cudaMemcpy(d_idx, idx.data(), idx.size() * 4, cudaMemcpyHostToDevice));
    const int *d_head_rows = d_idx + QRp + GUp + n_iota;
    const int *d_perm = d_idx, *d_gu = d_idx + QRp, *d_iota = d_idx + QRp + GUp;
    const int *d_seq = d_idx + QRp + GUp + n_iota + VP;      // 0, 1, .., I - 1
    SP_TRY(cudaMemcpyAsync(A + o_embed, w->embed, V * H * 2, cudaMemcpyDeviceToDevice, s));
    const __half *head_src = (const __half *)(c.tied_embeddings ? w->embed : w->lm_head);
    auto pack = [&](uint8_t *dst, const void *a, const void *as, int rows_a, const void *b, const void *bs,
                    const int *row_of, int N, int K, const StepOp &plan) {
        if (e->step_kernel && plan.fmt == WF_I8) {
            cudaError_t me = cudaMemsetAsync(dst, 0, step_gemv_bytes(plan), s);
            if (me != cudaSuccess) return me;
            return launch_pack_rows_i8(dst, (const int8_t *)a, (const __half *)as, rows_a, (const int8_t *)b,
                                       (const __half *)bs, row_of, plan, s);
        }
        const __half *ah = (const __half *)a, *bh = (const __half *)b;
        return e->step_kernel ? launch_pack_rows(dst, ah, rows_a, bh, row_of, plan, s)
               : e->tc        ? launch_pack_tc(dst, ah, rows_a, bh, row_of, N, K, s)
                              : launch_pack_fragments(dst, ah, rows_a, bh, row_of, N, K, s);
    };
    SP_TRY(pack(A + o_head, head_src, c.tied_embeddings ? nullptr : w->lm_head_s, (int)V, nullptr, nullptr,
                d_head_rows, (int)VP, (int)H, e->s_head));
    // int8 row-major copies: exponent k per matrix so that its largest weight times 2^k is near 2^15
    // (fp16 range, and the lo halves of the large weights stay normal); one alpha = 2^-k per matrix
    auto dequant = [&](size_t hi_off, size_t lo_off, const void *q1, const void *s1, int rows1, const void *q2,
                       const void *s2, int rows2, int K, PrefillMat &m, int pair_hd = 0) -> cudaError_t {
        // with a second matrix (gate_up: gate, then up) the rows are interleaved: 2i = q1 row i, 2i + 1 = q2 row i
        float mx = 0.f, mx2 = 0.f;
        cudaError_t er = launch_int8_absmax(d_absmax, (const __half *)s1, (long long)rows1 * (K / 32), s);
        if (er == cudaSuccess) er = cudaMemcpyAsync(&mx, d_absmax, 4, cudaMemcpyDeviceToHost, s);
        if (er == cudaSuccess && q2) er = launch_int8_absmax(d_absmax, (const __half *)s2, (long long)rows2 * (K / 32), s);
        if (er == cudaSuccess && q2) er = cudaMemcpyAsync(&mx2, d_absmax, 4, cudaMemcpyDeviceToHost, s);
        if (er == cudaSuccess) er = cudaStreamSynchronize(s);
        if (er != cudaSuccess) return er;
        mx = std::max(mx, mx2);
        int k = 0;
        if (mx > 0.f && std::isfinite(mx)) k = std::min(30, std::max(-30, (int)std::floor(std::log2(32768.0 / mx))));
        if (k < 0) return cudaErrorInvalidValue;      // block scales above 2^15 / 127: not this format
        int8_t *dq = (int8_t *)(A + hi_off);
        __half *dsc = (__half *)(A + lo_off);
        const int N = q2 ? rows1 + rows2 : rows1;
        er = cudaMemsetAsync(dsc, 0, (size_t)((K + 63) / 64) * N * 4, s);
        if (er == cudaSuccess)
            er = launch_repack_i8(dq, dsc, (const int8_t *)q1, (const __half *)s1, rows1, N, K, k, q2 ? 2 : 1, 0,
                                  pair_hd, s);
        if (er == cudaSuccess && q2)
            er = launch_repack_i8(dq, dsc, (const int8_t *)q2, (const __half *)s2, rows2, N, K, k, 2, 1, 0, s);
        m = PrefillMat{};
        m.q = dq;
        m.sc = dsc;
        m.alpha = ldexpf(1.0f, -k);
        return er;
    };
    if (e->prefill && i8) SP_TRY(cudaMalloc(&d_absmax, sizeof(float)));
    PrefillMat head_pf{c.tied_embeddings ? (const __half *)w->embed : nullptr, nullptr, 1.0f};
    if (e->prefill && !c.tied_embeddings) {
        if (i8) {
            SP_TRY(dequant(o_head_rm, o_head_rm_lo, w->lm_head, w->lm_head_s, (int)V, nullptr, nullptr, 0, (int)H,
                           head_pf));
        } else {
            SP_TRY(cudaMemcpyAsync(A + o_head_rm, w->lm_head, V * H * 2, cudaMemcpyDeviceToDevice, s));
            head_pf.hi = (const __half *)(A + o_head_rm);
        }
    }
    SP_TRY(cudaMemcpyAsync(A + o_fnorm, w->final_norm, H * 4, cudaMemcpyDeviceToDevice, s));
    for (int l = 0; l < c.layers; ++l) {
        const sp_layer_weights &Lw = w->layers[l];
        SP_TRY(pack(A + lo[l].qkv, Lw.qkv_w, Lw.qkv_s, (int)QR, nullptr, nullptr, d_perm, (int)QRp, (int)H, e->s_qkv));
        SP_TRY(pack(A + lo[l].o, Lw.o_w, Lw.o_s, (int)H, nullptr, nullptr, d_iota, (int)Hp, (int)H, e->s_o));
        SP_TRY(pack(A + lo[l].gu, Lw.gate_w, Lw.gate_s, (int)I, Lw.up_w, Lw.up_s, d_gu, (int)GUp, (int)H, e->s_gu));
        SP_TRY(pack(A + lo[l].dn, Lw.down_w, Lw.down_s, (int)H, nullptr, nullptr, d_iota, (int)Hp, (int)I, e->s_down));
        SP_TRY(cudaMemcpyAsync(A + lo[l].qkv_b, Lw.qkv_b, QR * 4, cudaMemcpyDeviceToDevice, s));
        SP_TRY(cudaMemcpyAsync(A + lo[l].inn, Lw.in_norm, H * 4, cudaMemcpyDeviceToDevice, s));
        SP_TRY(cudaMemcpyAsync(A + lo[l].post, Lw.post_norm, H * 4, cudaMemcpyDeviceToDevice, s));
        LayerDev L;
        if (e->prefill && i8) {
            const int A_ = c.heads * (int)HD;
            SP_TRY(dequant(lo[l].rqkv, lo[l].rqkv_lo, Lw.qkv_w, Lw.qkv_s, (int)QR, nullptr, nullptr, 0, (int)H, L.pf.qkv,
                           (int)HD));
            SP_TRY(dequant(lo[l].ro, lo[l].ro_lo, Lw.o_w, Lw.o_s, (int)H, nullptr, nullptr, 0, A_, L.pf.o));
            SP_TRY(dequant(lo[l].rgu, lo[l].rgu_lo, Lw.gate_w, Lw.gate_s, (int)I, Lw.up_w, Lw.up_s, (int)I, (int)H,
                           L.pf.gate_up));
            SP_TRY(dequant(lo[l].rdn, lo[l].rdn_lo, Lw.down_w, Lw.down_s, (int)H, nullptr, nullptr, 0, (int)I, L.pf.down));
        } else if (e->prefill) {
            // QKV rows with RoPE partners adjacent (the GEMM's QKV epilogue pairs them)
            SP_TRY(launch_gather_rows(A + lo[l].rqkv, (const uint8_t *)Lw.qkv_w, d_perm, (int)QR, (int)H * 2, 1, 0, s));
            SP_TRY(cudaMemcpyAsync(A + lo[l].ro, Lw.o_w, H * (size_t)c.heads * HD * 2, cudaMemcpyDeviceToDevice, s));
            // gate and up rows interleaved (2i = gate i, 2i + 1 = up i): the GEMM's SwiGLU epilogue pairs them
            SP_TRY(launch_gather_rows(A + lo[l].rgu, (const uint8_t *)Lw.gate_w, d_seq, (int)I, (int)H * 2, 2, 0, s));
            SP_TRY(launch_gather_rows(A + lo[l].rgu, (const uint8_t *)Lw.up_w, d_seq, (int)I, (int)H * 2, 2, 1, s));
            SP_TRY(cudaMemcpyAsync(A + lo[l].rdn, Lw.down_w, H * I * 2, cudaMemcpyDeviceToDevice, s));
            L.pf.qkv = PrefillMat{(const __half *)(A + lo[l].rqkv), nullptr, 1.0f};
            L.pf.o = PrefillMat{(const __half *)(A + lo[l].ro), nullptr, 1.0f};
            L.pf.gate_up = PrefillMat{(const __half *)(A + lo[l].rgu), nullptr, 1.0f};
            L.pf.down = PrefillMat{(const __half *)(A + lo[l].rdn), nullptr, 1.0f};
        }
        L.qkv = A + lo[l].qkv;
        L.o = A + lo[l].o;
        L.gate_up = A + lo[l].gu;
        L.down = A + lo[l].dn;
        L.qkv_b = (const float *)(A + lo[l].qkv_b);
        L.in_norm = (const float *)(A + lo[l].inn);
        L.post_norm = (const float *)(A + lo[l].post);
        L.off_qkv = lo[l].qkv;
        L.off_o = lo[l].o;
        L.off_gu = lo[l].gu;
        L.off_dn = lo[l].dn;
        if (e->prefill) {
            L.pf.qkv_b = L.qkv_b;
            L.pf.in_norm = L.in_norm;
            L.pf.post_norm = L.post_norm;
        }
        e->layers.push_back(L);
    }
    // RoPE table: the caller's (computed like the reference, qwen_engine.py:52,99-103), else double precision.
    {
        std::vector<float> rope;
        const float *host = w->rope_host;
        if (!host) {
            rope.resize((size_t)c.max_positions * (HD / 2) * 2);
            for (int pos = 0; pos < c.max_positions; ++pos)
                for (size_t i = 0; i < HD / 2; ++i) {
                    const float inv = (float)(1.0 / pow((double)c.rope_theta, (double)(2 * i) / (double)HD));
                    const float ph = (float)pos * inv;
                    rope[((size_t)pos * (HD / 2) + i) * 2] = (float)cos((double)ph);
                    rope[((size_t)pos * (HD / 2) + i) * 2 + 1] = (float)sin((double)ph);
                }
            host = rope.data();
        }
        SP_TRY(cudaMemcpy(A + o_rope, host, (size_t)c.max_positions * (HD / 2) * 2 * 4, cudaMemcpyHostToDevice));
    }
    SP_TRY(cudaStreamSynchronize(s));
    cudaFree(d_idx);
    d_idx = nullptr;
    cudaFree(d_absmax);
    d_absmax = nullptr;
    e->stream = A;
    e->stream_bytes = stream_end;
    e->embed = (const __half *)(A + o_embed);
    e->head = A + o_head;
    e->off_head = o_head;
    e->final_norm = (const float *)(A + o_fnorm);
    e->rope = (const float *)(A + o_rope);
    e->head_pf = head_pf;
    if (c.tied_embeddings) e->head_pf.hi = e->embed;

    // ---- GEMV plans -------------------------------------------------------------------------
    auto base = [&](size_t N, size_t K) {
        GemvParams p{};
        p.N = (int)N;
        p.K = (int)K;
        p.fmt = WF_F16;
        p.eps = c.rms_norm_eps;
        p.vocab = (int)V;
        p.rope = e->rope;
        p.max_pos = c.max_positions;
        p.nh = c.heads;
        p.nkv = c.kv_heads;
        p.hd = (int)HD;
        plan_gemv(p, e->num_sms, kRingBytes, kMaxUnitBytes);
        return p;
    };
    e->g_qkv = base(QR, H);
    e->g_o = base(H, H);
    e->g_gu = base(2 * I, H);
    e->g_down = base(H, I);
    e->g_head = base(VP, H);
    e->g_head.n_valid = (int)V;
    auto tbase = [&](size_t N, size_t K, int n_valid) {
        TcGemvParams t{};
        t.N = (int)N;
        t.K = (int)K;
        t.n_valid = n_valid;
        t.eps = c.rms_norm_eps;
        t.vocab = (int)V;
        t.rope = e->rope;
        t.max_pos = c.max_positions;
        t.nh = c.heads;
        t.nkv = c.kv_heads;
        t.hd = (int)HD;
        plan_gemv_tc(t, e->num_sms, kTcRingBytes, kTcBBudget);
        return t;
    };
    if (e->tc && !e->step_kernel) {
        e->t_qkv = tbase(QR, H, (int)QR);
        e->t_o = tbase(H, H, (int)H);
        e->t_gu = tbase(2 * I, H, (int)(2 * I));
        e->t_down = tbase(H, I, (int)H);
        e->t_head = tbase(VP, H, (int)V);
        for (const TcGemvParams *t : {&e->t_qkv, &e->t_o, &e->t_gu, &e->t_down, &e->t_head})
            if (t->max_items > gemv_tc_max_items() || gemv_tc_smem_bytes(*t) > 227 * 1024)
                return bail(fail(SP_ERR_UNSUPPORTED, "tensor-core GEMV plan for N=%d K=%d does not fit (%d strips per CTA, %zu B smem)",
                                 t->N, t->K, t->max_items, gemv_tc_smem_bytes(*t)));
    }
    if (env_flag("SEEDPLANE_VERBOSE", false) && e->step_kernel) {
        const char *names[] = {"qkv", "o", "gate_up", "down", "lm_head"};
        int k = 0;
        for (const StepOp *o : {&e->s_qkv, &e->s_o, &e->s_gu, &e->s_down, &e->s_head})
            fprintf(stderr, "[seedplane] step gemv %-8s %s N=%d K=%d grid=%d ksplit=%d pass_rows=%d chunk=%d\n",
                    names[k++], o->fmt == WF_I8 ? "i8" : "f16", o->N, o->K, o->grid, o->ksplit, o->pass_rows,
                    o->chunk_w);
    }
    if (env_flag("SEEDPLANE_VERBOSE", false) && e->tc && !e->step_kernel) {
        const char *names[] = {"qkv", "o", "gate_up", "down", "lm_head"};
        int k = 0;
        for (const TcGemvParams *t : {&e->t_qkv, &e->t_o, &e->t_gu, &e->t_down, &e->t_head})
            fprintf(stderr, "[seedplane] tc gemv %-8s N=%d K=%d grid=%d stages=%d b_full=%d b_tiles=%d contrib<=%d items<=%d smem=%zu\n",
                    names[k++], t->N, t->K, t->grid, t->stages, t->b_full, t->b_tiles, t->max_contrib, t->max_items,
                    gemv_tc_smem_bytes(*t));
    }
    if (env_flag("SEEDPLANE_VERBOSE", false) && !e->tc) {
        const char *names[] = {"qkv", "o", "gate_up", "down", "lm_head"};
        int k = 0;
        for (const GemvParams *p : {&e->g_qkv, &e->g_o, &e->g_gu, &e->g_down, &e->g_head})
            fprintf(stderr, "[seedplane] gemv %-8s N=%d K=%d tiles/unit=%d units/strip=%d stages=%d grid=%d smem=%zu\n",
                    names[k++], p->N, p->K, p->nt, p->ks, p->stages, p->grid, gemv_smem_bytes(*p));
    }

    // ---- workspace ------------------------------------------------------------------------
    size_t n_partial = 0, n_strips = 0;
    for (const GemvParams *p : {&e->g_qkv, &e->g_o, &e->g_gu, &e->g_down, &e->g_head}) {
        if (p->ks > 1) {
            n_partial = std::max(n_partial, (size_t)p->N * p->ks);
            n_strips = std::max(n_strips, (size_t)p->N / 16);
        }
    }
    if (e->tc)
        for (const TcGemvParams *t : {&e->t_qkv, &e->t_o, &e->t_gu, &e->t_down, &e->t_head}) {
            n_partial = std::max(n_partial, (size_t)t->N * t->max_contrib);
            n_strips = std::max(n_strips, (size_t)t->N / 128);
        }
    size_t woff = 0;
    auto wtake = [&](size_t bytes) { size_t o = woff; woff = align_up(woff + bytes, 256); return o; };
    // counters and split-strip state first: a device error clears exactly this prefix
    e->n_cnt = 5 * c.layers;
    // attention chunks per q head at most (SEEDPLANE_ATTN_MAX_CHUNKS lowers the cap: longer items,
    // e.g. to exercise many sub-chunks per item at small contexts)
    const int chunk_cap = (int)std::max(1L, env_long("SEEDPLANE_ATTN_MAX_CHUNKS", kStepMaxChunks));
    e->step_max_chunks = std::min({kStepMaxChunks, chunk_cap, e->num_sms / c.heads});
    // grouped items (one per kv head and chunk, all q heads of the group at once) from
    // SEEDPLANE_ATTN_GROUP_CTX visible positions on (0: always; a value above every context: never)
    // chunks: as many as leave one CTA per q head free for the merges (which then poll while the
    // items run instead of after them), SEEDPLANE_ATTN_GROUP_CHUNKS at most
    const int group_cap = (int)std::max(1L, env_long("SEEDPLANE_ATTN_GROUP_CHUNKS", kStepMaxChunks));
    const int group_fit = e->num_sms - c.heads >= c.kv_heads ? (e->num_sms - c.heads) / c.kv_heads
                                                             : e->num_sms / c.kv_heads;
    e->step_group_chunks = std::max(1, std::min({kStepMaxChunks, group_cap, group_fit}));
    // default (measured on the Qwen2 shapes): grouped items from the first position when a group
    // has 7 or more q heads (per-head items read every K/V row 7 times), else from 640 visible
    // positions on (Qwen2-1.5B's 6-head groups: per-head items are 0.3 % faster at 512-640
    // positions, grouped ones 1.5 % at 768-896, 2 % at 1,024 and 13 % at 4,096)
    const long group_dflt = c.heads / c.kv_heads >= 7 ? 0L : 640L;
    e->step_group_ctx = (int)std::max(0L, std::min<long>(INT_MAX, env_long("SEEDPLANE_ATTN_GROUP_CTX", group_dflt)));
    e->step_part_stride = std::max(e->step_max_chunks, e->step_group_chunks);
    const size_t w_cnt = wtake((size_t)e->n_cnt * 8), w_epoch = wtake(8);
    const size_t w_scnt = wtake(std::max<size_t>(n_strips, 1) * 4);
    const size_t w_lmcnt = wtake(4);
    const size_t w_am = wtake(argmax_scratch_bytes(kArgmaxChunkRows));
    // step hand-off words (a step after a device error must not see tags of the failed one)
    const size_t n_part = (size_t)c.heads * e->step_part_stride * (HD + 2);
    const size_t w_llxo = wtake(2 * H * 8), w_llxd = wtake(2 * H * 8);
    const size_t w_llq = wtake(2 * (size_t)c.heads * HD * 8), w_llkv = wtake(2 * (size_t)c.kv_heads * HD * 8);
    const size_t w_llpart = wtake(2 * n_part * 8), w_llattn = wtake(2 * (size_t)c.heads * HD * 8);
    const size_t w_llksp = wtake(2 * (kMaxKsplit - 1) *
                                 ((size_t)e->s_o.N + e->s_down.N + e->s_qkv.N + e->s_gu.N) * 8);
    e->ws_clear_bytes = woff;
    const size_t w_x = wtake(H * 4), w_q = wtake((size_t)c.heads * HD * 4);
    const size_t w_attn = wtake((size_t)c.heads * HD * 4), w_act = wtake(I * 4);
    const size_t w_partial = wtake(std::max<size_t>(n_partial, 1) * 4);
    const size_t lm_grid = std::max({(size_t)e->g_head.grid, (size_t)e->t_head.grid, (size_t)e->num_sms});
    const size_t w_lmval = wtake(lm_grid * 4), w_lmidx = wtake(lm_grid * 4);
    const size_t w_st = wtake(sizeof(DevState));
    const size_t w_acth = wtake(4 * I * 2);
    e->ws_bytes = woff;
    SP_TRY(cudaMalloc(&e->ws, e->ws_bytes));
    SP_TRY(cudaMemset(e->ws, 0, e->ws_bytes));
    if (e->prefill) {
        e->pf_dims = PrefillDims{(int)H, (int)I, c.heads, c.kv_heads, (int)HD, (int)V, c.max_positions,
                                 kPrefillMaxTokens, c.rms_norm_eps};
        e->pf_bytes = prefill_scratch_bytes(e->pf_dims);
        SP_TRY(cudaMalloc(&e->pf_mem, e->pf_bytes));
        e->pf = prefill_scratch_at(e->pf_mem, e->pf_dims);
        if (getenv("SEEDPLANE_MCOL_TRACE") && atoi(getenv("SEEDPLANE_MCOL_TRACE")) != 0) {
            SP_TRY(cudaMalloc(&e->mc_trace, (size_t)kPrefillMaxCtas * kMcolTraceWords * 8));
            SP_TRY(cudaMemset(e->mc_trace, 0, (size_t)kPrefillMaxCtas * kMcolTraceWords * 8));
        }
        SP_TRY(cudaMalloc(&e->vt, sizeof(VerifyIn) + kSmallNodes * sizeof(int32_t)));
        e->vt_argmax = reinterpret_cast<int32_t *>(e->vt + 1);
    }
    e->x = (float *)(e->ws + w_x);
    e->q = (float *)(e->ws + w_q);
    e->attn = (float *)(e->ws + w_attn);
    e->act = (float *)(e->ws + w_act);
    e->partial = (float *)(e->ws + w_partial);
    e->strip_cnt = (unsigned *)(e->ws + w_scnt);
    e->lm_cnt = (unsigned *)(e->ws + w_lmcnt);
    e->lm_val = (float *)(e->ws + w_lmval);
    e->lm_idx = (int *)(e->ws + w_lmidx);
    e->st = (DevState *)(e->ws + w_st);
    e->am = argmax_scratch_at(e->ws + w_am, kArgmaxChunkRows);
    e->cnt = (unsigned long long *)(e->ws + w_cnt);
    e->epoch = (unsigned long long *)(e->ws + w_epoch);
    e->ll_xo = (uint64_t *)(e->ws + w_llxo);
    e->ll_xd = (uint64_t *)(e->ws + w_llxd);
    e->ll_q = (uint64_t *)(e->ws + w_llq);
    e->ll_kv = (uint64_t *)(e->ws + w_llkv);
    e->ll_part = (uint64_t *)(e->ws + w_llpart);
    e->ll_attn = (uint64_t *)(e->ws + w_llattn);
    e->ll_ksp = (uint64_t *)(e->ws + w_llksp);
    e->act_h = (__half *)(e->ws + w_acth);        // parity p: hi at [2p I, 2p I + I), lo right after
    e->act_l = e->act_h + I;
    e->g_head.w = e->head;
    e->g_head.part_val = e->lm_val;
    e->g_head.part_idx = e->lm_idx;
    e->g_head.counter = e->lm_cnt;
    for (GemvParams *p : {&e->g_qkv, &e->g_o, &e->g_gu, &e->g_down, &e->g_head}) {
        p->st = e->st;
        p->partial = e->partial;
        p->strip_cnt = e->strip_cnt;
    }
    e->g_qkv.embed = e->embed;
    e->g_qkv.x_init = e->x;
    for (TcGemvParams *t : {&e->t_qkv, &e->t_o, &e->t_gu, &e->t_down, &e->t_head}) {
        t->st = e->st;
        t->partial = e->partial;
        t->strip_cnt = e->strip_cnt;
    }
    e->t_head.part_val = e->lm_val;
    e->t_head.part_idx = e->lm_idx;
    e->t_head.counter = e->lm_cnt;
    e->t_head.w = e->head;
    if (!e->tc) {
        SP_TRY(prepare_gemv(PRO_NORM, EPI_QKV, e->g_qkv));
        SP_TRY(prepare_gemv(PRO_EMBED_NORM, EPI_QKV, e->g_qkv));
        SP_TRY(prepare_gemv(PRO_PLAIN, EPI_RESID, e->g_o));
        SP_TRY(prepare_gemv(PRO_NORM, EPI_SWIGLU, e->g_gu));
        SP_TRY(prepare_gemv(PRO_PLAIN, EPI_RESID, e->g_down));
        SP_TRY(prepare_gemv(PRO_NORM, EPI_LMHEAD, e->g_head));
    }
    SP_TRY(prepare_attention());
    if (e->tc && !e->step_kernel) {
        SP_TRY(prepare_gemv_tc(PRO_NORM, EPI_QKV, e->t_qkv));
        SP_TRY(prepare_gemv_tc(PRO_EMBED_NORM, EPI_QKV, e->t_qkv));
        SP_TRY(prepare_gemv_tc(PRO_PLAIN, EPI_RESID, e->t_o));
        SP_TRY(prepare_gemv_tc(PRO_NORM, EPI_SWIGLU, e->t_gu));
        SP_TRY(prepare_gemv_tc(PRO_PLAIN, EPI_RESID, e->t_down));
        SP_TRY(prepare_gemv_tc(PRO_NORM, EPI_LMHEAD, e->t_head));
    }
    if (e->step_kernel) {
        if (e->step_max_chunks < 1 || c.heads * e->step_max_chunks > e->num_sms ||
            c.kv_heads * e->step_group_chunks > e->num_sms)
            return bail(fail(SP_ERR_UNSUPPORTED, "step kernel: %d q heads do not fit one attention item per CTA",
                             c.heads));
        SP_TRY(prepare_step((int)HD, e->step_lay.smem, i8));
        if (env_flag("SEEDPLANE_VERBOSE", false))
            fprintf(stderr, "[seedplane] step kernel: grid=%d stages=%d x %d B xmax=%d smem=%zu max_chunks=%d\n",
                    e->num_sms, e->step_lay.stages, e->step_lay.stage_bytes, e->step_xmax, e->step_lay.smem,
                    e->step_max_chunks);
    }
    for (const GemvParams *p : {&e->g_qkv, &e->g_o, &e->g_gu, &e->g_down, &e->g_head})
        if (!e->tc && gemv_smem_bytes(*p) > 227 * 1024) return bail(fail(SP_ERR_UNSUPPORTED, "GEMV needs %zu bytes of shared memory", gemv_smem_bytes(*p)));
    if (env_flag("SEEDPLANE_TRACE", false) && e->step_kernel) {
        const size_t words = (size_t)(5 * c.layers + 1) * e->num_sms * kStepTraceWords;
        SP_TRY(cudaMalloc(&e->step_trace, words * 8));
        SP_TRY(cudaMemset(e->step_trace, 0, words * 8));
    } else if (env_flag("SEEDPLANE_TRACE", false)) {
        e->trace_kernels = 4 * c.layers + 1;       // + 2 attention slots after the GEMVs
        SP_TRY(cudaMalloc(&e->trace, (size_t)(e->trace_kernels + 2) * e->num_sms * kTraceWords * 8));
        SP_TRY(cudaMemset(e->trace, 0, (size_t)(e->trace_kernels + 2) * e->num_sms * kTraceWords * 8));
    }
    e->cap_stream = s;
    s = nullptr;
#undef SP_TRY
    *out = e;
    return SP_OK;
}

void sp_engine_destroy(sp_engine *e) {
    if (!e) return;
    cudaSetDevice(e->device);
    for (auto &kv : e->graphs) cudaGraphExecDestroy(kv.second);
    for (auto &kv : e->step_ops) cudaFree(kv.second);
    cudaFree(e->step_trace);
    for (sp_kv *kv : e->caches) kv->e = nullptr;
    if (e->cap_stream) cudaStreamDestroy(e->cap_stream);
    cudaFree(e->arena);
    cudaFree(e->ws);
    cudaFree(e->trace);
    for (auto &g : e->vgraphs) cudaGraphExecDestroy(g.second);
    cudaFree(e->pf_mem);
    cudaFree(e->mc_trace);
    cudaFree(e->vt);
    cudaFree(e->acc_scratch);
    cudaFree(e->acc_rows);
    cudaFree(e->gr_buf);
    for (auto &g : e->bgraphs) cudaGraphExecDestroy(g.second);
    cudaFree(e->bt);
    cudaFree(e->bp);
    cudaFree(e->last_only_buf);
    delete e;
}

int64_t sp_engine_device_bytes(const sp_engine *e) {
    return e ? (int64_t)(e->arena_bytes + e->ws_bytes + e->pf_bytes) : 0;
}

int sp_kv_create(sp_engine *e, int32_t capacity, sp_kv **out) {
    if (!e || !out) return fail(SP_ERR_INVALID, "null argument");
    if (capacity < 1) return fail(SP_ERR_INVALID, "cache capacity must be positive");
    SP_CUDA(cudaSetDevice(e->device));
    const size_t n = (size_t)e->c.layers * e->c.kv_heads * capacity * e->c.head_dim;
    sp_kv *kv = new sp_kv();
    kv->e = e;
    kv->capacity = capacity;
    kv->length = 0;
    cudaError_t ce = cudaMalloc(&kv->k, n * 2);
    if (ce == cudaSuccess) ce = cudaMalloc(&kv->v, n * 2);
    if (ce == cudaSuccess) ce = cudaMemset(kv->k, 0, n * 2);
    if (ce == cudaSuccess) ce = cudaMemset(kv->v, 0, n * 2);
    if (ce != cudaSuccess) {
        cudaFree(kv->k);
        cudaFree(kv->v);
        delete kv;
        return fail(SP_ERR_CUDA, "KV cache of %d slots: %s", capacity, cudaGetErrorString(ce));
    }
    e->caches.push_back(kv);
    *out = kv;
    return SP_OK;
}

void sp_kv_destroy(sp_kv *kv) {
    if (!kv) return;
    if (kv->e) {
        sp_engine *e = kv->e;
        cudaSetDevice(e->device);
        for (auto g = e->graphs.begin(); g != e->graphs.end();) {
            if (g->first.first == kv) {
                cudaGraphExecDestroy(g->second);
                g = e->graphs.erase(g);
            } else {
                ++g;
            }
        }
        auto so = e->step_ops.find(kv);
        if (so != e->step_ops.end()) {
            cudaFree(so->second);
            e->step_ops.erase(so);
        }
        for (auto vg = e->vgraphs.begin(); vg != e->vgraphs.end();) {
            if (vg->first.first == kv) {
                cudaGraphExecDestroy(vg->second);
                vg = e->vgraphs.erase(vg);
            } else {
                ++vg;
            }
        }
        for (size_t i = 0; i < e->caches.size(); ++i)
            if (e->caches[i] == kv) { e->caches.erase(e->caches.begin() + i); break; }
    }
    cudaFree(kv->k);
    cudaFree(kv->v);
    delete kv;
}

int32_t sp_kv_length(const sp_kv *kv) { return kv ? kv->length : -1; }
int32_t sp_kv_capacity(const sp_kv *kv) { return kv ? kv->capacity : -1; }

int sp_kv_set_length(sp_kv *kv, int32_t length) {
    if (!kv) return fail(SP_ERR_INVALID, "null cache");
    if (length < 0 || length > kv->capacity) return fail(SP_ERR_CAPACITY, "length %d outside [0, %d]", length, kv->capacity);
    kv->length = length;
    return SP_OK;
}

static int check_engine_kv(sp_engine *e, sp_kv *kv) {
    if (!e || !kv) return fail(SP_ERR_INVALID, "null engine or cache");
    if (kv->e != e) return fail(SP_ERR_INVALID, "cache belongs to another engine");
    cudaError_t ce = cudaSetDevice(e->device);
    if (ce != cudaSuccess) return fail(SP_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(ce));
    return SP_OK;
}

// The batched pass: chunks of up to kPrefillMaxTokens tokens through all layers at once
// (prefill.cu), then the head in blocks of kPrefillLogitRows rows: logits (all rows, or the last
// row) and every row's argmax. The K/V of the block land at slots *slot_base + 0 .. n - 1 (the
// base is read on the device, so a captured graph serves any cache length). `mask`: tree-verify
// ancestor masks (n <= kSmallNodes), else causal.
static int forward_batched(sp_engine *e, sp_kv *kv, const int32_t *tok, const int32_t *pos, const uint64_t *mask,
                           const int32_t *slot_base, int32_t n, float *logits, bool all_logits, int32_t *argmax,
                           cudaStream_t s, bool last_only = false) {
    const sp_config &c = e->c;
    const size_t kv_layer = (size_t)c.kv_heads * kv->capacity * c.head_dim;
    const float scale = 1.0f / sqrtf((float)c.head_dim);
    for (int32_t b0 = 0; b0 < n; b0 += kPrefillMaxTokens) {
        const int T = std::min<int32_t>(kPrefillMaxTokens, n - b0);
        SP_CUDA(launch_prefill_embed(e->pf_dims, e->pf, e->embed, tok + b0, T, e->st, s));
        for (int l = 0; l < c.layers; ++l) {
            const PrefillLayer &L = e->layers[l].pf;
            SP_CUDA(launch_prefill_layer_front(e->pf_dims, L, e->pf, T, pos ? pos + b0 : nullptr,
                                               mask ? mask + b0 : nullptr, kv->k + l * kv_layer, kv->v + l * kv_layer,
                                               kv->capacity, slot_base, b0, scale, e->rope, e->st, s));
            SP_CUDA(launch_prefill_layer_ffn(e->pf_dims, L, e->pf, T, e->st, s));
        }
        // last_only: the head of the last token alone (argmax[0], logits [vocab])
        if (last_only) {
            if (b0 + T < n) continue;
            SP_CUDA(launch_prefill_logits(e->pf_dims, e->pf, e->final_norm, e->head_pf, T - 1, 1, e->pf.logits, e->st, s));
            if (argmax) SP_CUDA(launch_argmax_rows(e->pf.logits, 1, c.vocab, c.vocab, argmax, e->am, s));
            if (logits)
                SP_CUDA(cudaMemcpyAsync(logits, e->pf.logits, (size_t)c.vocab * 4, cudaMemcpyDeviceToDevice, s));
            continue;
        }
        for (int r0 = 0; r0 < T; r0 += kPrefillLogitRows) {
            const int rows = std::min(kPrefillLogitRows, T - r0);
            float *out = all_logits && logits ? logits + (size_t)(b0 + r0) * c.vocab : e->pf.logits;
            SP_CUDA(launch_prefill_logits(e->pf_dims, e->pf, e->final_norm, e->head_pf, r0, rows, out, e->st, s));
            SP_CUDA(launch_argmax_rows(out, rows, c.vocab, c.vocab, argmax + b0 + r0, e->am, s));
            if (!all_logits && logits && b0 + r0 + rows == n)
                SP_CUDA(cudaMemcpyAsync(logits, out + (size_t)(rows - 1) * c.vocab, (size_t)c.vocab * 4,
                                        cudaMemcpyDeviceToDevice, s));
        }
    }
    return SP_OK;
}

// One verify pass of n tree nodes as a CUDA graph per (cache, n): inputs in e->vt, argmaxes out
// in e->vt_argmax.
static int verify_graph(sp_engine *e, sp_kv *kv, int n, cudaGraphExec_t *out) {
    auto key = std::make_pair(kv, n);
    auto it = e->vgraphs.find(key);
    if (it != e->vgraphs.end()) {
        *out = it->second;
        return SP_OK;
    }
    cudaGraph_t g = nullptr;
    SP_CUDA(cudaStreamBeginCapture(e->cap_stream, cudaStreamCaptureModeThreadLocal));
    int rc = forward_batched(e, kv, e->vt->tok, e->vt->pos, e->vt->mask, &e->vt->slot0, n, nullptr, false,
                             e->vt_argmax, e->cap_stream);
    cudaError_t ce = cudaStreamEndCapture(e->cap_stream, &g);
    if (rc != SP_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (ce != cudaSuccess) return fail(SP_ERR_CUDA, "verify graph capture: %s", cudaGetErrorString(ce));
    cudaGraphExec_t ex = nullptr;
    ce = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return fail(SP_ERR_CUDA, "verify graph instantiate: %s", cudaGetErrorString(ce));
    e->vgraphs[key] = ex;
    *out = ex;
    return SP_OK;
}

int sp_forward(sp_engine *e, sp_kv *kv, const int32_t *tokens_dev, const int32_t *positions_dev, int32_t n,
               float *logits_dev, int32_t all_logits, int32_t *argmax_dev, void *stream) {
    int rc = check_engine_kv(e, kv);
    if (rc) return rc;
    if (n <= 0 || !tokens_dev) return fail(SP_ERR_INVALID, "input_ids cannot be empty");
    if (kv->length + n > kv->capacity) return fail(SP_ERR_CAPACITY, "KV cache capacity %d exceeded", kv->capacity);
    if (all_logits < 0 || all_logits > 2) return fail(SP_ERR_INVALID, "all_logits must be 0, 1 or 2");
    if (e->prefill && n >= kPrefillMin) {
        cudaStream_t s = (cudaStream_t)stream;
        const int32_t base = kv->length;
        SP_CUDA(cudaMemcpyAsync(&e->vt->slot0, &base, sizeof(base), cudaMemcpyHostToDevice, s));
        rc = forward_batched(e, kv, tokens_dev, positions_dev, nullptr, &e->vt->slot0, n, logits_dev, all_logits == 1,
                             argmax_dev, s, all_logits == 2);
        if (rc) return rc;
        kv->length += n;
        return SP_OK;
    }
    DevState d = base_state();
    d.n_forced = n;
    d.slot0 = kv->length;
    d.slot = kv->length;
    d.f_tok = tokens_dev;
    d.f_pos = positions_dev;
    d.logits = logits_dev;
    d.logits_stride = all_logits == 1 ? (long long)e->c.vocab : 0;
    d.logits_from = all_logits == 1 ? 0 : n - 1;
    d.out_tokens = argmax_dev;
    if (all_logits == 2 && argmax_dev && n > 1) {
        // the last token's argmax alone, at argmax_dev[0]: the steps write theirs to the engine's scratch
        if (e->last_only_cap < n) {
            cudaFree(e->last_only_buf);
            e->last_only_buf = nullptr;
            e->last_only_cap = 0;
            SP_CUDA(cudaMalloc(&e->last_only_buf, (size_t)n * sizeof(int32_t)));
            e->last_only_cap = n;
        }
        d.out_tokens = e->last_only_buf;
    }
    rc = run_steps(e, kv, d, n, (cudaStream_t)stream);
    if (!rc && all_logits == 2 && argmax_dev && n > 1)
        SP_CUDA(cudaMemcpyAsync(argmax_dev, e->last_only_buf + n - 1, sizeof(int32_t), cudaMemcpyDeviceToDevice,
                                (cudaStream_t)stream));
    if (rc) return rc;
    kv->length += n;
    return SP_OK;
}

int sp_decode(sp_engine *e, sp_kv *kv, int32_t token, int32_t pos, int32_t n_steps, int32_t *out_tokens_dev,
              float *logits_dev, void *stream) {
    int rc = check_engine_kv(e, kv);
    if (rc) return rc;
    if (n_steps <= 0) return fail(SP_ERR_INVALID, "n_steps must be positive");
    if (token < 0 || token >= e->c.vocab) return fail(SP_ERR_INVALID, "token %d outside the vocabulary", token);
    if (kv->length + n_steps > kv->capacity) return fail(SP_ERR_CAPACITY, "KV cache capacity %d exceeded", kv->capacity);
    if (pos < 0 || pos + n_steps > e->c.max_positions)
        return fail(SP_ERR_CAPACITY, "positions %d..%d outside the RoPE table", pos, pos + n_steps - 1);
    DevState d = base_state();
    d.token = token;
    d.pos = pos;
    d.slot = kv->length;
    d.slot0 = kv->length;
    d.logits = logits_dev;
    d.logits_from = n_steps - 1;
    d.out_tokens = out_tokens_dev;
    rc = run_steps(e, kv, d, n_steps, (cudaStream_t)stream);
    if (rc) return rc;
    kv->length += n_steps;
    return SP_OK;
}

// One greedy step of a batch of independent requests (e->bt): the batched pass over B tokens, each
// writing and attending to its own cache, every row's LM head and argmax, then the advance.
static int batch_step(sp_engine *e, int B, cudaStream_t s) {
    const sp_config &c = e->c;
    const float scale = 1.0f / sqrtf((float)c.head_dim);
    SP_CUDA(launch_prefill_embed(e->pf_dims, e->pf, e->embed, e->bt->tok, B, e->st, s));
    for (int l = 0; l < c.layers; ++l) {
        const PrefillLayer &L = e->layers[l].pf;
        SP_CUDA(launch_batch_layer_front(e->pf_dims, L, e->pf, B, e->bt->pos, e->bt->lanes, l, scale, e->rope, e->st, s));
        SP_CUDA(launch_prefill_layer_ffn(e->pf_dims, L, e->pf, B, e->st, s));
    }
    SP_CUDA(launch_prefill_logits(e->pf_dims, e->pf, e->final_norm, e->head_pf, 0, B, e->pf.logits, e->st, s));
    SP_CUDA(launch_argmax_rows(e->pf.logits, B, c.vocab, c.vocab, e->bt->argmax, e->am, s));
    SP_CUDA(launch_batch_advance(e->bt->lanes, e->bt->tok, e->bt->pos, e->bt->argmax, e->bt->out, B, c.max_positions,
                                 e->st, s));
    return SP_OK;
}

static int batch_graph(sp_engine *e, int B, cudaGraphExec_t *out) {
    auto it = e->bgraphs.find(B);
    if (it != e->bgraphs.end()) {
        *out = it->second;
        return SP_OK;
    }
    cudaGraph_t g = nullptr;
    SP_CUDA(cudaStreamBeginCapture(e->cap_stream, cudaStreamCaptureModeThreadLocal));
    int rc = batch_step(e, B, e->cap_stream);
    cudaError_t ce = cudaStreamEndCapture(e->cap_stream, &g);
    if (rc != SP_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (ce != cudaSuccess) return fail(SP_ERR_CUDA, "batch graph capture: %s", cudaGetErrorString(ce));
    cudaGraphExec_t ex = nullptr;
    ce = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return fail(SP_ERR_CUDA, "batch graph instantiate: %s", cudaGetErrorString(ce));
    e->bgraphs[B] = ex;
    *out = ex;
    return SP_OK;
}

int sp_decode_batch(sp_engine *e, sp_kv *const *kvs, int32_t B, const int32_t *tokens_host,
                    const int32_t *positions_host, int32_t n_steps, int32_t *out_tokens_dev, void *stream) {
    if (!e) return fail(SP_ERR_INVALID, "null engine");
    if (!kvs || !tokens_host || !positions_host || !out_tokens_dev) return fail(SP_ERR_INVALID, "null argument");
    if (B <= 0 || B > kBatchMax) return fail(SP_ERR_CAPACITY, "batch of %d requests (1..%d)", B, kBatchMax);
    if (n_steps <= 0) return fail(SP_ERR_INVALID, "n_steps must be positive");
    if (!e->prefill) return fail(SP_ERR_UNSUPPORTED, "batched decode needs the batched pass (SEEDPLANE_PREFILL=steps)");
    BatchIn in;
    memset(&in, 0, sizeof(in));
    for (int b = 0; b < B; ++b) {
        sp_kv *kv = kvs[b];
        if (!kv || kv->e != e) return fail(SP_ERR_INVALID, "request %d: null cache or a cache of another engine", b);
        for (int j = 0; j < b; ++j)
            if (kvs[j] == kv) return fail(SP_ERR_INVALID, "request %d: cache shared with request %d", b, j);
        if (kv->length + n_steps > kv->capacity)
            return fail(SP_ERR_CAPACITY, "request %d: KV cache capacity %d exceeded", b, kv->capacity);
        if (tokens_host[b] < 0 || tokens_host[b] >= e->c.vocab)
            return fail(SP_ERR_INVALID, "request %d: token %d outside the vocabulary", b, tokens_host[b]);
        if (positions_host[b] < 0 || positions_host[b] + n_steps > e->c.max_positions)
            return fail(SP_ERR_CAPACITY, "request %d: positions outside the RoPE table", b);
        in.lanes[b] = BatchLane{kv->k, kv->v, kv->capacity, kv->length};
        in.tok[b] = tokens_host[b];
        in.pos[b] = positions_host[b];
    }
    SP_CUDA(cudaSetDevice(e->device));
    cudaStream_t s = (cudaStream_t)stream;
    if (!e->bt) SP_CUDA(cudaMalloc(&e->bt, sizeof(BatchIn)));
    SP_CUDA(cudaMemcpyAsync(e->bt, &in, sizeof(in), cudaMemcpyHostToDevice, s));
    cudaGraphExec_t ex = nullptr;
    if (e->use_graph) {
        int rc = batch_graph(e, B, &ex);
        if (rc) return rc;
    }
    for (int i = 0; i < n_steps; ++i) {
        if (ex) {
            SP_CUDA(cudaGraphLaunch(ex, s));
        } else {
            int rc = batch_step(e, B, s);
            if (rc) return rc;
        }
        SP_CUDA(cudaMemcpyAsync(out_tokens_dev + (size_t)i * B, e->bt->out, (size_t)B * sizeof(int32_t),
                                cudaMemcpyDeviceToDevice, s));
    }
    for (int b = 0; b < B; ++b) kvs[b]->length += n_steps;
    return SP_OK;
}

// One packed pass: requests [r0, r1) whose prompts are the tokens [off, off + T) of tokens_dev.
static int prefill_pack(sp_engine *e, sp_kv *const *kvs, const int32_t *lens, int r0, int r1, const int32_t *tokens_dev,
                        int64_t off, int T, int32_t *argmax_dev, cudaStream_t s) {
    const sp_config &c = e->c;
    PrefillBatchIn in;
    int t = 0;
    for (int r = r0; r < r1; ++r) {
        sp_kv *kv = kvs[r];
        for (int i = 0; i < lens[r]; ++i, ++t) {
            in.lanes[t] = BatchLane{kv->k, kv->v, kv->capacity, kv->length + i};
            in.pos[t] = kv->length + i;
        }
        in.last[r - r0] = t - 1;
    }
    // only the filled part of the struct goes over (the lanes, positions and rows in use)
    SP_CUDA(cudaMemcpyAsync(e->bp->lanes, in.lanes, (size_t)T * sizeof(BatchLane), cudaMemcpyHostToDevice, s));
    SP_CUDA(cudaMemcpyAsync(e->bp->pos, in.pos, (size_t)T * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    SP_CUDA(cudaMemcpyAsync(e->bp->last, in.last, (size_t)(r1 - r0) * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    const float scale = 1.0f / sqrtf((float)c.head_dim);
    SP_CUDA(launch_prefill_embed(e->pf_dims, e->pf, e->embed, tokens_dev + off, T, e->st, s));
    for (int l = 0; l < c.layers; ++l) {
        const PrefillLayer &L = e->layers[l].pf;
        SP_CUDA(launch_batch_layer_front(e->pf_dims, L, e->pf, T, e->bp->pos, e->bp->lanes, l, scale, e->rope, e->st, s));
        SP_CUDA(launch_prefill_layer_ffn(e->pf_dims, L, e->pf, T, e->st, s));
    }
    // the prompts' last rows, gathered: the LM head and argmax for them alone
    PrefillScratch g = e->pf;
    g.x = e->pf.q;                         // free after the last layer's attention
    const int n = r1 - r0;
    SP_CUDA(launch_gather_rows(reinterpret_cast<uint8_t *>(g.x), reinterpret_cast<const uint8_t *>(e->pf.x), e->bp->last,
                               n, c.hidden * 4, 1, 0, s));
    for (int b0 = 0; b0 < n; b0 += kPrefillLogitRows) {
        const int rows = std::min(kPrefillLogitRows, n - b0);
        SP_CUDA(launch_prefill_logits(e->pf_dims, g, e->final_norm, e->head_pf, b0, rows, e->pf.logits, e->st, s));
        SP_CUDA(launch_argmax_rows(e->pf.logits, rows, c.vocab, c.vocab, argmax_dev + r0 + b0, e->am, s));
    }
    for (int r = r0; r < r1; ++r) kvs[r]->length += lens[r];
    return SP_OK;
}

int sp_prefill_batch(sp_engine *e, sp_kv *const *kvs, int32_t B, const int32_t *tokens_dev, const int32_t *lens_host,
                     int32_t *argmax_dev, void *stream) {
    if (!e) return fail(SP_ERR_INVALID, "null engine");
    if (!kvs || !tokens_dev || !lens_host || !argmax_dev) return fail(SP_ERR_INVALID, "null argument");
    if (B <= 0 || B > kPrefillBatchMax) return fail(SP_ERR_CAPACITY, "batch of %d prompts (1..%d)", B, kPrefillBatchMax);
    if (!e->prefill) return fail(SP_ERR_UNSUPPORTED, "packed prompts need the batched pass (SEEDPLANE_PREFILL=steps)");
    for (int b = 0; b < B; ++b) {
        sp_kv *kv = kvs[b];
        if (!kv || kv->e != e) return fail(SP_ERR_INVALID, "request %d: null cache or a cache of another engine", b);
        for (int j = 0; j < b; ++j)
            if (kvs[j] == kv) return fail(SP_ERR_INVALID, "request %d: cache shared with request %d", b, j);
        if (lens_host[b] <= 0) return fail(SP_ERR_INVALID, "request %d: empty prompt", b);
        if (kv->length + lens_host[b] > kv->capacity)
            return fail(SP_ERR_CAPACITY, "request %d: KV cache capacity %d exceeded", b, kv->capacity);
        if (kv->length + lens_host[b] > e->c.max_positions)
            return fail(SP_ERR_CAPACITY, "request %d: positions outside the RoPE table", b);
    }
    SP_CUDA(cudaSetDevice(e->device));
    cudaStream_t s = (cudaStream_t)stream;
    if (!e->bp) SP_CUDA(cudaMalloc(&e->bp, sizeof(PrefillBatchIn)));
    // pack whole prompts into passes of at most kPrefillMaxTokens tokens; a longer prompt runs alone
    int64_t off = 0, pack_off = 0;
    int r0 = 0, T = 0;
    for (int b = 0; b <= B; ++b) {
        const int len = b < B ? lens_host[b] : 0;
        if (b == B || T + len > kPrefillMaxTokens) {
            if (T > 0) {
                int rc = prefill_pack(e, kvs, lens_host, r0, b, tokens_dev, pack_off, T, argmax_dev, s);
                if (rc) return rc;
            }
            r0 = b;
            pack_off = off;
            T = 0;
        }
        if (b == B) break;
        if (len > kPrefillMaxTokens) {                  // alone, through the chunked pass
            sp_kv *kv = kvs[b];
            const int32_t base = kv->length;
            SP_CUDA(cudaMemcpyAsync(&e->vt->slot0, &base, sizeof(base), cudaMemcpyHostToDevice, s));
            int rc = forward_batched(e, kv, tokens_dev + off, nullptr, nullptr, &e->vt->slot0, len, nullptr, false,
                                     argmax_dev + b, s, true);
            if (rc) return rc;
            kv->length += len;
            off += len;
            r0 = b + 1;
            pack_off = off;
            continue;
        }
        T += len;
        off += len;
    }
    return SP_OK;
}

int sp_verify_tree(sp_engine *e, sp_kv *kv, const int32_t *tokens_host, const int32_t *parents_host, int32_t n,
                   int32_t base_pos, float *logits_dev, int32_t *argmax_dev, void *stream) {
    int rc = check_engine_kv(e, kv);
    if (rc) return rc;
    if (n <= 0 || !tokens_host || !parents_host) return fail(SP_ERR_INVALID, "empty tree");
    if (n > kSmallNodes) return fail(SP_ERR_CAPACITY, "tree of %d nodes exceeds %d", n, kSmallNodes);
    if (kv->length + n > kv->capacity) return fail(SP_ERR_CAPACITY, "KV cache capacity %d exceeded", kv->capacity);
    DevState d = base_state();
    int depth[kSmallNodes];
    for (int i = 0; i < n; ++i) {
        const int par = parents_host[i];
        if (par >= i || par < -1) return fail(SP_ERR_INVALID, "node %d: parent %d is not an earlier node", i, par);
        if (tokens_host[i] < 0 || tokens_host[i] >= e->c.vocab) return fail(SP_ERR_INVALID, "node %d: bad token", i);
        depth[i] = par < 0 ? 1 : depth[par] + 1;
        d.small_mask[i] = (par < 0 ? 0ull : d.small_mask[par]) | (1ull << i);
        d.small_tok[i] = tokens_host[i];
        d.small_pos[i] = base_pos + depth[i] - 1;
        if (d.small_pos[i] < 0 || d.small_pos[i] >= e->c.max_positions)
            return fail(SP_ERR_CAPACITY, "node %d: position outside the RoPE table", i);
    }
    if (e->prefill) {
        // one batched pass over the tree: node i at scratch slot length + i, its ancestors' bits as
        // the attention mask; the cache length does not move (sp_kv_commit keeps accepted nodes).
        // Inputs go to the device in one copy; without logits the pass replays a captured graph.
        cudaStream_t s = (cudaStream_t)stream;
        VerifyIn in;
        memset(&in, 0, sizeof(in));
        in.slot0 = kv->length;
        memcpy(in.tok, d.small_tok, n * sizeof(int32_t));
        memcpy(in.pos, d.small_pos, n * sizeof(int32_t));
        memcpy(in.mask, d.small_mask, n * sizeof(uint64_t));
        SP_CUDA(cudaMemcpyAsync(e->vt, &in, sizeof(in), cudaMemcpyHostToDevice, s));
        if (logits_dev)
            return forward_batched(e, kv, e->vt->tok, e->vt->pos, e->vt->mask, &e->vt->slot0, n, logits_dev, true,
                                   argmax_dev, s);
        cudaGraphExec_t ex;
        rc = verify_graph(e, kv, n, &ex);
        if (rc) return rc;
        SP_CUDA(cudaGraphLaunch(ex, s));
        SP_CUDA(cudaMemcpyAsync(argmax_dev, e->vt_argmax, n * sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
        return SP_OK;
    }
    d.use_small = 1;
    d.n_forced = n;
    d.slot0 = kv->length;
    d.tree_base = kv->length;
    d.token = d.small_tok[0];
    d.pos = d.small_pos[0];
    d.slot = kv->length;
    d.logits = logits_dev;
    d.logits_stride = e->c.vocab;
    d.out_tokens = argmax_dev;
    return run_steps(e, kv, d, n, (cudaStream_t)stream);
}

int sp_kv_commit(sp_kv *kv, const int32_t *src_slots_host, int32_t n, void *stream) {
    if (!kv || !kv->e) return fail(SP_ERR_INVALID, "null or orphaned cache");
    if (n < 0 || n > kSmallNodes) return fail(SP_ERR_CAPACITY, "commit of %d slots", n);
    if (n == 0) return SP_OK;
    if (!src_slots_host) return fail(SP_ERR_INVALID, "null slot list");
    if (kv->length + n > kv->capacity) return fail(SP_ERR_CAPACITY, "KV cache capacity %d exceeded", kv->capacity);
    for (int i = 0; i < n; ++i) {
        if (src_slots_host[i] < kv->length + i || src_slots_host[i] >= kv->capacity)
            return fail(SP_ERR_INVALID, "commit slot %d = %d outside [len+i, capacity)", i, src_slots_host[i]);
        if (i && src_slots_host[i] <= src_slots_host[i - 1])
            return fail(SP_ERR_INVALID, "commit slots must be increasing");
    }
    sp_engine *e = kv->e;
    SP_CUDA(cudaSetDevice(e->device));
    SP_CUDA(launch_kv_commit(kv->k, kv->v, e->c.layers, e->c.kv_heads, kv->capacity, e->c.head_dim, src_slots_host, n,
                             kv->length, (cudaStream_t)stream));
    kv->length += n;
    return SP_OK;
}

int sp_kv_copy(sp_kv *src, int32_t src_slot0, sp_kv *dst, int32_t dst_slot0, int32_t n, void *stream) {
    if (!src || !dst || !src->e || !dst->e) return fail(SP_ERR_INVALID, "null or orphaned cache");
    if (src->e != dst->e) return fail(SP_ERR_INVALID, "caches of different engines");
    if (n < 0 || src_slot0 < 0 || dst_slot0 < 0) return fail(SP_ERR_INVALID, "negative slot or count");
    if (n == 0) return SP_OK;
    if ((int64_t)src_slot0 + n > src->capacity || (int64_t)dst_slot0 + n > dst->capacity)
        return fail(SP_ERR_CAPACITY, "slots [%d, %d) -> [%d, %d) outside the capacities %d / %d", src_slot0, src_slot0 + n,
                    dst_slot0, dst_slot0 + n, src->capacity, dst->capacity);
    if (src == dst && src_slot0 < dst_slot0 + n && dst_slot0 < src_slot0 + n)
        return fail(SP_ERR_INVALID, "overlapping slot ranges in one cache");
    sp_engine *e = src->e;
    SP_CUDA(cudaSetDevice(e->device));
    // layout [layer][kv head][capacity][head_dim]: one row of n slots per (layer, kv head)
    const size_t row = (size_t)e->c.head_dim * sizeof(__half);
    const size_t rows = (size_t)e->c.layers * e->c.kv_heads;
    for (int which = 0; which < 2; ++which) {
        const __half *s = (which ? src->v : src->k) + (size_t)src_slot0 * e->c.head_dim;
        __half *d = (which ? dst->v : dst->k) + (size_t)dst_slot0 * e->c.head_dim;
        SP_CUDA(cudaMemcpy2DAsync(d, row * dst->capacity, s, row * src->capacity, row * n, rows, cudaMemcpyDeviceToDevice,
                                  (cudaStream_t)stream));
    }
    return SP_OK;
}

int sp_argmax(sp_engine *e, const float *logits_dev, int32_t rows, int32_t cols, int64_t ld, int32_t *argmax_dev,
              void *stream) {
    if (!e) return fail(SP_ERR_INVALID, "null engine");
    if (!logits_dev || !argmax_dev) return fail(SP_ERR_INVALID, "null logits or output");
    if (rows <= 0 || cols <= 0 || ld < cols) return fail(SP_ERR_INVALID, "bad shape rows=%d cols=%d ld=%lld", rows, cols,
                                                         (long long)ld);
    SP_CUDA(cudaSetDevice(e->device));
    // rows in chunks: the chunks share the engine's scratch in stream order
    for (int32_t r0 = 0; r0 < rows; r0 += kArgmaxChunkRows) {
        const int n = std::min<int32_t>(kArgmaxChunkRows, rows - r0);
        SP_CUDA(launch_argmax_rows(logits_dev + (size_t)r0 * ld, n, cols, ld, argmax_dev + r0, e->am,
                                   (cudaStream_t)stream));
    }
    return SP_OK;
}

int sp_mcol_gemm(sp_engine *e, int32_t mode, const void *w_dev, const void *w_lo_dev, float alpha, int32_t n, int32_t k,
                 const void *x_dev, int32_t x_rows, int32_t lo_row0, int32_t t, float *y_dev, int32_t ldy,
                 void *act_hi_dev, void *act_lo_dev, int32_t ld_act, void *stream) {
    if (!e) return fail(SP_ERR_INVALID, "null engine");
    if (!e->prefill) return fail(SP_ERR_UNSUPPORTED, "the engine was created without the batched pass");
    if (!w_dev || !x_dev || n <= 0 || k <= 0 || t <= 0 || t > x_rows || lo_row0 < t || lo_row0 + t > x_rows)
        return fail(SP_ERR_INVALID, "bad GEMM shape n=%d k=%d t=%d x_rows=%d lo_row0=%d", n, k, t, x_rows, lo_row0);
    if (t > kPrefillMaxTokens) return fail(SP_ERR_CAPACITY, "%d tokens exceed %d", t, kPrefillMaxTokens);
    if (mode < MC_STORE || mode > MC_SWIGLU) return fail(SP_ERR_INVALID, "mode %d", mode);
    if (mode == MC_SWIGLU ? (!act_hi_dev || !act_lo_dev || n % 2 || ld_act < n / 2) : (!y_dev || ldy < n))
        return fail(SP_ERR_INVALID, "bad GEMM output");
    SP_CUDA(cudaSetDevice(e->device));
    McolOp op{};
    op.mode = mode;
    op.w = (const __half *)w_dev;
    op.w_lo = (const __half *)w_lo_dev;
    op.alpha = alpha;
    op.N = n;
    op.K = k;
    op.x = (const __half *)x_dev;
    op.x_rows = x_rows;
    op.lo_row0 = lo_row0;
    op.T = t;
    op.y = y_dev;
    op.ldy = ldy;
    op.act_h = (__half *)act_hi_dev;
    op.act_l = (__half *)act_lo_dev;
    op.ld_act = ld_act;
    op.max_ctas = kPrefillMaxCtas;
    op.st = e->st;
    op.trace = e->mc_trace;
    SP_CUDA(launch_mcol(op, (cudaStream_t)stream, false));
    return SP_OK;
}

int sp_topk(sp_engine *e, const float *logits_dev, int32_t rows, int32_t cols, int64_t ld, int32_t k,
            int32_t *idx_dev, float *val_dev, float *lse_dev, void *stream) {
    if (!e || !logits_dev || !idx_dev || !val_dev || !lse_dev) return fail(SP_ERR_INVALID, "null argument");
    if (rows <= 0 || cols <= 0 || ld < cols) return fail(SP_ERR_INVALID, "bad logits shape");
    if (k < 1 || k > kTopkMax || k > cols) return fail(SP_ERR_INVALID, "k must be in 1..%d and <= cols", kTopkMax);
    SP_CUDA(cudaSetDevice(e->device));
    SP_CUDA(launch_topk_rows(logits_dev, rows, cols, ld, k, idx_dev, val_dev, lse_dev, (cudaStream_t)stream));
    return SP_OK;
}

int sp_sample_filter(const float *logits_dev, int32_t vocab, double temperature, int32_t top_k, double top_p,
                     float *z_dev, void *stream) {
    if (!logits_dev || !z_dev) return fail(SP_ERR_INVALID, "null argument");
    if (vocab <= 0 || vocab > kSampleFilterMaxVocab)
        return fail(SP_ERR_INVALID, "vocab %d outside [1, %d]", vocab, kSampleFilterMaxVocab);
    if (!(temperature > 0.0)) return fail(SP_ERR_INVALID, "temperature must be positive");
    if (top_k < 0 || !(top_p >= 0.0 && top_p <= 1.0)) return fail(SP_ERR_INVALID, "top_k < 0 or top_p outside [0, 1]");
    SP_CUDA(launch_sample_filter(logits_dev, vocab, temperature, top_k, top_p, z_dev, (cudaStream_t)stream));
    return SP_OK;
}

int sp_accept_stochastic(sp_engine *e, const float *target_logits_dev, const float *draft_logits_dev, int64_t ld,
                         int32_t vocab, const int32_t *tokens_host, const int32_t *parents_host, int32_t n,
                         double temperature, uint64_t seed, uint64_t counter, int32_t *out_host, void *stream) {
    if (!e || !target_logits_dev || !draft_logits_dev || !out_host || (n > 0 && (!tokens_host || !parents_host)))
        return fail(SP_ERR_INVALID, "null argument");
    if (n < 0 || n > kSmallNodes) return fail(SP_ERR_CAPACITY, "tree of %d nodes exceeds %d", n, kSmallNodes);
    if (vocab <= 0 || ld < vocab) return fail(SP_ERR_INVALID, "bad logits shape");
    if (!(temperature > 0.0)) return fail(SP_ERR_INVALID, "temperature must be positive");
    for (int i = 0; i < n; ++i) {
        if (parents_host[i] >= i || parents_host[i] < -1) return fail(SP_ERR_INVALID, "node %d: bad parent", i);
        if (tokens_host[i] < 0 || tokens_host[i] >= vocab) return fail(SP_ERR_INVALID, "node %d: bad token", i);
    }
    SP_CUDA(cudaSetDevice(e->device));
    cudaStream_t s = (cudaStream_t)stream;
    if (!e->acc_scratch) SP_CUDA(cudaMalloc(&e->acc_scratch, (size_t)(6 * kSmallNodes + 16) * 4));
    // the rows the walk can visit: the root's (0) and row i + 1 of every node i with children
    int32_t host[4 * kSmallNodes + 2] = {};
    int32_t *h_tok = host, *h_par = host + kSmallNodes, *h_rows = h_par + kSmallNodes, *h_slot = h_rows + kSmallNodes + 1;
    for (int r = 0; r <= n; ++r) h_slot[r] = -1;
    int nr = 0;
    h_slot[0] = nr;
    h_rows[nr++] = 0;
    for (int i = 0; i < n; ++i) {
        h_tok[i] = tokens_host[i];
        h_par[i] = parents_host[i];
        const int row = parents_host[i] + 1;
        if (h_slot[row] < 0) {
            h_slot[row] = nr;
            h_rows[nr++] = row;
        }
    }
    const size_t rows_bytes = ((size_t)4 * nr + (size_t)2 * nr * vocab) * 8;
    if (e->acc_rows_bytes < rows_bytes) {
        cudaFree(e->acc_rows);
        e->acc_rows = nullptr;
        e->acc_rows_bytes = 0;
        SP_CUDA(cudaMalloc(&e->acc_rows, rows_bytes));
        e->acc_rows_bytes = rows_bytes;
    }
    int32_t *dtok = e->acc_scratch;
    int32_t *dpar = dtok + kSmallNodes, *drows = dpar + kSmallNodes, *dslot = drows + kSmallNodes + 1;
    int32_t *dout = dslot + kSmallNodes + 1;
    SP_CUDA(cudaMemcpyAsync(dtok, host, sizeof(host), cudaMemcpyHostToDevice, s));
    double *ms = e->acc_rows, *ev = e->acc_rows + 4 * nr;
    SP_CUDA(launch_accept_stochastic(target_logits_dev, draft_logits_dev, ld, vocab, dtok, dpar, n, drows, dslot, nr,
                                     temperature, seed, counter, ms, ev, dout, s));
    SP_CUDA(cudaMemcpyAsync(out_host, dout, (size_t)(2 * n + 3) * 4, cudaMemcpyDeviceToHost, s));
    SP_CUDA(cudaStreamSynchronize(s));
    return SP_OK;
}

int sp_accept_greedy(sp_engine *e, const int32_t *node_pred_dev, int32_t root_pred, const int32_t *tokens_host,
                     const int32_t *parents_host, int32_t n, const int32_t *path_ends_host, int32_t n_paths,
                     int32_t *out_host, void *stream) {
    if (!e || !out_host || (n > 0 && (!node_pred_dev || !tokens_host || !parents_host)) ||
        (n_paths > 0 && !path_ends_host))
        return fail(SP_ERR_INVALID, "null argument");
    if (n < 0 || n > kSmallNodes) return fail(SP_ERR_CAPACITY, "tree of %d nodes exceeds %d", n, kSmallNodes);
    if (n_paths < 0 || n_paths > kGreedyMaxPaths)
        return fail(SP_ERR_CAPACITY, "%d paths exceed %d", n_paths, kGreedyMaxPaths);
    if (n_paths > 0 && n == 0) return fail(SP_ERR_INVALID, "paths without nodes");
    for (int i = 0; i < n; ++i)
        if (parents_host[i] >= i || parents_host[i] < -1) return fail(SP_ERR_INVALID, "node %d: bad parent", i);
    for (int j = 0; j < n_paths; ++j)
        if (path_ends_host[j] < 0 || path_ends_host[j] >= n) return fail(SP_ERR_INVALID, "path %d: bad end node", j);
    SP_CUDA(cudaSetDevice(e->device));
    cudaStream_t s = (cudaStream_t)stream;
    constexpr int kIn = 2 * kSmallNodes + kGreedyMaxPaths, kOut = 2 * kSmallNodes + 5;
    if (!e->gr_buf) SP_CUDA(cudaMalloc(&e->gr_buf, (size_t)(kIn + kOut) * sizeof(int32_t)));
    std::vector<int32_t> host(2 * kSmallNodes + n_paths, 0);
    if (n > 0) {
        memcpy(host.data(), tokens_host, n * 4);
        memcpy(host.data() + kSmallNodes, parents_host, n * 4);
    }
    if (n_paths > 0) memcpy(host.data() + 2 * kSmallNodes, path_ends_host, n_paths * 4);
    int32_t *dtok = e->gr_buf, *dpar = dtok + kSmallNodes, *dend = dpar + kSmallNodes, *dout = e->gr_buf + kIn;
    SP_CUDA(cudaMemcpyAsync(dtok, host.data(), host.size() * 4, cudaMemcpyHostToDevice, s));
    SP_CUDA(launch_accept_greedy(node_pred_dev, root_pred, dtok, dpar, n, dend, n_paths, dout, s));
    SP_CUDA(cudaMemcpyAsync(out_host, dout, (size_t)(2 * n + 5) * 4, cudaMemcpyDeviceToHost, s));
    SP_CUDA(cudaStreamSynchronize(s));
    return SP_OK;
}

int sp_argmax_noalloc(int device, const float *logits_dev, int32_t rows, int32_t cols, int64_t ld, int32_t *argmax_dev,
                      void *stream) {
    if (!logits_dev || !argmax_dev) return fail(SP_ERR_INVALID, "null logits or output");
    if (rows <= 0 || cols <= 0 || ld < cols) return fail(SP_ERR_INVALID, "bad shape rows=%d cols=%d ld=%lld", rows, cols,
                                                         (long long)ld);
    if (rows > argmax_noalloc_max_rows())
        return fail(SP_ERR_CAPACITY, "%d rows exceed the fixed scratch (at most %d rows)", rows, argmax_noalloc_max_rows());
    if (device < 0 || device >= kMaxDevices) return fail(SP_ERR_INVALID, "device %d", device);
    // the caller's current device is put back on every return
    struct DeviceRestore {
        int prev = -1;
        ~DeviceRestore() { if (prev >= 0) cudaSetDevice(prev); }
    } restore;
    SP_CUDA(cudaGetDevice(&restore.prev));
    SP_CUDA(cudaSetDevice(device));
    for (const void *ptr : {(const void *)logits_dev, (const void *)argmax_dev}) {
        cudaPointerAttributes at{};
        SP_CUDA(cudaPointerGetAttributes(&at, ptr));
        if (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged)
            return fail(SP_ERR_INVALID, "logits and output must be device memory");
        if (at.device != device)
            return fail(SP_ERR_INVALID, "a buffer lives on device %d, not on device %d", at.device, device);
    }
    // Per-device address of the module's scratch array, looked up once (before any stream capture);
    // it stays valid for the life of the device's primary context.
    static std::mutex mu;
    static void *base[kMaxDevices] = {};
    void *b = nullptr;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!base[device]) {
            void *p = nullptr;
            SP_CUDA(argmax_noalloc_scratch(&p));
            if (!p) return fail(SP_ERR_CUDA, "no address for the argmax scratch on device %d", device);
            base[device] = p;
        }
        b = base[device];
    }
    if (argmax_scratch_bytes(rows) > argmax_noalloc_scratch_bytes())
        return fail(SP_ERR_CAPACITY, "argmax scratch of %zu bytes is too small", argmax_noalloc_scratch_bytes());
    const ArgmaxScratch sc = argmax_scratch_at(b, rows);
    SP_CUDA(cudaMemsetAsync(sc.cnt, 0, (size_t)rows * sizeof(unsigned), (cudaStream_t)stream));   // counters start at 0
    SP_CUDA(launch_argmax_rows(logits_dev, rows, cols, ld, argmax_dev, sc, (cudaStream_t)stream));
    return SP_OK;
}

int64_t sp_trace_read(sp_engine *e, uint64_t *host_out, int64_t capacity) {
    if (!e) return fail(SP_ERR_INVALID, "null engine");
    if (!e->trace && !e->step_trace && !e->mc_trace) return 0;
    const int64_t n = e->step_trace ? (int64_t)(5 * e->c.layers + 1) * e->num_sms * kStepTraceWords
                      : e->trace ? (int64_t)(e->trace_kernels + 2) * e->num_sms * kTraceWords
                                 : (int64_t)kPrefillMaxCtas * kMcolTraceWords;
    if (!host_out) return n;
    if (capacity < n) return fail(SP_ERR_CAPACITY, "trace needs %lld words", (long long)n);
    cudaError_t ce = cudaSetDevice(e->device);
    if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
    const void *src = e->step_trace ? (const void *)e->step_trace : e->trace ? (const void *)e->trace : (const void *)e->mc_trace;
    if (ce == cudaSuccess) ce = cudaMemcpy(host_out, src, (size_t)n * 8, cudaMemcpyDeviceToHost);
    if (ce != cudaSuccess) return fail(SP_ERR_CUDA, "trace copy: %s", cudaGetErrorString(ce));
    return n;
}

int sp_device_status(sp_engine *e, void *stream) {
    if (!e) return fail(SP_ERR_INVALID, "null engine");
    SP_CUDA(cudaSetDevice(e->device));
    int err = 0;
    cudaStream_t s = (cudaStream_t)stream;
    SP_CUDA(cudaMemcpyAsync(&err, &e->st->err, 4, cudaMemcpyDeviceToHost, s));
    SP_CUDA(cudaStreamSynchronize(s));
    if (err) {
        // a step that gave up left counters and split-strip state undefined: start them afresh
        SP_CUDA(cudaMemsetAsync(e->ws, 0, e->ws_clear_bytes, s));
        SP_CUDA(cudaMemsetAsync(&e->st->err, 0, 4, s));
        SP_CUDA(cudaStreamSynchronize(s));
        const char *what = err == kErrMbarTimeout ? "a weight stage never arrived (bounded wait expired)"
                         : err == kErrBadToken    ? "token id outside the vocabulary"
                         : err == kErrBadSlot     ? "position or slot outside its table"
                                                  : "unknown";
        return fail(SP_ERR_DEVICE, "device error %d: %s", err, what);
    }
    return SP_OK;
}

}  // extern "C"
