// Persistent decode step for sm_100a: one launch per token, one CTA per SM.
//
// The kernel walks the step's op table (per layer: QKV GEMV, attention, O GEMV, gate_up GEMV,
// down GEMV; then the LM head). Weights are packed as tiles of 256 output rows x 64 inputs (32 KB,
// 128B-swizzled K-major rows); every CTA owns the tile range [T*c/C, T*(c+1)/C) of every GEMV.
// The weight tile is the B operand of tcgen05.mma (N = 256, K = 16, four per tile) and the
// activation is the A operand (M = 128): one 1 KB swizzle atom per 64 inputs holds row 0 = fp16(x)
// and row 1 = fp16(x - fp16(x)), and the descriptor's 8-row-group stride is 0, so every group of
// the 128 rows re-reads that atom. D rows 0 and 1 (and their copies in every warp's TMEM quarter)
// then hold W.hi and W.lo; y = their sum carries ~22 bits of the fp32 activation. Carrying 8 KB
// of weights per MMA instruction is what lets the tensor core keep up with HBM (measured: 4 KB
// per instruction as the A operand streams at about half the rate). Roles:
//
//   warp 4 (producer)  streams ALL of the CTA's tiles of the step, op after op, through one ring
//                      of 32 KB stages with 1-D bulk copies. It never waits for data, only for a
//                      free stage, so weight traffic continues while the other warps wait for
//                      activations (the ring then fills with the next ops' tiles).
//   warp 5 (MMA)       per GEMV op: waits until the activation atoms of that op are built, then
//                      issues four MMAs per tile into one of two 256-column TMEM accumulators
//                      (double-buffered with the epilogue: one accumulator per strip item).
//   warps 0-3          per GEMV op: wait on the op's dependency counter, build the activation
//                      atoms (RMSNorm fused), hand them to the MMA warp, then read the
//                      accumulators (warp w: columns 64w..64w+63) and run the epilogue on row pairs
//                      (bias + RoPE + K/V write / residual add / SwiGLU / logits + argmax). A strip
//                      split between CTAs is summed by its last contributor in fixed order.
//                      Finished strips are counted into the op's counter (fence, then atomic add).
//                      Attention: the epilogue warps of the first nkv * chunks CTAs each compute
//                      one (kv head, context chunk) item and publish an unnormalised partial
//                      (max, sum, acc); the O projection's prologue merges, per input it needs,
//                      the partials of that head (log-sum-exp, fixed chunk order).
//
// Counters are 64-bit and never reset: an op's consumers wait for units * (epoch + 1). All data
// another CTA produced is read through L2 (ld.global.cg / cp.async.cg), never from L1. Every
// wait is bounded; on expiry the CTA records an error in DevState::err, sets its abort flag and
// runs to the end without waiting again, so the kernel always terminates.
#include <algorithm>
#include <climits>
#include <cmath>

#include "kernels.cuh"
#include "tc.cuh"

namespace sp {

namespace {

constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;            // warps 0-3: TMEM lanes 0-127
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kTileRows = 256;              // output rows per weight tile (MMA N)
constexpr int kTileK = 64;                  // inputs per weight tile (one 128-byte swizzled row)
constexpr int kStepTileBytes = kTileRows * kTileK * 2;    // 32 KB per weight tile
constexpr int kStageTiles = 2;              // tiles per ring stage: one 64 KB bulk copy (a bulk copy costs
                                            // about the same time whatever its size, so big ones ingest faster)
constexpr int kStageBytes = kStageTiles * kStepTileBytes;
constexpr int kABlockBytes = 1024;          // activation atom (8 rows x 64 inputs) per k-block
constexpr int kMaxItems = 16;               // strips a CTA may touch in one op
constexpr int kTmemCols = 512;              // two accumulators of 256 fp32 columns
constexpr int kMaxUnits = 4;                // activation chunks (8 inputs) per epilogue thread
constexpr int kGroup = 8;                   // q heads per kv head, padded (zero q beyond G)
constexpr uint32_t kDepSpinLimit = 1u << 22;

SP_DEVINL void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

SP_DEVINL void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory"); }
SP_DEVINL void bready_sync() { asm volatile("bar.sync 2, %0;" ::"n"(kEpiThreads + 32) : "memory"); }

SP_DEVINL unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Cross-CTA hand-off. The writers of a CTA meet at a barrier, then one thread publishes with
// release semantics (cumulative over the writes the barrier ordered before it); a consumer thread
// acquires, then its CTA's barrier orders the other threads' reads after the acquire.
SP_DEVINL unsigned atom_add_acq_rel(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
SP_DEVINL void red_add_release(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

SP_DEVINL void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
SP_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
SP_DEVINL void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

SP_DEVINL float4 ldcg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }

// Abort state of the CTA: set on the first expired wait, after which no thread waits again.
struct Abort {
    volatile int *flag;
    DevState *st;
    SP_DEVINL bool on() const { return *flag != 0; }
    SP_DEVINL void raise(int code) const {
        *flag = 1;
        atomicCAS(&st->err, 0, code);
    }
};

SP_DEVINL bool wait_bar(uint64_t *bar, uint32_t parity, const Abort &ab) {
    for (uint32_t i = 0; i < kMbarSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && ab.on()) return false;
    }
    ab.raise(kErrMbarTimeout);
    return false;
}

// One thread waits until *cnt >= target (acquire). Gives up on abort or after the spin limit;
// also gives up when another CTA has already recorded an error, so a failure ends every CTA.
SP_DEVINL bool wait_counter(const unsigned long long *cnt, unsigned long long target, const Abort &ab) {
    for (uint32_t i = 0; i < kDepSpinLimit; ++i) {
        if (ld_acquire_u64(cnt) >= target) return true;
        if ((i & 63u) == 63u) {
            if (ab.on() || *reinterpret_cast<volatile int *>(&ab.st->err) != 0) {
                *ab.flag = 1;
                return false;
            }
            if (i >= 1024u) __nanosleep(64);      // back off only after the first ~1k polls
        }
    }
    ab.raise(kErrDepTimeout);
    return false;
}

// Attention staging region: K and V rows of one sub-chunk (fp16), q of the group (fp32, padded
// to kGroup heads), scores [rows][kGroup].
template <int HD>
struct AttnRegion {
    static constexpr int kRow = HD * 2;
    static constexpr size_t kOff = 0;
    static constexpr size_t vOff = kOff + (size_t)kStepAttnRows * kRow;
    static constexpr size_t qOff = vOff + (size_t)kStepAttnRows * kRow;
    static constexpr size_t sOff = qOff + (size_t)kGroup * HD * 4;
    static constexpr size_t bytes = sOff + (size_t)kStepAttnRows * kGroup * 4;
};

// cp.async K/V rows [lo, hi) of one kv head into the sub-chunk buffers (row j -> local j - base).
template <int HD>
SP_DEVINL void stage_rows(uint8_t *am, const __half *kb, const __half *vb, int base, int lo, int hi, int tid) {
    using L = AttnRegion<HD>;
    constexpr int kChunks = HD / 8;
    const int n = hi - lo;
    for (int i = tid; i < n * kChunks * 2; i += kEpiThreads) {
        const int which = i / (n * kChunks);
        const int r = (i - which * n * kChunks) / kChunks, ch = i % kChunks;
        const int j = lo + r;
        if (which == 0)
            cp_async16(am + L::kOff + (size_t)(j - base) * L::kRow + ch * 16, kb + (size_t)j * HD + ch * 8);
        else
            cp_async16(am + L::vOff + (size_t)(j - base) * L::kRow + ch * 16, vb + (size_t)j * HD + ch * 8);
    }
}

template <int DL>
SP_DEVINL void load_dims(const uint8_t *q, float (&f)[DL]) {
    if constexpr (DL == 4) {
        const uint2 u = *reinterpret_cast<const uint2 *>(q);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
        f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    } else {
        const uint32_t u = *reinterpret_cast<const uint32_t *>(q);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u));
        f[0] = a.x; f[1] = a.y;
    }
}

// Sum v[h] over the 32 lanes for 8 heads; lane l returns head l / 4 (exchange steps xor 16, 8, 4
// halve the values per lane, then xor 2, 1 finish the sums; fixed order).
SP_DEVINL float reduce_heads(const float (&v)[kGroup], int lane) {
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
    float w[4], x[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float send = b4 ? v[i] : v[i + 4], keep = b4 ? v[i + 4] : v[i];
        w[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float send = b3 ? w[i] : w[i + 2], keep = b3 ? w[i + 2] : w[i];
        x[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    const float send = b2 ? x[0] : x[1], keep = b2 ? x[1] : x[0];
    float y = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    y += __shfl_xor_sync(0xffffffffu, y, 2);
    y += __shfl_xor_sync(0xffffffffu, y, 1);
    return y;
}

// Attention chunking of the visible context [0, ctx): the same in the attention op and in the
// O projection's merge.
SP_DEVINL int attn_chunks(int ctx, int max_chunks) {
    return max(1, min(max_chunks, (ctx + kStepAttnRows - 1) / kStepAttnRows));
}

SP_DEVINL void stamp(unsigned long long *tr, int k, int C, int c, int i) {
    if (tr && threadIdx.x == 0) tr[((size_t)k * C + c) * kStepTraceWords + i] = globaltimer();
}



SP_DEVINL void prefetch_line_l2(const void *p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// While op k waits for its inputs, the epilogue warps warm L2 with this CTA's weight tiles that the
// ring cannot hold yet: op k's tiles beyond the ring's depth, then the next GEMV op's, at most
// `budget` tiles. Plain line prefetches (load/store path), so the copy engine keeps serving the ring;
// the ring's later bulk copies of these tiles then hit L2.
SP_DEVINL void warm_l2_for(const StepParams &p, const StepOp *ops, int k, int c, int tid, int skip, int budget) {
    for (int kk = k; kk < p.n_ops && budget > 0; ++kk) {
        const StepOp &op = ops[kk];
        if (op.kind != OP_GEMV) continue;
        if (c < op.grid) {
            const long long T = (long long)(op.N / kTileRows) * (op.K / kTileK);
            long long g0 = T * c / op.grid;
            const long long g1 = T * (c + 1) / op.grid;
            if (kk == k) g0 += skip;
            for (long long g = g0; g < g1 && budget > 0; ++g, --budget) {
                const uint8_t *t = op.w + (size_t)g * kStepTileBytes;
                for (int line = tid; line < kStepTileBytes / 128; line += kEpiThreads) prefetch_line_l2(t + (size_t)line * 128);
            }
        }
        if (kk != k) break;              // this op and the next GEMV op only
    }
}

// Per-step values every epilogue thread reads once (after the dependency on the previous step).
struct StepState {
    unsigned long long epoch;
    int token, pos, slot, tree_base;
    unsigned long long mask;
};

// ---- attention item of one CTA: (kv head g, chunk ch) ------------------------------------------
template <int HD>
__device__ void attention_item(const StepParams &p, const StepOp &op, const StepState &ss, uint8_t *am, int item,
                               int n_chunks, int rows_per, int ctx, const Abort &ab) {
    using L = AttnRegion<HD>;
    constexpr int DL = HD / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = p.nh / p.nkv;
    const int g = item / n_chunks, ch = item - g * n_chunks;
    const int j0 = ch * rows_per, j1 = min(ctx, j0 + rows_per);
    const __half *kb = op.kc + (size_t)g * p.cap * HD;
    const __half *vb = op.vc + (size_t)g * p.cap * HD;
    float *qs = reinterpret_cast<float *>(am + L::qOff);
    float *sc = reinterpret_cast<float *>(am + L::sOff);
    const int slot = ss.slot;

    for (int i = G * HD + tid; i < kGroup * HD; i += kEpiThreads) qs[i] = 0.f;
    // rows other than the current one do not depend on this step: stage them before the wait
    const int s1 = min(j1, j0 + kStepAttnRows);
    stage_rows<HD>(am, kb, vb, j0, j0, min(s1, slot), tid);
    cp_async_commit();
    if (tid == 0 && op.dep >= 0) wait_counter(p.cnt + op.dep, (unsigned long long)op.dep_n * (ss.epoch + 1), ab);
    epi_sync();
    if (slot >= j0 && slot < s1) stage_rows<HD>(am, kb, vb, j0, slot, slot + 1, tid);
    for (int i = tid; i < G * HD / 4; i += kEpiThreads) cp_async16(qs + 4 * i, p.q + (size_t)g * G * HD + 4 * i);
    cp_async_commit();
    cp_async_wait_all();
    epi_sync();

    float qr[kGroup][DL];
#pragma unroll
    for (int h = 0; h < kGroup; ++h)
#pragma unroll
        for (int i = 0; i < DL; ++i) qr[h][i] = qs[h * HD + DL * lane + i];
    // this warp's heads: warp and warp + 4 (of the group)
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    float acc[2][DL];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int i = 0; i < DL; ++i) acc[u][i] = 0.f;

    for (int a = j0; a < j1; a += kStepAttnRows) {
        const int b = min(j1, a + kStepAttnRows), nj = b - a;
        if (a != j0) {
            epi_sync();                       // everyone is done with the previous sub-chunk
            stage_rows<HD>(am, kb, vb, a, a, b, tid);
            cp_async_commit();
            cp_async_wait_all();
            epi_sync();
        }
        // scores: warp = position (two in flight), lane = HD/32 dims, all 8 heads
        for (int jl = warp; jl < nj; jl += 8) {
            const int jl2 = jl + 4;
            const bool has2 = jl2 < nj;
            float k1[DL], k2[DL];
            load_dims<DL>(am + L::kOff + (size_t)jl * L::kRow + lane * DL * 2, k1);
            if (has2) {
                load_dims<DL>(am + L::kOff + (size_t)jl2 * L::kRow + lane * DL * 2, k2);
            } else {
#pragma unroll
                for (int i = 0; i < DL; ++i) k2[i] = 0.f;
            }
            float v1[kGroup], v2[kGroup];
#pragma unroll
            for (int h = 0; h < kGroup; ++h) {
                float t1 = qr[h][0] * k1[0], t2 = qr[h][0] * k2[0];
#pragma unroll
                for (int i = 1; i < DL; ++i) {
                    t1 = fmaf(qr[h][i], k1[i], t1);
                    t2 = fmaf(qr[h][i], k2[i], t2);
                }
                v1[h] = t1;
                v2[h] = t2;
            }
            const float r1 = reduce_heads(v1, lane), r2 = reduce_heads(v2, lane);
            if ((lane & 3) == 0) {
                const int h = lane >> 2, j = a + jl, j2 = a + jl2;
                const bool vis1 = !(j >= ss.tree_base && !((ss.mask >> (j - ss.tree_base)) & 1ull));
                sc[jl * kGroup + h] = vis1 ? r1 * p.scale : -INFINITY;
                if (has2) {
                    const bool vis2 = !(j2 >= ss.tree_base && !((ss.mask >> (j2 - ss.tree_base)) & 1ull));
                    sc[jl2 * kGroup + h] = vis2 ? r2 * p.scale : -INFINITY;
                }
            }
        }
        epi_sync();
        // softmax (online) and values: this warp's heads only, so the warp needs no CTA barrier
        float corr[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int hh = warp + 4 * u;
            corr[u] = 1.f;
            if (hh >= G) continue;
            const float sv = lane < nj ? sc[lane * kGroup + hh] : -INFINITY;
            const float mx = warp_max(sv);
            const float mnew = fmaxf(m_run[u], mx);
            const float pe = mnew == -INFINITY ? 0.f : expf(sv - mnew);
            const float ls = warp_sum(lane < nj ? pe : 0.f);
            corr[u] = m_run[u] == -INFINITY ? 0.f : expf(m_run[u] - mnew);
            l_run[u] = l_run[u] * corr[u] + ls;
            m_run[u] = mnew;
            if (lane < nj) sc[lane * kGroup + hh] = pe;
        }
        __syncwarp();
        float part[2][2][DL];
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int v = 0; v < 2; ++v)
#pragma unroll
                for (int i = 0; i < DL; ++i) part[u][v][i] = 0.f;
        const uint8_t *vrow = am + L::vOff + lane * DL * 2;
        const bool two = warp + 4 < G;
        if (warp < G) {
            int q = 0;
            for (; q + 2 <= nj; q += 2) {
#pragma unroll
                for (int v = 0; v < 2; ++v) {
                    float vf[DL];
                    load_dims<DL>(vrow + (size_t)(q + v) * L::kRow, vf);
                    const float pa = sc[(q + v) * kGroup + warp];
                    const float pb = two ? sc[(q + v) * kGroup + warp + 4] : 0.f;
#pragma unroll
                    for (int i = 0; i < DL; ++i) {
                        part[0][v][i] = fmaf(pa, vf[i], part[0][v][i]);
                        part[1][v][i] = fmaf(pb, vf[i], part[1][v][i]);
                    }
                }
            }
            if (q < nj) {
                float vf[DL];
                load_dims<DL>(vrow + (size_t)q * L::kRow, vf);
                const float pa = sc[q * kGroup + warp];
                const float pb = two ? sc[q * kGroup + warp + 4] : 0.f;
#pragma unroll
                for (int i = 0; i < DL; ++i) {
                    part[0][0][i] = fmaf(pa, vf[i], part[0][0][i]);
                    part[1][0][i] = fmaf(pb, vf[i], part[1][0][i]);
                }
            }
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
                for (int i = 0; i < DL; ++i) acc[u][i] = fmaf(acc[u][i], corr[u], part[u][0][i] + part[u][1][i]);
        }
    }
    // publish this chunk's partial for each of this warp's heads
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int hh = warp + 4 * u;
        if (hh >= G) continue;
        const int h = g * G + hh;
        float *dst = p.attn_acc + ((size_t)h * p.max_chunks + ch) * HD + DL * lane;
#pragma unroll
        for (int i = 0; i < DL; ++i) dst[i] = acc[u][i];
        if (lane == 0) {
            p.attn_ml[((size_t)h * p.max_chunks + ch) * 2] = m_run[u];
            p.attn_ml[((size_t)h * p.max_chunks + ch) * 2 + 1] = l_run[u];
        }
    }
}

// ---- B operand: 8 inputs of one pair (k-tile t, half h) ------------------------------------------
// Merged attention output dims [k0, k0 + 8) (all inside one head): log-sum-exp over the chunks in
// fixed order. Two passes whose loads are independent of each other's arithmetic (max of the chunk
// maxima, then the weighted sums), so each pass costs about one L2 round trip.
template <int HD>
SP_DEVINL void merge_attention(const StepParams &p, int k0, int n_chunks, float (&v)[8]) {
    const int hq = k0 / HD, d0 = k0 - hq * HD;
    const float *ml = p.attn_ml + (size_t)hq * p.max_chunks * 2;
    const float *ac = p.attn_acc + (size_t)hq * p.max_chunks * HD + d0;
    float M = -INFINITY;
#pragma unroll 16
    for (int c = 0; c < n_chunks; ++c) M = fmaxf(M, __ldcg(ml + 2 * c));
    float Ls = 0.f;
    float A[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) A[i] = 0.f;
#pragma unroll 8
    for (int c = 0; c < n_chunks; ++c) {
        const float2 mlc = __ldcg(reinterpret_cast<const float2 *>(ml + 2 * c));
        const float4 a0 = ldcg4(ac + (size_t)c * HD), a1 = ldcg4(ac + (size_t)c * HD + 4);
        const float f = mlc.x == -INFINITY ? 0.f : expf(mlc.x - M);
        Ls = fmaf(mlc.y, f, Ls);
        A[0] = fmaf(a0.x, f, A[0]); A[1] = fmaf(a0.y, f, A[1]); A[2] = fmaf(a0.z, f, A[2]); A[3] = fmaf(a0.w, f, A[3]);
        A[4] = fmaf(a1.x, f, A[4]); A[5] = fmaf(a1.y, f, A[5]); A[6] = fmaf(a1.z, f, A[6]); A[7] = fmaf(a1.w, f, A[7]);
    }
    const float inv = 1.f / Ls;
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = A[i] * inv;
}

}  // namespace

template <int HD>
__global__ void __launch_bounds__(kThreads, 1) k_step(const StepParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint32_t s_tmem;
    __shared__ float s_val[4];
    __shared__ int s_idx[4];
    __shared__ int s_flag;
    __shared__ int s_abort;
    __shared__ int s_issued, s_consumed;      // stages the producer issued / the MMA warp consumed
    __shared__ __align__(8) uint64_t s_drain; // MMA completion before TMEM is released
    __shared__ __align__(8) uint64_t accf[2], tfree[2];   // accumulator full (MMA -> epilogue) / free
    __shared__ int it_strip[2][kMaxItems], it_a[2][kMaxItems], it_b[2][kMaxItems], it_boff[2][kMaxItems];
    __shared__ int s_nitems[2];
    __shared__ __align__(16) float ystage[4][2][64];    // per warp: hi and lo rows of its 64 columns

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = gridDim.x, c = blockIdx.x;
    const int S = p.stages;
    uint8_t *ring = smem;
    uint8_t *abuf = smem + (size_t)S * kStageBytes;                         // activation atoms, 1 KB per 64 inputs
    uint8_t *am = abuf + (size_t)p.a_blocks * kABlockBytes;
    StepOp *ops = reinterpret_cast<StepOp *>(am + AttnRegion<HD>::bytes);   // the op table, copied once
    uint64_t *full = reinterpret_cast<uint64_t *>(ops + p.n_ops);
    uint64_t *empty = full + S;
    const Abort ab{&s_abort, p.st};

    // Every role reads op descriptors on its critical path: keep them in shared memory.
    for (int i = tid; i < p.n_ops * (int)(sizeof(StepOp) / 16); i += kThreads)
        reinterpret_cast<uint4 *>(ops)[i] = __ldg(reinterpret_cast<const uint4 *>(p.ops) + i);

    if (tid == 0) {
        s_abort = 0;
        s_issued = 0;
        s_consumed = 0;
        mbar_init(&s_drain, 1);
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&accf[i], 1);
            mbar_init(&tfree[i], 4);        // one arrival per epilogue warp
        }
        fence_mbar_init();
    }
    // rows 2-7 of every activation atom stay zero; rows 0/1 are rewritten per op
    for (int i = tid; i < p.a_blocks * kABlockBytes / 16; i += kThreads)
        reinterpret_cast<uint4 *>(abuf)[i] = make_uint4(0u, 0u, 0u, 0u);
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == kProducerWarp) {
        // ---- producer: every tile of the step, in op order; waits only for free stages ----------
        if (lane == 0) {
            int s = 0, round = 0, issued = 0;
            const uint64_t pol = policy_evict_first();
            for (int k = 0; k < p.n_ops && !ab.on(); ++k) {
                const StepOp &op = ops[k];
                if (op.kind != OP_GEMV) continue;
                const long long T = (long long)(op.N / kTileRows) * (op.K / kTileK);
                const int Cg = op.grid;
                if (c >= Cg) continue;
                const long long g0 = T * c / Cg, g1 = T * (c + 1) / Cg;
                for (long long g = g0; g < g1; g += kStageTiles) {
                    if (round > 0 && !wait_bar(&empty[s], (uint32_t)(round - 1) & 1u, ab)) break;
                    const int n = (int)(g1 - g < kStageTiles ? g1 - g : kStageTiles);
                    const uint32_t nb = (uint32_t)(n * kStepTileBytes);
                    mbar_arrive_expect_tx(&full[s], nb);
                    if (p.evict_first)
                        bulk_g2s_hint(ring + (size_t)s * kStageBytes, op.w + (size_t)g * kStepTileBytes, nb, &full[s], pol);
                    else
                        bulk_g2s(ring + (size_t)s * kStageBytes, op.w + (size_t)g * kStepTileBytes, nb, &full[s]);
                    ++issued;
                    if (++s == S) {
                        s = 0;
                        ++round;
                    }
                }
            }
            s_issued = issued;
        }
    } else if (warp == kMmaWarp) {
        // ---- MMA issuer: per tile 4 x (M=128, N=256, K=16); accumulators double-buffered ----------
        const uint32_t ring_addr = smem_u32(ring), a_addr0 = smem_u32(abuf);
        int s = 0, round = 0, gi = 0, consumed = 0;
        uint32_t gj = 0;                      // items of the step so far (accumulator = gj & 1)
        for (int k = 0; k < p.n_ops; ++k) {
            const StepOp &op = ops[k];
            if (op.kind != OP_GEMV) continue;
            const int buf = gi & 1;
            ++gi;
            bready_sync();
            tc_fence_after();
            if (lane == 0 && p.trace) p.trace[((size_t)k * C + c) * kStepTraceWords + 6] = globaltimer();
            if (lane == 0 && !ab.on()) {
                const int nitems = s_nitems[buf];
                const long long T = (long long)(op.N / kTileRows) * (op.K / kTileK);
                const int Cg = op.grid;
                const int ntiles = c < Cg ? (int)(T * (c + 1) / Cg - T * c / Cg) : 0;
                int item = 0, t = it_a[buf][0];
                uint32_t a_blk = (uint32_t)it_boff[buf][0];
                bool ok = ntiles == 0 || gj < 2 || wait_bar(&tfree[gj & 1], ((gj >> 1) - 1) & 1u, ab);
                for (int i = 0; i < ntiles && ok; i += kStageTiles) {
                    if (!wait_bar(&full[s], (uint32_t)round & 1u, ab)) break;
                    if (i == 0 && p.trace) p.trace[((size_t)k * C + c) * kStepTraceWords + 7] = globaltimer();
                    ++consumed;
                    tc_fence_after();
                    const int n = ntiles - i < kStageTiles ? ntiles - i : kStageTiles;
                    for (int q = 0; q < n && ok; ++q) {
                        const uint32_t d = tmem + (gj & 1u) * 256u;
                        const uint32_t b_addr = ring_addr + (uint32_t)(s * kStageBytes + q * kStepTileBytes);
                        const uint32_t a_addr = a_addr0 + a_blk * (uint32_t)kABlockBytes;
                        const bool first = t == it_a[buf][item];
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            mma_f16_id(d, smem_desc_sw128(a_addr + 32u * j, 0u), smem_desc_sw128(b_addr + 32u * j, 1024u),
                                       kIdescM128N256, (first && j == 0) ? 0u : 1u);
                        ++t;
                        ++a_blk;
                        if (t == it_b[buf][item]) {
                            mma_commit(&accf[gj & 1u]);
                            ++gj;
                            if (item + 1 < nitems) {
                                ++item;
                                t = it_a[buf][item];
                                a_blk = (uint32_t)it_boff[buf][item];
                                if (gj >= 2 && !wait_bar(&tfree[gj & 1u], ((gj >> 1) - 1) & 1u, ab)) ok = false;
                            }
                        }
                    }
                    mma_commit(&empty[s]);
                    if (++s == S) {
                        s = 0;
                        ++round;
                    }
                }
            }
            __syncwarp();
        }
        if (lane == 0) {
            s_consumed = consumed;
            mma_commit(&s_drain);    // arrives once every MMA this thread issued has completed
        }
        __syncwarp();
    } else {
        // ---- warps 0-3: dependencies, prologues, epilogues, attention -----------------------------
        griddep_wait();
        griddep_launch_dependents();
        DevState *st = p.st;
        StepState ss;
        ss.epoch = *p.epoch;
        ss.token = st->token;
        ss.pos = st->pos;
        ss.slot = st->slot;
        ss.tree_base = st->tree_base;
        ss.mask = ss.slot >= ss.tree_base ? st->small_mask[ss.slot - ss.tree_base] : 0ull;
        if (ss.pos < 0 || ss.pos >= p.max_pos || ss.slot < 0 || ss.slot >= p.cap) {
            if (tid == 0 && c == 0) atomicCAS(&st->err, 0, kErrBadSlot);
            ss.pos = min(max(ss.pos, 0), p.max_pos - 1);
            ss.slot = min(max(ss.slot, 0), p.cap - 1);
        }
        if (ss.token < 0 || ss.token >= p.vocab) {
            if (tid == 0 && c == 0) atomicCAS(&st->err, 0, kErrBadToken);
            ss.token = 0;
        }
        const int ctx = min(ss.slot + 1, p.cap);
        const int n_chunks = attn_chunks(ctx, p.max_chunks);
        const int rows_per = (ctx + n_chunks - 1) / n_chunks;
        const int half_hd = HD / 2;
        uint32_t gj = 0;                // items of the step so far (accumulator = gj & 1)
        int gi = 0;

        for (int k = 0; k < p.n_ops; ++k) {
            const StepOp &op = ops[k];
            stamp(p.trace, k, C, c, 0);
            if (op.kind == OP_ATTN) {
                // items on the last CTAs: narrow GEMVs use the first ones, so these arrive early and
                // stage their K/V rows while the QKV projection is still running
                const int items = p.nkv * n_chunks, item = C - 1 - c;
                if (item < items && !ab.on()) attention_item<HD>(p, op, ss, am, item, n_chunks, rows_per, ctx, ab);
                epi_sync();
                stamp(p.trace, k, C, c, 3);
                if (tid == 0 && op.sig >= 0) red_add_release(p.cnt + op.sig, 1ull);
                continue;
            }
            const int buf = gi & 1;
            ++gi;
            const int K = op.K, KB = K / kTileK;
            const long long T = (long long)(op.N / kTileRows) * KB;
            const int Cg = op.grid;          // CTAs c >= Cg own no tile of this GEMV
            const long long g0 = c < Cg ? T * c / Cg : T, g1 = c < Cg ? T * (c + 1) / Cg : T;
            const int ntiles = (int)(g1 - g0);
            if (tid == 0) {
                // items: the CTA's tiles split at strip boundaries (at most kMaxItems, host-checked)
                int n = 0, boff = 0;
                long long gg = g0;
                while (gg < g1 && n < kMaxItems) {
                    const int s = (int)(gg / KB), a = (int)(gg % KB);
                    const long long rest = (long long)a + (g1 - gg);
                    const int b = rest < KB ? (int)rest : KB;
                    it_strip[buf][n] = s;
                    it_a[buf][n] = a;
                    it_b[buf][n] = b;
                    it_boff[buf][n] = op.b_full ? a : boff;
                    boff += b - a;
                    gg += b - a;
                    ++n;
                }
                s_nitems[buf] = n;
            }
            if (p.l2_ahead > 0 && op.dep >= 0) warm_l2_for(p, ops, k, c, tid, S * kStageTiles, p.l2_ahead);
            if (tid == 0 && op.dep >= 0 && !ab.on())
                wait_counter(p.cnt + op.dep, (unsigned long long)op.dep_n * (ss.epoch + 1), ab);
            epi_sync();
            stamp(p.trace, k, C, c, 1);
            const int nitems = s_nitems[buf];

            // ---- prologue: activation atoms (row 0 fp16 hi, row 1 fp16 lo) from one L2 round trip ---
            const int nb = op.b_full ? KB : ntiles;
            const int nunits = nb * 8;          // 8 inputs (one 16-byte chunk of a row) per unit
            float v[kMaxUnits][8], gg8[kMaxUnits][8];
            float sq = 0.f;
            const bool norm = op.pro == PRO_NORM || op.pro == PRO_EMBED_NORM;
            const __half *erow = p.embed + (size_t)ss.token * K;
#pragma unroll
            for (int q = 0; q < kMaxUnits; ++q) {
                const int u = tid + q * kEpiThreads;
                if (u >= nunits) continue;
                const int bt = u >> 3, ch = u & 7;
                int t = bt;
                if (!op.b_full) {
                    int j = 0;
                    while (j + 1 < nitems && bt >= it_boff[buf][j + 1]) ++j;
                    t = it_a[buf][j] + (bt - it_boff[buf][j]);
                }
                const int k0 = kTileK * t + 8 * ch;
                if (op.pro == PRO_EMBED_NORM) {
                    const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(erow + k0));
                    const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 t2 = __half22float2(h2[j]);
                        v[q][2 * j] = t2.x;
                        v[q][2 * j + 1] = t2.y;
                    }
                } else if (op.pro == PRO_ATTN) {
                    merge_attention<HD>(p, k0, n_chunks, v[q]);
                } else {
                    const float4 x0 = ldcg4(op.xin + k0), x1 = ldcg4(op.xin + k0 + 4);
                    v[q][0] = x0.x; v[q][1] = x0.y; v[q][2] = x0.z; v[q][3] = x0.w;
                    v[q][4] = x1.x; v[q][5] = x1.y; v[q][6] = x1.z; v[q][7] = x1.w;
                }
                if (norm) {
                    const float4 ga = __ldg(reinterpret_cast<const float4 *>(op.gain + k0));
                    const float4 gb = __ldg(reinterpret_cast<const float4 *>(op.gain + k0 + 4));
                    gg8[q][0] = ga.x; gg8[q][1] = ga.y; gg8[q][2] = ga.z; gg8[q][3] = ga.w;
                    gg8[q][4] = gb.x; gg8[q][5] = gb.y; gg8[q][6] = gb.z; gg8[q][7] = gb.w;
                    if (op.b_full) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) sq = fmaf(v[q][j], v[q][j], sq);
                    }
                }
            }
            float inv = 1.f;
            if (norm) {
                if (!op.b_full) {
                    // the sum of squares needs the whole vector
                    if (op.pro == PRO_EMBED_NORM) {
                        for (int vv = tid; vv < K / 8; vv += kEpiThreads) {
                            const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(erow) + vv);
                            const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const float2 t2 = __half22float2(h2[j]);
                                sq = fmaf(t2.x, t2.x, sq);
                                sq = fmaf(t2.y, t2.y, sq);
                            }
                        }
                    } else {
                        for (int vv = tid; vv < K / 4; vv += kEpiThreads) {
                            const float4 f = ldcg4(op.xin + 4 * vv);
                            sq = fmaf(f.x, f.x, sq);
                            sq = fmaf(f.y, f.y, sq);
                            sq = fmaf(f.z, f.z, sq);
                            sq = fmaf(f.w, f.w, sq);
                        }
                    }
                }
                sq = warp_sum(sq);
                if (lane == 0) s_val[warp] = sq;
                epi_sync();
                inv = 1.0f / sqrtf((s_val[0] + s_val[1] + s_val[2] + s_val[3]) / (float)K + p.eps);
            }
#pragma unroll
            for (int q = 0; q < kMaxUnits; ++q) {
                const int u = tid + q * kEpiThreads;
                if (u >= nunits) continue;
                const int bt = u >> 3, ch = u & 7;
                if (norm) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) v[q][j] = (v[q][j] * inv) * gg8[q][j];
                }
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const __half h0 = __float2half_rn(v[q][2 * j]), h1 = __float2half_rn(v[q][2 * j + 1]);
                    const __half l0 = __float2half_rn(v[q][2 * j] - __half2float(h0));
                    const __half l1 = __float2half_rn(v[q][2 * j + 1] - __half2float(h1));
                    hi[j] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
                    lo[j] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
                }
                // row 0 (hi) keeps chunk ch at position ch, row 1 (lo) at position ch ^ 1
                uint8_t *atom = abuf + (size_t)bt * kABlockBytes;
                *reinterpret_cast<uint4 *>(atom + ch * 16) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4 *>(atom + 128 + (ch ^ 1) * 16) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
            fence_proxy_async_smem();
            bready_sync();
            stamp(p.trace, k, C, c, 2);

            // ---- epilogue: warp w takes columns [64w, 64w + 64) of the item's 256 output rows ---------
            float *lg = nullptr;
            if (op.epi == EPI_LMHEAD && st->logits != nullptr && st->step >= st->logits_from)
                lg = st->logits + st->logits_stride * (long long)st->step;
            float bv = -INFINITY;
            int bi = INT_MAX;
            int n_final = 0;
            const int col = 64 * warp + 2 * lane;   // this thread's row pair (col, col + 1) of a strip
            for (int j = 0; j < nitems; ++j) {
                // epilogue operands that do not depend on the accumulator: load them before waiting
                const int strip = it_strip[buf][j];
                const int row = strip * kTileRows + col;
                float pre0 = 0.f, pre1 = 0.f, pcs = 1.f, psn = 0.f;
                if (row < op.n_valid) {
                    if (op.epi == EPI_RESID) {
                        if (op.resid_embed) {
                            const __half2 e2 = *reinterpret_cast<const __half2 *>(p.embed + (size_t)ss.token * p.hidden + row);
                            pre0 = __low2float(e2);
                            pre1 = __high2float(e2);
                        } else {
                            const float2 b2 = __ldcg(reinterpret_cast<const float2 *>(op.out + row));
                            pre0 = b2.x;
                            pre1 = b2.y;
                        }
                    } else if (op.epi == EPI_QKV) {
                        const int P = row / 2, hh = P / half_hd, dd = P - hh * half_hd;
                        pre0 = __ldg(op.bias + hh * HD + dd);
                        pre1 = __ldg(op.bias + hh * HD + dd + half_hd);
                        if (hh < p.nh + p.nkv) {
                            const float2 r2 = __ldg(reinterpret_cast<const float2 *>(p.rope + ((size_t)ss.pos * half_hd + dd) * 2));
                            pcs = r2.x;
                            psn = r2.y;
                        }
                    }
                }
                const uint32_t tb = gj & 1u;
                const bool ok = !ab.on() && wait_bar(&accf[tb], (gj >> 1) & 1u, ab);
                ++gj;
                if (!ok) continue;
                if (j == 0) stamp(p.trace, k, C, c, 4);
                if (j == nitems - 1) stamp(p.trace, k, C, c, 5);
                tc_fence_after();
                {
                    uint32_t r0[32], r1[32];
                    const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + tb * 256u + (uint32_t)(warp * 64);
                    tmem_ld32_nowait(taddr, r0);
                    tmem_ld32_nowait(taddr + 32u, r1);
                    tmem_wait_ld();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tfree[tb]);     // this warp's columns are read
                    if (lane < 2) {
                        float4 *dst = reinterpret_cast<float4 *>(&ystage[warp][lane][0]);
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            dst[i] = make_float4(__uint_as_float(r0[4 * i]), __uint_as_float(r0[4 * i + 1]),
                                                 __uint_as_float(r0[4 * i + 2]), __uint_as_float(r0[4 * i + 3]));
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            dst[8 + i] = make_float4(__uint_as_float(r1[4 * i]), __uint_as_float(r1[4 * i + 1]),
                                                     __uint_as_float(r1[4 * i + 2]), __uint_as_float(r1[4 * i + 3]));
                    }
                }
                __syncwarp();
                const float2 hv = *reinterpret_cast<const float2 *>(&ystage[warp][0][2 * lane]);
                const float2 lv = *reinterpret_cast<const float2 *>(&ystage[warp][1][2 * lane]);
                __syncwarp();
                float y0 = hv.x + lv.x, y1 = hv.y + lv.y;
                if (it_a[buf][j] != 0 || it_b[buf][j] != KB) {
                    // strip shared with other CTAs: post this part; the last contributor sums all
                    const long long first = (long long)strip * KB;
                    const int cf = tc_cta_of(first, T, Cg), cl = tc_cta_of(first + KB - 1, T, Cg);
                    float *slotp = p.partial + ((size_t)strip * op.max_contrib + (c - cf)) * kTileRows;
                    *reinterpret_cast<float2 *>(slotp + col) = make_float2(y0, y1);
                    epi_sync();
                    if (tid == 0) s_flag = atom_add_acq_rel(p.strip_cnt + strip, 1u) == (unsigned)(cl - cf);
                    epi_sync();
                    if (!s_flag) continue;
                    const float *all = p.partial + (size_t)strip * op.max_contrib * kTileRows + col;
                    y0 = 0.f;
                    y1 = 0.f;
                    const int ncon = cl - cf + 1;
                    for (int k2 = 0; k2 < ncon; k2 += 16) {
                        // sixteen contributors' loads in flight, summed in contributor order
                        float2 pv[16];
#pragma unroll
                        for (int u = 0; u < 16; ++u)
                            pv[u] = k2 + u < ncon ? __ldcg(reinterpret_cast<const float2 *>(all + (size_t)(k2 + u) * kTileRows))
                                                  : make_float2(0.f, 0.f);
#pragma unroll
                        for (int u = 0; u < 16; ++u) {
                            y0 += pv[u].x;
                            y1 += pv[u].y;
                        }
                    }
                    if (tid == 0) p.strip_cnt[strip] = 0u;
                }
                ++n_final;
                if (row >= op.n_valid) continue;
                if (op.epi == EPI_RESID) {
                    *reinterpret_cast<float2 *>(op.out + row) = make_float2(pre0 + y0, pre1 + y1);
                } else if (op.epi == EPI_LMHEAD) {
                    if (lg) lg[row] = y0;
                    if (y0 > bv) {
                        bv = y0;
                        bi = row;
                    }
                    if (row + 1 < op.n_valid) {
                        if (lg) lg[row + 1] = y1;
                        if (y1 > bv) {
                            bv = y1;
                            bi = row + 1;
                        }
                    }
                } else if (op.epi == EPI_SWIGLU) {
                    op.out[row / 2] = (y0 / (1.0f + expf(-y0))) * y1;
                } else {  // EPI_QKV: packed rows (2q, 2q+1) are dims (d, d + hd/2) of one head
                    const int P = row / 2;
                    const int hh = P / half_hd, dd = P - hh * half_hd;
                    const int lo = hh * HD + dd, hi = lo + half_hd;
                    const float a0 = y0 + pre0, a1 = y1 + pre1;
                    if (hh < p.nh + p.nkv) {
                        const float cs = pcs, sn = psn;
                        const float o0 = __fadd_rn(__fmul_rn(a0, cs), -__fmul_rn(a1, sn));
                        const float o1 = __fadd_rn(__fmul_rn(a1, cs), __fmul_rn(a0, sn));
                        if (hh < p.nh) {
                            op.out[lo] = o0;
                            op.out[hi] = o1;
                        } else {
                            __half *kr = op.kc + ((size_t)(hh - p.nh) * p.cap + ss.slot) * HD;
                            kr[dd] = __float2half_rn(o0);
                            kr[dd + half_hd] = __float2half_rn(o1);
                        }
                    } else {
                        __half *vr = op.vc + ((size_t)(hh - p.nh - p.nkv) * p.cap + ss.slot) * HD;
                        vr[dd] = __float2half_rn(a0);
                        vr[dd + half_hd] = __float2half_rn(a1);
                    }
                }
            }

            if (op.epi == EPI_LMHEAD) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    tc_argmax_merge(bv, bi, ov, oi);
                }
                if (lane == 0) {
                    s_val[warp] = bv;
                    s_idx[warp] = bi;
                }
                epi_sync();
                if (tid == 0) {
                    float vb = s_val[0];
                    int ib = s_idx[0];
                    for (int w = 1; w < 4; ++w) tc_argmax_merge(vb, ib, s_val[w], s_idx[w]);
                    p.part_val[c] = vb;
                    p.part_idx[c] = ib;
                    s_flag = atom_add_acq_rel(p.lm_cnt, 1u) == (unsigned)C - 1u;
                }
                epi_sync();
                if (s_flag) {
                    float vb = -INFINITY;
                    int ib = INT_MAX;
                    for (int j = tid; j < C; j += kEpiThreads)
                        tc_argmax_merge(vb, ib, __ldcg(p.part_val + j), __ldcg(p.part_idx + j));
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const float ov = __shfl_xor_sync(0xffffffffu, vb, o);
                        const int oi = __shfl_xor_sync(0xffffffffu, ib, o);
                        tc_argmax_merge(vb, ib, ov, oi);
                    }
                    epi_sync();
                    if (lane == 0) {
                        s_val[warp] = vb;
                        s_idx[warp] = ib;
                    }
                    epi_sync();
                    if (tid == 0) {
                        for (int w = 1; w < 4; ++w) tc_argmax_merge(s_val[0], s_idx[0], s_val[w], s_idx[w]);
                        int tok = s_idx[0];
                        if (tok < 0 || tok >= op.n_valid) {
                            atomicCAS(&st->err, 0, kErrBadToken);
                            tok = 0;
                        }
                        *p.lm_cnt = 0u;
                        const int step = st->step;
                        if (st->out_tokens) st->out_tokens[step] = tok;
                        const int nxt = step + 1;
                        st->step = nxt;
                        if (nxt < st->n_forced) {
                            st->slot = st->slot0 + nxt;
                            st->token = st->use_small ? st->small_tok[nxt] : st->f_tok[nxt];
                            st->pos = st->use_small ? st->small_pos[nxt] : (st->f_pos ? st->f_pos[nxt] : st->slot0 + nxt);
                        } else {
                            st->token = tok;
                            st->pos += 1;
                            st->slot += 1;
                        }
                        *p.epoch = ss.epoch + 1;
                    }
                }
            } else if (op.sig >= 0) {
                epi_sync();
                if (tid == 0 && n_final > 0) red_add_release(p.cnt + op.sig, (unsigned long long)n_final);
            }
            stamp(p.trace, k, C, c, 3);
        }
    }

    // producer and MMA warps are done; all TMEM reads are fenced: release TMEM
    __syncthreads();
    if (warp == kProducerWarp && lane == 0) {
        // after an abort, stages may still be in flight: let their copies land before exiting
        for (int i = s_consumed; i < s_issued; ++i) mbar_wait_bounded(&full[i % S], (uint32_t)(i / S) & 1u);
    }
    if (warp == kMmaWarp) {
        if (lane == 0) mbar_wait_bounded(&s_drain, 0u);
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// Pack an fp16 N x K matrix into 256 x 64 tiles of 128B-swizzled K-major rows: tile (strip s, k-block
// t) at (s * K/64 + t) * 32 KB; inside it row r (0..255) at r * 128 B with input chunk c (8 inputs)
// at chunk position c ^ (r & 7). Packed row `row` is source row row_of[row] of `a` (< rows_a) or of
// `b` (row_of - rows_a); row_of < 0 is a zero row. One thread per 16-byte chunk.
__global__ void k_pack_sw128(uint8_t *dst, const __half *a, int rows_a, const __half *b, const int *row_of, int N, int K) {
    const int KB = K / kTileK;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long total = (long long)N * K / 8;
    if (idx >= total) return;
    const long long tile = idx >> 11;                 // 2048 chunks of 16 B per 32 KB tile
    const int within = (int)(idx & 2047);
    const int r = within >> 3, pc = within & 7;
    const int ch = pc ^ (r & 7);
    const int s = (int)(tile / KB), t = (int)(tile % KB);
    const int row = kTileRows * s + r;
    const int src = row_of[row];
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (src >= 0) {
        const __half *rp = src < rows_a ? a + (size_t)src * K : b + (size_t)(src - rows_a) * K;
        v = *reinterpret_cast<const uint4 *>(rp + kTileK * t + 8 * ch);
    }
    *reinterpret_cast<uint4 *>(dst + (size_t)idx * 16) = v;
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
void plan_step_gemv(StepOp &o, int num_sms, int min_tiles) {
    const int KB = o.K / kTileK;
    const long long T = (long long)(o.N / kTileRows) * KB;
    // at least `min_tiles` tiles per CTA: fewer CTAs share a strip, so its last contributor sums
    // fewer partials and waits for fewer CTAs
    o.grid = (int)std::max<long long>(1, std::min<long long>(num_sms, T / std::max(1, min_tiles)));
    const long long per = (T + o.grid - 1) / o.grid;
    o.b_full = per >= KB ? 1 : 0;
    o.a_blocks = o.b_full ? KB : (int)per;
    const long long minper = std::max<long long>(1, T / o.grid);
    o.max_contrib = (int)((KB + minper - 1) / minper + 1);
    o.max_items = (int)(per / KB + 2);
}

int step_max_items() { return kMaxItems; }
int step_max_a_blocks() { return kMaxUnits * kEpiThreads / 8; }

size_t step_attn_smem_bytes(int hd) { return hd == 64 ? AttnRegion<64>::bytes : AttnRegion<128>::bytes; }

static size_t step_static_reserve() { return 4096; }   // static shared memory of k_step, rounded up

size_t step_smem_bytes(int stages, int a_blocks, int hd, int n_ops) {
    return (size_t)stages * kStageBytes + (size_t)a_blocks * kABlockBytes + step_attn_smem_bytes(hd) +
           (size_t)n_ops * sizeof(StepOp) + (size_t)(2 * stages) * 8;
}

int step_stages_for(int a_blocks, int hd, int n_ops) {
    const size_t budget = 227 * 1024 - step_static_reserve();
    const size_t fixed = (size_t)a_blocks * kABlockBytes + step_attn_smem_bytes(hd) + (size_t)n_ops * sizeof(StepOp);
    if (fixed >= budget) return 0;
    return (int)((budget - fixed) / (kStageBytes + 16));
}

cudaError_t launch_pack_sw128(uint8_t *dst, const __half *a, int rows_a, const __half *b, const int *row_of, int N, int K,
                              cudaStream_t s) {
    if (N % kTileRows || K % kTileK) return cudaErrorInvalidValue;
    const long long total = (long long)N * K / 8;
    k_pack_sw128<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(dst, a, rows_a, b, row_of, N, K);
    return cudaGetLastError();
}

template <int HD>
static cudaError_t step_launch_t(const StepParams *p, int grid, size_t smem, cudaStream_t s, bool pdl) {
    if (p == nullptr) {
        cudaError_t e = cudaFuncSetAttribute(k_step<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        return cudaFuncSetAttribute(k_step<HD>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    (int)cudaSharedmemCarveoutMaxShared);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeCooperative;
    attr[na].val.cooperative = 1;
    ++na;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k_step<HD>, *p);
}

cudaError_t prepare_step(int hd, size_t smem) {
    if (hd == 128) return step_launch_t<128>(nullptr, 0, smem, nullptr, false);
    if (hd == 64) return step_launch_t<64>(nullptr, 0, smem, nullptr, false);
    return cudaErrorInvalidValue;
}

cudaError_t launch_step(int hd, const StepParams &p, int grid, size_t smem, cudaStream_t s, bool pdl) {
    if (p.stages < 2 || p.a_blocks > step_max_a_blocks() || p.nh / p.nkv > kGroup || p.nkv * p.max_chunks > grid ||
        p.max_chunks > kStepMaxChunks)
        return cudaErrorInvalidValue;
    if (hd == 128) return step_launch_t<128>(&p, grid, smem, s, pdl);
    if (hd == 64) return step_launch_t<64>(&p, grid, smem, s, pdl);
    return cudaErrorInvalidValue;
}

}  // namespace sp
