// sm_100a decode kernels of the SeedPlane B200 engine.
//
// k_gemv    -- weight-streaming GEMV. One CTA per SM owns a contiguous range of weight rows and
//              streams it HBM -> shared memory through a ring of stages filled by 1-D bulk copies
//              (cp.async.bulk, TMA engine, mbarrier completion). The first stages are requested
//              BEFORE griddepcontrol.wait, so under programmatic dependent launch a kernel's weight
//              stream starts while the previous kernel is still finishing. Warps reduce rows in
//              fp32 from the staged fp16 (or int8 + fp16 block scale) weights and an fp32 input
//              vector held in shared memory. Prologues: RMSNorm of the residual stream, embedding
//              gather. Epilogues: bias + RoPE + K/V-cache write (QKV), residual add (O, down),
//              SiLU(gate)*up (gate_up), logits + greedy argmax with lowest-index ties (LM head).
//              Replaces the Vulkan gemv/swiglu/rope_kv/argmax shaders
//              (native/vulkan_decode/shaders/gemv.comp:23-51, swiglu.comp:20-44,
//              rope_kv.comp:14-32, argmax.comp:8-22).
// k_attn_decode -- GQA decode attention, split-K over the context: one CTA per (kv head, chunk)
//              serves all q heads of its group, partial (max, sum, acc) per chunk, and the last CTA
//              of a group to finish merges the partials (log-sum-exp) and writes the output.
//              Replaces attn_part.comp:15-44 + attn_combine.comp:8-19; the mask is the
//              reference's `slot <= own slot` (qwen_engine.py:131-135) or a tree-ancestor mask.
#include <algorithm>
#include <climits>
#include <cmath>
#include <utility>

#include "kernels.cuh"

namespace sp {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxTasks = 32;
constexpr int kTargetStage = 24 * 1024;

SP_DEVINL void argmax_merge(float &v, int &i, float ov, int oi) {
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
}

SP_DEVINL float dot16_i8(const uint4 q, const float4 *x, float acc) {
    const uint32_t wds[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float4 a = x[j];
        const uint32_t w = wds[j];
        acc = fmaf((float)(int8_t)(w & 0xff), a.x, acc);
        acc = fmaf((float)(int8_t)((w >> 8) & 0xff), a.y, acc);
        acc = fmaf((float)(int8_t)((w >> 16) & 0xff), a.z, acc);
        acc = fmaf((float)(int8_t)(w >> 24), a.w, acc);
    }
    return acc;
}

// Dot product of one staged row segment [v0, v0 + nv) (16-byte vectors) with the input vector.
template <int FMT>
SP_DEVINL float dot_segment(const uint8_t *stage, int r, int R, int K, int v0, int nv, const float *xs, int lane) {
    const float4 *x4 = reinterpret_cast<const float4 *>(xs);
    float a0 = 0.f, a1 = 0.f;
    if constexpr (FMT == WF_F16) {
        const uint4 *wr = reinterpret_cast<const uint4 *>(stage + (size_t)r * K * 2);
        int v = v0 + lane;
        const int ve = v0 + nv;
        for (; v + 32 < ve; v += 64) {
            a0 = dot8_f16(wr[v], x4[2 * v], x4[2 * v + 1], a0);
            a1 = dot8_f16(wr[v + 32], x4[2 * v + 64], x4[2 * v + 65], a1);
        }
        if (v < ve) a0 = dot8_f16(wr[v], x4[2 * v], x4[2 * v + 1], a0);
    } else {
        const uint4 *wr = reinterpret_cast<const uint4 *>(stage + (size_t)r * K);
        const __half *sc = reinterpret_cast<const __half *>(stage + (size_t)R * K) + (size_t)r * (K / 32);
        for (int v = v0 + lane; v < v0 + nv; v += 32) {
            const float t = dot16_i8(wr[v], x4 + 4 * v, 0.f);
            a0 = fmaf(__half2float(sc[v >> 1]), t, a0);
        }
    }
    return a0 + a1;
}

template <int PRO, int EPI, int FMT>
__global__ void __launch_bounds__(kThreads) k_gemv(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_val[kWarps];
    __shared__ int s_idx[kWarps];
    __shared__ int s_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = p.stages, SB = p.stage_bytes, K = p.K, R = p.rows_per_chunk, SPLIT = p.split;
    uint8_t *ring = smem;
    float *xs = reinterpret_cast<float *>(smem + (size_t)S * SB);
    float *red = xs + K;
    uint64_t *bars = reinterpret_cast<uint64_t *>(red + 2 * kMaxTasks);

    constexpr int RG = (EPI == EPI_QKV || EPI == EPI_SWIGLU) ? 2 : 1;
    const int C = gridDim.x, c = blockIdx.x;
    const int ngroups = p.N / RG;
    const int r0 = (int)((long long)ngroups * c / C) * RG;
    const int r1 = (int)((long long)ngroups * (c + 1) / C) * RG;
    const int nch = (r1 - r0 + R - 1) / R;
    const size_t row_bytes = FMT == WF_F16 ? (size_t)K * 2 : (size_t)K;
    const size_t srow_bytes = FMT == WF_I8 ? (size_t)(K / 32) * 2 : 0;

    auto issue = [&](int i) {
        const int s = i % S;
        const int cr0 = r0 + i * R;
        const int nr = min(R, r1 - cr0);
        uint8_t *dst = ring + (size_t)s * SB;
        const uint32_t wbytes = (uint32_t)(nr * row_bytes);
        const uint32_t sbytes = (uint32_t)(nr * srow_bytes);
        mbar_arrive_expect_tx(&bars[s], wbytes + sbytes);
        bulk_g2s(dst, p.w + (size_t)cr0 * row_bytes, wbytes, &bars[s]);
        if constexpr (FMT == WF_I8)
            bulk_g2s(dst + (size_t)R * row_bytes, reinterpret_cast<const uint8_t *>(p.ws) + (size_t)cr0 * srow_bytes,
                     sbytes, &bars[s]);
    };

    // Weights do not depend on the previous kernel: start streaming them before the dependency wait.
    if (tid == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        for (int i = 0; i < min(S, nch); ++i) issue(i);
    }
    __syncthreads();
    griddep_wait();
    griddep_launch_dependents();

    DevState *st = p.st;
    // ---- prologue: fp32 input vector in shared memory --------------------------------------
    if constexpr (PRO == PRO_EMBED_NORM) {
        int tok = st->token;
        if (tok < 0 || tok >= p.vocab) {
            if (tid == 0) atomicCAS(&st->err, 0, kErrBadToken);
            tok = 0;
        }
        const __half2 *e = reinterpret_cast<const __half2 *>(p.embed + (size_t)tok * K);
        for (int k = tid; k < K / 2; k += kThreads) {
            const float2 f = __half22float2(e[k]);
            xs[2 * k] = f.x;
            xs[2 * k + 1] = f.y;
            if (c == 0) {
                p.x_init[2 * k] = f.x;
                p.x_init[2 * k + 1] = f.y;
            }
        }
    } else {
        for (int k = tid * 4; k < K; k += kThreads * 4)
            *reinterpret_cast<float4 *>(xs + k) = *reinterpret_cast<const float4 *>(p.xin + k);
    }
    if constexpr (PRO != PRO_PLAIN) {
        __syncthreads();
        float ss = 0.f;
        for (int k = tid; k < K; k += kThreads) ss = fmaf(xs[k], xs[k], ss);
        ss = warp_sum(ss);
        if (lane == 0) s_val[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tot += s_val[w];
        const float inv = 1.0f / sqrtf(tot / (float)K + p.eps);
        for (int k = tid; k < K; k += kThreads) xs[k] = (xs[k] * inv) * p.gain[k];
    }
    __syncthreads();

    // ---- per-step values --------------------------------------------------------------------
    int pos = 0, slot = 0;
    float *lg = nullptr;
    if constexpr (EPI == EPI_QKV) {
        pos = st->pos;
        slot = st->slot;
        if (pos < 0 || pos >= p.max_pos || slot < 0 || slot >= p.cap) {
            if (tid == 0) atomicCAS(&st->err, 0, kErrBadSlot);
            pos = min(max(pos, 0), p.max_pos - 1);
            slot = min(max(slot, 0), p.cap - 1);
        }
    }
    if constexpr (EPI == EPI_LMHEAD) {
        if (st->logits != nullptr && st->step >= st->logits_from)
            lg = st->logits + st->logits_stride * (long long)st->step;
    }
    float bv = -INFINITY;
    int bi = INT_MAX;

    const int vec_per_row = FMT == WF_F16 ? K / 8 : K / 16;
    const int segv = vec_per_row / SPLIT;
    const int half_hd = p.hd / 2;

    for (int i = 0; i < nch; ++i) {
        const int s = i % S;
        const uint32_t par = (uint32_t)(i / S) & 1u;
        const bool ok = mbar_wait_bounded(&bars[s], par);
        const uint8_t *stage = ring + (size_t)s * SB;
        const int cr0 = r0 + i * R;
        const int nr = min(R, r1 - cr0);
        float *rb = red + (i & 1) * kMaxTasks;
        if (ok) {
            const int ntask = nr * SPLIT;
            for (int t = warp; t < ntask; t += kWarps) {
                const int r = t / SPLIT, sg = t - r * SPLIT;
                float acc = dot_segment<FMT>(stage, r, R, K, sg * segv, segv, xs, lane);
                acc = warp_sum(acc);
                if (lane == 0) rb[t] = acc;
            }
        }
        if (!__syncthreads_and(ok)) {
            // A stage never arrived: record it, wait (bounded) for copies still in flight, leave.
            if (tid == 0) {
                atomicCAS(&st->err, 0, kErrMbarTimeout);
                for (int j = i; j < min(i + S, nch); ++j) mbar_wait_bounded(&bars[j % S], (uint32_t)(j / S) & 1u);
            }
            __syncthreads();
            return;
        }
        if (tid == 0 && i + S < nch) issue(i + S);

        // ---- epilogue for the rows of this chunk ------------------------------------------
        if constexpr (EPI == EPI_RESID) {
            if (tid < nr) {
                float y = 0.f;
                for (int sg = 0; sg < SPLIT; ++sg) y += rb[tid * SPLIT + sg];
                const int row = cr0 + tid;
                p.out[row] = p.out[row] + y;
            }
        } else if constexpr (EPI == EPI_LMHEAD) {
            if (tid < nr) {
                float y = 0.f;
                for (int sg = 0; sg < SPLIT; ++sg) y += rb[tid * SPLIT + sg];
                const int row = cr0 + tid;
                if (lg) lg[row] = y;
                if (y > bv) { bv = y; bi = row; }
            }
        } else if constexpr (EPI == EPI_SWIGLU) {
            if (tid < nr / 2) {
                float g = 0.f, u = 0.f;
                for (int sg = 0; sg < SPLIT; ++sg) {
                    g += rb[(2 * tid) * SPLIT + sg];
                    u += rb[(2 * tid + 1) * SPLIT + sg];
                }
                p.out[cr0 / 2 + tid] = (g / (1.0f + expf(-g))) * u;
            }
        } else {  // EPI_QKV: packed rows come in RoPE pairs (d, d + hd/2) of one head
            if (tid < nr / 2) {
                float y0 = 0.f, y1 = 0.f;
                for (int sg = 0; sg < SPLIT; ++sg) {
                    y0 += rb[(2 * tid) * SPLIT + sg];
                    y1 += rb[(2 * tid + 1) * SPLIT + sg];
                }
                const int P = cr0 / 2 + tid;
                const int hh = P / half_hd, d = P - hh * half_hd;
                const int lo = hh * p.hd + d, hi = lo + half_hd;
                y0 += p.bias[lo];
                y1 += p.bias[hi];
                if (hh < p.nh + p.nkv) {
                    const float cs = p.rope[((size_t)pos * half_hd + d) * 2];
                    const float sn = p.rope[((size_t)pos * half_hd + d) * 2 + 1];
                    const float o0 = __fadd_rn(__fmul_rn(y0, cs), -__fmul_rn(y1, sn));
                    const float o1 = __fadd_rn(__fmul_rn(y1, cs), __fmul_rn(y0, sn));
                    if (hh < p.nh) {
                        p.out[lo] = o0;
                        p.out[hi] = o1;
                    } else {
                        __half *kr = p.kc + ((size_t)(hh - p.nh) * p.cap + slot) * p.hd;
                        kr[d] = __float2half_rn(o0);
                        kr[d + half_hd] = __float2half_rn(o1);
                    }
                } else {
                    __half *vr = p.vc + ((size_t)(hh - p.nh - p.nkv) * p.cap + slot) * p.hd;
                    vr[d] = __float2half_rn(y0);
                    vr[d + half_hd] = __float2half_rn(y1);
                }
            }
        }
    }

    if constexpr (EPI == EPI_LMHEAD) {
        // CTA argmax (lowest index among equal maxima), then the last CTA reduces all CTAs.
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            argmax_merge(bv, bi, ov, oi);
        }
        if (lane == 0) { s_val[warp] = bv; s_idx[warp] = bi; }
        __syncthreads();
        if (tid == 0) {
            float v = s_val[0];
            int ix = s_idx[0];
            for (int w = 1; w < kWarps; ++w) argmax_merge(v, ix, s_val[w], s_idx[w]);
            p.part_val[c] = v;
            p.part_idx[c] = ix;
            __threadfence();
            const unsigned old = atomicAdd(p.counter, 1u);
            s_flag = (old == (unsigned)C - 1u);
        }
        __syncthreads();
        if (!s_flag) return;
        __threadfence();
        float v = -INFINITY;
        int ix = INT_MAX;
        for (int j = tid; j < C; j += kThreads) argmax_merge(v, ix, __ldcg(p.part_val + j), __ldcg(p.part_idx + j));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, ix, o);
            argmax_merge(v, ix, ov, oi);
        }
        __syncthreads();
        if (lane == 0) { s_val[warp] = v; s_idx[warp] = ix; }
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < kWarps; ++w) argmax_merge(s_val[0], s_idx[0], s_val[w], s_idx[w]);
            int tok = s_idx[0];
            if (tok < 0 || tok >= p.N) {
                atomicCAS(&st->err, 0, kErrBadToken);
                tok = 0;
            }
            *p.counter = 0u;
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
        }
    }
}

// ---------------------------------------------------------------------------------------------
// GQA decode attention
// ---------------------------------------------------------------------------------------------
constexpr int kMaxGroup = 8;

template <int HD>
__global__ void __launch_bounds__(kThreads) k_attn_decode(const AttnParams p) {
    constexpr int DPL = HD / 32;
    __shared__ float sm_m[kWarps][kMaxGroup], sm_l[kWarps][kMaxGroup];
    __shared__ float sm_acc[kWarps][kMaxGroup][HD];
    __shared__ int s_flag;

    griddep_wait();
    griddep_launch_dependents();

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = blockIdx.y, c = blockIdx.x;
    const DevState *st = p.st;
    const int slot = st->slot, tree_base = st->tree_base;
    const unsigned long long mask = slot >= tree_base ? st->small_mask[slot - tree_base] : 0ull;
    const int ctx = min(slot + 1, p.cap);
    int nsplit = (ctx + p.min_chunk - 1) / p.min_chunk;
    nsplit = max(1, min(nsplit, p.max_split));
    const int chunk = (ctx + nsplit - 1) / nsplit;
    if (c >= nsplit) return;
    const int j0 = c * chunk, j1 = min(ctx, j0 + chunk);
    const int G = p.nh / p.nkv;

    float qr[kMaxGroup][DPL], m[kMaxGroup], l[kMaxGroup], acc[kMaxGroup][DPL];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
            acc[h][e] = 0.f;
            qr[h][e] = h < G ? p.q[(g * G + h) * HD + lane * DPL + e] : 0.f;
        }
    }
    const __half *kb = p.kc + (size_t)g * p.cap * HD;
    const __half *vb = p.vc + (size_t)g * p.cap * HD;
    for (int j = j0 + warp; j < j1; j += kWarps) {
        if (j >= tree_base && !((mask >> (j - tree_base)) & 1ull)) continue;
        float kf[DPL], vf[DPL];
        const __half2 *kp = reinterpret_cast<const __half2 *>(kb + (size_t)j * HD + lane * DPL);
        const __half2 *vp = reinterpret_cast<const __half2 *>(vb + (size_t)j * HD + lane * DPL);
#pragma unroll
        for (int e = 0; e < DPL / 2; ++e) {
            const float2 a = __half22float2(kp[e]), b = __half22float2(vp[e]);
            kf[2 * e] = a.x; kf[2 * e + 1] = a.y;
            vf[2 * e] = b.x; vf[2 * e + 1] = b.y;
        }
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) {
            if (h < G) {
                float s = 0.f;
#pragma unroll
                for (int e = 0; e < DPL; ++e) s = fmaf(qr[h][e], kf[e], s);
                s = warp_sum(s) * p.scale;
                const float mn = fmaxf(m[h], s);
                const float corr = expf(m[h] - mn);
                const float pe = expf(s - mn);
                l[h] = l[h] * corr + pe;
#pragma unroll
                for (int e = 0; e < DPL; ++e) acc[h][e] = fmaf(acc[h][e], corr, pe * vf[e]);
                m[h] = mn;
            }
        }
    }
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
        if (h < G) {
            if (lane == 0) { sm_m[warp][h] = m[h]; sm_l[warp][h] = l[h]; }
#pragma unroll
            for (int e = 0; e < DPL; ++e) sm_acc[warp][h][lane * DPL + e] = acc[h][e];
        }
    }
    __syncthreads();
    const int stride = HD + 2;
    for (int idx = tid; idx < G * HD; idx += kThreads) {
        const int h = idx / HD, d = idx - h * HD;
        float M = -INFINITY;
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm_m[w][h]);
        float L = 0.f, A = 0.f;
        if (M != -INFINITY) {
            for (int w = 0; w < kWarps; ++w) {
                const float f = expf(sm_m[w][h] - M);
                L = fmaf(sm_l[w][h], f, L);
                A = fmaf(sm_acc[w][h][d], f, A);
            }
        }
        float *pr = p.part + ((size_t)(g * G + h) * p.max_split + c) * stride;
        pr[d] = A;
        if (d == 0) { pr[HD] = M; pr[HD + 1] = L; }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned old = atomicAdd(p.counter + g, 1u);
        s_flag = (old == (unsigned)nsplit - 1u);
    }
    __syncthreads();
    if (!s_flag) return;
    __threadfence();
    for (int idx = tid; idx < G * HD; idx += kThreads) {
        const int h = idx / HD, d = idx - h * HD;
        const float *base = p.part + (size_t)(g * G + h) * p.max_split * stride;
        float M = -INFINITY;
        for (int k = 0; k < nsplit; ++k) M = fmaxf(M, __ldcg(base + (size_t)k * stride + HD));
        float L = 0.f, A = 0.f;
        for (int k = 0; k < nsplit; ++k) {
            const float mk = __ldcg(base + (size_t)k * stride + HD);
            if (mk == -INFINITY) continue;
            const float f = expf(mk - M);
            L = fmaf(__ldcg(base + (size_t)k * stride + HD + 1), f, L);
            A = fmaf(__ldcg(base + (size_t)k * stride + d), f, A);
        }
        p.out[(g * G + h) * HD + d] = A / L;
    }
    if (tid == 0) p.counter[g] = 0u;
}

// ---------------------------------------------------------------------------------------------
// Utility kernels
// ---------------------------------------------------------------------------------------------
// Writes the state of a step sequence; a forced sequence takes step 0's token and position from
// its forced sources (device arrays or the small tree tables).
__global__ void k_set_state(DevState *st, const DevState init) {
    const int *src = reinterpret_cast<const int *>(&init);
    int *dst = reinterpret_cast<int *>(st);
    for (int i = threadIdx.x; i < (int)(sizeof(DevState) / sizeof(int)); i += blockDim.x) dst[i] = src[i];
    __syncthreads();
    if (threadIdx.x == 0 && init.n_forced > 0) {
        st->slot = init.slot0;
        if (init.use_small) {
            st->token = init.small_tok[0];
            st->pos = init.small_pos[0];
        } else {
            st->token = init.f_tok[0];
            st->pos = init.f_pos ? init.f_pos[0] : init.slot0;
        }
    }
}

__global__ void k_gather_rows(uint8_t *dst, const uint8_t *src, const int *src_row, int row_bytes, int dst_mul,
                              int dst_add) {
    const int r = blockIdx.x;
    const uint4 *s = reinterpret_cast<const uint4 *>(src + (size_t)src_row[r] * row_bytes);
    uint4 *d = reinterpret_cast<uint4 *>(dst + ((size_t)r * dst_mul + dst_add) * row_bytes);
    for (int i = threadIdx.x; i < row_bytes / 16; i += blockDim.x) d[i] = s[i];
}

struct CommitSlots {
    int src[kSmallNodes];
};

// One CTA per (layer, kv head, K|V); slots are copied in increasing order (a destination slot is
// never the source of a later copy because accepted node indices are increasing).
__global__ void k_kv_commit(__half *k, __half *v, int nkv, int cap, int hd, const CommitSlots slots, int n, int dst0) {
    const int lg = blockIdx.x >> 1;
    __half *base = ((blockIdx.x & 1) ? v : k) + (size_t)lg * cap * hd;
    for (int i = 0; i < n; ++i) {
        const int sidx = slots.src[i], didx = dst0 + i;
        if (sidx != didx)
            for (int d = threadIdx.x; d < hd; d += blockDim.x) base[(size_t)didx * hd + d] = base[(size_t)sidx * hd + d];
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------------------------
// Host-side launchers
// ---------------------------------------------------------------------------------------------
template <typename... KArgs, typename... Args>
static cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, const LaunchCfg &lc,
                             Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = lc.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = lc.pdl ? attr : nullptr;
    cfg.numAttrs = lc.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

void plan_gemv(GemvParams &p, int rg, int num_sms, int ring_bytes) {
    const size_t row = p.fmt == WF_F16 ? (size_t)p.K * 2 : (size_t)p.K + (size_t)(p.K / 32) * 2;
    const int nvec = p.fmt == WF_F16 ? p.K / 8 : p.K / 16;
    int R = (int)(kTargetStage / row);
    R = R / rg * rg;
    R = std::max(rg, std::min(16, R));
    int split = 1;
    if (R < kWarps) {
        split = kWarps / R;
        while (split > 1 && nvec % split) --split;
    }
    p.rows_per_chunk = R;
    p.split = split;
    p.stage_bytes = (int)((R * row + 127) / 128 * 128);
    p.stages = std::max(2, std::min(8, ring_bytes / p.stage_bytes));
    const int groups = p.N / rg;
    p.grid = std::max(1, std::min(num_sms, groups));
}

size_t gemv_smem_bytes(const GemvParams &p) {
    return (size_t)p.stages * p.stage_bytes + (size_t)p.K * 4 + 2 * kMaxTasks * 4 + (size_t)p.stages * 8;
}

template <int PRO, int EPI, int FMT>
static cudaError_t gemv_t(const GemvParams &p, const LaunchCfg *lc) {
    const size_t smem = gemv_smem_bytes(p);
    if (lc == nullptr)
        return cudaFuncSetAttribute(k_gemv<PRO, EPI, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return launch_ex(k_gemv<PRO, EPI, FMT>, dim3(p.grid), dim3(kThreads), smem, *lc, p);
}

static cudaError_t gemv_dispatch(int pro, int epi, const GemvParams &p, const LaunchCfg *lc) {
#define SP_CASE(PRO, EPI)                                                                    \
    if (pro == PRO && epi == EPI)                                                            \
        return p.fmt == WF_F16 ? gemv_t<PRO, EPI, WF_F16>(p, lc) : gemv_t<PRO, EPI, WF_I8>(p, lc);
    SP_CASE(PRO_NORM, EPI_QKV)
    SP_CASE(PRO_EMBED_NORM, EPI_QKV)
    SP_CASE(PRO_PLAIN, EPI_RESID)
    SP_CASE(PRO_NORM, EPI_SWIGLU)
    SP_CASE(PRO_NORM, EPI_LMHEAD)
#undef SP_CASE
    return cudaErrorInvalidValue;
}

cudaError_t prepare_gemv(int pro, int epi, const GemvParams &p) { return gemv_dispatch(pro, epi, p, nullptr); }

cudaError_t launch_gemv(int pro, int epi, const GemvParams &p, const LaunchCfg &lc) {
    return gemv_dispatch(pro, epi, p, &lc);
}

cudaError_t launch_attention(const AttnParams &p, const LaunchCfg &lc) {
    if (p.nh / p.nkv > kMaxGroup) return cudaErrorInvalidValue;
    const dim3 grid(p.max_split, p.nkv);
    if (p.hd == 128) return launch_ex(k_attn_decode<128>, grid, dim3(kThreads), 0, lc, p);
    if (p.hd == 64) return launch_ex(k_attn_decode<64>, grid, dim3(kThreads), 0, lc, p);
    return cudaErrorInvalidValue;
}

cudaError_t launch_set_state(DevState *st, const DevState &init, cudaStream_t s) {
    k_set_state<<<1, 128, 0, s>>>(st, init);
    return cudaGetLastError();
}

cudaError_t launch_gather_rows(uint8_t *dst, const uint8_t *src, const int *src_row, int rows, int row_bytes,
                               int dst_mul, int dst_add, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    if (row_bytes % 16) return cudaErrorInvalidValue;
    k_gather_rows<<<rows, 128, 0, s>>>(dst, src, src_row, row_bytes, dst_mul, dst_add);
    return cudaGetLastError();
}

cudaError_t launch_kv_commit(__half *k, __half *v, int layers, int nkv, int cap, int hd, const int *src_slots,
                             int n, int dst0, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    if (n > kSmallNodes) return cudaErrorInvalidValue;
    CommitSlots cs;
    for (int i = 0; i < n; ++i) cs.src[i] = src_slots[i];
    k_kv_commit<<<layers * nkv * 2, 128, 0, s>>>(k, v, nkv, cap, hd, cs, n, dst0);
    return cudaGetLastError();
}

}  // namespace sp
