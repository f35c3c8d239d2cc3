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
// (The decode attention kernel is in attention.cu, the tensor-core GEMV in gemv_tc.cu.)
#include <algorithm>
#include <climits>
#include <cmath>
#include <type_traits>
#include <utility>

#include "kernels.cuh"

namespace sp {

constexpr int kThreads = 256;            // consumer threads (8 warps) of a GEMV; other kernels' block
constexpr int kWarps = kThreads / 32;
constexpr int kGemvThreads = kThreads + 32;   // + the producer warp
constexpr int kMaxUnitsPerCta = 1024;     // bounds the per-CTA array of unit row sums (64 KB)
constexpr int kMaxStages = 16;
static_assert(kMaxStages % 8 == 0, "GEMV stage counts are multiples of the 8 consumer warps");
constexpr int kUnitTiles = 16;            // tiles per unit at most (8 KB): one warp holds them in registers

// Barrier among the 8 consumer warps of a GEMV CTA (the producer warp does not take part).
SP_DEVINL void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }

SP_DEVINL void argmax_merge(float &v, int &i, float ov, int oi) {
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
}

// D += A(16x16 fp16) . B(16x8 fp16), fp32 accumulation (tensor cores). Used as a dot-product
// engine: B column 0 holds the fp16 "hi" part of the fp32 input, column 1 the "lo" remainder,
// so y = D[:,0] + D[:,1] carries ~22 bits of the fp32 activation (products are exact).
SP_DEVINL void mma_16816(float (&d)[4], const uint4 a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

SP_DEVINL uint32_t pack_half2(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// The CTA whose unit range [floor(U*c/C), floor(U*(c+1)/C)) contains unit u.
SP_DEVINL int cta_of(int u, int U, int C) {
    int c = (int)(((long long)u * C) / U);
    while (c > 0 && (long long)U * c / C > u) --c;
    while (c + 1 < C && (long long)U * (c + 1) / C <= u) ++c;
    return c;
}

template <int PRO, int EPI, int FMT>
__global__ void __launch_bounds__(kGemvThreads) k_gemv(const GemvParams p) {
    static_assert(FMT == WF_F16, "fragment GEMV streams fp16 weights");
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_val[kWarps];
    __shared__ int s_idx[kWarps];
    __shared__ int s_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool producer = warp == kWarps;        // warp 8 issues the bulk copies
    const int S = p.stages, K = p.K, NT = p.nt, KS = p.ks;
    const int KT = K / 16;
    const int unit_bytes = NT * kTileBytes;
    const int C = gridDim.x, c = blockIdx.x;
    const int U = (p.N / 16) * KS;
    const int u0 = (int)((long long)U * c / C), u1 = (int)((long long)U * (c + 1) / C);
    const int nu = u1 - u0;
    const int upc = (U + C - 1) / C;
    uint8_t *ring = smem;
    uint32_t *xb = reinterpret_cast<uint32_t *>(smem + (size_t)S * unit_bytes);   // KT x 16 words
    float *ysm = reinterpret_cast<float *>(xb + (size_t)KT * 16);                  // upc x 16 row sums
    uint64_t *full = reinterpret_cast<uint64_t *>(ysm + (size_t)upc * 16);
    uint64_t *empty = full + S;

    unsigned long long *tr = p.trace ? p.trace + (size_t)c * kTraceWords : nullptr;
    if (tr && tid == 0) tr[0] = globaltimer();
    auto issue = [&](int i, uint64_t policy) {
        if (tr && i < kTraceUnits) tr[8 + i] = globaltimer();
        const int u = u0 + i, st_ = i % S;
        const int strip = u / KS, seg = u - strip * KS;
        const uint8_t *src = p.w + ((size_t)strip * KT + (size_t)seg * NT) * kTileBytes;
        mbar_arrive_expect_tx(&full[st_], (uint32_t)unit_bytes);
        if (p.evict_first) bulk_g2s_hint(ring + (size_t)st_ * unit_bytes, src, (uint32_t)unit_bytes, &full[st_], policy);
        else bulk_g2s(ring + (size_t)st_ * unit_bytes, src, (uint32_t)unit_bytes, &full[st_]);
    };

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    DevState *st = p.st;

    if (producer) {
        // ---- producer warp: weights do not depend on the previous kernel, so the ring is filled
        // and L2 is warmed with the weight stream further ahead before any dependency wait. ------
        if (lane == 0) {
            const uint64_t policy = p.evict_first ? policy_evict_first() : 0ull;
            for (int i = 0; i < min(S, nu); ++i) issue(i, policy);
            for (int r = 0; r < p.pf_n; ++r) {
                const unsigned long long share = (p.pf_bytes[r] / C + 15) & ~15ull;
                const unsigned long long beg = share * c;
                if (beg >= p.pf_bytes[r]) continue;
                const unsigned long long end = min(beg + share, p.pf_bytes[r]) & ~15ull;
                for (unsigned long long o = beg; o < end; o += 32768)
                    prefetch_l2(p.pf_ptr[r] + o, (uint32_t)min(32768ull, end - o));
            }
            for (int i = S; i < nu; ++i) {
                // stage i % S is free once its previous unit (i - S) has been read by its warp
                if (!mbar_wait_bounded(&empty[i % S], (uint32_t)(i / S - 1) & 1u)) {
                    atomicCAS(&st->err, 0, kErrMbarTimeout);
                    break;
                }
                issue(i, policy);
            }
        }
    } else {
        griddep_wait();
        griddep_launch_dependents();
        if (tr && tid == 0) tr[1] = globaltimer();
        // ---- prologue: fp32 input -> RMSNorm -> hi/lo fp16 B fragments in shared memory ------
        // Pass A stores the raw fp32 input at its natural index in the fragment buffer (K floats
        // fill it exactly) with coalesced loads; pass B turns each k-tile's 16 floats (64 bytes)
        // into that tile's 64-byte fragment in place: lanes 0-3 hold the fp16 "hi" column,
        // lanes 4-7 the "lo" remainder.
        float *xs = reinterpret_cast<float *>(xb);
        float ss = 0.f;
        if constexpr (PRO == PRO_EMBED_NORM) {
            int tok = st->token;
            if (tok < 0 || tok >= p.vocab) {
                if (tid == 0) atomicCAS(&st->err, 0, kErrBadToken);
                tok = 0;
            }
            const uint4 *e4 = reinterpret_cast<const uint4 *>(p.embed + (size_t)tok * K);
            for (int v = tid; v < K / 8; v += kThreads) {
                const uint4 raw = e4[v];
                const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
                float f[8];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 t2 = __half22float2(h2[j]);
                    f[2 * j] = t2.x;
                    f[2 * j + 1] = t2.y;
                }
                float4 *dst = reinterpret_cast<float4 *>(xs + 8 * v);
                dst[0] = make_float4(f[0], f[1], f[2], f[3]);
                dst[1] = make_float4(f[4], f[5], f[6], f[7]);
                if (c == 0) {
                    float4 *xi = reinterpret_cast<float4 *>(p.x_init + 8 * v);
                    xi[0] = dst[0];
                    xi[1] = dst[1];
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
            }
        } else {
            const float4 *x4 = reinterpret_cast<const float4 *>(p.xin);
            for (int v = tid; v < K / 4; v += kThreads) {
                const float4 f = x4[v];
                reinterpret_cast<float4 *>(xs)[v] = f;
                if constexpr (PRO != PRO_PLAIN) {
                    ss = fmaf(f.x, f.x, ss);
                    ss = fmaf(f.y, f.y, ss);
                    ss = fmaf(f.z, f.z, ss);
                    ss = fmaf(f.w, f.w, ss);
                }
            }
        }
        float inv = 1.f;
        if constexpr (PRO != PRO_PLAIN) {
            ss = warp_sum(ss);
            if (lane == 0) s_val[warp] = ss;
        }
        consumer_sync();
        if constexpr (PRO != PRO_PLAIN) {
            float tot = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) tot += s_val[w];
            inv = 1.0f / sqrtf(tot / (float)K + p.eps);
        }
        for (int t = tid; t < KT; t += kThreads) {
            float v[16];
            const float4 *src = reinterpret_cast<const float4 *>(xs + 16 * t);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float4 f = src[j];
                v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
            }
            if constexpr (PRO != PRO_PLAIN) {
                const float4 *g4 = reinterpret_cast<const float4 *>(p.gain + 16 * t);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 gg = g4[j];
                    v[4 * j] = (v[4 * j] * inv) * gg.x;
                    v[4 * j + 1] = (v[4 * j + 1] * inv) * gg.y;
                    v[4 * j + 2] = (v[4 * j + 2] * inv) * gg.z;
                    v[4 * j + 3] = (v[4 * j + 3] * inv) * gg.w;
                }
            }
            __half hi[16], lo[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                hi[j] = __float2half_rn(v[j]);
                lo[j] = __float2half_rn(v[j] - __half2float(hi[j]));
            }
            uint32_t wds[16];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                const int k0 = 2 * cc;
                wds[cc * 2] = pack_half2(hi[k0], hi[k0 + 1]);
                wds[cc * 2 + 1] = pack_half2(hi[k0 + 8], hi[k0 + 9]);
                wds[8 + cc * 2] = pack_half2(lo[k0], lo[k0 + 1]);
                wds[8 + cc * 2 + 1] = pack_half2(lo[k0 + 8], lo[k0 + 9]);
            }
            uint4 *dst = reinterpret_cast<uint4 *>(xb + (size_t)t * 16);
#pragma unroll
            for (int j = 0; j < 4; ++j) dst[j] = make_uint4(wds[4 * j], wds[4 * j + 1], wds[4 * j + 2], wds[4 * j + 3]);
        }
        consumer_sync();
        if (tr && tid == 0) tr[2] = globaltimer();

        // ---- stream: warp w takes units w, w+8, ... Each unit: wait for its stage, copy the
        // unit's A fragments to registers, release the stage to the producer, then run the MMAs
        // with the B fragments of the unit's k-tiles. The unit's 16 row sums land in ysm. -------
        for (int i = warp; i < nu; i += kWarps) {
            const int sidx = i % S;
            if (!mbar_wait_bounded(&full[sidx], (uint32_t)(i / S) & 1u)) {
                if (lane == 0) atomicCAS(&st->err, 0, kErrMbarTimeout);
                break;
            }
            if (tr && lane == 0 && i < kTraceUnits) tr[8 + kTraceUnits + i] = globaltimer();
            const uint8_t *stage = ring + (size_t)sidx * unit_bytes;
            uint4 af[kUnitTiles];
#pragma unroll
            for (int q = 0; q < kUnitTiles; ++q)
                af[q] = q < NT ? *reinterpret_cast<const uint4 *>(stage + (size_t)q * kTileBytes + lane * 16)
                               : make_uint4(0u, 0u, 0u, 0u);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[sidx]);
            const int seg = (u0 + i) % KS;
            const uint32_t *xw = xb + (size_t)seg * NT * 16;
            float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int q = 0; q < kUnitTiles; q += 2) {
                if (q < NT) {
                    uint2 b = make_uint2(0u, 0u);
                    if (lane < 8) b = *reinterpret_cast<const uint2 *>(xw + q * 16 + lane * 2);
                    mma_16816(d0, af[q], b.x, b.y);
                }
                if (q + 1 < NT) {
                    uint2 b = make_uint2(0u, 0u);
                    if (lane < 8) b = *reinterpret_cast<const uint2 *>(xw + (q + 1) * 16 + lane * 2);
                    mma_16816(d1, af[q + 1], b.x, b.y);
                }
            }
            if ((lane & 3) == 0) {
                ysm[i * 16 + (lane >> 2)] = (d0[0] + d0[1]) + (d1[0] + d1[1]);
                ysm[i * 16 + (lane >> 2) + 8] = (d0[2] + d0[3]) + (d1[2] + d1[3]);
            }
        }
    }
    __syncthreads();
    if (tr && tid == 0) tr[3] = globaltimer();
    if (producer) return;

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
    const int half_hd = p.hd / 2;

    // ---- epilogues: every strip this CTA touched, 16 rows per half-warp -----------------------
    // Units of one strip are summed in unit order. A strip whose units all lie in this CTA is
    // finished here; a strip shared with neighbouring CTAs (at most the first and the last) posts
    // its contribution and the last contributor sums all of them in segment order.
    const int sA = u0 / KS, sB = (u1 - 1) / KS;
    const int rows_here = (sB - sA + 1) * 16;
    const unsigned half_mask = 0xffffu << (lane & 16);
    for (int base = 0; base < rows_here; base += kThreads) {
        const int t = base + tid;
        if (t >= rows_here) continue;       // whole half-warps drop out together
        const int r = t & 15, strip = sA + (t >> 4);
        const int ua = max(u0, strip * KS), ub = min(u1, (strip + 1) * KS);
        float y = 0.f;
        for (int u = ua; u < ub; ++u) y += ysm[(u - u0) * 16 + r];
        if (ua != strip * KS || ub != (strip + 1) * KS) {
            float *slot = p.partial + ((size_t)strip * KS + (ua - strip * KS)) * 16;
            slot[r] = y;
            __threadfence();
            __syncwarp(half_mask);
            unsigned last = 0;
            if (r == 0) {
                const int need = cta_of(strip * KS + KS - 1, U, C) - cta_of(strip * KS, U, C) + 1;
                last = atomicAdd(p.strip_cnt + strip, 1u) == (unsigned)(need - 1);
            }
            last = __shfl_sync(half_mask, last, lane & 16);
            if (!last) continue;
            __threadfence();
            float* all = p.partial + (size_t)strip * KS * 16;
            y = 0.f;
            for (int k2 = 0; k2 < KS; ++k2) {
                y += __ldcg(all + k2 * 16 + r);
                all[k2 * 16 + r] = 0.f;      // leave the slots zeroed for the next launch
            }
            if (r == 0) p.strip_cnt[strip] = 0u;
        }
        const int row = strip * 16 + r;
        const float other = __shfl_xor_sync(half_mask, y, 1);   // pair partner (row ^ 1)
        if constexpr (EPI == EPI_RESID) {
            p.out[row] = p.out[row] + y;
        } else if constexpr (EPI == EPI_LMHEAD) {
            if (row < p.n_valid) {
                if (lg) lg[row] = y;
                if (y > bv) { bv = y; bi = row; }
            }
        } else if constexpr (EPI == EPI_SWIGLU) {
            if ((r & 1) == 0) p.out[row / 2] = (y / (1.0f + expf(-y))) * other;
        } else {  // EPI_QKV: packed rows (2q, 2q+1) are dims (d, d + hd/2) of one head
            if ((r & 1) == 0) {
                const int P = row / 2;
                const int hh = P / half_hd, dd = P - hh * half_hd;
                const int lo = hh * p.hd + dd, hi = lo + half_hd;
                const float y0 = y + p.bias[lo], y1 = other + p.bias[hi];
                if (hh < p.nh + p.nkv) {
                    const float cs = p.rope[((size_t)pos * half_hd + dd) * 2];
                    const float sn = p.rope[((size_t)pos * half_hd + dd) * 2 + 1];
                    const float o0 = __fadd_rn(__fmul_rn(y0, cs), -__fmul_rn(y1, sn));
                    const float o1 = __fadd_rn(__fmul_rn(y1, cs), __fmul_rn(y0, sn));
                    if (hh < p.nh) {
                        p.out[lo] = o0;
                        p.out[hi] = o1;
                    } else {
                        __half *kr = p.kc + ((size_t)(hh - p.nh) * p.cap + slot) * p.hd;
                        kr[dd] = __float2half_rn(o0);
                        kr[dd + half_hd] = __float2half_rn(o1);
                    }
                } else {
                    __half *vr = p.vc + ((size_t)(hh - p.nh - p.nkv) * p.cap + slot) * p.hd;
                    vr[dd] = __float2half_rn(y0);
                    vr[dd + half_hd] = __float2half_rn(y1);
                }
            }
        }
    }

    if (tr) {
        consumer_sync();
        if (tid == 0) tr[4] = globaltimer();
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
        consumer_sync();
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
        consumer_sync();
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
        consumer_sync();
        if (lane == 0) { s_val[warp] = v; s_idx[warp] = ix; }
        consumer_sync();
        if (tid == 0) {
            for (int w = 1; w < kWarps; ++w) argmax_merge(s_val[0], s_idx[0], s_val[w], s_idx[w]);
            int tok = s_idx[0];
            if (tok < 0 || tok >= p.n_valid) {
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

// One warp per 16x16 tile; lane l writes its A-fragment registers a0..a3 (16 bytes):
// a0 = (row g, cols 2c, 2c+1), a1 = (row g+8, same cols), a2 = (row g, cols 2c+8, 2c+9), a3 = (row g+8, ...),
// with g = l/4, c = l%4 (the mma.m16n8k16 row-major A layout).
__global__ void k_pack_fragments(uint8_t *dst, const __half *a, int rows_a, const __half *b, const int *row_of,
                                 int N, int K) {
    const int KT = K / 16;
    const long long tile = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (tile >= (long long)(N / 16) * KT) return;
    const int lane = threadIdx.x & 31, g = lane >> 2, cc = lane & 3;
    const int s = (int)(tile / KT), t = (int)(tile % KT);
    auto row_ptr = [&](int r) -> const __half * {
        const int src = row_of[r];
        if (src < 0) return nullptr;
        return src < rows_a ? a + (size_t)src * K : b + (size_t)(src - rows_a) * K;
    };
    auto pair = [](const __half *row, int k) -> uint32_t {
        return row ? *reinterpret_cast<const uint32_t *>(row + k) : 0u;
    };
    const __half *r0 = row_ptr(16 * s + g), *r1 = row_ptr(16 * s + g + 8);
    const int k0 = 16 * t + 2 * cc;
    uint4 v;
    v.x = pair(r0, k0);
    v.y = pair(r1, k0);
    v.z = pair(r0, k0 + 8);
    v.w = pair(r1, k0 + 8);
    *reinterpret_cast<uint4 *>(dst + ((size_t)tile * 32 + lane) * 16) = v;
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

// Units per CTA the busiest CTA streams.
static long long max_units_per_cta(long long U, long long C) { return (U + C - 1) / C; }

void plan_gemv(GemvParams &p, int num_sms, int ring_bytes, int max_unit_bytes) {
    // A unit is one warp's work item: the largest divisor of K/16 up to kUnitTiles tiles (8 KB),
    // so a 12-deep ring of units keeps ~96 KB per SM in flight; units are spread evenly over
    // one CTA per SM.
    (void)max_unit_bytes;
    const int KT = p.K / 16, strips = p.N / 16;
    p.nt = 1;
    for (int nt = std::min(KT, kUnitTiles); nt >= 1; --nt)
        if (KT % nt == 0) { p.nt = nt; break; }
    p.ks = KT / p.nt;
    const long long U = (long long)strips * p.ks;
    p.grid = (int)std::min<long long>(num_sms, U);
    // Unit i lives in stage i % S and is consumed by warp i % 8. S must be a multiple of 8 so a
    // stage is always consumed by the same warp, in order: a warp then never waits on a stage's
    // full barrier more than one phase ahead (a parity wait cannot tell phase k+1 from k-1).
    const int fit = std::min(kMaxStages, ring_bytes / (p.nt * kTileBytes));
    p.stages = std::max(kWarps, fit / kWarps * kWarps);
}

size_t gemv_smem_bytes(const GemvParams &p) {
    const long long U = (long long)(p.N / 16) * p.ks;
    const size_t upc = (size_t)max_units_per_cta(U, p.grid);
    return (size_t)p.stages * p.nt * kTileBytes + (size_t)(p.K / 16) * 64 + upc * 16 * 4 + (size_t)p.stages * 16;
}

template <int PRO, int EPI, int FMT>
static cudaError_t gemv_t(const GemvParams &p, const LaunchCfg *lc) {
    const size_t smem = gemv_smem_bytes(p);
    if (lc == nullptr) {
        // One instantiation serves several matrices (O and down): only ever raise its opt-in.
        cudaFuncAttributes fa;
        cudaError_t e = cudaFuncSetAttribute(k_gemv<PRO, EPI, FMT>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                             (int)cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        e = cudaFuncGetAttributes(&fa, k_gemv<PRO, EPI, FMT>);
        if (e != cudaSuccess) return e;
        if ((size_t)fa.maxDynamicSharedSizeBytes >= smem) return cudaSuccess;
        return cudaFuncSetAttribute(k_gemv<PRO, EPI, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    }
    return launch_ex(k_gemv<PRO, EPI, FMT>, dim3(p.grid), dim3(kGemvThreads), smem, *lc, p);
}

static cudaError_t gemv_dispatch(int pro, int epi, const GemvParams &p, const LaunchCfg *lc) {
    if (p.stages % kWarps || p.stages > kMaxStages || p.nt > kUnitTiles) return cudaErrorInvalidValue;
#define SP_CASE(PRO, EPI)                                                                    \
    if (pro == PRO && epi == EPI)                                                            \
        return p.fmt == WF_F16 ? gemv_t<PRO, EPI, WF_F16>(p, lc) : cudaErrorNotSupported;
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

cudaError_t launch_pack_fragments(uint8_t *dst, const __half *a, int rows_a, const __half *b, const int *row_of,
                                  int N, int K, cudaStream_t s) {
    if (N % 16 || K % 16) return cudaErrorInvalidValue;
    const long long tiles = (long long)(N / 16) * (K / 16);
    const int per_block = 8;
    k_pack_fragments<<<(unsigned)((tiles + per_block - 1) / per_block), per_block * 32, 0, s>>>(dst, a, rows_a, b, row_of,
                                                                                            N, K);
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
