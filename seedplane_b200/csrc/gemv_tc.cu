// Weight-streaming GEMV on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// y = W . in(x) for one token. W is packed in HBM in the canonical K-major, non-swizzled UMMA
// layout, as tiles of 128 rows x 16 inputs (4 KB): tile (strip s, k-tile t) lives at
// (s * K/16 + t) * 4096, and inside a tile the 8-row x 16-byte core matrix (r, h) (rows 8r..8r+7,
// inputs 16t+8h..+7) is at (2r + h) * 128 -- so LBO = 128 B (K direction) and SBO = 256 B (M).
//
// The activation is the B operand of an M=128, N=8, K=16 tcgen05.mma: row 0 holds the fp16
// rounding of the fp32 input ("hi"), row 1 the fp16 rounding of the remainder ("lo"), rows 2-7
// are zero, and the fp32 accumulator in TMEM gives y = D[:,0] + D[:,1] with ~22 bits of the
// activation (fp16 x fp16 products are exact). The tensor core reads both operands straight from
// shared memory, so the SMs issue almost no instructions per weight byte.
//
// Roles (192 threads): warps 0-3 build the B operand and run the epilogues (one TMEM lane = one
// row each), warp 4 streams the CTA's tiles through a ring of 16 KB stages with 1-D bulk copies
// (started before the programmatic-dependent-launch wait: weights do not depend on the previous
// kernel), warp 5 allocates TMEM and issues the MMAs (one thread). Each CTA owns a contiguous
// range of tiles, split at strip boundaries into items with one 8-column TMEM accumulator each;
// a strip split between CTAs is summed by its last contributor in fixed order.
#include <algorithm>
#include <climits>
#include <cmath>

#include "kernels.cuh"
#include "tc.cuh"

namespace sp {

namespace {

constexpr int kTcWarps = 6;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kEpiThreads = 128;          // warps 0-3: TMEM lanes 0-127
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kTcStageTiles = 4;          // 16 KB per stage
constexpr int kTcStageBytes = kTcStageTiles * kTcTileBytes;
constexpr int kTcMaxItems = 16;           // TMEM accumulators per CTA (8 columns each)
constexpr int kTcTmemCols = kTcMaxItems * 8;
constexpr int kMaxPairs = 4;              // B pairs (k-tile, half) per prologue thread: K/8 <= 512

SP_DEVINL void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory"); }
// warps 0-3 + the MMA warp: the B operand is ready
SP_DEVINL void bready_sync() { asm volatile("bar.sync 2, %0;" ::"n"(kEpiThreads + 32) : "memory"); }

}  // namespace

template <int PRO, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1) k_gemv_tc(const TcGemvParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint32_t s_tmem;
    __shared__ float s_val[4];
    __shared__ int s_idx[4];
    __shared__ int s_flag;
    __shared__ int it_strip[kTcMaxItems], it_a[kTcMaxItems], it_b[kTcMaxItems], it_boff[kTcMaxItems];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = p.K, KT = K / 16;
    const int C = gridDim.x, c = blockIdx.x;
    const long long T = (long long)(p.N / 128) * KT;
    const long long g0 = T * c / C, g1 = T * (c + 1) / C;
    const int ntiles = (int)(g1 - g0);
    const int nstage = (ntiles + kTcStageTiles - 1) / kTcStageTiles;
    const int S = p.stages;
    uint8_t *ring = smem;
    uint8_t *bbuf = smem + (size_t)S * kTcStageBytes;                      // B operand, 256 B per k-tile
    uint64_t *full = reinterpret_cast<uint64_t *>(bbuf + (size_t)p.b_tiles * 256);
    uint64_t *empty = full + S;
    uint64_t *accf = empty + S;
    DevState *st = p.st;
    unsigned long long *tr = p.trace ? p.trace + (size_t)c * kTraceWords : nullptr;
    if (tr && tid == 0) tr[0] = globaltimer();

    // Items: the CTA's tiles split at strip boundaries (at most kTcMaxItems, checked on the host).
    int nitems = 0;
    if (tid == 0) {
        long long g = g0;
        int boff = 0;
        while (g < g1 && nitems < kTcMaxItems) {
            const int s = (int)(g / KT), a = (int)(g % KT);
            const long long rest = (long long)a + (g1 - g);
            const int b = rest < KT ? (int)rest : KT;
            it_strip[nitems] = s;
            it_a[nitems] = a;
            it_b[nitems] = b;
            it_boff[nitems] = p.b_full ? a : boff;     // B tile index of the item's first k-tile
            boff += b - a;
            g += b - a;
            ++nitems;
        }
        s_flag = nitems;
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < kTcMaxItems; ++i) mbar_init(&accf[i], 1);
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kTcTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    nitems = s_flag;
    const uint32_t tmem = s_tmem;

    if (warp == kProducerWarp) {
        // ---- producer: fill the ring and warm L2 further ahead, before any dependency wait ----
        if (lane == 0) {
            auto issue = [&](int i) {
                if (tr && i < kTraceUnits) tr[8 + i] = globaltimer();
                const int s = i % S;
                const int n = min((int)kTcStageTiles, ntiles - i * (int)kTcStageTiles);
                mbar_arrive_expect_tx(&full[s], (uint32_t)(n * kTcTileBytes));
                bulk_g2s(ring + (size_t)s * kTcStageBytes, p.w + (size_t)(g0 + (long long)i * kTcStageTiles) * kTcTileBytes,
                         (uint32_t)(n * kTcTileBytes), &full[s]);
            };
            for (int i = 0; i < min(S, nstage); ++i) issue(i);
            for (int r = 0; r < p.pf_n; ++r) {
                const unsigned long long share = (p.pf_bytes[r] / C + 15) & ~15ull;
                const unsigned long long beg = share * c;
                if (beg >= p.pf_bytes[r]) continue;
                const unsigned long long end = min(beg + share, p.pf_bytes[r]) & ~15ull;
                for (unsigned long long o = beg; o < end; o += 32768)
                    prefetch_l2(p.pf_ptr[r] + o, (uint32_t)min(32768ull, end - o));
            }
            for (int i = S; i < nstage; ++i) {
                if (!mbar_wait_bounded(&empty[i % S], (uint32_t)(i / S - 1) & 1u)) {
                    atomicCAS(&st->err, 0, kErrMbarTimeout);
                    break;
                }
                issue(i);
            }
        }
    } else if (warp == kMmaWarp) {
        // ---- MMA issuer: one thread walks the tiles in order ----------------------------------
        bready_sync();
        tc_fence_after();
        if (lane == 0) {
            // Walk the tiles with running (item, k-tile) counters: no division on the issue path.
            const uint32_t ring_addr = smem_u32(ring), b_addr = smem_u32(bbuf);
            int item = 0, t = it_a[0];
            uint32_t b_tile = (uint32_t)it_boff[0];      // B tile of the current k-tile
            int s = 0, par = 0;
            for (int i = 0; i < nstage; ++i) {
                if (!mbar_wait_bounded(&full[s], (uint32_t)par)) {
                    atomicCAS(&st->err, 0, kErrMbarTimeout);
                    break;
                }
                tc_fence_after();
                if (tr && i < kTraceUnits) tr[8 + kTraceUnits + i] = globaltimer();
                const int n = min((int)kTcStageTiles, ntiles - i * (int)kTcStageTiles);
                uint32_t a_addr = ring_addr + (uint32_t)(s * kTcStageBytes);
                for (int q = 0; q < n; ++q) {
                    const uint64_t ad = smem_desc(a_addr, 128, 256);
                    const uint64_t bd = smem_desc(b_addr + b_tile * 256u, 128, 256);
                    mma_f16(tmem + (uint32_t)(item * 8), ad, bd, t != it_a[item] ? 1u : 0u);
                    a_addr += kTcTileBytes;
                    ++t;
                    ++b_tile;
                    if (t == it_b[item]) {                      // accumulator complete
                        mma_commit(&accf[item]);
                        if (item + 1 < nitems) {
                            ++item;
                            t = it_a[item];
                            b_tile = (uint32_t)it_boff[item];
                        }
                    }
                }
                mma_commit(&empty[s]);   // the stage is free once these MMAs have read it
                if (++s == S) {
                    s = 0;
                    par ^= 1;
                }
            }
        }
        __syncwarp();
    } else {
        // ---- warps 0-3: input vector -> B operand (rows hi / lo / 0 x 6) ----------------------
        // One L2 round trip: every thread first loads the 8 inputs (and 8 norm gains) of each of
        // its B "pairs" (k-tile, half), plus, when the B operand covers only part of K, its share
        // of the whole vector for the RMSNorm sum of squares; then one reduction, then the fp16
        // hi / lo rows are built from registers.
        griddep_wait();
        griddep_launch_dependents();
        if (tr && tid == 0) tr[1] = globaltimer();
        const __half *erow = nullptr;
        if constexpr (PRO == PRO_EMBED_NORM) {
            int tok = st->token;
            if (tok < 0 || tok >= p.vocab) {
                if (tid == 0) atomicCAS(&st->err, 0, kErrBadToken);
                tok = 0;
            }
            erow = p.embed + (size_t)tok * K;
        }
        const int nb = p.b_full ? KT : ntiles;
        const int npairs = nb * 2;
        float v[kMaxPairs][8];
        float ss = 0.f;
#pragma unroll
        for (int q = 0; q < kMaxPairs; ++q) {
            const int idx = tid + q * kEpiThreads;
            if (idx < npairs) {
                const int bt = idx >> 1, h = idx & 1;
                int t = bt;                                  // k-tile of this B tile
                if (!p.b_full) {
                    int j = 0;
                    while (j + 1 < nitems && bt >= it_boff[j + 1]) ++j;
                    t = it_a[j] + (bt - it_boff[j]);
                }
                const int k0 = 16 * t + 8 * h;
                if constexpr (PRO == PRO_EMBED_NORM) {
                    const uint4 raw = *reinterpret_cast<const uint4 *>(erow + k0);
                    const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 t2 = __half22float2(h2[j]);
                        v[q][2 * j] = t2.x;
                        v[q][2 * j + 1] = t2.y;
                    }
                } else {
                    const float4 x0 = *reinterpret_cast<const float4 *>(p.xin + k0);
                    const float4 x1 = *reinterpret_cast<const float4 *>(p.xin + k0 + 4);
                    v[q][0] = x0.x; v[q][1] = x0.y; v[q][2] = x0.z; v[q][3] = x0.w;
                    v[q][4] = x1.x; v[q][5] = x1.y; v[q][6] = x1.z; v[q][7] = x1.w;
                }
                if (PRO != PRO_PLAIN && p.b_full) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) ss = fmaf(v[q][j], v[q][j], ss);
                }
            }
        }
        if constexpr (PRO != PRO_PLAIN) {
            if (!p.b_full || (PRO == PRO_EMBED_NORM && c == 0)) {
                // the whole vector: sum of squares (B covers part of K) and / or the residual init
                if constexpr (PRO == PRO_EMBED_NORM) {
                    const uint4 *e4 = reinterpret_cast<const uint4 *>(erow);
                    for (int vv = tid; vv < K / 8; vv += kEpiThreads) {
                        const uint4 raw = e4[vv];
                        const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
                        float f[8];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float2 t2 = __half22float2(h2[j]);
                            f[2 * j] = t2.x;
                            f[2 * j + 1] = t2.y;
                        }
                        if (c == 0) {
                            float4 *xi = reinterpret_cast<float4 *>(p.x_init + 8 * vv);
                            xi[0] = make_float4(f[0], f[1], f[2], f[3]);
                            xi[1] = make_float4(f[4], f[5], f[6], f[7]);
                        }
                        if (!p.b_full) {
#pragma unroll
                            for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
                        }
                    }
                } else {
                    const float4 *x4 = reinterpret_cast<const float4 *>(p.xin);
                    for (int vv = tid; vv < K / 4; vv += kEpiThreads) {
                        const float4 f = x4[vv];
                        ss = fmaf(f.x, f.x, ss);
                        ss = fmaf(f.y, f.y, ss);
                        ss = fmaf(f.z, f.z, ss);
                        ss = fmaf(f.w, f.w, ss);
                    }
                }
            }
        }
        float inv = 1.f;
        if constexpr (PRO != PRO_PLAIN) {
            ss = warp_sum(ss);
            if (tr && tid == 0) tr[5] = globaltimer();
            if (lane == 0) s_val[warp] = ss;
            epi_sync();
            if (tr && tid == 0) tr[6] = globaltimer();
            inv = 1.0f / sqrtf((s_val[0] + s_val[1] + s_val[2] + s_val[3]) / (float)K + p.eps);
        }
#pragma unroll
        for (int q = 0; q < kMaxPairs; ++q) {
            const int idx = tid + q * kEpiThreads;
            if (idx < npairs) {
                const int bt = idx >> 1, h = idx & 1;
                if constexpr (PRO != PRO_PLAIN) {
                    int t = bt;
                    if (!p.b_full) {
                        int j = 0;
                        while (j + 1 < nitems && bt >= it_boff[j + 1]) ++j;
                        t = it_a[j] + (bt - it_boff[j]);
                    }
                    const int k0 = 16 * t + 8 * h;
                    const float4 ga = *reinterpret_cast<const float4 *>(p.gain + k0);
                    const float4 gb = *reinterpret_cast<const float4 *>(p.gain + k0 + 4);
                    const float gg[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
                    for (int j = 0; j < 8; ++j) v[q][j] = (v[q][j] * inv) * gg[j];
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
                uint4 *core = reinterpret_cast<uint4 *>(bbuf + (size_t)bt * 256 + h * 128);
                core[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                core[1] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
#pragma unroll
                for (int r = 2; r < 8; ++r) core[r] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        fence_proxy_async_smem();   // generic-proxy writes -> visible to the tensor core
        bready_sync();
        if (tr && tid == 0) tr[2] = globaltimer();
    }

    if (warp >= 4) {
        // producer and MMA warps are done; wait for the epilogue, then release TMEM
        __syncthreads();
        if (warp == kMmaWarp) {
            tc_fence_after();
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols));
        }
        return;
    }

    // ---- epilogues (warps 0-3): thread = row (TMEM lane) of the item's strip -------------------
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
    for (int j = 0; j < nitems; ++j) {
        const bool ok = mbar_wait_bounded(&accf[j], 0u);
        if (!ok) {
            if (tid == 0) atomicCAS(&st->err, 0, kErrMbarTimeout);
            break;
        }
        tc_fence_after();
        float v[8];
        tmem_ld8(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(j * 8), v);
        float y = v[0] + v[1];
        const int strip = it_strip[j];
        if (it_a[j] != 0 || it_b[j] != KT) {
            // strip shared with other CTAs: post this contribution, the last one sums them all
            const long long first = (long long)strip * KT;
            const int cf = tc_cta_of(first, T, C), cl = tc_cta_of(first + KT - 1, T, C);
            float *slotp = p.partial + ((size_t)strip * p.max_contrib + (c - cf)) * 128;
            slotp[tid] = y;
            __threadfence();
            epi_sync();
            if (tid == 0) s_flag = atomicAdd(p.strip_cnt + strip, 1u) == (unsigned)(cl - cf);
            epi_sync();
            if (!s_flag) continue;
            __threadfence();
            const float *all = p.partial + (size_t)strip * p.max_contrib * 128;
            y = 0.f;
            for (int k2 = 0; k2 <= cl - cf; ++k2) y += __ldcg(all + (size_t)k2 * 128 + tid);
            if (tid == 0) p.strip_cnt[strip] = 0u;
        }
        const int row = strip * 128 + tid;
        const float other = __shfl_xor_sync(0xffffffffu, y, 1);   // pair partner (row ^ 1)
        if (row >= p.n_valid) continue;
        if constexpr (EPI == EPI_RESID) {
            p.out[row] = p.out[row] + y;
        } else if constexpr (EPI == EPI_LMHEAD) {
            if (lg) lg[row] = y;
            if (y > bv) { bv = y; bi = row; }
        } else if constexpr (EPI == EPI_SWIGLU) {
            if ((row & 1) == 0) p.out[row / 2] = (y / (1.0f + expf(-y))) * other;
        } else {  // EPI_QKV: packed rows (2q, 2q+1) are dims (d, d + hd/2) of one head
            if ((row & 1) == 0) {
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
    tc_fence_before();
    if (tr && tid == 0) tr[3] = globaltimer();

    if constexpr (EPI == EPI_LMHEAD) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            tc_argmax_merge(bv, bi, ov, oi);
        }
        if (lane == 0) { s_val[warp] = bv; s_idx[warp] = bi; }
        epi_sync();
        if (tid == 0) {
            float v = s_val[0];
            int ix = s_idx[0];
            for (int w = 1; w < 4; ++w) tc_argmax_merge(v, ix, s_val[w], s_idx[w]);
            p.part_val[c] = v;
            p.part_idx[c] = ix;
            __threadfence();
            s_flag = atomicAdd(p.counter, 1u) == (unsigned)C - 1u;
        }
        epi_sync();
        if (s_flag) {
            __threadfence();
            float v = -INFINITY;
            int ix = INT_MAX;
            for (int j = tid; j < C; j += kEpiThreads) tc_argmax_merge(v, ix, __ldcg(p.part_val + j), __ldcg(p.part_idx + j));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, v, o);
                const int oi = __shfl_xor_sync(0xffffffffu, ix, o);
                tc_argmax_merge(v, ix, ov, oi);
            }
            epi_sync();
            if (lane == 0) { s_val[warp] = v; s_idx[warp] = ix; }
            epi_sync();
            if (tid == 0) {
                for (int w = 1; w < 4; ++w) tc_argmax_merge(s_val[0], s_idx[0], s_val[w], s_idx[w]);
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
    if (tr && tid == 0) tr[4] = globaltimer();
    __syncthreads();    // TMEM reads are done (fenced above); the MMA warp may deallocate
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
void plan_gemv_tc(TcGemvParams &p, int num_sms, int ring_bytes, int b_budget_bytes) {
    const int KT = p.K / 16;
    const long long T = (long long)(p.N / 128) * KT;
    p.grid = (int)std::min<long long>(num_sms, T);
    const long long per = (T + p.grid - 1) / p.grid;           // tiles of the busiest CTA
    // B operand: the whole K when a CTA can cover a full strip (and it fits), else the CTA's tiles.
    p.b_full = (per >= KT && (long long)KT * 256 <= b_budget_bytes) ? 1 : 0;
    if (per >= KT && !p.b_full) p.b_full = 1;                  // rejected later by the smem check
    p.b_tiles = p.b_full ? KT : (int)per;
    p.stages = std::max(2, std::min(8, ring_bytes / kTcStageBytes));
    // strips split between CTAs: at most ceil(KT / min tiles per CTA) + 1 contributors
    const long long minper = std::max<long long>(1, T / p.grid);
    p.max_contrib = (int)((KT + minper - 1) / minper + 1);
    p.max_items = (int)(per / KT + 2);
}

int gemv_tc_max_pairs() { return kMaxPairs * kEpiThreads; }

size_t gemv_tc_smem_bytes(const TcGemvParams &p) {
    return (size_t)p.stages * kTcStageBytes + (size_t)p.b_tiles * 256 + (size_t)(2 * p.stages + kTcMaxItems) * 8;
}

int gemv_tc_max_items() { return kTcMaxItems; }

template <int PRO, int EPI>
static cudaError_t gemv_tc_t(const TcGemvParams &p, const LaunchCfg *lc) {
    const size_t smem = gemv_tc_smem_bytes(p);
    if (lc == nullptr) {
        cudaError_t e = cudaFuncSetAttribute(k_gemv_tc<PRO, EPI>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                             (int)cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        cudaFuncAttributes fa;
        e = cudaFuncGetAttributes(&fa, k_gemv_tc<PRO, EPI>);
        if (e != cudaSuccess) return e;
        if ((size_t)fa.maxDynamicSharedSizeBytes >= smem) return cudaSuccess;
        return cudaFuncSetAttribute(k_gemv_tc<PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = lc->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = lc->pdl ? attr : nullptr;
    cfg.numAttrs = lc->pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_gemv_tc<PRO, EPI>, p);
}

static cudaError_t gemv_tc_dispatch(int pro, int epi, const TcGemvParams &p, const LaunchCfg *lc) {
    if (p.max_items > kTcMaxItems || p.N % 128 || p.K % 16 || p.b_tiles * 2 > kMaxPairs * kEpiThreads)
        return cudaErrorInvalidValue;
#define SP_CASE(PRO, EPI) \
    if (pro == PRO && epi == EPI) return gemv_tc_t<PRO, EPI>(p, lc);
    SP_CASE(PRO_NORM, EPI_QKV)
    SP_CASE(PRO_EMBED_NORM, EPI_QKV)
    SP_CASE(PRO_PLAIN, EPI_RESID)
    SP_CASE(PRO_NORM, EPI_SWIGLU)
    SP_CASE(PRO_NORM, EPI_LMHEAD)
#undef SP_CASE
    return cudaErrorInvalidValue;
}

cudaError_t prepare_gemv_tc(int pro, int epi, const TcGemvParams &p) { return gemv_tc_dispatch(pro, epi, p, nullptr); }
cudaError_t launch_gemv_tc(int pro, int epi, const TcGemvParams &p, const LaunchCfg &lc) {
    return gemv_tc_dispatch(pro, epi, p, &lc);
}

// Pack an fp16 matrix into 128 x 16 tiles of canonical K-major core matrices. One thread per
// 16-byte core row: row i of core (r, h) of tile (s, t) holds W[128s + 8r + i][16t + 8h .. +7].
__global__ void k_pack_tc(uint8_t *dst, const __half *a, int rows_a, const __half *b, const int *row_of, int N, int K) {
    const int KT = K / 16;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;   // 16-byte row index
    const long long total = (long long)N * K / 8;
    if (idx >= total) return;
    const long long tile = idx >> 8;             // 256 rows of 16 B per 4 KB tile
    const int within = (int)(idx & 255);
    const int core = within >> 3, i = within & 7;
    const int r = core >> 1, h = core & 1;
    const int s = (int)(tile / KT), t = (int)(tile % KT);
    const int row = 128 * s + 8 * r + i;
    const int src = row_of[row];
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (src >= 0) {
        const __half *rp = src < rows_a ? a + (size_t)src * K : b + (size_t)(src - rows_a) * K;
        v = *reinterpret_cast<const uint4 *>(rp + 16 * t + 8 * h);
    }
    *reinterpret_cast<uint4 *>(dst + (size_t)idx * 16) = v;
}

cudaError_t launch_pack_tc(uint8_t *dst, const __half *a, int rows_a, const __half *b, const int *row_of, int N, int K,
                           cudaStream_t s) {
    if (N % 128 || K % 16) return cudaErrorInvalidValue;
    const long long total = (long long)N * K / 8;
    k_pack_tc<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(dst, a, rows_a, b, row_of, N, K);
    return cudaGetLastError();
}

}  // namespace sp
