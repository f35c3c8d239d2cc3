// Multi-column GEMM of the batched pass (prompt chunks and tree verification) on the 5th-generation
// tensor cores, sm_100a.
//
//   Y[t][n] = alpha * sum_k W[n][k] * x[t][k]        t < T tokens, n < N rows, k < K inputs
//
// W is a row-major fp16 matrix (or two: W = hi + lo, the exact halves of dequantized int8 weights);
// x is given as two fp16 row sets, hi = fp16(x) and lo = fp16(x - hi), which carry ~22 bits of the
// fp32 activation against the fp16 weights (the decode step's precision). Swap-AB: the weights are
// the M = 128 operand A, the tokens the N operand B, with the hi rows of TN tokens followed by their
// lo rows (N = 2 TN <= 256 columns); D[n][t] + D[n][TN + t] is the product.
//
//   warp 4   producer: TMA (cp.async.bulk.tensor.2d, 128-byte swizzle, no multicast) of a 128 x 64
//            weight tile and the 2 x TN x 64 token tile of every k-block into a ring of stages
//   warp 5   allocates TMEM and issues tcgen05.mma (M 128, N 2 TN, K 16; four per k-block) into one
//            of two accumulators, commits each stage back to the producer and each finished
//            accumulator to the epilogue
//   warps 6-9  int8 weights only: each k-block's int8 tile and block scales into fp16 hi / lo tiles
//   warps 0-3  epilogue: tcgen05.ld of the hi / lo columns and the fused epilogue of the op: store,
//            residual add, SwiGLU of interleaved gate / up rows written as the down projection's
//            fp16 hi / lo input, or QKV bias + RoPE + K/V cache write
//
// Work: tiles of 128 rows x TN tokens, each over K in k-blocks of 64 inputs. With enough tiles to
// keep half the SMs busy, every CTA takes whole tiles in turn (thread = output row, accumulators
// double-buffered so a tile's epilogue overlaps the next tile's MMAs). Otherwise (the small
// projections of a verify pass) each tile goes to a thread-block cluster of cs CTAs that split its
// k-blocks: every CTA leaves its partial sums in its own shared memory, the cluster meets at a
// barrier, and CTA r adds the cs partials of rows [r 128 / cs, (r + 1) 128 / cs) in rank order
// through distributed shared memory and runs the epilogue on them. No global workspace, no atomics,
// the same result whichever CTA finishes first. Every mbarrier wait is bounded; an expired wait
// records kErrMbarTimeout in DevState::err and the CTA stops waiting (the cluster barriers still
// complete: every thread reaches them).
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "kernels.cuh"
#include "tc.cuh"

namespace sp {

namespace {

constexpr int kMcConvWarps = 4;         // int8 weights: dequantization warps (8 measured no faster)
constexpr int kMcConvThreads = 32 * kMcConvWarps;
constexpr int kMcThreads = 192 + kMcConvThreads;   // warps 0-3 epilogue, 4 producer, 5 MMA, 6.. dequantization
constexpr int kMcThreadsF16 = 192;      // fp16 weights: no dequantization warps
constexpr int kMcConv0 = 6;
constexpr int kMcEpiThreads = 128;
constexpr int kMcProducer = 4;
constexpr int kMcMma = 5;
constexpr int kBK = 64;                  // inputs per k-block: one 128-byte swizzle row of fp16
constexpr int kBM = 128;
constexpr int kATileBytes = kBM * kBK * 2;
constexpr int kI8TileBytes = kBM * kBK;  // an int8 weight tile (rows of 64 bytes, no swizzle)
constexpr int kABufs = 2;                // int8 weights: fp16 hi / lo tile buffers (the MMA's A operand)
constexpr int kABufBytes = 2 * kATileBytes;
constexpr int kScaleBytes = 1024;        // int8 weights: a stage's block scales (128 rows x 2 fp16), padded
constexpr int kMcMaxStages = 12;
constexpr int kMcMaxCluster = 8;         // portable cluster size
constexpr uint32_t kMcSpin = 1u << 22;

// Phase stamp i of this CTA (%globaltimer, ns) when the launch carries a trace buffer:
// 0 entry, 1 set-up done, 2 first TMA issued, 3 dependency wait done, 4 first stage landed (MMA
// warp), 5 first accumulator committed, 6 first accumulator seen by the epilogue, 7 partial in
// shared memory (cluster split), 8 cluster partials reduced, 9 epilogue done, 10 exit.
SP_DEVINL void mstamp(unsigned long long *tr, int i) {
    if (tr) tr[(size_t)blockIdx.x * kMcolTraceWords + i] = globaltimer();
}

SP_DEVINL void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kMcEpiThreads) : "memory"); }

SP_DEVINL void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
SP_DEVINL void tma_load_2d_hint(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
SP_DEVINL void prefetch_map(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Thread-block cluster: every thread of every CTA arrives (release) and waits (acquire). Not the
// .aligned form: the producer and MMA warps reach it from divergent code.
SP_DEVINL void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
SP_DEVINL uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The address of this CTA's shared-memory word `addr` in the CTA of rank `rank` of the cluster.
SP_DEVINL uint32_t dsmem_addr(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
SP_DEVINL float ld_dsmem(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// kind::f16 instruction descriptor: D fp32, A / B fp16, both K-major, M = 128, N = n.
SP_DEVINL uint32_t idesc_m128(int n) { return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24); }

struct Flag {
    volatile int *abort;
    DevState *st;
    SP_DEVINL bool on() const { return *abort != 0; }
    SP_DEVINL void raise() const {
        *abort = 1;
        if (st) atomicCAS(&st->err, 0, kErrMbarTimeout);
    }
};
SP_DEVINL bool wait_phase(uint64_t *bar, uint32_t parity, const Flag &f) {
    for (uint32_t i = 0; i < kMcSpin; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 127u) == 127u && f.on()) return false;
    }
    f.raise();
    return false;
}

// The cache slot of token 0 of the block (device-side base + offset), checked against the cache.
SP_DEVINL int qkv_slot0(const McolParams &p) {
    const McolQkv &a = p.qkv;
    if (a.lanes) return 0;               // batched decode: every token's slot comes from its lane
    int s0 = *a.slot_base + a.slot_off;
    if (s0 < 0 || s0 + p.T > a.cap) {
        if (p.st && threadIdx.x == 0) atomicCAS(&p.st->err, 0, kErrBadSlot);
        s0 = min(max(s0, 0), max(a.cap - p.T, 0));
    }
    return s0;
}

// The fused epilogue of one output y = alpha * sum (row n, token t). Rows 2i and 2i + 1 are in
// lanes 2m and 2m + 1 of one warp for the same token (every lane calls this, valid or not: the pair
// is exchanged by shuffle).
//   MC_STORE / MC_RESID: y[t ldy + n] = / += value
//   MC_SWIGLU: rows 2i (gate i), 2i + 1 (up i): act[t ld_act + i] = SiLU(gate) * up as fp16 hi / lo
//   MC_QKV: rows 2p, 2p + 1 = dims d, d + hd / 2 of one head (p = head * hd / 2 + d): bias, RoPE on
//     q and k with the token's position, q fp32 [t][heads * hd], k / v fp16 into the cache
//     (as the decode step's QKV epilogue computes them)
template <int MODE>
SP_DEVINL void epilogue_one(const McolParams &p, float v, int n, int t, int lane, int slot0) {
    const float y = p.alpha * v;
    const bool ok = n < p.N && t < p.T;
    if (MODE == MC_STORE || MODE == MC_RESID) {
        if (ok) {
            float *dst = p.y + (size_t)t * p.ldy + n;
            *dst = MODE == MC_RESID ? *dst + y : y;
        }
    } else if (MODE == MC_SWIGLU) {
        const float up = __shfl_xor_sync(0xffffffffu, y, 1);
        if ((lane & 1) == 0 && ok && n + 1 < p.N) {
            const float a = (y / (1.0f + expf(-y))) * up;
            const __half ah = __float2half_rn(a);
            p.act_h[(size_t)t * p.ld_act + (n >> 1)] = ah;
            p.act_l[(size_t)t * p.ld_act + (n >> 1)] = __float2half_rn(a - __half2float(ah));
        }
    } else {
        const McolQkv &a = p.qkv;
        const float other = __shfl_xor_sync(0xffffffffu, y, 1);
        if ((lane & 1) != 0 || !ok || n + 1 >= p.N) return;
        const int half_hd = a.hd / 2;
        const int P2 = n >> 1, hh = P2 / half_hd, dd = P2 - hh * half_hd;
        const float a0 = y + __ldg(a.bias + hh * a.hd + dd), a1 = other + __ldg(a.bias + hh * a.hd + dd + half_hd);
        const int slot = a.lanes ? a.lanes[t].slot : slot0 + t;
        __half *kbase = a.kc, *vbase = a.vc;
        int cap = a.cap;
        if (a.lanes) {                    // batched decode: the token's own cache, this layer
            cap = a.lanes[t].cap;
            kbase = a.lanes[t].k + (size_t)a.layer * a.nkv * cap * a.hd;
            vbase = a.lanes[t].v + (size_t)a.layer * a.nkv * cap * a.hd;
            if (slot < 0 || slot >= cap) {
                if (p.st) atomicCAS(&p.st->err, 0, kErrBadSlot);
                return;
            }
        }
        if (hh < a.nh + a.nkv) {
            int pos = a.pos ? a.pos[t] : slot;
            if (pos < 0 || pos >= a.max_pos) {
                if (p.st) atomicCAS(&p.st->err, 0, kErrBadSlot);
                pos = min(max(pos, 0), a.max_pos - 1);
            }
            const float2 r2 = __ldg(reinterpret_cast<const float2 *>(a.rope + ((size_t)pos * half_hd + dd) * 2));
            const float o0 = __fadd_rn(__fmul_rn(a0, r2.x), -__fmul_rn(a1, r2.y));
            const float o1 = __fadd_rn(__fmul_rn(a1, r2.x), __fmul_rn(a0, r2.y));
            if (hh < a.nh) {
                float *qr = a.q + (size_t)t * a.nh * a.hd + hh * a.hd;
                qr[dd] = o0;
                qr[dd + half_hd] = o1;
            } else {
                __half *kr = kbase + ((size_t)(hh - a.nh) * cap + slot) * a.hd;
                kr[dd] = __float2half_rn(o0);
                kr[dd + half_hd] = __float2half_rn(o1);
            }
        } else {
            __half *vr = vbase + ((size_t)(hh - a.nh - a.nkv) * cap + slot) * a.hd;
            vr[dd] = __float2half_rn(a0);
            vr[dd + half_hd] = __float2half_rn(a1);
        }
    }
}

}  // namespace

template <int MODE, bool I8>
__global__ void __launch_bounds__(I8 ? kMcThreads : kMcThreadsF16, 1)
    k_mcol(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w2,
           const __grid_constant__ CUtensorMap tm_x, const McolParams p) {
    extern __shared__ uint8_t mc_smem_raw[];
    __shared__ __align__(8) uint64_t full[kMcMaxStages], empty[kMcMaxStages], conv[kABufs], aempty[kABufs], accf[2],
        acce[2], drain;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int TN = p.tn, S = p.stages, cs = p.cs;
    const int kbx = (p.K + kBK - 1) / kBK;              // k-blocks of the input
    const int kbe = p.two_w ? 2 * kbx : kbx;            // k-blocks of a tile
    const int mtiles = (p.N + kBM - 1) / kBM, ntiles = (p.T + TN - 1) / TN;
    const long long tiles = (long long)mtiles * ntiles;
    // this CTA's k-blocks [u0, u1) of the flattened (tile, k-block) order
    long long u0, u1;
    int rank = 0;
    if (cs > 1) {
        rank = (int)cluster_rank();
        const long long tile = blockIdx.x / cs;
        u0 = tile * kbe + (long long)kbe * rank / cs;
        u1 = tile * kbe + (long long)kbe * (rank + 1) / cs;
    } else {
        u0 = tiles * blockIdx.x / gridDim.x * kbe;
        u1 = tiles * (blockIdx.x + 1) / gridDim.x * kbe;
    }
    const uint32_t base = (smem_u32(mc_smem_raw) + 1023u) & ~1023u;
    // a stage of the ring: the weight tile and the token tile. int8 weights: the token tile and the
    // TMA's int8 tile, which the epilogue warps turn into fp16 hi / lo tiles in one of kABufs
    // buffers ahead of the ring (a deep ring of 1-byte weights; the 4-byte tiles only where the MMA
    // reads them)
    constexpr bool i8w = I8;               // the int8-weight build (dequantization warps 6-9)
    const uint32_t qbase = base + (i8w ? (uint32_t)(kABufs * kABufBytes) : 0u);
    const uint32_t boff = i8w ? 0u : (uint32_t)kATileBytes;
    const uint32_t qoff = boff + (uint32_t)(2 * TN * kBK * 2);
    const uint32_t soff = qoff + (uint32_t)kI8TileBytes;              // int8: the tile's block scales
    const uint32_t stage_bytes = i8w ? soff + (uint32_t)kScaleBytes : qoff;
    const Flag fl{&s_abort, p.st};
    if (tid == 0) mstamp(p.trace, 0);

    if (tid == 0) {
        s_abort = 0;
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < kABufs; ++i) {
            mbar_init(&conv[i], kMcConvWarps);
            mbar_init(&aempty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&accf[i], 1);
            mbar_init(&acce[i], 1);
        }
        mbar_init(&drain, 1);
        fence_mbar_init();
    }
    if (warp == kMcMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"((uint32_t)p.tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (warp == kMcProducer && lane == 0) {
        prefetch_map(&tm_w);
        if (p.two_w) prefetch_map(&tm_w2);
        prefetch_map(&tm_x);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    griddep_launch_dependents();
    if (tid == 0) mstamp(p.trace, 1);

    // int8 weights, warps 6-9: the k-blocks [ua, ub) of the CTA's order, in the ring order of
    // the producer and the MMA warp. Per stage: wait for the TMA, turn the int8 tile into the fp16
    // hi / lo tiles, make the writes visible to the tensor core (fence.proxy.async) and arrive on
    // conv[stage]. w = q * sc with sc the block scale times 2^k (fp16, exact): hi = fp16(q sc) and
    // lo = fp16(q sc - hi), both single roundings of exact values (HMUL2 / HFMA2 on q as fp16, exact
    // for an int8), the same halves fp32 arithmetic gives. q to fp16 two at a time: the bytes
    // biased by 128 go into the mantissas of 1024.0 (0x64xx), then 1152 is subtracted (exact). The
    // tiles are 128-byte swizzled like a TMA tile: 16-byte piece j of row r at
    // r * 128 + ((j ^ (r & 7)) << 4). Thread item i of 512: row i / 4, inputs 16 (i % 4) .. + 15
    // (a warp reads 512 contiguous bytes of the int8 tile).
    int cv_s = 0, cv_a = 0;
    uint32_t cv_ph = 0u, cv_aph[kABufs] = {0u, 0u};
    long long cv_n = 0;
    const auto convert = [&](long long ua, long long ub) -> bool {
        const __half2 bias = __halves2half2(__ushort_as_half((unsigned short)0x6480u), __ushort_as_half((unsigned short)0x6480u));
        for (long long u = ua; u < ub; ++u) {
            if (!wait_phase(&full[cv_s], cv_ph, fl)) return false;
            if (cv_n >= kABufs) {                      // the MMAs that read this buffer are done
                if (!wait_phase(&aempty[cv_a], cv_aph[cv_a], fl)) return false;
                cv_aph[cv_a] ^= 1u;
            }
            const int mt = (int)(u / kbe) / ntiles;
            const uint32_t stg = qbase + (uint32_t)cv_s * stage_bytes;     // shared-space addresses
            const uint32_t abuf = base + (uint32_t)(cv_a * kABufBytes);
            constexpr int NI = kBM * 4 / kMcConvThreads;         // items a thread
            uint4 raw[NI];
            uint32_t sw[NI];
#pragma unroll
            for (int j = 0; j < NI; ++j) {                       // every load first, then the math
                const int i = (tid - kMcConv0 * 32) + j * kMcConvThreads, r = i >> 2, c = i & 3;
                asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                             : "=r"(raw[j].x), "=r"(raw[j].y), "=r"(raw[j].z), "=r"(raw[j].w)
                             : "r"(stg + qoff + (uint32_t)(r * kBK + c * 16)));
                // the two block scales of the row's k-block (staged with the tile)
                asm volatile("ld.shared.u32 %0, [%1];" : "=r"(sw[j]) : "r"(stg + soff + (uint32_t)(r * 4)));
            }
#pragma unroll
            for (int j = 0; j < NI; ++j) {
                const int i = (tid - kMcConv0 * 32) + j * kMcConvThreads, r = i >> 2, c = i & 3;
                const int n = mt * kBM + r;
                // this item's block is c / 2; rows past N read stale scale bytes: their int8 are zeros
                // from the TMA, and a zero scale keeps them zero
                const uint32_t sbits = n < p.N ? __byte_perm(sw[j], 0u, (c >> 1) ? 0x3232u : 0x1010u) : 0u;
                const __half2 s2 = *reinterpret_cast<const __half2 *>(&sbits);
                const uint32_t words[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
                uint32_t hw[8], lw[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const uint32_t x = words[e] ^ 0x80808080u;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t pb = __byte_perm(x, 0x64646464u, h ? 0x7362u : 0x5140u);
                        const __half2 q2 = __hsub2(*reinterpret_cast<const __half2 *>(&pb), bias);
                        const __half2 hi2 = __hmul2(q2, s2);
                        const __half2 lo2 = __hfma2(q2, s2, __hneg2(hi2));
                        hw[2 * e + h] = *reinterpret_cast<const uint32_t *>(&hi2);
                        lw[2 * e + h] = *reinterpret_cast<const uint32_t *>(&lo2);
                    }
                }
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const uint32_t off = (uint32_t)(r * 128 + (((2 * c + hh) ^ (r & 7)) << 4));
                    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(abuf + off), "r"(hw[4 * hh]),
                                 "r"(hw[4 * hh + 1]), "r"(hw[4 * hh + 2]), "r"(hw[4 * hh + 3]) : "memory");
                    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(abuf + (uint32_t)kATileBytes + off),
                                 "r"(lw[4 * hh]), "r"(lw[4 * hh + 1]), "r"(lw[4 * hh + 2]), "r"(lw[4 * hh + 3]) : "memory");
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&conv[cv_a]);
            if (++cv_s == S) {
                cv_s = 0;
                cv_ph ^= 1u;
            }
            cv_a = (cv_a + 1) % kABufs;
            ++cv_n;
        }
        return true;
    };

    if (warp == kMcProducer) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int s = 0;
            uint32_t ph = 0;
            long long issued = 0;
            // weights do not depend on the previous kernel; the tokens do
            bool waited = false;
            for (long long u = u0; u < u1 && !fl.on(); ++u) {
                const int tile = (int)(u / kbe), kb = (int)(u % kbe);
                const int mt = tile / ntiles, nt = tile % ntiles;
                if (issued >= S && !wait_phase(&empty[s], ph ^ 1u, fl)) break;
                const uint32_t st = qbase + (uint32_t)s * stage_bytes;
                // int8: the scales of the tile's rows below N (a multiple of 4 rows: 16-byte pieces)
                const uint32_t sc_bytes = i8w ? (uint32_t)min(kBM, p.N - mt * kBM) * 4u : 0u;
                mbar_arrive_expect_tx(&full[s], i8w ? qoff + (uint32_t)kI8TileBytes + sc_bytes : stage_bytes);
                const bool second = kb >= kbx;
                const int kx = (second ? kb - kbx : kb) * kBK;
                tma_load_2d_hint(i8w ? st + qoff : st, second ? &tm_w2 : &tm_w, kx, mt * kBM, &full[s], pol);
                if (i8w)
                    bulk_g2s_hint(mc_smem_raw + (st + soff - smem_u32(mc_smem_raw)),
                                  reinterpret_cast<const uint8_t *>(p.wsc) + ((size_t)kb * p.N + (size_t)mt * kBM) * 4, sc_bytes,
                                  &full[s], pol);
                if (!waited) {
                    mstamp(p.trace, 2);
                    griddep_wait();
                    mstamp(p.trace, 3);
                    waited = true;
                }
                tma_load_2d(st + boff, &tm_x, kx, nt * TN, &full[s]);
                tma_load_2d(st + boff + (uint32_t)(TN * kBK * 2), &tm_x, kx, p.lo_row0 + nt * TN, &full[s]);
                ++issued;
                if (++s == S) {
                    s = 0;
                    ph ^= 1u;
                }
            }
            if (!waited) griddep_wait();
            // loads still in flight land before the CTA may exit (after an abort)
            for (long long i = issued > S ? issued - S : 0; i < issued; ++i)
                mbar_wait_bounded(&full[i % S], (uint32_t)((i / S) & 1));
        }
    } else if (warp == kMcMma) {
        if (lane == 0) {
            const uint32_t idesc = idesc_m128(2 * TN), idesc_lo = idesc_m128(TN);
            int s = 0, buf = 0, ab = 0;
            uint32_t ph = 0, eph[2] = {0u, 0u}, cph[kABufs] = {0u, 0u};
            int nseg = 0;
            long long u = u0;
            while (u < u1 && !fl.on()) {
                const int tile = (int)(u / kbe);
                const long long tile_end = (long long)(tile + 1) * kbe;
                const long long v1 = u1 < tile_end ? u1 : tile_end;
                if (nseg >= 2) {                            // the epilogue has read this buffer out
                    if (!wait_phase(&acce[buf], eph[buf], fl)) break;
                    eph[buf] ^= 1u;
                }
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(buf * 2 * TN);
                bool first = true;
                for (; u < v1; ++u) {
                    if (!wait_phase(&full[s], ph, fl)) break;
                    if (i8w) {                              // and the stage's weights as fp16 hi / lo
                        if (!wait_phase(&conv[ab], cph[ab], fl)) break;
                        cph[ab] ^= 1u;
                    }
                    if (u == u0) mstamp(p.trace, 4);
                    tc_fence_after();
                    const uint32_t st = qbase + (uint32_t)s * stage_bytes;
                    const uint32_t at = i8w ? base + (uint32_t)(ab * kABufBytes) : st;
                    const uint64_t ad = smem_desc_sw128(at, 1024);
                    const uint64_t bd = smem_desc_sw128(st + boff, 1024);
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k)
                        mma_f16_id(acc, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, first && k == 0 ? 0u : 1u);
                    if (i8w) {
                        // the lo tile times the tokens' hi rows only (N = TN: columns 0 .. TN - 1); lo x lo
                        // is below 2^-22 of a product and is left out (a quarter of the MMA work)
                        const uint64_t ad2 = smem_desc_sw128(at + kATileBytes, 1024);
#pragma unroll
                        for (int k = 0; k < kBK / 16; ++k)
                            mma_f16_id(acc, ad2 + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc_lo, 1u);
                        mma_commit(&aempty[ab]);
                        ab = (ab + 1) % kABufs;
                    }
                    first = false;
                    mma_commit(&empty[s]);
                    if (++s == S) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (u < v1) break;                          // aborted
                mma_commit(&accf[buf]);
                if (nseg == 0) mstamp(p.trace, 5);
                ++nseg;
                buf ^= 1;
            }
            // every MMA issued has completed before TMEM is freed (matters after an abort)
            mma_commit(&drain);
            mbar_wait_bounded(&drain, 0u);
        }
    } else if (warp >= kMcConv0) {
        // ---- int8 weights: every k-block of the CTA, as the ring brings them --------------------------
        if constexpr (I8) convert(u0, u1);
    } else if (cs == 1) {
        // ---- whole tiles: thread = output row, 16 tokens per TMEM read ------------------------------
        const int row = warp * 32 + lane;
        int buf = 0;
        uint32_t fph[2] = {0u, 0u};
        const int slot0 = MODE == MC_QKV ? qkv_slot0(p) : 0;
        for (long long u = u0; u < u1 && !fl.on(); u += kbe) {
            const int tile = (int)(u / kbe);
            const int mt = tile / ntiles, nt = tile % ntiles;
            const int n = mt * kBM + row;
            if (!wait_phase(&accf[buf], fph[buf], fl)) break;
            if (u == u0 && tid == 0) mstamp(p.trace, 6);
            fph[buf] ^= 1u;
            tc_fence_after();
            const uint32_t tacc = tmem + (uint32_t)(buf * 2 * TN) + ((uint32_t)(warp * 32) << 16);
            for (int c0 = 0; c0 < TN; c0 += 16) {
                uint32_t h[16], l[16];
                tmem_ld16_nowait(tacc + (uint32_t)c0, h);
                tmem_ld16_nowait(tacc + (uint32_t)(TN + c0), l);
                tmem_wait_ld();
                const int t0 = nt * TN + c0;
                if (MODE == MC_RESID) {
                    if (n < p.N) {
                        // all loads before the stores (a store could alias a later load for the compiler)
                        float *dst = p.y + (size_t)t0 * p.ldy + n;
                        float old[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) old[j] = t0 + j < p.T ? __ldcg(dst + (size_t)j * p.ldy) : 0.f;
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (t0 + j < p.T)
                                dst[(size_t)j * p.ldy] = old[j] + p.alpha * (__uint_as_float(h[j]) + __uint_as_float(l[j]));
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        epilogue_one<MODE>(p, __uint_as_float(h[j]) + __uint_as_float(l[j]), n, t0 + j, lane, slot0);
                }
            }
            tc_fence_before();
            epi_bar();
            if (tid == 0) mbar_arrive(&acce[buf]);
            buf ^= 1;
        }
        if (tid == 0) mstamp(p.trace, 9);
    } else {
        // ---- cluster split: this CTA's partial of its tile into its own shared memory ---------------
        // P [row][TN] fp32 at the ring's start (every stage has been consumed once the accumulator is
        // committed: this CTA has exactly one segment)
        const int row = warp * 32 + lane;
        if (u0 < u1 && wait_phase(&accf[0], 0u, fl)) {
            if (tid == 0) mstamp(p.trace, 6);
            tc_fence_after();
            const uint32_t tacc = tmem + ((uint32_t)(warp * 32) << 16);
            float4 *mine = reinterpret_cast<float4 *>(mc_smem_raw + (base - smem_u32(mc_smem_raw))) + (size_t)row * (TN / 4);
            for (int c0 = 0; c0 < TN; c0 += 16) {
                uint32_t h[16], l[16];
                tmem_ld16_nowait(tacc + (uint32_t)c0, h);
                tmem_ld16_nowait(tacc + (uint32_t)(TN + c0), l);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    mine[c0 / 4 + j] = make_float4(__uint_as_float(h[4 * j]) + __uint_as_float(l[4 * j]),
                                                   __uint_as_float(h[4 * j + 1]) + __uint_as_float(l[4 * j + 1]),
                                                   __uint_as_float(h[4 * j + 2]) + __uint_as_float(l[4 * j + 2]),
                                                   __uint_as_float(h[4 * j + 3]) + __uint_as_float(l[4 * j + 3]));
            }
            tc_fence_before();
        }
        if (tid == 0) mstamp(p.trace, 7);
    }

    if (cs > 1) {
        // ---- cluster split: reduce rows [rank rp, (rank + 1) rp) of the tile over the cs partials ----
        cluster_sync();                                     // every partial of the cluster is written
        if (warp < kMcEpiThreads / 32) {
            const int rp = kBM / cs;
            const long long tile = blockIdx.x / cs;
            const int mt = (int)(tile / ntiles), nt = (int)(tile % ntiles);
            const int slot0 = MODE == MC_QKV ? qkv_slot0(p) : 0;
            // element e = tid + 128 i: row rank rp + e % rp, token e / rp (adjacent lanes, adjacent rows)
            for (int e = tid; e < rp * TN; e += kMcEpiThreads) {
                const int rl = e % rp, t = e / rp;
                const uint32_t off = base + (uint32_t)(((rank * rp + rl) * TN + t) * 4);
                // every partial is loaded before the first add (the remote loads overlap), then the
                // sum runs in rank order
                float part[kMcMaxCluster];
#pragma unroll
                for (int q = 0; q < kMcMaxCluster; ++q)
                    part[q] = q < cs ? ld_dsmem(dsmem_addr(off, (uint32_t)q)) : 0.f;
                float v = 0.f;
#pragma unroll
                for (int q = 0; q < kMcMaxCluster; ++q)
                    if (q < cs) v += part[q];
                const int n = mt * kBM + rank * rp + rl;
                epilogue_one<MODE>(p, v, n, nt * TN + t, lane, slot0);
            }
            if (tid == 0) mstamp(p.trace, 8);
        }
        cluster_sync();                                     // no CTA leaves while its partial is read
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMcMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)p.tmem_cols));
    }
    if (tid == 0) mstamp(p.trace, 10);
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
namespace {

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

// A row-major fp16 [rows, K] matrix as 64-input x box_rows tiles, 128-byte swizzle, zeros outside.
cudaError_t map_rows(CUtensorMap *m, const __half *ptr, int rows, int K, int box_rows) {
    EncodeTiled enc = encoder();
    if (!enc) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) || (K * 2) % 16 || box_rows < 8 || box_rows > 256)
        return cudaErrorInvalidValue;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// A row-major int8 [rows, K] matrix as 64-input x box_rows tiles of 64-byte rows (no swizzle: the
// epilogue warps read it and write the swizzled fp16 tiles), zeros outside.
cudaError_t map_rows_i8(CUtensorMap *m, const int8_t *ptr, int rows, int K, int box_rows) {
    EncodeTiled enc = encoder();
    if (!enc) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) || K % 16 || box_rows < 8 || box_rows > 256) return cudaErrorInvalidValue;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

int env_int(const char *name, int fallback) {
    const char *v = getenv(name);
    return v && *v ? atoi(v) : fallback;
}

int sm_count() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// The kernel's dynamic shared-memory limit, raised once per device.
template <int MODE, bool I8>
cudaError_t set_max_smem(int dev) {
    static std::atomic<unsigned long long> configured{0};       // one bit per device
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(configured.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(k_mcol<MODE, I8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mcol_max_smem());
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    return cudaSuccess;
}

template <int MODE, bool I8>
cudaError_t launch_mode(const CUtensorMap &a, const CUtensorMap &a2, const CUtensorMap &x, const McolParams &p,
                        int grid, size_t smem, cudaStream_t s, bool pdl) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = set_max_smem<MODE, I8>(dev);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(I8 ? kMcThreads : kMcThreadsF16);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (p.cs > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = (unsigned)p.cs;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k_mcol<MODE, I8>, a, a2, x, p);
}

// Clusters of cs CTAs of k_mcol<mode> (`threads` a CTA) with `smem` bytes of dynamic shared memory that
// can be resident at once on this device (cudaOccupancyMaxActiveClusters), cached per (device, mode,
// cs, smem, threads).
template <bool I8>
int max_active_clusters_t(int mode, int cs, size_t smem) {
    const int threads = I8 ? kMcThreads : kMcThreadsF16;
    static std::mutex mu;
    static std::map<std::tuple<int, int, int, size_t, int>, int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    const auto key = std::make_tuple(dev, mode, cs, smem, threads);
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs * kPrefillMaxCtas);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    cudaError_t e = cudaSuccess;
    switch (mode) {
        case MC_STORE: e = set_max_smem<MC_STORE, I8>(dev); if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n, k_mcol<MC_STORE, I8>, &cfg); break;
        case MC_RESID: e = set_max_smem<MC_RESID, I8>(dev); if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n, k_mcol<MC_RESID, I8>, &cfg); break;
        case MC_SWIGLU: e = set_max_smem<MC_SWIGLU, I8>(dev); if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n, k_mcol<MC_SWIGLU, I8>, &cfg); break;
        default: e = set_max_smem<MC_QKV, I8>(dev); if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n, k_mcol<MC_QKV, I8>, &cfg); break;
    }
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        n = 0;                                  // unknown: no cluster split
    }
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = n;
    return n;
}
int max_active_clusters(int mode, int cs, size_t smem, bool i8) {
    return i8 ? max_active_clusters_t<true>(mode, cs, smem) : max_active_clusters_t<false>(mode, cs, smem);
}

}  // namespace

size_t mcol_max_smem() { return 227 * 1024 - 1024; }   // 1 KB for the static barriers

int mcol_tile_tokens(int T) { return T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : 128; }

cudaError_t launch_mcol(const McolOp &op, cudaStream_t s, bool pdl) {
    if (op.T <= 0 || op.N <= 0 || op.K <= 0 || op.T > op.x_rows || op.lo_row0 < op.T) return cudaErrorInvalidValue;
    if (op.mode == MC_SWIGLU && (op.N % 2 || !op.act_h || !op.act_l)) return cudaErrorInvalidValue;
    if ((op.mode == MC_STORE || op.mode == MC_RESID) && !op.y) return cudaErrorInvalidValue;
    if (op.mode == MC_QKV) {
        const McolQkv &a = op.qkv;
        if (!a.bias || !a.rope || !a.q || a.hd <= 0 || a.hd % 2 || a.nh <= 0 || a.nkv <= 0 ||
            op.N != (a.nh + 2 * a.nkv) * a.hd || a.max_pos <= 0)
            return cudaErrorInvalidValue;
        if (!a.lanes && (!a.slot_base || !a.kc || !a.vc || a.cap < op.T)) return cudaErrorInvalidValue;
        if (a.lanes && (!a.pos || a.layer < 0)) return cudaErrorInvalidValue;
    }
    // int8: N a multiple of 4 (the block scales of a tile go by 16-byte bulk copies)
    if (op.wq && (op.w || op.w_lo || !op.wsc || op.N % 4 || (reinterpret_cast<uintptr_t>(op.wsc) & 15u)))
        return cudaErrorInvalidValue;
    if (!op.wq && !op.w) return cudaErrorInvalidValue;
    McolParams p{};
    p.N = op.N;
    p.K = op.K;
    p.T = op.T;
    p.tn = mcol_tile_tokens(op.T);
    p.lo_row0 = op.lo_row0;
    p.two_w = op.w_lo != nullptr;
    p.i8w = op.wq != nullptr;
    p.wsc = op.wsc;
    p.alpha = op.alpha;
    p.y = op.y;
    p.ldy = op.ldy;
    p.act_h = op.act_h;
    p.act_l = op.act_l;
    p.ld_act = op.ld_act;
    p.st = op.st;
    p.qkv = op.qkv;
    p.trace = op.trace;
    p.tmem_cols = 4 * p.tn < 32 ? 32 : 4 * p.tn;
    const int stage_bytes = (p.i8w ? kI8TileBytes + kScaleBytes : kATileBytes) + 2 * p.tn * kBK * 2;
    const size_t abytes = p.i8w ? (size_t)kABufs * kABufBytes : 0;       // int8: the hi / lo tile buffers
    static const int stage_cap = env_int("SEEDPLANE_MCOL_STAGES", kMcMaxStages);
    const int fit = (int)((mcol_max_smem() - 1024 - abytes) / stage_bytes);          // 1 KB: alignment
    p.stages = std::max(2, std::min(std::min(stage_cap, kMcMaxStages), fit));
    const long long mtiles = (op.N + kBM - 1) / kBM, ntiles = (op.T + p.tn - 1) / p.tn;
    const long long tiles = mtiles * ntiles;
    const long long kbe = (long long)((op.K + kBK - 1) / kBK) * (op.w_lo ? 2 : 1);
    // Whole tiles when they keep at least half the SMs busy; else the largest cluster (<= 8 CTAs, <= the
    // tile's k-blocks) whose tiles x cluster CTAs fit the SMs in one wave splits each tile's k-blocks:
    // the clusters must all be resident at once (a cluster's CTAs share one GPC, so fewer clusters
    // of 8 fit than 148 / 8), which the occupancy query of the launch says.
    const int C = std::min(sm_count(), op.max_ctas);
    static const int cs_cap = std::max(1, std::min(kMcMaxCluster, env_int("SEEDPLANE_MCOL_CLUSTER", kMcMaxCluster)));
    const size_t smem = abytes + (size_t)p.stages * stage_bytes + 1024;
    p.cs = 1;
    if (2 * tiles <= C)
        for (int cs = cs_cap; cs >= 2; cs /= 2)
            if (tiles * cs <= C && cs <= kbe &&
                tiles <= max_active_clusters(op.mode, cs, smem, p.i8w != 0)) {
                p.cs = cs;
                break;
            }
    const int grid = p.cs > 1 ? (int)(tiles * p.cs) : (int)std::min<long long>(C, tiles);
    CUtensorMap a, a2, x;
    cudaError_t e = p.i8w ? map_rows_i8(&a, op.wq, op.N, op.K, kBM) : map_rows(&a, op.w, op.N, op.K, kBM);
    if (e == cudaSuccess) {
        if (p.i8w)
            a2 = a;
        else
            e = map_rows(&a2, op.w_lo ? op.w_lo : op.w, op.N, op.K, kBM);
    }
    if (e == cudaSuccess) e = map_rows(&x, op.x, op.x_rows, op.K, p.tn);
    if (e != cudaSuccess) return e;
    if (p.i8w) {
        switch (op.mode) {
            case MC_STORE: return launch_mode<MC_STORE, true>(a, a2, x, p, grid, smem, s, pdl);
            case MC_RESID: return launch_mode<MC_RESID, true>(a, a2, x, p, grid, smem, s, pdl);
            case MC_SWIGLU: return launch_mode<MC_SWIGLU, true>(a, a2, x, p, grid, smem, s, pdl);
            case MC_QKV: return launch_mode<MC_QKV, true>(a, a2, x, p, grid, smem, s, pdl);
            default: return cudaErrorInvalidValue;
        }
    }
    switch (op.mode) {
        case MC_STORE: return launch_mode<MC_STORE, false>(a, a2, x, p, grid, smem, s, pdl);
        case MC_RESID: return launch_mode<MC_RESID, false>(a, a2, x, p, grid, smem, s, pdl);
        case MC_SWIGLU: return launch_mode<MC_SWIGLU, false>(a, a2, x, p, grid, smem, s, pdl);
        case MC_QKV: return launch_mode<MC_QKV, false>(a, a2, x, p, grid, smem, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace sp
