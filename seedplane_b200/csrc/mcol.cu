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
//   warps 0-3  epilogue: thread = output row (TMEM lane), tcgen05.ld of its hi / lo columns, the
//            fused epilogue of the op: store, residual add, or SwiGLU of interleaved gate / up rows
//            written as the down projection's fp16 hi / lo input
//
// Work: tiles of 128 rows x TN tokens, each over K in k-blocks of 64 inputs. With at least as many
// tiles as CTAs, every CTA takes whole tiles. Otherwise (the small projections of a verify pass)
// the k-blocks of all tiles are dealt out as one contiguous range per CTA (stream-K): a CTA whose
// range covers part of a tile writes its partial sums to a workspace slot and counts itself in on
// the tile's counter; the last contributor adds all partials in contributor order (so the result
// does not depend on which CTA finishes last) and runs the epilogue. Every wait is bounded; an
// expired wait records kErrMbarTimeout in DevState::err and the CTA leaves without waiting again.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <mutex>

#include "kernels.cuh"
#include "tc.cuh"

namespace sp {

namespace {

constexpr int kMcThreads = 192;
constexpr int kMcEpiThreads = 128;
constexpr int kMcProducer = 4;
constexpr int kMcMma = 5;
constexpr int kBK = 64;                  // inputs per k-block: one 128-byte swizzle row of fp16
constexpr int kBM = 128;
constexpr int kATileBytes = kBM * kBK * 2;
constexpr int kMcMaxStages = 8;
constexpr uint32_t kMcSpin = 1u << 22;

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

// The unit (k-block) range [u0, u1) of CTA c out of C over W units.
SP_DEVINL long long unit_start(long long W, int C, int c) { return W * c / C; }
SP_DEVINL int cta_of_unit(long long W, int C, long long u) {
    int c = (int)((u * C) / W);
    while (c > 0 && unit_start(W, C, c) > u) --c;
    while (c + 1 < C && unit_start(W, C, c + 1) <= u) ++c;
    return c;
}

}  // namespace

template <int MODE>
__global__ void __launch_bounds__(kMcThreads, 1)
    k_mcol(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w2,
           const __grid_constant__ CUtensorMap tm_x, const McolParams p) {
    extern __shared__ uint8_t mc_smem_raw[];
    __shared__ __align__(8) uint64_t full[kMcMaxStages], empty[kMcMaxStages], accf[2], acce[2], drain;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort, s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = gridDim.x, c = blockIdx.x;
    const int TN = p.tn, S = p.stages;
    const int kbx = (p.K + kBK - 1) / kBK;              // k-blocks of the input
    const int kbe = p.two_w ? 2 * kbx : kbx;            // k-blocks of a tile
    const int mtiles = (p.N + kBM - 1) / kBM, ntiles = (p.T + TN - 1) / TN;
    const long long tiles = (long long)mtiles * ntiles;
    const long long W = tiles * kbe;
    long long u0, u1;
    if (p.split) {
        u0 = unit_start(W, C, c);
        u1 = unit_start(W, C, c + 1);
    } else {
        u0 = tiles * c / C * kbe;
        u1 = tiles * (c + 1) / C * kbe;
    }
    const uint32_t base = (smem_u32(mc_smem_raw) + 1023u) & ~1023u;
    const uint32_t stage_bytes = (uint32_t)(kATileBytes + 2 * TN * kBK * 2);
    const Flag fl{&s_abort, p.st};

    if (tid == 0) {
        s_abort = 0;
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
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
                const uint32_t st = base + (uint32_t)s * stage_bytes;
                mbar_arrive_expect_tx(&full[s], stage_bytes);
                const bool second = kb >= kbx;
                const int kx = (second ? kb - kbx : kb) * kBK;
                tma_load_2d_hint(st, second ? &tm_w2 : &tm_w, kx, mt * kBM, &full[s], pol);
                if (!waited) {
                    griddep_wait();
                    waited = true;
                }
                tma_load_2d(st + kATileBytes, &tm_x, kx, nt * TN, &full[s]);
                tma_load_2d(st + kATileBytes + (uint32_t)(TN * kBK * 2), &tm_x, kx, p.lo_row0 + nt * TN, &full[s]);
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
            const uint32_t idesc = idesc_m128(2 * TN);
            int s = 0, buf = 0;
            uint32_t ph = 0, eph[2] = {0u, 0u};
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
                    tc_fence_after();
                    const uint32_t st = base + (uint32_t)s * stage_bytes;
                    const uint64_t ad = smem_desc_sw128(st, 1024);
                    const uint64_t bd = smem_desc_sw128(st + kATileBytes, 1024);
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k)
                        mma_f16_id(acc, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, first && k == 0 ? 0u : 1u);
                    first = false;
                    mma_commit(&empty[s]);
                    if (++s == S) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (u < v1) break;                          // aborted
                mma_commit(&accf[buf]);
                ++nseg;
                buf ^= 1;
            }
            // every MMA issued has completed before TMEM is freed (matters after an abort)
            mma_commit(&drain);
            mbar_wait_bounded(&drain, 0u);
        }
    } else {
        // ---- epilogue: warps 0-3, thread = row of the tile ----------------------------------------
        const int row = warp * 32 + lane;
        int buf = 0;
        uint32_t fph[2] = {0u, 0u};
        long long u = u0;
        while (u < u1 && !fl.on()) {
            const int tile = (int)(u / kbe), kb0 = (int)(u % kbe);
            const long long tile_end = (long long)(tile + 1) * kbe;
            const long long v1 = u1 < tile_end ? u1 : tile_end;
            const bool whole = kb0 == 0 && v1 == tile_end;
            u = v1;
            const int mt = tile / ntiles, nt = tile % ntiles;
            const int n = mt * kBM + row;
            if (!wait_phase(&accf[buf], fph[buf], fl)) break;
            fph[buf] ^= 1u;
            tc_fence_after();
            const uint32_t tacc = tmem + (uint32_t)(buf * 2 * TN) + ((uint32_t)(warp * 32) << 16);
            // this segment's position among the tile's contributors (split tiles only)
            // (the host makes every CTA's range non-empty, so the contributors are consecutive CTAs)
            int first_c = 0, nctr = 1;
            if (!whole) {
                first_c = cta_of_unit(W, C, (long long)tile * kbe);
                nctr = cta_of_unit(W, C, tile_end - 1) - first_c + 1;
            }
            float *wsl = nullptr;
            if (!whole) {
                const int slot = 2 * c + ((long long)tile == unit_start(W, C, c) / kbe ? 0 : 1);
                wsl = p.ws + (size_t)slot * kBM * TN;
            }
            // the tile's columns in chunks of 16 tokens: v[j] = hi + lo of token c0 + j
            bool last = true;
            if (!whole) {
                for (int c0 = 0; c0 < TN; c0 += 16) {
                    uint32_t h[16], l[16];
                    tmem_ld16_nowait(tacc + (uint32_t)c0, h);
                    tmem_ld16_nowait(tacc + (uint32_t)(TN + c0), l);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        __stcg(wsl + (size_t)(c0 + j) * kBM + row, __uint_as_float(h[j]) + __uint_as_float(l[j]));
                }
                tc_fence_before();
                __threadfence();
                epi_bar();
                if (tid == 0) {
                    __threadfence();
                    const unsigned prev = atomicAdd(p.cnt + tile, 1u);
                    s_last = prev == (unsigned)(nctr - 1);
                    if (s_last) p.cnt[tile] = 0u;                       // ready for the next launch
                    __threadfence();
                }
                epi_bar();
                last = s_last != 0;
                if (tid == 0) mbar_arrive(&acce[buf]);                  // the accumulator is read out
                if (last) __threadfence();
            }
            if (last) {
                for (int c0 = 0; c0 < TN; c0 += 16) {
                    float v[16];
                    if (whole) {
                        uint32_t h[16], l[16];
                        tmem_ld16_nowait(tacc + (uint32_t)c0, h);
                        tmem_ld16_nowait(tacc + (uint32_t)(TN + c0), l);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(h[j]) + __uint_as_float(l[j]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = 0.f;
                        for (int q = 0; q < nctr; ++q) {             // contributors in CTA order
                            const int cq = first_c + q;
                            const int slot = 2 * cq + ((long long)tile == unit_start(W, C, cq) / kbe ? 0 : 1);
                            const float *src = p.ws + (size_t)slot * kBM * TN + (size_t)c0 * kBM + row;
#pragma unroll
                            for (int j = 0; j < 16; ++j) v[j] += __ldcg(src + (size_t)j * kBM);
                        }
                    }
                    const int t0 = nt * TN + c0;
                    if (MODE == MC_SWIGLU) {
                        // rows 2i (gate i) and 2i + 1 (up i) sit in lanes 2m, 2m + 1 of one warp
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const float y = p.alpha * v[j];
                            const float up = __shfl_xor_sync(0xffffffffu, y, 1);
                            const int t = t0 + j;
                            if ((lane & 1) == 0 && t < p.T && n + 1 < p.N) {
                                const float a = (y / (1.0f + expf(-y))) * up;
                                const __half ah = __float2half_rn(a);
                                p.act_h[(size_t)t * p.ld_act + (n >> 1)] = ah;
                                p.act_l[(size_t)t * p.ld_act + (n >> 1)] = __float2half_rn(a - __half2float(ah));
                            }
                        }
                    } else if (n < p.N) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int t = t0 + j;
                            if (t < p.T) {
                                float *dst = p.y + (size_t)t * p.ldy + n;
                                if (MODE == MC_RESID)
                                    *dst += p.alpha * v[j];
                                else
                                    *dst = p.alpha * v[j];
                            }
                        }
                    }
                }
            }
            if (whole) {
                tc_fence_before();
                epi_bar();
                if (tid == 0) mbar_arrive(&acce[buf]);
            }
            buf ^= 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMcMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)p.tmem_cols));
    }
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

template <int MODE>
cudaError_t launch_mode(const CUtensorMap &a, const CUtensorMap &a2, const CUtensorMap &x, const McolParams &p,
                        int grid, size_t smem, cudaStream_t s, bool pdl) {
    static std::atomic<unsigned long long> configured{0};       // one bit per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(configured.load() & bit)) {
        e = cudaFuncSetAttribute(k_mcol<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mcol_max_smem());
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kMcThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_mcol<MODE>, a, a2, x, p);
}

}  // namespace

size_t mcol_max_smem() { return 227 * 1024 - 1024; }   // 1 KB for the static barriers

int mcol_tile_tokens(int T) { return T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : 128; }

size_t mcol_workspace_bytes(int max_ctas, int max_tokens) {
    return (size_t)2 * max_ctas * kBM * mcol_tile_tokens(max_tokens) * sizeof(float);
}

size_t mcol_counter_count(int max_rows, int max_tokens) {
    const int tn = mcol_tile_tokens(max_tokens);
    return (size_t)((max_rows + kBM - 1) / kBM) * ((max_tokens + tn - 1) / tn);
}

cudaError_t launch_mcol(const McolOp &op, cudaStream_t s, bool pdl) {
    if (op.T <= 0 || op.N <= 0 || op.K <= 0 || op.T > op.x_rows || op.lo_row0 < op.T) return cudaErrorInvalidValue;
    if (op.mode == MC_SWIGLU && (op.N % 2 || !op.act_h || !op.act_l)) return cudaErrorInvalidValue;
    if (op.mode != MC_SWIGLU && !op.y) return cudaErrorInvalidValue;
    McolParams p{};
    p.N = op.N;
    p.K = op.K;
    p.T = op.T;
    p.tn = mcol_tile_tokens(op.T);
    p.lo_row0 = op.lo_row0;
    p.two_w = op.w_lo != nullptr;
    p.alpha = op.alpha;
    p.y = op.y;
    p.ldy = op.ldy;
    p.act_h = op.act_h;
    p.act_l = op.act_l;
    p.ld_act = op.ld_act;
    p.ws = op.ws;
    p.cnt = op.cnt;
    p.st = op.st;
    p.tmem_cols = 4 * p.tn < 32 ? 32 : 4 * p.tn;
    const int stage_bytes = kATileBytes + 2 * p.tn * kBK * 2;
    p.stages = std::min(kMcMaxStages, (int)((mcol_max_smem() - 1024) / stage_bytes));   // 1 KB: alignment
    const long long mtiles = (op.N + kBM - 1) / kBM, ntiles = (op.T + p.tn - 1) / p.tn;
    const long long tiles = mtiles * ntiles;
    const int C = std::min(sm_count(), op.max_ctas);
    int grid;
    if (tiles >= C) {
        p.split = 0;
        grid = C;
    } else {
        // every CTA gets at least one k-block, so a split tile's contributors are consecutive CTAs
        p.split = 1;
        const long long kbe = (long long)((op.K + kBK - 1) / kBK) * (op.w_lo ? 2 : 1);
        grid = (int)std::min<long long>(C, tiles * kbe);
        if (!op.ws || !op.cnt || tiles > op.cnt_count) return cudaErrorInvalidValue;
    }
    if (p.split && (size_t)2 * grid * kBM * p.tn * sizeof(float) > op.ws_bytes) return cudaErrorInvalidValue;
    CUtensorMap a, a2, x;
    cudaError_t e = map_rows(&a, op.w, op.N, op.K, kBM);
    if (e == cudaSuccess) e = map_rows(&a2, op.w_lo ? op.w_lo : op.w, op.N, op.K, kBM);
    if (e == cudaSuccess) e = map_rows(&x, op.x, op.x_rows, op.K, p.tn);
    if (e != cudaSuccess) return e;
    const size_t smem = (size_t)p.stages * stage_bytes + 1024;
    switch (op.mode) {
        case MC_STORE: return launch_mode<MC_STORE>(a, a2, x, p, grid, smem, s, pdl);
        case MC_RESID: return launch_mode<MC_RESID>(a, a2, x, p, grid, smem, s, pdl);
        case MC_SWIGLU: return launch_mode<MC_SWIGLU>(a, a2, x, p, grid, smem, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace sp
