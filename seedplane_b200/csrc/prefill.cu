// Batched prompt pass (prefill) for sm_100a: T prompt tokens per chunk through all layers at once.
//
// The projections of T tokens go to the multi-column tcgen05 GEMM of mcol.cu (weights as the
// M = 128 operand, the tokens as the N operand) with fused epilogues: the O and down projections
// add into the fp32 residual stream, gate_up (rows interleaved gate / up) writes SwiGLU straight
// into the down projection's input, QKV and the LM head store fp32. Around them: embedding gather,
// RMSNorm to fp16 hi / lo halves, bias + RoPE + K/V cache write, causal GQA attention over the
// cache. Every GEMM input is split like the decode step's: hi = fp16(x), lo = fp16(x - hi), token
// t's hi row at t and its lo row at kPrefillMaxTokens + t of the input buffer, so the products carry
// ~22 bits of the fp32 activation against the fp16 weights (the precision greedy token identity
// with the fp32 reference depends on). The residual stream stays fp32.
//
// The same pass verifies a draft tree: the T tokens are tree nodes (K/V at scratch slots) and
// node t attends to the committed prefix and to the nodes whose bits its ancestor mask holds.
#include <algorithm>
#include <atomic>
#include <cmath>

#include "kernels.cuh"

namespace sp {

namespace {

constexpr int kNormThreads = 256;
constexpr int kShortBlockT = 64;            // blocks up to this many tokens: one query per warp

__device__ __forceinline__ void set_err(DevState *st, int code) {
    if (st) atomicCAS(&st->err, 0, code);
}

// Kernels of the pass are launched with programmatic dependent launch: each may start while its
// predecessor finishes, and waits for it (griddepcontrol.wait) before its first global access.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
// The same with dynamic shared memory; the kernel's limit is raised once per device when the size
// is above the default 48 KB.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_smem(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args... args) {
    if (smem > 48 * 1024) {
        static std::atomic<unsigned long long> raised{0};     // one bit per device, per kernel
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        const unsigned long long bit = 1ull << (dev & 63);
        if (!(raised.load() & bit)) {
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            raised.fetch_or(bit);
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
SP_DEVINL void pdl_enter() {
    griddep_wait();
    griddep_launch_dependents();
}

// First cache slot of the block: device-side base (so a captured graph serves any cache length)
// plus the chunk offset; a block that would not fit the cache records an error and is clamped.
__device__ __forceinline__ int block_slot0(const int *slot_base, int slot_off, int T, int cap, DevState *st) {
    int s0 = *slot_base + slot_off;
    if (s0 < 0 || s0 + T > cap) {
        if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) set_err(st, kErrBadSlot);
        s0 = min(max(s0, 0), max(cap - T, 0));
    }
    return s0;
}

// x[t] = embedding row of token t (ids outside the vocabulary record an error and read row 0)
__global__ void k_embed_rows(float *x, const __half *embed, const int32_t *tok, int H, int vocab, DevState *st) {
    pdl_enter();
    const int t = blockIdx.x;
    int id = tok[t];
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) set_err(st, kErrBadToken);
        id = 0;
    }
    const __half *row = embed + (size_t)id * H;
    for (int j = threadIdx.x; j < H; j += blockDim.x) x[(size_t)t * H + j] = __half2float(row[j]);
}

// hi / lo halves of RMSNorm(x[t]) * gain: v = (x * inv) * g, inv = 1 / sqrt(mean(x^2) + eps)
__global__ void __launch_bounds__(kNormThreads) k_rmsnorm_hilo(__half *xh, __half *xl, const float *x,
                                                                const float *gain, int H, float eps) {
    pdl_enter();
    const int t = blockIdx.x;
    const float *r = x + (size_t)t * H;
    __shared__ float s_part[kNormThreads / 32];
    float sq = 0.f;
    for (int j = threadIdx.x; j < H; j += kNormThreads) sq = fmaf(r[j], r[j], sq);
    sq = warp_sum(sq);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = sq;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < kNormThreads / 32; ++w) tot += s_part[w];
    const float inv = 1.0f / sqrtf(tot / (float)H + eps);
    for (int j = threadIdx.x; j < H; j += kNormThreads) {
        const float v = (r[j] * inv) * gain[j];
        const __half h = __float2half_rn(v);
        xh[(size_t)t * H + j] = h;
        xl[(size_t)t * H + j] = __float2half_rn(v - __half2float(h));
    }
}

// Attention of a block of T queries over the cache (a short verify tree or prompt chunk over a
// short cache; k_attn_gqa below takes the rest). CTA = (q head, 4 QW queries), warp w = queries
// q0 + w QW .. + QW - 1 (the pass uses QW = 1). The visible keys go through shared memory in tiles of 64 (K and V rows padded by
// 16 bytes, so the lanes of a quarter warp reading 16 bytes of 8 different rows hit distinct
// banks), two tiles in flight: tile i + 1 is copied with cp.async while tile i is used. Per tile
// and warp: lane = keys lane and lane + 32 (full dot products over the row, each K chunk read once
// for the warp's QW queries), online softmax per query (running max / sum in fp32), then lane =
// HD / 32 output dims summed over the tile's keys in order with the probabilities broadcast from
// shared memory. Query t sees the slots before slot0 and, among the block's own slots,
// [slot0, slot0 + t] (causal, mask == null) or the slots slot0 + j whose bit j its ancestor mask
// holds (tree, T <= 64). The output goes out as fp16 hi / lo halves (the O projection's input).
constexpr int kTreeKeys = 64;
template <int HD>
struct TreeSmem {
    static constexpr int kRow = HD * 2 + 16;                       // bytes of a padded K / V row
    static constexpr int kTile = kTreeKeys * kRow;                 // one tile of K (or V)
    static constexpr int kBytes = 2 * 2 * kTile;                   // two stages of K and V
};
template <int HD, int QW>
__global__ void __launch_bounds__(128) k_attn_block(__half *oh, __half *ol, const float *q, const __half *kc,
                                                    const __half *vc, const uint64_t *mask, int T, int nh, int nkv,
                                                    int cap, const int *slot_base, int slot_off, float scale,
                                                    DevState *st) {
    using L = TreeSmem<HD>;
    constexpr int QC = 4 * QW;                                     // queries per CTA
    extern __shared__ __align__(16) uint8_t tsm[];
    __shared__ __align__(16) float qs[QC][HD];
    __shared__ float ps[QC][kTreeKeys];
    pdl_enter();
    const int slot0 = block_slot0(slot_base, slot_off, T, cap, st);
    constexpr int DL = HD / 32;
    constexpr int CH = HD / 8;                                     // 16-byte chunks per row
    const int h = blockIdx.x, q0 = blockIdx.y * QC;
    const int g = h / (nh / nkv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tw = q0 + warp * QW;                                 // this warp's first query
    const __half *kb = kc + (size_t)g * cap * HD, *vb = vc + (size_t)g * cap * HD;
    const int last = slot0 + min(T, q0 + QC) - 1;                  // the last key any query of this CTA sees
    const int ntiles = last / kTreeKeys + 1;
    auto stage = [&](int tile) {                                   // cp.async of tile `tile` into its stage
        uint8_t *ks = tsm + (tile & 1) * 2 * L::kTile, *vs = ks + L::kTile;
        const int k0 = tile * kTreeKeys;
        for (int i = threadIdx.x; i < kTreeKeys * CH; i += 128) {
            const int j = i / CH, c = i - j * CH;
            if (k0 + j <= last) {
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(ks + j * L::kRow + c * 16)),
                             "l"(kb + (size_t)(k0 + j) * HD + c * 8) : "memory");
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(vs + j * L::kRow + c * 16)),
                             "l"(vb + (size_t)(k0 + j) * HD + c * 8) : "memory");
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    stage(0);
    for (int i = threadIdx.x; i < QC * HD; i += 128) {
        const int qq = i / HD, d = i - qq * HD;
        qs[qq][d] = q0 + qq < T ? q[(size_t)(q0 + qq) * nh * HD + h * HD + d] * scale : 0.f;
    }
    float m[QW], l[QW], acc[QW][DL];
    uint64_t tmask[QW];
#pragma unroll
    for (int i = 0; i < QW; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
        tmask[i] = (mask && tw + i < T) ? mask[tw + i] : 0ull;
#pragma unroll
        for (int d = 0; d < DL; ++d) acc[i][d] = 0.f;
    }
    // the last key any query of this warp sees: tiles past it are skipped by the warp
    const int wlast = slot0 + min(T - 1, tw + QW - 1);
    for (int tile = 0; tile < ntiles; ++tile) {
        if (tile + 1 < ntiles) {
            stage(tile + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();                                           // tile `tile` (and q) visible to all
        const uint8_t *ks = tsm + (tile & 1) * 2 * L::kTile, *vs = ks + L::kTile;
        const int k0 = tile * kTreeKeys;
        if (k0 <= wlast && tw < T) {                               // warp-uniform
            float s0[QW], s1[QW];
#pragma unroll
            for (int i = 0; i < QW; ++i) s0[i] = s1[i] = 0.f;
            const uint8_t *r0 = ks + lane * L::kRow, *r1 = ks + (lane + 32) * L::kRow;
#pragma unroll 2
            for (int c = 0; c < CH; ++c) {
                const uint4 a = *reinterpret_cast<const uint4 *>(r0 + c * 16);
                const uint4 b = *reinterpret_cast<const uint4 *>(r1 + c * 16);
                const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
                float fa[8], fb[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 x = __half22float2(*reinterpret_cast<const __half2 *>(&aw[e]));
                    const float2 y = __half22float2(*reinterpret_cast<const __half2 *>(&bw[e]));
                    fa[2 * e] = x.x;
                    fa[2 * e + 1] = x.y;
                    fb[2 * e] = y.x;
                    fb[2 * e + 1] = y.y;
                }
#pragma unroll
                for (int i = 0; i < QW; ++i) {
                    const float4 qa = *reinterpret_cast<const float4 *>(&qs[warp * QW + i][8 * c]);
                    const float4 qb = *reinterpret_cast<const float4 *>(&qs[warp * QW + i][8 * c + 4]);
                    const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        s0[i] = fmaf(qv[e], fa[e], s0[i]);
                        s1[i] = fmaf(qv[e], fb[e], s1[i]);
                    }
                }
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < QW; ++i) {
                const int t = tw + i;
                auto visible = [&](int key) {
                    bool vis = t < T && key <= slot0 + t;
                    if (mask && vis && key >= slot0) vis = (tmask[i] >> (key - slot0)) & 1ull;
                    return vis;
                };
                const float v0 = visible(k0 + lane) ? s0[i] : -INFINITY;
                const float v1 = visible(k0 + 32 + lane) ? s1[i] : -INFINITY;
                const float mnew = fmaxf(m[i], warp_max(fmaxf(v0, v1)));
                const float p0 = mnew == -INFINITY ? 0.f : expf(v0 - mnew);
                const float p1 = mnew == -INFINITY ? 0.f : expf(v1 - mnew);
                const float corr = m[i] == -INFINITY ? 0.f : expf(m[i] - mnew);
                l[i] = l[i] * corr + warp_sum(p0 + p1);
                m[i] = mnew;
                ps[warp * QW + i][lane] = p0;
                ps[warp * QW + i][lane + 32] = p1;
#pragma unroll
                for (int d = 0; d < DL; ++d) acc[i][d] *= corr;
            }
            __syncwarp();
            const int nk = min(kTreeKeys, wlast + 1 - k0);         // keys of the tile this warp may see
#pragma unroll 4
            for (int j = 0; j < nk; ++j) {
                const uint8_t *vr = vs + j * L::kRow + lane * DL * 2;
                float vf[DL];
                if constexpr (DL == 4) {
                    const uint2 vv = *reinterpret_cast<const uint2 *>(vr);
                    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&vv.x));
                    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&vv.y));
                    vf[0] = a.x;
                    vf[1] = a.y;
                    vf[2] = b.x;
                    vf[3] = b.y;
                } else {
                    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(vr));
                    vf[0] = a.x;
                    vf[1] = a.y;
                }
#pragma unroll
                for (int i = 0; i < QW; ++i) {
                    const float pj = ps[warp * QW + i][j];
#pragma unroll
                    for (int d = 0; d < DL; ++d) acc[i][d] = fmaf(pj, vf[d], acc[i][d]);
                }
            }
        }
        __syncthreads();                                           // the stage is rewritten two tiles on
    }
#pragma unroll
    for (int i = 0; i < QW; ++i) {
        const int t = tw + i;
        if (t >= T) continue;
#pragma unroll
        for (int d = 0; d < DL; ++d) {
            const float o = acc[i][d] / l[i];
            const __half hv = __float2half_rn(o);
            const size_t idx = (size_t)t * nh * HD + h * HD + lane * DL + d;
            oh[idx] = hv;
            ol[idx] = __float2half_rn(o - __half2float(hv));
        }
    }
}

// Attention of a block of T queries on the tensor cores, by GQA group and context chunk (the long-
// context form of k_attn_block, same visibility rule and output). Rows are (query t, head r) pairs
// of kv head g's group, pair p = t G + r; an m-tile of the MMAs is 8 pairs: row i < 8 = fp16 hi
// of pair i's q * scale, row 8 + i = its fp16 lo, so
//   scores  S (16 x 8 keys) = Q K^T, mma.sync m16n8k16 (B = K rows by ldmatrix), pair i's score
//           = D[i] + D[8 + i];
//   values  O (16 x HD) += P V, mma.sync m16n8k16 with A = the probabilities' fp16 hi (rows i) and
//           lo (rows 8 + i) taken straight from the score accumulators, B = V rows by
//           ldmatrix.trans; pair i's output = O[i] + O[8 + i].
// CTA = (kv head g, 32 pairs = one m-tile per warp, key chunk z): the chunk's keys go through
// shared memory in tiles of 64 (rows XOR-swizzled in 16-byte pieces, two tiles in flight), and
// every warp multiplies its m-tile with each tile; online softmax per pair in fp32. Chunks: the
// visible keys [0, slot0 + T) are cut into nz pieces of >= 256 keys (nz <= gridDim.z, computed on
// the device from slot0, so one captured graph serves any cache length). One chunk: the output as
// fp16 hi / lo halves; several: an unnormalised partial (max, sum, acc[HD]) per (pair, chunk) that
// k_attn_merge folds in chunk order.
constexpr int kGqaKeys = 64;                // keys per shared-memory tile
constexpr int kGqaChunkKeys = 256;          // keys per chunk at least
constexpr int kShortCacheKeys = 1024;       // caches this short: verify blocks use k_attn_block
constexpr int kGqaPairs = 32;               // (query, head) pairs per CTA: 8 a warp
constexpr int kGqaMaxChunks = 64;           // chunks of the keys at most
template <int HD>
struct GqaSmem {
    static constexpr int kRow = HD * 2;                            // bytes of a K / V row
    static constexpr int kTile = kGqaKeys * kRow;
    static constexpr int kBytes = 2 * 2 * kTile;                   // two stages of K and V
};
SP_DEVINL void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
SP_DEVINL void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
SP_DEVINL void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
SP_DEVINL uint32_t h2bits(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}
// byte offset of 16-byte piece c of row r in a swizzled tile (pieces XOR-permuted by r within each
// 128-byte segment: the 8 rows an ldmatrix reads hit 8 different bank groups)
template <int HD>
SP_DEVINL uint32_t gqa_off(int r, int c) {
    return (uint32_t)(r * GqaSmem<HD>::kRow + (((c & ~7) | ((c & 7) ^ (r & 7))) << 4));
}
// Chunk size and count for `keys` visible keys over at most zmax chunks (the same in every kernel).
SP_DEVINL void gqa_chunks(int keys, int zmax, int &chunk, int &nz) {
    chunk = max(kGqaChunkKeys, (keys + zmax - 1) / zmax);
    chunk = (chunk + kGqaKeys - 1) / kGqaKeys * kGqaKeys;
    nz = (keys + chunk - 1) / chunk;
}

template <int HD>
__global__ void __launch_bounds__(128) k_attn_gqa(__half *oh, __half *ol, float *part, const float *q,
                                                  const __half *kc, const __half *vc, const uint64_t *mask, int T,
                                                  int nh, int nkv, int cap, const int *slot_base, int slot_off,
                                                  float scale, DevState *st) {
    using L = GqaSmem<HD>;
    constexpr int KS = HD / 16;             // k-steps of a score MMA
    constexpr int NT = HD / 8;              // output n-tiles
    constexpr int CH = HD / 8;              // 16-byte pieces of a row
    extern __shared__ __align__(128) uint8_t gsm[];
    pdl_enter();
    const int slot0 = block_slot0(slot_base, slot_off, T, cap, st);
    const int G = nh / nkv, g = blockIdx.x, z = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
    const int keys = slot0 + T;             // every key any query sees is below this
    int chunk, nz;
    gqa_chunks(keys, (int)gridDim.z, chunk, nz);
    if (z >= nz) return;                    // uniform: this chunk holds no key
    const int np = T * G, p0 = blockIdx.y * kGqaPairs;
    // the last key the CTA's pairs see, and this chunk's keys
    const int last = slot0 + min(T - 1, (min(np, p0 + kGqaPairs) - 1) / G);
    const int k_lo = z * chunk, k_hi = min(keys, min(k_lo + chunk, last + 1));
    // this thread's pair (row gq of the warp's m-tile): query, head, visibility
    const int pr = p0 + warp * 8 + gq;
    const bool live = pr < np;
    const int tr = live ? pr / G : 0, hr = g * G + (live ? pr % G : 0);
    const uint64_t tm = (mask && live) ? mask[tr] : 0ull;
    const __half *kb = kc + (size_t)g * cap * HD, *vb = vc + (size_t)g * cap * HD;
    const int ntiles = k_hi > k_lo ? (k_hi - k_lo + kGqaKeys - 1) / kGqaKeys : 0;
    auto stage = [&](int tile) {
        uint8_t *ks = gsm + (tile & 1) * 2 * L::kTile, *vs = ks + L::kTile;
        const int j0 = k_lo + tile * kGqaKeys;
        for (int i = threadIdx.x; i < kGqaKeys * CH; i += 128) {
            const int r = i / CH, c = i - r * CH;
            const int j = min(j0 + r, keys - 1);     // past the chunk: a valid row, masked
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(ks + gqa_off<HD>(r, c))),
                         "l"(kb + (size_t)j * HD + c * 8) : "memory");
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(vs + gqa_off<HD>(r, c))),
                         "l"(vb + (size_t)j * HD + c * 8) : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (ntiles > 0) stage(0);
    // q fragments of the warp's m-tile: row gq hi / lo at dims 16 kk + 2 tq + {0, 1} and + 8
    uint32_t qa[KS][4];
    {
        const float *qr = q + (size_t)tr * nh * HD + (size_t)hr * HD;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const float2 x = live ? *reinterpret_cast<const float2 *>(qr + 16 * kk + 8 * hf + 2 * tq)
                                      : make_float2(0.f, 0.f);
                const float a = x.x * scale, b = x.y * scale;
                const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
                qa[kk][2 * hf] = h2bits(ha, hb);
                qa[kk][2 * hf + 1] = h2bits(__float2half_rn(a - __half2float(ha)), __float2half_rn(b - __half2float(hb)));
            }
        }
    }
    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m_run = -INFINITY, l_part = 0.f;
    const int wlast = slot0 + min(T - 1, (min(np, p0 + warp * 8 + 8) - 1) / G);   // the warp's last key
    const auto visible = [&](int j) {
        if (!live || j >= keys) return false;
        if (j < slot0) return true;
        return mask ? (((tm >> (j - slot0)) & 1ull) != 0ull) : j <= slot0 + tr;
    };
    for (int tile = 0; tile < ntiles; ++tile) {
        if (tile + 1 < ntiles) {
            stage(tile + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();                    // tile `tile` visible to all
        const uint32_t ks = smem_u32(gsm + (tile & 1) * 2 * L::kTile), vs = ks + L::kTile;
        const int j0 = k_lo + tile * kGqaKeys;
        if (j0 <= wlast && pr - gq < np) {  // warp-uniform
            // scores of the tile: 8 n-tiles of 8 keys
            float s[8][4];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
                for (int kk = 0; kk < KS; kk += 2) {
                    uint32_t b0, b1, b2, b3;   // keys 8 nt .. + 7, pieces 2 kk .. 2 kk + 3
                    ldsm_x4(ks + gqa_off<HD>(8 * nt + (lane & 7), 2 * kk + (lane >> 3)), b0, b1, b2, b3);
                    mma16816(s[nt], qa[kk], b0, b1);
                    mma16816(s[nt], qa[kk + 1], b2, b3);
                }
            }
            float mt = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float v = s[nt][e] + s[nt][2 + e];
                    if (!visible(j0 + 8 * nt + 2 * tq + e)) v = -INFINITY;
                    s[nt][e] = v;
                    mt = fmaxf(mt, v);
                }
            }
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
            const float mn = fmaxf(m_run, mt);
            const float corr = m_run == -INFINITY ? 0.f : expf(m_run - mn);
            m_run = mn;
            float ls = 0.f;
            uint32_t pa[4][4];                // P as the A operand: 4 k-steps of 16 keys
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                float pe[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    pe[e] = s[nt][e] == -INFINITY ? 0.f : expf(s[nt][e] - mn);
                    ls += pe[e];
                }
                const __half h0 = __float2half_rn(pe[0]), h1 = __float2half_rn(pe[1]);
                pa[nt >> 1][2 * (nt & 1)] = h2bits(h0, h1);
                pa[nt >> 1][2 * (nt & 1) + 1] =
                    h2bits(__float2half_rn(pe[0] - __half2float(h0)), __float2half_rn(pe[1] - __half2float(h1)));
            }
            l_part = fmaf(l_part, corr, ls);
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                o[n][0] *= corr;
                o[n][1] *= corr;
                o[n][2] *= corr;
                o[n][3] *= corr;
            }
            // values: 4 k-steps of 16 keys x NT n-tiles of 8 dims
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                for (int n = 0; n < NT; n += 2) {
                    uint32_t b0, b1, b2, b3;   // keys 16 kk + {0..7, 8..15} x dims 8 n .. 8 n + 15
                    const int mtx = lane >> 3;
                    ldsm_x4_t(vs + gqa_off<HD>(16 * kk + 8 * (mtx & 1) + (lane & 7), n + (mtx >> 1)), b0, b1, b2, b3);
                    mma16816(o[n], pa[kk], b0, b1);
                    mma16816(o[n + 1], pa[kk], b2, b3);
                }
            }
        }
        __syncthreads();                    // the stage is rewritten two tiles on
    }
    // pair gq of the warp: dims 8 n + 2 tq + e
    float l = l_part + __shfl_xor_sync(0xffffffffu, l_part, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (!live) return;
    if (nz == 1) {
        const float inv = 1.f / l;
        const size_t base = (size_t)tr * nh * HD + (size_t)hr * HD + 2 * tq;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float v = (o[n][e] + o[n][2 + e]) * inv;
                const __half hv = __float2half_rn(v);
                oh[base + 8 * n + e] = hv;
                ol[base + 8 * n + e] = __float2half_rn(v - __half2float(hv));
            }
        }
    } else {
        float *pp = part + (((size_t)tr * nh + hr) * gridDim.z + z) * (HD + 2);
        if (tq == 0) {
            pp[0] = m_run;
            pp[1] = l;
        }
#pragma unroll
        for (int n = 0; n < NT; ++n)
            *reinterpret_cast<float2 *>(pp + 2 + 8 * n + 2 * tq) = make_float2(o[n][0] + o[n][2], o[n][1] + o[n][3]);
    }
}

// The chunks' partials of each (query, head) -> the attention output as fp16 hi / lo halves, chunks
// folded in order (log-sum-exp). CTA = one (query, head), thread d = output dim d.
template <int HD>
__global__ void __launch_bounds__(HD) k_attn_merge(__half *oh, __half *ol, const float *part, int T, int nh, int cap,
                                                   const int *slot_base, int slot_off, int zmax, DevState *st) {
    pdl_enter();
    const int slot0 = block_slot0(slot_base, slot_off, T, cap, st);
    int chunk, nz;
    gqa_chunks(slot0 + T, zmax, chunk, nz);
    if (nz == 1) return;                    // k_attn_gqa wrote the output
    const int t = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    const float *pp = part + ((size_t)t * nh + h) * zmax * (HD + 2);
    float M = -INFINITY;
    for (int z = 0; z < nz; ++z) M = fmaxf(M, pp[(size_t)z * (HD + 2)]);
    float Ls = 0.f, A = 0.f;
    if (M != -INFINITY) {
        for (int z = 0; z < nz; ++z) {
            const float *q = pp + (size_t)z * (HD + 2);
            const float f = q[0] == -INFINITY ? 0.f : expf(q[0] - M);
            Ls = fmaf(q[1], f, Ls);
            A = fmaf(q[2 + d], f, A);
        }
    }
    const float v = A / Ls;
    const __half hv = __float2half_rn(v);
    const size_t idx = (size_t)t * nh * HD + (size_t)h * HD + d;
    oh[idx] = hv;
    ol[idx] = __float2half_rn(v - __half2float(hv));
}

// Attention of a batched decode step: token b of request lanes[b] attends to slots [0, slot] of
// its own cache. CTA = (kv head g, token b): the group's G = nh / nkv query heads share the K / V
// tiles, which go through shared memory as in k_attn_block (64 keys per tile, two in flight, padded
// rows); warp w takes heads g G + w and g G + w + 4 (G <= 8). Output as fp16 hi / lo halves.
constexpr int kBatchHeadsPerWarp = 2;
template <int HD>
__global__ void __launch_bounds__(128) k_attn_batch(__half *oh, __half *ol, const float *q, const BatchLane *lanes,
                                                    int layer, int nh, int nkv, float scale, DevState *st) {
    using L = TreeSmem<HD>;
    extern __shared__ __align__(16) uint8_t tsm[];
    __shared__ __align__(16) float qs[4 * kBatchHeadsPerWarp][HD];
    __shared__ float ps[4 * kBatchHeadsPerWarp][kTreeKeys];
    pdl_enter();
    constexpr int DL = HD / 32;
    constexpr int CH = HD / 8;
    const int g = blockIdx.x, b = blockIdx.y, G = nh / nkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const BatchLane ln = lanes[b];
    int last = ln.slot;
    if (last < 0 || last >= ln.cap) {
        if (threadIdx.x == 0) set_err(st, kErrBadSlot);
        last = min(max(last, 0), ln.cap - 1);
    }
    const size_t head_off = ((size_t)layer * nkv + g) * ln.cap * HD;
    const __half *kb = ln.k + head_off, *vb = ln.v + head_off;
    const int ntiles = last / kTreeKeys + 1;
    auto stage = [&](int tile) {
        uint8_t *ks = tsm + (tile & 1) * 2 * L::kTile, *vs = ks + L::kTile;
        const int k0 = tile * kTreeKeys;
        for (int i = threadIdx.x; i < kTreeKeys * CH; i += 128) {
            const int j = i / CH, c = i - j * CH;
            if (k0 + j <= last) {
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(ks + j * L::kRow + c * 16)),
                             "l"(kb + (size_t)(k0 + j) * HD + c * 8) : "memory");
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(vs + j * L::kRow + c * 16)),
                             "l"(vb + (size_t)(k0 + j) * HD + c * 8) : "memory");
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    stage(0);
    for (int i = threadIdx.x; i < 4 * kBatchHeadsPerWarp * HD; i += 128) {
        const int r = i / HD, d = i - r * HD;               // row r: head g G + (r % 4) + 4 (r / 4)
        const int hl = (r & 3) + 4 * (r >> 2);
        qs[r][d] = hl < G ? q[(size_t)b * nh * HD + (g * G + hl) * HD + d] * scale : 0.f;
    }
    float m[kBatchHeadsPerWarp], l[kBatchHeadsPerWarp], acc[kBatchHeadsPerWarp][DL];
#pragma unroll
    for (int i = 0; i < kBatchHeadsPerWarp; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int d = 0; d < DL; ++d) acc[i][d] = 0.f;
    }
    for (int tile = 0; tile < ntiles; ++tile) {
        if (tile + 1 < ntiles) {
            stage(tile + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const uint8_t *ks = tsm + (tile & 1) * 2 * L::kTile, *vs = ks + L::kTile;
        const int k0 = tile * kTreeKeys;
        const bool in0 = k0 + lane <= last, in1 = k0 + 32 + lane <= last;
        const uint8_t *r0 = ks + lane * L::kRow, *r1 = ks + (lane + 32) * L::kRow;
#pragma unroll
        for (int i = 0; i < kBatchHeadsPerWarp; ++i) {
            const int r = warp + 4 * i;
            if (warp + 4 * i >= G) break;                   // warp-uniform
            float s0 = 0.f, s1 = 0.f;
#pragma unroll 4
            for (int c = 0; c < CH; ++c) {
                const uint4 a = *reinterpret_cast<const uint4 *>(r0 + c * 16);
                const uint4 bb = *reinterpret_cast<const uint4 *>(r1 + c * 16);
                const float4 qa = *reinterpret_cast<const float4 *>(&qs[r][8 * c]);
                const float4 qb = *reinterpret_cast<const float4 *>(&qs[r][8 * c + 4]);
                const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {bb.x, bb.y, bb.z, bb.w};
                const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 fa = __half22float2(*reinterpret_cast<const __half2 *>(&aw[e]));
                    const float2 fb = __half22float2(*reinterpret_cast<const __half2 *>(&bw[e]));
                    s0 = fmaf(qv[2 * e], fa.x, s0);
                    s0 = fmaf(qv[2 * e + 1], fa.y, s0);
                    s1 = fmaf(qv[2 * e], fb.x, s1);
                    s1 = fmaf(qv[2 * e + 1], fb.y, s1);
                }
            }
            const float v0 = in0 ? s0 : -INFINITY, v1 = in1 ? s1 : -INFINITY;
            __syncwarp();
            const float mnew = fmaxf(m[i], warp_max(fmaxf(v0, v1)));
            const float p0 = mnew == -INFINITY ? 0.f : expf(v0 - mnew);
            const float p1 = mnew == -INFINITY ? 0.f : expf(v1 - mnew);
            const float corr = m[i] == -INFINITY ? 0.f : expf(m[i] - mnew);
            l[i] = l[i] * corr + warp_sum(p0 + p1);
            m[i] = mnew;
            ps[r][lane] = p0;
            ps[r][lane + 32] = p1;
#pragma unroll
            for (int d = 0; d < DL; ++d) acc[i][d] *= corr;
        }
        __syncwarp();
        const int nk = min(kTreeKeys, last + 1 - k0);
#pragma unroll 4
        for (int j = 0; j < nk; ++j) {
            const uint8_t *vr = vs + j * L::kRow + lane * DL * 2;
            float vf[DL];
            if constexpr (DL == 4) {
                const uint2 vv = *reinterpret_cast<const uint2 *>(vr);
                const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&vv.x));
                const float2 c = __half22float2(*reinterpret_cast<const __half2 *>(&vv.y));
                vf[0] = a.x;
                vf[1] = a.y;
                vf[2] = c.x;
                vf[3] = c.y;
            } else {
                const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(vr));
                vf[0] = a.x;
                vf[1] = a.y;
            }
#pragma unroll
            for (int i = 0; i < kBatchHeadsPerWarp; ++i) {
                if (warp + 4 * i >= G) break;
                const float pj = ps[warp + 4 * i][j];
#pragma unroll
                for (int d = 0; d < DL; ++d) acc[i][d] = fmaf(pj, vf[d], acc[i][d]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < kBatchHeadsPerWarp; ++i) {
        const int hl = warp + 4 * i;
        if (hl >= G) break;
#pragma unroll
        for (int d = 0; d < DL; ++d) {
            const float o = acc[i][d] / l[i];
            const __half hv = __float2half_rn(o);
            const size_t idx = (size_t)b * nh * HD + (g * G + hl) * HD + lane * DL + d;
            oh[idx] = hv;
            ol[idx] = __float2half_rn(o - __half2float(hv));
        }
    }
}

__global__ void k_batch_advance(BatchLane *lanes, int32_t *tok, int32_t *pos, const int32_t *argmax, int32_t *out,
                                int B, int max_pos, DevState *st) {
    pdl_enter();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int t = argmax[b];
    out[b] = t;
    tok[b] = t;
    const int np = pos[b] + 1, ns = lanes[b].slot + 1;
    if (np >= max_pos || ns >= lanes[b].cap) set_err(st, kErrBadSlot);
    pos[b] = min(np, max_pos - 1);
    lanes[b].slot = min(ns, lanes[b].cap - 1);
}

// The int8 rows and their scales for the batched pass (launch_repack_i8): one thread per 8 inputs
// of a row; the thread of a 32-input block's first 8 writes its scale times 2^k.
__global__ void k_repack_i8(int8_t *dq, __half *dsc, const int8_t *q, const __half *scales, int rows, int N, int K,
                            float p2, int dst_mul, int dst_add, int pair_hd) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)rows * (K / 8)) return;
    const long long e0 = idx * 8;
    const long long r = e0 / K;
    const int k0 = (int)(e0 - r * K);
    long long dr = r * dst_mul + dst_add;
    if (pair_hd > 0) {                                    // RoPE partners adjacent
        const long long hh = r / pair_hd, dd = r - hh * pair_hd;
        dr = hh * pair_hd + (dd < pair_hd / 2 ? 2 * dd : 2 * (dd - pair_hd / 2) + 1);
    }
    *reinterpret_cast<uint2 *>(dq + dr * K + k0) = *reinterpret_cast<const uint2 *>(q + e0);
    if ((k0 & 31) == 0)
        dsc[((size_t)(k0 >> 6) * N + dr) * 2 + ((k0 >> 5) & 1)] = __float2half_rn(__half2float(scales[e0 / 32]) * p2);
}

// max |scale| over n fp16 scales, times 127, into *out (non-negative floats compare as unsigned)
__global__ void k_int8_absmax(float *out, const __half *scales, long long n) {
    float m = 0.f;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(__half2float(scales[i])));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<unsigned *>(out), __float_as_uint(m * 127.0f));
}

}  // namespace

namespace {
size_t up256(size_t v) { return (v + 255) / 256 * 256; }
size_t kmax_of(const PrefillDims &d) {
    return std::max({(size_t)d.hidden, (size_t)d.inter, (size_t)d.heads * d.head_dim});
}
size_t qrows_of(const PrefillDims &d) { return (size_t)(d.heads + 2 * d.kv_heads) * d.head_dim; }
}  // namespace

size_t prefill_scratch_bytes(const PrefillDims &d) {
    const size_t T = d.max_tokens;
    return up256(T * d.hidden * 4) + up256(2 * T * kmax_of(d) * 2) + up256(2 * T * d.inter * 2) +
           up256(T * d.heads * d.head_dim * 4) + up256((size_t)kPrefillLogitRows * d.vocab * 4) + kAttnPartBytes;
}

PrefillScratch prefill_scratch_at(void *base, const PrefillDims &d) {
    const size_t T = d.max_tokens;
    uint8_t *p = static_cast<uint8_t *>(base);
    PrefillScratch s{};
    auto take = [&](size_t bytes) { uint8_t *q = p; p += up256(bytes); return q; };
    s.x = reinterpret_cast<float *>(take(T * d.hidden * 4));
    s.xa = reinterpret_cast<__half *>(take(2 * T * kmax_of(d) * 2));
    s.xb = reinterpret_cast<__half *>(take(2 * T * d.inter * 2));
    s.q = reinterpret_cast<float *>(take(T * d.heads * d.head_dim * 4));
    s.logits = reinterpret_cast<float *>(take((size_t)kPrefillLogitRows * d.vocab * 4));
    s.part = reinterpret_cast<float *>(take(kAttnPartBytes));
    return s;
}

namespace {
// One projection of the chunk: x = rows of `in` (hi at t, lo at max_tokens + t, row stride K).
McolOp proj(const PrefillDims &d, const PrefillScratch &s, const PrefillMat &w, int mode, int N, int K, const __half *in,
            int T, DevState *st) {
    McolOp op{};
    op.mode = mode;
    op.w = w.hi;
    op.w_lo = w.lo;
    op.wq = w.q;
    op.wsc = w.sc;
    op.alpha = w.alpha;
    op.N = N;
    op.K = K;
    op.x = in;
    op.x_rows = 2 * d.max_tokens;
    op.lo_row0 = d.max_tokens;
    op.T = T;
    op.max_ctas = kPrefillMaxCtas;
    op.st = st;
    return op;
}
}  // namespace

cudaError_t launch_prefill_layer_front(const PrefillDims &d, const PrefillLayer &L, const PrefillScratch &s, int T,
                                       const int32_t *pos, const uint64_t *mask, __half *kc, __half *vc, int cap,
                                       const int *slot_base, int slot_off, float scale, const float *rope,
                                       DevState *st, cudaStream_t stream) {
    const int H = d.hidden, QR = (int)qrows_of(d), A = d.heads * d.head_dim;
    const size_t lo = (size_t)d.max_tokens;
    cudaError_t e = launch_pdl(k_rmsnorm_hilo, T, kNormThreads, stream, s.xa, s.xa + lo * H, s.x, L.in_norm, H, d.eps);
    if (e != cudaSuccess) return e;
    // QKV with bias, RoPE and the K/V cache write in the epilogue (q to s.q)
    McolOp qkv = proj(d, s, L.qkv, MC_QKV, QR, H, s.xa, T, st);
    qkv.qkv = McolQkv{L.qkv_b, rope, pos, slot_base, slot_off, cap, d.heads, d.kv_heads, d.head_dim, d.max_pos,
                      s.q, kc, vc};
    e = launch_mcol(qkv, stream, true);
    if (e != cudaSuccess) return e;
    if (mask && T > kShortBlockT) return cudaErrorInvalidValue;    // trees have at most 64 nodes
    if (T <= kShortBlockT && cap <= kShortCacheKeys) {
        // short blocks over a short cache (the cfg2 verify): per (head, 4 queries) CTAs keep more of the
        // GPU busy than the grouped kernel's few CTAs (1.17 against 1.26 ms a 0.5B verify pass)
        const dim3 grid(d.heads, (T + 3) / 4);
        if (d.head_dim == 128)
            e = launch_pdl_smem(k_attn_block<128, 1>, grid, 128, TreeSmem<128>::kBytes, stream, s.xa, s.xa + lo * A,
                                s.q, kc, vc, mask, T, d.heads, d.kv_heads, cap, slot_base, slot_off, scale, st);
        else
            e = launch_pdl_smem(k_attn_block<64, 1>, grid, 128, TreeSmem<64>::kBytes, stream, s.xa, s.xa + lo * A,
                                s.q, kc, vc, mask, T, d.heads, d.kv_heads, cap, slot_base, slot_off, scale, st);
    } else {
        // chunks of the visible keys (at most zmax; the kernels cut the keys on the device): one per
        // 256 keys the cache holds, within the partials' scratch
        const size_t per_chunk = (size_t)T * d.heads * (d.head_dim + 2) * 4;
        const int groups = (T * (d.heads / d.kv_heads) + kGqaPairs - 1) / kGqaPairs;
        const int zmax = (int)std::max<size_t>(1, std::min<size_t>({(size_t)(cap + kGqaChunkKeys - 1) / kGqaChunkKeys,
                                                                     (size_t)kGqaMaxChunks, kAttnPartBytes / per_chunk}));
        const dim3 grid(d.kv_heads, groups, zmax);
        const dim3 mgrid(T, d.heads);
        if (d.head_dim == 128) {
            e = launch_pdl_smem(k_attn_gqa<128>, grid, 128, GqaSmem<128>::kBytes, stream, s.xa, s.xa + lo * A, s.part,
                                s.q, kc, vc, mask, T, d.heads, d.kv_heads, cap, slot_base, slot_off, scale, st);
            if (e == cudaSuccess && zmax > 1)
                e = launch_pdl(k_attn_merge<128>, mgrid, 128, stream, s.xa, s.xa + lo * A, s.part, T, d.heads, cap,
                               slot_base, slot_off, zmax, st);
        } else {
            e = launch_pdl_smem(k_attn_gqa<64>, grid, 128, GqaSmem<64>::kBytes, stream, s.xa, s.xa + lo * A, s.part,
                                s.q, kc, vc, mask, T, d.heads, d.kv_heads, cap, slot_base, slot_off, scale, st);
            if (e == cudaSuccess && zmax > 1)
                e = launch_pdl(k_attn_merge<64>, mgrid, 64, stream, s.xa, s.xa + lo * A, s.part, T, d.heads, cap,
                               slot_base, slot_off, zmax, st);
        }
    }
    if (e != cudaSuccess) return e;
    // O projection into the residual stream
    McolOp o = proj(d, s, L.o, MC_RESID, H, A, s.xa, T, st);
    o.y = s.x;
    o.ldy = H;
    e = launch_mcol(o, stream, true);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t launch_batch_layer_front(const PrefillDims &d, const PrefillLayer &L, const PrefillScratch &s, int B,
                                     const int32_t *pos, const BatchLane *lanes, int layer, float scale,
                                     const float *rope, DevState *st, cudaStream_t stream) {
    const int H = d.hidden, QR = (int)qrows_of(d), A = d.heads * d.head_dim;
    const size_t lo = (size_t)d.max_tokens;
    if (B <= 0 || B > d.max_tokens || !lanes || !pos || d.heads / d.kv_heads > 4 * kBatchHeadsPerWarp)
        return cudaErrorInvalidValue;
    cudaError_t e = launch_pdl(k_rmsnorm_hilo, B, kNormThreads, stream, s.xa, s.xa + lo * H, s.x, L.in_norm, H, d.eps);
    if (e != cudaSuccess) return e;
    McolOp qkv = proj(d, s, L.qkv, MC_QKV, QR, H, s.xa, B, st);
    qkv.qkv = McolQkv{L.qkv_b, rope, pos, nullptr, 0, 0, d.heads, d.kv_heads, d.head_dim, d.max_pos,
                      s.q, nullptr, nullptr, lanes, layer};
    e = launch_mcol(qkv, stream, true);
    if (e != cudaSuccess) return e;
    const dim3 grid(d.kv_heads, B);
    if (d.head_dim == 128)
        e = launch_pdl_smem(k_attn_batch<128>, grid, 128, TreeSmem<128>::kBytes, stream, s.xa, s.xa + lo * A, s.q,
                            lanes, layer, d.heads, d.kv_heads, scale, st);
    else
        e = launch_pdl_smem(k_attn_batch<64>, grid, 128, TreeSmem<64>::kBytes, stream, s.xa, s.xa + lo * A, s.q,
                            lanes, layer, d.heads, d.kv_heads, scale, st);
    if (e != cudaSuccess) return e;
    McolOp o = proj(d, s, L.o, MC_RESID, H, A, s.xa, B, st);
    o.y = s.x;
    o.ldy = H;
    e = launch_mcol(o, stream, true);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t launch_batch_advance(BatchLane *lanes, int32_t *tok, int32_t *pos, const int32_t *argmax, int32_t *out,
                                 int B, int max_pos, DevState *st, cudaStream_t stream) {
    return launch_pdl(k_batch_advance, (B + 127) / 128, 128, stream, lanes, tok, pos, argmax, out, B, max_pos, st);
}

cudaError_t launch_prefill_layer_ffn(const PrefillDims &d, const PrefillLayer &L, const PrefillScratch &s, int T,
                                     DevState *st, cudaStream_t stream) {
    const int H = d.hidden, I = d.inter;
    const size_t lo = (size_t)d.max_tokens;
    cudaError_t e = launch_pdl(k_rmsnorm_hilo, T, kNormThreads, stream, s.xa, s.xa + lo * H, s.x, L.post_norm, H, d.eps);
    if (e != cudaSuccess) return e;
    // gate_up (rows interleaved: 2i gate, 2i + 1 up) -> SiLU(gate) * up as the down projection's input
    McolOp gu = proj(d, s, L.gate_up, MC_SWIGLU, 2 * I, H, s.xa, T, st);
    gu.act_h = s.xb;
    gu.act_l = s.xb + lo * I;
    gu.ld_act = I;
    e = launch_mcol(gu, stream, true);
    if (e != cudaSuccess) return e;
    McolOp dn = proj(d, s, L.down, MC_RESID, H, I, s.xb, T, st);
    dn.y = s.x;
    dn.ldy = H;
    e = launch_mcol(dn, stream, true);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t launch_prefill_embed(const PrefillDims &d, const PrefillScratch &s, const __half *embed,
                                 const int32_t *tok, int T, DevState *st, cudaStream_t stream) {
    return launch_pdl(k_embed_rows, T, 256, stream, s.x, embed, tok, d.hidden, d.vocab, st);
}

// Logits of rows [r0, r0 + n) of the chunk (n <= kPrefillLogitRows) into `out` (row stride vocab):
// final RMSNorm, then the head GEMM.
cudaError_t launch_prefill_logits(const PrefillDims &d, const PrefillScratch &s, const float *final_norm,
                                  const PrefillMat &head, int r0, int n, float *out, DevState *st, cudaStream_t stream) {
    const int H = d.hidden;
    cudaError_t e = launch_pdl(k_rmsnorm_hilo, n, kNormThreads, stream, s.xa, s.xa + (size_t)d.max_tokens * H,
                               s.x + (size_t)r0 * H, final_norm, H, d.eps);
    if (e != cudaSuccess) return e;
    McolOp hd = proj(d, s, head, MC_STORE, d.vocab, H, s.xa, n, st);
    hd.y = out;
    hd.ldy = d.vocab;
    e = launch_mcol(hd, stream, true);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t launch_repack_i8(int8_t *dq, __half *dsc, const int8_t *q, const __half *scales, int rows, int N, int K,
                             int k, int dst_mul, int dst_add, int pair_hd, cudaStream_t s) {
    if (K % 32 || k < 0 || k > 30 || dst_mul < 1 || dst_add < 0 || dst_add >= dst_mul || pair_hd < 0 || pair_hd % 2 ||
        (pair_hd > 0 && (rows % pair_hd || dst_mul != 1)) || (long long)(rows - 1) * dst_mul + dst_add >= N)
        return cudaErrorInvalidValue;
    const long long n = (long long)rows * (K / 8);
    k_repack_i8<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(dq, dsc, q, scales, rows, N, K, ldexpf(1.0f, k), dst_mul,
                                                            dst_add, pair_hd);
    return cudaGetLastError();
}

cudaError_t launch_int8_absmax(float *out, const __half *scales, long long n, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float), s);
    if (e != cudaSuccess) return e;
    k_int8_absmax<<<256, 256, 0, s>>>(out, scales, n);
    return cudaGetLastError();
}

}  // namespace sp
