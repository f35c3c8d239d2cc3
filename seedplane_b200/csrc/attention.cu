// GQA decode attention for sm_100a: one thread-block cluster of kAttnCluster CTAs per kv head.
//
// Each CTA of the cluster owns 1/8 of the visible context [0, slot] and serves all q heads of
// its group. The K/V rows it needs are copied into shared memory with cp.async; rows other than
// the current one are immutable during a step (only the step's own QKV kernel writes row `slot`,
// and `slot` itself is advanced by the previous step), so they are fetched BEFORE the
// programmatic-dependent-launch wait, overlapping the QKV projection. After the wait the CTA
// fetches q and the current row, then per sub-chunk of up to 128 positions:
//   scores  s[j][h] = scale * q_h . k_j   (warp = position, lane = HD/32 dims, q in registers;
//                                          a 3-step butterfly leaves head lane/4 in each lane)
//   softmax running max / sum per head (fp32, online across sub-chunks; warp = head)
//   values  acc[h][d] += p[j][h] v_j[d]    (warp = head, lane = HD/32 dims, 4 partial sums)
// Heads of the group beyond G are computed on a zero q (branch-free inner loops) and dropped.
// The CTAs' partials (max, sum, acc) are merged by log-sum-exp through distributed shared memory.
// Mask: the reference's `key slot <= own slot` (seedplane/qwen_engine.py:131-135), or, for
// speculative nodes (slot >= tree_base), the node's ancestor-or-self bits.
// Replaces native/vulkan_decode/shaders/attn_part.comp:15-44 and attn_combine.comp:8-19.
#include <cmath>

#include <cooperative_groups.h>

#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace sp {

namespace {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kMaxGroup = 8;          // q heads per kv head (== kAttnWarps: softmax/values use warp = head)
constexpr int kSub = 128;             // positions per shared-memory sub-chunk
static_assert(kMaxGroup == kAttnWarps, "one warp per head of the group");

SP_DEVINL void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
SP_DEVINL void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

template <int HD>
struct AttnSmem {
    static constexpr int kRow = HD * 2;                   // K and V rows, fp16, unpadded
    static constexpr size_t kOff = 0;
    static constexpr size_t vOff = kOff + (size_t)kSub * kRow;
    static constexpr size_t qOff = vOff + (size_t)kSub * kRow;
    static constexpr size_t sOff = qOff + (size_t)kMaxGroup * HD * 4;
    static constexpr size_t bytes = sOff + (size_t)kSub * kMaxGroup * 4;
};

// Copy K/V rows [lo, hi) of this kv head into the sub-chunk buffers (row lo -> local row lo - base).
template <int HD>
SP_DEVINL void stage_rows(uint8_t *sm, const __half *kb, const __half *vb, int base, int lo, int hi, int tid) {
    constexpr int kChunks = HD / 8;       // 16-byte chunks per row
    using L = AttnSmem<HD>;
    const int n = hi - lo;
    for (int i = tid; i < n * kChunks * 2; i += kAttnThreads) {
        const int which = i / (n * kChunks);              // 0: K, 1: V
        const int r = (i - which * n * kChunks) / kChunks, ch = i % kChunks;
        const int j = lo + r;
        if (which == 0)
            cp_async16(sm + L::kOff + (size_t)(j - base) * L::kRow + ch * 16, kb + (size_t)j * HD + ch * 8);
        else
            cp_async16(sm + L::vOff + (size_t)(j - base) * L::kRow + ch * 16, vb + (size_t)j * HD + ch * 8);
    }
}

// DL consecutive fp16 values at `p` (8- or 4-byte aligned) as fp32.
template <int DL>
SP_DEVINL void load_dims(const uint8_t *p, float (&f)[DL]) {
    static_assert(DL == 4 || DL == 2, "head_dim 128 or 64");
    if constexpr (DL == 4) {
        const uint2 u = *reinterpret_cast<const uint2 *>(p);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
        f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    } else {
        const uint32_t u = *reinterpret_cast<const uint32_t *>(p);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u));
        f[0] = a.x; f[1] = a.y;
    }
}

// Sum v[h] over the 32 lanes for all 8 heads; lane l returns the sum of head l / 4.
// Three exchange steps halve the values each lane carries (xor 16, 8, 4), two plain steps
// (xor 2, 1) finish the sums: 9 shuffles instead of 40. The summation order is fixed.
SP_DEVINL float reduce_heads(const float (&v)[kMaxGroup], int lane) {
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

}  // namespace

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(const AttnParams p) {
    using L = AttnSmem<HD>;
    constexpr int DL = HD / 32;             // dims per lane
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ float m_run[kMaxGroup], l_run[kMaxGroup], corr[kMaxGroup];
    __shared__ float c_m[kMaxGroup], c_l[kMaxGroup];     // this CTA's partial, read by the cluster
    __shared__ float c_acc[kMaxGroup][HD];

    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank(), nrank = (int)cluster.num_blocks();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = blockIdx.y;
    const int G = p.nh / p.nkv;
    unsigned long long *tr = p.trace ? p.trace + ((size_t)blockIdx.y * gridDim.x + blockIdx.x) * kTraceWords : nullptr;
    if (tr && tid == 0) tr[0] = globaltimer();

    // The step's slot and mask were written before this step began (previous step / set-state).
    const DevState *st = p.st;
    const int slot = st->slot, tree_base = st->tree_base;
    const unsigned long long mask = slot >= tree_base ? st->small_mask[slot - tree_base] : 0ull;
    const int ctx = min(slot + 1, p.cap);
    const int chunk = (ctx + nrank - 1) / nrank;
    const int j0 = min(ctx, rank * chunk), j1 = min(ctx, j0 + chunk);
    const __half *kb = p.kc + (size_t)g * p.cap * HD;
    const __half *vb = p.vc + (size_t)g * p.cap * HD;
    float *qs = reinterpret_cast<float *>(sm + L::qOff);
    float *sc = reinterpret_cast<float *>(sm + L::sOff);

    if (tid < kMaxGroup) {
        m_run[tid] = -INFINITY;
        l_run[tid] = 0.f;
    }
    for (int i = G * HD + tid; i < kMaxGroup * HD; i += kAttnThreads) qs[i] = 0.f;
    // first sub-chunk: every row except the current one can be fetched before the wait
    const int s1 = min(j1, j0 + kSub);
    stage_rows<HD>(sm, kb, vb, j0, j0, min(s1, slot), tid);
    griddep_wait();
    griddep_launch_dependents();
    if (tr && tid == 0) tr[1] = globaltimer();
    if (slot >= j0 && slot < s1) stage_rows<HD>(sm, kb, vb, j0, slot, slot + 1, tid);
    for (int i = tid; i < G * HD / 4; i += kAttnThreads)
        cp_async16(qs + 4 * i, p.q + (size_t)g * G * HD + 4 * i);
    cp_async_wait_all();
    __syncthreads();
    if (tr && tid == 0) tr[6] = globaltimer();

    float qr[kMaxGroup][DL];                // this lane's dims of every head's q
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
#pragma unroll
        for (int i = 0; i < DL; ++i) qr[h][i] = qs[h * HD + DL * lane + i];
    float acc[DL];                          // warp = head (< G), lane = dims [DL*lane, DL*lane + DL)
#pragma unroll
    for (int i = 0; i < DL; ++i) acc[i] = 0.f;

    for (int a = j0; a < j1; a += kSub) {
        const int b = min(j1, a + kSub), nj = b - a;
        if (a != j0) {                      // later sub-chunks (long contexts): fetch now
            stage_rows<HD>(sm, kb, vb, a, a, b, tid);
            cp_async_wait_all();
            __syncthreads();
        }
        // ---- scores: warp = position, two positions in flight --------------------------------------
        for (int jl = warp; jl < nj; jl += 2 * kAttnWarps) {
            const int jl2 = jl + kAttnWarps;
            const bool has2 = jl2 < nj;     // warp-uniform
            float k1[DL], k2[DL];
            load_dims<DL>(sm + L::kOff + (size_t)jl * L::kRow + lane * DL * 2, k1);
            if (has2) {
                load_dims<DL>(sm + L::kOff + (size_t)jl2 * L::kRow + lane * DL * 2, k2);
            } else {
#pragma unroll
                for (int i = 0; i < DL; ++i) k2[i] = 0.f;
            }
            float v1[kMaxGroup], v2[kMaxGroup];
#pragma unroll
            for (int h = 0; h < kMaxGroup; ++h) {
                float t1 = qr[h][0] * k1[0], t2 = qr[h][0] * k2[0];
#pragma unroll
                for (int i = 1; i < DL; ++i) {
                    t1 = fmaf(qr[h][i], k1[i], t1);
                    t2 = fmaf(qr[h][i], k2[i], t2);
                }
                v1[h] = t1;
                v2[h] = t2;
            }
            const float s1v = reduce_heads(v1, lane), s2v = reduce_heads(v2, lane);
            if ((lane & 3) == 0) {
                const int h = lane >> 2;
                const int j = a + jl, j2 = a + jl2;
                const bool vis1 = !(j >= tree_base && !((mask >> (j - tree_base)) & 1ull));
                sc[jl * kMaxGroup + h] = vis1 ? s1v * p.scale : -INFINITY;
                if (has2) {
                    const bool vis2 = !(j2 >= tree_base && !((mask >> (j2 - tree_base)) & 1ull));
                    sc[jl2 * kMaxGroup + h] = vis2 ? s2v * p.scale : -INFINITY;
                }
            }
        }
        __syncthreads();
        if (tr && tid == 0 && a == j0) tr[7] = globaltimer();
        // ---- softmax statistics: warp h owns head h ----------------------------------------------
        if (warp < G) {
            const int h = warp;
            float mx = -INFINITY;
            for (int q = lane; q < nj; q += 32) mx = fmaxf(mx, sc[q * kMaxGroup + h]);
            mx = warp_max(mx);
            const float mold = m_run[h];
            const float mnew = fmaxf(mold, mx);
            float ls = 0.f;
            for (int q = lane; q < nj; q += 32) {
                const float pe = mnew == -INFINITY ? 0.f : expf(sc[q * kMaxGroup + h] - mnew);
                sc[q * kMaxGroup + h] = pe;
                ls += pe;
            }
            ls = warp_sum(ls);
            if (lane == 0) {
                const float cf = mold == -INFINITY ? 0.f : expf(mold - mnew);
                corr[h] = cf;
                l_run[h] = l_run[h] * cf + ls;
                m_run[h] = mnew;
            }
        }
        __syncthreads();
        if (tr && tid == 0 && a == j0) tr[8] = globaltimer();
        // ---- values: warp h owns head h, four independent partial sums ---------------------------
        if (warp < G) {
            const int h = warp;
            float part[4][DL];
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int i = 0; i < DL; ++i) part[u][i] = 0.f;
            const uint8_t *vrow = sm + L::vOff + lane * DL * 2;
            int q = 0;
            for (; q + 4 <= nj; q += 4) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float pe = sc[(q + u) * kMaxGroup + h];
                    float vf[DL];
                    load_dims<DL>(vrow + (size_t)(q + u) * L::kRow, vf);
#pragma unroll
                    for (int i = 0; i < DL; ++i) part[u][i] = fmaf(pe, vf[i], part[u][i]);
                }
            }
            for (; q < nj; ++q) {
                const float pe = sc[q * kMaxGroup + h];
                float vf[DL];
                load_dims<DL>(vrow + (size_t)q * L::kRow, vf);
#pragma unroll
                for (int i = 0; i < DL; ++i) part[0][i] = fmaf(pe, vf[i], part[0][i]);
            }
            const float cf = corr[h];
#pragma unroll
            for (int i = 0; i < DL; ++i) acc[i] = fmaf(acc[i], cf, (part[0][i] + part[1][i]) + (part[2][i] + part[3][i]));
        }
        __syncthreads();
    }
    if (tr && tid == 0) tr[2] = globaltimer();
    // ---- this CTA's partial, then the cluster merge ------------------------------------------------
    if (warp < G) {
#pragma unroll
        for (int i = 0; i < DL; ++i) c_acc[warp][DL * lane + i] = acc[i];
    }
    if (tid < G) {
        c_m[tid] = m_run[tid];
        c_l[tid] = l_run[tid];
    }
    if (tr && tid == 0) tr[3] = globaltimer();
    cluster.sync();
    if (tr && tid == 0) tr[4] = globaltimer();
    const int E = G * HD;
    const int per = (E + kAttnCluster - 1) / kAttnCluster;
    for (int e = rank * per + tid; e < min(E, (rank + 1) * per); e += kAttnThreads) {
        const int h = e / HD, d = e - h * HD;
        float mr[kAttnCluster], lr[kAttnCluster], ar[kAttnCluster];
#pragma unroll
        for (int r = 0; r < kAttnCluster; ++r) {
            mr[r] = *cluster.map_shared_rank(&c_m[h], r);
            lr[r] = *cluster.map_shared_rank(&c_l[h], r);
            ar[r] = *cluster.map_shared_rank(&c_acc[h][d], r);
        }
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < kAttnCluster; ++r) M = fmaxf(M, mr[r]);
        float Ls = 0.f, A = 0.f;
#pragma unroll
        for (int r = 0; r < kAttnCluster; ++r) {
            const float f = mr[r] == -INFINITY ? 0.f : expf(mr[r] - M);
            Ls = fmaf(lr[r], f, Ls);
            A = fmaf(ar[r], f, A);
        }
        p.out[(g * G + h) * HD + d] = A / Ls;
    }
    if (tr && tid == 0) tr[5] = globaltimer();
    cluster.sync();      // keep this CTA's shared memory alive until the cluster has read it
}

template <int HD>
static cudaError_t launch_attention_t(const AttnParams &p, const LaunchCfg *lc) {
    const size_t smem = AttnSmem<HD>::bytes;
    if (lc == nullptr) {
        cudaError_t e = cudaFuncSetAttribute(k_attn_decode<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        return cudaFuncSetAttribute(k_attn_decode<HD>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    (int)cudaSharedmemCarveoutMaxShared);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kAttnCluster, p.nkv);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = lc->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kAttnCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = lc->pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, k_attn_decode<HD>, p);
}

cudaError_t prepare_attention() {
    cudaError_t e = launch_attention_t<128>(AttnParams{}, nullptr);
    if (e != cudaSuccess) return e;
    return launch_attention_t<64>(AttnParams{}, nullptr);
}

cudaError_t launch_attention(const AttnParams &p, const LaunchCfg &lc) {
    if (p.nh / p.nkv > kMaxGroup) return cudaErrorInvalidValue;
    if (p.hd == 128) return launch_attention_t<128>(p, &lc);
    if (p.hd == 64) return launch_attention_t<64>(p, &lc);
    return cudaErrorInvalidValue;
}

}  // namespace sp
