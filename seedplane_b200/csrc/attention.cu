// GQA decode attention for sm_100a: one thread-block cluster of kAttnCluster CTAs per kv head.
//
// Each CTA of the cluster owns 1/8 of the visible context [0, slot] and serves all q heads of
// its group. The K/V rows it needs are copied into shared memory with cp.async; rows other than
// the current one are immutable during a step (only the step's own QKV kernel writes row `slot`,
// and `slot` itself is advanced by the previous step), so they are fetched BEFORE the
// programmatic-dependent-launch wait, overlapping the QKV projection. After the wait the CTA
// fetches q and the current row, then per sub-chunk of up to 128 positions:
//   scores  s[j][h] = scale * q_h . k_j   (lane = position, q broadcast from shared memory)
//   softmax running max / sum per head (fp32, online across sub-chunks)
//   values  acc[h][d] += p[j][h] v_j[d]    (thread = output element)
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
constexpr int kMaxGroup = 8;          // q heads per kv head
constexpr int kSub = 128;             // positions per shared-memory sub-chunk

SP_DEVINL void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
SP_DEVINL void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

template <int HD>
struct AttnSmem {
    static constexpr int kRow = HD * 2 + 16;              // padded K row (bank-conflict-free lane-per-row reads)
    static constexpr int vRow = HD * 2;
    static constexpr size_t kOff = 0;
    static constexpr size_t vOff = kOff + (size_t)kSub * kRow;
    static constexpr size_t qOff = vOff + (size_t)kSub * vRow;
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
            cp_async16(sm + L::vOff + (size_t)(j - base) * L::vRow + ch * 16, vb + (size_t)j * HD + ch * 8);
    }
}

}  // namespace

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(const AttnParams p) {
    using L = AttnSmem<HD>;
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

    const int E = G * HD;                   // outputs of this group, thread t owns t, t+256, ...
    float acc[kMaxGroup * HD / kAttnThreads];
#pragma unroll
    for (int k = 0; k < kMaxGroup * HD / kAttnThreads; ++k) acc[k] = 0.f;

    for (int a = j0; a < j1; a += kSub) {
        const int b = min(j1, a + kSub), nj = b - a;
        if (a != j0) {                      // later sub-chunks (long contexts): fetch now
            stage_rows<HD>(sm, kb, vb, a, a, b, tid);
            cp_async_wait_all();
            __syncthreads();
        }
        // ---- scores: lane = position -----------------------------------------------------------
        const int jl = warp * 32 + lane;
        if (jl < nj) {
            float s[kMaxGroup];
#pragma unroll
            for (int h = 0; h < kMaxGroup; ++h) s[h] = 0.f;
            const uint4 *krow = reinterpret_cast<const uint4 *>(sm + L::kOff + (size_t)jl * L::kRow);
#pragma unroll 4
            for (int c8 = 0; c8 < HD / 8; ++c8) {
                const uint4 kv = krow[c8];
                const __half2 *kh = reinterpret_cast<const __half2 *>(&kv);
                float kf[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(kh[e]);
                    kf[2 * e] = f.x;
                    kf[2 * e + 1] = f.y;
                }
#pragma unroll
                for (int h = 0; h < kMaxGroup; ++h) {
                    if (h < G) {
                        const float4 q0 = *reinterpret_cast<const float4 *>(qs + h * HD + 8 * c8);
                        const float4 q1 = *reinterpret_cast<const float4 *>(qs + h * HD + 8 * c8 + 4);
                        float t = s[h];
                        t = fmaf(q0.x, kf[0], t); t = fmaf(q0.y, kf[1], t); t = fmaf(q0.z, kf[2], t); t = fmaf(q0.w, kf[3], t);
                        t = fmaf(q1.x, kf[4], t); t = fmaf(q1.y, kf[5], t); t = fmaf(q1.z, kf[6], t); t = fmaf(q1.w, kf[7], t);
                        s[h] = t;
                    }
                }
            }
            const int j = a + jl;
            const bool vis = !(j >= tree_base && !((mask >> (j - tree_base)) & 1ull));
#pragma unroll
            for (int h = 0; h < kMaxGroup; ++h) sc[jl * kMaxGroup + h] = vis ? s[h] * p.scale : -INFINITY;
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
        // ---- values: thread = output element ----------------------------------------------------
#pragma unroll
        for (int k = 0; k < kMaxGroup * HD / kAttnThreads; ++k) {
            const int e = tid + k * kAttnThreads;
            if (e < E) {
                const int h = e / HD, d = e - h * HD;
                float t = acc[k] * corr[h];
                const __half *vcol = reinterpret_cast<const __half *>(sm + L::vOff) + d;
                for (int q = 0; q < nj; ++q) t = fmaf(sc[q * kMaxGroup + h], __half2float(vcol[(size_t)q * HD]), t);
                acc[k] = t;
            }
        }
        __syncthreads();
    }
    if (tr && tid == 0) tr[2] = globaltimer();
    // ---- this CTA's partial, then the cluster merge ------------------------------------------------
#pragma unroll
    for (int k = 0; k < kMaxGroup * HD / kAttnThreads; ++k) {
        const int e = tid + k * kAttnThreads;
        if (e < E) c_acc[e / HD][e % HD] = acc[k];
    }
    if (tid < G) {
        c_m[tid] = m_run[tid];
        c_l[tid] = l_run[tid];
    }
    if (tr && tid == 0) tr[3] = globaltimer();
    cluster.sync();
    if (tr && tid == 0) tr[4] = globaltimer();
    const int per = (E + nrank - 1) / nrank;
    for (int e = rank * per + tid; e < min(E, (rank + 1) * per); e += kAttnThreads) {
        const int h = e / HD, d = e - h * HD;
        float M = -INFINITY;
        for (int r = 0; r < nrank; ++r) M = fmaxf(M, *cluster.map_shared_rank(&c_m[h], r));
        float Ls = 0.f, A = 0.f;
        for (int r = 0; r < nrank; ++r) {
            const float mr = *cluster.map_shared_rank(&c_m[h], r);
            if (mr == -INFINITY) continue;
            const float f = expf(mr - M);
            Ls = fmaf(*cluster.map_shared_rank(&c_l[h], r), f, Ls);
            A = fmaf(*cluster.map_shared_rank(&c_acc[h][d], r), f, A);
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
