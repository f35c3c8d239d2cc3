// Device helpers shared by the sm_100a kernels: bulk-copy (TMA engine) staging with mbarriers,
// programmatic dependent launch, warp reductions, and the device-side state of one decode step.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#define SP_DEVINL __device__ __forceinline__
#define SP_HOSTDEV __host__ __device__ __forceinline__

namespace sp {

// ---------------------------------------------------------------------------------------------
// Device state of the step sequence. One instance per engine, written by the host-side launch of
// k_set_state before a sequence of step replays, advanced on the device by the LM-head kernel.
// Every kernel of a step reads it after griddepcontrol.wait, so a CUDA graph of one step can be
// replayed for decode, teacher-forced prefill and tree verification alike.
// ---------------------------------------------------------------------------------------------
constexpr int kSmallNodes = 64;          // tree nodes per verify pass (ancestor bitmask = 64 bits)

struct DevState {
    int token;             // token fed at this step
    int pos;               // its RoPE position
    int slot;              // cache slot its K/V is written to
    int step;              // index of this step within the sequence
    int n_forced;          // steps [0, n_forced) take token/pos/slot from the forced sources
    int slot0;             // slot of step 0 (forced step i writes slot0 + i)
    int tree_base;         // slots >= tree_base are speculative nodes (INT32_MAX: none)
    int use_small;         // forced tokens/positions come from small_tok/small_pos
    const int *f_tok;      // forced tokens (device) when !use_small
    const int *f_pos;      // forced positions (device) or null = slot
    float *logits;         // logits destination or null
    long long logits_stride;   // elements between steps (0 = overwrite)
    int logits_from;       // write logits for steps >= logits_from
    int err;               // device-side error code (0 = ok)
    int *out_tokens;       // argmax of every step or null
    int pad_[3];
    int small_tok[kSmallNodes];
    int small_pos[kSmallNodes];
    unsigned long long small_mask[kSmallNodes];   // ancestor-or-self bits over nodes
};

// ---------------------------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------------------------
SP_DEVINL uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

SP_DEVINL void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
SP_DEVINL void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

SP_DEVINL void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
SP_DEVINL void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
SP_DEVINL void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
SP_DEVINL void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
SP_DEVINL void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Non-blocking probe of a phase (mbarrier.try_wait may suspend the thread for a while; this never does).
SP_DEVINL bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok)
                 : "r"(smem_u32(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}

SP_DEVINL bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase. try_wait suspends the thread for a hardware-defined interval
// per attempt, so the bound is a few seconds at most; on expiry the caller gets `false` and is
// expected to record an error and leave without touching the stage.
constexpr uint32_t kMbarSpinLimit = 1u << 22;
SP_DEVINL bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < kMbarSpinLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// 1-D bulk copy global -> shared (TMA engine), completion signalled on `bar` as transaction bytes.
// src, dst 16-byte aligned; bytes a multiple of 16.
SP_DEVINL void bulk_g2s(void *dst_smem, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst_smem)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// Same, with an L2 eviction-priority hint (streamed weights: evict first).
SP_DEVINL void bulk_g2s_hint(void *dst_smem, const void *src, uint32_t bytes, uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(dst_smem)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
SP_DEVINL uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// Warm L2 with [src, src+bytes) (bytes multiple of 16, src 16-byte aligned).
SP_DEVINL void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

SP_DEVINL unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

SP_DEVINL float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
SP_DEVINL float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// fp32 dot of 8 fp16 weights (one 16-byte vector) with 8 fp32 activations.
SP_DEVINL float dot8_f16(const uint4 w, const float4 a, const float4 b, float acc) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&w);
    float2 f0 = __half22float2(h[0]), f1 = __half22float2(h[1]);
    float2 f2 = __half22float2(h[2]), f3 = __half22float2(h[3]);
    acc = fmaf(f0.x, a.x, acc); acc = fmaf(f0.y, a.y, acc);
    acc = fmaf(f1.x, a.z, acc); acc = fmaf(f1.y, a.w, acc);
    acc = fmaf(f2.x, b.x, acc); acc = fmaf(f2.y, b.y, acc);
    acc = fmaf(f3.x, b.z, acc); acc = fmaf(f3.y, b.w, acc);
    return acc;
}

// Device error codes written to DevState::err.
constexpr int kErrMbarTimeout = 1;
constexpr int kErrBadToken = 2;
constexpr int kErrBadSlot = 3;
constexpr int kErrDepTimeout = 4;        // a cross-CTA dependency counter never reached its target

}  // namespace sp
