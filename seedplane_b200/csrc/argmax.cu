// Row-wise greedy argmax of fp32 logits (the reference's `sample`: `logits.argmax()`,
// seedplane/qwen_engine.py:147-148; Vulkan native/vulkan_decode/shaders/argmax.comp:8-22), for
// logits that come from outside the fused LM head (all-logits verification, external heads).
//
// A row is split over `ctas` CTAs (HBM-bound: 4 bytes per logit, float4 loads when the row is
// 16-byte aligned). Each CTA reduces its chunk to (max, lowest index), posts it to scratch and
// counts itself in; the last CTA of the row reduces the posted partials and resets the counter,
// so the scratch is clean again when the kernel ends. Lowest index wins ties; NaN compares false
// and is never selected (an all-NaN row yields 0), as in the fused LM-head argmax.
#include <algorithm>
#include <climits>
#include <cmath>

#include "kernels.cuh"

namespace sp {

namespace {

constexpr int kArgmaxThreads = 256;

SP_DEVINL void am_take(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

}  // namespace

__global__ void __launch_bounds__(kArgmaxThreads) k_argmax_rows(const float *logits, int cols, long long ld, int *out,
                                                                const ArgmaxScratch sc) {
    griddep_wait();               // launched after the pass's head GEMM (programmatic launch)
    griddep_launch_dependents();
    __shared__ float s_v[kArgmaxThreads / 32];
    __shared__ int s_i[kArgmaxThreads / 32];
    const int row = blockIdx.y, cta = blockIdx.x, nct = gridDim.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *r = logits + (size_t)row * ld;
    const int per = ((cols + nct - 1) / nct + 3) & ~3;       // multiple of 4: chunks start 16-byte aligned
    const int c0 = min(cols, cta * per), c1 = min(cols, c0 + per);
    float bv = -INFINITY;
    int bi = INT_MAX;
    if ((reinterpret_cast<uintptr_t>(r) & 15) == 0) {
        const int nvec = (c1 - c0) >> 2;
        const float4 *r4 = reinterpret_cast<const float4 *>(r + c0);
        for (int i = tid; i < nvec; i += kArgmaxThreads) {
            const float4 v = __ldg(r4 + i);
            const int j = c0 + 4 * i;
            am_take(bv, bi, v.x, j);
            am_take(bv, bi, v.y, j + 1);
            am_take(bv, bi, v.z, j + 2);
            am_take(bv, bi, v.w, j + 3);
        }
        for (int j = c0 + 4 * nvec + tid; j < c1; j += kArgmaxThreads) am_take(bv, bi, __ldg(r + j), j);
    } else {
        for (int j = c0 + tid; j < c1; j += kArgmaxThreads) am_take(bv, bi, __ldg(r + j), j);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        am_take(bv, bi, ov, oi);
    }
    if (lane == 0) {
        s_v[warp] = bv;
        s_i[warp] = bi;
    }
    __syncthreads();
    if (tid != 0) return;
    for (int w = 1; w < kArgmaxThreads / 32; ++w) am_take(s_v[0], s_i[0], s_v[w], s_i[w]);
    bv = s_v[0];
    bi = s_i[0];
    if (nct == 1) {
        out[row] = bi == INT_MAX ? 0 : bi;
        return;
    }
    sc.val[(size_t)row * kArgmaxMaxCtas + cta] = bv;
    sc.idx[(size_t)row * kArgmaxMaxCtas + cta] = bi;
    __threadfence();
    if (atomicAdd(sc.cnt + row, 1u) != (unsigned)(nct - 1)) return;    // not the row's last CTA
    __threadfence();
    bv = -INFINITY;
    bi = INT_MAX;
    for (int k = 0; k < nct; ++k)
        am_take(bv, bi, __ldcg(sc.val + (size_t)row * kArgmaxMaxCtas + k), __ldcg(sc.idx + (size_t)row * kArgmaxMaxCtas + k));
    out[row] = bi == INT_MAX ? 0 : bi;
    sc.cnt[row] = 0u;
}

int argmax_ctas(int cols) { return std::max(1, std::min(kArgmaxMaxCtas, (cols + 8191) / 8192)); }

size_t argmax_scratch_bytes(int rows) {
    const size_t part = ((size_t)rows * kArgmaxMaxCtas * 4 + 255) & ~(size_t)255;
    return 2 * part + (((size_t)rows * 4 + 255) & ~(size_t)255);
}

ArgmaxScratch argmax_scratch_at(void *base, int rows) {
    const size_t part = ((size_t)rows * kArgmaxMaxCtas * 4 + 255) & ~(size_t)255;
    uint8_t *b = static_cast<uint8_t *>(base);
    ArgmaxScratch s;
    s.val = reinterpret_cast<float *>(b);
    s.idx = reinterpret_cast<int *>(b + part);
    s.cnt = reinterpret_cast<unsigned *>(b + 2 * part);
    return s;
}

// Scratch of the allocation-free entry point (sp_argmax_noalloc): a fixed array in the module's
// global memory, sized for kNoAllocMaxRows rows (val / idx [128][32] + 128 counters = 33,280 B).
// Zero at module load; the caller clears the counters it uses before each launch.
namespace {
constexpr int kNoAllocMaxRows = 128;
constexpr size_t kNoAllocScratchBytes =
    2 * (size_t)kNoAllocMaxRows * kArgmaxMaxCtas * 4 + (size_t)kNoAllocMaxRows * 4;
static __device__ __align__(256) uint8_t g_argmax_scratch[kNoAllocScratchBytes];
}  // namespace

int argmax_noalloc_max_rows() { return kNoAllocMaxRows; }
size_t argmax_noalloc_scratch_bytes() { return kNoAllocScratchBytes; }
cudaError_t argmax_noalloc_scratch(void **base) { return cudaGetSymbolAddress(base, g_argmax_scratch); }

cudaError_t launch_argmax_rows(const float *logits, int rows, int cols, long long ld, int *out, const ArgmaxScratch &sc,
                               cudaStream_t s) {
    if (rows <= 0 || rows > 65535 || cols <= 0 || ld < cols) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(argmax_ctas(cols), rows);
    cfg.blockDim = dim3(kArgmaxThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_argmax_rows, logits, cols, ld, out, sc);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace sp
