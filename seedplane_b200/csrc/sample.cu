// Draft-token selection for speculative decoding: per-row top-k of fp32 logits with the row's
// log-sum-exp, so a drafter's candidates and their log-probabilities (value - lse) come from one
// pass over the vocabulary. One CTA per row: every thread keeps a sorted top-k of its strided
// elements and an online (max, sum of exp) pair; the CTA merges the threads' lists by k rounds of
// a block-wide argmax over the list heads. Order: larger value first, lower index on ties (the
// greedy argmax's rule); NaN never enters a list.
#include <cfloat>
#include <climits>
#include <cmath>

#include "kernels.cuh"

namespace sp {

namespace {

constexpr int kTopkThreads = 256;

SP_DEVINL bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

template <int K>
__global__ void __launch_bounds__(kTopkThreads) k_topk_rows(const float *logits, int cols, long long ld, int kout,
                                                            int *idx_out, float *val_out, float *lse_out) {
    __shared__ float s_v[kTopkThreads / 32];
    __shared__ int s_i[kTopkThreads / 32];
    __shared__ int s_t[kTopkThreads / 32];
    __shared__ float s_m[kTopkThreads / 32], s_s[kTopkThreads / 32];
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *r = logits + (size_t)row * ld;
    float tv[K];
    int ti[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
        tv[j] = -INFINITY;
        ti[j] = INT_MAX;
    }
    float m = -INFINITY, s = 0.f;
    for (int c = tid; c < cols; c += kTopkThreads) {
        const float v = __ldg(r + c);
        if (v > m) {                                   // online log-sum-exp (NaN compares false)
            s = s * expf(m - v) + 1.0f;
            m = v;
        } else if (v >= -FLT_MAX) {
            s += expf(v - m);
        }
        if (better(v, c, tv[K - 1], ti[K - 1])) {     // insert into the sorted list
            tv[K - 1] = v;
            ti[K - 1] = c;
#pragma unroll
            for (int j = K - 1; j > 0; --j) {
                if (better(tv[j], ti[j], tv[j - 1], ti[j - 1])) {
                    const float fv = tv[j];
                    tv[j] = tv[j - 1];
                    tv[j - 1] = fv;
                    const int fi = ti[j];
                    ti[j] = ti[j - 1];
                    ti[j - 1] = fi;
                }
            }
        }
    }
    // log-sum-exp across the CTA
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
        const float nm = fmaxf(m, om);
        s = (m == -INFINITY ? 0.f : s * expf(m - nm)) + (om == -INFINITY ? 0.f : os * expf(om - nm));
        m = nm;
    }
    if (lane == 0) {
        s_m[warp] = m;
        s_s[warp] = s;
    }
    // k rounds: the best list head of the CTA wins and its thread advances
    int head = 0;
    for (int round = 0; round < K; ++round) {
        __syncwarp();                                  // reconverged after the previous pop
        float bv = head < K ? tv[0] : -INFINITY;
        int bi = head < K ? ti[0] : INT_MAX;
        int bt = tid;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const int ot = __shfl_xor_sync(0xffffffffu, bt, o);
            if (better(ov, oi, bv, bi)) {
                bv = ov;
                bi = oi;
                bt = ot;
            }
        }
        __syncthreads();                               // the previous round's s_* are consumed
        if (lane == 0) {
            s_v[warp] = bv;
            s_i[warp] = bi;
            s_t[warp] = bt;
        }
        __syncthreads();
        float wv = s_v[0];
        int wi = s_i[0], wt = s_t[0];
        for (int w = 1; w < kTopkThreads / 32; ++w) {
            if (better(s_v[w], s_i[w], wv, wi)) {
                wv = s_v[w];
                wi = s_i[w];
                wt = s_t[w];
            }
        }
        if (tid == 0 && round < kout) {
            idx_out[(size_t)row * kout + round] = wi == INT_MAX ? 0 : wi;
            val_out[(size_t)row * kout + round] = wv;
        }
        if (tid == wt && wi != INT_MAX) {              // pop the winner's head
#pragma unroll
            for (int j = 0; j < K - 1; ++j) {
                tv[j] = tv[j + 1];
                ti[j] = ti[j + 1];
            }
            tv[K - 1] = -INFINITY;
            ti[K - 1] = INT_MAX;
            ++head;
        }
    }
    if (tid == 0) {
        float M = -INFINITY, S = 0.f;
        for (int w = 0; w < kTopkThreads / 32; ++w) {
            const float nm = fmaxf(M, s_m[w]);
            S = (M == -INFINITY ? 0.f : S * expf(M - nm)) + (s_m[w] == -INFINITY ? 0.f : s_s[w] * expf(s_m[w] - nm));
            M = nm;
        }
        lse_out[row] = M == -INFINITY ? -INFINITY : M + logf(S);
    }
}

}  // namespace

cudaError_t launch_topk_rows(const float *logits, int rows, int cols, long long ld, int k, int *idx, float *val,
                             float *lse, cudaStream_t s) {
    if (rows <= 0 || cols <= 0 || k < 1 || k > kTopkMax) return cudaErrorInvalidValue;
    switch (k) {
        case 1: k_topk_rows<1><<<rows, kTopkThreads, 0, s>>>(logits, cols, ld, k, idx, val, lse); break;
        case 2: k_topk_rows<2><<<rows, kTopkThreads, 0, s>>>(logits, cols, ld, k, idx, val, lse); break;
        case 3: case 4: k_topk_rows<4><<<rows, kTopkThreads, 0, s>>>(logits, cols, ld, k, idx, val, lse); break;
        default: k_topk_rows<8><<<rows, kTopkThreads, 0, s>>>(logits, cols, ld, k, idx, val, lse); break;
    }
    return cudaGetLastError();
}

}  // namespace sp
