// Batched prompt pass (prefill) for sm_100a: T prompt tokens per chunk through all layers at once.
//
// The projections of T tokens are plain GEMMs, [T, K] x [K, N], compute-bound at prompt lengths,
// so they go to cuBLAS (fp16 operands, fp32 accumulation and output) on row-major copies of the
// weights. Everything around them is this file's kernels: embedding gather, RMSNorm to fp16
// hi / lo halves, bias + RoPE + K/V cache write, causal GQA attention over the cache, SwiGLU.
// The activation of every GEMM is split like the decode step's: hi = fp16(x), lo = fp16(x - hi),
// stacked as 2T columns [hi rows; lo rows] so ONE GEMM reads the weights once, and the epilogues
// add the two halves (W x = W hi + W lo): the products carry ~22 bits of the fp32 activation
// against the fp16 weights — the decode step's precision, which greedy token identity with the
// fp32 reference depends on. The residual stream stays fp32.
//
// The same pass verifies a draft tree: the T tokens are tree nodes (K/V at scratch slots) and
// node t attends to the committed prefix and to the nodes whose bits its ancestor mask holds.
#include <cublas_v2.h>

#include <algorithm>
#include <cmath>

#include "kernels.cuh"

namespace sp {

namespace {

constexpr int kNormThreads = 256;
constexpr int kAttnQ = 16;                  // queries per attention CTA (4 per warp)
constexpr int kAttnKeys = 32;               // keys per staged tile (one per lane)

__device__ __forceinline__ void set_err(DevState *st, int code) {
    if (st) atomicCAS(&st->err, 0, code);
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

// y[t] = [q heads | k heads | v heads] (natural row order): bias, RoPE on q and k with the
// position of token t, q -> fp32, k and v -> the fp16 cache at slot slot0 + t.
__global__ void k_qkv_rope_kv(float *q, __half *kc, __half *vc, const float *y, const float *bias, const float *rope,
                              const int32_t *pos, int T, int nh, int nkv, int hd, int cap, const int *slot_base,
                              int slot_off, int max_pos, DevState *st) {
    const int t = blockIdx.x, half_hd = hd / 2, heads = nh + 2 * nkv;
    const int slot0 = block_slot0(slot_base, slot_off, T, cap, st);
    int p = pos ? pos[t] : slot0 + t;
    if (p < 0 || p >= max_pos) {
        if (threadIdx.x == 0) set_err(st, kErrBadSlot);
        p = min(max(p, 0), max_pos - 1);
    }
    const float *yr = y + (size_t)t * heads * hd, *yl = y + (size_t)(T + t) * heads * hd;
    const int slot = slot0 + t;
    for (int i = threadIdx.x; i < heads * half_hd; i += blockDim.x) {
        const int hh = i / half_hd, d = i - hh * half_hd;
        const int lo = hh * hd + d, hi = lo + half_hd;
        const float a0 = (yr[lo] + yl[lo]) + bias[lo], a1 = (yr[hi] + yl[hi]) + bias[hi];
        if (hh < nh + nkv) {
            const float cs = rope[((size_t)p * half_hd + d) * 2], sn = rope[((size_t)p * half_hd + d) * 2 + 1];
            const float o0 = __fadd_rn(__fmul_rn(a0, cs), -__fmul_rn(a1, sn));
            const float o1 = __fadd_rn(__fmul_rn(a1, cs), __fmul_rn(a0, sn));
            if (hh < nh) {
                q[(size_t)t * nh * hd + lo] = o0;
                q[(size_t)t * nh * hd + hi] = o1;
            } else {
                __half *kr = kc + ((size_t)(hh - nh) * cap + slot) * hd;
                kr[d] = __float2half_rn(o0);
                kr[d + half_hd] = __float2half_rn(o1);
            }
        } else {
            __half *vr = vc + ((size_t)(hh - nh - nkv) * cap + slot) * hd;
            vr[d] = __float2half_rn(a0);
            vr[d + half_hd] = __float2half_rn(a1);
        }
    }
}

// GQA attention of T queries (slots slot0 .. slot0 + T - 1) over the cache. Query t sees the slots
// before slot0 and, among the block's own slots, [slot0, slot0 + t] (causal, mask == null) or the
// slots slot0 + j whose bit j its ancestor mask holds (tree, T <= 64). CTA = (q head, 16 queries),
// warp = 4 queries; keys in tiles of 32 staged
// in shared memory (K rows padded by 8 bytes: lane j reads row j without bank conflicts). Scores,
// online softmax (running max / sum per query) and the value sums in fp32 (the tile's
// probabilities go through shared memory: each lane then sums its dims over the keys); the output
// goes out as fp16 hi / lo halves (the O projection's input).
template <int HD>
__global__ void __launch_bounds__(128) k_attn_prefill(__half *oh, __half *ol, const float *q, const __half *kc,
                                                      const __half *vc, const uint64_t *mask, int T, int nh, int nkv,
                                                      int cap, const int *slot_base, int slot_off, float scale,
                                                      DevState *st) {
    const int slot0 = block_slot0(slot_base, slot_off, T, cap, st);
    constexpr int DL = HD / 32;                       // output dims per lane
    constexpr int KROW = HD * 2 + 8;                  // padded K row (bytes): 8-byte reads, lanes on distinct banks
    __shared__ __align__(16) float qs[kAttnQ][HD];
    __shared__ __align__(16) uint8_t ks[kAttnKeys * KROW];
    __shared__ __align__(16) __half vs[kAttnKeys][HD];
    __shared__ float ps[kAttnQ][kAttnKeys];            // this tile's probabilities
    const int h = blockIdx.x, q0 = blockIdx.y * kAttnQ;
    const int g = h / (nh / nkv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < kAttnQ * HD; i += 128) {
        const int qq = i / HD, d = i - qq * HD;
        qs[qq][d] = q0 + qq < T ? q[(size_t)(q0 + qq) * nh * HD + h * HD + d] * scale : 0.f;
    }
    const __half *kb = kc + (size_t)g * cap * HD, *vb = vc + (size_t)g * cap * HD;
    float m[4], l[4], acc[4][DL];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int d = 0; d < DL; ++d) acc[i][d] = 0.f;
    }
    const int last = slot0 + min(T, q0 + kAttnQ) - 1;    // the last key any query of this CTA sees
    for (int k0 = 0; k0 <= last; k0 += kAttnKeys) {
        __syncthreads();                                  // previous tile consumed (and q staged)
        for (int i = threadIdx.x; i < kAttnKeys * (HD / 8); i += 128) {
            const int j = i / (HD / 8), c = i - j * (HD / 8);
            uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = make_uint4(0u, 0u, 0u, 0u);
            if (k0 + j <= last) {
                kv = *reinterpret_cast<const uint4 *>(kb + (size_t)(k0 + j) * HD + c * 8);
                vv = *reinterpret_cast<const uint4 *>(vb + (size_t)(k0 + j) * HD + c * 8);
            }
            uint32_t *kd = reinterpret_cast<uint32_t *>(ks + (size_t)j * KROW + c * 16);
            kd[0] = kv.x;
            kd[1] = kv.y;
            kd[2] = kv.z;
            kd[3] = kv.w;
            *reinterpret_cast<uint4 *>(&vs[j][c * 8]) = vv;
        }
        __syncthreads();
        __syncwarp();                                     // reconverged before the shuffles below
        // scores: lane = key k0 + lane, four queries of this warp, four dims per step
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        const uint8_t *kr = ks + (size_t)lane * KROW;
#pragma unroll 8
        for (int d = 0; d < HD; d += 4) {
            const uint2 kk = *reinterpret_cast<const uint2 *>(kr + d * 2);
            const float2 ka = __half22float2(*reinterpret_cast<const __half2 *>(&kk.x));
            const float2 kb2 = __half22float2(*reinterpret_cast<const __half2 *>(&kk.y));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 qf = *reinterpret_cast<const float4 *>(&qs[warp * 4 + i][d]);
                s[i] = fmaf(qf.x, ka.x, s[i]);
                s[i] = fmaf(qf.y, ka.y, s[i]);
                s[i] = fmaf(qf.z, kb2.x, s[i]);
                s[i] = fmaf(qf.w, kb2.y, s[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int t = q0 + warp * 4 + i;
            const int key = k0 + lane;
            bool vis = t < T && key <= slot0 + t;
            if (mask && vis && key >= slot0) vis = (mask[t] >> (key - slot0)) & 1ull;
            const float sv = vis ? s[i] : -INFINITY;
            const float mnew = fmaxf(m[i], warp_max(sv));
            const float p = mnew == -INFINITY ? 0.f : expf(sv - mnew);
            const float corr = m[i] == -INFINITY ? 0.f : expf(m[i] - mnew);
            l[i] = l[i] * corr + warp_sum(p);
            m[i] = mnew;
#pragma unroll
            for (int d = 0; d < DL; ++d) acc[i][d] *= corr;
            ps[warp * 4 + i][lane] = p;
        }
        __syncwarp();
        // values: lane = DL dims, keys in order, the warp's four queries per key (probabilities from
        // shared memory, a broadcast; no shuffles, no branches)
        for (int j = 0; j < kAttnKeys; ++j) {
            float vf[DL];
            if constexpr (DL == 4) {
                const uint2 vv = *reinterpret_cast<const uint2 *>(&vs[j][lane * 4]);
                const float2 v0 = __half22float2(*reinterpret_cast<const __half2 *>(&vv.x));
                const float2 v1 = __half22float2(*reinterpret_cast<const __half2 *>(&vv.y));
                vf[0] = v0.x;
                vf[1] = v0.y;
                vf[2] = v1.x;
                vf[3] = v1.y;
            } else {
#pragma unroll
                for (int d = 0; d < DL; ++d) vf[d] = __half2float(vs[j][lane * DL + d]);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float pj = ps[warp * 4 + i][j];
#pragma unroll
                for (int d = 0; d < DL; ++d) acc[i][d] = fmaf(pj, vf[d], acc[i][d]);
            }
        }
        __syncwarp();                                     // ps is rewritten by the next tile
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = q0 + warp * 4 + i;
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

// act = SiLU(gate) * up as fp16 hi / lo; rows t and T + t of y are the two halves of [gate | up]
__global__ void k_swiglu_hilo(__half *ah, __half *al, const float *y, int T, int I) {
    const int t = blockIdx.x;
    const float *g = y + (size_t)t * 2 * I, *u = g + I;
    const float *gl = y + (size_t)(T + t) * 2 * I, *ul = gl + I;
    for (int j = threadIdx.x; j < I; j += blockDim.x) {
        const float y0 = g[j] + gl[j], y1 = u[j] + ul[j];
        const float a = (y0 / (1.0f + expf(-y0))) * y1;
        const __half hv = __float2half_rn(a);
        ah[(size_t)t * I + j] = hv;
        al[(size_t)t * I + j] = __float2half_rn(a - __half2float(hv));
    }
}

// out[t] = y[t] + y[n + t] (rows of `cols`); in place when out == y
__global__ void k_sum_halves(float *out, const float *y, int n, int cols) {
    const int t = blockIdx.y;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < cols; j += gridDim.x * blockDim.x)
        out[(size_t)t * cols + j] = y[(size_t)t * cols + j] + y[(size_t)(n + t) * cols + j];
}

// x[t] += y[t] + y[T + t]: the two halves of a projection into the residual stream
__global__ void k_resid_add(float *x, const float *y, int T, int H) {
    const int t = blockIdx.x;
    for (int j = threadIdx.x; j < H; j += blockDim.x)
        x[(size_t)t * H + j] += y[(size_t)t * H + j] + y[(size_t)(T + t) * H + j];
}

// Y2[2T, N] (row-major) = W[N, K] (row-major) . X2[2T, K]^T, X2 = [hi rows; lo rows]: one GEMM per
// weight half (W = alpha (hi + lo); fp16 checkpoints have no lo half)
cublasStatus_t gemm_stacked(cublasHandle_t hb, const PrefillMat &w, int N, int K, const __half *x2, int T, float *y2) {
    const float zero = 0.0f, one = 1.0f;
    cublasStatus_t st = cublasGemmEx(hb, CUBLAS_OP_T, CUBLAS_OP_N, N, 2 * T, K, &w.alpha, w.hi, CUDA_R_16F, K, x2,
                                     CUDA_R_16F, K, &zero, y2, CUDA_R_32F, N, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
    if (st != CUBLAS_STATUS_SUCCESS || w.lo == nullptr) return st;
    return cublasGemmEx(hb, CUBLAS_OP_T, CUBLAS_OP_N, N, 2 * T, K, &w.alpha, w.lo, CUDA_R_16F, K, x2, CUDA_R_16F, K,
                        &one, y2, CUDA_R_32F, N, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
}

// Y[T, N] (row-major, ldy) = beta * Y + W[N, K] (row-major) . (Xh + Xl)[T, K]^T, one GEMM per input
// half and weight half
cublasStatus_t gemm_hilo(cublasHandle_t hb, const PrefillMat &w, int N, int K, const __half *xh, const __half *xl, int T,
                         float *y, int ldy, float beta) {
    const float one = 1.0f;
    const __half *wh[2] = {w.hi, w.lo};
    const __half *xs[2] = {xh, xl};
    bool first = true;
    for (int i = 0; i < 2; ++i) {
        if (wh[i] == nullptr) continue;
        for (int j = 0; j < 2; ++j) {
            cublasStatus_t st = cublasGemmEx(hb, CUBLAS_OP_T, CUBLAS_OP_N, N, T, K, &w.alpha, wh[i], CUDA_R_16F, K,
                                             xs[j], CUDA_R_16F, K, first ? &beta : &one, y, CUDA_R_32F, ldy,
                                             CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
            if (st != CUBLAS_STATUS_SUCCESS) return st;
            first = false;
        }
    }
    return CUBLAS_STATUS_SUCCESS;
}

// w = q * scale (exact in fp32), times 2^k (exact), split into fp16 hi = fp16(w') and lo =
// fp16(w' - hi): hi + lo = w' exactly while w' and its remainder stay in fp16's normal range, which
// the caller's k arranges for the matrix's largest weights. One thread per 8 inputs of a row.
__global__ void k_dequant_hilo(__half *hi, __half *lo, const int8_t *q, const __half *scales, int rows, int K, float p2) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)rows * (K / 8)) return;
    const long long e0 = idx * 8;
    const float sc = __half2float(scales[e0 / 32]) * p2;
    const uint2 raw = *reinterpret_cast<const uint2 *>(q + e0);
    const int8_t *b = reinterpret_cast<const int8_t *>(&raw);
    __align__(16) __half h[8], l[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float w = (float)b[j] * sc;
        h[j] = __float2half_rn(w);
        l[j] = __float2half_rn(w - __half2float(h[j]));
    }
    *reinterpret_cast<uint4 *>(hi + e0) = *reinterpret_cast<const uint4 *>(h);
    *reinterpret_cast<uint4 *>(lo + e0) = *reinterpret_cast<const uint4 *>(l);
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

size_t prefill_scratch_bytes(const PrefillDims &d) {
    const size_t T = d.max_tokens;
    const size_t kmax = std::max({(size_t)d.hidden, (size_t)d.inter, (size_t)d.heads * d.head_dim});
    const size_t nmax = std::max((size_t)(d.heads + 2 * d.kv_heads) * d.head_dim, 2 * (size_t)d.inter);
    return T * d.hidden * 4 + 2 * T * kmax * 2 + 2 * T * nmax * 4 + T * d.heads * d.head_dim * 4 +
           (size_t)kPrefillLogitRows * d.vocab * 4 + 5 * 256;
}

PrefillScratch prefill_scratch_at(void *base, const PrefillDims &d) {
    auto up = [](size_t v) { return (v + 255) / 256 * 256; };
    const size_t T = d.max_tokens;
    const size_t kmax = std::max({(size_t)d.hidden, (size_t)d.inter, (size_t)d.heads * d.head_dim});
    const size_t nmax = std::max((size_t)(d.heads + 2 * d.kv_heads) * d.head_dim, 2 * (size_t)d.inter);
    uint8_t *p = static_cast<uint8_t *>(base);
    PrefillScratch s{};
    s.x = reinterpret_cast<float *>(p);
    p += up(T * d.hidden * 4);
    s.xh = reinterpret_cast<__half *>(p);      // [2T, kmax] halves: hi rows, then lo rows
    p += up(2 * T * kmax * 2);
    s.xl = nullptr;
    s.y = reinterpret_cast<float *>(p);
    p += up(2 * T * nmax * 4);
    s.q = reinterpret_cast<float *>(p);
    p += up(T * d.heads * d.head_dim * 4);
    s.logits = reinterpret_cast<float *>(p);
    return s;
}

cudaError_t launch_prefill_layer_front(const PrefillDims &d, const PrefillLayer &L, const PrefillScratch &s, int T,
                                       const int32_t *pos, const uint64_t *mask, __half *kc, __half *vc, int cap,
                                       const int *slot_base, int slot_off, float scale, const float *rope,
                                       DevState *st, void *cublas, cudaStream_t stream) {
    cublasHandle_t hb = static_cast<cublasHandle_t>(cublas);
    const int H = d.hidden, QR = (d.heads + 2 * d.kv_heads) * d.head_dim, A = d.heads * d.head_dim;
    k_rmsnorm_hilo<<<T, kNormThreads, 0, stream>>>(s.xh, s.xh + (size_t)T * H, s.x, L.in_norm, H, d.eps);
    if (gemm_stacked(hb, L.qkv, QR, H, s.xh, T, s.y) != CUBLAS_STATUS_SUCCESS) return cudaErrorUnknown;
    k_qkv_rope_kv<<<T, 256, 0, stream>>>(s.q, kc, vc, s.y, L.qkv_b, rope, pos, T, d.heads, d.kv_heads, d.head_dim,
                                         cap, slot_base, slot_off, d.max_pos, st);
    const dim3 grid(d.heads, (T + kAttnQ - 1) / kAttnQ);
    if (d.head_dim == 128)
        k_attn_prefill<128><<<grid, 128, 0, stream>>>(s.xh, s.xh + (size_t)T * A, s.q, kc, vc, mask, T, d.heads,
                                                      d.kv_heads, cap, slot_base, slot_off, scale, st);
    else
        k_attn_prefill<64><<<grid, 128, 0, stream>>>(s.xh, s.xh + (size_t)T * A, s.q, kc, vc, mask, T, d.heads,
                                                     d.kv_heads, cap, slot_base, slot_off, scale, st);
    // O projection into the residual stream
    if (gemm_stacked(hb, L.o, H, A, s.xh, T, s.y) != CUBLAS_STATUS_SUCCESS) return cudaErrorUnknown;
    k_resid_add<<<T, 256, 0, stream>>>(s.x, s.y, T, H);
    return cudaGetLastError();
}

cudaError_t launch_prefill_layer_ffn(const PrefillDims &d, const PrefillLayer &L, const PrefillScratch &s, int T,
                                     void *cublas, cudaStream_t stream) {
    cublasHandle_t hb = static_cast<cublasHandle_t>(cublas);
    const int H = d.hidden, I = d.inter;
    k_rmsnorm_hilo<<<T, kNormThreads, 0, stream>>>(s.xh, s.xh + (size_t)T * H, s.x, L.post_norm, H, d.eps);
    if (gemm_stacked(hb, L.gate_up, 2 * I, H, s.xh, T, s.y) != CUBLAS_STATUS_SUCCESS) return cudaErrorUnknown;
    k_swiglu_hilo<<<T, 256, 0, stream>>>(s.xh, s.xh + (size_t)T * I, s.y, T, I);
    if (gemm_stacked(hb, L.down, H, I, s.xh, T, s.y) != CUBLAS_STATUS_SUCCESS) return cudaErrorUnknown;
    k_resid_add<<<T, 256, 0, stream>>>(s.x, s.y, T, H);
    return cudaGetLastError();
}

cudaError_t launch_prefill_embed(const PrefillDims &d, const PrefillScratch &s, const __half *embed,
                                 const int32_t *tok, int T, DevState *st, cudaStream_t stream) {
    k_embed_rows<<<T, 256, 0, stream>>>(s.x, embed, tok, d.hidden, d.vocab, st);
    return cudaGetLastError();
}

// Logits of rows [r0, r0 + n) of the chunk (n <= kPrefillLogitRows) into `out` (row stride vocab):
// final RMSNorm, then the head GEMM.
cudaError_t launch_prefill_logits(const PrefillDims &d, const PrefillScratch &s, const float *final_norm,
                                  const PrefillMat &head, int r0, int n, float *out, void *cublas, cudaStream_t stream) {
    cublasHandle_t hb = static_cast<cublasHandle_t>(cublas);
    const int H = d.hidden;
    k_rmsnorm_hilo<<<n, kNormThreads, 0, stream>>>(s.xh, s.xh + (size_t)n * H, s.x + (size_t)r0 * H, final_norm, H,
                                                    d.eps);
    if (2 * n <= kPrefillLogitRows) {
        // one pass over the head: [hi rows; lo rows] into the scratch, then the halves summed
        if (gemm_stacked(hb, head, d.vocab, H, s.xh, n, s.logits) != CUBLAS_STATUS_SUCCESS) return cudaErrorUnknown;
        k_sum_halves<<<dim3(64, n), 256, 0, stream>>>(out, s.logits, n, d.vocab);
    } else if (gemm_hilo(hb, head, d.vocab, H, s.xh, s.xh + (size_t)n * H, n, out, d.vocab, 0.0f) !=
               CUBLAS_STATUS_SUCCESS) {
        return cudaErrorUnknown;
    }
    return cudaGetLastError();
}

cudaError_t launch_dequant_hilo(__half *hi, __half *lo, const int8_t *q, const __half *scales, int rows, int K, int k,
                                cudaStream_t s) {
    if (K % 32 || k < -30 || k > 30) return cudaErrorInvalidValue;
    const long long n = (long long)rows * (K / 8);
    k_dequant_hilo<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(hi, lo, q, scales, rows, K, ldexpf(1.0f, k));
    return cudaGetLastError();
}

cudaError_t launch_int8_absmax(float *out, const __half *scales, long long n, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float), s);
    if (e != cudaSuccess) return e;
    k_int8_absmax<<<256, 256, 0, s>>>(out, scales, n);
    return cudaGetLastError();
}

cudaError_t prefill_blas_create(void **handle, void *workspace, size_t workspace_bytes) {
    cublasHandle_t h = nullptr;
    if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS) return cudaErrorUnknown;
    // a fixed workspace: no allocation inside a captured graph
    if (cublasSetWorkspace(h, workspace, workspace_bytes) != CUBLAS_STATUS_SUCCESS) {
        cublasDestroy(h);
        return cudaErrorUnknown;
    }
    *handle = h;
    return cudaSuccess;
}

cudaError_t prefill_blas_stream(void *handle, cudaStream_t s) {
    return cublasSetStream(static_cast<cublasHandle_t>(handle), s) == CUBLAS_STATUS_SUCCESS ? cudaSuccess
                                                                                             : cudaErrorUnknown;
}

void prefill_blas_destroy(void *handle) {
    if (handle) cublasDestroy(static_cast<cublasHandle_t>(handle));
}

}  // namespace sp
