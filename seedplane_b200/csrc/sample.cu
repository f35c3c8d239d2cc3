// Draft-token selection for speculative decoding: per-row top-k of fp32 logits with the row's
// log-sum-exp, so a drafter's candidates and their log-probabilities (value - lse) come from one
// pass over the vocabulary. One CTA per row: every thread keeps a sorted top-k of its strided
// elements and an online (max, sum of exp) pair; the CTA merges the threads' lists by k rounds of
// a block-wide argmax over the list heads. Order: larger value first, lower index on ties (the
// greedy argmax's rule); NaN never enters a list.
#include <algorithm>
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


// ---------------------------------------------------------------------------------------------
// Stochastic tree acceptance (recursive rejection sampling over a draft tree, temperature T).
//
// Rule (written here; the reference has none, so its CPU restatement in
// oracle/speculative_oracle.py is the oracle): start at the root (row 0 of the logits, the
// distributions after the committed prefix). At a node with target distribution p and drafter
// distribution q, try its children in node order: child x is accepted with probability
// min(1, p(x) / q(x)) (uniform u < p(x) / q(x)); on rejection p becomes max(p - q, 0) normalised
// (unchanged if that is all zero) and the next child is tried. An accepted child becomes the
// current node (rows i + 1: the distributions after node i); when it has no children the pass
// ends with the accepted drafts only. When every child is rejected, one token is drawn from p
// and the pass ends. Every number is fp64 with a fixed operation order, so decisions are
// reproducible bit for bit on the CPU:
//   p_j = e_j / S, e_j = exp((l_j / T) - max), S = sum of e over contiguous blocks of
//   ceil(V / 256) entries (block b summed in index order, then the 256 block sums in order);
//   exp: Cody-Waite reduction by ln 2 (two-part constant) and a degree-13 Taylor polynomial in
//   Horner form, no fused multiply-add, then scaling by 2^k;
//   u: splitmix64 (Vigna) of seed ^ (counter * 0x9E3779B97F4A7C15) advanced once per draw, the
//   top 53 bits times 2^-53; a draw from p walks the same blocks: the first index whose running
//   sum exceeds u * S.
// Launches: four grid-wide kernels give every row the walk can visit (the root's, and those of
// nodes with children) its max, e_j, S and then p (target) or q (drafter) in place; the walk is
// one CTA that reads them. It modifies a row's p in place when a child is rejected, which is safe
// because it visits each row once.
// ---------------------------------------------------------------------------------------------
namespace {

constexpr int kAccThreads = 256;

SP_DEVINL double dexp_ref(double x) {
    // Cody-Waite: x = k ln2 + r, |r| <= ln2 / 2 (ln 2 split in two parts, the published values of
    // fdlibm's e_exp.c); exp(r) by its Taylor series to r^13 / 13!
    const double ln2_hi = 6.93147180369123816490e-01, ln2_lo = 1.90821492927058770002e-10;
    const double inv_ln2 = 1.44269504088896338700e+00;
    if (x < -745.0) return 0.0;
    const double k = rint(__dmul_rn(x, inv_ln2));
    const double r = __dadd_rn(__dadd_rn(x, -__dmul_rn(k, ln2_hi)), -__dmul_rn(k, ln2_lo));
    double pw = 1.0 / 6227020800.0;                 // 1/13!
    const double inv_fact[13] = {1.0 / 479001600.0, 1.0 / 39916800.0, 1.0 / 3628800.0, 1.0 / 362880.0,
                                 1.0 / 40320.0,     1.0 / 5040.0,     1.0 / 720.0,      1.0 / 120.0,
                                 1.0 / 24.0,        1.0 / 6.0,        0.5,              1.0,
                                 1.0};
#pragma unroll
    for (int i = 0; i < 13; ++i) pw = __dadd_rn(__dmul_rn(pw, r), inv_fact[i]);
    return scalbn(pw, (int)k);
}

SP_DEVINL unsigned long long splitmix_next(unsigned long long &s) {
    s += 0x9E3779B97F4A7C15ull;
    unsigned long long z = s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
SP_DEVINL double uniform53(unsigned long long &s) { return (double)(splitmix_next(s) >> 11) * 0x1.0p-53; }

// sum over contiguous blocks (block b = thread b), then the block sums in order (thread 0)
template <typename F>
SP_DEVINL double block_sum(F f, int V, double *s_part) {
    const int B = (V + kAccThreads - 1) / kAccThreads;
    double acc = 0.0;
    for (int i = 0; i < B; ++i) {
        const int j = threadIdx.x * B + i;
        if (j < V) acc = __dadd_rn(acc, f(j));
    }
    s_part[threadIdx.x] = acc;
    __syncthreads();
    double tot = 0.0;
    for (int t = 0; t < kAccThreads; ++t) tot = __dadd_rn(tot, s_part[t]);
    __syncthreads();
    return tot;
}

SP_DEVINL double block_max(const float *row, int V, double inv_t, double *s_part) {
    double m = -INFINITY;
    for (int j = threadIdx.x; j < V; j += kAccThreads) m = fmax(m, __dmul_rn((double)row[j], inv_t));
    s_part[threadIdx.x] = m;
    __syncthreads();
    double mx = -INFINITY;
    for (int t = 0; t < kAccThreads; ++t) mx = fmax(mx, s_part[t]);
    __syncthreads();
    return mx;
}

// ---- the rows' distributions ahead of the walk, over the whole GPU ---------------------------
// The walk can visit the root's row and the rows of nodes with children (nr rows, rows[r] = the
// logits row). For each and for both models (w = 0 target, 1 drafter): MS[w][r] = (max, S) and
// E[w][r][j] = e_j, with the walk's own arithmetic (the same max, exponentials and block-ordered
// sum), so every number the walk reads is the one it would have computed itself.
SP_DEVINL const float *stoch_row(const float *tlog, const float *dlog, long long ld, const int *rows, int nr, int wr) {
    return (wr < nr ? tlog : dlog) + (size_t)rows[wr % nr] * ld;
}

__global__ void __launch_bounds__(kAccThreads) k_stoch_max(const float *tlog, const float *dlog, long long ld, int V,
                                                           const int *rows, int nr, double inv_t, double *MS) {
    __shared__ double s_part[kAccThreads];
    const double m = block_max(stoch_row(tlog, dlog, ld, rows, nr, blockIdx.x), V, inv_t, s_part);
    if (threadIdx.x == 0) MS[2 * blockIdx.x] = m;
}

// grid (2 nr) x chunks: e_j of chunk c of row wr
__global__ void __launch_bounds__(kAccThreads) k_stoch_exp(const float *tlog, const float *dlog, long long ld, int V,
                                                           const int *rows, int nr, double inv_t, const double *MS,
                                                           double *E) {
    const int wr = blockIdx.y;
    const float *row = stoch_row(tlog, dlog, ld, rows, nr, wr);
    const double m = MS[2 * wr];
    double *e = E + (size_t)wr * V;
    for (int j = blockIdx.x * kAccThreads + threadIdx.x; j < V; j += gridDim.x * kAccThreads)
        e[j] = dexp_ref(__dadd_rn(__dmul_rn((double)row[j], inv_t), -m));
}

__global__ void __launch_bounds__(kAccThreads) k_stoch_sum(int V, const double *E, double *MS) {
    __shared__ double s_part[kAccThreads];
    const double *e = E + (size_t)blockIdx.x * V;
    const double S = block_sum([&](int j) { return e[j]; }, V, s_part);
    if (threadIdx.x == 0) MS[2 * blockIdx.x + 1] = S;
}

// the rows' probabilities in place: p_j = e_j / S (target rows), q_j = e_j / S (drafter rows)
__global__ void __launch_bounds__(kAccThreads) k_stoch_div(int V, const double *MS, double *E) {
    const int wr = blockIdx.y;
    const double S = MS[2 * wr + 1];
    double *e = E + (size_t)wr * V;
    for (int j = blockIdx.x * kAccThreads + threadIdx.x; j < V; j += gridDim.x * kAccThreads) e[j] = __ddiv_rn(e[j], S);
}

// The walk's sums: the block structure of block_sum (256 contiguous blocks, each in index order, then
// the block sums in order) with a CTA of kWalkThreads (threads 0-255 sum the blocks).
constexpr int kWalkThreads = 1024;
template <typename F>
SP_DEVINL double walk_sum(F f, int V, double *s_part) {
    if (threadIdx.x < kAccThreads) {
        const int B = (V + kAccThreads - 1) / kAccThreads;
        double acc = 0.0;
        for (int i = 0; i < B; ++i) {
            const int j = threadIdx.x * B + i;
            if (j < V) acc = __dadd_rn(acc, f(j));
        }
        s_part[threadIdx.x] = acc;
    }
    __syncthreads();
    double tot = 0.0;
    for (int t = 0; t < kAccThreads; ++t) tot = __dadd_rn(tot, s_part[t]);
    __syncthreads();
    return tot;
}

__global__ void __launch_bounds__(kWalkThreads) k_accept_stochastic(int V, const int *tok, const int *parent, int n,
                                                                    const int *slot, int nr, double *E,
                                                                    unsigned long long seed, unsigned long long counter,
                                                                    int *out) {
    __shared__ double s_part[kAccThreads];
    __shared__ int s_tok;
    unsigned long long rng = seed ^ (counter * 0x9E3779B97F4A7C15ull);
    int cur = -1;                                         // -1: the root
    int n_out = 0, n_acc = 0;
    for (int depth = 0; depth <= n; ++depth) {
        // the row's p (updated in place on rejections: a row is visited once) and q
        const int r = slot[cur + 1];                          // a row the host listed (the root or a parent)
        double *P = E + (size_t)r * V;
        const double *Q = E + (size_t)(nr + r) * V;
        int next = -1;
        bool any_child = false;
        for (int c = 0; c < n && next < 0; ++c) {
            if (parent[c] != cur) continue;
            any_child = true;
            const int x = tok[c];
            const double q = Q[x];
            const double u = uniform53(rng);                  // the same in every thread
            const double px = P[x];
            if (u < __ddiv_rn(px, q)) {
                next = c;
            } else {                                          // residual max(p - q, 0), normalised
                const double Z = walk_sum([&](int j) { return fmax(__dadd_rn(P[j], -Q[j]), 0.0); }, V, s_part);
                if (Z > 0.0) {
                    for (int j = threadIdx.x; j < V; j += kWalkThreads)
                        P[j] = __ddiv_rn(fmax(__dadd_rn(P[j], -Q[j]), 0.0), Z);
                }
                __syncthreads();
            }
        }
        if (next >= 0) {                                      // accepted: descend
            if (threadIdx.x == 0) {
                out[2 + n_out] = tok[next];
                out[2 + n + 1 + n_acc] = next;
            }
            ++n_out;
            ++n_acc;
            cur = next;
            bool leaf = true;
            for (int c = 0; c < n; ++c) leaf &= parent[c] != cur;
            if (leaf) break;
            continue;
        }
        // every child rejected (or none): draw from p
        const double u = uniform53(rng);
        const double S = walk_sum([&](int j) { return P[j]; }, V, s_part);
        if (threadIdx.x == 0) {
            const double target = __dmul_rn(u, S);
            const int B = (V + kAccThreads - 1) / kAccThreads;
            double run = 0.0;
            int pick = V - 1;
            bool found = false;
            for (int t = 0; t < kAccThreads && !found; ++t) {
                if (__dadd_rn(run, s_part[t]) > target || t == kAccThreads - 1) {
                    for (int i = 0; i < B; ++i) {             // inside block t, in index order
                        const int j = t * B + i;
                        if (j >= V) break;
                        run = __dadd_rn(run, P[j]);
                        if (run > target) {
                            pick = j;
                            found = true;
                            break;
                        }
                    }
                    if (!found) {                             // rounding: the last index of positive
                        int j = min(V - 1, t * B + B - 1);    // probability up to the block's end
                        while (j > 0 && !(P[j] > 0.0)) --j;
                        pick = P[j] > 0.0 ? j : min(V - 1, t * B + B - 1);
                        found = true;
                    }
                } else {
                    run = __dadd_rn(run, s_part[t]);
                }
            }
            s_tok = pick;
            out[2 + n_out] = pick;
        }
        __syncthreads();
        ++n_out;
        (void)any_child;
        break;
    }
    if (threadIdx.x == 0) {
        out[0] = n_out;
        out[1] = n_acc;
    }
}

// ---- top-k / top-p filter of one row (the masking steps of the reference's sample()) ----------
// z = logits / T in fp32. top_k > 0 keeps z >= the k-th largest z (ties at the cut kept, as
// `z < cutoff` drops only smaller values). top_p < 1 then keeps, in descending order, every value
// whose preceding probability mass (softmax over what top-k kept) is at most top_p: the cut is the
// value at which the inclusive mass first exceeds top_p * S (a tie group at the cut stays whole).
// Dropped entries become -inf. One CTA; both cuts are radix selects over order-preserving 32-bit
// keys, 8 bits a pass: by count for top-k, by mass for top-p. Masses are exp(z - max) in fixed
// point (2^44 units, 64-bit integer sums: exact and independent of the atomics' order, so the cut
// is deterministic; the rounding moves a mass by at most V 2^-45 of the largest entry's).
constexpr int kFiltThreads = 1024;
constexpr double kMassScale = 17592186044416.0;      // 2^44

SP_DEVINL uint32_t order_key(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(kFiltThreads) k_sample_filter(const float *logits, int V, float temp, int top_k,
                                                                double top_p, float *z) {
    __shared__ unsigned long long s_bin[256];
    __shared__ unsigned long long s_red[kFiltThreads / 32];
    __shared__ float s_fmax[kFiltThreads / 32];
    __shared__ uint32_t s_digit;
    __shared__ unsigned long long s_rest;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int j = tid; j < V; j += kFiltThreads) z[j] = __fdiv_rn(logits[j], temp);
    __syncthreads();

    // radix select over the keys of the kept entries (key >= lo): the key at which the running
    // weight from the top first reaches `need` (weight 1 per entry: rank; mass: strictly exceeds)
    auto select = [&](uint32_t lo, bool by_mass, float mx, unsigned long long need) -> uint32_t {
        uint32_t prefix = 0u, pmask = 0u;
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int b = tid; b < 256; b += kFiltThreads) s_bin[b] = 0ull;
            __syncthreads();
            // a warp's entries of one bin go in as one atomic (most entries share a few top bins, whose
            // per-entry atomics serialised): the bin's lanes meet by __match_any_sync, the lowest adds
            // their weights (integers: the sum does not depend on the order)
            for (int j = tid; j - lane < V; j += kFiltThreads) {
                uint32_t bin = 256u;
                unsigned long long w = 0ull;
                if (j < V) {
                    const float v = z[j];
                    const uint32_t key = order_key(v);
                    if (key >= lo && (key & pmask) == prefix) {
                        w = by_mass ? __double2ull_rn(exp((double)v - (double)mx) * kMassScale) : 1ull;
                        if (w) bin = (key >> shift) & 255u;
                    }
                }
                const unsigned peers = __match_any_sync(0xffffffffu, bin);
                unsigned long long sum = 0ull;
                if (by_mass) {
                    for (int i = 0; i < 32; ++i) {
                        const unsigned long long wi = __shfl_sync(0xffffffffu, w, i);
                        if ((peers >> i) & 1u) sum += wi;
                    }
                } else {
                    sum = (unsigned long long)__popc(peers);
                }
                if (bin < 256u && lane == __ffs(peers) - 1) atomicAdd(&s_bin[bin], sum);
            }
            __syncthreads();
            if (tid == 0) {
                unsigned long long acc = 0ull;
                int d = 255;
                for (; d > 0; --d) {
                    const unsigned long long nx = acc + s_bin[d];
                    if (by_mass ? nx > need : nx >= need) break;
                    acc = nx;
                }
                s_digit = (uint32_t)d;
                s_rest = need - acc;
            }
            __syncthreads();
            prefix |= s_digit << shift;
            pmask |= 255u << shift;
            need = s_rest;
            __syncthreads();
        }
        return prefix;
    };

    uint32_t cut = 0u;                                    // keep keys >= cut
    if (top_k > 0 && top_k < V) cut = select(0u, false, 0.f, (unsigned long long)top_k);
    if (top_p < 1.0) {
        float m = -INFINITY;
        for (int j = tid; j < V; j += kFiltThreads)
            if (order_key(z[j]) >= cut) m = fmaxf(m, z[j]);
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) s_fmax[warp] = m;
        __syncthreads();
        m = s_fmax[0];
        for (int w = 1; w < kFiltThreads / 32; ++w) m = fmaxf(m, s_fmax[w]);
        unsigned long long tot = 0ull;
        for (int j = tid; j < V; j += kFiltThreads)
            if (order_key(z[j]) >= cut) tot += __double2ull_rn(exp((double)z[j] - (double)m) * kMassScale);
        for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
        if (lane == 0) s_red[warp] = tot;
        __syncthreads();
        tot = 0ull;
        for (int w = 0; w < kFiltThreads / 32; ++w) tot += s_red[w];
        __syncthreads();
        // mass above the cut at most top_p * S: the cut is where the inclusive mass first exceeds it
        const unsigned long long need = (unsigned long long)fmax(0.0, floor(top_p * (double)tot));
        if (need < tot) cut = max(cut, select(cut, true, m, need));
    }
    for (int j = tid; j < V; j += kFiltThreads)
        if (order_key(z[j]) < cut) z[j] = -INFINITY;
}

}  // namespace

cudaError_t launch_sample_filter(const float *logits, int V, double temperature, int top_k, double top_p, float *z,
                                 cudaStream_t s) {
    if (V <= 0 || V > kSampleFilterMaxVocab || !(temperature > 0.0) || top_k < 0 || !(top_p >= 0.0 && top_p <= 1.0))
        return cudaErrorInvalidValue;
    k_sample_filter<<<1, kFiltThreads, 0, s>>>(logits, V, (float)temperature, top_k, top_p, z);
    return cudaGetLastError();
}

cudaError_t launch_accept_stochastic(const float *tlog, const float *dlog, long long ld, int V, const int *tok,
                                     const int *parent, int n, const int *rows, const int *slot, int nr,
                                     double temperature, unsigned long long seed, unsigned long long counter,
                                     double *MS, double *E, int *out, cudaStream_t s) {
    if (V <= 0 || n < 0 || nr < 1 || nr > n + 1 || !(temperature > 0.0)) return cudaErrorInvalidValue;
    const double inv_t = 1.0 / temperature;
    k_stoch_max<<<2 * nr, kAccThreads, 0, s>>>(tlog, dlog, ld, V, rows, nr, inv_t, MS);
    const int chunks = std::max(1, std::min(64, (V + 8 * kAccThreads - 1) / (8 * kAccThreads)));
    k_stoch_exp<<<dim3(chunks, 2 * nr), kAccThreads, 0, s>>>(tlog, dlog, ld, V, rows, nr, inv_t, MS, E);
    k_stoch_sum<<<2 * nr, kAccThreads, 0, s>>>(V, E, MS);
    k_stoch_div<<<dim3(chunks, 2 * nr), kAccThreads, 0, s>>>(V, MS, E);
    k_accept_stochastic<<<1, kWalkThreads, 0, s>>>(V, tok, parent, n, slot, nr, E, seed, counter, out);
    return cudaGetLastError();
}

// ---- greedy acceptance of a verified tree ----------------------------------------------------
// The reference's rule (seedplane/speculative.py:55-92) over per-node target argmaxes: every draft
// path is walked from its root while the target's token after the previous node (after the
// committed prefix for the root) equals the node's token; the first disagreement emits the
// target's token and ends the path; a fully agreed path emits its draft tokens only. The chosen
// path has the most accepted draft tokens, then the most emitted tokens, then the lowest input
// position. One warp: lane j walks paths j, j + 32, ...; the keys (accepted, emitted, -position)
// meet in a warp maximum; lane 0 writes the chosen path's result.
namespace {

SP_DEVINL int greedy_walk(const int *pred, int root_pred, const int *tok, const int *parent, int end, int *chain,
                          int &emitted) {
    int d = 0;
    for (int v = end; v >= 0 && d < kSmallNodes; v = parent[v]) chain[d++] = v;   // end .. root
    int prev = -1, acc = 0;
    emitted = 0;
    for (int i = d - 1; i >= 0; --i) {
        const int nid = chain[i];
        const int want = prev < 0 ? root_pred : pred[prev];
        ++emitted;
        if (want != tok[nid]) return acc;
        ++acc;
        prev = nid;
    }
    return acc;
}

__global__ void __launch_bounds__(32) k_accept_greedy(const int *pred, int root_pred, const int *tok, const int *parent,
                                                      int n, const int *ends, int n_paths, int *out) {
    const int lane = threadIdx.x;
    int chain[kSmallNodes];
    unsigned best = 0u;                     // (accepted << 20) | (emitted << 10) | (1023 - position), + 1
    for (int p = lane; p < n_paths; p += 32) {
        int em = 0;
        const int acc = greedy_walk(pred, root_pred, tok, parent, ends[p], chain, em);
        best = max(best, (((unsigned)acc << 20) | ((unsigned)em << 10) | (unsigned)(1023 - p)) + 1u);
    }
    best = __reduce_max_sync(0xffffffffu, best);
    if (lane != 0) return;
    int *emit = out + 4, *nodes = out + 4 + n + 1;
    if (n_paths == 0) {                     // no draft: one target token
        out[0] = 1;
        out[1] = 0;
        out[2] = -1;
        out[3] = -1;
        emit[0] = root_pred;
        return;
    }
    const int p = 1023 - (int)((best - 1u) & 1023u);
    int d = 0;
    for (int v = ends[p]; v >= 0 && d < kSmallNodes; v = parent[v]) chain[d++] = v;
    int prev = -1, acc = 0, em = 0;
    for (int i = d - 1; i >= 0; --i) {
        const int nid = chain[i];
        const int want = prev < 0 ? root_pred : pred[prev];
        emit[em++] = want;
        if (want != tok[nid]) break;
        nodes[acc++] = nid;
        prev = nid;
    }
    out[0] = em;
    out[1] = acc;
    out[2] = p;
    out[3] = (acc == d && acc > 0) ? pred[prev] : -1;    // the target's token after a fully accepted path
}

}  // namespace

cudaError_t launch_accept_greedy(const int *pred, int root_pred, const int *tok, const int *parent, int n,
                                 const int *ends, int n_paths, int *out, cudaStream_t s) {
    if (n < 0 || n > kSmallNodes || n_paths < 0 || n_paths > kGreedyMaxPaths) return cudaErrorInvalidValue;
    k_accept_greedy<<<1, 32, 0, s>>>(pred, root_pred, tok, parent, n, ends, n_paths, out);
    return cudaGetLastError();
}

}  // namespace sp
