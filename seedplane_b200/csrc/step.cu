// Persistent decode step for sm_100a: one launch per token, one CTA per SM.
//
// The kernel walks the step's op table (per layer: QKV GEMV, attention, O GEMV, gate_up GEMV,
// down GEMV; then the LM head). Batch-1 decode reads every weight once per token; it is bound by
// HBM bandwidth and by the latency of the hand-offs between ops, so the design is about moving
// bytes and hiding latency:
//
//   rows       every CTA owns whole output rows of every GEMV (row pairs, so a RoPE pair or a
//              gate/up pair stays in one thread): no split-K, no cross-CTA partial sums. Its rows
//              are packed as units of (up to 64 rows) x (a chunk of the inputs), one ring stage
//              at most.
//   warp 4     (producer) streams ALL of the CTA's units of the step, op after op, through a
//              ring of stages with 1-D bulk copies (one copy per unit). It never waits for data,
//              only for a free stage, so weights stream while the other warps wait for
//              activations; it starts while the previous step is still finishing (programmatic
//              dependent launch).
//   warps 0-3  per GEMV op: build the input vector in shared memory as fp16 hi / lo halves
//              (RMSNorm fused), multiply each unit on the tensor cores (mma.sync m16n8k16:
//              A = 16 weight rows from the swizzled unit, B = the hi / lo columns), add up the
//              four warps' k-step partials in shared memory and run the pair epilogue (bias +
//              RoPE + K/V write / residual add / SwiGLU / logits + argmax).
//              Attention: the last nh * chunks CTAs each compute one (q head, context chunk)
//              item and publish an unnormalised partial (max, sum, acc); the chunk-0 item of a
//              head merges the head's chunks (log-sum-exp, fixed order).
//
// Hand-offs. The vectors that the CTAs of the next op read (the residual stream x, q, the new
// K/V rows, attention partials and the attention output) are LL words: one 64-bit store carries
// a 32-bit payload and the 32-bit tag of the writing op and step. A reader polls the words
// themselves until every tag matches, so a hand-off costs about one L2 round trip and no fence.
// The SwiGLU activation (the largest vector, read whole by every down-projection CTA) is plain
// fp16 hi / lo published through a 64-bit counter: its writers meet at a barrier, one thread
// release-adds, a reader acquires. Counters never reset: the target is CTAs x (epoch + 1), where
// the epoch counts finished steps (advanced by the LM head's last CTA). Buffers alternate by
// layer parity. All data another CTA produced is read through L2. Every wait is bounded; on
// expiry the CTA records an error in DevState::err, sets its abort flag and runs to the end
// without waiting again, so the kernel always terminates.
#include <algorithm>
#include <climits>
#include <cmath>
#include <type_traits>

#include "kernels.cuh"
#include "tc.cuh"

namespace sp {

namespace {

constexpr int kEpiThreads = 128;            // warps 0-3: compute, epilogues, attention
constexpr int kProducerWarp = 4;
constexpr int kThreads = kEpiThreads + 32;
constexpr int kMaxStageBytes = 64 * 1024;   // one unit per stage (a bulk copy costs about the same
                                            // time whatever its size, so big ones ingest faster)
constexpr int kPassRows = kStepPassRows;    // rows per pass: 16 per warp
constexpr int kPassRowsI8 = 128;            // int8 passes: one M = 128 tensor-core tile
constexpr int kUnitBlocksI8 = 32;           // int8 32-input blocks per unit: 8 TMEM columns each
constexpr uint32_t kStepTmemCols = 2 * 8 * kUnitBlocksI8;   // two unit buffers
static_assert(kPassRowsI8 <= 4 * kPassRows, "int8 pass rows go through red[]");
constexpr int kGroup = 8;                   // q heads per kv head at most
constexpr int kGroupTileRows = 64;          // grouped attention items: positions per chunk at least
constexpr int kNormRegs = 8;                // float4s per thread in the RMSNorm prologue: K <= 4096
constexpr int kLLBatch = 7;                 // LL word pairs per thread in flight (plain prologues, merge)
constexpr int kMergeBatch = 32;            // attention chunks merged per batch (staged in shared memory)
constexpr uint32_t kDepSpinLimit = 1u << 22;
constexpr int kOpWords = (int)(sizeof(StepOp) / 16);
static_assert(kLLBatch <= 32, "poll masks are 32-bit");
static_assert(kStepAttnRows <= kEpiThreads - 32, "attention scores run on threads 32 ..");

SP_DEVINL void ldmatrix_x4(uint32_t addr, uint32_t &a0, uint32_t &a1, uint32_t &a2, uint32_t &a3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3)
                 : "r"(addr));
}
// D (16x8 fp32) += A (16x16 fp16, row-major) * B (16x8 fp16, column-major)
SP_DEVINL void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// x[k .. k + 3] -> hi = fp16(x), lo = fp16(x - hi)
SP_DEVINL void store_hilo4(__half *xh, __half *xl, int k, float4 v) {
    const __half2 h01 = __floats2half2_rn(v.x, v.y), h23 = __floats2half2_rn(v.z, v.w);
    const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
    const __half2 l01 = __floats2half2_rn(v.x - f01.x, v.y - f01.y), l23 = __floats2half2_rn(v.z - f23.x, v.w - f23.y);
    *reinterpret_cast<__half2 *>(xh + k) = h01;
    *reinterpret_cast<__half2 *>(xh + k + 2) = h23;
    *reinterpret_cast<__half2 *>(xl + k) = l01;
    *reinterpret_cast<__half2 *>(xl + k + 2) = l23;
}

// One weight unit of a pass through the tensor cores. This warp takes k-steps warp, warp + 4, ...
// in groups of U (= 4 / row tiles): accumulator slot sl = rt * U + u holds row tile rt's sum over
// the group's u-th k-step, so four independent MMA chains run and four ldmatrix are in flight.
template <int U>
SP_DEVINL void unit_mma(float (&d)[4][4], uint32_t unit, int rs, int nks, int rows_p, int nrt, int q0, const __half *xh,
                        const __half *xl, int warp, int lane) {
    const int lm = lane >> 3, lr = lane & 7;               // ldmatrix: matrix, row within it
    for (int ks = warp; ks < nks; ks += 4 * U) {
        uint32_t b[U][2];
        uint32_t a[4][4];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            b[u][0] = 0u;
            b[u][1] = 0u;
            const int kk = ks + 4 * u;
            if (kk < nks && lane < 8) {                     // B column 0 = hi, column 1 = lo
                const __half *xv = lane < 4 ? xh : xl;
                const int kr = q0 + 16 * kk + 2 * (lane & 3);
                b[u][0] = *reinterpret_cast<const uint32_t *>(xv + kr);
                b[u][1] = *reinterpret_cast<const uint32_t *>(xv + kr + 8);
            }
        }
#pragma unroll
        for (int sl = 0; sl < 4; ++sl) {
            const int rt = sl / U, kk = ks + 4 * (sl % U);
            if (rt < nrt && kk < nks) {
                const int r = min(rt * 16 + ((lm & 1) << 3) + lr, rows_p - 1);
                const int j = 2 * kk + (lm >> 1);           // 16-byte chunk of the row
                const int pj = (j & ~7) | ((j & 7) ^ (r & 7));
                ldmatrix_x4(unit + (uint32_t)(r * rs + pj * 16), a[sl][0], a[sl][1], a[sl][2], a[sl][3]);
            }
        }
#pragma unroll
        for (int sl = 0; sl < 4; ++sl) {
            const int rt = sl / U, kk = ks + 4 * (sl % U);
            if (rt < nrt && kk < nks) mma_16816(d[sl], a[sl][0], a[sl][1], a[sl][2], a[sl][3], b[sl % U][0], b[sl % U][1]);
        }
    }
}

// Integer digits of a GEMV input for int8 weights. A 32-input block with max |x| in [2^E, 2^E+1)
// gets the scale 2^(E - 26): q = rint(x * 2^(26 - E)) is an integer below 2^27 in magnitude, written
// as q = d0 2^21 + d1 2^14 + d2 2^7 + d3 with d0 in [-64, 63] and d1..d3 in [0, 127] (the bits of
// q), so every digit is an int8 and x = scale * q to 2^-28 of the block's largest input. Layout:
// 128 bytes per block, [half h][digit c][16 inputs] (input k at (k / 32) * 128 + ((k / 16) & 1) *
// 64 + c * 16 + k % 16): each 16-input half is a K-major 8-row core matrix whose rows 0-3 are the
// digits (rows 4-7, the next 64 bytes, give output columns that are not read). The block's scale
// goes to bsc[k / 32]. The 32 inputs of a block are the float4s of 8 consecutive lanes (lane & 7 =
// position in the block); the whole warp calls digitize4_n.
// This thread's N float4s, x[u] = inputs k0 + u * kstride .. + 3 for the u with bit u of vmask set
// (warp-uniform), into digits: the N block maxima first (N shuffle chains interleaved after one reconvergence),
// then the N conversions; one float4 at a time would serialise N latency chains.
template <int N>
SP_DEVINL void digitize4_n(const float4 (&x)[N], int k0, int kstride, uint32_t vmask, int8_t *dg, float *bsc) {
    float m[N];
#pragma unroll
    for (int u = 0; u < N; ++u) m[u] = fmaxf(fmaxf(fabsf(x[u].x), fabsf(x[u].y)), fmaxf(fabsf(x[u].z), fabsf(x[u].w)));
    __syncwarp();                   // a warp left split by earlier divergent code pays ~8x per shuffle
#pragma unroll
    for (int sh = 1; sh <= 4; sh <<= 1)
#pragma unroll
        for (int u = 0; u < N; ++u) m[u] = fmaxf(m[u], __shfl_xor_sync(0xffffffffu, m[u], sh));
#pragma unroll
    for (int u = 0; u < N; ++u) {
        if ((vmask >> u) & 1u) {
            const int k = k0 + u * kstride;
            // biased exponent of m, at least 26 (blocks below 2^-101 become zero: multiplier 2^127)
            const int eb = max((int)((__float_as_uint(m[u]) >> 23) & 0xffu), 26);
            const float mul = __uint_as_float((uint32_t)(280 - eb) << 23);       // 2^(153 - eb)
            if ((threadIdx.x & 7) == 0) bsc[k >> 5] = __uint_as_float((uint32_t)(eb - 26) << 23);   // 2^(eb - 153)
            uint32_t sp[4];
            const float xv[4] = {x[u].x, x[u].y, x[u].z, x[u].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int q = __float2int_rn(xv[e] * mul);
                // bytes (low to high): d3, d2, d1, d0 = q's 7-bit groups, the top one signed
                sp[e] = ((uint32_t)q & 0x7fu) | (((uint32_t)q << 1) & 0x7f00u) | (((uint32_t)q << 2) & 0x7f0000u) |
                        (((uint32_t)q << 3) & 0xff000000u);
            }
            // transpose: word c = byte (3 - c) of the four inputs (c = 0: the top digit)
            const uint32_t t0 = __byte_perm(sp[0], sp[1], 0x5140), t1 = __byte_perm(sp[0], sp[1], 0x7362);
            const uint32_t t2 = __byte_perm(sp[2], sp[3], 0x5140), t3 = __byte_perm(sp[2], sp[3], 0x7362);
            int8_t *w = dg + (k >> 5) * 128 + ((k >> 4) & 1) * 64 + (k & 15);
            *reinterpret_cast<uint32_t *>(w) = __byte_perm(t1, t3, 0x7632);
            *reinterpret_cast<uint32_t *>(w + 16) = __byte_perm(t1, t3, 0x5410);
            *reinterpret_cast<uint32_t *>(w + 32) = __byte_perm(t0, t2, 0x7632);
            *reinterpret_cast<uint32_t *>(w + 48) = __byte_perm(t0, t2, 0x5410);
        }
    }
}

// The MMAs of one int8 unit. A unit of rows_p rows x 32 nb inputs holds, per 32-input
// block b, the rows' 32 bytes as two K-major halves: [half][row][16 bytes] (rows at 16 B, 8-row
// core groups 128 B apart, halves rows_p * 16 B apart; no padding rows: the rows past rows_p of the
// M = 64 or 128 tile read whatever follows and land in TMEM lanes nobody reads), then the scales
// [row][block] fp16. Block b: D (TMEM columns 8b .. 8b + 7) = A (M x 32 s8) * B (the 8-row digit
// cores of the same 32 inputs), exact s32, not accumulated: every block keeps its own sums. M = 64
// for passes of at most 64 rows (~32 cycles of tensor core per MMA, ~48 for M = 128, whatever the
// row count). Issued by lane 0 of each compute warp w for blocks w, w + 4, ... (four issuers keep
// the tensor core fed), descriptors advanced in place.
SP_DEVINL void unit_i8_issue(uint32_t tmem, uint32_t unit, int rows_p, int nb, uint32_t dgb, int b0) {
    const uint32_t idesc = rows_p <= 64 ? kIdescI8M64N8 : kIdescI8M128N8;
    uint64_t ad = smem_desc(unit + (uint32_t)(b0 * rows_p * 32), (uint32_t)(rows_p * 16), 128);
    uint64_t bd = smem_desc(dgb + (uint32_t)(b0 * 128), 64, 128);
    const uint64_t da = (uint64_t)((4 * rows_p * 32) >> 4), db = (uint64_t)((4 * 128) >> 4);
    uint32_t t = tmem + (uint32_t)(8 * b0);
    for (int b = b0; b < nb; b += 4) {
        mma_i8(t, ad, bd, idesc);
        ad += da;                                           // start-address field (bits 0-13) only
        bd += db;
        t += 32;
    }
}

// This thread's row (its TMEM lane) of one int8 unit of nb blocks (nb even): sum over blocks b of
// row scale (sc2: fp16 pairs of blocks 2j, 2j + 1) * input block scale * (2^14 (128 d0 + d1) +
// (128 d2 + d3)), the d's the block's digit columns 0-3 (the pairs are exact in s32), in fp32 and
// block order. Whole warp (tcgen05.ld is warp-wide): one 32-column load per 4 blocks (the
// readout's cost follows the number of load instructions: x16 pairs were 2 % slower). A last pair
// of blocks reads 16 columns past them, inside the unit's buffer.
SP_DEVINL float unit_i8_row(uint32_t tmem_lane, const uint32_t (&sc2)[kUnitBlocksI8 / 2], int nb, const float *bsc) {
    float y = 0.f;
#pragma unroll
    for (int b0 = 0; b0 < kUnitBlocksI8; b0 += 4) {
        if (b0 < nb) {                                          // warp-uniform
            uint32_t v[32];
            tmem_ld32_nowait(tmem_lane + (uint32_t)(8 * b0), v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int b = b0 + e;
                if (b < nb) {
                    const uint32_t *r = &v[8 * e];
                    const int hi = (int)r[0] * 128 + (int)r[1], lo = (int)r[2] * 128 + (int)r[3];
                    const float ds = fmaf(16384.f, (float)hi, (float)lo);
                    const __half2 s2 = *reinterpret_cast<const __half2 *>(&sc2[b >> 1]);
                    const float sc = (b & 1) ? __high2float(s2) : __low2float(s2);
                    y = fmaf(sc * bsc[b], ds, y);
                }
            }
        }
    }
    return y;
}

// Row sums of a pass from the accumulator slots (lanes 4i: rows i and i + 8 of each tile; columns
// 0 = hi, 1 = lo), tile rt's U slots added in slot order.
template <int U>
SP_DEVINL void rows_from_acc(const float (&d)[4][4], float *red_w, int nrt, int lane) {
#pragma unroll
    for (int rt = 0; rt < 4 / U; ++rt) {
        if (rt < nrt) {
            float ya = 0.f, yb = 0.f;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                ya += d[rt * U + u][0] + d[rt * U + u][1];
                yb += d[rt * U + u][2] + d[rt * U + u][3];
            }
            red_w[rt * 16 + (lane >> 2)] = ya;
            red_w[rt * 16 + (lane >> 2) + 8] = yb;
        }
    }
}

SP_DEVINL void argmax_merge(float &v, int &i, float ov, int oi) {
    if (ov > v || (ov == v && oi < i)) {
        v = ov;
        i = oi;
    }
}

// The compute warps' barrier. A warp can leave bar.sync with its lanes still split (they arrived
// from divergent code), and a warp-collective instruction after that (shuffle reductions) then
// pays a resynchronisation of hundreds of cycles: code that reduces across a warp right after
// divergent code reconverges first with __syncwarp() (measured: the softmax phase 2900 -> 550
// cycles). It is not added here or to the ring wait: measured, that costs more than it saves.
SP_DEVINL void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory"); }

SP_DEVINL unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Cross-CTA hand-off. The writers of a CTA meet at a barrier, then one thread publishes with
// release semantics (cumulative over the writes the barrier ordered before it); a consumer thread
// acquires, then its CTA's barrier orders the other threads' reads after the acquire.
SP_DEVINL unsigned atom_add_acq_rel(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
SP_DEVINL void red_add_release(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

SP_DEVINL void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
SP_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
SP_DEVINL void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }


// Abort state of the CTA: set on the first expired wait, after which no thread waits again.
struct Abort {
    volatile int *flag;
    DevState *st;
    SP_DEVINL bool on() const { return *flag != 0; }
    SP_DEVINL void raise(int code) const {
        *flag = 1;
        atomicCAS(&st->err, 0, code);
    }
};

SP_DEVINL bool wait_bar(uint64_t *bar, uint32_t parity, const Abort &ab) {
    for (uint32_t i = 0; i < kMbarSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && ab.on()) return false;
    }
    ab.raise(kErrMbarTimeout);
    return false;
}

// One thread waits until *cnt >= target (acquire). Gives up on abort or after the spin limit;
// also gives up when another CTA has already recorded an error, so a failure ends every CTA.
SP_DEVINL bool wait_counter(const unsigned long long *cnt, unsigned long long target, const Abort &ab) {
    for (uint32_t i = 0; i < kDepSpinLimit; ++i) {
        if (ld_acquire_u64(cnt) >= target) return true;
        if ((i & 63u) == 63u) {
            if (ab.on() || *reinterpret_cast<volatile int *>(&ab.st->err) != 0) {
                *ab.flag = 1;
                return false;
            }
            if (i >= 1024u) __nanosleep(64);      // back off only after the first ~1k polls
        }
    }
    ab.raise(kErrDepTimeout);
    return false;
}

// ---- LL words: (payload, tag) in one single-copy-atomic 64-bit store -------------------------
// Tag of the words op k writes in the step of `epoch`: never 0 (zeroed buffers never match) and
// different for every op of the last 2^31 / n_ops steps.
SP_DEVINL uint32_t ll_tag(unsigned long long epoch, int n_ops, int k) {
    return 0x80000000u | (((uint32_t)epoch * (uint32_t)n_ops + (uint32_t)k) & 0x7fffffffu);
}
SP_DEVINL uint64_t ll_word(uint32_t payload, uint32_t tag) { return ((uint64_t)tag << 32) | payload; }
SP_DEVINL uint64_t ll_wordf(float v, uint32_t tag) { return ll_word(__float_as_uint(v), tag); }
SP_DEVINL float ll_f(uint64_t w) { return __uint_as_float((uint32_t)w); }
SP_DEVINL bool ll_ok(uint64_t w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
SP_DEVINL void ll_st1(uint64_t *p, uint64_t a) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(a) : "memory");
}
SP_DEVINL void ll_st2(uint64_t *p, uint64_t a, uint64_t b) {
    asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
SP_DEVINL void ll_ld2(const uint64_t *p, uint64_t &a, uint64_t &b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p));
}
// fp16 hi = fp16(x) in the low half, lo = fp16(x - hi) in the high half
SP_DEVINL uint32_t hilo_bits(float x) {
    const __half h = __float2half_rn(x);
    const __half l = __float2half_rn(x - __half2float(h));
    return (uint32_t)__half_as_ushort(h) | ((uint32_t)__half_as_ushort(l) << 16);
}
SP_DEVINL uint32_t half2_bits(float a, float b) {
    return (uint32_t)__half_as_ushort(__float2half_rn(a)) | ((uint32_t)__half_as_ushort(__float2half_rn(b)) << 16);
}

// Polls the word pairs j < N with bit j of `valid` set (pair j at addr(j), 16-byte aligned) until
// both words of every pair carry `tag`; the words are left in w. Every round re-loads all pending
// pairs at once (the pairs of one thread come from different writers), so the poll ends about
// one round trip after the last writer's words land. Bounded; false when the CTA aborts.
template <int N, typename Addr>
SP_DEVINL bool ll_poll(uint64_t (&w)[N][2], uint32_t valid, Addr addr, uint32_t tag, const Abort &ab) {
    uint32_t pend = valid, todo = valid;
    for (uint32_t it = 0; pend != 0u; ++it) {
#pragma unroll
        for (int j = 0; j < N; ++j)
            if ((todo >> j) & 1u) ll_ld2(addr(j), w[j][0], w[j][1]);
        uint32_t got = 0u;
#pragma unroll
        for (int j = 0; j < N; ++j)
            if (((todo >> j) & 1u) && ll_ok(w[j][0], tag) && ll_ok(w[j][1], tag)) got |= 1u << j;
        pend &= ~got;
        todo = pend;
        if ((it & 63u) == 63u && pend != 0u) {
            if (ab.on() || *reinterpret_cast<volatile int *>(&ab.st->err) != 0) {
                *ab.flag = 1;
                return false;
            }
            if (it >= kDepSpinLimit) {
                ab.raise(kErrDepTimeout);
                return false;
            }
        }
    }
    return true;
}

// Prologue input of a norm op: this thread's float4s q of the residual stream (elements
// 4 (tid + q kEpiThreads) ..., K <= 4 x kNormRegs x kEpiThreads) from LL words, kNormRound
// float4s (2 kNormRound word pairs) per round trip.
// HILO: the payloads are fp16 (hi, lo) pairs, x = hi + lo; else fp32.
constexpr int kNormRound = 3;
SP_DEVINL float ll_x(uint64_t w, bool hilo) {
    if (!hilo) return ll_f(w);
    const uint32_t u = (uint32_t)w;
    return __half2float(__ushort_as_half((unsigned short)(u & 0xffffu))) + __half2float(__ushort_as_half((unsigned short)(u >> 16)));
}
template <bool HILO>
SP_DEVINL bool ll_norm_input(float4 (&v)[kNormRegs], const uint64_t *lin, int K, uint32_t tag, const Abort &ab) {
    const int tid = threadIdx.x;
#pragma unroll
    for (int q0 = 0; q0 < kNormRegs; q0 += kNormRound) {
        if (4 * (tid + q0 * kEpiThreads) >= K) break;
        uint64_t w[2 * kNormRound][2];
        uint32_t valid = 0u;
#pragma unroll
        for (int j = 0; j < 2 * kNormRound; ++j)
            if (q0 + (j >> 1) < kNormRegs && 4 * (tid + (q0 + (j >> 1)) * kEpiThreads) < K) valid |= 1u << j;
        if (!ll_poll<2 * kNormRound>(
                w, valid, [&](int j) { return lin + 4 * (tid + (q0 + (j >> 1)) * kEpiThreads) + 2 * (j & 1); }, tag, ab))
            return false;
#pragma unroll
        for (int q = 0; q < kNormRound; ++q)
            if (q0 + q < kNormRegs)
                v[q0 + q] = make_float4(ll_x(w[2 * q][0], HILO), ll_x(w[2 * q][1], HILO), ll_x(w[2 * q + 1][0], HILO),
                                        ll_x(w[2 * q + 1][1], HILO));
    }
    return true;
}

// Prologue input of the O projection: the merged attention output, LL words whose payload is the
// fp16 hi / lo pair, into the shared hi / lo vectors.
SP_DEVINL void ll_hilo_input(__half *xh, __half *xl, const uint64_t *lin, int K, uint32_t tag,
                                           const Abort &ab) {
    const int tid = threadIdx.x;
    for (int b0 = 0; b0 < K; b0 += 2 * kEpiThreads * kLLBatch) {
        uint64_t w[kLLBatch][2];
        uint32_t valid = 0u;
#pragma unroll
        for (int j = 0; j < kLLBatch; ++j)
            if (b0 + 2 * (tid + j * kEpiThreads) < K) valid |= 1u << j;
        if (!ll_poll<kLLBatch>(w, valid, [&](int j) { return lin + b0 + 2 * (tid + j * kEpiThreads); }, tag, ab)) return;
#pragma unroll
        for (int j = 0; j < kLLBatch; ++j) {
            if ((valid >> j) & 1u) {
                const int e = b0 + 2 * (tid + j * kEpiThreads);
                const uint32_t u0 = (uint32_t)w[j][0], u1 = (uint32_t)w[j][1];
                *reinterpret_cast<uint32_t *>(xh + e) = (u0 & 0xffffu) | (u1 << 16);
                *reinterpret_cast<uint32_t *>(xl + e) = (u0 >> 16) | (u1 & 0xffff0000u);
            }
        }
    }
}

// Int8 prologues (out of line: they run once per op and keep the kernel's register budget for
// the unit loop). The merged attention output (LL words of fp16 hi / lo payloads) into digits:
__device__ __noinline__ void attn_digits(const uint64_t *lin, int K, uint32_t tag, const Abort &ab, int8_t *dg,
                                         float *bsc) {
    // all of this thread's float4s (K <= 4 kNormRegs kEpiThreads) in one round trip
    const int tid = threadIdx.x;
    uint64_t w[2 * kNormRegs][2];
    uint32_t valid = 0u;
#pragma unroll
    for (int j = 0; j < 2 * kNormRegs; ++j)
        if (4 * (tid + (j >> 1) * kEpiThreads) < K) valid |= 1u << j;
    if (!ll_poll<2 * kNormRegs>(w, valid, [&](int j) { return lin + 4 * (tid + (j >> 1) * kEpiThreads) + 2 * (j & 1); },
                                tag, ab))
        return;
    float4 xs[kNormRegs];
    int nvalid = 0;
#pragma unroll
    for (int q = 0; q < kNormRegs; ++q) {
        xs[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (4 * (tid + q * kEpiThreads) < K) {                   // warp-uniform (K % 128 == 0)
            xs[q] = make_float4(ll_x(w[2 * q][0], true), ll_x(w[2 * q][1], true), ll_x(w[2 * q + 1][0], true),
                                ll_x(w[2 * q + 1][1], true));
            nvalid = q + 1;
        }
    }
    digitize4_n<kNormRegs>(xs, 4 * tid, 4 * kEpiThreads, (1u << nvalid) - 1u, dg, bsc);
}

// PRO_PLAIN into digits: the fp16 hi / lo vectors behind the counter (written by other CTAs in
// this launch). The digits of a 32-input block take 128 bytes, as many as its fp16 hi and lo
// halves: every 16-byte piece of the input goes in flight at once (cp.async through L2) into its
// block's own 128 bytes (hi at +0, lo at +64), one wait, then each block turns into digits in
// place. One round trip to L2 instead of one per batch of registers: under the weight stream a
// round trip takes microseconds. A block's 8 threads sit in one warp and read all of it before the
// warp barrier inside digitize4_n; its digit stores come after.
constexpr int kPlainBatch = 12;
__device__ __noinline__ void plain_digits(const __half *xin_h, const __half *xin_l, int K, int8_t *dg, float *bsc) {
    const int tid = threadIdx.x;
    for (int i = tid; i < K / 8; i += kEpiThreads) {                // piece i = inputs 8i .. 8i + 7
        int8_t *d = dg + 128 * (i >> 2) + 16 * (i & 3);
        cp_async16(d, reinterpret_cast<const uint4 *>(xin_h) + i);
        cp_async16(d + 64, reinterpret_cast<const uint4 *>(xin_l) + i);
    }
    cp_async_commit();
    cp_async_wait_all();
    epi_sync();
    for (int i0 = tid; 4 * i0 < K; i0 += kPlainBatch * kEpiThreads) {
        float4 xs[kPlainBatch];
        int nvalid = 0;
#pragma unroll
        for (int u = 0; u < kPlainBatch; ++u) {
            const int k = 4 * (i0 + u * kEpiThreads);
            xs[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k < K) {                                            // warp-uniform (K % 128 == 0)
                const int8_t *s = dg + 128 * (k >> 5) + 2 * (k & 31);
                const uint2 h = *reinterpret_cast<const uint2 *>(s);
                const uint2 l = *reinterpret_cast<const uint2 *>(s + 64);
                const float2 h0 = __half22float2(*reinterpret_cast<const __half2 *>(&h.x));
                const float2 h1 = __half22float2(*reinterpret_cast<const __half2 *>(&h.y));
                const float2 l0 = __half22float2(*reinterpret_cast<const __half2 *>(&l.x));
                const float2 l1 = __half22float2(*reinterpret_cast<const __half2 *>(&l.y));
                xs[u] = make_float4(h0.x + l0.x, h0.y + l0.y, h1.x + l1.x, h1.y + l1.y);
                nvalid = u + 1;
            }
        }
        digitize4_n<kPlainBatch>(xs, 4 * i0, 4 * kEpiThreads, (1u << nvalid) - 1u, dg, bsc);
    }
}

// Attention staging region of one (q head, chunk) item: K and V rows of one sub-chunk (fp16), the
// scores, q (fp32) and the four warps' value sums.
template <int HD>
struct AttnRegion {
    static constexpr int kRow = HD * 2;
    static constexpr size_t kOff = 0;                                   // K rows of the sub-chunk
    static constexpr size_t vOff = kOff + (size_t)kStepAttnRows * kRow; // V rows
    static constexpr size_t sOff = vOff + (size_t)kStepAttnRows * kRow; // scores / probabilities [rows]
    static constexpr size_t qOff = sOff + (size_t)kStepAttnRows * 4;    // q of the head [HD] fp32
    static constexpr size_t rOff = qOff + (size_t)HD * 4;               // per-warp PV partials [4][HD]
    static constexpr size_t bytes = rOff + (size_t)4 * HD * 4;
};

// cp.async K/V rows [lo, hi) of one kv head into the sub-chunk buffers (row j -> local j - base).
// In K rows the 16-byte chunks are XOR-permuted by (local row & 7): a thread per row reads chunk c
// of 8 consecutive rows from 8 different bank groups. V rows keep their order.
template <int HD>
SP_DEVINL void stage_rows(uint8_t *am, const __half *kb, const __half *vb, int base, int lo, int hi, int tid) {
    using L = AttnRegion<HD>;
    constexpr int kChunks = HD / 8;
    const int n = hi - lo;
    for (int i = tid; i < n * kChunks * 2; i += kEpiThreads) {
        const int which = i / (n * kChunks);
        const int r = (i - which * n * kChunks) / kChunks, ch = i % kChunks;
        const int j = lo + r;
        if (which == 0)
            cp_async16(am + L::kOff + (size_t)(j - base) * L::kRow + (ch ^ ((j - base) & 7)) * 16, kb + (size_t)j * HD + ch * 8);
        else
            cp_async16(am + L::vOff + (size_t)(j - base) * L::kRow + ch * 16, vb + (size_t)j * HD + ch * 8);
    }
}

// The K (V = false, chunks XOR-permuted by row like stage_rows) or V rows [lo, hi) of a sub-chunk
// starting at position `base`, with cp.async.
template <int HD, bool V>
SP_DEVINL void stage_half(uint8_t *am, const __half *src, int base, int lo, int hi, int tid) {
    using L = AttnRegion<HD>;
    constexpr int kChunks = HD / 8;
    for (int i = tid; i < (hi - lo) * kChunks; i += kEpiThreads) {
        const int j = lo + i / kChunks, ch = i % kChunks;
        if (V)
            cp_async16(am + L::vOff + (size_t)(j - base) * L::kRow + ch * 16, src + (size_t)j * HD + ch * 8);
        else
            cp_async16(am + L::kOff + (size_t)(j - base) * L::kRow + (ch ^ ((j - base) & 7)) * 16, src + (size_t)j * HD + ch * 8);
    }
}
SP_DEVINL void cp_async_wait_but1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

template <int DL>
SP_DEVINL void load_dims(const uint8_t *q, float (&f)[DL]) {
    if constexpr (DL == 4) {
        const uint2 u = *reinterpret_cast<const uint2 *>(q);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
        f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    } else {
        const uint32_t u = *reinterpret_cast<const uint32_t *>(q);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u));
        f[0] = a.x; f[1] = a.y;
    }
}

// Attention chunking of the visible context [0, ctx), the same in every CTA.
SP_DEVINL int attn_chunks(int ctx, int max_chunks) {
    return max(1, min(max_chunks, (ctx + kStepAttnRows - 1) / kStepAttnRows));
}

SP_DEVINL void stamp(unsigned long long *tr, int k, int C, int c, int i) {
    if (tr && threadIdx.x == 0) tr[((size_t)k * C + c) * kStepTraceWords + i] = globaltimer();
}
// SM clock at phase boundary i (0..7) of op k: cycle-exact durations inside one CTA
SP_DEVINL void stamp_clk(unsigned long long *tr, int k, int C, int c, int i) {
    if (tr && threadIdx.x == 0) tr[((size_t)k * C + c) * kStepTraceWords + 8 + i] = clock64();
}
// The same two from the calling thread (the attention warps' first thread)
SP_DEVINL void stamp_lead(unsigned long long *tr, int k, int C, int c, int i) {
    if (tr) tr[((size_t)k * C + c) * kStepTraceWords + i] = globaltimer();
}
SP_DEVINL void stamp_clk_lead(unsigned long long *tr, int k, int C, int c, int i) {
    if (tr) tr[((size_t)k * C + c) * kStepTraceWords + 8 + i] = clock64();
}

// One int8 pass (rows_p rows, all K inputs in units of chunk_w) on the 5th-generation tensor cores,
// pipelined: lane 0 of each compute warp issues its share of unit u + 1's block MMAs (TMEM buffer
// (u + 1) & 1) while every thread reads unit u's sums out of TMEM; a unit's stage goes back to the
// producer once its MMAs are done and its row scales are in registers. Out of line: the loop gets
// its own register budget instead of the step kernel's. Returns this thread's row sum.
SP_DEVINL int i8_row_of_thread(int rows_p, int tid) {
    return rows_p <= 64 ? ((tid & 31) < 16 ? 16 * (tid >> 5) + (tid & 31) : -1) : tid;
}
struct I8Ring {
    uint8_t *ring;
    uint64_t *full, *empty, *accb;
    int S, SB;
    int s, round, consumed;          // in / out: the ring position
    uint32_t acc_par;                // in / out: phases of accb[0] (bit 0), accb[1] (bit 1)
};
__device__ __noinline__ float i8_pass(I8Ring &rg, uint32_t tmem, const int8_t *dg, const float *bsc, int rows_p, int K,
                                      int chunk_w, const Abort ab) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // this thread's row (its TMEM lane): M = 128 tiles put row r at lane r, M = 64 tiles (passes of
    // at most 64 rows) at lane r % 16 + 32 (r / 16)
    const int row = i8_row_of_thread(rows_p, tid);
    const int S = rg.S, SB = rg.SB, s0 = rg.s, round0 = rg.round;
    uint32_t acc_par = rg.acc_par;
    const int nun = (K + chunk_w - 1) / chunk_w;
    auto issue = [&](int u) {                                   // lane 0 of each compute warp
        const int x = s0 + u, su = x % S;
        if (!wait_bar(&rg.full[su], (uint32_t)(round0 + x / S) & 1u, ab)) return;
        tc_fence_after();
        const int q0 = u * chunk_w;
        unit_i8_issue(tmem + (uint32_t)((u & 1) * 8 * kUnitBlocksI8), smem_u32(rg.ring + (size_t)su * SB), rows_p,
                      min(chunk_w, K - q0) >> 5, smem_u32(dg) + (uint32_t)((q0 >> 5) * 128), warp);
        mma_commit(&rg.accb[u & 1]);
    };
    if (lane == 0) issue(0);
    float y = 0.f;
    int u = 0;
    for (; u < nun; ++u) {
        const int q0 = u * chunk_w, wq = min(chunk_w, K - q0), nb = wq >> 5;
        const int su = (s0 + u) % S;
        if (!wait_bar(&rg.accb[u & 1], (acc_par >> (u & 1)) & 1u, ab)) break;
        acc_par ^= 1u << (u & 1);
        tc_fence_after();
        // this row's scales: [row][block] fp16 after the unit's weights
        uint32_t sc2[kUnitBlocksI8 / 2];
        const uint32_t *sr = reinterpret_cast<const uint32_t *>(rg.ring + (size_t)su * SB + (size_t)rows_p * wq) +
                             (size_t)max(0, min(row, rows_p - 1)) * (nb >> 1);
#pragma unroll
        for (int j = 0; j < kUnitBlocksI8 / 2; ++j) sc2[j] = 2 * j < nb ? sr[j] : 0u;
        epi_sync();                                             // the stage is read
        if (tid == 0) mbar_arrive(&rg.empty[su]);
        if (lane == 0 && u + 1 < nun) issue(u + 1);
        y += unit_i8_row(tmem + (uint32_t)((u & 1) * 8 * kUnitBlocksI8) + ((uint32_t)(warp * 32) << 16), sc2, nb,
                         bsc + (q0 >> 5));
        tc_fence_before();
    }
    rg.consumed += u;
    rg.s = (s0 + u) % S;
    rg.round = round0 + (s0 + u) / S;
    rg.acc_par = acc_par;
    return y;
}

// Per-step values every epilogue thread reads once (after the dependency on the previous step).
struct StepState {
    unsigned long long epoch;
    int token, pos, slot, tree_base;
    unsigned long long mask;
};

// ---- attention item of one CTA: (q head h, context chunk ch) -----------------------------------
// Staging that does not depend on the step: the first sub-chunk's K/V rows other than the current
// one (only the step's QKV projection writes row `slot`). Issued before the QKV projection's
// input is ready; `qkv` is that projection's op (same layer caches).
template <int HD>
__device__ void attn_prestage(const StepParams &p, const StepOp &qkv, const StepState &ss, uint8_t *am, int item,
                              int n_chunks, int rows_per, int ctx) {
    const int G = p.nh / p.nkv;
    const int h = item / n_chunks, ch = item - h * n_chunks, g = h / G;
    const int j0 = ch * rows_per, j1 = min(ctx, j0 + rows_per);
    const int s1 = min(j1, j0 + kStepAttnRows);
    stage_rows<HD>(am, qkv.kc + (size_t)g * p.cap * HD, qkv.vc + (size_t)g * p.cap * HD, j0, j0, min(s1, ss.slot),
                   threadIdx.x);
    cp_async_commit();
}

// One q head over one chunk of the context, in sub-chunks of up to kStepAttnRows positions:
//   scores  thread 32 + t = position t, a full HD-dim dot product against q in shared memory
//   softmax warp 1, running max / sum across sub-chunks (fp32)
//   values  warp = every fourth position, lane = HD/32 dims; the four warps' sums meet in shared
//           memory and thread t < HD keeps output dim t
// Publishes the chunk's unnormalised partial (max, sum, acc[HD]) as LL words.
template <int HD>
__device__ void attention_item(const StepParams &p, const StepOp &op, const StepState &ss, uint8_t *am, int item,
                               int n_chunks, int rows_per, int ctx, const Abort &ab, int k) {
    using L = AttnRegion<HD>;
    constexpr int DL = HD / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = p.nh / p.nkv;
    const int h = item / n_chunks, ch = item - h * n_chunks, g = h / G;
    const int j0 = ch * rows_per, j1 = min(ctx, j0 + rows_per);
    const __half *kb = op.kc + (size_t)g * p.cap * HD;
    const __half *vb = op.vc + (size_t)g * p.cap * HD;
    float *qs = reinterpret_cast<float *>(am + L::qOff);
    float *sc = reinterpret_cast<float *>(am + L::sOff);
    float *rd = reinterpret_cast<float *>(am + L::rOff);
    __shared__ float s_corr;
    const int slot = ss.slot;
    const int s1 = min(j1, j0 + kStepAttnRows);
    // the step's own position (the last of the context) is the one K / V row this step writes: it
    // comes from the QKV projection's LL words (thread t < HD / 2 holds one pair of each), never
    // from the cache, wherever it falls in the chunk
    const bool has_slot = slot >= j0 && slot < j1;
    uint32_t kvw[2] = {0u, 0u};
    auto put_slot = [&](int base) {
        if (tid < HD / 2) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int i = 2 * tid + e, which = i / (HD / 2), dd = i - which * (HD / 2);
                const int r = slot - base;
                __half *row = reinterpret_cast<__half *>(am + (which ? L::vOff : L::kOff) + (size_t)r * L::kRow);
                // dims dd and dd + HD/2; K chunks permuted like stage_rows'
                const int d0 = which ? dd : ((((dd >> 3) ^ (r & 7)) << 3) | (dd & 7));
                const int d1 = which ? dd + HD / 2 : (((((dd + HD / 2) >> 3) ^ (r & 7)) << 3) | (dd & 7));
                row[d0] = __ushort_as_half((unsigned short)(kvw[e] & 0xffffu));
                row[d1] = __ushort_as_half((unsigned short)(kvw[e] >> 16));
            }
        }
    };
    {
        // q of the head and, when the chunk holds the step's position, its new K / V row
        const bool cur = slot >= j0 && slot < s1;
        const uint64_t *qw = op.lin + (size_t)h * HD + 2 * tid;
        const uint64_t *kw = op.lkv + (size_t)g * HD + 2 * tid;
        uint64_t w[2][2];
        const uint32_t valid = tid < HD / 2 ? (has_slot ? 3u : 1u) : 0u;
        stamp_clk(p.trace, k, gridDim.x, blockIdx.x, 0);
        ll_poll<2>(w, valid, [&](int j) { return j == 0 ? qw : kw; }, ll_tag(ss.epoch, p.n_ops, op.lin_k), ab);
        stamp(p.trace, k, gridDim.x, blockIdx.x, 1);
        stamp_clk(p.trace, k, gridDim.x, blockIdx.x, 1);
        if (tid < HD / 2) {
            qs[2 * tid] = ll_f(w[0][0]);
            qs[2 * tid + 1] = ll_f(w[0][1]);
            kvw[0] = (uint32_t)w[1][0];
            kvw[1] = (uint32_t)w[1][1];
        }
        if (cur) put_slot(j0);
    }
    cp_async_wait_all();
    epi_sync();
    stamp(p.trace, k, gridDim.x, blockIdx.x, 2);
    stamp_clk(p.trace, k, gridDim.x, blockIdx.x, 2);
    __syncwarp();

    float qr[DL];
#pragma unroll
    for (int i = 0; i < DL; ++i) qr[i] = qs[DL * lane + i];
    float m_run = -INFINITY, l_run = 0.f;       // warp 1 (lane-uniform)
    float acc = 0.f;                            // thread t < HD: output dim t

    // Sub-chunks are pipelined: the next sub-chunk's K rows load while this one's softmax and
    // values run, its V rows while its own scores run (cp.async groups complete in order).
    for (int a = j0; a < j1; a += kStepAttnRows) {
        const int b = min(j1, a + kStepAttnRows), nj = b - a;
        const int a2 = b, b2 = min(j1, b + kStepAttnRows);  // the next sub-chunk (a2 < j1: exists)
        if (a != j0) {
            cp_async_wait_but1();               // K rows of [a, b) (its V rows may still load)
            if (slot >= a && slot < b) put_slot(a);
            epi_sync();
        }
        // scores: thread 32 + t = position t of the sub-chunk (nj <= kStepAttnRows <= 96), a full
        // dot product over HD dims: 16-byte K chunks (permuted by row, conflict-free) against q from
        // shared memory (the same address in every lane: a broadcast). No shuffles. Warps 1-3 do
        // the scores and the softmax: warp 0 shares its scheduler with the producer warp, and the
        // softmax ran ~5x slower there in some builds.
        const int sp = tid - 32;
        if (sp >= 0 && sp < nj) {
            const uint8_t *kr = am + L::kOff + (size_t)sp * L::kRow;
            float sv = 0.f;
#pragma unroll
            for (int c = 0; c < HD / 8; ++c) {
                const uint4 kq = *reinterpret_cast<const uint4 *>(kr + ((c ^ (sp & 7)) << 4));
                const float4 qa = *reinterpret_cast<const float4 *>(qs + 8 * c);
                const float4 qb = *reinterpret_cast<const float4 *>(qs + 8 * c + 4);
                const float2 k0 = __half22float2(*reinterpret_cast<const __half2 *>(&kq.x));
                const float2 k1 = __half22float2(*reinterpret_cast<const __half2 *>(&kq.y));
                const float2 k2 = __half22float2(*reinterpret_cast<const __half2 *>(&kq.z));
                const float2 k3 = __half22float2(*reinterpret_cast<const __half2 *>(&kq.w));
                sv = fmaf(qa.x, k0.x, sv);
                sv = fmaf(qa.y, k0.y, sv);
                sv = fmaf(qa.z, k1.x, sv);
                sv = fmaf(qa.w, k1.y, sv);
                sv = fmaf(qb.x, k2.x, sv);
                sv = fmaf(qb.y, k2.y, sv);
                sv = fmaf(qb.z, k3.x, sv);
                sv = fmaf(qb.w, k3.y, sv);
            }
            const int jj = a + sp;
            const bool vis = !(jj >= ss.tree_base && !((ss.mask >> (jj - ss.tree_base)) & 1ull));
            sc[sp] = vis ? sv * p.scale : -INFINITY;
        }
        epi_sync();                             // the K rows are free
        if (a2 < j1) {
            stage_half<HD, false>(am, kb, a2, a2, min(b2, slot), tid);
            cp_async_commit();
        }
        if (a == j0) {
            stamp(p.trace, k, gridDim.x, blockIdx.x, 5);
            stamp_clk(p.trace, k, gridDim.x, blockIdx.x, 3);
        }
        if (warp == 1) {                        // softmax statistics over the sub-chunk
            __syncwarp();
            const float v0 = lane < nj ? sc[lane] : -INFINITY;
            const float v1 = lane + 32 < nj ? sc[lane + 32] : -INFINITY;
            const float mnew = fmaxf(m_run, warp_max(fmaxf(v0, v1)));
            const float p0 = mnew == -INFINITY ? 0.f : expf(v0 - mnew);
            const float p1 = mnew == -INFINITY ? 0.f : expf(v1 - mnew);
            const float ls = warp_sum((lane < nj ? p0 : 0.f) + (lane + 32 < nj ? p1 : 0.f));
            const float corr = m_run == -INFINITY ? 0.f : expf(m_run - mnew);
            l_run = l_run * corr + ls;
            m_run = mnew;
            if (lane < nj) sc[lane] = p0;
            if (lane + 32 < nj) sc[lane + 32] = p1;
            if (lane == 0) s_corr = corr;
        }
        if (a != j0) {                          // the V rows of [a, b)
            if (a2 < j1)
                cp_async_wait_but1();           // (the next K rows may still load)
            else
                cp_async_wait_all();
        }
        epi_sync();
        if (a == j0) stamp_clk(p.trace, k, gridDim.x, blockIdx.x, 4);
        // values: warp w sums positions w, w + 4, ...; lane = DL output dims
        float pa[DL];
#pragma unroll
        for (int i = 0; i < DL; ++i) pa[i] = 0.f;
        const uint8_t *vrow = am + L::vOff + lane * DL * 2;
        for (int j = warp; j < nj; j += 4) {
            float vf[DL];
            load_dims<DL>(vrow + (size_t)j * L::kRow, vf);
            const float pj = sc[j];
#pragma unroll
            for (int i = 0; i < DL; ++i) pa[i] = fmaf(pj, vf[i], pa[i]);
        }
#pragma unroll
        for (int i = 0; i < DL; ++i) rd[warp * HD + DL * lane + i] = pa[i];
        epi_sync();                             // the V rows are free
        if (a2 < j1) {
            stage_half<HD, true>(am, vb, a2, a2, min(b2, slot), tid);
            cp_async_commit();
        }
        if (tid < HD) acc = fmaf(acc, s_corr, ((rd[tid] + rd[HD + tid]) + rd[2 * HD + tid]) + rd[3 * HD + tid]);
    }
    stamp(p.trace, k, gridDim.x, blockIdx.x, 4);
    stamp_clk(p.trace, k, gridDim.x, blockIdx.x, 5);
    uint64_t *pw = op.lpart + ((size_t)h * p.part_stride + ch) * (HD + 2);
    const uint32_t tag = ll_tag(ss.epoch, p.n_ops, k);
    if (tid < HD) ll_st1(pw + 2 + tid, ll_wordf(acc, tag));
    if (tid == 32) ll_st2(pw, ll_wordf(m_run, tag), ll_wordf(l_run, tag));
}

// A merge CTA folds q head h's chunks: out[d] = sum_c w_c acc_c[d] with
// w_c = exp(m_c - M) / sum_c l_c exp(m_c - M), chunks in a fixed order. In batches of up to
// kMergeBatch chunks, the NTH threads of the group (thread index t, their barrier) poll the batch's
// LL words (max, sum, acc[HD] per chunk; one round trip) into the free K staging rows, then the
// thread of output d folds the batch into a running (M, sum, acc[d]). The output goes out as LL
// words whose payload is the fp16 hi / lo pair the O projection multiplies.
template <int NTH>
SP_DEVINL void group_sync() {
    if constexpr (NTH == kEpiThreads)
        epi_sync();
    else
        asm volatile("bar.sync 2, %0;" ::"n"(NTH) : "memory");
}
// NB: word pairs a thread polls per round trip; MB: chunks staged per batch.
template <int HD, int NTH, int NB, int MB>
__device__ void merge_head(const StepParams &p, const StepOp &op, const StepState &ss, uint8_t *am, int h,
                           int n_chunks, int k, const Abort &ab, int t) {
    using L = AttnRegion<HD>;
    constexpr int kW = HD + 2;                  // words per chunk
    constexpr int ND = (HD + NTH - 1) / NTH;    // outputs per thread
    const uint32_t tag = ll_tag(ss.epoch, p.n_ops, k);
    const uint64_t *base = op.lpart + (size_t)h * p.part_stride * kW;
    static_assert((size_t)MB * (kW + 1) * 4 <= L::sOff, "a merge batch and its weights fit the K/V staging rows");
    static_assert(MB <= NTH, "a thread per chunk weight");
    float *mp = reinterpret_cast<float *>(am + L::kOff);
    float *fw = mp + (size_t)MB * kW;             // chunk weights of the batch
    float M = -INFINITY, Ls = 0.f, A[ND];
#pragma unroll
    for (int i = 0; i < ND; ++i) A[i] = 0.f;
    for (int c0 = 0; c0 < n_chunks; c0 += MB) {
        const int nc = min(MB, n_chunks - c0);
        const int nw = nc * kW;                 // even
        const uint64_t *bw = base + (size_t)c0 * kW;
        for (int b0 = 0; b0 < nw; b0 += 2 * NTH * NB) {
            uint64_t w[NB][2];
            uint32_t valid = 0u;
#pragma unroll
            for (int j = 0; j < NB; ++j)
                if (b0 + 2 * (t + j * NTH) < nw) valid |= 1u << j;
            // on abort every thread still passes the barriers below (the results are then unused)
            if (!ll_poll<NB>(w, valid, [&](int j) { return bw + b0 + 2 * (t + j * NTH); }, tag, ab))
                valid = 0u;
#pragma unroll
            for (int j = 0; j < NB; ++j) {
                if ((valid >> j) & 1u) {
                    const int e = b0 + 2 * (t + j * NTH);
                    *reinterpret_cast<float2 *>(mp + e) = make_float2(ll_f(w[j][0]), ll_f(w[j][1]));
                }
            }
        }
        group_sync<NTH>();
        // the batch's running max, then one weight exp(m_c - max) per chunk (thread c) for everyone
        float Mb = M;
        for (int cc = 0; cc < nc; ++cc) Mb = fmaxf(Mb, mp[cc * kW]);
        if (t < nc) {
            const float mc = mp[t * kW];
            fw[t] = (mc == -INFINITY || Mb == -INFINITY) ? 0.f : expf(mc - Mb);
        }
        group_sync<NTH>();
        if (t < HD && Mb != -INFINITY) {
            const float r = M == -INFINITY ? 0.f : expf(M - Mb);
            Ls *= r;
#pragma unroll
            for (int i = 0; i < ND; ++i) A[i] *= r;
            for (int cc = 0; cc < nc; ++cc) {
                const float f = fw[cc];
                Ls = fmaf(mp[cc * kW + 1], f, Ls);
#pragma unroll
                for (int i = 0; i < ND; ++i)
                    if (t + i * NTH < HD) A[i] = fmaf(mp[cc * kW + 2 + t + i * NTH], f, A[i]);
            }
        }
        M = Mb;
        group_sync<NTH>();                      // the staging rows are reused by the next batch
    }
#pragma unroll
    for (int i = 0; i < ND; ++i)
        if (t + i * NTH < HD) ll_st1(op.lout + (size_t)h * HD + t + i * NTH, ll_word(hilo_bits(A[i] / Ls), tag));
}

// ---- grouped attention: items (kv head g, context chunk ch), all G <= 8 q heads of the group ----
// In the grouped build the attention runs on three warps of its own (warps 5-7), which walk the
// step's attention ops while warps 0-3 do the GEMVs: the attention code keeps its registers out of
// the GEMV loop's budget, and a CTA's attention warps start each layer early (L2 prefetch of the
// item's K/V rows, its first tiles in flight) and wait for q.
// The K/V rows of a chunk are read from HBM once for the whole group (the per-head items read them
// once per q head) and the products run on the tensor cores, with fp32-grade sums:
//   scores  S (16 x 8 positions) = Q (16 x HD) K^T, mma.sync m16n8k16: A row r < 8 = fp16 hi of
//           q_r * scale, row 8 + r = its fp16 lo (q - hi); B = the K rows. Score of head r =
//           D[r] + D[8 + r].
//   values  O (16 x HD) += P (16 x 8 positions) V, mma.sync m16n8k8: A row r = fp16 hi of the
//           head's probabilities, row 8 + r = their lo; B = the V rows transposed with movmatrix.
//           Output of head r = O[r] + O[8 + r].
// The contraction index is permuted so that thread (row g, quad t) reads whole 16-byte pieces of
// the K row of position g: pieces t, t + 4, ... (8 dims each; the quad reads 64 contiguous bytes
// per load). Its j-th dim is dim 32 (j / 8) + 8 t + j % 8 of the row, and logical k =
// 16 kk + 2 t + 8 h + e is its dim j = 4 kk + 2 h + e, in q and in K alike; output n-tile nn,
// column 2 t + e is its dim 2 nn + e, so V is read in the same pieces. K/V go straight from
// global memory (L2) into registers, D tiles in flight while one computes; no shared-memory
// staging and no barriers inside the loop. Warp w takes tiles w, w + 3, ... of the chunk with its
// own running max / sum per head; the warps' partials meet once in shared memory and the item
// publishes one partial (max, sum, acc[HD]) per q head in the per-head items' format, so the same
// merge follows.
constexpr int kAttnWarps = 3;
constexpr int kAttnThreads = 32 * kAttnWarps;
constexpr int kAttnWarp0 = kProducerWarp + 1;
constexpr int kThreadsGR = kThreads + kAttnThreads;
static_assert(kThreadsGR * 255 <= 65536, "the grouped build keeps 255 registers a thread");
constexpr int kAttnMergePairs = 12;         // the attention warps' merge: word pairs in flight a thread
template <int HD>
constexpr int kAttnMergeChunks = HD == 128 ? 46 : 45;   // chunks staged per merge batch (region size)
template <int HD>
struct GroupRegion {
    static constexpr size_t qOff = 0;                                    // q [8][HD] fp32 (scaled)
    static constexpr size_t sOff = qOff + (size_t)kGroup * HD * 4;       // own K / V row [2][HD] fp16
    static constexpr size_t fOff = sOff + (size_t)2 * HD * 2;            // q fragments [HD / 16][32] uint4
    static constexpr size_t oOff = fOff + (size_t)HD / 16 * 32 * 16;     // warps' outputs [3][8][HD] fp32
    static constexpr size_t mOff = oOff + (size_t)kAttnWarps * kGroup * HD * 4;   // (max, sum) [3][8]
    static constexpr size_t bytes = mOff + (size_t)kAttnWarps * kGroup * 2 * 4;
};
static_assert(GroupRegion<64>::bytes <= AttnRegion<64>::bytes && GroupRegion<128>::bytes <= AttnRegion<128>::bytes,
              "grouped items use the per-head items' staging region");

// D (16x8 fp32) += A (16x8 fp16, row-major) * B (8x8 fp16, column-major)
SP_DEVINL void mma_1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(b0));
}
// 8x8 fp16 transpose across the warp (lane 4 r + t holds elements (r, 2t), (r, 2t + 1))
SP_DEVINL uint32_t movmatrix_t(uint32_t a) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}
SP_DEVINL uint32_t pack_half2(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}
// L2 prefetch of [src, src + bytes) (16-byte aligned, bytes a multiple of 16)
SP_DEVINL void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Chunk ch = item % n_chunks of kv head g = item / n_chunks: positions [j0, j1) of that head's rows.
struct GroupRows {
    const __half *kb, *vb;
    int g, ch, j0, j1;
};
template <int HD>
SP_DEVINL GroupRows group_rows(const StepParams &p, const StepOp &op, int item, int n_chunks, int rows_per, int ctx) {
    GroupRows r;
    r.g = item / n_chunks;
    r.ch = item - r.g * n_chunks;
    r.kb = op.kc + (size_t)r.g * p.cap * HD;
    r.vb = op.vc + (size_t)r.g * p.cap * HD;
    r.j0 = r.ch * rows_per;
    r.j1 = min(ctx, r.j0 + rows_per);
    return r;
}

// The item's K and V rows other than the step's own into L2 (threads t of nth), ahead of the item.
template <int HD>
SP_DEVINL void group_prefetch_t(const GroupRows &r, int slot, int t, int nth) {
    constexpr uint32_t kPiece = 4096;
    const int hi = min(r.j1, slot);
    if (hi <= r.j0) return;
    const uint32_t bytes = (uint32_t)(hi - r.j0) * HD * 2, n = (bytes + kPiece - 1) / kPiece;
    for (uint32_t i = (uint32_t)t; i < 2 * n; i += (uint32_t)nth) {
        const uint32_t piece = i % n, off = piece * kPiece;
        const __half *base = (i < n ? r.kb : r.vb) + (size_t)r.j0 * HD;
        bulk_prefetch_l2(reinterpret_cast<const uint8_t *>(base) + off, min(kPiece, bytes - off));
    }
}

// One pair of LL words (16-byte aligned) until both carry `tag`, with a back-off: the attention
// warps reach a layer long before its q exists and must not take issue slots from the GEMV warps.
// Bounded; false on abort.
SP_DEVINL bool ll_wait_pair(const uint64_t *w2, uint32_t tag, const Abort &ab) {
    for (uint32_t it = 0; it < kDepSpinLimit; ++it) {
        uint64_t a, b;
        ll_ld2(w2, a, b);
        if (ll_ok(a, tag) && ll_ok(b, tag)) return true;
        if ((it & 15u) == 15u && (ab.on() || *reinterpret_cast<volatile int *>(&ab.st->err) != 0)) {
            *ab.flag = 1;
            return false;
        }
        __nanosleep(200);
    }
    ab.raise(kErrDepTimeout);
    return false;
}

// The attention warps' item; t = thread index among them.
template <int HD>
SP_DEVINL void group_item(const StepParams &p, const StepOp &op, int item, int n_chunks, int rows_per, int ctx,
                          const StepState &ss, uint32_t tag, uint8_t *am, const Abort &ab, int k, int t) {
    using L = GroupRegion<HD>;
    const GroupRows gr = group_rows<HD>(p, op, item, n_chunks, rows_per, ctx);
    const int G = p.nh / p.nkv;
    const int j0 = gr.j0, j1 = gr.j1, slot = ss.slot;
    const __half *kb = gr.kb, *vb = gr.vb;
    constexpr int KS = HD / 16;             // k-steps of a score MMA
    constexpr int NT = HD / 8;              // output n-tiles
    constexpr int LD = HD / 32;             // 16-byte pieces of a thread per row
    constexpr int D = HD == 128 ? 1 : 3;    // K / V tiles in flight per warp beyond the current one
    const int warp = t >> 5, lane = t & 31, gq = lane >> 2, tq = lane & 3;
    const bool lead = t == 0;
    const int C = gridDim.x, c = blockIdx.x;
    float *qs = reinterpret_cast<float *>(am + L::qOff);
    __half *srow = reinterpret_cast<__half *>(am + L::sOff);
    const bool has_slot = slot >= j0 && slot < j1;
    const int ntiles = max(0, (j1 - j0 + 7) / 8);
    group_prefetch_t<HD>(gr, slot, t, kAttnThreads);
    // row of position gq of tile tt (past the chunk: a valid row, masked)
    const auto row_at = [&](int tt) { return (size_t)min(j0 + 8 * tt + gq, j1 - 1) * HD; };
    uint4 kq[D][LD], vq[D][LD];
    const auto load = [&](int tt, uint4 (&kr)[LD], uint4 (&vr)[LD]) {
        const size_t r = row_at(tt);
#pragma unroll
        for (int i = 0; i < LD; ++i) {
            kr[i] = __ldcg(reinterpret_cast<const uint4 *>(kb + r + 32 * i + 8 * tq));
            vr[i] = __ldcg(reinterpret_cast<const uint4 *>(vb + r + 32 * i + 8 * tq));
        }
    };
    // the first tiles go in flight before q exists (the step's own row is replaced later)
#pragma unroll
    for (int u = 0; u < D; ++u)
        if (warp + kAttnWarps * u < ntiles) load(warp + kAttnWarps * u, kq[u], vq[u]);
    const uint32_t qtag = ll_tag(ss.epoch, p.n_ops, op.lin_k);
    const uint64_t *lq = op.lin + (size_t)gr.g * G * HD, *lkv = op.lkv + (size_t)gr.g * HD;
    if (lead) stamp_clk_lead(p.trace, k, C, c, 0);
    ll_wait_pair(lq, qtag, ab);
    {
        // q of the group's heads (rows G.. are zero) and, when the chunk holds the step's position,
        // its K / V row; word pairs: q first (8 HD / 2), then K / V (HD / 2)
        constexpr int QP = kGroup * HD / 2, NPAIR = QP + HD / 2;
        constexpr int NP = (NPAIR + kAttnThreads - 1) / kAttnThreads;
        uint64_t w[NP][2];
        uint32_t valid = 0u;
#pragma unroll
        for (int j = 0; j < NP; ++j) {
            const int i = t + j * kAttnThreads;
            if (i < QP ? 2 * i < G * HD : (i < NPAIR && has_slot)) valid |= 1u << j;
        }
        const auto addr = [&](int j) {
            const int i = t + j * kAttnThreads;
            return i < QP ? lq + 2 * i : lkv + 2 * (i - QP);
        };
        // one tag: q and the K / V rows come from the same QKV projection
        if (!ll_poll<NP>(w, valid, addr, qtag, ab)) valid = 0u;
        if (lead) {
            stamp_lead(p.trace, k, C, c, 1);
            stamp_clk_lead(p.trace, k, C, c, 1);
        }
#pragma unroll
        for (int j = 0; j < NP; ++j) {
            const int i = t + j * kAttnThreads;
            if (i < QP) {
                const bool v = (valid >> j) & 1u;
                qs[2 * i] = v ? ll_f(w[j][0]) * p.scale : 0.f;
                qs[2 * i + 1] = v ? ll_f(w[j][1]) * p.scale : 0.f;
            } else if ((valid >> j) & 1u) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {     // word = (dim dd, dim dd + HD / 2) of K (which 0) or V
                    const int wi = 2 * (i - QP) + e, which = wi / (HD / 2), dd = wi - which * (HD / 2);
                    const uint32_t u = (uint32_t)w[j][e];
                    srow[which * HD + dd] = __ushort_as_half((unsigned short)(u & 0xffffu));
                    srow[which * HD + dd + HD / 2] = __ushort_as_half((unsigned short)(u >> 16));
                }
            }
        }
    }
    group_sync<kAttnThreads>();
    // q fragments of lane l: row l / 4 hi / lo at its dims 4 kk + {0, 1} (columns 2 (l % 4) + {0, 1})
    // and 4 kk + {2, 3}; the same for every warp, built once into [kk][lane] uint4
    uint4 *qf = reinterpret_cast<uint4 *>(am + L::fOff);
    for (int i = t; i < KS * 32; i += kAttnThreads) {
        const int kk = i >> 5, l = i & 31;
        const float4 x = *reinterpret_cast<const float4 *>(qs + (l >> 2) * HD + 32 * (kk >> 1) + 8 * (l & 3) + 4 * (kk & 1));
        const __half h0 = __float2half_rn(x.x), h1 = __float2half_rn(x.y), h2 = __float2half_rn(x.z),
                     h3 = __float2half_rn(x.w);
        qf[i] = make_uint4(pack_half2(h0, h1),
                           pack_half2(__float2half_rn(x.x - __half2float(h0)), __float2half_rn(x.y - __half2float(h1))),
                           pack_half2(h2, h3),
                           pack_half2(__float2half_rn(x.z - __half2float(h2)), __float2half_rn(x.w - __half2float(h3))));
    }
    group_sync<kAttnThreads>();
    if (lead) {
        stamp_lead(p.trace, k, C, c, 2);
        stamp_clk_lead(p.trace, k, C, c, 2);
        stamp_clk_lead(p.trace, k, C, c, 3);
        stamp_clk_lead(p.trace, k, C, c, 4);
    }
    float o[NT][4];
#pragma unroll
    for (int nn = 0; nn < NT; ++nn) o[nn][0] = o[nn][1] = o[nn][2] = o[nn][3] = 0.f;
    float m_run = -INFINITY, l_part = 0.f;  // head gq (m quad-uniform; l this thread's positions)
    const auto tile = [&](int tt, uint4 (&kc)[LD], uint4 (&vc)[LD]) {
        const int a = j0 + 8 * tt;
        const bool own = a + gq == slot;    // the step's own row: from the QKV projection's words
        if (own) {
#pragma unroll
            for (int i = 0; i < LD; ++i) {
                kc[i] = *reinterpret_cast<const uint4 *>(srow + 32 * i + 8 * tq);
                vc[i] = *reinterpret_cast<const uint4 *>(srow + HD + 32 * i + 8 * tq);
            }
        }
        const uint32_t *kw = reinterpret_cast<const uint32_t *>(kc);
        float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};   // even / odd k-steps
#pragma unroll
        for (int kk = 0; kk < KS; kk += 2) {
            const uint4 f0 = qf[kk * 32 + lane], f1 = qf[(kk + 1) * 32 + lane];
            mma_16816(sa, f0.x, f0.y, f0.z, f0.w, kw[2 * kk], kw[2 * kk + 1]);
            mma_16816(sb, f1.x, f1.y, f1.z, f1.w, kw[2 * kk + 2], kw[2 * kk + 3]);
        }
        // positions a + 2 tq, a + 2 tq + 1
        float s0 = (sa[0] + sb[0]) + (sa[2] + sb[2]), s1 = (sa[1] + sb[1]) + (sa[3] + sb[3]);
        const auto vis = [&](int jj) {
            if (jj >= j1) return false;
            const int d = jj - ss.tree_base;
            return !(d >= 0 && (d >= 64 || !((ss.mask >> d) & 1ull)));
        };
        if (!vis(a + 2 * tq)) s0 = -INFINITY;
        if (!vis(a + 2 * tq + 1)) s1 = -INFINITY;
        float mt = fmaxf(s0, s1);
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
        const float mn = fmaxf(m_run, mt);
        const float corr = m_run == -INFINITY ? 0.f : expf(m_run - mn);
        const float e0 = s0 == -INFINITY ? 0.f : expf(s0 - mn), e1 = s1 == -INFINITY ? 0.f : expf(s1 - mn);
        l_part = fmaf(l_part, corr, e0 + e1);
        m_run = mn;
        const __half p0 = __float2half_rn(e0), p1 = __float2half_rn(e1);
        const uint32_t pa0 = pack_half2(p0, p1);
        const uint32_t pa1 = pack_half2(__float2half_rn(e0 - __half2float(p0)), __float2half_rn(e1 - __half2float(p1)));
        const uint32_t *vw = reinterpret_cast<const uint32_t *>(vc);
#pragma unroll
        for (int nn = 0; nn < NT; ++nn) {
            o[nn][0] *= corr;
            o[nn][1] *= corr;
            o[nn][2] *= corr;
            o[nn][3] *= corr;
            mma_1688(o[nn], pa0, pa1, movmatrix_t(vw[nn]));
        }
    };
    for (int t0 = warp; t0 < ntiles; t0 += kAttnWarps * D) {
#pragma unroll
        for (int u = 0; u < D; ++u) {
            const int tt = t0 + kAttnWarps * u;
            if (tt < ntiles) {              // warp-uniform
                uint4 kc[LD], vc[LD];
#pragma unroll
                for (int i = 0; i < LD; ++i) {
                    kc[i] = kq[u][i];
                    vc[i] = vq[u][i];
                }
                if (tt + kAttnWarps * D < ntiles) load(tt + kAttnWarps * D, kq[u], vq[u]);
                tile(tt, kc, vc);
            }
        }
    }
    // the warp's partial of head gq (the thread's dims 2 nn + e)
    float l = l_part + __shfl_xor_sync(0xffffffffu, l_part, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    float *ow = reinterpret_cast<float *>(am + L::oOff) + ((size_t)warp * kGroup + gq) * HD + 8 * tq;
#pragma unroll
    for (int nn = 0; nn < NT; ++nn)
        *reinterpret_cast<float2 *>(ow + 32 * (nn >> 2) + 2 * (nn & 3)) =
            make_float2(o[nn][0] + o[nn][2], o[nn][1] + o[nn][3]);
    float *mw = reinterpret_cast<float *>(am + L::mOff);
    if (tq == 0) *reinterpret_cast<float2 *>(mw + 2 * (warp * kGroup + gq)) = make_float2(m_run, l);
    group_sync<kAttnThreads>();
    if (lead) {
        stamp_lead(p.trace, k, C, c, 5);
        stamp_clk_lead(p.trace, k, C, c, 5);
    }
    // the warps' partials -> one per q head, in the per-head items' format
    const float *oo = reinterpret_cast<const float *>(am + L::oOff);
    uint64_t *part = op.lpart + ((size_t)gr.g * G * p.part_stride + gr.ch) * (HD + 2);
    for (int i = t; i < G * HD; i += kAttnThreads) {
        const int r = i / HD, d = i - r * HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, mw[2 * (w * kGroup + r)]);
        float Ls = 0.f, A = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kAttnWarps; ++w) {
                const float mwr = mw[2 * (w * kGroup + r)];
                const float f = mwr == -INFINITY ? 0.f : expf(mwr - M);
                Ls = fmaf(mw[2 * (w * kGroup + r) + 1], f, Ls);
                A = fmaf(oo[((size_t)w * kGroup + r) * HD + d], f, A);
            }
        }
        uint64_t *pw = part + (size_t)r * p.part_stride * (HD + 2);
        ll_st1(pw + 2 + d, ll_wordf(A, tag));
        if (d == 0) ll_st2(pw, ll_wordf(M, tag), ll_wordf(Ls, tag));
    }
    group_sync<kAttnThreads>();             // the region is reused by the merge
}

// The LM head's argmax across CTAs (last arriver) and the device state of the next step; once
// per step, so out of line (it keeps the step's hot code smaller).
__device__ __noinline__ void lmhead_finish(const StepParams &p, const StepOp &op, const StepState &ss, DevState *st,
                                           float bv, int bi, int c) {
    __shared__ float s_val[4];
    __shared__ int s_idx[4];
    __shared__ int s_flag;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, ov, oi);
    }
    if (lane == 0) {
        s_val[warp] = bv;
        s_idx[warp] = bi;
    }
    epi_sync();
    if (tid == 0) {
        float vb = s_val[0];
        int ib = s_idx[0];
        for (int w = 1; w < 4; ++w) argmax_merge(vb, ib, s_val[w], s_idx[w]);
        p.part_val[c] = vb;
        p.part_idx[c] = ib;
        s_flag = atom_add_acq_rel(p.lm_cnt, 1u) == (unsigned)op.grid - 1u;
    }
    epi_sync();
    if (s_flag) {
        float vb = -INFINITY;
        int ib = INT_MAX;
        for (int j = tid; j < op.grid; j += kEpiThreads)
            argmax_merge(vb, ib, __ldcg(p.part_val + j), __ldcg(p.part_idx + j));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, vb, o);
            const int oi = __shfl_xor_sync(0xffffffffu, ib, o);
            argmax_merge(vb, ib, ov, oi);
        }
        epi_sync();
        if (lane == 0) {
            s_val[warp] = vb;
            s_idx[warp] = ib;
        }
        epi_sync();
        if (tid == 0) {
            for (int w = 1; w < 4; ++w) argmax_merge(s_val[0], s_idx[0], s_val[w], s_idx[w]);
            int tok = s_idx[0];
            if (tok < 0 || tok >= op.n_valid) {
                atomicCAS(&st->err, 0, kErrBadToken);
                tok = 0;
            }
            *p.lm_cnt = 0u;
            const int step = st->step;
            if (st->out_tokens) st->out_tokens[step] = tok;
            const int nxt = step + 1;
            st->step = nxt;
            if (nxt < st->n_forced) {
                st->slot = st->slot0 + nxt;
                st->token = st->use_small ? st->small_tok[nxt] : st->f_tok[nxt];
                st->pos = st->use_small ? st->small_pos[nxt] : (st->f_pos ? st->f_pos[nxt] : st->slot0 + nxt);
            } else {
                st->token = tok;
                st->pos += 1;
                st->slot += 1;
            }
            *p.epoch = ss.epoch + 1;
        }
    }
}

// Bytes of one unit of `rows` rows x `w` inputs: fp16 rows, or int8 rows plus their fp16 scales
// (one per row and 32-input block), padded to 16 bytes.
SP_HOSTDEV uint32_t step_unit_bytes(int fmt, int rows, int w) {
    return fmt == WF_I8 ? (uint32_t)(rows * w + (((w / 32) * rows * 2 + 15) & ~15)) : (uint32_t)(rows * w * 2);
}

// The CTA's weight units of the step in consumption order (op, pass, chunk). A unit's bytes are
// contiguous and follow the previous unit of the same op (see k_pack_rows). Op fields are read
// from the table in global memory when the cursor enters an op, lazily (at the next call), so a
// unit is handed out without waiting for the next op's descriptor.
struct UnitCursor {
    const StepOp *ops;
    int n_ops, c;
    int k = -1;                     // current op; n_ops: exhausted
    int K = 0, cw = 0, prw = 0, R = 0, p0 = 0, q0 = 0, fmt = WF_F16;
    bool pending = false;           // the current op is used up: seek the next one first
    const uint8_t *src = nullptr;

    SP_DEVINL void seek(int from) {
        for (k = from; k < n_ops; ++k) {
            const StepOp *o = ops + k;
            if (__ldg(&o->kind) != OP_GEMV) continue;
            const int grid = __ldg(&o->grid);
            if (c >= grid) continue;
            const GemvShare sh = gemv_share(__ldg(&o->N), __ldg(&o->K), grid, __ldg(&o->ksplit), c);
            const int R0 = sh.R0;
            R = sh.R;
            if (R <= 0) continue;
            K = sh.Kc;
            cw = __ldg(&o->chunk_w);
            prw = __ldg(&o->pass_rows);
            fmt = __ldg(&o->fmt);
            src = reinterpret_cast<const uint8_t *>(__ldg(reinterpret_cast<const unsigned long long *>(&o->w))) +
                  (fmt == WF_I8 ? (size_t)c * __ldg(&o->cta_bytes) : (size_t)R0 * K * 2);
            p0 = 0;
            q0 = 0;
            return;
        }
    }
    SP_DEVINL bool next(const uint8_t *&unit, uint32_t &bytes) {
        if (pending) {
            pending = false;
            seek(k + 1);
        }
        if (k >= n_ops) return false;
        bytes = step_unit_bytes(fmt, min(prw, R - p0), min(cw, K - q0));
        unit = src;
        src += bytes;
        q0 += cw;
        if (q0 >= K) {
            q0 = 0;
            p0 += prw;
            if (p0 >= R) pending = true;
        }
        return true;
    }
};

}  // namespace

// Q8: the build with the blockwise-int8 unit path (a separate instantiation, so the fp16-only
// kernel keeps its register allocation).
template <int HD, bool Q8, bool GR>
__global__ void __launch_bounds__(GR ? kThreadsGR : kThreads, 1) k_step(const StepParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ float s_val[4];
    __shared__ int s_abort;
    __shared__ int s_issued, s_consumed;      // stages the producer issued / the compute warps consumed
    __shared__ float red[4][kPassRows];       // per-warp row partials of a pass (k-steps split over warps)
    __shared__ uint64_t s_accb[2];            // Q8: the int8 MMAs of a unit (TMEM buffer 0 / 1) are done
    __shared__ uint32_t s_tmem;               // Q8: TMEM accumulator base (kStepTmemCols columns)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = gridDim.x, c = blockIdx.x;
    const int S = p.stages;
    const int SB = p.stage_bytes;
    uint8_t *ring = smem;
    // the input vector of a GEMV as two fp16 vectors: hi = fp16(x) at xh, lo = fp16(x - hi) at
    // xh + K (~22 bits of x); the attention region follows the QKV projection's input
    uint8_t *vec = smem + (size_t)S * SB;
    __half *xh = reinterpret_cast<__half *>(vec);
    uint8_t *am = vec + p.attn_off;
    StepOp *opc = reinterpret_cast<StepOp *>(vec + p.vec_bytes);     // ops k and k + 1 (warps 0-3)
    uint64_t *full = reinterpret_cast<uint64_t *>(opc + 2);
    uint64_t *empty = full + S;
    const Abort ab{&s_abort, p.st};

    if (tid == 0) {
        s_abort = 0;
        s_issued = 0;
        s_consumed = 0;
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        if (Q8) {                             // one commit from each compute warp's issuing lane
            mbar_init(&s_accb[0], kEpiThreads / 32);
            mbar_init(&s_accb[1], kEpiThreads / 32);
        }
        fence_mbar_init();
    }
    if (Q8 && warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kStepTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid < kOpWords) cp_async16(reinterpret_cast<uint4 *>(opc) + tid, reinterpret_cast<const uint4 *>(p.ops) + tid);
    cp_async_commit();
    cp_async_wait_all();
    if (Q8) tc_fence_before();
    __syncthreads();
    if (Q8) tc_fence_after();
    const uint32_t tmem = Q8 ? s_tmem : 0u;
    uint32_t acc_par = 0u;                    // Q8: phases of s_accb[0] (bit 0) and s_accb[1] (bit 1)

    if (warp == kProducerWarp) {
        // ---- producer: every unit of the step, in op order; waits only for free stages. While it
        // waits (the ring is full: the other warps are in a hand-off or a small op), it warms L2 with
        // the CTA's next units, up to p.l2_ahead bytes beyond the issue point, so HBM keeps
        // streaming through the latency-bound phases and the big ops later read from L2. ---------
        if (lane == 0) {
            int s = 0, round = 0, issued = 0;
            const int F = p.max_inflight > 0 ? min(p.max_inflight, S) : S;
            const uint64_t pol = policy_evict_first();
            UnitCursor ic{p.ops, p.n_ops, c};
            ic.seek(0);
            // the warm-ahead cursor walks the same units on its own; pf_pos / is_pos are the bytes
            // of the CTA's stream it has passed / that have been issued
            UnitCursor pc{p.ops, p.n_ops, c};
            pc.seek(0);
            unsigned long long pf_pos = 0, is_pos = 0;
            bool pf_more = p.l2_ahead > 0;
            const uint8_t *u;
            uint32_t nb;
            while (!ab.on() && ic.next(u, nb)) {
                is_pos += nb;
                if (round > 0) {
                    const uint32_t par = (uint32_t)(round - 1) & 1u;
                    bool ok = false;
                    for (uint32_t i = 0; i < kMbarSpinLimit; ++i) {
                        // with warm-ahead budget left, probe without blocking and prefetch in between
                        const bool pf = pf_more && pf_pos < is_pos + (unsigned long long)p.l2_ahead;
                        if (pf ? mbar_test_wait(&empty[s], par) : mbar_try_wait(&empty[s], par)) {
                            ok = true;
                            break;
                        }
                        if (pf) {
                            const uint8_t *pu;
                            uint32_t pnb;
                            if (pc.next(pu, pnb)) {
                                if (pf_pos >= is_pos) prefetch_l2(pu, pnb);     // units not issued yet only
                                pf_pos += pnb;
                            } else {
                                pf_more = false;
                            }
                        }
                        if ((i & 255u) == 255u && ab.on()) break;
                    }
                    if (!ok) {
                        if (!ab.on()) ab.raise(kErrMbarTimeout);
                        break;
                    }
                }
                // at most F copies in flight: unit issued - F must have landed (its stage is not
                // refilled before this one is issued, so its phase parity is exact)
                if (issued >= F) {
                    const int uu = issued - F;
                    if (!wait_bar(&full[uu % S], (uint32_t)(uu / S) & 1u, ab)) break;
                }
                mbar_arrive_expect_tx(&full[s], nb);
                if (p.evict_first)
                    bulk_g2s_hint(ring + (size_t)s * SB, u, nb, &full[s], pol);
                else
                    bulk_g2s(ring + (size_t)s * SB, u, nb, &full[s]);
                ++issued;
                if (++s == S) {
                    s = 0;
                    ++round;
                }
            }
            s_issued = issued;
        }
    } else if (GR && warp >= kAttnWarp0) {
        // ---- grouped build, warps 5-7: the step's attention ops, one layer after the other -------
        griddep_wait();
        const int t = tid - kAttnWarp0 * 32;
        DevState *st = p.st;
        StepState ss;
        ss.epoch = *p.epoch;
        ss.slot = min(max(st->slot, 0), p.cap - 1);          // warps 0-3 report bad slots
        ss.tree_base = st->tree_base;
        ss.mask = ss.slot >= ss.tree_base ? st->small_mask[ss.slot - ss.tree_base] : 0ull;
        ss.token = 0;
        ss.pos = 0;
        const int ctx = min(ss.slot + 1, p.cap);
        const int n_chunks = max(1, min(p.group_chunks, (ctx + kGroupTileRows - 1) / kGroupTileRows));
        const int rows_per = (ctx + n_chunks - 1) / n_chunks;
        const int n_items = p.nkv * n_chunks;
        // items on the last CTAs, one per CTA; head h's merge on the CTA before them (or on the CTA
        // of item h, after its item, when the grid has no room)
        const int item = C - 1 - c;
        const int mh = n_items + p.nh <= C ? C - 1 - n_items - c : item;
        for (int k = 0; k < p.n_ops; ++k) {
            const StepOp &op = p.ops[k];
            if (op.kind != OP_ATTN) continue;
            if (ab.on()) break;
            const uint32_t tag = ll_tag(ss.epoch, p.n_ops, k);
            if (item < n_items) {
                group_item<HD>(p, op, item, n_chunks, rows_per, ctx, ss, tag, am, ab, k, t);
                if (t == 0) stamp_lead(p.trace, k, C, c, 4);
            }
            if (mh >= 0 && mh < p.nh && !ab.on()) {
                if (t == 0) stamp_lead(p.trace, k, C, c, 6);
                ll_wait_pair(op.lpart + (size_t)mh * p.part_stride * (HD + 2), tag, ab);   // back-off first
                merge_head<HD, kAttnThreads, kAttnMergePairs, kAttnMergeChunks<HD>>(p, op, ss, am, mh, n_chunks, k, ab, t);
                if (t == 0) {
                    stamp_lead(p.trace, k, C, c, 7);
                    stamp_clk_lead(p.trace, k, C, c, 7);
                }
            }
        }
    } else {
        // ---- warps 0-3: hand-offs, prologues, GEMV compute, epilogues, attention ------------------
        griddep_wait();
        griddep_launch_dependents();
        DevState *st = p.st;
        StepState ss;
        ss.epoch = *p.epoch;
        ss.token = st->token;
        ss.pos = st->pos;
        ss.slot = st->slot;
        ss.tree_base = st->tree_base;
        ss.mask = ss.slot >= ss.tree_base ? st->small_mask[ss.slot - ss.tree_base] : 0ull;
        if (ss.pos < 0 || ss.pos >= p.max_pos || ss.slot < 0 || ss.slot >= p.cap) {
            if (tid == 0 && c == 0) atomicCAS(&st->err, 0, kErrBadSlot);
            ss.pos = min(max(ss.pos, 0), p.max_pos - 1);
            ss.slot = min(max(ss.slot, 0), p.cap - 1);
        }
        if (ss.token < 0 || ss.token >= p.vocab) {
            if (tid == 0 && c == 0) atomicCAS(&st->err, 0, kErrBadToken);
            ss.token = 0;
        }
        const int ctx = min(ss.slot + 1, p.cap);
        // attention items: per (q head, chunk), or (GR) per (kv head, chunk)
        const int n_chunks = GR ? max(1, min(p.group_chunks, (ctx + kGroupTileRows - 1) / kGroupTileRows))
                                : attn_chunks(ctx, p.max_chunks);
        const int rows_per = (ctx + n_chunks - 1) / n_chunks;
        const int n_items = (GR ? p.nkv : p.nh) * n_chunks;
        const int half_hd = HD / 2;
        int s = 0, round = 0, consumed = 0;       // ring position of the compute warps

        for (int k = 0; k < p.n_ops; ++k) {
            cp_async_wait_all();
            epi_sync();                           // op k is in opc[k & 1]; everyone is done with op k - 1
            const StepOp &op = opc[k & 1];
            if (k + 1 < p.n_ops && tid < kOpWords)
                cp_async16(reinterpret_cast<uint4 *>(opc + ((k + 1) & 1)) + tid,
                           reinterpret_cast<const uint4 *>(p.ops + k + 1) + tid);
            cp_async_commit();
            stamp(p.trace, k, C, c, 0);
            const uint32_t tag = ll_tag(ss.epoch, p.n_ops, k);
            if (GR && op.kind == OP_ATTN) {       // the attention warps' op
                stamp(p.trace, k, C, c, 3);
                continue;
            }
            if (!GR && op.kind == OP_ATTN) {
                // items on the last CTAs: (q head, context chunk), one per CTA
                const int items = n_items, item = C - 1 - c;
                if (item < items && !ab.on()) {
                    attention_item<HD>(p, op, ss, am, item, n_chunks, rows_per, ctx, ab, k);
                    const int h = item / n_chunks;
                    if (item == h * n_chunks) {          // chunk 0 of the head: merge all of them
                        stamp(p.trace, k, C, c, 6);
                        stamp_clk(p.trace, k, C, c, 6);
                        merge_head<HD, kEpiThreads, kLLBatch, kMergeBatch>(p, op, ss, am, h, n_chunks, k, ab, tid);
                        stamp(p.trace, k, C, c, 7);
                        stamp_clk(p.trace, k, C, c, 7);
                    }
                }
                stamp(p.trace, k, C, c, 3);
                continue;
            }
            if (op.epi == EPI_QKV) {
                // this CTA's attention item of the layer: stage its immutable K/V rows now
                const int item = C - 1 - c;
                if (!GR && item < n_items) attn_prestage<HD>(p, op, ss, am, item, n_chunks, rows_per, ctx);
            }
            if (c >= op.grid) continue;          // no rows of this GEMV
            stamp_clk(p.trace, k, C, c, 0);
            // split inputs exist for int8 units only: the fp16 build keeps the unsplit code (the split
            // branches cost its decode step ~4.5 %)
            const GemvShare sh = gemv_share(op.N, op.K, op.grid, Q8 ? op.ksplit : 1, c);
            const int K = sh.Kc;                 // this CTA's inputs: [sh.K0, sh.K0 + K) of op.K
            const int KF = op.K;                 // the whole input (a norm prologue normalizes all of it)
            const bool fin = sh.K0 == 0;         // finishes its rows (split: adds the partners' partials)
            __half *xl = xh + K;
            // int8 weights: the input's digit rows (stride K + 16 bytes) and block scales instead
            int8_t *dg = reinterpret_cast<int8_t *>(vec);
            float *bsc = reinterpret_cast<float *>(vec + 4 * (K + 16));
            const bool q8 = Q8 && op.fmt == WF_I8;
            const bool norm = op.pro == PRO_NORM || op.pro == PRO_EMBED_NORM;
            const int R0 = sh.R0, R = sh.R;
            // epilogue operands that do not depend on the products (residual rows, bias, RoPE
            // factors): thread t < npairs finishes pair t (rows 2t, 2t + 1) of a pass. Pass 0's are
            // loaded before the input wait, where their round trip costs nothing.
            auto preload = [&](int p0, float &pre0, float &pre1, float &pcs, float &psn) {
                const int rows_p = min(op.pass_rows, R - p0);
                const int row = R0 + p0 + 2 * tid;                  // packed row (row, row + 1)
                pre0 = 0.f;
                pre1 = 0.f;
                pcs = 1.f;
                psn = 0.f;
                if (tid < rows_p / 2 && row < op.n_valid) {
                    if (op.epi == EPI_RESID) {
                        if (!fin) {                                 // the partner adds the residual
                        } else if (op.lres == nullptr) {                   // layer 0: the token's embedding row
                            const __half2 e2 = *reinterpret_cast<const __half2 *>(p.embed + (size_t)ss.token * p.hidden + row);
                            pre0 = __low2float(e2);
                            pre1 = __high2float(e2);
                        } else {
                            uint64_t w[1][2];
                            ll_poll<1>(w, 1u, [&](int) { return op.lres + row; }, ll_tag(ss.epoch, p.n_ops, op.lres_k), ab);
                            pre0 = ll_f(w[0][0]);
                            pre1 = ll_f(w[0][1]);
                        }
                    } else if (op.epi == EPI_QKV) {
                        const int P2 = row / 2, hh = P2 / half_hd, dd = P2 - hh * half_hd;
                        pre0 = __ldg(op.bias + hh * HD + dd);
                        pre1 = __ldg(op.bias + hh * HD + dd + half_hd);
                        if (hh < p.nh + p.nkv) {
                            const float2 r2 = __ldg(reinterpret_cast<const float2 *>(p.rope + ((size_t)ss.pos * half_hd + dd) * 2));
                            pcs = r2.x;
                            psn = r2.y;
                        }
                    }
                }
                __syncwarp();                                       // after the per-pair loads
            };
            float pre0, pre1, pcs, psn;
            preload(0, pre0, pre1, pcs, psn);
            float4 gn[kNormRegs];
            if (norm) {
#pragma unroll
                for (int q = 0; q < kNormRegs; ++q) {
                    const int i = tid + q * kEpiThreads;
                    gn[q] = 4 * i < KF ? __ldg(reinterpret_cast<const float4 *>(op.gain) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            if (op.dep >= 0) {
                if (tid == 0 && !ab.on())
                    wait_counter(p.cnt + op.dep, (unsigned long long)op.dep_n * (ss.epoch + 1), ab);
                epi_sync();
            }
            stamp(p.trace, k, C, c, 1);

            // ---- prologue: the input vector in shared memory as hi / lo halves ----------------------
            if (norm) {
                // K <= kNormRegs * 4 * kEpiThreads (host-checked): each thread holds its float4s in registers
                float4 v[kNormRegs];
#pragma unroll
                for (int q = 0; q < kNormRegs; ++q) v[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (op.pro == PRO_EMBED_NORM) {
#pragma unroll
                    for (int q = 0; q < kNormRegs; ++q) {
                        const int i = tid + q * kEpiThreads;
                        if (4 * i < KF) {
                            const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(p.embed + (size_t)ss.token * KF) + i);
                            const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
                            const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
                            v[q] = make_float4(a.x, a.y, b.x, b.y);
                        }
                    }
                } else {
                    ll_norm_input<false>(v, op.lin, KF, ll_tag(ss.epoch, p.n_ops, op.lin_k), ab);
                }
                __syncwarp();
                float sq = 0.f;
#pragma unroll
                for (int q = 0; q < kNormRegs; ++q) {
                    if (4 * (tid + q * kEpiThreads) < KF) {
                        sq = fmaf(v[q].x, v[q].x, sq);
                        sq = fmaf(v[q].y, v[q].y, sq);
                        sq = fmaf(v[q].z, v[q].z, sq);
                        sq = fmaf(v[q].w, v[q].w, sq);
                    }
                }
                sq = warp_sum(sq);
                if (lane == 0) s_val[warp] = sq;
                epi_sync();
                const float inv = 1.0f / sqrtf((s_val[0] + s_val[1] + s_val[2] + s_val[3]) / (float)KF + p.eps);
                if (Q8 && q8) {
                    // the whole vector is normalized; this CTA's inputs [sh.K0, sh.K0 + K) become digits
                    uint32_t vm = 0u;
#pragma unroll
                    for (int q = 0; q < kNormRegs; ++q) {
                        const int i4 = 4 * (tid + q * kEpiThreads) - sh.K0;
                        if (i4 >= 0 && i4 < K) {                    // warp-uniform (K0, K multiples of 128)
                            v[q] = make_float4((v[q].x * inv) * gn[q].x, (v[q].y * inv) * gn[q].y,
                                               (v[q].z * inv) * gn[q].z, (v[q].w * inv) * gn[q].w);
                            vm |= 1u << q;
                        }
                    }
                    digitize4_n<kNormRegs>(v, 4 * tid - sh.K0, 4 * kEpiThreads, vm, dg, bsc);
                } else {
#pragma unroll
                    for (int q = 0; q < kNormRegs; ++q) {
                        const int i = tid + q * kEpiThreads;
                        if (4 * i < K)
                            store_hilo4(xh, xl, 4 * i,
                                        make_float4((v[q].x * inv) * gn[q].x, (v[q].y * inv) * gn[q].y,
                                                    (v[q].z * inv) * gn[q].z, (v[q].w * inv) * gn[q].w));
                    }
                }
            } else if (q8 && op.pro == PRO_ATTN) {
                attn_digits(op.lin + sh.K0, K, ll_tag(ss.epoch, p.n_ops, op.lin_k), ab, dg, bsc);
            } else if (op.pro == PRO_ATTN) {
                ll_hilo_input(xh, xl, op.lin, K, ll_tag(ss.epoch, p.n_ops, op.lin_k), ab);
            } else if (q8) {
                plain_digits(op.xin_h + sh.K0, op.xin_l + sh.K0, K, dg, bsc);
            } else {
                // PRO_PLAIN: fp16 hi / lo vectors behind the dependency counter: every 16-byte piece
                // in flight at once (cp.async through L2), one wait
                for (int i = tid; i < K / 8; i += kEpiThreads) {
                    cp_async16(reinterpret_cast<uint4 *>(xh) + i, reinterpret_cast<const uint4 *>(op.xin_h) + i);
                    cp_async16(reinterpret_cast<uint4 *>(xl) + i, reinterpret_cast<const uint4 *>(op.xin_l) + i);
                }
                cp_async_commit();
                cp_async_wait_all();
            }
            if (q8) fence_proxy_async_smem();                       // digits -> visible to the tensor core
            epi_sync();
            stamp(p.trace, k, C, c, 2);
            stamp_clk(p.trace, k, C, c, 1);

            // ---- rows: passes of up to kPassRows rows, each over all inputs in chunks ---------------
            float *lg = nullptr;
            if (op.epi == EPI_LMHEAD && st->logits != nullptr && st->step >= st->logits_from)
                lg = st->logits + st->logits_stride * (long long)st->step;
            float bv = -INFINITY;
            int bi = INT_MAX;
            for (int p0 = 0; p0 < R && !ab.on(); p0 += op.pass_rows) {
                const int rows_p = min(op.pass_rows, R - p0);
                const int nrt = (rows_p + 15) >> 4;                 // 16-row tiles of the pass (<= 4)
                const int row = R0 + p0 + 2 * tid;                  // packed row (row, row + 1)
                const bool mine = tid < rows_p / 2 && row < op.n_valid;
                if (p0 > 0) preload(p0, pre0, pre1, pcs, psn);      // pass 0: preloaded before the input
                // tensor-core products: A = 16 weight rows x 16 inputs (ldmatrix from the swizzled
                // unit), B column 0 = hi, column 1 = lo of the inputs, fp32 accumulators; warp w
                // takes k-steps w, w + 4, ... of every row tile
                float d[4][4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) d[i][j] = 0.f;
                float yrow = 0.f;                                   // int8: this thread's row of the pass
                if (q8) {
                    I8Ring rg{ring, full, empty, s_accb, S, SB, s, round, consumed, acc_par};
                    if (p0 == 0) {
                        stamp(p.trace, k, C, c, 4);
                        stamp_clk(p.trace, k, C, c, 2);
                    }
                    yrow = i8_pass(rg, tmem, dg, bsc, rows_p, K, op.chunk_w, ab);
                    s = rg.s;
                    round = rg.round;
                    consumed = rg.consumed;
                    acc_par = rg.acc_par;
                } else {
                for (int q0 = 0; q0 < K; q0 += op.chunk_w) {
                    const int wq = min(op.chunk_w, K - q0);
                    if (!wait_bar(&full[s], (uint32_t)round & 1u, ab)) break;
                    if (p0 == 0 && q0 == 0) {
                        stamp(p.trace, k, C, c, 4);
                        stamp_clk(p.trace, k, C, c, 2);
                    }
                    const uint32_t unit = smem_u32(ring + (size_t)s * SB);
                    // row stride 2 wq bytes, 16-input k-steps
                    if (nrt == 1)
                        unit_mma<4>(d, unit, wq * 2, wq >> 4, rows_p, nrt, q0, xh, xl, warp, lane);
                    else
                        unit_mma<1>(d, unit, wq * 2, wq >> 4, rows_p, nrt, q0, xh, xl, warp, lane);
                    epi_sync();                                     // every warp is done with the unit
                    if (tid == 0) mbar_arrive(&empty[s]);
                    ++consumed;
                    if (++s == S) {
                        s = 0;
                        ++round;
                    }
                }
                }
                if (p0 == 0) stamp_clk(p.trace, k, C, c, 3);
                // row sums: lanes 4i hold rows i and i + 8 of each tile (columns 0 = hi, 1 = lo);
                // tile rt's U accumulator slots are summed in slot order
                if (q8) {
                    const int r8 = i8_row_of_thread(rows_p, tid);    // this thread's row (<= 128 rows)
                    if (r8 >= 0 && r8 < rows_p) (&red[0][0])[r8] = yrow;
                } else if ((lane & 3) == 0) {
                    if (nrt == 1)
                        rows_from_acc<4>(d, red[warp], nrt, lane);
                    else
                        rows_from_acc<1>(d, red[warp], nrt, lane);
                }
                epi_sync();
                if (!mine) continue;
                const int r2 = 2 * tid;
                float y0 = q8 ? (&red[0][0])[r2] : ((red[0][r2] + red[1][r2]) + red[2][r2]) + red[3][r2];
                float y1 = q8 ? (&red[0][0])[r2 + 1] : ((red[0][r2 + 1] + red[1][r2 + 1]) + red[2][r2 + 1]) + red[3][r2 + 1];
                if (Q8 && op.ksplit > 1) {
                    // split inputs: CTA h > 0 of the row group hands its row partials to CTA 0
                    // (region h - 1 of lksp, op.N words each), which adds them in h order and runs
                    // the epilogue
                    if (!fin) {
                        ll_st2(op.lksp + (size_t)(sh.K0 / K - 1) * op.N + row, ll_wordf(y0, tag), ll_wordf(y1, tag));
                        continue;
                    }
                    uint64_t w[kMaxKsplit - 1][2];
                    ll_poll<kMaxKsplit - 1>(w, (1u << (op.ksplit - 1)) - 1u,
                                            [&](int j) { return op.lksp + (size_t)j * op.N + row; }, tag, ab);
#pragma unroll
                    for (int j = 0; j < kMaxKsplit - 1; ++j)
                        if (j < op.ksplit - 1) {
                            y0 += ll_f(w[j][0]);
                            y1 += ll_f(w[j][1]);
                        }
                }
                if (op.epi == EPI_RESID) {
                    ll_st2(op.lout + row, ll_wordf(pre0 + y0, tag), ll_wordf(pre1 + y1, tag));
                } else if (op.epi == EPI_LMHEAD) {
                    if (lg) lg[row] = y0;
                    if (y0 > bv) {
                        bv = y0;
                        bi = row;
                    }
                    if (row + 1 < op.n_valid) {
                        if (lg) lg[row + 1] = y1;
                        if (y1 > bv) {
                            bv = y1;
                            bi = row + 1;
                        }
                    }
                } else if (op.epi == EPI_SWIGLU) {
                    const float a = (y0 / (1.0f + expf(-y0))) * y1;
                    const __half ah = __float2half_rn(a);
                    op.out_h[row / 2] = ah;
                    op.out_l[row / 2] = __float2half_rn(a - __half2float(ah));
                } else {  // EPI_QKV: packed rows (2q, 2q+1) are dims (d, d + hd/2) of one head
                    const int P2 = row / 2;
                    const int hh = P2 / half_hd, dd = P2 - hh * half_hd;
                    const float a0 = y0 + pre0, a1 = y1 + pre1;
                    if (hh < p.nh + p.nkv) {
                        const float o0 = __fadd_rn(__fmul_rn(a0, pcs), -__fmul_rn(a1, psn));
                        const float o1 = __fadd_rn(__fmul_rn(a1, pcs), __fmul_rn(a0, psn));
                        if (hh < p.nh) {
                            ll_st1(op.lout + hh * HD + dd, ll_wordf(o0, tag));
                            ll_st1(op.lout + hh * HD + dd + half_hd, ll_wordf(o1, tag));
                        } else {
                            const int g = hh - p.nh;
                            __half *kr = op.kc + ((size_t)g * p.cap + ss.slot) * HD;
                            kr[dd] = __float2half_rn(o0);
                            kr[dd + half_hd] = __float2half_rn(o1);
                            ll_st1(op.lkv + (size_t)g * HD + dd, ll_word(half2_bits(o0, o1), tag));
                        }
                    } else {
                        const int g = hh - p.nh - p.nkv;
                        __half *vr = op.vc + ((size_t)g * p.cap + ss.slot) * HD;
                        vr[dd] = __float2half_rn(a0);
                        vr[dd + half_hd] = __float2half_rn(a1);
                        ll_st1(op.lkv + (size_t)g * HD + half_hd + dd, ll_word(half2_bits(a0, a1), tag));
                    }
                }
            }
            epi_sync();                                             // `red` is reused by the next op
            stamp(p.trace, k, C, c, 5);
            stamp_clk(p.trace, k, C, c, 4);

            if (op.epi == EPI_LMHEAD) {
                lmhead_finish(p, op, ss, st, bv, bi, c);
            } else if (op.sig >= 0) {
                if (tid == 0) red_add_release(p.cnt + op.sig, 1ull);   // after the barrier above
            }
            stamp(p.trace, k, C, c, 3);
            stamp_clk(p.trace, k, C, c, 5);
        }
        cp_async_wait_all();
        if (tid == 0) s_consumed = consumed;
    }

    if (Q8 && warp < kEpiThreads / 32 && lane == 0) {
        // every MMA issued has completed (one more commit per issuer tracks all of them) before
        // TMEM goes back
        mma_commit(&s_accb[0]);
        mbar_wait_bounded(&s_accb[0], acc_par & 1u);
    }
    if (Q8) tc_fence_before();
    __syncthreads();
    if (Q8 && warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kStepTmemCols));
    }
    if (warp == kProducerWarp && lane == 0) {
        // after an abort, stages may still be in flight: let their copies land before exiting
        for (int i = s_consumed; i < s_issued; ++i) mbar_wait_bounded(&full[i % S], (uint32_t)(i / S) & 1u);
    }
}

// Pack an fp16 N x K matrix into the row-block layout of the step kernel. Packed row r is source
// row row_of[r] of `a` (< rows_a) or of `b` (row_of - rows_a); row_of < 0 is a zero row. The rows
// of CTA c are [R0, R0 + R) (R0 = 2 floor(P c / grid), P = N / 2), stored from byte R0 * K * 2 as
// units in (pass, chunk) order: pass i covers rows [i * pass_rows, ...) of the CTA, chunk j inputs
// [j * chunk_w, ...); a unit is [its rows][its inputs] fp16 in which the 16-byte chunks of each
// 128-byte segment of row r are XOR-permuted by r & 7 (8 rows read by one ldmatrix hit 8 different
// bank groups). One thread per 8 inputs of a row.
__global__ void k_pack_rows(uint8_t *dst, const __half *a, int rows_a, const __half *b, const int *row_of, int N, int K,
                            int grid, int pass_rows, int chunk_w) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long total = (long long)N * K / 8;
    if (idx >= total) return;
    const int row = (int)(idx / (K / 8));
    const int k = (int)(idx - (long long)row * (K / 8)) * 8;
    const int P = N / 2, pair = row / 2;
    int c = (int)(((long long)pair * grid) / P);
    while (c > 0 && (long long)P * c / grid > pair) --c;
    while (c + 1 < grid && (long long)P * (c + 1) / grid <= pair) ++c;
    const int R0 = 2 * (int)((long long)P * c / grid);
    const int R = 2 * (int)((long long)P * (c + 1) / grid) - R0;
    const int lr = row - R0;
    const int pi = lr / pass_rows;
    const int rows_p = min(pass_rows, R - pi * pass_rows);
    const int qi = k / chunk_w;
    const int wq = min(chunk_w, K - qi * chunk_w);
    const int r = lr - pi * pass_rows;                    // row within the unit
    const int j = (k - qi * chunk_w) / 8;                   // 16-byte chunk within the unit's row
    const int pj = (j & ~7) | ((j & 7) ^ (r & 7));          // 128-byte segments XOR-swizzled by row
    const size_t off = (size_t)R0 * K * 2 + (size_t)pi * pass_rows * K * 2 + (size_t)rows_p * qi * chunk_w * 2 +
                       (size_t)r * wq * 2 + (size_t)pj * 16;
    const int src = row_of[row];
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (src >= 0) {
        const __half *rp = src < rows_a ? a + (size_t)src * K : b + (size_t)(src - rows_a) * K;
        v = *reinterpret_cast<const uint4 *>(rp + k);
    }
    *reinterpret_cast<uint4 *>(dst + off) = v;
}

// Pack a blockwise-int8 N x K matrix (an fp16 scale per row and 32 inputs) into the step kernel's
// int8 units; CTA c holds its share (gemv_share: its row group's rows over its part of the inputs)
// from c * cta_bytes, in (pass, chunk) order. A unit of rows_p rows x wq inputs holds, per 32-input block, [half][row][16 bytes] (the
// tensor core's K-major core matrices, see unit_i8_issue), then the scales [row][block]. One
// thread per row and 32-input block.
__global__ void k_pack_rows_i8(uint8_t *dst, const int8_t *a, const __half *as, int rows_a, const int8_t *b,
                               const __half *bs, const int *row_of, int N, int K, int grid, int ksplit,
                               int pass_rows, int chunk_w, int cta_bytes) {
    const int nbk = K / 32;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)N * nbk) return;
    const int row = (int)(idx / nbk);
    const int kg = (int)(idx - (long long)row * nbk) * 32;  // input of the whole row
    const int P = N / 2, pair = row / 2, G = grid / ksplit;
    int g = (int)(((long long)pair * G) / P);               // the row group owning the pair
    while (g > 0 && (long long)P * g / G > pair) --g;
    while (g + 1 < G && (long long)P * (g + 1) / G <= pair) ++g;
    const int Kc = K / ksplit, c = g * ksplit + kg / Kc;     // the CTA owning the input's part
    const int k = kg - (kg / Kc) * Kc;                       // input within the CTA's part
    const GemvShare sh = gemv_share(N, K, grid, ksplit, c);
    const int R0 = sh.R0, R = sh.R;
    const int lr = row - R0;
    const int pi = lr / pass_rows;
    const int rows_p = min(pass_rows, R - pi * pass_rows);
    const int qi = k / chunk_w;
    const int wq = min(chunk_w, Kc - qi * chunk_w);
    const int r = lr - pi * pass_rows;
    size_t pass_full = 0;                                  // bytes of a full pass (pass_rows rows)
    for (int q0 = 0; q0 < Kc; q0 += chunk_w) pass_full += step_unit_bytes(WF_I8, pass_rows, min(chunk_w, Kc - q0));
    uint8_t *unit = dst + (size_t)c * cta_bytes + (size_t)pi * pass_full +
                    (size_t)qi * step_unit_bytes(WF_I8, rows_p, chunk_w);
    const int bl = (k - qi * chunk_w) / 32;                // block within the unit
    uint4 v0 = make_uint4(0u, 0u, 0u, 0u), v1 = v0;
    __half sc = __ushort_as_half(0);
    const int src = row_of[row];
    if (src >= 0) {
        const int8_t *rp = src < rows_a ? a + (size_t)src * K : b + (size_t)(src - rows_a) * K;
        sc = src < rows_a ? as[(size_t)src * nbk + kg / 32] : bs[(size_t)(src - rows_a) * nbk + kg / 32];
        v0 = *reinterpret_cast<const uint4 *>(rp + kg);
        v1 = *reinterpret_cast<const uint4 *>(rp + kg + 16);
    }
    uint8_t *blk = unit + (size_t)bl * rows_p * 32;
    *reinterpret_cast<uint4 *>(blk + (size_t)r * 16) = v0;
    *reinterpret_cast<uint4 *>(blk + (size_t)rows_p * 16 + (size_t)r * 16) = v1;
    reinterpret_cast<__half *>(unit + (size_t)rows_p * wq)[(size_t)r * (wq / 32) + bl] = sc;
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Packed int8 bytes of R rows (passes of pass_rows rows, each all K inputs in chunks of chunk_w).
static size_t i8_rows_bytes(int R, int K, int pass_rows, int chunk_w) {
    size_t b = 0;
    for (int p0 = 0; p0 < R; p0 += pass_rows)
        for (int q0 = 0; q0 < K; q0 += chunk_w)
            b += step_unit_bytes(WF_I8, std::min(pass_rows, R - p0), std::min(chunk_w, K - q0));
    return b;
}

// Rows per pass and inputs per unit, each unit at most one stage: for fp16 the fewest units for
// the busiest CTA (ties: more rows per pass); for int8 the least tensor-core time, every 32-input
// block of a pass one MMA (~48 cycles at M = 128, ~32 at M = 64) plus ~1,000 cycles a unit.
// An int8 op (not the LM head) whose CTAs would hold few rows (<= 32) is split over its inputs:
// two CTAs share a row group, each over half of K, so a block MMA covers twice the rows and a CTA
// issues and reads back half the block MMAs and digitizes half the input; the second CTA hands
// its row partials to the first. A long input (K >= 16,384, or any K when max_ksplit >= 8) is
// split four ways when a row group then fits one M = 128 pass.
void plan_step_gemv(StepOp &o, int num_sms, int stage_bytes, int max_ksplit) {
    const int P = o.N / 2;
    const bool i8 = o.fmt == WF_I8;
    o.ksplit = 1;
    o.grid = std::max(1, std::min(num_sms, P));
    if (i8 && max_ksplit >= 2 && o.epi != EPI_LMHEAD && o.K % 256 == 0 && num_sms >= 2) {
        const int G = std::min(num_sms / 2, P);
        if (2 * ((P + G - 1) / G) <= 64) {
            o.ksplit = 2;
            o.grid = 2 * G;
        }
    }
    if (o.ksplit == 2 && max_ksplit >= 4 && o.K % 512 == 0 && num_sms >= 4 && (o.K >= 16384 || max_ksplit >= 8)) {
        const int G = std::min(num_sms / 4, P);
        if (2 * ((P + G - 1) / G) <= kPassRowsI8) {
            o.ksplit = 4;
            o.grid = 4 * G;
        }
    }
    const int G = o.grid / o.ksplit, Kc = o.K / o.ksplit;
    const int rmax = 2 * ((P + G - 1) / G);                                 // rows of the busiest CTA
    const int gran = i8 ? 64 : 256;                                          // chunk_w granule (int8: even blocks)
    long long best = -1;
    for (int pr = std::min(i8 ? kPassRowsI8 : kPassRows, rmax); pr >= 2; pr -= 2) {
        // widest unit within a stage (int8: at most kUnitBlocksI8 blocks, one TMEM column group each)
        int w = i8 ? std::min((stage_bytes - 16) / (pr + pr / 16 + 1), 32 * kUnitBlocksI8) : stage_bytes / (pr * 2);
        w = w / gran * gran;
        if (w >= Kc) w = Kc;
        if (w < gran && w != Kc) continue;
        while (i8 && w > gran && step_unit_bytes(WF_I8, pr, w) > (uint32_t)stage_bytes) w -= gran;
        const long long passes = (rmax + pr - 1) / pr, units = passes * ((Kc + w - 1) / w);
        const long long cost = i8 ? passes * (Kc / 32) * (pr > 64 ? 48 : 32) + units * 1000 : units;
        if (best < 0 || cost < best) {
            best = cost;
            o.pass_rows = pr;
            o.chunk_w = w;
        }
    }
    if (best < 0) {
        o.pass_rows = 2;
        o.chunk_w = gran;
    }
    const size_t cb = i8 ? i8_rows_bytes(rmax, Kc, o.pass_rows, o.chunk_w) : 0;
    o.cta_bytes = cb <= (size_t)INT_MAX ? (int)cb : -1;
}

size_t step_gemv_bytes(const StepOp &o) {
    return o.fmt == WF_I8 ? (size_t)o.grid * (size_t)std::max(o.cta_bytes, 0) : (size_t)o.N * o.K * 2;
}

bool step_gemv_supported(const StepOp &o, int stage_bytes) {
    const bool i8 = o.fmt == WF_I8;
    const int ks = std::max(o.ksplit, 1);
    if (ks > kMaxKsplit || (ks & (ks - 1)) || o.grid % ks || (ks > 1 && (!i8 || o.epi == EPI_LMHEAD || o.K % (128 * ks))))
        return false;
    if (i8 && (o.K % 128 || o.chunk_w % 64 || o.chunk_w > 32 * kUnitBlocksI8 || o.cta_bytes <= 0)) return false;
    if (!i8 && (o.fmt != WF_F16 || (o.chunk_w != o.K && o.chunk_w % 256))) return false;
    return o.N % 2 == 0 && o.K % 64 == 0 && o.pass_rows % 2 == 0 && o.pass_rows >= 2 &&
           o.pass_rows <= (i8 ? kPassRowsI8 : kPassRows) &&
           step_unit_bytes(o.fmt, o.pass_rows, o.chunk_w) <= (uint32_t)stage_bytes &&
           (o.pro == PRO_NORM || o.pro == PRO_EMBED_NORM || (i8 && o.pro == PRO_ATTN) ? o.K <= kNormRegs * 4 * kEpiThreads
                                                                                      : true);
}

size_t step_attn_smem_bytes(int hd) { return hd == 64 ? AttnRegion<64>::bytes : AttnRegion<128>::bytes; }

static size_t step_static_reserve() { return 2048; }   // static shared memory of k_step, rounded up

// Dynamic shared memory: ring [stages x stage_bytes] | vector region | ops k, k + 1 | barriers.
// The vector region holds a GEMV's input halves (4 K bytes) and, from attn_off on (after the QKV
// projection's input, 4 hidden bytes), the attention staging region.
StepLayout step_layout(int hidden, int xmax, int hd, int stages, bool i8) {
    StepLayout L{};
    L.stages = stages;
    // a GEMV input of K values: fp16 hi / lo halves (4 K bytes) or, for int8 weights, four digit
    // rows of K + 16 bytes and K / 32 block scales
    auto in_bytes = [&](size_t K) { return i8 ? 4 * (K + 16) + K / 8 : 4 * K; };
    L.attn_off = (int)align_up(in_bytes((size_t)hidden), 128);
    L.vec_bytes = (int)align_up(std::max(in_bytes((size_t)xmax), (size_t)L.attn_off + step_attn_smem_bytes(hd)), 128);
    const size_t fixed = (size_t)L.vec_bytes + 2 * sizeof(StepOp) + (size_t)stages * 16;
    const size_t budget = 227 * 1024 - step_static_reserve();
    if (stages < 2 || fixed >= budget) return L;
    L.stage_bytes = (int)std::min<size_t>(kMaxStageBytes, (budget - fixed) / stages / 1024 * 1024);
    L.smem = (size_t)stages * L.stage_bytes + fixed;
    return L;
}

cudaError_t launch_pack_rows(uint8_t *dst, const __half *a, int rows_a, const __half *b, const int *row_of,
                             const StepOp &plan, cudaStream_t s) {
    if (plan.N % 2 || plan.K % 8) return cudaErrorInvalidValue;
    const long long total = (long long)plan.N * plan.K / 8;
    k_pack_rows<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(dst, a, rows_a, b, row_of, plan.N, plan.K, plan.grid,
                                                                plan.pass_rows, plan.chunk_w);
    return cudaGetLastError();
}

cudaError_t launch_pack_rows_i8(uint8_t *dst, const int8_t *a, const __half *as, int rows_a, const int8_t *b,
                                const __half *bs, const int *row_of, const StepOp &plan, cudaStream_t s) {
    if (plan.fmt != WF_I8 || plan.N % 2 || plan.K % 128 || plan.cta_bytes <= 0) return cudaErrorInvalidValue;
    const long long total = (long long)plan.N * (plan.K / 32);
    k_pack_rows_i8<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(dst, a, as, rows_a, b, bs, row_of, plan.N, plan.K,
                                                                   plan.grid, std::max(plan.ksplit, 1),
                                                                   plan.pass_rows, plan.chunk_w, plan.cta_bytes);
    return cudaGetLastError();
}

template <int HD, bool Q8, bool GR>
static cudaError_t step_launch_t(const StepParams *p, int grid, size_t smem, cudaStream_t s, bool pdl) {
    if (p == nullptr) {
        cudaError_t e = cudaFuncSetAttribute(k_step<HD, Q8, GR>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        return cudaFuncSetAttribute(k_step<HD, Q8, GR>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    (int)cudaSharedmemCarveoutMaxShared);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GR ? kThreadsGR : kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeCooperative;
    attr[na].val.cooperative = 1;
    ++na;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k_step<HD, Q8, GR>, *p);
}

template <bool Q8, bool GR>
static cudaError_t step_launch_hd(int hd, const StepParams *p, int grid, size_t smem, cudaStream_t s, bool pdl) {
    if (hd == 128) return step_launch_t<128, Q8, GR>(p, grid, smem, s, pdl);
    if (hd == 64) return step_launch_t<64, Q8, GR>(p, grid, smem, s, pdl);
    return cudaErrorInvalidValue;
}

cudaError_t prepare_step(int hd, size_t smem, bool q8) {
    for (const bool gr : {false, true}) {
        const cudaError_t e = q8 ? (gr ? step_launch_hd<true, true>(hd, nullptr, 0, smem, nullptr, false)
                                       : step_launch_hd<true, false>(hd, nullptr, 0, smem, nullptr, false))
                                 : (gr ? step_launch_hd<false, true>(hd, nullptr, 0, smem, nullptr, false)
                                       : step_launch_hd<false, false>(hd, nullptr, 0, smem, nullptr, false));
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_step(int hd, const StepParams &p, int grid, size_t smem, cudaStream_t s, bool pdl, bool q8,
                        bool grouped) {
    if (p.stages < 2 || p.stage_bytes < 1024 || p.stage_bytes % 1024 || p.stage_bytes > kMaxStageBytes ||
        p.nh / p.nkv > kGroup || p.nh * p.max_chunks > grid || p.max_chunks > kStepMaxChunks || p.attn_off % 128 ||
        p.group_chunks < 1 || p.nkv * p.group_chunks > grid || p.group_chunks > kStepMaxChunks ||
        p.part_stride < std::max(p.max_chunks, p.group_chunks) ||
        p.vec_bytes % 128 || (size_t)p.attn_off + step_attn_smem_bytes(hd) > (size_t)p.vec_bytes)
        return cudaErrorInvalidValue;
    if (q8) return grouped ? step_launch_hd<true, true>(hd, &p, grid, smem, s, pdl)
                           : step_launch_hd<true, false>(hd, &p, grid, smem, s, pdl);
    return grouped ? step_launch_hd<false, true>(hd, &p, grid, smem, s, pdl)
                   : step_launch_hd<false, false>(hd, &p, grid, smem, s, pdl);
}

}  // namespace sp
