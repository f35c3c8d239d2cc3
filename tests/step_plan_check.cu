// Host-only check of the step kernel's GEMV plans (no GPU): plans every GEMV of a model shape the
// way sp_engine_create does (input splits first, then the shared-memory layout, then the units)
// with the library's own plan_step_gemv / step_layout / step_gemv_supported, and checks:
//   * every plan is supported and its unit fits a ring stage;
//   * split GEMVs: ksplit divides the grid, K / ksplit is a multiple of 128, only int8 and never
//     the LM head; the row groups (gemv_share) cover the row pairs [0, N / 2) once, the CTAs of a
//     group share its rows and cover [0, K) once;
//   * a CTA's input share fits the layout's vector region;
//   * int8: cta_bytes holds the units of the busiest CTA.
// Usage: step_plan_check H I heads kv_heads head_dim vocab tied i8 [expected ksplit x5 | -]
// Prints "ok" and exits 0, or names the broken check and exits 1.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "kernels.cuh"

using namespace sp;

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
static size_t unit_bytes(bool i8, int rows, int w) {   // the unit size rule of the step kernel
    return i8 ? (size_t)rows * w + (((size_t)(w / 32) * rows * 2 + 15) & ~(size_t)15) : (size_t)rows * w * 2;
}

static int fails = 0;
#define CHECK(cond, ...)                                                                                 \
    do {                                                                                                 \
        if (!(cond)) {                                                                                   \
            std::printf("FAIL %s:%d ", __FILE__, __LINE__);                                              \
            std::printf(__VA_ARGS__);                                                                    \
            std::printf("\n");                                                                           \
            ++fails;                                                                                     \
        }                                                                                                \
    } while (0)

int main(int argc, char **argv) {
    if (argc < 9) {
        std::printf("usage: %s H I heads kv_heads head_dim vocab tied i8 [ks x5]\n", argv[0]);
        return 2;
    }
    const size_t H = atoi(argv[1]), I = atoi(argv[2]), nh = atoi(argv[3]), nkv = atoi(argv[4]), HD = atoi(argv[5]);
    const size_t V = atoi(argv[6]);
    const bool tied = atoi(argv[7]) != 0, i8 = atoi(argv[8]) != 0;
    const int sms = 148, max_ks = kMaxKsplit;
    const size_t QR = (nh + 2 * nkv) * HD, QRp = align_up(QR, 2), Hp = align_up(H, 2), GUp = align_up(2 * I, 2);
    const size_t VP = align_up(V, 2);
    auto base = [&](size_t N, size_t K, int pro, int epi, bool q8, int stage) {
        StepOp o{};
        o.kind = OP_GEMV;
        o.fmt = q8 ? WF_I8 : WF_F16;
        o.pro = pro;
        o.epi = epi;
        o.N = (int)N;
        o.K = (int)K;
        plan_step_gemv(o, sms, stage, max_ks);
        return o;
    };
    auto share_k = [&](size_t N, size_t K, int pro, int epi) {
        return K / (size_t)std::max(base(N, K, pro, epi, i8, 64 * 1024).ksplit, 1);
    };
    const int xmax = (int)align_up(std::max({H, share_k(Hp, I, PRO_PLAIN, EPI_RESID),
                                             share_k(Hp, nh * HD, PRO_ATTN, EPI_RESID)}), 8);
    StepLayout L = step_layout((int)H, xmax, (int)HD, 3, i8);
    if (L.stage_bytes < 16 * 1024) L = step_layout((int)H, xmax, (int)HD, 2, i8);
    CHECK(L.stage_bytes >= 16 * 1024, "no room for the ring (stage %d)", L.stage_bytes);
    const StepOp ops[5] = {base(QRp, H, PRO_NORM, EPI_QKV, i8, L.stage_bytes),
                           base(Hp, H, PRO_ATTN, EPI_RESID, i8, L.stage_bytes),
                           base(GUp, H, PRO_NORM, EPI_SWIGLU, i8, L.stage_bytes),
                           base(Hp, I, PRO_PLAIN, EPI_RESID, i8, L.stage_bytes),
                           base(VP, H, PRO_NORM, EPI_LMHEAD, i8 && !tied, L.stage_bytes)};
    const char *names[5] = {"qkv", "o", "gate_up", "down", "lm_head"};
    for (int n = 0; n < 5; ++n) {
        const StepOp &o = ops[n];
        const bool q8 = o.fmt == WF_I8;
        const int ks = std::max(o.ksplit, 1);
        CHECK(step_gemv_supported(o, L.stage_bytes), "%s: plan not supported", names[n]);
        CHECK(unit_bytes(q8, o.pass_rows, o.chunk_w) <= (size_t)L.stage_bytes, "%s: unit above a stage", names[n]);
        CHECK(o.grid >= 1 && o.grid <= sms && o.grid % ks == 0, "%s: grid %d, ksplit %d", names[n], o.grid, ks);
        if (ks > 1) {
            CHECK(q8 && o.epi != EPI_LMHEAD && o.K % (128 * ks) == 0, "%s: bad split %d", names[n], ks);
        }
        if (argc >= 14 && argv[9][0] != '-') CHECK(ks == atoi(argv[9 + n]), "%s: ksplit %d, expected %s", names[n], ks, argv[9 + n]);
        // row groups and input parts
        const int P = o.N / 2, G = o.grid / ks;
        std::vector<int> owner(P, -1);
        int rmax = 0;
        for (int g = 0; g < G; ++g) {
            const GemvShare s0 = gemv_share(o.N, o.K, o.grid, ks, g * ks);
            rmax = std::max(rmax, s0.R);
            int k_next = 0;
            for (int h = 0; h < ks; ++h) {
                const GemvShare s = gemv_share(o.N, o.K, o.grid, ks, g * ks + h);
                CHECK(s.R0 == s0.R0 && s.R == s0.R, "%s: CTAs of group %d own different rows", names[n], g);
                CHECK(s.K0 == k_next && s.Kc == o.K / ks, "%s: group %d input parts", names[n], g);
                k_next = s.K0 + s.Kc;
            }
            CHECK(k_next == o.K, "%s: group %d covers %d of %d inputs", names[n], g, k_next, o.K);
            CHECK(s0.R0 % 2 == 0 && s0.R % 2 == 0, "%s: odd rows", names[n]);
            for (int pr = s0.R0 / 2; pr < (s0.R0 + s0.R) / 2; ++pr) {
                CHECK(pr >= 0 && pr < P && owner[pr] < 0, "%s: pair %d owned twice or out of range", names[n], pr);
                if (pr >= 0 && pr < P) owner[pr] = g;
            }
        }
        CHECK(std::count(owner.begin(), owner.end(), -1) == 0, "%s: unowned row pairs", names[n]);
        // the CTA's input share in the vector region
        const size_t kc = (size_t)o.K / ks;
        const size_t in = q8 ? 4 * (kc + 16) + kc / 8 : 4 * (size_t)o.K;
        CHECK(in <= (size_t)L.vec_bytes, "%s: input share %zu above the vector region %d", names[n], in, L.vec_bytes);
        if (q8) {   // the busiest CTA's units
            size_t b = 0;
            for (int p0 = 0; p0 < rmax; p0 += o.pass_rows)
                for (int q0 = 0; q0 < (int)kc; q0 += o.chunk_w)
                    b += unit_bytes(true, std::min(o.pass_rows, rmax - p0), std::min(o.chunk_w, (int)kc - q0));
            CHECK(o.cta_bytes > 0 && (size_t)o.cta_bytes >= b, "%s: cta_bytes %d < %zu", names[n], o.cta_bytes, b);
        }
        std::printf("%s %s N=%d K=%d grid=%d ksplit=%d pass_rows=%d chunk=%d\n", names[n], q8 ? "i8" : "f16", o.N, o.K,
                    o.grid, ks, o.pass_rows, o.chunk_w);
    }
    std::printf("stage=%d stages=%d vec=%d\n", L.stage_bytes, L.stages, L.vec_bytes);
    if (fails) return 1;
    std::printf("ok\n");
    return 0;
}
