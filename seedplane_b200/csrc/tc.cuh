// tcgen05 (5th-generation tensor core) helpers shared by the weight-streaming kernels, sm_100a.
//
// The streamed matrices are packed as 128 x 16 fp16 tiles (4 KB) in the canonical K-major,
// non-swizzled UMMA layout: core matrix (r, h) (rows 8r..8r+7, inputs 8h..8h+7 of the tile) at
// (2r + h) * 128 bytes, i.e. LBO = 128 B between the two K halves, SBO = 256 B between row groups.
// The activation (B operand, N = 8) uses the same core layout: 256 bytes per k-tile.
#pragma once

#include <climits>

#include "common.cuh"

namespace sp {

SP_DEVINL uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);   // version 1, no swizzle
}

// kind::f16 instruction descriptor: D fp32, A/B fp16, both K-major, M = 128, N = 8.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | ((8u >> 3) << 17) | ((128u >> 4) << 24);

SP_DEVINL void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate));
}
SP_DEVINL void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
SP_DEVINL void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
SP_DEVINL void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

SP_DEVINL void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- 128B-swizzled K-major operands (the persistent step kernel) --------------------------------
// A row of 64 fp16 inputs is 128 bytes; 8 rows form a 1024-byte atom in which the 16-byte chunk c of
// row r is stored at chunk position c ^ r. K advances by 16 inputs (32 bytes) inside the atom by
// moving the start address; 8-row groups follow each other at `sbo` bytes (0: every group reads the
// same atom, which is how one 1 KB activation atom feeds all 128 rows of the A operand).
SP_DEVINL uint64_t smem_desc_sw128(uint32_t addr, uint32_t sbo) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | (1ull << 16) | ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) |
           (1ull << 46) | (2ull << 61);
}
// kind::f16 instruction descriptor: D fp32, A/B fp16, both K-major, M = 128, N = 256.
constexpr uint32_t kIdescM128N256 = (1u << 4) | ((256u >> 3) << 17) | ((128u >> 4) << 24);

SP_DEVINL void mma_f16_id(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// 32 consecutive TMEM columns of this thread's lane (no wait: call tmem_wait_ld before use).
SP_DEVINL void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// 16 consecutive TMEM columns of this thread's lane (no wait).
SP_DEVINL void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
}

SP_DEVINL void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- kind::i8 (the step kernel's int8 units) ---------------------------------------------------
// D s32, A and B signed 8-bit, both K-major, N = 8; one MMA covers K = 32 (32 bytes a row).
// M = 64 (rows r at TMEM lanes r % 16 + 32 (r / 16)) costs about two thirds of M = 128 per MMA.
constexpr uint32_t kIdescI8M128N8 = (2u << 4) | (1u << 7) | (1u << 10) | ((8u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescI8M64N8 = (2u << 4) | (1u << 7) | (1u << 10) | ((8u >> 3) << 17) | ((64u >> 4) << 24);

SP_DEVINL void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc = kIdescI8M128N8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0u));
}
// 4 consecutive TMEM columns of this thread's lane (no wait).
SP_DEVINL void tmem_ld4_nowait(uint32_t taddr, uint32_t (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}

SP_DEVINL void tc_argmax_merge(float &v, int &i, float ov, int oi) {
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
}

// The CTA whose tile range [floor(T*c/C), floor(T*(c+1)/C)) contains tile g.
SP_DEVINL int tc_cta_of(long long g, long long T, int C) {
    int c = (int)((g * C) / T);
    while (c > 0 && T * c / C > g) --c;
    while (c + 1 < C && T * (c + 1) / C <= g) ++c;
    return c;
}

}  // namespace sp
