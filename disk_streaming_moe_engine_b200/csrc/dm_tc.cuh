// dm_tc.cuh — 5th-generation tensor core (tcgen05) helpers for sm_100a: tensor-memory
// allocation, shared-memory matrix descriptors, the kind::f16 MMA with fp32 accumulation
// in tensor memory, completion through mbarriers, and tensor-memory loads.
//
// Operand layout used by every caller: K-major tiles of 64 bf16 (128 bytes) per row with
// the 128-byte swizzle, rows in 8-row groups of 1024 bytes: the 16-byte unit u of row r
// sits at (r / 8) * 1024 + (r % 8) * 128 + ((u ^ (r % 8)) * 16).  A tile starts on a
// 1024-byte boundary.  One MMA consumes K = 16 (32 bytes of each row); the next K step of
// the same tile advances the descriptor's start address by 32 bytes.
#pragma once
#include <cstdint>

#include "dm_common.cuh"

namespace dm {

// Shared-memory matrix descriptor (tcgen05 format): start address >> 4 in bits [0,14),
// leading byte offset (16 bytes, unused by swizzled K-major layouts) >> 4 in [16,30),
// stride byte offset (1024 bytes between 8-row groups) >> 4 in [32,46), version 1 in
// [46,48), layout SWIZZLE_128B (2) in [61,64).
DM_DEV uint64_t tc_desc_sw128(uint32_t smem_addr) {
    return static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulator (bits [4,6) = 1), A and B bf16
// (bits [7,10) and [10,13) = 1), both K-major, N >> 3 in [17,23), M >> 4 in [24,29).
DM_DEV uint32_t tc_idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// The same with A and B fp16 (bits [7,10) and [10,13) = 0).
DM_DEV uint32_t tc_idesc_f16(int M, int N) {
    return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
DM_DEV void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, issued by one thread (kind::f16: bf16 or fp16 operands,
// as the instruction descriptor says).  A (M = 128) sits in tensor memory with row m in
// lane m and two consecutive 16-bit K elements per 32-bit column (the lower one in the low
// half); one K = 16 step reads 8 columns.
DM_DEV void tc_mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
        : "memory");
}

// The mbarrier receives one arrival once every tcgen05 operation this thread issued
// before the commit has completed (their shared-memory reads included).
DM_DEV void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

DM_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DM_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Allocation by one whole warp; the base address is written to *slot (shared memory).
DM_DEV void tc_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
DM_DEV void tc_dealloc(uint32_t base, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}

// 16 consecutive fp32 columns of this thread's lane (warp w reads lanes 32 (w % 4) ..).
DM_DEV void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// This thread's lane, 16 consecutive 32-bit columns from registers.
DM_DEV void tc_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
DM_DEV void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
DM_DEV void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Byte offset of element k (0..63) of row r in a 128-byte-swizzled K-major tile.
DM_DEV uint32_t sw128_off(int r, int k) {
    return static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((((k >> 3) ^ (r & 7)) & 7) << 4) + (k & 7) * 2);
}

// Phase-parity bookkeeping of an mbarrier ring: use u of a ring of n stages waits for
// parity (u / n) & 1 on its "full" barrier and (u / n) & 1 ^ 1 on its "empty" barrier.
DM_DEV uint32_t ring_parity(uint32_t use, uint32_t n) { return (use / n) & 1u; }

}  // namespace dm
