// lt_umma.cuh — 5th-generation tensor-core (tcgen05) helpers for sm_100a:
// shared-memory operand layout and descriptors, the f16 MMA with f32
// accumulation in tensor memory (TMEM), TMEM allocation and loads.
//
// Operand tiles are K-major with the 128-byte swizzle: a "swizzle atom" is
// 8 rows of 64 f16 (128 bytes each) = 1024 bytes at a 1024-byte boundary;
// the 16-byte chunk c of row r sits at chunk position c ^ (r % 8).  Rows
// beyond 8 stack at 1024-byte steps (the descriptor's stride offset), and
// K beyond 64 lives in further atoms.  One MMA consumes K = 16 (32 bytes of
// each row): step s of an atom starts 32*s bytes into it.
#pragma once

#include "lt_common.cuh"

namespace lt {

// Byte offset of element (r, k), k < 64, inside a K-major 128B-swizzled tile.
LT_DEVINL uint32_t sw128_offset(uint32_t r, uint32_t k) {
    return r * 128 + ((((k >> 3) ^ r) & 7) << 4) + ((k & 7) << 1);
}

// Shared-memory matrix descriptor for a K-major 128B-swizzled operand that
// starts at shared address saddr (the atom base must be 1024-byte aligned;
// saddr may add a 32*s step inside the atom): start >> 4 in bits [0,14),
// leading offset 1 (unused with swizzling), stride offset 1024 >> 4 in bits
// [32,46), version 1 in bits [46,48), layout "128B swizzle" (2) in [61,64).
LT_DEVINL uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor for kind::f16: A, B f16 (format 0), D f32 (format 1
// in bits [4,6)), both K-major, N >> 3 in bits [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t umma_idesc_f16_f32(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A * B^T, issued by one thread.
LT_DEVINL void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Arrive on an mbarrier once all MMAs this thread issued so far complete.
LT_DEVINL void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// TMEM allocation (whole warp): writes the base address to shared memory.
LT_DEVINL void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
LT_DEVINL void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
LT_DEVINL void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
LT_DEVINL void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LT_DEVINL void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Generic-proxy shared-memory writes before the tensor core reads them.
LT_DEVINL void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive 32-bit TMEM columns of this thread's lane: warp w of a
// warpgroup reads lanes [32 (w % 4), +32); taddr carries lane << 16 | column.
LT_DEVINL void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}
LT_DEVINL void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace lt
