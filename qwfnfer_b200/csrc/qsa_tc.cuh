// qsa_tc.cuh -- 5th-generation tensor core (tcgen05) helpers: TMEM allocation, shared-memory
// matrix descriptors for 128-byte-swizzled K-major f16 operands, the kind::f16 MMA, commit and
// TMEM loads.
#pragma once
#include "qsa_common.cuh"

namespace qsa {

// Byte offset of element (r, k) of a K-major, 128-byte-swizzled f16 tile of `rows` rows: atoms of
// 64 columns, each rows x 128 B in groups of 8 rows (1024 B); inside a group, the 16-byte chunk c
// of row r sits at chunk position c ^ (r % 8).  The tile base must be 1024-byte aligned.
__device__ __forceinline__ uint32_t sw128_off(int rows, int r, int k) {
    const int atom = k >> 6, c = (k >> 3) & 7;
    return (uint32_t) (atom * rows * 128 + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4) + ((k & 7) << 1));
}

// Shared-memory matrix descriptor: start address >> 4, leading byte offset 1 (unused for swizzled
// K-major), stride byte offset 1024 >> 4 between 8-row groups, version 1, layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
    return (uint64_t) ((smem_addr >> 4) & 0x3FFFu) | ((uint64_t) 1 << 16) | ((uint64_t) 64 << 32) |
           ((uint64_t) 1 << 46) | ((uint64_t) 2 << 61);
}

// Instruction descriptor, kind::f16: D f32, A and B f16, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t) (N >> 3) << 17) | ((uint32_t) (M >> 4) << 24);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// One warp: allocate `ncols` TMEM columns (a power of two >= 32); the address goes to *slot.
__device__ __forceinline__ void tmem_alloc_warp(uint32_t * slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_warp(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}

// D (TMEM) = A x B (+ D when accumulate), issued by one thread.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, bool accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
                 :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(0u) : "memory");
}
// The mbarrier receives one arrive when every MMA issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

// 32 consecutive f32 columns of this thread's TMEM lane (warp w reads lanes 32 (w % 4) ..).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                   "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
                   "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
                   "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace qsa
