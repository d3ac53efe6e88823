// Blackwell 5th-generation tensor core primitives (tcgen05) as inline PTX:
// tensor-memory allocation, the f16 MMA with shared-memory operand
// descriptors, completion through mbarriers, and accumulator reads.
//
// Shared-memory operands are K-major with the 128-byte swizzle: a tile row
// is 64 f16 (128 bytes), rows are packed, eight rows make a 1,024-byte
// swizzle atom, and 16-byte chunk c of row r sits at chunk c ^ (r mod 8).
// Descriptor fields (PTX ISA, tcgen05 shared memory descriptor; the same
// layout as CUTLASS's cute::UMMA::SmemDescriptor): start address >> 4 in
// bits 0-13, leading byte offset >> 4 in 16-29, stride byte offset >> 4 in
// 32-45, version 1 in 46-47, swizzle mode in 61-63 (2 = 128-byte).
#pragma once

#include <cstdint>

#include "tma.cuh"

namespace cb {

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// K-major, 128-byte swizzle, atoms of 8 rows 1,024 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_byte_addr) {
    return static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3FFFu) | (1ull << 16) |   // LBO (unused for swizzled K-major)
           (static_cast<uint64_t>(1024u >> 4) << 32) |                                // SBO: 8-row atoms
           (1ull << 46) |                                                               // version (Blackwell)
           (2ull << 61);                                                                // 128-byte swizzle
}

// Instruction descriptor of kind::f16 with f16 A and B, f32 accumulate,
// both operands K-major, an M × N tile.
__host__ __device__ constexpr uint32_t umma_idesc_f16(uint32_t M, uint32_t N) {
    return (1u << 4)                  // D format: f32
           | (0u << 7) | (0u << 10)   // A, B format: f16
           | (0u << 15) | (0u << 16)  // A, B K-major
           | ((N >> 3) << 17) | ((M >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t columns) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
                 "r"(columns)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t columns) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A·Bᵀ, issued by one thread.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                         uint32_t accumulate) {
    const uint32_t mask0 = 0, mask1 = 0, mask2 = 0, mask3 = 0;
    asm volatile(
        "{\n\t"
        ".reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t"
        "}\n" ::"r"(tmem_d),
        "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(mask0), "r"(mask1), "r"(mask2), "r"(mask3)
        : "memory");
}

// Arrives on `bar` once every tcgen05 operation this thread issued before
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// 32 consecutive f32 columns of this thread's TMEM lane (a warp reads its
// own 32 lanes: lanes 32·(warp mod 4) ...). The wait for the load is in the
// same asm statement, so the registers are never read before they land.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace cb
