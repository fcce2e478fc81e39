// tcgen05 (5th-generation tensor core) building blocks shared by the kernels that
// run matrix products on sm_100a: shared-memory operand descriptors for K-major
// tiles in the 128-byte swizzled layout, the instruction descriptors of kind::tf32
// and kind::f16 with an FP32 accumulator, MMA issue and commit, and tensor-memory
// (TMEM) allocation and loads.
//
// Operand tiles: rows of 128 bytes (32 fp32 or 64 fp16 elements, one K block), 8-row groups
// of 1024 bytes; inside a group the 16-byte chunk c of row r sits at chunk
// position c ^ (r % 8) (the layout the TMA engine writes for SWIZZLE_128B). A tile
// starts on a 1024-byte boundary.
#pragma once
#include <cstdint>

#include "common.cuh"

namespace mpb {

// K-major, 128-byte swizzle UMMA shared-memory descriptor: start address >> 4,
// LBO (ignored for swizzled K-major) 1, SBO = 1024 B between 8-row groups,
// version 1 (sm_100), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc(const void* tile) {
    const uint64_t addr = smem_u32(tile);
    uint64_t d = (addr >> 4) & 0x3FFFull;
    d |= uint64_t(1) << 16;
    d |= uint64_t(1024 >> 4) << 32;
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

// Byte offset of the 16-byte chunk `chunk` (0..7) of row `row` in a swizzled tile.
__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk) {
    return uint32_t(row) * 128u + uint32_t((chunk ^ (row & 7)) << 4);
}

// Instruction descriptor: D f32 (1 @ bit 4), A/B tf32 (2 @ bits 7, 10), both
// K-major, N >> 3 @ bit 17, M >> 4 @ bit 24.
template <int M, int N>
__host__ __device__ constexpr uint32_t umma_idesc_tf32() {
    return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// Instruction descriptor of kind::f16 with FP16 A and B (format 0 @ bits 7, 10)
// and an FP32 accumulator (1 @ bit 4), both K-major.
template <int M, int N>
__host__ __device__ constexpr uint32_t umma_idesc_f16() {
    return (1u << 4) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// D (TMEM) (+)= A . B^T, one K step of 16 fp16 elements (32 bytes of each operand
// row); `accumulate` 0 overwrites.
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// D (TMEM) (+)= A . B^T, one K step of 8 tf32 elements; `accumulate` 0 overwrites.
__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// Arrive on `bar` once every MMA this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// Whole-warp TMEM allocation of `cols` columns (power of two >= 32); the base
// address is written to shared memory at `holder`.
__device__ __forceinline__ void tmem_alloc(uint32_t* holder, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t tmem, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(cols) : "memory");
}

// 32 consecutive columns of this warp's 32 TMEM lanes: thread = lane, r = columns.
// Warp-collective (.sync.aligned): all 32 lanes must execute it convergently, never
// under a lane-dependent condition.
__device__ __forceinline__ void tmem_load32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace mpb
