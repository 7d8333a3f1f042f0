// umma.cuh - 5th-generation tensor core (tcgen05) and TMA tensor-copy helpers, sm_100a.
//
// Each MMA is issued for one CTA (cta_group::1) on operands in that CTA's own shared memory,
// and every TMA copy fills only its own CTA's shared memory (no multicast). (Split-K GEMMs
// group CTAs in clusters only to add their finished partial tiles through distributed
// shared memory; see voc_conv.cuh.) Operands are K-major tiles that a
// TMA tensor copy wrote into shared memory with the 64-byte swizzle; accumulators
// live in tensor memory (TMEM) and come back to registers with tcgen05.ld.
//
// Bit layouts (PTX ISA, "Matrix Descriptors" and "Instruction descriptor" of the
// tcgen05 family; the same fields as cute::UMMA::SmemDescriptor / InstrDescriptor):
//   shared-memory descriptor (64 bits)
//     [0,14)  start address >> 4        [16,30) leading byte offset >> 4
//     [32,46) stride byte offset >> 4   [46,48) version, 1 on sm_100
//     [49,52) base offset               [52]    LBO mode
//     [61,64) swizzle: 0 none, 1 128B/32B-atom, 2 128B, 4 64B, 6 32B
//   instruction descriptor, kind::tf32 / kind::f16 (32 bits)
//     [4,6) D format (1 = F32)   [7,10) A format   [10,13) B format (2 = TF32)
//     [15] A MN-major   [16] B MN-major   [17,23) N >> 3   [24,29) M >> 4
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "bulk_copy.cuh"

namespace lai {
namespace umma {

using bulk::smem_addr;

// ---- TMEM allocation: executed by one whole warp; the base address lands in *slot ----
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// Order tcgen05 operations against thread synchronisation (barriers, mbarrier waits).
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// K-major operand tile written by TMA with CU_TENSOR_MAP_SWIZZLE_64B: rows of 64 bytes,
// 8-row groups 512 bytes apart. The tile base must be 512-byte aligned; a start
// address advanced by 32 bytes within the row selects the second 8-element K step.
__device__ __forceinline__ uint64_t desc_kmajor_sw64(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4)  // start address
           | (uint64_t)1 << 16                   // leading byte offset (unused when swizzled)
           | (uint64_t)(512u >> 4) << 32         // stride byte offset: 8 rows x 64 B
           | (uint64_t)1 << 46                   // descriptor version
           | (uint64_t)4 << 61;                  // 64-byte swizzle
}

// kind::tf32, F32 accumulate, both operands K-major, M x N tile.
template <int M, int N>
__host__ __device__ constexpr uint32_t idesc_tf32() {
    static_assert(M == 128, "cta_group::1 tiles here are 128 rows");
    static_assert(N % 16 == 0 && N >= 16 && N <= 256, "M = 128 needs N % 16 == 0, 16..256");
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// D[tmem] = A * B^T (+ D when accumulate != 0); issued by one thread.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// One arrival on *bar once every MMA this thread issued before has completed.
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_addr(bar))
        : "memory");
}

// Lane i of the warp receives TMEM lane (taddr.lane + i), 32 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
        "[%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}
// Lane i of the warp receives TMEM lane (taddr.lane + i), 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- TMA tensor copies global -> shared (tiled mode, no multicast) ----
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y,
                                            int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int x, int y,
                                            int z, int w, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w),
        "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// FP32 -> nearest TF32 value (low 13 mantissa bits zero), ties away from zero, on the
// integer pipe (the conversion instruction runs on the narrow XU pipe, which limited the
// epilogues that split every output): IEEE bit patterns order magnitudes, so adding half a
// TF32 unit (bit 12) to the bits and clearing the low 13 rounds the magnitude to nearest
// with ties up; a carry out of the mantissa steps into the next binade, and past FLT_MAX
// to inf, as the rounding does. NaN is returned unchanged (the add could carry a NaN with
// a full mantissa into the sign bit).
__device__ __forceinline__ float tf32_round(float x) {
    const uint32_t u = __float_as_uint(x);
    const uint32_t r = (u + 0x1000u) & 0xffffe000u;
    return (u & 0x7fffffffu) > 0x7f800000u ? x : __uint_as_float(r);
}

}  // namespace umma
}  // namespace lai
