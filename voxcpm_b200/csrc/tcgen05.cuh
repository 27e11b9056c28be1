// Fifth-generation tensor core (tcgen05) and tensor memory (TMEM) wrappers
// for sm_100a, as inline PTX. Used by the tensor-core product kernel
// (products_tc.cu).
//
// TMEM is 128 lanes x 512 columns of 32 bits per SM. An address is
// (lane << 16) | column. A warp reaches only the 32 lanes of its quarter,
// 32 * (warp id % 4).
#pragma once

#include <cuda.h>

#include <cstdint>

#include "vx_common.cuh"

namespace vx {

/// Allocates `columns` TMEM columns (a power of two, 32..512) for this CTA
/// and writes the base address to `*dst` (shared memory). One whole warp.
__device__ inline void TmemAlloc(std::uint32_t* dst, std::uint32_t columns) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          SmemAddr(dst)),
      "r"(columns)
      : "memory");
}

/// Lets other CTAs on this SM allocate once this one has. One whole warp.
__device__ inline void TmemRelinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}

/// Frees an allocation; the warp that allocated, before the CTA exits.
__device__ inline void TmemDealloc(std::uint32_t base, std::uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   base),
               "r"(columns)
               : "memory");
}

/// Orders this thread's earlier tcgen05 operations before a following
/// thread synchronization (barrier or mbarrier arrive).
__device__ inline void TcFenceBefore() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

/// Orders tcgen05 operations after a preceding thread synchronization.
__device__ inline void TcFenceAfter() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

/// Stores 16 registers of each lane into 16 consecutive columns of the
/// lane's TMEM row (shape 32x32b) and waits until the stores are done.
__device__ inline void TmemStore16(std::uint32_t address,
                                   const std::uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, "
      "%7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n"
      "tcgen05.wait::st.sync.aligned;" ::"r"(address),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]),
      "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]),
      "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

/// Loads 16, 24 or 32 consecutive columns of each lane's TMEM row (shape
/// 32x32b) and waits for them; the registers are valid on return.
template <int kColumns>
__device__ inline void TmemLoad(std::uint32_t address,
                                std::uint32_t (&v)[kColumns]) {
  static_assert(kColumns == 16 || kColumns == 24 || kColumns == 32,
                "16, 24 or 32 columns");
  if constexpr (kColumns == 16) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, "
        "%7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]),
          "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]),
          "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15])
        : "r"(address)
        : "memory");
  } else if constexpr (kColumns == 24) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, "
        "%7, %8, %9, %10, %11, %12, %13, %14, %15}, [%24];\n"
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16, %17, %18, %19, %20, %21, "
        "%22, %23}, [%25];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]),
          "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]),
          "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
          "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23])
        : "r"(address), "r"(address + 16)
        : "memory");
  } else {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, "
        "%7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, "
        "%21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]),
          "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]),
          "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
          "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
          "=r"(v[30]), "=r"(v[31])
        : "r"(address)
        : "memory");
  }
}

/// Instruction descriptor of a dense kind::f16 MMA: bf16 A and B, both
/// K-major, fp32 accumulator, M x N.
__host__ __device__ constexpr std::uint32_t MmaBf16Descriptor(int m, int n) {
  return (1u << 4)      // accumulator format: fp32
         | (1u << 7)    // A: bf16
         | (1u << 10)   // B: bf16
         | (static_cast<std::uint32_t>(n >> 3) << 17) |
         (static_cast<std::uint32_t>(m >> 4) << 24);
}

/// Shared-memory matrix descriptor, no swizzle, K-major: 8-row x 16-byte
/// core matrices; `k_stride` bytes between the two core matrices of one
/// 16-element K step, `row_stride` bytes between 8-row groups.
__device__ inline std::uint64_t SmemDescriptorNoSwizzle(const void* start,
                                                        std::uint32_t k_stride,
                                                        std::uint32_t row_stride) {
  return static_cast<std::uint64_t>((SmemAddr(start) >> 4) & 0x3FFFu) |
         (static_cast<std::uint64_t>((k_stride >> 4) & 0x3FFFu) << 16) |
         (static_cast<std::uint64_t>((row_stride >> 4) & 0x3FFFu) << 32) |
         (1ull << 46);  // descriptor version for sm_100
}

/// Shared-memory matrix descriptor, 128-byte swizzle, K-major: rows of 128
/// bytes (64 bf16 values) in 8-row, 1024-byte swizzle atoms, as the TMA's
/// CU_TENSOR_MAP_SWIZZLE_128B writes them. `start` is a 1024-byte aligned
/// atom base plus the K offset within the row in bytes (32 per 16-element
/// K step); `group_stride` bytes between 8-row groups. The leading-dimension
/// offset is unused for this layout (one MMA's K stays inside a row).
__device__ inline std::uint64_t SmemDescriptorSw128(const void* start,
                                                    std::uint32_t group_stride) {
  return static_cast<std::uint64_t>((SmemAddr(start) >> 4) & 0x3FFFu) |
         (1ull << 16) |
         (static_cast<std::uint64_t>((group_stride >> 4) & 0x3FFFu) << 32) |
         (1ull << 46) |  // descriptor version for sm_100
         (2ull << 61);   // layout: 128-byte swizzle
}

/// D (TMEM) = A (TMEM) x B (shared memory) [+ D when `accumulate`]. One
/// thread issues it; it completes asynchronously (see MmaCommit).
__device__ inline void MmaBf16TmemA(std::uint32_t d, std::uint32_t a,
                                    std::uint64_t b_descriptor,
                                    std::uint32_t instruction,
                                    std::uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
      "}\n" ::"r"(d),
      "r"(a), "l"(b_descriptor), "r"(instruction), "r"(accumulate)
      : "memory");
}

/// Tiled 2-D TMA load (no multicast) of the box at element coordinates
/// (c0, c1) of `map` into shared memory, completing on `bar`. c0 times the
/// element size is a multiple of 16 bytes.
__device__ inline void TmaLoad2D(void* dst, const CUtensorMap* map, int c0,
                                 int c1, std::uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(SmemAddr(dst)),
      "l"(reinterpret_cast<std::uint64_t>(map)), "r"(c0), "r"(c1),
      "r"(SmemAddr(bar))
      : "memory");
}

/// Tiled 3-D TMA load (no multicast), as TmaLoad2D.
__device__ inline void TmaLoad3D(void* dst, const CUtensorMap* map, int c0,
                                 int c1, int c2, std::uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(SmemAddr(dst)),
      "l"(reinterpret_cast<std::uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
      "r"(SmemAddr(bar))
      : "memory");
}

/// Arrives once on `bar` when every tcgen05.mma this thread issued before
/// has completed.
__device__ inline void MmaCommit(std::uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(SmemAddr(bar))
      : "memory");
}

}  // namespace vx
