// Shared device helpers of the sm_100a hot path: bf16 rounding, fp16 decode,
// mbarrier / bulk-copy (TMA) / cluster PTX wrappers, bounded waits and the
// library's status plumbing.
//
// Rounding semantics follow the reference's device math
// (kernels/device_math.hpp:12-24, kernels/generator_kernels.hip:18-28):
// float -> bf16 rounds to nearest even, a NaN stays a quiet NaN.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstddef>
#include <cstdint>

#include "vx_status.h"

namespace vx {

using Bf16 = std::uint16_t;

// Device error bits, or-ed into g_vx_device_error by a kernel whose bounded
// wait expired. The host reads and clears them with vx_device_error().
enum DeviceError : unsigned {
  kErrWeightWait = 1u << 0,
  kErrActivationWait = 1u << 1,
  kErrDrainWait = 1u << 2,
  kErrBarrierWait = 1u << 3,
  kErrPublishWait = 1u << 4,
  kErrPeerWait = 1u << 5,
};

/// The device word the library's kernels or their error bits into; defined
/// in products.cu (DeviceErrorWord gives its address for other units).
unsigned* DeviceErrorWord();
/// Reads and clears the device error word (synchronizes the device).
int ReadDeviceError(unsigned* bits);

// ---------------------------------------------------------------- bf16 / fp16

__host__ __device__ inline float Bf16ToFloat(Bf16 bits) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(static_cast<std::uint32_t>(bits) << 16U);
#else
  std::uint32_t v = static_cast<std::uint32_t>(bits) << 16U;
  float f;
  __builtin_memcpy(&f, &v, 4);
  return f;
#endif
}

/// float -> bf16 bits, round to nearest even, NaN kept quiet.
__device__ inline Bf16 FloatToBf16(float value) {
  const std::uint32_t bits = __float_as_uint(value);
  if ((bits & 0x7F800000U) == 0x7F800000U && (bits & 0x007FFFFFU) != 0)
    return static_cast<Bf16>((bits >> 16U) | 0x40U);
  const std::uint32_t rounding = 0x7FFFU + ((bits >> 16U) & 1U);
  return static_cast<Bf16>((bits + rounding) >> 16U);
}

__device__ inline float HalfBitsToFloat(std::uint16_t bits) {
  return __half2float(__ushort_as_half(bits));
}

// ---------------------------------------------------------------- PTX wrappers

__device__ inline std::uint32_t SmemAddr(const void* p) {
  return static_cast<std::uint32_t>(__cvta_generic_to_shared(p));
}

__device__ inline void MbarInit(std::uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(SmemAddr(bar)),
               "r"(count)
               : "memory");
}

__device__ inline void FenceMbarInit() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ inline void FenceProxyAsync() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

/// Arrives once on `bar` and raises its expected transaction bytes.
__device__ inline void MbarArriveExpectTx(std::uint64_t* bar, unsigned bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          SmemAddr(bar)),
      "r"(bytes)
      : "memory");
}

/// Arrives once on `bar` (no transaction bytes).
__device__ inline void MbarArrive(std::uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(SmemAddr(bar))
               : "memory");
}

/// Tests phase `parity` of `bar`; a thread whose phase is not complete is
/// suspended by the hardware until it completes or `suspend_ns` pass, so a
/// waiting warp takes no issue slots from the warps that compute.
__device__ inline bool MbarTryWait(std::uint64_t* bar, unsigned parity,
                                   std::uint32_t suspend_ns = 10000000u) {
  std::uint32_t done;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(done)
      : "r"(SmemAddr(bar)), "r"(parity), "r"(suspend_ns)
      : "memory");
  return done != 0;
}

__device__ inline std::uint64_t GlobalTimerNs() {
  std::uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

/// Waits for phase `parity` of `bar` for at most `limit_ns`; on expiry
/// ors `error` into `*error_word` and returns false.
__device__ inline bool MbarWaitBounded(std::uint64_t* bar, unsigned parity,
                                       unsigned* error_word, unsigned error,
                                       std::uint64_t limit_ns = 2000000000ull) {
  if (MbarTryWait(bar, parity))
    return true;
  const std::uint64_t start = GlobalTimerNs();
  while (true) {
    if (MbarTryWait(bar, parity))
      return true;
    if (GlobalTimerNs() - start > limit_ns) {
      atomicOr(error_word, error);
      return false;
    }
  }
}

/// Bulk copy (TMA, 1-D) of `bytes` from global memory into this CTA's
/// shared memory, completing on `bar`. Both addresses 16-byte aligned and
/// `bytes` a multiple of 16.
__device__ inline void BulkLoad(void* smem_dst, const void* gmem_src,
                                unsigned bytes, std::uint64_t* bar,
                                std::uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::"
      "cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(SmemAddr(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(SmemAddr(bar)), "l"(policy)
      : "memory");
}

/// Asks L2 to fetch `bytes` of global memory (no copy to the SM; nothing
/// waits for it). 16-byte aligned address, `bytes` a multiple of 16.
__device__ inline void PrefetchL2Bulk(const void* gmem, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem),
               "r"(bytes)
               : "memory");
}

__device__ inline std::uint64_t PolicyEvictFirst() {
  std::uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;"
               : "=l"(policy));
  return policy;
}

__device__ inline std::uint64_t PolicyEvictLast() {
  std::uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;"
               : "=l"(policy));
  return policy;
}

// Programmatic dependent launch: a kernel launched with the
// programmatic-stream-serialization attribute may start before its
// predecessor ends; it must wait before touching the predecessor's outputs.
__device__ inline void GridDependencyWait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ inline void GridLaunchDependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Thread-block cluster helpers.
__device__ inline unsigned ClusterRank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ inline void ClusterSync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
/// Address of the same shared-memory variable in cluster CTA `rank`.
__device__ inline std::uint32_t MapShared(const void* p, unsigned rank) {
  std::uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(out)
               : "r"(SmemAddr(p)), "r"(rank));
  return out;
}
__device__ inline float4 LoadSharedCluster4(std::uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Packed fp32 pairs (sm_100a): two lanes of work per instruction.
__device__ inline float2 Add2(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 a, b, d;\nmov.b64 a, {%2,%3};\nmov.b64 b, {%4,%5};\n"
      "add.rn.f32x2 d, a, b;\nmov.b64 {%0,%1}, d;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
/// a * b + c per lane, fused, round to nearest.
__device__ inline float2 Fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n.reg .b64 a, b, c, d;\nmov.b64 a, {%2,%3};\nmov.b64 b, {%4,%5};\n"
      "mov.b64 c, {%6,%7};\nfma.rn.f32x2 d, a, b, c;\nmov.b64 {%0,%1}, d;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ inline std::uint32_t Prmt(std::uint32_t a, std::uint32_t b,
                                     std::uint32_t selector) {
  std::uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(selector));
  return d;
}

}  // namespace vx
