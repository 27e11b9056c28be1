// Device machinery shared by the persistent kernels (persistent_dit.cu,
// persistent_lm.cu): sixteen consumer warps with named-barrier syncs, bounded
// waits that give up when any CTA aborted, monotone counters polled with
// acquire loads, a publisher warp that does the release-adds, and the
// in-CTA reduction of split warps' accumulators.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "vx_common.cuh"

namespace vx {
namespace {

constexpr int kConsumerWarps = 16;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kRedFloats = 32 * 12;  // one warp's accumulators, 3 column tiles
constexpr int kPubSlots = 8;
constexpr std::uint64_t kWaitLimitNs = 2000000000ull;
constexpr std::uint32_t kSuspendNs = 100000u;
constexpr int kSyncAbort = 0;  // sync word 0: any CTA aborted

/// One request to the publisher warp: add `value` to `counter`.
struct PubEntry {
  unsigned* counter;
  unsigned value;
  unsigned pad;
};

// ---------------------------------------------------------------- helpers

__device__ inline void ConsumerSync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}

/// Consumer barrier that also ORs a predicate over the consumer threads.
__device__ inline bool ConsumerSyncOr(bool value) {
  unsigned result;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\n"
      "bar.red.or.pred p, 1, %2, q;\nselp.u32 %0, 1, 0, p;\n}"
      : "=r"(result)
      : "r"(static_cast<unsigned>(value)), "n"(kConsumers)
      : "memory");
  return result != 0;
}

/// Arrives on the mbarrier at shared::cluster address `addr` (a peer's),
/// releasing this thread's prior writes at cluster scope.
__device__ inline void MbarArriveCluster(std::uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr)
               : "memory");
}

/// try_wait with acquire at cluster scope (arrivals from the peer CTA).
__device__ inline bool MbarTryWaitCluster(std::uint64_t* bar, unsigned parity,
                                          std::uint32_t suspend_ns) {
  std::uint32_t done;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(SmemAddr(bar)), "r"(parity), "r"(suspend_ns)
      : "memory");
  return done != 0;
}

__device__ inline void StoreSharedCluster(std::uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ inline unsigned LoadAcquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];"
               : "=r"(v)
               : "l"(p)
               : "memory");
  return v;
}

__device__ inline unsigned LoadRelaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];"
               : "=r"(v)
               : "l"(p)
               : "memory");
  return v;
}

__device__ inline void RedRelease(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v)
               : "memory");
}

__device__ inline float WarpAllSum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

/// Two floats -> packed bf16 pair (lo in the low half), round to nearest
/// even (the hardware conversion; equal to the software rounding for every
/// non-NaN input).
__device__ inline unsigned PackBf16x2(float lo, float hi) {
  unsigned d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

__device__ inline uint2 PackBf16x4(float a, float b, float c, float d) {
  return make_uint2(PackBf16x2(a, b), PackBf16x2(c, d));
}

__device__ inline Bf16 ToBf16(float v) {
  return static_cast<Bf16>(PackBf16x2(v, 0.0f) & 0xFFFFu);
}

__device__ inline float RoundBf16(float v) {
  return Bf16ToFloat(ToBf16(v));
}

/// Abort state shared by the CTA's warps and, through `sync`, all CTAs.
struct Control {
  unsigned* sync;
  unsigned* error_word;
  volatile int* aborted;  // shared
};

__device__ inline void Abort(const Control& c, unsigned error) {
  if (error != 0)
    atomicOr(c.error_word, error);
  atomicExch(c.sync + kSyncAbort, 1u);
  *c.aborted = 1;
}

/// Waits for phase `parity` of `bar`, giving up when any CTA aborted or
/// after the time limit (which aborts the launch).
__device__ bool WaitSlot(std::uint64_t* bar, unsigned parity,
                         const Control& c, unsigned error) {
  if (MbarTryWait(bar, parity, kSuspendNs))
    return true;
  const std::uint64_t start = GlobalTimerNs();
  while (true) {
    if (MbarTryWait(bar, parity, kSuspendNs))
      return true;
    if (*c.aborted != 0 || LoadRelaxed(c.sync + kSyncAbort) != 0) {
      *c.aborted = 1;
      return false;
    }
    if (GlobalTimerNs() - start > kWaitLimitNs) {
      Abort(c, error);
      return false;
    }
  }
}

/// Consumer-wide wait for phase `parity` of the local mbarrier `bar` that
/// the peer CTA arrives on. Returns false, uniformly, once aborted.
__device__ bool WaitPeer(std::uint64_t* bar, unsigned parity, const Control& c) {
  bool aborted = false;
  if (threadIdx.x == 0) {
    if (*c.aborted == 0 && !MbarTryWaitCluster(bar, parity, kSuspendNs)) {
      const std::uint64_t start = GlobalTimerNs();
      while (!MbarTryWaitCluster(bar, parity, kSuspendNs)) {
        if (*c.aborted != 0 || LoadRelaxed(c.sync + kSyncAbort) != 0) {
          *c.aborted = 1;
          break;
        }
        if (GlobalTimerNs() - start > kWaitLimitNs) {
          Abort(c, kErrPeerWait);
          break;
        }
      }
    }
    aborted = *c.aborted != 0;
  }
  return !ConsumerSyncOr(aborted);
}

/// Consumer-wide wait until `*counter >= target` (thread 0 polls with
/// acquire loads). Returns false, uniformly, once the launch aborted.
__device__ bool WaitCount(const Control& c, const unsigned* counter,
                          unsigned target) {
  bool aborted = false;
  if (threadIdx.x == 0) {
    if (*c.aborted == 0 && LoadAcquire(counter) < target) {
      // Acquire polls; the abort flag and the time limit every 32 polls.
      const std::uint64_t start = GlobalTimerNs();
      unsigned spins = 0;
      while (LoadAcquire(counter) < target) {
        if ((++spins & 31u) == 0) {
          if (LoadRelaxed(c.sync + kSyncAbort) != 0) {
            *c.aborted = 1;
            break;
          }
          if (GlobalTimerNs() - start > kWaitLimitNs) {
            Abort(c, kErrBarrierWait);
            break;
          }
        }
      }
    }
    aborted = *c.aborted != 0;
  }
  return !ConsumerSyncOr(aborted);
}

/// (output feature within the 16-row group, activation row) of reduced
/// accumulator `t` for `ntiles` column tiles.
__device__ inline void Decode(int t, int ntiles, int& feature, int& row) {
  const int per_lane = ntiles * 4;
  const int lane = t / per_lane;
  const int jq = t % per_lane;
  const int q = jq & 3;
  feature = (lane >> 2) + 8 * (q >> 1);
  row = 8 * (jq >> 2) + 2 * (lane & 3) + (q & 1);
}

/// Sum over warps [first, first + count) of the reduction buffer, in order.
__device__ inline float Reduce(const float* red, int t, int stride,
                              int first = 0, int count = kConsumerWarps) {
  float s = red[first * stride + t];
  for (int w = 1; w < count; ++w)
    s += red[(first + w) * stride + t];
  return s;
}

// ---------------------------------------------------------------- publisher

/// Lane 0 of the publisher warp: for each request of the consumers, in
/// order, adds to the counter with release semantics (device scope), which
/// makes the CTA's writes before the request visible to whoever acquires the
/// counter. The consumers never wait for the release.
__device__ void Publish(PubEntry* entries, std::uint64_t* pub_full,
                        std::uint64_t* pub_empty, const Control& c) {
  for (unsigned k = 0;; ++k) {
    const unsigned slot = k % kPubSlots;
    if (!WaitSlot(&pub_full[slot], (k / kPubSlots) & 1u, c, kErrPublishWait))
      return;
    const volatile PubEntry* e = entries + slot;
    unsigned* counter = e->counter;
    const unsigned value = e->value;
    if (counter == nullptr)
      return;
    // The consumers' writes precede their barrier and the queue entry's
    // release-arrive; this release-add is ordered after them, so whoever
    // acquires the counter sees them.
    RedRelease(counter, value);
    MbarArrive(&pub_empty[slot]);
  }
}

/// Brings `bytes` of global memory into L2 ahead of use (one 128-byte line
/// per consumer thread, no register or wait).
__device__ inline void PrefetchL2(const void* p, int bytes, int tid) {
  const char* base = static_cast<const char*>(p);
  for (int at = tid * 128; at < bytes; at += kConsumers * 128)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(base + at));
}

}  // namespace

/// The most CTAs a persistent kernel launches (0: no cap; below a kernel's
/// minimum the minimum). A tuning and profiling knob: a profiler may hold
/// back resources, so fewer CTAs than the occupancy query gives co-reside.
void SetPersistentMaxCtas(int ctas);
int PersistentMaxCtas();
/// Whether the persistent kernels launch with the cooperative attribute
/// (default on). Off, their co-residency rests on the grid fitting an idle
/// GPU (one CTA per SM); if it does not, the bounded waits end the launch
/// with the abort word set. For profilers that cannot replay cooperative
/// cluster launches.
void SetPersistentCooperative(bool enabled);
bool PersistentCooperative();

}  // namespace vx
