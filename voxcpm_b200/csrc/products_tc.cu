// The tensor-core (tcgen05) skinny product for Q8_0 tiles on sm_100a.
//
// y[rows][out] (+)= x[rows][in] * W[out][in]^T for 9..32 activation rows,
// with the reference's per-block arithmetic (kernels/wmma_products.hip:
// 139-296): every 32-column block of a weight row is summed in fp32 over
// exact bf16 values of q, then added into the row's accumulator as
// fmaf(scale, block sum, acc).
//
// Why tensor memory: at 22 rows the legacy mma.sync path needs six
// m16n8k16 MMAs per 16 x 32 weight tile, and on sm_100 those alone take
// about 24 SM cycles per tile, which caps the product near the HBM rate.
// Here one thread issues 128 x N x 16 tcgen05 MMAs, so the SM's issue slots
// go to the exact dequantisation only.
//
// One CTA per SM owns 128 weight rows (8 tile groups) over a slice of at
// most 24 blocks of the reduction; the CTAs of a thread-block cluster take
// consecutive slices of the same rows and add up in cluster-rank order
// through distributed shared memory (the reference's ordered split sum,
// kernels/wmma_products.hip:249-295). Per CTA, a three-stage pipeline over
// ten TMEM slots (A: 16 columns, block sums: 32 columns each):
// - a producer warp brings the whole weight slice in with one 1-D TMA bulk
//   copy per tile group and 8-block part, from eight lanes at once (L2
//   evict-first), and x, after the programmatic-launch wait, with one 3-D
//   tensor-map copy per part that lands as the MMA's B operand in the
//   no-swizzle K-major layout (8-row x 16-byte core matrices; rows past the
//   activation rows are zero-filled by the copy);
// - three conversion teams of four warps (one warp per TMEM lane quarter)
//   take every third block: each thread owns one weight row, turns its 32
//   biased int8 values into bf16 exactly and stores them into the block's
//   TMEM A slot (tcgen05.st); the team meets at a named barrier and one lane
//   issues D[slot] = A[slot] x x_block (two K=16 steps, fresh accumulator),
//   committing to the slot's mbarrier;
// - two read teams take alternate blocks: they read the block sums back
//   (tcgen05.ld), free the slot and add the sums into their rows'
//   accumulators with the rows' fp16 scales.
// A TMA request or a tcgen05.mma costs its issuing thread 30-40 ns whatever
// its size: hence few, large copies and one MMA issuer per team.
#include "products.cuh"
#include "product_math.cuh"
#include "tcgen05.cuh"
#include "tensor_map.cuh"
#include "vx_common.cuh"

#include <cuda.h>

#include <algorithm>
#include <mutex>

namespace vx {

namespace {

constexpr int kTcGroups = 8;                  // 16-row tile groups per CTA
constexpr int kTcRows = 16 * kTcGroups;       // = the MMA's M (TMEM lanes)
constexpr int kTcPartBlocks = 8;              // blocks per weight / x copy
constexpr int kTcParts = kTensorCoreMaxBlocks / kTcPartBlocks;
constexpr int kTcSlots = 10;                  // TMEM A / accumulator slots
constexpr int kTcConvertTeams = 3;            // teams of four warps: int8 -> TMEM
constexpr int kTcReadTeams = 2;               // teams of four warps: sums back
constexpr int kTcConvertWarps = 4 * kTcConvertTeams;
constexpr int kTcWorkerWarps = kTcConvertWarps + 4 * kTcReadTeams;
constexpr int kTcProducerWarp = kTcWorkerWarps;
constexpr int kTcThreads = 32 * (kTcWorkerWarps + 1);
constexpr int kTcXRows = 32;                  // B rows staged (M <= 32)
constexpr int kTcXChunkBytes = kTcXRows * 16; // 8 K-values of all 32 rows
constexpr int kTcXPartBytes = kTcPartBlocks * 4 * kTcXChunkBytes;
constexpr int kTcXBytes = kTcParts * kTcXPartBytes;
constexpr int kTcWeightBytes = kTcGroups * kTensorCoreMaxBlocks * kQ8TileBytes;
constexpr int kTcBarriers = 2 * kTcParts + 2 * kTcSlots;
constexpr int kTcSmemBytes = kTcXBytes + kTcWeightBytes + kTcBarriers * 8 + 16;
constexpr std::uint32_t kTcColumns = 512;     // one CTA per SM
constexpr int kTcDColumn = 0;                 // slot t: columns 32t..32t+31
constexpr int kTcAColumn = 32 * kTcSlots;     // slot t: columns +16t..+15

static_assert(kTensorCoreMaxBlocks % kTcPartBlocks == 0, "whole parts");
static_assert(kTcAColumn + 16 * kTcSlots <= static_cast<int>(kTcColumns),
              "TMEM slots exceed the allocation");
static_assert(kTcReadTeams * kTcRows * 32 * 4 <= kTcWeightBytes,
              "the reduction buffers reuse the weight area");
static_assert(kTcSmemBytes > 114 * 1024 && kTcSmemBytes <= 227 * 1024,
              "exactly one CTA per SM, which owns all 512 TMEM columns");

struct TcArgs {
  const Bf16* x;
  const unsigned char* w;
  float* y;
  Bf16* y_bf16;
  int m;
  int k;
  int n;
  int k_blocks;
  int splits;
  int blocks_per_split;
  int accumulate;
  int wait;
  int x_boxes;      // 1: one 3-D box per part; 32: 2-D boxes of 8 columns
  unsigned* error;  // the library's device error word
};

/// Waits for phase `parity` of `bar` (bounded) in every lane of the warp;
/// the warp agrees on the outcome.
__device__ inline bool WarpWait(std::uint64_t* bar, unsigned parity,
                                unsigned* word, unsigned error) {
  const bool ok = MbarWaitBounded(bar, parity, word, error);
  return __all_sync(0xFFFFFFFFu, ok) != 0;
}

/// Named barrier of one conversion team (its 128 threads, id 1 + team)
/// that ands `value` over them.
__device__ inline bool TeamAll(int team, bool value) {
  unsigned result;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\n"
      "bar.red.and.pred p, %2, 128, q;\nselp.u32 %0, 1, 0, p;\n}"
      : "=r"(result)
      : "r"(static_cast<unsigned>(value)), "r"(team + 1)
      : "memory");
  return result != 0;
}

__device__ inline float4 LoadFloat4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

template <int kRead>
__global__ void __launch_bounds__(kTcThreads, 1)
    TcProductKernel(const TcArgs p, const __grid_constant__ CUtensorMap x_map) {
  constexpr int kN = kRead <= 16 ? 16 : 32;  // the MMA's N (x rows, padded)
  constexpr std::uint32_t kInstruction = MmaBf16Descriptor(kTcRows, kN);
  extern __shared__ __align__(1024) unsigned char smem[];
  const int warp = static_cast<int>(threadIdx.x) >> 5;
  const int lane = static_cast<int>(threadIdx.x) & 31;
  const int split = static_cast<int>(blockIdx.x) % p.splits;
  const int panel = static_cast<int>(blockIdx.x) / p.splits;
  const int first = split * p.blocks_per_split;
  const int nb = max(0, min(p.k_blocks - first, p.blocks_per_split));
  const int parts = (nb + kTcPartBlocks - 1) / kTcPartBlocks;
  const int group0 = panel * kTcGroups;
  const int my_groups = min(kTcGroups, (p.n + 15) / 16 - group0);

  unsigned char* xs = smem;                 // [part][32 chunks][32 rows][16 B]
  unsigned char* wts = smem + kTcXBytes;    // [group][nb blocks] tiles
  std::uint64_t* wfull = reinterpret_cast<std::uint64_t*>(wts + kTcWeightBytes);
  std::uint64_t* xfull = wfull + kTcParts;
  std::uint64_t* dfull = xfull + kTcParts;
  std::uint64_t* tfree = dfull + kTcSlots;
  std::uint32_t* tmem_word = reinterpret_cast<std::uint32_t*>(tfree + kTcSlots);
  volatile std::uint32_t* aborted = tmem_word + 1;

  if (threadIdx.x == 0) {
    for (int q = 0; q < kTcParts; ++q) {
      MbarInit(&wfull[q], 1);
      MbarInit(&xfull[q], 1);
    }
    for (int t = 0; t < kTcSlots; ++t) {
      MbarInit(&dfull[t], 1);
      MbarInit(&tfree[t], 4);
    }
    *aborted = 0;
    FenceMbarInit();
  }
  if (warp == kTcProducerWarp) {
    TmemAlloc(tmem_word, kTcColumns);
    TmemRelinquish();
  }
  TcFenceBefore();
  __syncthreads();
  TcFenceAfter();
  const std::uint32_t tmem = *tmem_word;
  GridLaunchDependents();

  const int quarter = warp & 3;
  const int row = 32 * quarter + lane;  // CTA-local weight row (workers)
  const bool reader = warp >= kTcConvertWarps && warp < kTcWorkerWarps;
  const int read_team = (warp - kTcConvertWarps) >> 2;
  float acc[kRead];
#pragma unroll
  for (int c = 0; c < kRead; ++c)
    acc[c] = 0.0f;

  if (warp == kTcProducerWarp) {
    // Weights: one copy per group and part, from eight lanes at once (a TMA
    // request costs its issuing thread some 30-40 ns).
    if (lane == 0) {
      for (int q = 0; q < parts; ++q)
        MbarArriveExpectTx(&wfull[q],
                           my_groups * min(kTcPartBlocks, nb - kTcPartBlocks * q) *
                               kQ8TileBytes);
    }
    __syncwarp();
    if (lane < my_groups) {
      const std::uint64_t policy = PolicyEvictFirst();
      for (int q = 0; q < parts; ++q) {
        const int b0 = kTcPartBlocks * q;
        const int count = min(kTcPartBlocks, nb - b0);
        BulkLoad(wts + (lane * nb + b0) * kQ8TileBytes,
                 p.w + (static_cast<std::size_t>(group0 + lane) * p.k_blocks +
                        first + b0) * kQ8TileBytes,
                 count * kQ8TileBytes, &wfull[q], policy);
      }
    }
    // x after the preceding kernel (which may write it) has finished.
    if (p.wait)
      GridDependencyWait();
    if (lane == 0) {
      for (int q = 0; q < parts; ++q)
        MbarArriveExpectTx(&xfull[q], kTcXPartBytes);
    }
    __syncwarp();
    if (p.x_boxes == 1) {
      if (lane < parts)
        TmaLoad3D(xs + lane * kTcXPartBytes, &x_map, 0, 0,
                  (first + kTcPartBlocks * lane) * 4, &xfull[lane]);
    } else {
      for (int q = 0; q < parts; ++q)
        TmaLoad2D(xs + q * kTcXPartBytes + lane * kTcXChunkBytes, &x_map,
                  (first + kTcPartBlocks * q) * 32 + 8 * lane, 0, &xfull[q]);
    }
    // Copies still in flight land before the shared memory is released.
    if (lane == 0) {
      for (int q = 0; q < parts; ++q) {
        (void)MbarWaitBounded(&wfull[q], 0, p.error, kErrDrainWait,
                              100000000ull);
        (void)MbarWaitBounded(&xfull[q], 0, p.error, kErrDrainWait,
                              100000000ull);
      }
    }
    __syncwarp();
  } else if (warp < kTcConvertWarps) {
    // Conversion team `team` takes blocks team, team + 3, ...: each thread
    // turns its row's 32 values into bf16 in the block's TMEM A slot, the
    // team meets, and its issuer sends the block's two K=16 MMAs.
    const int team = warp >> 2;
    const int g = row >> 4;
    const int r = row & 15;
    const bool live = g < my_groups;
    // Rows 4..7 of each 8 read their two 16-byte halves in the other order,
    // so the eight lanes of a shared-memory phase hit distinct banks.
    const int swap = (r >> 2) & 1;
    const std::uint32_t lanes = static_cast<std::uint32_t>(32 * quarter) << 16;
    const bool issuer = quarter == 0 && lane == 0;
    int w_parts_ready = 0;  // parts of the weights known to have landed
    int x_parts_ready = 0;  // issuer: parts of x known to have landed
    for (int b = team; b < nb; b += kTcConvertTeams) {
      // Warp-uniform view of the abort flag (the .sync.aligned tcgen05
      // operations below need the whole warp).
      const bool quit = __shfl_sync(0xFFFFFFFFu, *aborted, 0) != 0u;
      const int t = b % kTcSlots;
      bool stored = false;
      if (!quit) {
        bool ok = true;
        for (; w_parts_ready <= b / kTcPartBlocks && ok; ++w_parts_ready)
          ok = WarpWait(&wfull[w_parts_ready], 0, p.error, kErrWeightWait);
        if (ok && b >= kTcSlots)
          ok = WarpWait(&tfree[t], (b / kTcSlots - 1) & 1, p.error,
                        kErrWeightWait);
        if (!ok) {
          *aborted = 1;
        } else {
          const unsigned char* tile = wts + (g * nb + b) * kQ8TileBytes;
          uint4 c0 = *reinterpret_cast<const uint4*>(tile + 32 * r + 16 * swap);
          uint4 c1 =
              *reinterpret_cast<const uint4*>(tile + 32 * r + 16 * (swap ^ 1));
          if (swap) {
            const uint4 tmp = c0;
            c0 = c1;
            c1 = tmp;
          }
          std::uint32_t a[16];
          DequantWord(c0.x, a[0], a[1]);
          DequantWord(c0.y, a[2], a[3]);
          DequantWord(c0.z, a[4], a[5]);
          DequantWord(c0.w, a[6], a[7]);
          DequantWord(c1.x, a[8], a[9]);
          DequantWord(c1.y, a[10], a[11]);
          DequantWord(c1.z, a[12], a[13]);
          DequantWord(c1.w, a[14], a[15]);
          if (!live) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              a[j] = 0u;
          }
          TmemStore16(tmem + lanes + kTcAColumn + 16 * t, a);
          TcFenceBefore();
          stored = true;
        }
      }
      // Every iteration meets, so the barrier counts match.
      const bool all_stored = TeamAll(team, stored);
      if (all_stored && issuer) {
        bool ok = true;
        for (; x_parts_ready <= b / kTcPartBlocks && ok; ++x_parts_ready)
          ok = MbarWaitBounded(&xfull[x_parts_ready], 0, p.error,
                               kErrActivationWait);
        if (!ok) {
          *aborted = 1;
        } else {
          TcFenceAfter();
#pragma unroll
          for (int s = 0; s < 2; ++s)
            MmaBf16TmemA(tmem + kTcDColumn + 32 * t,
                         tmem + kTcAColumn + 16 * t + 8 * s,
                         SmemDescriptorNoSwizzle(
                             xs + (4 * b + 2 * s) * kTcXChunkBytes,
                             kTcXChunkBytes, 128),
                         kInstruction, static_cast<std::uint32_t>(s));
          MmaCommit(&dfull[t]);
        }
      }
      __syncwarp();
    }
  } else {
    // Read team `read_team` takes blocks read_team, read_team + 2, ...: it
    // waits for the block's sums, frees the slot and adds them into the
    // rows' accumulators with the rows' fp16 scales (still in shared
    // memory with the weights).
    const int g = row >> 4;
    const int r = row & 15;
    const bool live = g < my_groups;
    const int scale_offset = 512 + (r < 8 ? 4 * r : 4 * (r - 8) + 2);
    const std::uint32_t lanes = static_cast<std::uint32_t>(32 * quarter) << 16;
    int w_parts_ready = 0;  // parts of the weights (and scales) seen landed
    for (int b = read_team; b < nb; b += kTcReadTeams) {
      const bool quit = __shfl_sync(0xFFFFFFFFu, *aborted, 0) != 0u;
      if (quit)
        break;
      const int t = b % kTcSlots;
      bool ok = true;
      for (; w_parts_ready <= b / kTcPartBlocks && ok; ++w_parts_ready)
        ok = WarpWait(&wfull[w_parts_ready], 0, p.error, kErrWeightWait);
      if (!ok) {
        *aborted = 1;
        break;
      }
      if (!WarpWait(&dfull[t], (b / kTcSlots) & 1, p.error, kErrWeightWait)) {
        *aborted = 1;
        break;
      }
      TcFenceAfter();
      std::uint32_t d[kRead];
      TmemLoad<kRead>(tmem + lanes + kTcDColumn + 32 * t, d);
      TcFenceBefore();
      __syncwarp();
      if (lane == 0)
        MbarArrive(&tfree[t]);
      const std::uint16_t bits = *reinterpret_cast<const std::uint16_t*>(
          wts + (g * nb + b) * kQ8TileBytes + scale_offset);
      const float scale = live ? HalfBitsToFloat(bits) : 0.0f;
#pragma unroll
      for (int c = 0; c < kRead; c += 2) {
        const float2 v = Fma2(make_float2(scale, scale),
                              make_float2(__uint_as_float(d[c]),
                                          __uint_as_float(d[c + 1])),
                              make_float2(acc[c], acc[c + 1]));
        acc[c] = v.x;
        acc[c + 1] = v.y;
      }
    }
  }

  // Every wait above is bounded, so every thread gets here.
  __syncthreads();
  TcFenceAfter();
  if (warp == kTcProducerWarp)
    TmemDealloc(tmem, kTcColumns);

  // The read teams, then the cluster's splits, add up in a fixed order.
  float* red = reinterpret_cast<float*>(wts);  // [read team - 1][128][kRead]
  float* part = red + (kTcReadTeams - 1) * kTcRows * kRead;  // [128][kRead]
  if (reader && read_team != 0) {
#pragma unroll
    for (int c = 0; c < kRead; c += 4)
      *reinterpret_cast<float4*>(red + ((read_team - 1) * kTcRows + row) *
                                           kRead + c) =
          make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
  }
  __syncthreads();
  if (reader && read_team == 0) {
    for (int other = 1; other < kTcReadTeams; ++other) {
#pragma unroll
      for (int c = 0; c < kRead; c += 4) {
        const float4 v =
            LoadFloat4(red + ((other - 1) * kTcRows + row) * kRead + c);
        acc[c] += v.x;
        acc[c + 1] += v.y;
        acc[c + 2] += v.z;
        acc[c + 3] += v.w;
      }
    }
  }
  if (p.splits > 1) {
    if (reader && read_team == 0 && split != 0) {
#pragma unroll
      for (int c = 0; c < kRead; c += 4)
        *reinterpret_cast<float4*>(part + row * kRead + c) =
            make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
    }
    ClusterSync();
    if (reader && read_team == 0 && split == 0) {
      for (int rank = 1; rank < p.splits; ++rank) {
#pragma unroll
        for (int c = 0; c < kRead; c += 4) {
          const float4 v = LoadSharedCluster4(
              MapShared(part + row * kRead + c, static_cast<unsigned>(rank)));
          acc[c] += v.x;
          acc[c + 1] += v.y;
          acc[c + 2] += v.z;
          acc[c + 3] += v.w;
        }
      }
    }
    ClusterSync();  // the others keep their shared memory until it was read
  }
  if (!reader || read_team != 0 || split != 0 || *aborted != 0)
    return;
  const int n = group0 * 16 + row;
  if (n >= p.n)
    return;
  if (p.accumulate && p.wait)
    GridDependencyWait();  // y may be the preceding kernel's output
#pragma unroll
  for (int m = 0; m < kRead; ++m) {
    if (m < p.m) {
      const std::size_t index = static_cast<std::size_t>(m) * p.n + n;
      float value = acc[m];
      if (p.y != nullptr) {
        if (p.accumulate)
          value = p.y[index] + value;
        p.y[index] = value;
      } else {
        if (p.accumulate)
          value = Bf16ToFloat(p.y_bf16[index]) + value;
        p.y_bf16[index] = FloatToBf16(value);
      }
    }
  }
}

/// The tensor map of x [rows][in] bf16 for the B operand. Preferred: x
/// viewed as 3-D {8 columns, rows, in / 8 chunks} (strides in*2 and 16
/// bytes) with a box of {8, 32, 32}, which lands one part (32 chunks of all
/// 32 rows, 16 KB) as K-major core matrices in one request (`*boxes` = 1).
/// If the driver does not take that view: 2-D with a box of 8 columns x 32
/// rows, 32 requests per part (`*boxes` = 32).
bool EncodeActivations(const std::uint16_t* x, std::size_t rows,
                       std::size_t in, CUtensorMap* map, int* boxes) {
  {
    const std::uint64_t dims[3] = {8, rows, in / 8};
    const std::uint64_t strides[2] = {in * 2, 16};
    const std::uint32_t box[3] = {8, static_cast<std::uint32_t>(kTcXRows),
                                  4 * kTcPartBlocks};
    if (EncodeBf16TensorMap(map, x, 3, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_NONE)) {
      *boxes = 1;
      return true;
    }
  }
  const std::uint64_t dims[2] = {in, rows};
  const std::uint64_t strides[1] = {in * 2};
  const std::uint32_t box[2] = {8, static_cast<std::uint32_t>(kTcXRows)};
  *boxes = 32;
  return EncodeBf16TensorMap(map, x, 2, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_NONE);
}

}  // namespace

ProductPlan PlanTensorCoreProduct(std::size_t rows, std::size_t in,
                                  std::size_t out, int sms) {
  ProductPlan plan;
  if (rows < 1 || rows > kTensorCoreMaxRows || in == 0 ||
      in % kTileColumns != 0 || out == 0)
    return plan;
  const int k_blocks = static_cast<int>(in / kTileColumns);
  const int panels = static_cast<int>(((out + 15) / 16 + kTcGroups - 1) /
                                      kTcGroups);
  int splits = std::max((k_blocks + kTensorCoreMaxBlocks - 1) /
                            kTensorCoreMaxBlocks,
                        (sms + panels / 2) / std::max(panels, 1));
  splits = std::max(1, std::min({splits, 8, k_blocks}));
  const int bps = (k_blocks + splits - 1) / splits;
  if (bps > kTensorCoreMaxBlocks)
    return plan;
  plan.variant = kTensorCoreVariant;
  plan.blocks_per_split = bps;
  plan.splits = (k_blocks + bps - 1) / bps;
  return plan;
}

int LaunchTensorCoreProduct(const std::uint16_t* x, const void* w, float* y,
                            std::uint16_t* y_bf16, std::size_t rows,
                            std::size_t in, std::size_t out, bool accumulate,
                            const ProductPlan& plan, cudaStream_t stream,
                            bool independent, bool programmatic) {
  const int k_blocks = static_cast<int>(in / kTileColumns);
  if (rows < 1 || rows > kTensorCoreMaxRows || plan.splits < 1 ||
      plan.splits > 8 || plan.blocks_per_split < 1 ||
      plan.blocks_per_split > kTensorCoreMaxBlocks ||
      (k_blocks + plan.blocks_per_split - 1) / plan.blocks_per_split !=
          plan.splits)
    return kUnsupported;
  const int read = rows <= 16 ? 16 : rows <= 24 ? 24 : 32;
  void (*kernel)(const TcArgs, const CUtensorMap) =
      read == 16   ? TcProductKernel<16>
                                 : read == 24 ? TcProductKernel<24>
                                              : TcProductKernel<32>;
  unsigned* error_word = nullptr;
  {
    // Per device: the kernels' shared-memory limit and the error word.
    static std::mutex mutex;
    static bool configured[8][3] = {};
    static unsigned* words[8] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess)
      return kCudaError;
    std::lock_guard<std::mutex> lock(mutex);
    bool& done = configured[device & 7][read / 8 - 2];
    if (!done) {
      if (cudaFuncSetAttribute(kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kTcSmemBytes) != cudaSuccess)
        return kCudaError;
      done = true;
    }
    if (words[device & 7] == nullptr)
      words[device & 7] = DeviceErrorWord();
    error_word = words[device & 7];
  }
  if (error_word == nullptr)
    return kCudaError;
  TcArgs args;
  args.x = x;
  args.w = static_cast<const unsigned char*>(w);
  args.y = y;
  args.y_bf16 = y != nullptr ? nullptr : y_bf16;
  args.m = static_cast<int>(rows);
  args.k = static_cast<int>(in);
  args.n = static_cast<int>(out);
  args.k_blocks = k_blocks;
  args.splits = plan.splits;
  args.blocks_per_split = plan.blocks_per_split;
  args.accumulate = accumulate ? 1 : 0;
  args.wait = independent ? 0 : 1;
  args.error = error_word;
  const int panels = static_cast<int>(((out + 15) / 16 + kTcGroups - 1) /
                                      kTcGroups);
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(static_cast<unsigned>(panels * plan.splits));
  config.blockDim = dim3(kTcThreads);
  config.dynamicSmemBytes = kTcSmemBytes;
  config.stream = stream;
  cudaLaunchAttribute attributes[2];
  int count = 0;
  if (plan.splits > 1) {
    attributes[count].id = cudaLaunchAttributeClusterDimension;
    attributes[count].val.clusterDim.x = static_cast<unsigned>(plan.splits);
    attributes[count].val.clusterDim.y = 1;
    attributes[count].val.clusterDim.z = 1;
    ++count;
  }
  if (programmatic) {
    attributes[count].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attributes[count].val.programmaticStreamSerializationAllowed = 1;
    ++count;
  }
  config.attrs = attributes;
  config.numAttrs = count;
  CUtensorMap x_map;
  if (!EncodeActivations(x, rows, in, &x_map, &args.x_boxes))
    return kInvalid;
  if (cudaLaunchKernelEx(&config, kernel, args, x_map) != cudaSuccess)
    return kCudaError;
  return kOk;
}

namespace {

/// cuTensorMapEncodeTiled through the runtime's driver entry point.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType,
                                   cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn TensorMapEncoder() {
  static const EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult found;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f,
                                cudaEnableDefault, &found) != cudaSuccess ||
        found != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

}  // namespace

bool EncodeBf16TensorMap(CUtensorMap* map, const void* base, int rank,
                         const std::uint64_t* dims,
                         const std::uint64_t* strides,
                         const std::uint32_t* box, CUtensorMapSwizzle swizzle) {
  const EncodeTiledFn encode = TensorMapEncoder();
  if (encode == nullptr || rank < 1 || rank > 5)
    return false;
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank)
      st[i] = strides[i];
  }
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, st,
                b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace vx
