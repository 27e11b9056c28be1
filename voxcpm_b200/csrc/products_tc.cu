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
// One CTA owns 128 weight rows (8 tile groups) over a slice of at most 24
// blocks of the reduction; the CTAs of a thread-block cluster take
// consecutive slices of the same rows and add up in cluster-rank order
// through distributed shared memory (the reference's ordered split sum,
// kernels/wmma_products.hip:249-295). Per CTA:
// - a producer warp streams the rows' tiles, two blocks per stage, into a
//   ring of 1-D TMA bulk copies (L2 evict-first);
// - eight worker warps, two per TMEM lane quarter, take alternate blocks:
//   each thread owns one weight row, turns its 32 biased int8 values into
//   bf16 exactly, and stores them into a TMEM A slot (tcgen05.st);
// - an MMA warp issues D[slot] = A[slot] x x_block (two K=16 steps, fresh
//   accumulator) and commits to the slot's mbarrier;
// - the worker reads the block sums back (tcgen05.ld) and adds them into its
//   registers with the row's fp16 scale;
// - the producer also brings the CTA's slice of x in with 2-D TMA, one box
//   of 8 columns x 32 rows per copy, which lands as the MMA's B operand in
//   the no-swizzle K-major layout (8-row x 16-byte core matrices); rows past
//   the activation rows are zero-filled by the copy.
// Weights do not depend on earlier kernels, so the first ring of them
// streams (and is converted) before the programmatic-launch wait; x is
// read after it.
#include "products.cuh"
#include "product_math.cuh"
#include "tcgen05.cuh"
#include "vx_common.cuh"

#include <cuda.h>

#include <algorithm>
#include <mutex>

namespace vx {

namespace {

constexpr int kTcGroups = 8;                  // 16-row tile groups per CTA
constexpr int kTcRows = 16 * kTcGroups;       // = the MMA's M (TMEM lanes)
constexpr int kTcStage = 2;                   // blocks per ring stage
constexpr int kTcRing = 5;                    // ring stages
constexpr int kTcSlots = 5;                   // TMEM A / accumulator slots
constexpr int kTcWorkerWarps = 8;
constexpr int kTcProducerWarp = kTcWorkerWarps;
constexpr int kTcMmaWarp = kTcWorkerWarps + 1;
constexpr int kTcThreads = 32 * (kTcWorkerWarps + 2);
constexpr int kTcXRows = 32;                  // B rows staged (M <= 32)
constexpr int kTcXChunkBytes = kTcXRows * 16; // 8 K-values of all 32 rows
constexpr int kTcXBytes = kTcXRows * kTensorCoreMaxBlocks * 32 * 2;
constexpr int kTcStageBytes = kTcGroups * kTcStage * kQ8TileBytes;
constexpr int kTcRingBytes = kTcRing * kTcStageBytes;
constexpr int kTcBarriers = 2 * kTcRing + 3 * kTcSlots + 1;
constexpr int kTcSmemBytes = kTcXBytes + kTcRingBytes + kTcBarriers * 8 + 16;
constexpr std::uint32_t kTcColumns = 256;     // two CTAs fit on one SM
constexpr int kTcDColumn = 0;                 // slot t: columns 32t..32t+31
constexpr int kTcAColumn = 32 * kTcSlots;     // slot t: columns +16t..+15

static_assert(kTcAColumn + 16 * kTcSlots <= static_cast<int>(kTcColumns),
              "TMEM slots exceed the allocation");
static_assert(2 * kTcRows * 32 * 4 <= kTcRingBytes,
              "the reduction buffers reuse the ring");
static_assert(kTcSmemBytes <= 113 * 1024, "two CTAs per SM");

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
  unsigned* error;  // the library's device error word
};

/// Waits for phase `parity` of `bar` (bounded) in every lane of the warp;
/// the warp agrees on the outcome.
__device__ inline bool WarpWait(std::uint64_t* bar, unsigned parity,
                                unsigned* word, unsigned error) {
  const bool ok = MbarWaitBounded(bar, parity, word, error);
  return __all_sync(0xFFFFFFFFu, ok) != 0;
}

__device__ inline float4 LoadFloat4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

template <int kRead>
__global__ void __launch_bounds__(kTcThreads, 2)
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
  const int group0 = panel * kTcGroups;
  const int my_groups = min(kTcGroups, (p.n + 15) / 16 - group0);

  unsigned char* xs = smem;
  unsigned char* ring = smem + kTcXBytes;
  std::uint64_t* wfull = reinterpret_cast<std::uint64_t*>(ring + kTcRingBytes);
  std::uint64_t* wempty = wfull + kTcRing;
  std::uint64_t* aready = wempty + kTcRing;
  std::uint64_t* dfull = aready + kTcSlots;
  std::uint64_t* tfree = dfull + kTcSlots;
  std::uint64_t* xready = tfree + kTcSlots;
  std::uint32_t* tmem_word = reinterpret_cast<std::uint32_t*>(xready + 1);
  volatile std::uint32_t* aborted = tmem_word + 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcRing; ++i) {
      MbarInit(&wfull[i], 1);
      MbarInit(&wempty[i], kTcWorkerWarps);
    }
    for (int t = 0; t < kTcSlots; ++t) {
      MbarInit(&aready[t], 4);
      MbarInit(&dfull[t], 1);
      MbarInit(&tfree[t], 4);
    }
    MbarInit(xready, 1);
    *aborted = 0;
    FenceMbarInit();
  }
  if (warp == kTcMmaWarp) {
    TmemAlloc(tmem_word, kTcColumns);
    TmemRelinquish();
  }
  TcFenceBefore();
  __syncthreads();
  TcFenceAfter();
  const std::uint32_t tmem = *tmem_word;
  GridLaunchDependents();

  const bool worker = warp < kTcWorkerWarps;
  const int quarter = warp & 3;
  const int half = (warp >> 2) & 1;
  const int row = 32 * quarter + lane;  // CTA-local weight row (workers)
  float acc[kRead];
#pragma unroll
  for (int c = 0; c < kRead; ++c)
    acc[c] = 0.0f;

  if (warp == kTcProducerWarp) {
    if (lane == 0) {
      const std::uint64_t policy = PolicyEvictFirst();
      const int stages = (nb + kTcStage - 1) / kTcStage;
      int issued = 0;
      auto issue = [&](int i) {
        const int slot = i % kTcRing;
        const int b0 = first + i * kTcStage;
        const int count = min(kTcStage, first + nb - b0);
        MbarArriveExpectTx(&wfull[slot], my_groups * count * kQ8TileBytes);
        for (int g = 0; g < my_groups; ++g)
          BulkLoad(ring + slot * kTcStageBytes + g * kTcStage * kQ8TileBytes,
                   p.w + (static_cast<std::size_t>(group0 + g) * p.k_blocks +
                          b0) * kQ8TileBytes,
                   count * kQ8TileBytes, &wfull[slot], policy);
      };
      // The first ring of weights before the wait for the preceding kernel.
      for (; issued < min(stages, kTcRing); ++issued)
        issue(issued);
      if (p.wait)
        GridDependencyWait();
      // x: four boxes of 8 columns per block, 32 rows each (rows past
      // p.m read as zeros).
      MbarArriveExpectTx(xready, 4 * nb * kTcXChunkBytes);
      for (int c = 0; c < 4 * nb; ++c)
        TmaLoad2D(xs + c * kTcXChunkBytes, &x_map, first * 32 + 8 * c, 0,
                  xready);
      for (; issued < stages && *aborted == 0; ++issued) {
        const int slot = issued % kTcRing;
        if (!MbarWaitBounded(&wempty[slot], (issued / kTcRing - 1) & 1,
                             p.error, kErrWeightWait)) {
          *aborted = 1;
          break;
        }
        issue(issued);
      }
      // Copies still in flight land before the shared memory is released.
      (void)MbarWaitBounded(xready, 0, p.error, kErrDrainWait, 100000000ull);
      for (int i = max(0, issued - kTcRing); i < issued; ++i)
        (void)MbarWaitBounded(&wfull[i % kTcRing], (i / kTcRing) & 1,
                              p.error, kErrDrainWait, 100000000ull);
    }
    __syncwarp();
  } else if (warp == kTcMmaWarp) {
    if (lane == 0) {
      int issued = 0;
      if (!MbarWaitBounded(xready, 0, p.error,
                           kErrActivationWait))
        *aborted = 1;
      for (int b = 0; b < nb && *aborted == 0; ++b) {
        const int t = b % kTcSlots;
        if (!MbarWaitBounded(&aready[t], (b / kTcSlots) & 1,
                             p.error, kErrWeightWait)) {
          *aborted = 1;
          break;
        }
        TcFenceAfter();
        const std::uint32_t a = tmem + kTcAColumn + 16 * t;
        const std::uint32_t d = tmem + kTcDColumn + 32 * t;
#pragma unroll
        for (int s = 0; s < 2; ++s)
          MmaBf16TmemA(d, a + 8 * s,
                       SmemDescriptorNoSwizzle(
                           xs + (4 * b + 2 * s) * kTcXChunkBytes,
                           kTcXChunkBytes, 128),
                       kInstruction, static_cast<std::uint32_t>(s));
        MmaCommit(&dfull[t]);
        ++issued;
      }
      // Every MMA has completed before the columns are freed.
      if (issued > 0)
        (void)MbarWaitBounded(&dfull[(issued - 1) % kTcSlots],
                              ((issued - 1) / kTcSlots) & 1,
                              p.error, kErrDrainWait,
                              100000000ull);
    }
    __syncwarp();
  } else {
    const int g = row >> 4;
    const int r = row & 15;
    const bool live = g < my_groups;
    const int scale_offset = 512 + (r < 8 ? 4 * r : 4 * (r - 8) + 2);
    // Rows 4..7 of each 8 read their two 16-byte halves in the other order,
    // so the eight lanes of a shared-memory phase hit distinct banks.
    const int swap = (r >> 2) & 1;
    const std::uint32_t lanes = static_cast<std::uint32_t>(32 * quarter) << 16;
    int prev = -1;
    float prev_scale = 0.0f;
    for (int b = half; b < nb + 2; b += 2) {
      // Warp-uniform view of the abort flag (the .sync.aligned tcgen05
      // operations below need the whole warp).
      const bool quit = __shfl_sync(0xFFFFFFFFu, *aborted, 0) != 0u;
      const bool has = b < nb && !quit;
      float scale = 0.0f;
      bool stored = false;
      if (has) {
        const int i = b / kTcStage;
        const int rs = i % kTcRing;
        if (!WarpWait(&wfull[rs], (i / kTcRing) & 1, p.error, kErrWeightWait)) {
          *aborted = 1;
        } else {
          const unsigned char* tile =
              ring + rs * kTcStageBytes +
              (g * kTcStage + (b % kTcStage)) * kQ8TileBytes;
          uint4 c0 = *reinterpret_cast<const uint4*>(tile + 32 * r + 16 * swap);
          uint4 c1 =
              *reinterpret_cast<const uint4*>(tile + 32 * r + 16 * (swap ^ 1));
          const std::uint16_t bits =
              *reinterpret_cast<const std::uint16_t*>(tile + scale_offset);
          __syncwarp();
          if (lane == 0)
            MbarArrive(&wempty[rs]);
          if (swap) {
            const uint4 t = c0;
            c0 = c1;
            c1 = t;
          }
          scale = live ? HalfBitsToFloat(bits) : 0.0f;
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
          const int t = b % kTcSlots;
          if (b >= kTcSlots &&
              !WarpWait(&tfree[t], (b / kTcSlots - 1) & 1, p.error,
                        kErrWeightWait)) {
            *aborted = 1;
          } else {
            TmemStore16(tmem + lanes + kTcAColumn + 16 * t, a);
            TcFenceBefore();
            __syncwarp();
            if (lane == 0)
              MbarArrive(&aready[t]);
            stored = true;
          }
        }
      }
      if (prev >= 0 && !quit) {
        const int t = prev % kTcSlots;
        if (!WarpWait(&dfull[t], (prev / kTcSlots) & 1, p.error,
                      kErrWeightWait)) {
          *aborted = 1;
        } else {
          TcFenceAfter();
          std::uint32_t d[kRead];
          TmemLoad<kRead>(tmem + lanes + kTcDColumn + 32 * t, d);
          TcFenceBefore();
          __syncwarp();
          if (lane == 0)
            MbarArrive(&tfree[t]);
#pragma unroll
          for (int c = 0; c < kRead; c += 2) {
            const float2 v = Fma2(make_float2(prev_scale, prev_scale),
                                  make_float2(__uint_as_float(d[c]),
                                              __uint_as_float(d[c + 1])),
                                  make_float2(acc[c], acc[c + 1]));
            acc[c] = v.x;
            acc[c + 1] = v.y;
          }
        }
      }
      prev = stored ? b : -1;
      prev_scale = scale;
    }
  }

  // Every wait above is bounded, so every thread gets here.
  __syncthreads();
  TcFenceAfter();
  if (warp == kTcMmaWarp)
    TmemDealloc(tmem, kTcColumns);

  // The two halves, then the cluster's splits, add up in a fixed order.
  float* red = reinterpret_cast<float*>(ring);      // [128][kRead]
  float* part = red + kTcRows * kRead;              // [128][kRead]
  if (worker && half == 1) {
#pragma unroll
    for (int c = 0; c < kRead; c += 4)
      *reinterpret_cast<float4*>(red + row * kRead + c) =
          make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
  }
  __syncthreads();
  if (worker && half == 0) {
#pragma unroll
    for (int c = 0; c < kRead; c += 4) {
      const float4 v = LoadFloat4(red + row * kRead + c);
      acc[c] += v.x;
      acc[c + 1] += v.y;
      acc[c + 2] += v.z;
      acc[c + 3] += v.w;
    }
  }
  if (p.splits > 1) {
    if (worker && half == 0 && split != 0) {
#pragma unroll
      for (int c = 0; c < kRead; c += 4)
        *reinterpret_cast<float4*>(part + row * kRead + c) =
            make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
    }
    ClusterSync();
    if (worker && half == 0 && split == 0) {
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
  if (!worker || half != 0 || split != 0 || *aborted != 0)
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

/// cuTensorMapEncodeTiled, reached through the runtime's driver entry
/// point (no link against the driver library).
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

/// The tensor map of x [rows][in] bf16 with a box of 8 columns x 32 rows.
bool EncodeActivations(const std::uint16_t* x, std::size_t rows,
                       std::size_t in, CUtensorMap* map) {
  const EncodeTiledFn encode = TensorMapEncoder();
  if (encode == nullptr)
    return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(in),
                              static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(in) * 2};
  const cuuint32_t box[2] = {8, static_cast<cuuint32_t>(kTcXRows)};
  const cuuint32_t element_strides[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                const_cast<std::uint16_t*>(x), dims, strides, box,
                element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

ProductPlan PlanTensorCoreProduct(std::size_t rows, std::size_t in,
                                  std::size_t out, int sms) {
  ProductPlan plan;
  if (rows < 1 || rows > kMaxProductRows || in == 0 ||
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
  if (rows < 1 || rows > kMaxProductRows || plan.splits < 1 ||
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
  if (!EncodeActivations(x, rows, in, &x_map))
    return kInvalid;
  if (cudaLaunchKernelEx(&config, kernel, args, x_map) != cudaSuccess)
    return kCudaError;
  return kOk;
}

}  // namespace vx
