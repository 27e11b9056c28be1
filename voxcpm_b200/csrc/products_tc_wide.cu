// The tensor-core (tcgen05) product for 33..128 activation rows and Q8_0
// tiles on sm_100a: y[rows][out] (+)= x[rows][in] * W[out][in]^T with the
// reference's per-block arithmetic (kernels/wmma_products.hip:139-296):
// every 32-column block of a weight row is summed in fp32 over exact bf16
// values of q, then added into the row's accumulator as
// fmaf(scale, block sum, acc), block after block in order.
//
// Why: at 64 or 128 rows the legacy mma.sync path needs 16 or 32 MMAs per
// 16 x 32 weight tile and is compute-bound far below the HBM rate, and
// long reductions fall back to 32-row launches that re-read the weights.
// Here one thread issues a 128 x N x 16 tcgen05 MMA (N = the rows rounded up
// to 64, 96 or 128) per K step, so every weight byte is read once and the
// tensor pipe has room to spare.
//
// One CTA per SM owns 128 weight rows (8 tile groups, the MMA's M) over a
// slice of the reduction; the CTAs of a thread-block cluster take
// consecutive slices and add up in cluster-rank order through distributed
// shared memory. Per CTA:
// - a producer warp streams the slice in parts of 8 blocks through a
//   two-stage ring: per part one bulk copy per tile group (weights) and four
//   tensor-map copies of 64 columns x N rows of x with the 128-byte swizzle,
//   which land as the MMA's K-major B operand in 128-byte rows (rows past
//   the activation rows are zero-filled). 128-byte rows keep the copy's
//   request count low: 16-byte pieces, one per row and 8 columns, took the
//   copy engine about 7 ns each;
// - two conversion teams of four warps take alternate blocks: each thread
//   owns one weight row, turns its 32 biased int8 values into bf16 exactly
//   and stores them into the block's TMEM A slot; the team meets at a named
//   barrier and one lane issues D[slot] = A[slot] x x_block (two K = 16
//   steps), committing to the slot's mbarrier;
// - one read team of four warps per 32 columns of N reads its columns of
//   every block's sums back (tcgen05.ld) in block order and adds them into
//   its rows' accumulators with the rows' fp16 scales; the last reader of a
//   part frees its ring stage.
// Every wait is bounded: on a timeout the kernel records an error bit,
// stops, lets its copies and MMAs land, frees its TMEM and returns.
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

constexpr int kWGroups = 8;             // 16-row tile groups per CTA
constexpr int kWRows = 16 * kWGroups;   // = the MMA's M (TMEM lanes)
constexpr int kWPartBlocks = 8;         // blocks per ring stage
constexpr int kWStages = 2;
constexpr int kWConvertTeams = 2;
constexpr int kWConvertWarps = 4 * kWConvertTeams;
constexpr std::uint32_t kWColumns = 512;  // one CTA per SM

template <int kChunks>
struct Wide {
  static constexpr int kN = 32 * kChunks;          // the MMA's N
  static constexpr int kReadWarps = 4 * kChunks;   // one team per 32 columns
  static constexpr int kProducerWarp = kWConvertWarps + kReadWarps;
  static constexpr int kThreads = 32 * (kProducerWarp + 1);
  static constexpr int kSlots = 512 / (kN + 16);   // TMEM D + A slots
  static constexpr int kXBoxBytes = kN * 128;      // 64 K-values of all N rows
  static constexpr int kXPartBytes = (kWPartBlocks / 2) * kXBoxBytes;
  static constexpr int kWPartBytes = kWGroups * kWPartBlocks * kQ8TileBytes;
  static constexpr int kStageBytes = kXPartBytes + kWPartBytes;
  static constexpr int kBarriers = 2 * kWStages + 2 * kSlots;
  static constexpr int kSmemBytes = kWStages * kStageBytes + kBarriers * 8 + 16;
  static constexpr int kAColumn = kSlots * kN;     // slot t: +16t..+16t+15
  static_assert(kSlots >= 3, "a pipeline needs three TMEM slots");
  static_assert(kAColumn + 16 * kSlots <= static_cast<int>(kWColumns),
                "TMEM slots exceed the allocation");
  static_assert(kStageBytes % 1024 == 0 && kXBoxBytes % 1024 == 0,
                "stages and swizzle atoms stay 1 KB aligned");
  static_assert(kWRows * kN * 4 <= kWStages * kStageBytes,
                "the split sums reuse the ring");
  static_assert(kSmemBytes > 114 * 1024 && kSmemBytes <= 227 * 1024,
                "exactly one CTA per SM, which owns all 512 TMEM columns");
};

struct WideArgs {
  const unsigned char* w;
  float* y;
  Bf16* y_bf16;
  int m;
  int n;
  int k_blocks;
  int splits;
  int blocks_per_split;
  int accumulate;
  int wait;
  unsigned* error;
};

__device__ inline bool WarpWaitW(std::uint64_t* bar, unsigned parity,
                                 unsigned* word, unsigned error) {
  const bool ok = MbarWaitBounded(bar, parity, word, error);
  return __all_sync(0xFFFFFFFFu, ok) != 0;
}

/// Named barrier of one conversion team (128 threads, id 1 + team) that
/// ands `value` over them.
__device__ inline bool TeamAllW(int team, bool value) {
  unsigned result;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\n"
      "bar.red.and.pred p, %2, 128, q;\nselp.u32 %0, 1, 0, p;\n}"
      : "=r"(result)
      : "r"(static_cast<unsigned>(value)), "r"(team + 1)
      : "memory");
  return result != 0;
}

template <int kChunks>
__global__ void __launch_bounds__(Wide<kChunks>::kThreads, 1)
    TcWideKernel(const WideArgs p, const __grid_constant__ CUtensorMap x_map) {
  using S = Wide<kChunks>;
  constexpr std::uint32_t kInstruction = MmaBf16Descriptor(kWRows, S::kN);
  extern __shared__ __align__(1024) unsigned char smem[];
  const int warp = static_cast<int>(threadIdx.x) >> 5;
  const int lane = static_cast<int>(threadIdx.x) & 31;
  const int split = static_cast<int>(blockIdx.x) % p.splits;
  const int panel = static_cast<int>(blockIdx.x) / p.splits;
  const int first = split * p.blocks_per_split;
  const int nb = max(0, min(p.k_blocks - first, p.blocks_per_split));
  const int parts = (nb + kWPartBlocks - 1) / kWPartBlocks;
  const int group0 = panel * kWGroups;
  const int my_groups = min(kWGroups, (p.n + 15) / 16 - group0);

  std::uint64_t* full = reinterpret_cast<std::uint64_t*>(smem + kWStages * S::kStageBytes);
  std::uint64_t* empty = full + kWStages;
  std::uint64_t* dfull = empty + kWStages;
  std::uint64_t* tfree = dfull + S::kSlots;
  std::uint32_t* tmem_word = reinterpret_cast<std::uint32_t*>(tfree + S::kSlots);
  volatile std::uint32_t* aborted = tmem_word + 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) {
      MbarInit(&full[s], 1);
      MbarInit(&empty[s], S::kReadWarps);
    }
    for (int t = 0; t < S::kSlots; ++t) {
      MbarInit(&dfull[t], 1);
      MbarInit(&tfree[t], S::kReadWarps);
    }
    *aborted = 0;
    FenceMbarInit();
  }
  if (warp == S::kProducerWarp) {
    TmemAlloc(tmem_word, kWColumns);
    TmemRelinquish();
  }
  TcFenceBefore();
  __syncthreads();
  TcFenceAfter();
  const std::uint32_t tmem = *tmem_word;
  GridLaunchDependents();

  const int quarter = warp & 3;
  const int row = 32 * quarter + lane;  // CTA-local weight row (workers)
  const bool reader = warp >= kWConvertWarps && warp < S::kProducerWarp;
  const int chunk = (warp - kWConvertWarps) >> 2;  // readers: columns 32c..
  float acc[32];
#pragma unroll
  for (int c = 0; c < 32; ++c)
    acc[c] = 0.0f;

  if (warp == S::kProducerWarp) {
    int issued = 0;
    bool waited = false;
    for (int q = 0; q < parts; ++q) {
      const int stage = q % kWStages;
      if (q >= kWStages) {
        const bool ok = WarpWaitW(&empty[stage], ((q / kWStages) - 1) & 1,
                                  p.error, kErrWeightWait);
        if (!ok || *aborted != 0) {
          *aborted = 1;
          break;
        }
      }
      unsigned char* xs = smem + stage * S::kStageBytes;
      unsigned char* ws = xs + S::kXPartBytes;
      const int b0 = kWPartBlocks * q;
      const int count = min(kWPartBlocks, nb - b0);
      if (lane == 0)
        MbarArriveExpectTx(&full[stage],
                           my_groups * count * kQ8TileBytes + S::kXPartBytes);
      __syncwarp();
      if (lane < my_groups)
        BulkLoad(ws + lane * kWPartBlocks * kQ8TileBytes,
                 p.w + (static_cast<std::size_t>(group0 + lane) * p.k_blocks +
                        first + b0) * kQ8TileBytes,
                 count * kQ8TileBytes, &full[stage], PolicyEvictFirst());
      // x after the preceding kernel (which may write it) has finished.
      if (p.wait && !waited) {
        GridDependencyWait();
        waited = true;
      }
      // x: four boxes of 64 columns x N rows (128-byte swizzled rows).
      if (lane < 4)
        TmaLoad2D(xs + lane * S::kXBoxBytes, &x_map, (first + b0) * 32 + 64 * lane,
                  0, &full[stage]);
      __syncwarp();
      issued = q + 1;
    }
    // Copies still in flight land before the shared memory is released.
    if (lane == 0) {
      for (int q = max(0, issued - kWStages); q < issued; ++q)
        (void)MbarWaitBounded(&full[q % kWStages], (q / kWStages) & 1, p.error,
                              kErrDrainWait, 100000000ull);
    }
    __syncwarp();
  } else if (warp < kWConvertWarps) {
    const int team = warp >> 2;
    const int g = row >> 4;
    const int r = row & 15;
    const bool live = g < my_groups;
    const int swap = (r >> 2) & 1;
    const std::uint32_t lanes = static_cast<std::uint32_t>(32 * quarter) << 16;
    const bool issuer = quarter == 0 && lane == 0;
    int last_slot = -1;
    int last_parity = 0;
    for (int b = team; b < nb; b += kWConvertTeams) {
      const bool quit = __shfl_sync(0xFFFFFFFFu, *aborted, 0) != 0u;
      const int t = b % S::kSlots;
      const int q = b / kWPartBlocks;
      const int stage = q % kWStages;
      const int j = b % kWPartBlocks;
      unsigned char* xs = smem + stage * S::kStageBytes;
      const unsigned char* ws = xs + S::kXPartBytes;
      bool stored = false;
      if (!quit) {
        bool ok = WarpWaitW(&full[stage], (q / kWStages) & 1, p.error,
                            kErrWeightWait);
        if (ok && b >= S::kSlots)
          ok = WarpWaitW(&tfree[t], ((b / S::kSlots) - 1) & 1, p.error,
                         kErrWeightWait);
        if (!ok) {
          *aborted = 1;
        } else {
          const unsigned char* tile = ws + (g * kWPartBlocks + j) * kQ8TileBytes;
          uint4 c0 = *reinterpret_cast<const uint4*>(tile + 32 * r + 16 * swap);
          uint4 c1 = *reinterpret_cast<const uint4*>(tile + 32 * r + 16 * (swap ^ 1));
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
            for (int i = 0; i < 16; ++i)
              a[i] = 0u;
          }
          TmemStore16(tmem + lanes + S::kAColumn + 16 * t, a);
          TcFenceBefore();
          stored = true;
        }
      }
      // Every iteration meets, so the barrier counts match.
      const bool all_stored = TeamAllW(team, stored);
      if (all_stored && issuer) {
        TcFenceAfter();
#pragma unroll
        for (int s = 0; s < 2; ++s)
          MmaBf16TmemA(tmem + S::kN * t, tmem + S::kAColumn + 16 * t + 8 * s,
                       SmemDescriptorSw128(xs + (j >> 1) * S::kXBoxBytes +
                                               64 * (j & 1) + 32 * s,
                                           1024),
                       kInstruction, static_cast<std::uint32_t>(s));
        MmaCommit(&dfull[t]);
        last_slot = t;
        last_parity = (b / S::kSlots) & 1;
      }
      __syncwarp();
    }
    // MMAs still in flight finish before the TMEM is released.
    if (issuer && last_slot >= 0)
      (void)MbarWaitBounded(&dfull[last_slot], last_parity, p.error,
                            kErrDrainWait, 100000000ull);
  } else {
    // Read team `chunk` adds columns 32 chunk.. of every block, in order.
    const int g = row >> 4;
    const int r = row & 15;
    const bool live = g < my_groups;
    const int scale_offset = 512 + (r < 8 ? 4 * r : 4 * (r - 8) + 2);
    const std::uint32_t lanes = static_cast<std::uint32_t>(32 * quarter) << 16;
    for (int b = 0; b < nb; ++b) {
      const bool quit = __shfl_sync(0xFFFFFFFFu, *aborted, 0) != 0u;
      if (quit)
        break;
      const int t = b % S::kSlots;
      const int q = b / kWPartBlocks;
      const int stage = q % kWStages;
      const int j = b % kWPartBlocks;
      // The part's scales (with its weights) have landed; the stage is not
      // refilled before this warp frees it.
      if (j == 0 && !WarpWaitW(&full[stage], (q / kWStages) & 1, p.error,
                               kErrWeightWait)) {
        *aborted = 1;
        break;
      }
      if (!WarpWaitW(&dfull[t], (b / S::kSlots) & 1, p.error, kErrWeightWait)) {
        *aborted = 1;
        break;
      }
      TcFenceAfter();
      std::uint32_t d[32];
      TmemLoad<32>(tmem + lanes + S::kN * t + 32 * chunk, d);
      TcFenceBefore();
      __syncwarp();
      if (lane == 0)
        MbarArrive(&tfree[t]);
      const unsigned char* ws = smem + stage * S::kStageBytes + S::kXPartBytes;
      const std::uint16_t bits = *reinterpret_cast<const std::uint16_t*>(
          ws + (g * kWPartBlocks + j) * kQ8TileBytes + scale_offset);
      const float scale = live ? HalfBitsToFloat(bits) : 0.0f;
#pragma unroll
      for (int c = 0; c < 32; ++c)
        acc[c] = fmaf(scale, __uint_as_float(d[c]), acc[c]);
      // The last block of a part: its stage may be refilled.
      if (j == kWPartBlocks - 1 || b == nb - 1) {
        __syncwarp();
        if (lane == 0)
          MbarArrive(&empty[stage]);
      }
    }
  }

  // Every wait above is bounded, so every thread gets here.
  __syncthreads();
  TcFenceAfter();
  if (warp == S::kProducerWarp)
    TmemDealloc(tmem, kWColumns);

  // The cluster's splits add up in rank order.
  float* part = reinterpret_cast<float*>(smem);  // [128 rows][N]
  if (p.splits > 1) {
    if (reader && split != 0) {
#pragma unroll
      for (int c = 0; c < 32; c += 4)
        *reinterpret_cast<float4*>(part + row * S::kN + 32 * chunk + c) =
            make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
    }
    ClusterSync();
    if (reader && split == 0) {
      for (int rank = 1; rank < p.splits; ++rank) {
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
          const float4 v = LoadSharedCluster4(MapShared(
              part + row * S::kN + 32 * chunk + c, static_cast<unsigned>(rank)));
          acc[c] += v.x;
          acc[c + 1] += v.y;
          acc[c + 2] += v.z;
          acc[c + 3] += v.w;
        }
      }
    }
    ClusterSync();  // the others keep their shared memory until it was read
  }
  if (!reader || split != 0 || *aborted != 0)
    return;
  const int n = group0 * 16 + row;
  if (n >= p.n)
    return;
  if (p.accumulate && p.wait)
    GridDependencyWait();  // y may be the preceding kernel's output
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    const int m = 32 * chunk + c;
    if (m < p.m) {
      const std::size_t index = static_cast<std::size_t>(m) * p.n + n;
      float value = acc[c];
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

/// x [rows][in] bf16 with a box of 64 columns x N rows and the 128-byte
/// swizzle: each box lands as N 128-byte rows in 8-row swizzle atoms, the
/// MMA's K-major B layout (rows past the activation rows read as zero).
bool EncodeWideActivations(const std::uint16_t* x, std::size_t rows,
                           std::size_t in, int n, CUtensorMap* map) {
  const std::uint64_t dims[2] = {in, rows};
  const std::uint64_t strides[1] = {in * 2};
  const std::uint32_t box[2] = {64, static_cast<std::uint32_t>(n)};
  return EncodeBf16TensorMap(map, x, 2, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B);
}

bool g_wide = true;

}  // namespace

void SetWideTensorCoreProducts(bool enabled) { g_wide = enabled; }

bool WideProductPays(std::size_t rows, std::size_t in, std::size_t out) {
  // Measured on B200 against the mma.sync path at 33..128 rows over the
  // config-1 and DiT shapes: the wide kernel wins for more than 64 rows over
  // short reductions into many outputs (1024 -> 8192 at 88..128 rows: 18-22
  // against 48-52 us; 1024 -> 3072: 19-23 against 25-27 us), where the
  // mma.sync kernels' activation slice leaves few CTAs; elsewhere the
  // per-block read-back of its sums keeps it slower.
  return rows > 64 && rows <= static_cast<std::size_t>(kWideMaxRows) &&
         in <= 1024 && out >= 3072;
}
bool WideTensorCoreProducts() { return g_wide; }

ProductPlan PlanWideProduct(std::size_t rows, std::size_t in, std::size_t out,
                            int sms) {
  ProductPlan plan;
  if (rows < kWideMinRows || rows > kWideMaxRows || in == 0 ||
      in % kTileColumns != 0 || out == 0)
    return plan;
  const int k_blocks = static_cast<int>(in / kTileColumns);
  const int panels = static_cast<int>(((out + 15) / 16 + kWGroups - 1) / kWGroups);
  // About one CTA per SM; each split keeps at least one whole part.
  int splits = (sms + panels / 2) / std::max(panels, 1);
  splits = std::max(1, std::min({splits, 8, (k_blocks + kWPartBlocks - 1) / kWPartBlocks}));
  const int bps = (k_blocks + splits - 1) / splits;
  plan.variant = kTensorCoreWideVariant;
  plan.blocks_per_split = bps;
  plan.splits = (k_blocks + bps - 1) / bps;
  return plan;
}

int LaunchWideProduct(const std::uint16_t* x, const void* w, float* y,
                      std::uint16_t* y_bf16, std::size_t rows, std::size_t in,
                      std::size_t out, bool accumulate, const ProductPlan& plan,
                      cudaStream_t stream, bool independent, bool programmatic) {
  const int k_blocks = static_cast<int>(in / kTileColumns);
  if (rows < 1 || rows > kWideMaxRows || in % kTileColumns != 0 ||
      plan.splits < 1 || plan.splits > 8 || plan.blocks_per_split < 1 ||
      (k_blocks + plan.blocks_per_split - 1) / plan.blocks_per_split != plan.splits)
    return kUnsupported;
  const int chunks = rows <= 64 ? 2 : rows <= 96 ? 3 : 4;
  void (*kernel)(const WideArgs, const CUtensorMap) =
      chunks == 2 ? TcWideKernel<2> : chunks == 3 ? TcWideKernel<3> : TcWideKernel<4>;
  const int smem = chunks == 2 ? Wide<2>::kSmemBytes
                   : chunks == 3 ? Wide<3>::kSmemBytes
                                 : Wide<4>::kSmemBytes;
  const int threads = chunks == 2 ? Wide<2>::kThreads
                      : chunks == 3 ? Wide<3>::kThreads
                                    : Wide<4>::kThreads;
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
    bool& done = configured[device & 7][chunks - 2];
    if (!done) {
      if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               smem) != cudaSuccess)
        return kCudaError;
      done = true;
    }
    if (words[device & 7] == nullptr)
      words[device & 7] = DeviceErrorWord();
    error_word = words[device & 7];
  }
  if (error_word == nullptr)
    return kCudaError;
  WideArgs args;
  args.w = static_cast<const unsigned char*>(w);
  args.y = y;
  args.y_bf16 = y != nullptr ? nullptr : y_bf16;
  args.m = static_cast<int>(rows);
  args.n = static_cast<int>(out);
  args.k_blocks = k_blocks;
  args.splits = plan.splits;
  args.blocks_per_split = plan.blocks_per_split;
  args.accumulate = accumulate ? 1 : 0;
  args.wait = independent ? 0 : 1;
  args.error = error_word;
  const int panels = static_cast<int>(((out + 15) / 16 + kWGroups - 1) / kWGroups);
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(static_cast<unsigned>(panels * plan.splits));
  config.blockDim = dim3(static_cast<unsigned>(threads));
  config.dynamicSmemBytes = static_cast<std::size_t>(smem);
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
  if (!EncodeWideActivations(x, rows, in, 32 * chunks, &x_map))
    return kInvalid;
  if (cudaLaunchKernelEx(&config, kernel, args, x_map) != cudaSuccess)
    return kCudaError;
  return kOk;
}

}  // namespace vx
