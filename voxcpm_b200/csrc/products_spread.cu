// Spread products: one wave of CTAs over a product's whole weight stream.
//
// The product's work is the grid of units (panel, block): a panel is 128
// weight rows (eight 16-row groups, one per warp), a block is 32 columns of
// the reduction. The units are numbered panel-major and cut into one
// contiguous run per CTA, at most one SM's worth of CTAs, so every SM streams
// the same number of weight bytes (within one unit) whatever the shape: no
// CTA waits on a partly filled last wave, and no cluster has to find free SM
// pairs. A run is at most one panel's reduction long, so it touches at most
// two panels: the end of one and the start of the next.
//
// A panel whose reduction lies in one CTA is written by that CTA. A panel cut
// between CTAs is added up as the reference's split-K products do
// (kernels/wmma_products.hip:136-138, 249-295): every part stores its fp32
// partial sums in the caller's scratch and counts itself in on the panel's
// counter; the CTA that counts last adds all parts in part order (so the sum
// never depends on which CTA finished last) and resets the counter to zero for
// the next launch. Nothing spins: no CTA waits for another.
//
// Measured on B200 in dependent chains (one launch waiting for the one
// before), it is slower than the whole-reduction plans of products.cu for
// nearly every shape: the CTA that counts in last pays two more trips
// through L2 (its partial loads after the counter), and every CTA waits for
// its activations after the previous kernel. It is therefore opt-in
// (SetSpreadProducts, or an explicit plan with split scratch).
//
// Everything else is the skinny product's machinery (products.cu): 1-D TMA
// bulk copies of each warp's weight runs into a ring of stages, exact Q8_0
// dequantization into mma.sync m16n8k16 tiles with per-block fp32 sums scaled
// into the accumulator (kernels/wmma_products.hip:201-209), activations in
// shared memory, and programmatic dependent launch: a CTA issues its first
// weight stages before it waits for the previous kernel, so consecutive
// products keep HBM busy across kernel boundaries. The scratch, the counters,
// the activations and the output are touched only after that wait.
#include "product_math.cuh"
#include "products.cuh"
#include "vx_common.cuh"

#include <algorithm>
#include <atomic>
#include <mutex>

namespace vx {

namespace {

constexpr int kSpreadWarps = 8;  // warps per CTA: one 16-row group each
constexpr int kPanelGroups = kSpreadWarps;
constexpr int kPanelRows = kPanelGroups * kTileRows;  // 128
constexpr int kSpreadDepth = 2;   // ring stages per warp
constexpr int kMinUnitsPerCta = 4;
/// Dynamic shared memory a spread CTA may take. Most shapes need less than
/// half an SM's, so the next launch's CTAs fit beside this one's and start
/// streaming their weights while it computes.
constexpr std::size_t kSpreadSmemLimit = 220 * 1024;
/// Floats of scratch per (CTA, end of its run): every warp's accumulators of
/// up to four 8-row activation tiles.
constexpr int kSlotFloats = kSpreadWarps * 32 * 4 * 4;

__host__ __device__ constexpr int SpreadStage(int format) {
  // Blocks per stage: 4.3 KB Q8 runs; 4 KB bf16 runs.
  return format == static_cast<int>(WeightFormat::kQ8Tiles) ? 8 : 4;
}

__host__ __device__ constexpr int SpreadRowStride(int stage) {
  return stage * 64 + ((stage % 2 == 0) ? 64 : 0);
}

__host__ __device__ constexpr int SpreadGroupBytes(int format, int stage) {
  return format == static_cast<int>(WeightFormat::kQ8Tiles)
             ? stage * kQ8TileBytes
             : (format == static_cast<int>(WeightFormat::kBf16Tiles)
                    ? stage * kBf16TileBytes
                    : 16 * SpreadRowStride(stage));
}

inline int SpreadXStride(int columns) {
  const int bytes = columns * 2;
  return (bytes % 128 == 64) ? bytes : (bytes + 127) / 128 * 128 + 64;
}

struct SpreadArgs {
  const Bf16* x;
  const unsigned char* w;
  float* y;
  Bf16* y_bf16;
  float* partials;
  unsigned* counters;
  unsigned* error_word;  // the library's device error word
  int m;
  int k;
  int n;
  int k_blocks;
  int groups_total;
  int units;  // panels * k_blocks
  int ctas;
  int accumulate;
  int x_stride;
  int ring_bytes;  // one warp's ring
  int wait;
};

/// Most units of one product (so that the run arithmetic below stays in 32
/// bits: CTAs x units < 2^32).
constexpr int kSpreadMaxUnits = 1 << 22;

/// First unit of CTA `c`'s run.
__host__ __device__ inline int RunStart(int c, int units, int ctas) {
  return static_cast<int>(static_cast<unsigned>(c) *
                          static_cast<unsigned>(units) /
                          static_cast<unsigned>(ctas));
}

/// The CTA whose run holds unit `u`.
__device__ inline int RunOf(int u, int units, int ctas) {
  return static_cast<int>((static_cast<unsigned>(u + 1) *
                               static_cast<unsigned>(ctas) +
                           static_cast<unsigned>(units) - 1u) /
                          static_cast<unsigned>(units)) -
         1;
}

/// Adds `v` to the counter at device scope with acquire-release order: the
/// CTA's writes before its barrier are published with the add, and the
/// writes of every part counted in before are visible after it.
__device__ inline unsigned AddAcqRel(unsigned* counter, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(counter), "r"(v)
               : "memory");
  return old;
}

template <int kFormat, int kNTiles>
__global__ void __launch_bounds__(kSpreadWarps * 32)
    SpreadProductKernel(const SpreadArgs p) {
  constexpr int kStage = SpreadStage(kFormat);
  constexpr int kGroupBytes = SpreadGroupBytes(kFormat, kStage);
  constexpr bool kQ8 = kFormat == static_cast<int>(WeightFormat::kQ8Tiles);
  constexpr bool kRows = kFormat == static_cast<int>(WeightFormat::kBf16);
  constexpr int kTileBytes = kQ8 ? kQ8TileBytes : kBf16TileBytes;
  constexpr int kRowStride = SpreadRowStride(kStage);

  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int last_part[2];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int gid = lane >> 2;
  const int tig = lane & 3;
  const int cta = static_cast<int>(blockIdx.x);
  const int kb = p.k_blocks;
  const int u0 = RunStart(cta, p.units, p.ctas);
  const int u1 = RunStart(cta + 1, p.units, p.ctas);
  const int run = u1 - u0;
  // The run's (at most two) segments: panel, first block, length.
  const int panel0 = u0 / kb;
  const int b0 = u0 - panel0 * kb;
  const int len0 = min(run, kb - b0);
  const int len1 = run - len0;
  const int panel1 = panel0 + 1;
  const int stages0 = (len0 + kStage - 1) / kStage;
  const int stages = stages0 + (len1 + kStage - 1) / kStage;
  const int x_rows = kNTiles * 8;

  unsigned char* xs = smem;
  unsigned char* rings = smem + ((x_rows * p.x_stride + 127) / 128) * 128;
  std::uint64_t* bars =
      reinterpret_cast<std::uint64_t*>(rings + kSpreadWarps * p.ring_bytes);
  std::uint64_t* xbar = bars + kSpreadWarps * kSpreadDepth;
  unsigned char* ring = rings + warp * p.ring_bytes;
  std::uint64_t* full = bars + warp * kSpreadDepth;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSpreadWarps * kSpreadDepth + 1; ++i)
      MbarInit(&bars[i], 1);
    FenceMbarInit();
  }
  {
    uint4* pad = reinterpret_cast<uint4*>(xs + p.m * p.x_stride);
    const int count = (x_rows - p.m) * p.x_stride / 16;
    for (int i = threadIdx.x; i < count; i += blockDim.x)
      pad[i] = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();

  // Stage i: segment, first block within the panel, blocks, first unit of
  // the run (its column in the activation slice / 32), and this warp's
  // group (or -1 when the panel has no group for this warp).
  auto stage_of = [&](int i, int& block, int& nb, int& unit, int& group) {
    if (i < stages0) {
      block = b0 + i * kStage;
      nb = min(kStage, b0 + len0 - block);
      unit = block - b0;
      group = panel0 * kPanelGroups + warp;
    } else {
      block = (i - stages0) * kStage;
      nb = min(kStage, len1 - block);
      unit = len0 + block;
      group = panel1 * kPanelGroups + warp;
    }
    if (group >= p.groups_total)
      group = -1;
  };

  const std::uint64_t evict_first = PolicyEvictFirst();
  auto issue = [&](int i) {
    int block, nb, unit, group;
    stage_of(i, block, nb, unit, group);
    const int slot = i % kSpreadDepth;
    std::uint64_t* bar = &full[slot];
    unsigned char* dst = ring + slot * kGroupBytes;
    if (group < 0) {
      // No weights for this warp here: complete the phase at once so the
      // ring's phases stay in step with the stage numbers.
      if (lane == 0)
        MbarArrive(bar);
      return;
    }
    if constexpr (!kRows) {
      if (lane == 0) {
        MbarArriveExpectTx(bar, nb * kTileBytes);
        const unsigned char* src =
            p.w + (static_cast<std::size_t>(group) * kb + block) * kTileBytes;
        BulkLoad(dst, src, nb * kTileBytes, bar, evict_first);
      }
    } else {
      const int valid = min(16, p.n - group * 16);
      if (lane == 0)
        MbarArriveExpectTx(bar, valid * nb * 64);
      __syncwarp();
      if (lane < valid) {
        const unsigned char* src =
            p.w + (static_cast<std::size_t>(group * 16 + lane) * p.k +
                   block * 32) *
                      2;
        BulkLoad(dst + lane * kRowStride, src, nb * 64, bar, evict_first);
      }
    }
  };

  int issued = 0;
  for (; issued < min(kSpreadDepth, stages); ++issued)
    issue(issued);
  // Weights never depend on earlier kernels; activations, output, scratch
  // and counters may be in use by the previous launch until it completes.
  GridLaunchDependents();
  if (p.wait)
    GridDependencyWait();
  if (warp == 0 && run > 0) {
    if (lane == 0)
      MbarArriveExpectTx(xbar, p.m * run * 64);
    __syncwarp();
    for (int row = lane; row < p.m; row += 32) {
      const Bf16* src = p.x + static_cast<std::size_t>(row) * p.k;
      unsigned char* dst = xs + row * p.x_stride;
      BulkLoad(dst, src + b0 * 32, len0 * 64, xbar, PolicyEvictLast());
      if (len1 > 0)
        BulkLoad(dst + len0 * 64, src, len1 * 64, xbar, PolicyEvictLast());
    }
  }

  float acc[1][kNTiles][4];
  auto clear = [&]() {
#pragma unroll
    for (int j = 0; j < kNTiles; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c)
        acc[0][j][c] = 0.0f;
  };
  clear();

  // Writes the accumulators of `group` to the output (a panel held whole).
  auto store_output = [&](int group, const float (&v)[kNTiles][4]) {
#pragma unroll
    for (int j = 0; j < kNTiles; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int n = group * 16 + gid + 8 * (c >> 1);
        const int m = 8 * j + 2 * tig + (c & 1);
        if (m < p.m && n < p.n) {
          const std::size_t index = static_cast<std::size_t>(m) * p.n + n;
          float value = v[j][c];
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
  };
  auto slot_of = [&](int c, int end) {
    return reinterpret_cast<float4*>(
        p.partials +
        (static_cast<std::size_t>(c) * 2 + end) * kSlotFloats +
        static_cast<std::size_t>(warp) * (32 * 4 * kNTiles));
  };
  // Ends a segment: a whole panel goes to the output, a part to scratch.
  auto finish_segment = [&](int end, int group, bool whole) {
    if (group >= 0) {
      if (whole) {
        store_output(group, acc[0]);
      } else {
        float4* slot = slot_of(cta, end);
#pragma unroll
        for (int j = 0; j < kNTiles; ++j)
          slot[j * 32 + lane] =
              make_float4(acc[0][j][0], acc[0][j][1], acc[0][j][2],
                          acc[0][j][3]);
      }
    }
    clear();
  };
  const bool whole0 = b0 == 0 && len0 == kb;
  const bool whole1 = len1 == kb;

  bool failed = false;
  int waited = 0;
  if (run > 0 &&
      !MbarWaitBounded(xbar, 0, p.error_word, kErrActivationWait))
    failed = true;
  for (int i = 0; i < stages && !failed; ++i) {
    const int slot = i % kSpreadDepth;
    if (!MbarWaitBounded(&full[slot], (i / kSpreadDepth) & 1,
                         p.error_word, kErrWeightWait)) {
      failed = true;
      break;
    }
    ++waited;
    int block, nb, unit, group;
    stage_of(i, block, nb, unit, group);
    if (group >= 0) {
      const unsigned char* base = ring + slot * kGroupBytes;
      auto one = [&](int b) {
        uint4 frag[kNTiles];
        const int column = (unit + b) * 32 + 8 * tig;
#pragma unroll
        for (int j = 0; j < kNTiles; ++j)
          frag[j] = *reinterpret_cast<const uint4*>(
              xs + (8 * j + gid) * p.x_stride + column * 2);
        BlockProduct<kFormat, kNTiles, kRowStride>(base, b, gid, tig, frag,
                                                   acc[0]);
      };
      if (nb == kStage) {
#pragma unroll
        for (int b = 0; b < kStage; ++b)
          one(b);
      } else {
#pragma unroll 1
        for (int b = 0; b < nb; ++b)
          one(b);
      }
    }
    __syncwarp();
    if (issued < stages) {
      issue(issued);
      ++issued;
    }
    if (i == stages0 - 1)
      finish_segment(0, group, whole0);
  }
  if (failed) {
    for (int i = waited; i < issued; ++i)
      (void)MbarWaitBounded(&full[i % kSpreadDepth], (i / kSpreadDepth) & 1,
                            p.error_word, kErrDrainWait, 100000000ull);
  } else if (len1 > 0) {
    const int group1 = panel1 * kPanelGroups + warp;
    finish_segment(1, group1 < p.groups_total ? group1 : -1, whole1);
  }

  // Parts of split panels: count in, and the last part adds them all. The
  // barrier orders every warp's partial stores before thread 0's
  // acquire-release add, which publishes them at device scope.
  const bool split0 = run > 0 && !whole0;
  const bool split1 = len1 > 0 && !whole1;
  if (!split0 && !split1)
    return;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int end = 0; end < 2; ++end) {
      const bool split = end == 0 ? split0 : split1;
      const int panel = end == 0 ? panel0 : panel1;
      last_part[end] = 0;
      if (!split)
        continue;
      const int first = RunOf(panel * kb, p.units, p.ctas);
      const int last = RunOf(panel * kb + kb - 1, p.units, p.ctas);
      const unsigned parts = static_cast<unsigned>(last - first + 1);
      if (AddAcqRel(&p.counters[panel], 1u) == parts - 1) {
        last_part[end] = 1;
        p.counters[panel] = 0;  // ready for the next launch
      }
    }
  }
  __syncthreads();
  constexpr int kBatch = 4;  // parts whose partials are in flight at once
  for (int end = 0; end < 2; ++end) {
    if (!last_part[end])
      continue;
    const int panel = end == 0 ? panel0 : panel1;
    const int group = panel * kPanelGroups + warp;
    if (group >= p.groups_total)
      continue;
    const int first = RunOf(panel * kb, p.units, p.ctas);
    const int last = RunOf(panel * kb + kb - 1, p.units, p.ctas);
    float sum[kNTiles][4];
    for (int c0 = first; c0 <= last; c0 += kBatch) {
      float4 v[kBatch][kNTiles];
#pragma unroll
      for (int q = 0; q < kBatch; ++q) {
        const int c = c0 + q;
        if (c <= last) {
          // The part's end of its run: its first segment if the panel
          // starts there, else its second.
          const int part_end =
              RunStart(c, p.units, p.ctas) / kb == panel ? 0 : 1;
          const float4* slot = slot_of(c, part_end);
#pragma unroll
          for (int j = 0; j < kNTiles; ++j)
            v[q][j] = __ldcg(&slot[j * 32 + lane]);
        }
      }
      // Added in part order, whichever CTA counted in last.
#pragma unroll
      for (int q = 0; q < kBatch; ++q) {
        if (c0 + q > last)
          break;
#pragma unroll
        for (int j = 0; j < kNTiles; ++j) {
          if (c0 + q == first) {
            sum[j][0] = v[q][j].x;
            sum[j][1] = v[q][j].y;
            sum[j][2] = v[q][j].z;
            sum[j][3] = v[q][j].w;
          } else {
            sum[j][0] += v[q][j].x;
            sum[j][1] += v[q][j].y;
            sum[j][2] += v[q][j].z;
            sum[j][3] += v[q][j].w;
          }
        }
      }
    }
    store_output(group, sum);
  }
}

using SpreadFn = void (*)(const SpreadArgs);

template <int kFormat>
SpreadFn SpreadFor(int ntiles) {
  switch (ntiles) {
    case 1:
      return SpreadProductKernel<kFormat, 1>;
    case 2:
      return SpreadProductKernel<kFormat, 2>;
    case 3:
      return SpreadProductKernel<kFormat, 3>;
    default:
      return SpreadProductKernel<kFormat, 4>;
  }
}

SpreadFn SpreadKernelFor(int format, int ntiles) {
  switch (format) {
    case 0:
      return SpreadFor<0>(ntiles);
    case 1:
      return SpreadFor<1>(ntiles);
    default:
      return SpreadFor<2>(ntiles);
  }
}

struct SpreadShape {
  int ctas = 0;
  int run = 0;  // most units in one CTA's run
  int x_stride = 0;
  int ring_bytes = 0;
  std::size_t smem = 0;
};

SpreadShape ShapeOf(int format, std::size_t rows, std::size_t in,
                    std::size_t out, int sms) {
  SpreadShape s;
  const int k_blocks = static_cast<int>(in / kTileColumns);
  const int panels = static_cast<int>((out + kPanelRows - 1) / kPanelRows);
  const long long units = static_cast<long long>(panels) * k_blocks;
  if (units <= 0 || units > kSpreadMaxUnits)
    return s;
  // At least kMinUnitsPerCta units per CTA where there are few, and at
  // least one CTA per panel, so no run is longer than one panel's reduction.
  int ctas = static_cast<int>(
      std::min<long long>(sms, (units + kMinUnitsPerCta - 1) / kMinUnitsPerCta));
  ctas = std::max({ctas, panels, 1});
  if (ctas > sms || panels > kSpreadMaxPanels)
    return s;
  const int run = static_cast<int>((units + ctas - 1) / ctas);
  if (run > k_blocks)
    return s;
  const int ntiles = static_cast<int>((rows + 7) / 8);
  const int stage = SpreadStage(format);
  s.ctas = ctas;
  s.run = run;
  s.x_stride = SpreadXStride(run * kTileColumns);
  s.ring_bytes = kSpreadDepth * SpreadGroupBytes(format, stage);
  s.smem = (static_cast<std::size_t>(ntiles) * 8 * s.x_stride + 127) / 128 *
               128 +
           static_cast<std::size_t>(kSpreadWarps) * s.ring_bytes +
           (kSpreadWarps * kSpreadDepth + 1) * 8;
  if (s.smem > kSpreadSmemLimit)
    return SpreadShape();
  return s;
}

int Sms() {
  static int count = [] {
    int device = 0;
    int sms = 148;
    if (cudaGetDevice(&device) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    return sms;
  }();
  return count;
}

std::atomic<bool> g_spread{false};

}  // namespace

void SetSpreadProducts(bool enabled) { g_spread = enabled; }
bool SpreadProducts() { return g_spread; }

bool SpreadProductPays(WeightFormat format, std::size_t rows, std::size_t in,
                       std::size_t out) {
  if (!g_spread || rows == 0 || rows > kSpreadMaxRows)
    return false;
  return SpreadScratchNeeds(format, rows, in, out).ok;
}

SpreadNeeds SpreadScratchNeeds(WeightFormat format, std::size_t rows,
                               std::size_t in, std::size_t out) {
  SpreadNeeds needs;
  if (rows == 0 || rows > kSpreadMaxRows || in == 0 || out == 0 ||
      in % kTileColumns != 0)
    return needs;
  const SpreadShape s = ShapeOf(static_cast<int>(format), rows, in, out, Sms());
  if (s.ctas == 0)
    return needs;
  needs.ok = true;
  needs.ctas = s.ctas;
  needs.run = s.run;
  needs.partial_floats = static_cast<std::size_t>(s.ctas) * 2 * kSlotFloats;
  needs.counters = (out + kPanelRows - 1) / kPanelRows;
  return needs;
}

std::size_t SpreadScratchFloatsFor(int ctas) {
  return static_cast<std::size_t>(ctas) * 2 * kSlotFloats;
}

int MaxSpreadCtas() { return Sms(); }

int LaunchSpreadProduct(WeightFormat format, const std::uint16_t* x,
                        const void* w, float* y, std::uint16_t* y_bf16,
                        std::size_t rows, std::size_t in, std::size_t out,
                        bool accumulate, const SplitScratch& scratch,
                        cudaStream_t stream, bool independent,
                        bool programmatic) {
  const SpreadNeeds needs = SpreadScratchNeeds(format, rows, in, out);
  if (!needs.ok)
    return kUnsupported;
  if (scratch.partials == nullptr || scratch.counters == nullptr ||
      scratch.partial_floats < needs.partial_floats ||
      scratch.counter_count < needs.counters)
    return kInvalid;
  if (reinterpret_cast<std::uintptr_t>(scratch.partials) % 16 != 0)
    return kInvalid;
  const int f = static_cast<int>(format);
  const SpreadShape s = ShapeOf(f, rows, in, out, Sms());
  const int ntiles = static_cast<int>((rows + 7) / 8);
  SpreadFn kernel = SpreadKernelFor(f, ntiles);
  {
    static std::mutex mutex;
    static bool configured[64][3][4] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64)
      return kCudaError;
    std::lock_guard<std::mutex> lock(mutex);
    bool& done = configured[device][f][ntiles - 1];
    if (!done) {
      // All of the SM's on-chip memory as shared memory, so two CTAs (this
      // launch's and the next's) fit side by side.
      if (cudaFuncSetAttribute(kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kSpreadSmemLimit)) !=
              cudaSuccess ||
          cudaFuncSetAttribute(kernel,
                               cudaFuncAttributePreferredSharedMemoryCarveout,
                               100) != cudaSuccess)
        return kCudaError;
      done = true;
    }
  }
  SpreadArgs a;
  a.x = x;
  a.w = static_cast<const unsigned char*>(w);
  a.y = y;
  a.y_bf16 = y != nullptr ? nullptr : y_bf16;
  a.partials = scratch.partials;
  a.counters = scratch.counters;
  a.error_word = DeviceErrorWord();
  if (a.error_word == nullptr)
    return kCudaError;
  a.m = static_cast<int>(rows);
  a.k = static_cast<int>(in);
  a.n = static_cast<int>(out);
  a.k_blocks = static_cast<int>(in / kTileColumns);
  a.groups_total = static_cast<int>((out + 15) / 16);
  a.units = static_cast<int>((out + kPanelRows - 1) / kPanelRows) * a.k_blocks;
  a.ctas = s.ctas;
  a.accumulate = accumulate ? 1 : 0;
  a.x_stride = s.x_stride;
  a.ring_bytes = s.ring_bytes;
  a.wait = independent ? 0 : 1;

  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(static_cast<unsigned>(s.ctas));
  config.blockDim = dim3(kSpreadWarps * 32);
  config.dynamicSmemBytes = s.smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  config.numAttrs = 0;
  if (programmatic) {
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
  }
  if (cudaLaunchKernelEx(&config, kernel, a) != cudaSuccess)
    return kCudaError;
  return kOk;
}

}  // namespace vx
