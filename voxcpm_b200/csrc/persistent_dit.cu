// The persistent DiT patch kernel (see persistent_dit.cuh).
//
// Arithmetic follows the per-kernel path it replaces, operation by
// operation (kernels/generator_kernels.hip:91-360 for the norms, RoPE,
// attention, SwiGLU, biases and the CFG-Zero* update; transformer.cpp:55-100
// for the layer order): bf16 roundings sit at the same points, products
// accumulate in fp32 per 32-column block with the Q8 scale applied per
// block. Only float summation orders differ (products split over warps and
// CTAs, two-pass softmax), so results agree with the per-kernel path to
// float32 rounding noise, and are bit-for-bit repeatable run to run.
#include "persistent_dit.cuh"

#include <cmath>
#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>

#include "persistent_common.cuh"
#include "product_math.cuh"
#include "vx_common.cuh"
#include "vx_status.h"

namespace vx {
namespace {

using Shape = DitShape;

constexpr int kChunk = 1024;                        // reduction columns per unit
constexpr int kUnitTiles = kChunk / kTileColumns;   // 32 tiles per unit
constexpr int kQkvWidth =
    (Shape::kHeads + 2 * Shape::kKvHeads) * Shape::kHeadDim;  // 2560
constexpr int kAttWidth = Shape::kHeads * Shape::kHeadDim;    // 2048
constexpr int kRows = Shape::kRows;                           // 22
constexpr int kSeq = Shape::kSequence;                        // 11
constexpr int kHidden = Shape::kHidden;
constexpr int kInter = Shape::kIntermediate;
constexpr int kThreads = kConsumers + 64;  // + producer and publisher warps
constexpr int kXRows = 8;                  // staged rows of the patch boundary
constexpr int kXStride = kChunk * 2 + 64;  // bytes per staged row (bank skew)
constexpr int kOParts = kAttWidth / kChunk;   // 2
constexpr int kDownParts = kInter / kChunk;   // 4
constexpr int kDitInSlots = (kHidden / 16) * (Shape::kFeat / 32) / kUnitTiles;
constexpr int kDitOutSlots = Shape::kFeat / 16;
constexpr int kKvGroups = 2 * Shape::kKvHeads * Shape::kHeadDim / 16;  // 32
constexpr int kHeadGroups = Shape::kHeadDim / 16;                       // 8
constexpr int kHeadsPerKv = Shape::kHeads / Shape::kKvHeads;            // 8
constexpr int kHeadsPerChunk = kChunk / Shape::kHeadDim;                // 8
constexpr int kAttentionTasks = 2 * Shape::kHeads;  // (head, sequence)
constexpr int kGuPerChunk = kChunk / 16;            // 64
constexpr int kGroups = kHidden / 16;               // 64

// Sync words (zeroed per launch), all monotone over the launch: the abort
// flag; per query head the count of its q groups done, per KV head the
// count of its k and v groups; per 1024-column chunk of the attention
// output the count of (head, sequence) tasks done; the count of residual
// groups folded; the count of assembled evaluations; per chunk of the
// SwiGLU activation the count of gate/up units done. One thread per CTA
// polls a counter, so the polling load on L2 stays small.
constexpr int kSyncNever = 8;       // set by no CTA (the stall test hook)
constexpr int kSyncQ = 32;          // [16]
constexpr int kSyncKv = 48;         // [2]
constexpr int kSyncAtt = 64;        // [2]
constexpr int kSyncHidden = 96;
constexpr int kSyncAssembled = 97;
constexpr int kSyncAct = 128;       // [4]

// O and down groups belong to a CTA pair (a cluster of two): rank r takes
// O part r and down parts r and r + 2; rank 1 sends its reduced parts to
// rank 0 through distributed shared memory, and rank 0 folds.
constexpr int kPairParts = kDownParts / 2;

static_assert(kHidden == kChunk, "QKV and gate/up reduce over one chunk");
static_assert(2 * Shape::kPatch <= kXRows, "the boundary stages the output rows");
static_assert(kSyncAct + kDownParts <= kDitSyncWords, "act counters");
static_assert(kOParts == 2 && kDownParts == 4, "pair split");
static_assert(kSyncQ + Shape::kHeads <= kSyncKv, "head counters");
static_assert(Shape::kHeadDim == 128, "attention lanes hold 4 of 128");
static_assert(kConsumerWarps * 64 == kChunk, "a warp owns 64 columns");
static_assert(2 * Shape::kPatch <= 8, "DiT outputs fit one column tile");
static_assert(kDitInSlots * kUnitTiles == (kHidden / 16) * (Shape::kFeat / 32),
              "dit_in tiles fill whole slots");
static_assert(kRows == 22 && kHidden == 1024, "fragment layouts");

enum Phase : int { kQkv = 0, kO = 1, kGu = 2, kDown = 3 };

__host__ __device__ constexpr int PhaseUnits(int phase) {
  return phase == kQkv  ? kQkvWidth / 16
         : phase == kO  ? kGroups * kOParts
         : phase == kGu ? kInter / 16
                        : kGroups * kDownParts;
}
__host__ __device__ constexpr int SlotsPerUnit(int phase) {
  return phase == kGu ? 2 : 1;  // gate group and up group
}
/// QKV units take the key and value groups first.
__host__ __device__ constexpr int QkvGroup(int u) {
  return u < kKvGroups ? kAttWidth / 16 + u : u - kKvGroups;
}

template <int kFormat>
struct RingShape {
  static constexpr bool kQ8 =
      kFormat == static_cast<int>(WeightFormat::kQ8Tiles);
  static constexpr int kTile = kQ8 ? kQ8TileBytes : kBf16TileBytes;
  static constexpr int kSlots = kQ8 ? 8 : 4;
  static constexpr int kSlotBytes = kTile * kUnitTiles;
  static constexpr int kXsOffset = kSlots * kSlotBytes;
  static constexpr int kRedOffset = kXsOffset + kXRows * kXStride;
  // red[2][16 warps][384]: gate/up units reduce both slots at once.
  static constexpr int kVelOffset =
      kRedOffset + 2 * kConsumerWarps * kRedFloats * 4;
  static constexpr int kSumsOffset =
      kVelOffset + 2 * Shape::kPatch * Shape::kFeat * 4;
  // sums: [22][16] per-warp row partials, [22] inverse norms, scratch.
  static constexpr int kPubOffset = kSumsOffset + 512 * 4;
  static constexpr int kRecvOffset = kPubOffset + kPubSlots * 16;
  static constexpr int kBarOffset = kRecvOffset + kPairParts * kRedFloats * 4;
  // full[kSlots], empty[kSlots], pub_full[8], pub_empty[8], recv, done
  static constexpr int kFlagOffset =
      kBarOffset + (2 * (kSlots + kPubSlots) + 2) * 8;
  static constexpr int kSmemBytes = kFlagOffset + 16;
  static_assert(kSlotBytes % 128 == 0 && kXsOffset % 128 == 0, "alignment");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
  // Attention keys and values of one (head, sequence) use the first
  // reduction buffer.
  static_assert(2 * kSeq * Shape::kHeadDim * 4 <= kConsumerWarps * kRedFloats * 4,
                "attention staging");
};

__device__ inline int FirstUnit(int cta, int ctas, int base) {
  return (cta - base + ctas) % ctas;
}

/// Source of one slot: unit `u` of `phase` (`which`: gate 0 / up 1).
template <int kTile>
__device__ inline const unsigned char* SlotSource(const DitLayer& layer,
                                                  int phase, int u,
                                                  int which) {
  std::size_t tile;
  const unsigned char* base;
  switch (phase) {
    case kQkv:
      base = layer.qkv;
      tile = static_cast<std::size_t>(QkvGroup(u)) * kUnitTiles;
      break;
    case kO:
      base = layer.o;
      tile = static_cast<std::size_t>(u / kOParts) * (kAttWidth / 32) +
             (u % kOParts) * kUnitTiles;
      break;
    case kGu:
      base = layer.gate_up;
      tile = static_cast<std::size_t>(u + which * (kInter / 16)) * kUnitTiles;
      break;
    default:
      base = layer.down;
      tile = static_cast<std::size_t>(u / kDownParts) * (kInter / 32) +
             (u % kDownParts) * kUnitTiles;
      break;
  }
  return base + tile * kTile;
}

/// `kTiles` consecutive tiles from `kb0` of a 32-tile slot against the
/// staged rows; the accumulators go to red[warp].
template <int kFormat, int kNTiles, int kTiles>
__device__ __forceinline__ void SlotProduct(const unsigned char* slot,
                                            int kb0, const unsigned char* xs,
                                            int warp, int lane, float* red) {
  const int gid = lane >> 2;
  const int tig = lane & 3;
  float acc[kNTiles][4];
#pragma unroll
  for (int j = 0; j < kNTiles; ++j)
    acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
#pragma unroll
  for (int t = 0; t < kTiles; ++t) {
    const int kb = kb0 + t;
    uint4 b[kNTiles];
#pragma unroll
    for (int j = 0; j < kNTiles; ++j)
      b[j] = *reinterpret_cast<const uint4*>(xs + (8 * j + gid) * kXStride +
                                             (kb * 32 + 8 * tig) * 2);
    BlockProduct<kFormat, kNTiles, 0>(slot, kb, gid, tig, b, acc);
  }
  float* out = red + warp * (32 * kNTiles * 4) + lane * (kNTiles * 4);
#pragma unroll
  for (int j = 0; j < kNTiles; ++j)
    *reinterpret_cast<float4*>(out + 4 * j) =
        make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
}

/// bf16(w * x * rsqrt(mean(x^2) + eps)) of one 1024-wide row into a staged
/// row (kernels/generator_kernels.hip:91-108); one warp.
__device__ inline void StageNormRow(const float* src, const Bf16* weight,
                                    float eps, unsigned char* dst, int lane) {
  float4 v[8];
  uint2 wb[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    v[k] = __ldcg(reinterpret_cast<const float4*>(src) + lane + 32 * k);
    wb[k] = __ldg(reinterpret_cast<const uint2*>(weight) + lane + 32 * k);
  }
  float sum = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k)
    sum += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z +
           v[k].w * v[k].w;
  sum = WarpAllSum(sum);
  const float inverse = rsqrtf(sum / static_cast<float>(kHidden) + eps);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int i = 4 * (lane + 32 * k);
    const float o0 = v[k].x * inverse * Bf16ToFloat(static_cast<Bf16>(wb[k].x & 0xFFFFu));
    const float o1 = v[k].y * inverse * Bf16ToFloat(static_cast<Bf16>(wb[k].x >> 16));
    const float o2 = v[k].z * inverse * Bf16ToFloat(static_cast<Bf16>(wb[k].y & 0xFFFFu));
    const float o3 = v[k].w * inverse * Bf16ToFloat(static_cast<Bf16>(wb[k].y >> 16));
    *reinterpret_cast<uint2*>(dst + i * 2) = PackBf16x4(o0, o1, o2, o3);
  }
}

/// B fragments of this warp's two tiles (reduction columns column0 + 64w ..
/// + 63) for three column tiles of 8 rows: lane (gid, tig) holds, for tile
/// t and column tile j, the 8 columns 32t + 8tig .. of row 8j + gid.
using Fragments = uint4[2][3];

/// Fragments from bf16 rows [22][ld] (rows 22, 23 zero).
__device__ inline void BfFragments(const Bf16* src, int ld, int column0,
                                   int warp, int lane, Fragments& b) {
  const int gid = lane >> 2;
  const int tig = lane & 3;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int row = 8 * j + gid;
#pragma unroll
    for (int t = 0; t < 2; ++t)
      b[t][j] = row < kRows
                    ? __ldcg(reinterpret_cast<const uint4*>(
                          src + static_cast<std::size_t>(row) * ld + column0 +
                          64 * warp + 32 * t + 8 * tig))
                    : make_uint4(0u, 0u, 0u, 0u);
  }
}

/// Fragments of bf16(w * x * rsqrt(mean(x^2) + eps)) of the fp32 rows
/// `hidden` [22][1024] (kernels/generator_kernels.hip:91-108): each warp
/// loads its 64 columns, row sums go through `sums` ([22][16] warp partials
/// summed in warp order, then [22] inverse norms), one CTA barrier each.
/// `weight`: this lane's 16 norm weights (two runs of 8 columns).
__device__ void NormFragments(const float* hidden, const uint4 (&weight)[2],
                              float eps, float* sums, int tid, int warp,
                              int lane, Fragments& b) {
  const int gid = lane >> 2;
  const int tig = lane & 3;
  float4 v[3][2][2];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int row = 8 * j + gid;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float* src = hidden + static_cast<std::size_t>(row) * kHidden +
                         64 * warp + 32 * t + 8 * tig;
      v[j][t][0] = row < kRows ? __ldcg(reinterpret_cast<const float4*>(src))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
      v[j][t][1] = row < kRows ? __ldcg(reinterpret_cast<const float4*>(src) + 1)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    float s = 0.0f;
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        s += v[j][t][h].x * v[j][t][h].x + v[j][t][h].y * v[j][t][h].y +
             v[j][t][h].z * v[j][t][h].z + v[j][t][h].w * v[j][t][h].w;
    s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);
    s += __shfl_xor_sync(0xFFFFFFFFu, s, 2);
    const int row = 8 * j + gid;
    if (tig == 0 && row < kRows)
      sums[row * kConsumerWarps + warp] = s;
  }
  ConsumerSync();
  float* inverse = sums + kRows * kConsumerWarps;
  if (tid < kRows) {
    float total = sums[tid * kConsumerWarps];
#pragma unroll
    for (int w = 1; w < kConsumerWarps; ++w)
      total += sums[tid * kConsumerWarps + w];
    inverse[tid] = rsqrtf(total / static_cast<float>(kHidden) + eps);
  }
  ConsumerSync();
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int row = 8 * j + gid;
    const float r = row < kRows ? inverse[row] : 0.0f;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const uint4 w = weight[t];
      const float4 lo = v[j][t][0];
      const float4 hi = v[j][t][1];
      b[t][j].x = PackBf16x2(lo.x * r * Bf16ToFloat(static_cast<Bf16>(w.x & 0xFFFFu)),
                             lo.y * r * Bf16ToFloat(static_cast<Bf16>(w.x >> 16)));
      b[t][j].y = PackBf16x2(lo.z * r * Bf16ToFloat(static_cast<Bf16>(w.y & 0xFFFFu)),
                             lo.w * r * Bf16ToFloat(static_cast<Bf16>(w.y >> 16)));
      b[t][j].z = PackBf16x2(hi.x * r * Bf16ToFloat(static_cast<Bf16>(w.z & 0xFFFFu)),
                             hi.y * r * Bf16ToFloat(static_cast<Bf16>(w.z >> 16)));
      b[t][j].w = PackBf16x2(hi.z * r * Bf16ToFloat(static_cast<Bf16>(w.w & 0xFFFFu)),
                             hi.w * r * Bf16ToFloat(static_cast<Bf16>(w.w >> 16)));
    }
  }
}

/// This warp's two tiles (2w, 2w + 1) of a 32-tile slot against its
/// fragments; the accumulators go to red[warp].
template <int kFormat>
__device__ __forceinline__ void FragProduct(const unsigned char* slot,
                                            const Fragments& b, int warp,
                                            int lane, float* red) {
  const int gid = lane >> 2;
  const int tig = lane & 3;
  float acc[3][4];
#pragma unroll
  for (int j = 0; j < 3; ++j)
    acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const uint4 bt[3] = {b[t][0], b[t][1], b[t][2]};
    BlockProduct<kFormat, 3, 0>(slot, 2 * warp + t, gid, tig, bt, acc);
  }
  float* out = red + warp * kRedFloats + lane * 12;
#pragma unroll
  for (int j = 0; j < 3; ++j)
    *reinterpret_cast<float4*>(out + 4 * j) =
        make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
}

/// Attention of one (query head, CFG sequence): RoPE on q and k at
/// positions 0..10, keys/values rounded as the cache stores them, scale
/// 1/sqrt(128), non-causal over the sequence's 11 rows, bf16 output
/// (kernels/generator_kernels.hip:110-241). Keys and values are staged in
/// `kv` ([2][11][128] fp32); warp w < 11 takes query row w.
__device__ void AttentionTask(const DitPatchParams& p, int head, int sequence,
                              float* kv, int tid, int warp, int lane) {
  constexpr int kD = Shape::kHeadDim;
  constexpr int kHalf = kD / 2;
  const int kv_head = head / kHeadsPerKv;
  const float* rows = p.qkv + static_cast<std::size_t>(sequence) * kSeq * kQkvWidth;
  float* ks = kv;
  float* vs = kv + kSeq * kD;
  // Everything this thread reads, in flight at once: its warp's query row
  // with its rotary factors, its share of key pairs (with factors) and of
  // values.
  const bool has_query = warp < kSeq;
  float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 qc = q, qs = q;
  if (has_query) {
    q = __ldcg(reinterpret_cast<const float4*>(rows + warp * kQkvWidth + head * kD) + lane);
    if (p.rope != nullptr) {
      const int d = 4 * (lane & 15);
      qc = *reinterpret_cast<const float4*>(p.rope + warp * kD + d);
      qs = *reinterpret_cast<const float4*>(p.rope + warp * kD + kHalf + d);
    }
  }
  constexpr int kPairs = kSeq * kHalf;   // 704
  constexpr int kValues = kSeq * kD;     // 1408
  constexpr int kPerThread = (kPairs + kValues + kConsumers - 1) / kConsumers;
  float a[kPerThread], b[kPerThread], cs[kPerThread], sn[kPerThread];
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) {
    const int i = tid + k * kConsumers;
    cs[k] = 1.0f;
    sn[k] = 0.0f;
    if (i < kPairs) {
      const int row = i / kHalf;
      const int d = i % kHalf;
      const float* src = rows + row * kQkvWidth + kAttWidth + kv_head * kD + d;
      a[k] = __ldcg(src);
      b[k] = __ldcg(src + kHalf);
      if (p.rope != nullptr) {
        cs[k] = p.rope[row * kD + d];
        sn[k] = p.rope[row * kD + kHalf + d];
      }
    } else if (i < kPairs + kValues) {
      const int j = i - kPairs;
      a[k] = __ldcg(rows + (j / kD) * kQkvWidth + kAttWidth +
                    (Shape::kKvHeads + kv_head) * kD + j % kD);
    }
  }
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) {
    const int i = tid + k * kConsumers;
    if (i < kPairs) {
      const int row = i / kHalf;
      const int d = i % kHalf;
      float first = a[k];
      float second = b[k];
      if (p.rope != nullptr) {
        first = a[k] * cs[k] - b[k] * sn[k];
        second = b[k] * cs[k] + a[k] * sn[k];
      }
      if (p.bf16_kv) {
        first = RoundBf16(first);
        second = RoundBf16(second);
      }
      ks[row * kD + d] = first;
      ks[row * kD + kHalf + d] = second;
    } else if (i < kPairs + kValues) {
      vs[i - kPairs] = p.bf16_kv ? RoundBf16(a[k]) : a[k];
    }
  }
  // The query: lane l holds dims 4l..4l+3; its RoPE partner dims are in
  // lane l ^ 16 (first = a c - b s below 64, second = b c + a s above).
  if (has_query && p.rope != nullptr) {
    const float4 partner = make_float4(__shfl_xor_sync(0xFFFFFFFFu, q.x, 16),
                                       __shfl_xor_sync(0xFFFFFFFFu, q.y, 16),
                                       __shfl_xor_sync(0xFFFFFFFFu, q.z, 16),
                                       __shfl_xor_sync(0xFFFFFFFFu, q.w, 16));
    if (lane < 16)
      q = make_float4(q.x * qc.x - partner.x * qs.x, q.y * qc.y - partner.y * qs.y,
                      q.z * qc.z - partner.z * qs.z, q.w * qc.w - partner.w * qs.w);
    else
      q = make_float4(q.x * qc.x + partner.x * qs.x, q.y * qc.y + partner.y * qs.y,
                      q.z * qc.z + partner.z * qs.z, q.w * qc.w + partner.w * qs.w);
  }
  ConsumerSync();
  if (has_query) {
    q.x *= p.attention_scale;
    q.y *= p.attention_scale;
    q.z *= p.attention_scale;
    q.w *= p.attention_scale;
    float score[kSeq];
    float maximum = -INFINITY;
#pragma unroll
    for (int key = 0; key < kSeq; ++key) {
      const float4 k = reinterpret_cast<const float4*>(ks + key * kD)[lane];
      score[key] = WarpAllSum(q.x * k.x + q.y * k.y + q.z * k.z + q.w * k.w);
      maximum = fmaxf(maximum, score[key]);
    }
    float total = 0.0f;
    float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int key = 0; key < kSeq; ++key) {
      const float weight = expf(score[key] - maximum);
      const float4 v = reinterpret_cast<const float4*>(vs + key * kD)[lane];
      total += weight;
      out.x += weight * v.x;
      out.y += weight * v.y;
      out.z += weight * v.z;
      out.w += weight * v.w;
    }
    const float inverse = 1.0f / total;
    *reinterpret_cast<uint2*>(
        p.att + static_cast<std::size_t>(sequence * kSeq + warp) * kAttWidth +
        head * kD + lane * 4) =
        PackBf16x4(out.x * inverse, out.y * inverse, out.z * inverse,
                   out.w * inverse);
  }
  ConsumerSync();
}

// ---------------------------------------------------------------- producer

template <int kFormat>
__device__ void Produce(const DitPatchParams& p, unsigned char* ring,
                        std::uint64_t* full, std::uint64_t* empty,
                        const Control& c) {
  using R = RingShape<kFormat>;
  const std::uint64_t policy = PolicyEvictFirst();
  const int cta = static_cast<int>(blockIdx.x);
  const int ctas = static_cast<int>(gridDim.x);
  unsigned issued = 0;
  bool stop = false;
  auto issue = [&](const unsigned char* source) {
    if (stop)
      return;
    const unsigned slot = issued % R::kSlots;
    if (issued >= static_cast<unsigned>(R::kSlots) &&
        !WaitSlot(&empty[slot], ((issued / R::kSlots) - 1) & 1u, c,
                  kErrWeightWait)) {
      stop = true;
      return;
    }
    MbarArriveExpectTx(&full[slot], R::kSlotBytes);
    BulkLoad(ring + slot * R::kSlotBytes, source, R::kSlotBytes, &full[slot],
             policy);
    ++issued;
  };
  auto dit_in = [&]() {
    for (int s = 0; s < kDitInSlots; ++s)
      issue(p.dit_in + static_cast<std::size_t>(s) * R::kSlotBytes);
  };
  if (cta == 0)
    dit_in();
  const int pair = cta >> 1;
  const int rank = cta & 1;
  const int pairs = ctas >> 1;
  int base = 0;
  int pair_base = 0;
  for (int e = 0; e < p.evaluations && !stop; ++e) {
    for (int l = 0; l < p.layers && !stop; ++l) {
      const DitLayer layer = p.layer[l];
      for (int phase = kQkv; phase <= kDown; ++phase) {
        if (phase == kO || phase == kDown) {
          for (int g = FirstUnit(pair, pairs, pair_base); g < kGroups; g += pairs) {
            if (phase == kO) {
              issue(SlotSource<R::kTile>(layer, kO, g * kOParts + rank, 0));
            } else {
              for (int k = 0; k < kPairParts; ++k)
                issue(SlotSource<R::kTile>(layer, kDown,
                                           g * kDownParts + rank + 2 * k, 0));
            }
          }
          pair_base = (pair_base + kGroups) % pairs;
          continue;
        }
        const int units = PhaseUnits(phase);
        for (int u = FirstUnit(cta, ctas, base); u < units; u += ctas)
          for (int which = 0; which < SlotsPerUnit(phase); ++which)
            issue(SlotSource<R::kTile>(layer, phase, u, which));
        base = (base + units) % ctas;
      }
    }
    if (cta == 0) {
      for (int g = 0; g < kDitOutSlots; ++g)
        issue(p.dit_out + static_cast<std::size_t>(g) * R::kSlotBytes);
      if (e + 1 < p.evaluations)
        dit_in();
    }
  }
  // Every copy this warp started lands before the CTA may exit.
  const unsigned first =
      issued > static_cast<unsigned>(R::kSlots) ? issued - R::kSlots : 0u;
  for (unsigned k = first; k < issued; ++k)
    (void)MbarWaitBounded(&full[k % R::kSlots], (k / R::kSlots) & 1u,
                          c.error_word, kErrDrainWait);
}

// ---------------------------------------------------------------- consumers

template <int kFormat>
__device__ void Consume(const DitPatchParams& p, unsigned char* smem,
                        const Control& c) {
  using R = RingShape<kFormat>;
  unsigned char* ring = smem;
  unsigned char* xs = smem + R::kXsOffset;
  float* red = reinterpret_cast<float*>(smem + R::kRedOffset);
  float* vel = reinterpret_cast<float*>(smem + R::kVelOffset);
  float* sums = reinterpret_cast<float*>(smem + R::kSumsOffset);
  PubEntry* entries = reinterpret_cast<PubEntry*>(smem + R::kPubOffset);
  std::uint64_t* full = reinterpret_cast<std::uint64_t*>(smem + R::kBarOffset);
  std::uint64_t* empty = full + R::kSlots;
  std::uint64_t* pub_full = empty + R::kSlots;
  std::uint64_t* pub_empty = pub_full + kPubSlots;
  std::uint64_t* recv_bar = pub_empty + kPubSlots;
  float* recv = reinterpret_cast<float*>(smem + R::kRecvOffset);
  const int tid = static_cast<int>(threadIdx.x);
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int gid = lane >> 2;
  const int tig = lane & 3;
  const int cta = static_cast<int>(blockIdx.x);
  const int ctas = static_cast<int>(gridDim.x);
  const int pair = cta >> 1;
  const int rank = cta & 1;
  const int pairs = ctas >> 1;
  unsigned* sync = p.sync;
  unsigned consumed = 0;
  unsigned published = 0;
  unsigned folds = 0;  // pair folds this CTA took part in
  // The peer's receive buffer and barrier (rank 1 sends to rank 0).
  const std::uint32_t peer_recv = MapShared(recv, rank ^ 1);
  const std::uint32_t peer_recv_bar = MapShared(recv_bar, rank ^ 1);

  // Slot `consumed + ahead` of the ring, once it landed.
  auto acquire = [&](unsigned ahead = 0) -> const unsigned char* {
    const unsigned item = consumed + ahead;
    const unsigned slot = item % R::kSlots;
    if (*c.aborted == 0)
      (void)WaitSlot(&full[slot], (item / R::kSlots) & 1u, c, kErrWeightWait);
    return ring + slot * R::kSlotBytes;
  };
  // This warp is done with the next `count` slots.
  auto release = [&](unsigned count = 1) {
    __syncwarp();
    if (lane == 0)
      for (unsigned k = 0; k < count; ++k)
        MbarArrive(&empty[(consumed + k) % R::kSlots]);
    consumed += count;
  };
  // After a consumer barrier that follows the writes: queue a release-add
  // of `value` to `counter` for the publisher warp (null ends its loop).
  auto publish = [&](unsigned* counter, unsigned value) {
    if (tid == 0) {
      const unsigned slot = published % kPubSlots;
      if (published >= static_cast<unsigned>(kPubSlots))
        (void)WaitSlot(&pub_empty[slot], ((published / kPubSlots) - 1) & 1u, c,
                       kErrPublishWait);
      volatile PubEntry* entry = entries + slot;
      entry->counter = counter;
      entry->value = value;
      MbarArrive(&pub_full[slot]);
    }
    ++published;
  };
  // One product unit's reduced values: `store(feature, row, value)` for
  // rows < 22, then a consumer barrier.
  auto reduce_store = [&](auto&& store) {
    ConsumerSync();
    if (tid < kRedFloats) {
      int feature, row;
      Decode(tid, 3, feature, row);
      if (row < kRows)
        store(feature, row, Reduce(red, tid, kRedFloats));
    }
    ConsumerSync();
  };

  // dit_in(bf16(x)) + bias into the x rows of both sequences, then the
  // other rows [mu_a, mu_b, time, cond x4] (uncond: zero mu); publishes the
  // assembled evaluation (kernels/generator_kernels.hip:320-340;
  // generator.cpp:297-310).
  auto boundary_in = [&](int e) {
    for (int i = tid; i < 8 * Shape::kFeat; i += kConsumers) {
      const int r = i / Shape::kFeat;
      const int col = i % Shape::kFeat;
      const float v = r < Shape::kPatch ? __ldcg(p.x + r * Shape::kFeat + col) : 0.0f;
      *reinterpret_cast<Bf16*>(xs + r * kXStride + col * 2) = ToBf16(v);
    }
    ConsumerSync();
    for (int s = 0; s < kDitInSlots; ++s) {
      const unsigned char* slot = acquire();
      float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
      // Warp w: row group 16 s + w, its two tiles (the whole 64 columns).
#pragma unroll
      for (int kb = 0; kb < Shape::kFeat / 32; ++kb) {
        uint4 b[1];
        b[0] = *reinterpret_cast<const uint4*>(xs + gid * kXStride +
                                               (kb * 32 + 8 * tig) * 2);
        BlockProduct<kFormat, 1, 0>(slot + warp * (Shape::kFeat / 32) * R::kTile,
                                    kb, gid, tig, b, acc);
      }
      release();
      const int group = s * kConsumerWarps + warp;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int row = 2 * tig + (q & 1);
        const int feature = group * 16 + gid + 8 * (q >> 1);
        if (row < Shape::kPatch) {
          const float v = acc[0][q] + Bf16ToFloat(p.dit_in_bias[feature]);
          const int x_row = 3 + Shape::kPatch + row;
          p.hidden[static_cast<std::size_t>(x_row) * kHidden + feature] = v;
          p.hidden[static_cast<std::size_t>(kSeq + x_row) * kHidden + feature] = v;
        }
      }
    }
    const float* time = p.time_vectors[e];
    constexpr int kFixed = 3 + Shape::kPatch;
    for (int i = tid; i < 2 * kFixed * kHidden; i += kConsumers) {
      const int sequence = i / (kFixed * kHidden);
      const int row = (i / kHidden) % kFixed;
      const int col = i % kHidden;
      float v;
      if (row < 2)
        v = sequence == 0 ? p.mu[row * kHidden + col] : 0.0f;
      else if (row == 2)
        v = time[col];
      else
        v = p.cond_rows[(row - 3) * kHidden + col];
      p.hidden[static_cast<std::size_t>(sequence * kSeq + row) * kHidden + col] = v;
    }
    ConsumerSync();
    publish(sync + kSyncAssembled, 1u);
  };

  // Final norm of the 2P output rows, dit_out + bias, CFG-Zero* Euler
  // update of x (kernels/generator_kernels.hip:342-360).
  auto boundary_out = [&](int e) {
    if (warp < 2 * Shape::kPatch) {
      const int k = warp;
      const int row = (k < Shape::kPatch ? 0 : kSeq - Shape::kPatch) + 3 +
                      Shape::kPatch + k;
      StageNormRow(p.hidden + static_cast<std::size_t>(row) * kHidden,
                   p.final_norm, p.eps, xs + k * kXStride, lane);
    }
    ConsumerSync();
    for (int g = 0; g < kDitOutSlots; ++g) {
      SlotProduct<kFormat, 1, 2>(acquire(), 2 * warp, xs, warp, lane, red);
      release();
      ConsumerSync();
      if (tid < 32 * 4) {
        int feature, row;
        Decode(tid, 1, feature, row);
        feature += g * 16;
        vel[row * Shape::kFeat + feature] =
            Reduce(red, tid, 32 * 4) + Bf16ToFloat(p.dit_out_bias[feature]);
      }
      ConsumerSync();
    }
    constexpr int kCount = Shape::kPatch * Shape::kFeat;  // 256
    float cv = 0.f, uv = 0.f;
    if (tid < kCount) {
      cv = vel[tid];
      uv = vel[kCount + tid];
      const float dot = WarpAllSum(cv * uv);
      const float norm = WarpAllSum(uv * uv);
      if (lane == 0) {
        sums[warp] = dot;
        sums[16 + warp] = norm;
      }
    }
    ConsumerSync();
    if (tid < kCount) {
      float dot = sums[0];
      float norm = sums[16];
      for (int w = 1; w < kCount / 32; ++w) {
        dot += sums[w];
        norm += sums[16 + w];
      }
      const float s = dot / (norm + 1e-8f);
      const float guided = uv * s + p.cfg * (cv - uv * s);
      p.x[tid] -= p.dts[e] * guided;
    }
    ConsumerSync();
  };

  // A pair's split product: rank 1 stores its reduced part `k` into rank
  // 0's receive buffer; rank 0 keeps its own in `keep`.
  auto reduce_part = [&](int k, float& keep) {
    ConsumerSync();
    if (tid < kRedFloats) {
      const float v = Reduce(red, tid, kRedFloats);
      if (rank == 1)
        StoreSharedCluster(peer_recv + static_cast<std::uint32_t>(
                                           (k * kRedFloats + tid) * 4), v);
      else
        keep = v;
    }
    ConsumerSync();
  };
  // Rank 1: signal rank 0. Rank 0: wait, then hidden[:, group] += the
  // parts in part order (kept ones at even parts, received ones at odd),
  // and publish one folded group.
  auto fold_pair = [&](int group, int parts, const float* keep) {
    if (rank == 1) {
      if (tid == 0)
        MbarArriveCluster(peer_recv_bar);
      ++folds;
      return true;
    }
    // This thread's residual value, loaded while the peer finishes.
    std::size_t at = 0;
    float h = 0.0f;
    bool mine = false;
    if (tid < kRedFloats) {
      int feature, row;
      Decode(tid, 3, feature, row);
      mine = row < kRows;
      at = static_cast<std::size_t>(row) * kHidden + group * 16 + feature;
      if (mine)
        h = __ldcg(p.hidden + at);
    }
    if (!WaitPeer(recv_bar, folds & 1u, c))
      return false;
    ++folds;
    if (mine) {
      float sum = keep[0] + recv[tid];  // parts 0 and 1
      if (parts == kDownParts) {
        sum += keep[1];                 // part 2
        sum += recv[kRedFloats + tid];  // part 3
      }
      p.hidden[at] = h + sum;
    }
    ConsumerSync();
    publish(sync + kSyncHidden, 1u);
    return true;
  };

  if (cta == 0)
    boundary_in(0);
  int base = 0;
  int pair_base = 0;
  float* red2 = red + kConsumerWarps * kRedFloats;  // second reduction buffer
  // Norm weights of this lane's 16 columns (two runs of 8).
  auto norm_weights = [&](const Bf16* weight, uint4 (&w)[2]) {
#pragma unroll
    for (int t = 0; t < 2; ++t)
      w[t] = __ldg(reinterpret_cast<const uint4*>(weight + 64 * warp + 32 * t +
                                                  8 * tig));
  };
  auto check = [&]() { return !ConsumerSyncOr(*c.aborted != 0); };
  Fragments frag;
  for (int e = 0; e < p.evaluations; ++e) {
    for (int l = 0; l < p.layers; ++l) {
      const DitLayer layer = p.layer[l];
      const unsigned index = static_cast<unsigned>(e * p.layers + l);
      // This layer's post norm and the next layer's input norm (or the
      // final norm) into L2 now, so the norm stages wait on L2, not HBM.
      PrefetchL2(layer.post_norm, kHidden * 2, tid);
      if (l + 1 < p.layers) {
        PrefetchL2(p.layer[l + 1].input_norm, kHidden * 2, tid);
      } else {
        PrefetchL2(p.final_norm, kHidden * 2, tid);
        PrefetchL2(p.layer[0].input_norm, kHidden * 2, tid);
      }

      // QKV: norm(hidden) x W_qkv -> qkv (fp32), then this CTA's attention
      // task when it has one.
      {
        const int units = PhaseUnits(kQkv);
        const int mine = FirstUnit(cta, ctas, base);
        if (mine < units) {
          uint4 w[2];
          norm_weights(layer.input_norm, w);
          const bool ready =
              l == 0 ? WaitCount(c, sync + kSyncAssembled, e + 1)
                     : WaitCount(c, sync + kSyncHidden, 2 * kGroups * index);
          if (!ready)
            return;
          NormFragments(p.hidden, w, p.eps, sums, tid, warp, lane, frag);
        }
        for (int u = mine; u < units; u += ctas) {
          const int group = QkvGroup(u);
          FragProduct<kFormat>(acquire(), frag, warp, lane, red);
          release();
          reduce_store([&](int feature, int row, float v) {
            p.qkv[static_cast<std::size_t>(row) * kQkvWidth + group * 16 + feature] = v;
          });
          const int q_groups = kAttWidth / 16;
          publish(group < q_groups
                      ? sync + kSyncQ + group / kHeadGroups
                      : sync + kSyncKv + ((group - q_groups) % (kKvGroups / 2)) / kHeadGroups,
                  1u);
        }
        if (!check())
          return;
        // Attention: 32 (head, sequence) tasks on CTAs holding one unit.
        const int task = mine - (units > ctas ? units - ctas : 0);
        if (mine < units && task >= 0 && task < kAttentionTasks) {
          const int head = task >> 1;
          const int sequence = task & 1;
          if (!WaitCount(c, sync + kSyncKv + head / kHeadsPerKv,
                         2 * kHeadGroups * (index + 1)) ||
              !WaitCount(c, sync + kSyncQ + head, kHeadGroups * (index + 1)))
            return;
          AttentionTask(p, head, sequence, red, tid, warp, lane);
          publish(sync + kSyncAtt + head / kHeadsPerChunk, 1u);
        }
        base = (base + units) % ctas;
      }

      // O: att x W_o, the two column chunks on the two CTAs of a pair,
      // folded into hidden by rank 0. Warp w's columns belong to head
      // 8 rank + w / 2.
      {
        for (int g = FirstUnit(pair, pairs, pair_base); g < kGroups; g += pairs) {
          if (!WaitCount(c, sync + kSyncAtt + rank,
                         2 * kHeadsPerChunk * (index + 1)))
            return;
          BfFragments(p.att, kAttWidth, rank * kChunk, warp, lane, frag);
          FragProduct<kFormat>(acquire(), frag, warp, lane, red);
          release();
          float keep[kPairParts] = {0.f, 0.f};
          reduce_part(0, keep[0]);
          if (!check() || !fold_pair(g, kOParts, keep))
            return;
        }
        pair_base = (pair_base + kGroups) % pairs;
      }

      // gate/up: norm(hidden) x W_gate, W_up -> bf16(silu(g) * u); all
      // warps take both slots.
      {
        const int units = PhaseUnits(kGu);
        const int mine = FirstUnit(cta, ctas, base);
        if (mine < units) {
          uint4 w[2];
          norm_weights(layer.post_norm, w);
          if (!WaitCount(c, sync + kSyncHidden, kGroups * (2 * index + 1)))
            return;
          NormFragments(p.hidden, w, p.eps, sums, tid, warp, lane, frag);
        }
        for (int u = mine; u < units; u += ctas) {
          FragProduct<kFormat>(acquire(0), frag, warp, lane, red);
          FragProduct<kFormat>(acquire(1), frag, warp, lane, red2);
          release(2);
          ConsumerSync();
          if (tid < kRedFloats) {
            int feature, row;
            Decode(tid, 3, feature, row);
            if (row < kRows) {
              const float g = Reduce(red, tid, kRedFloats);
              const float up = Reduce(red2, tid, kRedFloats);
              p.act[static_cast<std::size_t>(row) * kInter + u * 16 + feature] =
                  ToBf16(g / (1.0f + expf(-g)) * up);
            }
          }
          ConsumerSync();
          publish(sync + kSyncAct + u / kGuPerChunk, 1u);
        }
        if (!check())
          return;
        base = (base + units) % ctas;
      }

      // down: act x W_down over four column chunks, parts r and r + 2 on
      // rank r of a pair, folded into hidden by rank 0. Warp w's columns of
      // chunk c come from gate/up units 64 c + 4 w .. + 3.
      {
        for (int g = FirstUnit(pair, pairs, pair_base); g < kGroups; g += pairs) {
          float keep[kPairParts] = {0.f, 0.f};
          if (!WaitCount(c, sync + kSyncAct + rank, kGuPerChunk * (index + 1)) ||
              !WaitCount(c, sync + kSyncAct + rank + 2, kGuPerChunk * (index + 1)))
            return;
          Fragments frag2;
          BfFragments(p.act, kInter, rank * kChunk, warp, lane, frag);
          BfFragments(p.act, kInter, (rank + 2) * kChunk, warp, lane, frag2);
          FragProduct<kFormat>(acquire(), frag, warp, lane, red);
          release();
          reduce_part(0, keep[0]);
          FragProduct<kFormat>(acquire(), frag2, warp, lane, red);
          release();
          reduce_part(1, keep[1]);
          if (!check() || !fold_pair(g, kDownParts, keep))
            return;
        }
        pair_base = (pair_base + kGroups) % pairs;
      }
    }
    if (cta == 0) {
      // Every residual group folded by the last layer's down.
      if (!WaitCount(c, sync + kSyncHidden,
                     2 * kGroups * static_cast<unsigned>((e + 1) * p.layers)))
        return;
      boundary_out(e);
      if (e + 1 < p.evaluations)
        boundary_in(e + 1);
    }
  }
  publish(nullptr, 0u);
}

template <int kFormat>
__global__ void __launch_bounds__(kThreads, 1)
    DitPatchKernel(const DitPatchParams p, unsigned* error_word) {
  using R = RingShape<kFormat>;
  extern __shared__ __align__(128) unsigned char smem[];
  std::uint64_t* full = reinterpret_cast<std::uint64_t*>(smem + R::kBarOffset);
  std::uint64_t* empty = full + R::kSlots;
  std::uint64_t* pub_full = empty + R::kSlots;
  std::uint64_t* pub_empty = pub_full + kPubSlots;
  volatile int* aborted = reinterpret_cast<volatile int*>(smem + R::kFlagOffset);
  const Control c{p.sync, error_word, aborted};
  if (threadIdx.x == 0) {
    for (int s = 0; s < R::kSlots; ++s) {
      MbarInit(&full[s], 1);
      MbarInit(&empty[s], kConsumerWarps);
    }
    for (int s = 0; s < kPubSlots; ++s) {
      MbarInit(&pub_full[s], 1);
      MbarInit(&pub_empty[s], 1);
    }
    MbarInit(pub_empty + kPubSlots, 1);      // recv: one arrival per fold
    MbarInit(pub_empty + kPubSlots + 1, 1);  // done: the peer's teardown
    *aborted = 0;
    FenceMbarInit();
  }
  // Staged rows start at zero; rows 22 and 23 stay zero for the whole patch.
  uint4* xs = reinterpret_cast<uint4*>(smem + R::kXsOffset);
  for (int i = threadIdx.x; i < kXRows * kXStride / 16; i += kThreads)
    xs[i] = make_uint4(0u, 0u, 0u, 0u);
  // Both CTAs of the pair see each other's initialized barriers.
  ClusterSync();
  if (threadIdx.x >= kConsumers) {
    if (threadIdx.x == kConsumers)
      Produce<kFormat>(p, smem, full, empty, c);
    else if (threadIdx.x == kConsumers + 32)
      Publish(reinterpret_cast<PubEntry*>(smem + R::kPubOffset), pub_full,
              pub_empty, c);
    return;
  }
  if (p.stall_limit_ns != 0 && blockIdx.x == 0 && threadIdx.x == 0) {
    // The test hook: a bounded wait that runs out, then the abort every
    // other wait of the launch watches for.
    const std::uint64_t start = GlobalTimerNs();
    while (LoadAcquire(p.sync + kSyncNever) == 0u) {
      if (GlobalTimerNs() - start > p.stall_limit_ns) {
        Abort(c, kErrBarrierWait);
        break;
      }
    }
  }
  Consume<kFormat>(p, smem, c);
  // Teardown: neither CTA of the pair exits while its peer may still write
  // into its shared memory. Each signals the other, then waits (bounded)
  // for the peer's signal.
  if (threadIdx.x == 0) {
    std::uint64_t* done = pub_empty + kPubSlots + 1;
    MbarArriveCluster(MapShared(done, (blockIdx.x & 1) ^ 1));
    const std::uint64_t start = GlobalTimerNs();
    while (!MbarTryWaitCluster(done, 0, kSuspendNs))
      if (GlobalTimerNs() - start > kWaitLimitNs) {
        atomicOr(error_word, kErrPeerWait);
        break;
      }
  }
}

constexpr std::size_t Align256(std::size_t n) { return (n + 255) & ~std::size_t{255}; }

struct DeviceState {
  bool probed = false;
  bool configured[2] = {false, false};
  int ctas[2] = {0, 0};  // CTAs of the launch (two per co-resident cluster)
};

}  // namespace

std::size_t DitWorkBytes() {
  return Align256(kRows * kHidden * 4) + Align256(kRows * kQkvWidth * 4) +
         Align256(kRows * kAttWidth * 2) + Align256(kRows * kInter * 2) +
         Align256(kDitSyncWords * 4);
}

void DitWorkLayout(void* base, DitPatchParams& params) {
  auto* at = static_cast<unsigned char*>(base);
  auto take = [&](std::size_t bytes) {
    unsigned char* p = at;
    at += Align256(bytes);
    return p;
  };
  params.hidden = reinterpret_cast<float*>(take(kRows * kHidden * 4));
  params.qkv = reinterpret_cast<float*>(take(kRows * kQkvWidth * 4));
  params.att = reinterpret_cast<std::uint16_t*>(take(kRows * kAttWidth * 2));
  params.act = reinterpret_cast<std::uint16_t*>(take(kRows * kInter * 2));
  params.sync = reinterpret_cast<unsigned*>(take(kDitSyncWords * 4));
}

namespace {

void (*DitKernel(bool q8))(const DitPatchParams, unsigned*) {
  return q8 ? DitPatchKernel<static_cast<int>(WeightFormat::kQ8Tiles)>
            : DitPatchKernel<static_cast<int>(WeightFormat::kBf16Tiles)>;
}

int DitSmem(bool q8) {
  return q8 ? RingShape<static_cast<int>(WeightFormat::kQ8Tiles)>::kSmemBytes
            : RingShape<static_cast<int>(WeightFormat::kBf16Tiles)>::kSmemBytes;
}

cudaLaunchConfig_t DitConfig(bool q8, unsigned ctas, cudaStream_t stream,
                             cudaLaunchAttribute (&attribute)[2]) {
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(ctas);
  config.blockDim = dim3(kThreads);
  config.dynamicSmemBytes = static_cast<std::size_t>(DitSmem(q8));
  config.stream = stream;
  attribute[0].id = cudaLaunchAttributeClusterDimension;
  attribute[0].val.clusterDim.x = 2;
  attribute[0].val.clusterDim.y = 1;
  attribute[0].val.clusterDim.z = 1;
  attribute[1].id = cudaLaunchAttributeCooperative;
  attribute[1].val.cooperative = 1;
  config.attrs = attribute;
  config.numAttrs = 2;
  return config;
}

/// CTAs of a launch on the current device (0 when it cannot run: no
/// cooperative launch, or fewer co-resident CTA pairs than residual groups).
int DitCtas(bool q8) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64)
    return 0;
  static std::mutex mutex;
  static DeviceState states[64];
  std::lock_guard<std::mutex> lock(mutex);
  DeviceState& state = states[device];
  const int which = q8 ? 0 : 1;
  if (!state.configured[which]) {
    state.configured[which] = true;
    int cooperative = 0;
    if (cudaDeviceGetAttribute(&cooperative, cudaDevAttrCooperativeLaunch,
                               device) != cudaSuccess ||
        cooperative == 0)
      return 0;
    if (cudaFuncSetAttribute(DitKernel(q8),
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DitSmem(q8)) != cudaSuccess)
      return 0;
    cudaLaunchAttribute attribute[2];
    cudaLaunchConfig_t config = DitConfig(q8, 2, nullptr, attribute);
    config.numAttrs = 1;  // the occupancy query takes the cluster shape only
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, DitKernel(q8), &config) !=
        cudaSuccess)
      return 0;
    state.ctas[which] = clusters >= kGroups ? 2 * clusters : 0;
  }
  const int cap = PersistentMaxCtas();
  if (cap > 0 && state.ctas[which] > 0)
    return std::min(state.ctas[which], std::max(cap / 2 * 2, 2 * kGroups));
  return state.ctas[which];
}

}  // namespace

bool DitPatchSupported(WeightFormat format) {
  if (format != WeightFormat::kQ8Tiles && format != WeightFormat::kBf16Tiles)
    return false;
  const bool ok = DitCtas(format == WeightFormat::kQ8Tiles) > 0;
  (void)cudaGetLastError();  // a failed query leaves no sticky error behind
  return ok;
}

// ---------------------------------------------------------------- static scratch

namespace {

/// The work buffers of the allocation-free patch live in this fixed device
/// array instead of memory the caller allocated. One array per process and
/// device: launches that overlap on the GPU share it and race.
constexpr std::size_t kDitStaticScratchBytes = std::size_t{1} << 20;
static __device__ __align__(256) unsigned char g_dit_static_scratch[kDitStaticScratchBytes];

/// The static array's device address on the current device, looked up once
/// per device (with that device current) on the first call there.
int StaticScratchAddress(void** scratch) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64)
    return Fail(kCudaError, "allocation-free DiT patch: no current device");
  static std::mutex mutex;
  static void* addresses[64] = {};
  std::lock_guard<std::mutex> lock(mutex);
  if (addresses[device] == nullptr) {
    void* address = nullptr;
    const cudaError_t error =
        cudaGetSymbolAddress(&address, g_dit_static_scratch);
    if (error != cudaSuccess || address == nullptr)
      return Fail(kCudaError,
                  std::string("allocation-free DiT patch: static scratch "
                              "address: ") +
                      cudaGetErrorString(error));
    addresses[device] = address;
  }
  *scratch = addresses[device];
  return kOk;
}

std::atomic<std::uint64_t> g_dit_stall_ns{0};

}  // namespace

void SetDitStall(std::uint64_t limit_ns) { g_dit_stall_ns = limit_ns; }

namespace {
std::atomic<int> g_persistent_max_ctas{0};
std::atomic<bool> g_persistent_cooperative{true};
}  // namespace

void SetPersistentMaxCtas(int ctas) { g_persistent_max_ctas = ctas > 0 ? ctas : 0; }
int PersistentMaxCtas() { return g_persistent_max_ctas; }
void SetPersistentCooperative(bool enabled) { g_persistent_cooperative = enabled; }
bool PersistentCooperative() { return g_persistent_cooperative; }

int DitLaunchAborted(const DitPatchParams& params, cudaStream_t stream,
                     bool* aborted) {
  *aborted = false;
  if (params.sync == nullptr)
    return kOk;
  unsigned word = 0;
  if (cudaMemcpyAsync(&word, params.sync + kSyncAbort, sizeof(word),
                      cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return Fail(kCudaError, "persistent DiT: reading the abort word");
  if (word != 0) {
    *aborted = true;
    if (cudaMemsetAsync(params.sync + kSyncAbort, 0, sizeof(unsigned),
                        stream) != cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess)
      return Fail(kCudaError, "persistent DiT: clearing the abort word");
  }
  return kOk;
}

int DitStaticLaunchAborted(cudaStream_t stream, bool* aborted) {
  *aborted = false;
  void* scratch = nullptr;
  const int status = StaticScratchAddress(&scratch);
  if (status != kOk)
    return status;
  DitPatchParams p;
  DitWorkLayout(scratch, p);
  return DitLaunchAborted(p, stream, aborted);
}

int LaunchDitPatchStatic(const DitPatchParams& base, cudaStream_t stream) {
  if (DitWorkBytes() > kDitStaticScratchBytes)
    return Fail(kInvalid,
                "allocation-free DiT patch: the work buffers need " +
                    std::to_string(DitWorkBytes()) + " bytes, more than the " +
                    std::to_string(kDitStaticScratchBytes) +
                    "-byte static scratch");
  void* scratch = nullptr;
  const int status = StaticScratchAddress(&scratch);
  if (status != kOk)
    return status;
  DitPatchParams p = base;
  DitWorkLayout(scratch, p);  // the sync words are zeroed by LaunchDitPatch
  return LaunchDitPatch(p, stream);
}

int LaunchDitPatch(const DitPatchParams& p, cudaStream_t stream) {
  const bool q8 = p.format == WeightFormat::kQ8Tiles;
  if (!q8 && p.format != WeightFormat::kBf16Tiles)
    return Fail(kInvalid, "persistent DiT: weights must be Q8 or bf16 tiles");
  if (p.layers < 1 || p.evaluations < 1 || p.layer == nullptr ||
      p.final_norm == nullptr || p.dit_in == nullptr ||
      p.dit_in_bias == nullptr || p.dit_out == nullptr ||
      p.dit_out_bias == nullptr || p.mu == nullptr || p.cond_rows == nullptr ||
      p.time_vectors == nullptr || p.dts == nullptr || p.x == nullptr ||
      p.hidden == nullptr || p.qkv == nullptr || p.att == nullptr ||
      p.act == nullptr || p.sync == nullptr)
    return Fail(kInvalid, "persistent DiT: missing argument");
  const int ctas = DitCtas(q8);
  if (ctas == 0)
    return Fail(kUnsupported,
                "persistent DiT: the device cannot hold one CTA pair per "
                "residual group co-resident");
  unsigned* error_word = DeviceErrorWord();
  if (error_word == nullptr)
    return Fail(kCudaError, "persistent DiT: device error word");
  if (cudaMemsetAsync(p.sync, 0, kDitSyncWords * sizeof(unsigned), stream) !=
      cudaSuccess)
    return Fail(kCudaError, "persistent DiT: memset");
  cudaLaunchAttribute attribute[2];
  const cudaLaunchConfig_t config =
      DitConfig(q8, static_cast<unsigned>(ctas), stream, attribute);
  cudaLaunchConfig_t launch_config = config;
  if (!PersistentCooperative())
    launch_config.numAttrs = 1;  // the cluster shape only
  DitPatchParams launch = p;
  launch.stall_limit_ns = g_dit_stall_ns;
  return FromCuda(
      cudaLaunchKernelEx(&launch_config, DitKernel(q8), launch, error_word),
      "persistent DiT launch");
}

}  // namespace vx
