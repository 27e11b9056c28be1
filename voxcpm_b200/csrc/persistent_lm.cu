// The persistent one-row decoder stack (see persistent_lm.cuh).
//
// Arithmetic follows ForwardStack at one row operation by operation
// (transformer.cpp:55-100; kernels/generator_kernels.hip:91-254): RMSNorm to
// bf16, products with fp32 accumulation per 32-column block (the Q8 scale
// applied per block), RoPE on q and k at the row's position, keys and values
// rounded as the cache stores them, softmax attention over every cached row
// and the new one, bf16 attention output, residual adds in fp32, SwiGLU to
// bf16. Only float summation orders differ from the per-kernel path.
#include "persistent_lm.cuh"

#include <cmath>
#include <algorithm>
#include <mutex>
#include <string>

#include "persistent_common.cuh"
#include "product_math.cuh"
#include "vx_common.cuh"
#include "vx_status.h"

namespace vx {
namespace {

using Shape = LmShape;

constexpr int kChunk = 1024;                       // reduction columns per slot
constexpr int kUnitTiles = kChunk / kTileColumns;  // 32 tiles per slot
constexpr int kHidden = Shape::kHidden;
constexpr int kInter = Shape::kIntermediate;
constexpr int kD = Shape::kHeadDim;
constexpr int kHeads = Shape::kHeads;
constexpr int kKvHeads = Shape::kKvHeads;
constexpr int kQkvWidth = (kHeads + 2 * kKvHeads) * kD;  // 2560
constexpr int kAttWidth = kHeads * kD;                   // 2048
constexpr int kHiddenChunks = kHidden / kChunk;          // 2
constexpr int kInterChunks = kInter / kChunk;            // 6
constexpr int kQkvUnits = kQkvWidth / 16;                // 160
constexpr int kOUnits = kHidden / 16;                    // 128
constexpr int kGuUnits = kInter / 16;                    // 384
constexpr int kDownUnits = kHidden / 16;                 // 128
constexpr int kSplits = Shape::kKeySplits;               // 8
constexpr int kTasks = kHeads * kSplits;                 // 128
constexpr int kPartFloats = kD + 4;                      // o[128], max, sum
constexpr int kHeadsPerKv = kHeads / kKvHeads;           // 8
constexpr int kThreads = kConsumers + 64;  // + producer and publisher warps
constexpr int kTile = kQ8TileBytes;
constexpr int kSlots = 10;
constexpr int kSlotBytes = kTile * kUnitTiles;
constexpr int kRed1 = 32 * 4;  // one warp's accumulators, one column tile

// Sync words (zeroed per launch), monotone over the launch: the abort flag
// (word 0), QKV units done, attention tasks done, residual groups updated
// (O and down, 128 each per layer), gate/up units done.
constexpr int kSyncQkv = 8;
constexpr int kSyncAtt = 16;
constexpr int kSyncHidden = 24;
constexpr int kSyncAct = 32;

static_assert(kSyncAct < kLmSyncWords, "sync words");
static_assert(kConsumerWarps * 64 == kChunk, "a warp owns 64 columns per chunk");
static_assert(kD == 128, "attention lanes hold 4 of 128");
static_assert(kTasks <= 148, "one attention task per CTA");

// Shared memory: ring | red[2][16][128] | sums[64] | pub queue | barriers | flag
constexpr int kRedOffset = kSlots * kSlotBytes;
constexpr int kSumsOffset = kRedOffset + 2 * kConsumerWarps * kRed1 * 4;
constexpr int kPubOffset = kSumsOffset + 64 * 4;
constexpr int kBarOffset = kPubOffset + kPubSlots * 16;
constexpr int kFlagOffset = kBarOffset + 2 * (kSlots + kPubSlots) * 8;
constexpr int kSmemBytes = kFlagOffset + 16;
static_assert(kSmemBytes <= 227 * 1024, "shared memory");
static_assert(kRedOffset % 128 == 0, "alignment");
// Attention: per-warp partials (o[128], max, sum) in the reduction buffers.
static_assert(kConsumerWarps * kPartFloats <= 2 * kConsumerWarps * kRed1,
              "attention partials");
static_assert(kHeads * 32 == kConsumers, "a thread per 4 dims of the attention row");
static_assert(kAttWidth * 2 <= kConsumerWarps * kRed1 * 4, "attention row in red2");

enum Phase : int { kQkv = 0, kO = 1, kGu = 2, kDown = 3 };

__host__ __device__ constexpr int PhaseUnits(int phase) {
  return phase == kQkv ? kQkvUnits
         : phase == kO ? kOUnits
         : phase == kGu ? kGuUnits
                       : kDownUnits;
}
__host__ __device__ constexpr int PhaseSlots(int phase) {
  return phase == kQkv ? kHiddenChunks
         : phase == kO ? kAttWidth / kChunk
         : phase == kGu ? 2 * kHiddenChunks
                       : kInterChunks;
}

__device__ inline int FirstUnit(int cta, int ctas, int base) {
  return (cta - base + ctas) % ctas;
}

/// Source of slot `s` of unit `u` of `phase`.
__device__ inline const unsigned char* SlotSource(const LmLayer& layer,
                                                  int phase, int u, int s) {
  std::size_t tile;
  const unsigned char* base;
  switch (phase) {
    case kQkv:
      base = layer.qkv;
      tile = static_cast<std::size_t>(u) * (kHidden / 32) + s * kUnitTiles;
      break;
    case kO:
      base = layer.o;
      tile = static_cast<std::size_t>(u) * (kAttWidth / 32) + s * kUnitTiles;
      break;
    case kGu: {  // gate chunk 0, gate chunk 1, up chunk 0, up chunk 1
      base = layer.gate_up;
      const int group = u + (s / kHiddenChunks) * kGuUnits;
      tile = static_cast<std::size_t>(group) * (kHidden / 32) +
             (s % kHiddenChunks) * kUnitTiles;
      break;
    }
    default:
      base = layer.down;
      tile = static_cast<std::size_t>(u) * (kInter / 32) + s * kUnitTiles;
      break;
  }
  return base + tile * kTile;
}

/// One row's fragments: lanes 0..3 hold, for tile t, the 8 columns
/// 32 t + 8 lane of this warp's 64 (every other lane holds zeros).
using RowFragments = uint4[2];

/// This warp's two tiles of a slot against its fragments, accumulated.
__device__ __forceinline__ void RowProduct(const unsigned char* slot,
                                           const RowFragments& b, int warp,
                                           int lane, float (&acc)[1][4]) {
  const int gid = lane >> 2;
  const int tig = lane & 3;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const uint4 bt[1] = {b[t]};
    BlockProduct<static_cast<int>(WeightFormat::kQ8Tiles), 1, 0>(
        slot, 2 * warp + t, gid, tig, bt, acc);
  }
}

__device__ inline void StoreAcc(float* red, int warp, int lane,
                                const float (&acc)[1][4]) {
  *reinterpret_cast<float4*>(red + warp * kRed1 + lane * 4) =
      make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
}

/// Fragments of bf16(w * x * rsqrt(mean(x^2) + eps)) of the row `x`
/// [2048] for both hidden chunks (kernels/generator_kernels.hip:91-108).
/// `weight`: this lane's norm weights [chunk][tile] (lanes 0..3).
__device__ void NormRow(const float* x, const uint4 (&weight)[2][2], float eps,
                        float* sums, int tid, int warp, int lane,
                        RowFragments (&b)[2]) {
  float4 v[2][2][2];
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float* src = x + c * kChunk + 64 * warp + 32 * t + 8 * lane;
      v[c][t][0] = lane < 4 ? __ldcg(reinterpret_cast<const float4*>(src))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
      v[c][t][1] = lane < 4 ? __ldcg(reinterpret_cast<const float4*>(src) + 1)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  float s = 0.0f;
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        s += v[c][t][h].x * v[c][t][h].x + v[c][t][h].y * v[c][t][h].y +
             v[c][t][h].z * v[c][t][h].z + v[c][t][h].w * v[c][t][h].w;
  s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);
  s += __shfl_xor_sync(0xFFFFFFFFu, s, 2);
  if (lane == 0)
    sums[warp] = s;
  ConsumerSync();
  if (tid == 0) {
    float total = sums[0];
    for (int w = 1; w < kConsumerWarps; ++w)
      total += sums[w];
    sums[32] = rsqrtf(total / static_cast<float>(kHidden) + eps);
  }
  ConsumerSync();
  const float r = sums[32];
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const uint4 w = weight[c][t];
      const float4 lo = v[c][t][0];
      const float4 hi = v[c][t][1];
      b[c][t] = lane < 4
                    ? make_uint4(
                          PackBf16x2(lo.x * r * Bf16ToFloat(static_cast<Bf16>(w.x & 0xFFFFu)),
                                     lo.y * r * Bf16ToFloat(static_cast<Bf16>(w.x >> 16))),
                          PackBf16x2(lo.z * r * Bf16ToFloat(static_cast<Bf16>(w.y & 0xFFFFu)),
                                     lo.w * r * Bf16ToFloat(static_cast<Bf16>(w.y >> 16))),
                          PackBf16x2(hi.x * r * Bf16ToFloat(static_cast<Bf16>(w.z & 0xFFFFu)),
                                     hi.y * r * Bf16ToFloat(static_cast<Bf16>(w.z >> 16))),
                          PackBf16x2(hi.z * r * Bf16ToFloat(static_cast<Bf16>(w.w & 0xFFFFu)),
                                     hi.w * r * Bf16ToFloat(static_cast<Bf16>(w.w >> 16))))
                    : make_uint4(0u, 0u, 0u, 0u);
    }
}

/// A cache row's 4 dims of this lane as stored (fp32: float4, bf16: uint2).
template <typename CacheT>
struct CacheRaw;
template <>
struct CacheRaw<float> {
  using Type = float4;
  __device__ static Type Load(const void* base, std::size_t row, int lane) {
    return __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(base) +
                                                  row * kD) +
                  lane);
  }
  __device__ static float4 Widen(Type v) { return v; }
  __device__ static Type Narrow(float4 v) { return v; }
};
template <>
struct CacheRaw<Bf16> {
  using Type = uint2;
  __device__ static Type Load(const void* base, std::size_t row, int lane) {
    return __ldcg(reinterpret_cast<const uint2*>(static_cast<const Bf16*>(base) +
                                                 row * kD) +
                  lane);
  }
  __device__ static float4 Widen(Type v) {
    return make_float4(Bf16ToFloat(static_cast<Bf16>(v.x & 0xFFFFu)),
                       Bf16ToFloat(static_cast<Bf16>(v.x >> 16)),
                       Bf16ToFloat(static_cast<Bf16>(v.y & 0xFFFFu)),
                       Bf16ToFloat(static_cast<Bf16>(v.y >> 16)));
  }
  __device__ static Type Narrow(float4 v) { return PackBf16x4(v.x, v.y, v.z, v.w); }
};

/// RoPE of a 128-wide vector held 4 dims per lane: the pair of dim d < 64
/// is d + 64, held by lane ^ 16 (first = a c - b s, second = b c + a s).
__device__ inline float4 Rope(float4 x, const float* table, int lane) {
  const float4 partner = make_float4(__shfl_xor_sync(0xFFFFFFFFu, x.x, 16),
                                     __shfl_xor_sync(0xFFFFFFFFu, x.y, 16),
                                     __shfl_xor_sync(0xFFFFFFFFu, x.z, 16),
                                     __shfl_xor_sync(0xFFFFFFFFu, x.w, 16));
  const int d = 4 * (lane & 15);
  const float4 c = __ldg(reinterpret_cast<const float4*>(table + d));
  const float4 s = __ldg(reinterpret_cast<const float4*>(table + kD / 2 + d));
  if (lane < 16)
    return make_float4(x.x * c.x - partner.x * s.x, x.y * c.y - partner.y * s.y,
                       x.z * c.z - partner.z * s.z, x.w * c.w - partner.w * s.w);
  return make_float4(x.x * c.x + partner.x * s.x, x.y * c.y + partner.y * s.y,
                     x.z * c.z + partner.z * s.z, x.w * c.w + partner.w * s.w);
}

__device__ inline float4 RoundBf16x4(float4 v) {
  return make_float4(RoundBf16(v.x), RoundBf16(v.y), RoundBf16(v.z),
                     RoundBf16(v.w));
}

/// One attention task: query head `head` over key chunk `split` of the
/// `position` + 1 keys (every cached row and the new one), online softmax
/// (kernels/generator_kernels.hip:160-241). Warp w takes keys k0 + w,
/// + 16, ...; the warps' partials merge in warp order into
/// att_parts[head][split]. The task holding the new row of the first head
/// of a KV group appends the row's key (roped, rounded) and value.
template <typename CacheT>
__device__ void AttentionTask(const LmStackParams& p, const LmLayer& layer,
                              int head, int split, int position,
                              float* scratch, int tid, int warp, int lane) {
  const int kv = head / kHeadsPerKv;
  const int keys = position + 1;
  const int chunk = (keys + kSplits - 1) / kSplits;
  const int k0 = split * chunk;
  const int k1 = min(keys, k0 + chunk);
  const float* table =
      p.rope != nullptr ? p.rope + static_cast<std::size_t>(position) * kD : nullptr;
  float4 q = __ldcg(reinterpret_cast<const float4*>(p.qkv + head * kD) + lane);
  const bool has_new = k0 <= position && position < k1;
  float4 new_k = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 new_v = new_k;
  if (has_new) {
    new_k = __ldcg(reinterpret_cast<const float4*>(p.qkv + kAttWidth + kv * kD) + lane);
    new_v = __ldcg(reinterpret_cast<const float4*>(p.qkv + kAttWidth + (kKvHeads + kv) * kD) +
                   lane);
  }
  if (table != nullptr) {
    q = Rope(q, table, lane);
    if (has_new)
      new_k = Rope(new_k, table, lane);
  }
  if (p.bf16_kv && has_new) {
    new_k = RoundBf16x4(new_k);
    new_v = RoundBf16x4(new_v);
  }
  q.x *= p.attention_scale;
  q.y *= p.attention_scale;
  q.z *= p.attention_scale;
  q.w *= p.attention_scale;
  const std::size_t base = static_cast<std::size_t>(kv) * p.capacity;
  float maximum = -INFINITY;
  float sum = 0.0f;
  float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
  // This warp's keys k0 + warp, + 16, ... in batches whose rows are all in
  // flight before the first is used.
  using Raw = CacheRaw<CacheT>;
  constexpr int kBatch = sizeof(CacheT) == 2 ? 8 : 4;
  // The new row as stored (already rounded to the cache's type).
  const typename Raw::Type new_kr = Raw::Narrow(new_k);
  const typename Raw::Type new_vr = Raw::Narrow(new_v);
  for (int first = k0 + warp; first < k1; first += kBatch * kConsumerWarps) {
    typename Raw::Type kr[kBatch], vr[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int key = first + i * kConsumerWarps;
      if (key < k1 && key != position) {
        kr[i] = Raw::Load(layer.keys, base + key, lane);
        vr[i] = Raw::Load(layer.values, base + key, lane);
      } else {
        kr[i] = new_kr;
        vr[i] = new_vr;
      }
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      if (first + i * kConsumerWarps >= k1)
        break;
      const float4 ki = Raw::Widen(kr[i]);
      const float4 vi = Raw::Widen(vr[i]);
      const float score =
          WarpAllSum(q.x * ki.x + q.y * ki.y + q.z * ki.z + q.w * ki.w);
      const float next = fmaxf(maximum, score);
      const float decay = expf(maximum - next);
      const float weight = expf(score - next);
      sum = sum * decay + weight;
      out.x = out.x * decay + weight * vi.x;
      out.y = out.y * decay + weight * vi.y;
      out.z = out.z * decay + weight * vi.z;
      out.w = out.w * decay + weight * vi.w;
      maximum = next;
    }
  }
  float* mine = scratch + warp * kPartFloats;
  reinterpret_cast<float4*>(mine)[lane] = out;
  if (lane == 0) {
    mine[kD] = maximum;
    mine[kD + 1] = sum;
  }
  ConsumerSync();
  if (warp == 0) {
    float m = -INFINITY;
    for (int w = 0; w < kConsumerWarps; ++w)
      m = fmaxf(m, scratch[w * kPartFloats + kD]);
    float total = 0.0f;
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float mw = scratch[w * kPartFloats + kD];
      const float f = mw == -INFINITY ? 0.0f : expf(mw - m);
      total += scratch[w * kPartFloats + kD + 1] * f;
      const float4 o = reinterpret_cast<const float4*>(scratch + w * kPartFloats)[lane];
      r.x += o.x * f;
      r.y += o.y * f;
      r.z += o.z * f;
      r.w += o.w * f;
    }
    float* part = p.att_parts + (static_cast<std::size_t>(head) * kSplits + split) * kPartFloats;
    reinterpret_cast<float4*>(part)[lane] = r;
    if (lane == 0) {
      part[kD] = m;
      part[kD + 1] = total;
    }
  } else if (warp == 1 && has_new && head % kHeadsPerKv == 0) {
    // Append the new row to this layer's cache (for the next steps).
    const std::size_t row = base + position;
    if constexpr (sizeof(CacheT) == 4) {
      reinterpret_cast<float4*>(static_cast<float*>(layer.keys) + row * kD)[lane] = new_k;
      reinterpret_cast<float4*>(static_cast<float*>(layer.values) + row * kD)[lane] = new_v;
    } else {
      reinterpret_cast<uint2*>(static_cast<Bf16*>(layer.keys) + row * kD)[lane] =
          PackBf16x4(new_k.x, new_k.y, new_k.z, new_k.w);
      reinterpret_cast<uint2*>(static_cast<Bf16*>(layer.values) + row * kD)[lane] =
          PackBf16x4(new_v.x, new_v.y, new_v.z, new_v.w);
    }
  }
  ConsumerSync();
}

/// The attention output row (bf16 [2048]) into `row`: thread t merges the
/// split partials of head t / 32 for dims 4 (t % 32) .. + 3, every load in
/// flight at once (split order fixed, so the merge is deterministic).
__device__ void MergeAttention(const float* parts, Bf16* row, int tid) {
  const int head = tid >> 5;
  const int d = 4 * (tid & 31);
  const float* hp = parts + static_cast<std::size_t>(head) * kSplits * kPartFloats;
  float mx[kSplits], sm[kSplits];
  float4 o[kSplits];
#pragma unroll
  for (int s = 0; s < kSplits; ++s) {
    mx[s] = __ldcg(hp + s * kPartFloats + kD);
    sm[s] = __ldcg(hp + s * kPartFloats + kD + 1);
    o[s] = __ldcg(reinterpret_cast<const float4*>(hp + s * kPartFloats + d));
  }
  float m = -INFINITY;
#pragma unroll
  for (int s = 0; s < kSplits; ++s)
    m = fmaxf(m, mx[s]);
  float total = 0.0f;
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int s = 0; s < kSplits; ++s) {
    const float f = mx[s] == -INFINITY ? 0.0f : expf(mx[s] - m);
    total += sm[s] * f;
    r.x += o[s].x * f;
    r.y += o[s].y * f;
    r.z += o[s].z * f;
    r.w += o[s].w * f;
  }
  const float inverse = 1.0f / total;
  *reinterpret_cast<uint2*>(row + head * kD + d) =
      PackBf16x4(r.x * inverse, r.y * inverse, r.z * inverse, r.w * inverse);
}

/// Fragments of a bf16 row held in shared memory (lanes 0..3).
__device__ inline void SharedRowFragments(const Bf16* row, int chunk, int warp,
                                          int lane, RowFragments& b) {
#pragma unroll
  for (int t = 0; t < 2; ++t)
    b[t] = lane < 4 ? *reinterpret_cast<const uint4*>(row + chunk * kChunk + 64 * warp +
                                                      32 * t + 8 * lane)
                    : make_uint4(0u, 0u, 0u, 0u);
}

/// Fragments of bf16 row `src` for chunk `chunk` (lanes 0..3).
__device__ inline void Bf16RowFragments(const Bf16* src, int chunk, int warp,
                                        int lane, RowFragments& b) {
#pragma unroll
  for (int t = 0; t < 2; ++t)
    b[t] = lane < 4 ? __ldcg(reinterpret_cast<const uint4*>(
                          src + chunk * kChunk + 64 * warp + 32 * t + 8 * lane))
                    : make_uint4(0u, 0u, 0u, 0u);
}

// ---------------------------------------------------------------- producer

__device__ void Produce(const LmStackParams& p, unsigned char* ring,
                        std::uint64_t* full, std::uint64_t* empty,
                        const Control& c) {
  const std::uint64_t policy = PolicyEvictFirst();
  const int cta = static_cast<int>(blockIdx.x);
  const int ctas = static_cast<int>(gridDim.x);
  unsigned issued = 0;
  bool stop = false;
  auto issue = [&](const unsigned char* source) {
    if (stop)
      return;
    const unsigned slot = issued % kSlots;
    if (issued >= static_cast<unsigned>(kSlots) &&
        !WaitSlot(&empty[slot], ((issued / kSlots) - 1) & 1u, c,
                  kErrWeightWait)) {
      stop = true;
      return;
    }
    MbarArriveExpectTx(&full[slot], kSlotBytes);
    BulkLoad(ring + slot * kSlotBytes, source, kSlotBytes, &full[slot], policy);
    ++issued;
  };
  int base = 0;
  for (int l = 0; l < p.layers && !stop; ++l) {
    const LmLayer layer = p.layer[l];
    for (int phase = kQkv; phase <= kDown; ++phase) {
      const int units = PhaseUnits(phase);
      for (int u = FirstUnit(cta, ctas, base); u < units; u += ctas)
        for (int s = 0; s < PhaseSlots(phase); ++s)
          issue(SlotSource(layer, phase, u, s));
      base = (base + units) % ctas;
    }
  }
  const unsigned first = issued > static_cast<unsigned>(kSlots) ? issued - kSlots : 0u;
  for (unsigned k = first; k < issued; ++k)
    (void)MbarWaitBounded(&full[k % kSlots], (k / kSlots) & 1u, c.error_word,
                          kErrDrainWait);
}

// ---------------------------------------------------------------- consumers

__device__ void Consume(const LmStackParams& p, unsigned char* smem,
                        const Control& c) {
  unsigned char* ring = smem;
  float* red = reinterpret_cast<float*>(smem + kRedOffset);
  float* red2 = red + kConsumerWarps * kRed1;
  float* sums = reinterpret_cast<float*>(smem + kSumsOffset);
  PubEntry* entries = reinterpret_cast<PubEntry*>(smem + kPubOffset);
  std::uint64_t* full = reinterpret_cast<std::uint64_t*>(smem + kBarOffset);
  std::uint64_t* empty = full + kSlots;
  std::uint64_t* pub_full = empty + kSlots;
  std::uint64_t* pub_empty = pub_full + kPubSlots;
  const int tid = static_cast<int>(threadIdx.x);
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int cta = static_cast<int>(blockIdx.x);
  const int ctas = static_cast<int>(gridDim.x);
  unsigned* sync = p.sync;
  unsigned consumed = 0;
  unsigned published = 0;
  const int position = *p.position;

  auto acquire = [&]() -> const unsigned char* {
    const unsigned slot = consumed % kSlots;
    if (*c.aborted == 0)
      (void)WaitSlot(&full[slot], (consumed / kSlots) & 1u, c, kErrWeightWait);
    return ring + slot * kSlotBytes;
  };
  auto release = [&]() {
    __syncwarp();
    if (lane == 0)
      MbarArrive(&empty[consumed % kSlots]);
    ++consumed;
  };
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
  // The 16 outputs of a unit (row 0 of the one column tile), reduced over
  // the warps in order: `store(feature, value)`.
  auto reduce_row = [&](const float* buffer, auto&& store) {
    if (tid < kRed1) {
      int feature, row;
      Decode(tid, 1, feature, row);
      if (row == 0)
        store(feature, Reduce(buffer, tid, kRed1));
    }
  };
  auto check = [&]() { return !ConsumerSyncOr(*c.aborted != 0); };
  auto norm_weights = [&](const Bf16* weight, uint4 (&w)[2][2]) {
#pragma unroll
    for (int ch = 0; ch < 2; ++ch)
#pragma unroll
      for (int t = 0; t < 2; ++t)
        w[ch][t] = lane < 4 ? __ldg(reinterpret_cast<const uint4*>(
                                  weight + ch * kChunk + 64 * warp + 32 * t + 8 * lane))
                            : make_uint4(0u, 0u, 0u, 0u);
  };

  int base = 0;
  for (int l = 0; l < p.layers; ++l) {
    const LmLayer layer = p.layer[l];
    const unsigned index = static_cast<unsigned>(l);
    // This layer's post norm and the next layer's input norm (or the final
    // norm) into L2 now, so the norm stages wait on L2, not HBM.
    PrefetchL2(layer.post_norm, kHidden * 2, tid);
    PrefetchL2(l + 1 < p.layers ? p.layer[l + 1].input_norm : p.final_norm,
               kHidden * 2, tid);

    // QKV: norm(row) x W_qkv -> qkv (fp32).
    {
      const int mine = FirstUnit(cta, ctas, base);
      if (mine < kQkvUnits) {
        uint4 w[2][2];
        norm_weights(layer.input_norm, w);
        if (l > 0 && !WaitCount(c, sync + kSyncHidden, 2 * kOUnits * index))
          return;
        RowFragments b[2];
        NormRow(p.hidden, w, p.eps, sums, tid, warp, lane, b);
        for (int u = mine; u < kQkvUnits; u += ctas) {
          float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
          for (int ch = 0; ch < kHiddenChunks; ++ch) {
            RowProduct(acquire(), b[ch], warp, lane, acc);
            release();
          }
          StoreAcc(red, warp, lane, acc);
          ConsumerSync();
          reduce_row(red, [&](int feature, float v) { p.qkv[u * 16 + feature] = v; });
          ConsumerSync();
          publish(sync + kSyncQkv, 1u);
        }
      }
      base = (base + kQkvUnits) % ctas;
    }
    if (!check())
      return;

    // Attention: 16 heads x 8 key chunks on CTAs 0..127.
    if (cta < kTasks) {
      if (!WaitCount(c, sync + kSyncQkv, kQkvUnits * (index + 1)))
        return;
      if (p.bf16_kv)
        AttentionTask<Bf16>(p, layer, cta / kSplits, cta % kSplits, position,
                            red, tid, warp, lane);
      else
        AttentionTask<float>(p, layer, cta / kSplits, cta % kSplits, position,
                             red, tid, warp, lane);
      publish(sync + kSyncAtt, 1u);
    }

    // O: merged attention x W_o, added into the row by the unit's CTA.
    {
      const int mine = FirstUnit(cta, ctas, base);
      for (int u = mine; u < kOUnits; u += ctas) {
        if (!WaitCount(c, sync + kSyncAtt, kTasks * (index + 1)))
          return;
        Bf16* att_row = reinterpret_cast<Bf16*>(red2);
        MergeAttention(p.att_parts, att_row, tid);
        ConsumerSync();
        float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
        for (int ch = 0; ch < kAttWidth / kChunk; ++ch) {
          RowFragments b;
          SharedRowFragments(att_row, ch, warp, lane, b);
          RowProduct(acquire(), b, warp, lane, acc);
          release();
        }
        StoreAcc(red, warp, lane, acc);
        ConsumerSync();
        reduce_row(red, [&](int feature, float v) {
          const int at = u * 16 + feature;
          p.hidden[at] = __ldcg(p.hidden + at) + v;
        });
        ConsumerSync();
        publish(sync + kSyncHidden, 1u);
      }
      base = (base + kOUnits) % ctas;
    }

    // gate/up: norm(row) x W_gate, W_up -> bf16(silu(g) * u).
    {
      const int mine = FirstUnit(cta, ctas, base);
      if (mine < kGuUnits) {
        uint4 w[2][2];
        norm_weights(layer.post_norm, w);
        if (!WaitCount(c, sync + kSyncHidden, 2 * kOUnits * index + kOUnits))
          return;
        RowFragments b[2];
        NormRow(p.hidden, w, p.eps, sums, tid, warp, lane, b);
        for (int u = mine; u < kGuUnits; u += ctas) {
          float gate[1][4] = {{0.f, 0.f, 0.f, 0.f}};
          float up[1][4] = {{0.f, 0.f, 0.f, 0.f}};
          for (int ch = 0; ch < kHiddenChunks; ++ch) {
            RowProduct(acquire(), b[ch], warp, lane, gate);
            release();
          }
          for (int ch = 0; ch < kHiddenChunks; ++ch) {
            RowProduct(acquire(), b[ch], warp, lane, up);
            release();
          }
          StoreAcc(red, warp, lane, gate);
          StoreAcc(red2, warp, lane, up);
          ConsumerSync();
          if (tid < kRed1) {
            int feature, row;
            Decode(tid, 1, feature, row);
            if (row == 0) {
              const float g = Reduce(red, tid, kRed1);
              const float v = Reduce(red2, tid, kRed1);
              p.act[u * 16 + feature] = ToBf16(g / (1.0f + expf(-g)) * v);
            }
          }
          ConsumerSync();
          publish(sync + kSyncAct, 1u);
        }
      }
      base = (base + kGuUnits) % ctas;
    }
    if (!check())
      return;

    // down: act x W_down, added into the row by the unit's CTA.
    {
      const int mine = FirstUnit(cta, ctas, base);
      for (int u = mine; u < kDownUnits; u += ctas) {
        if (!WaitCount(c, sync + kSyncAct, kGuUnits * (index + 1)))
          return;
        float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
        RowFragments b[2];
        Bf16RowFragments(p.act, 0, warp, lane, b[0]);
        for (int ch = 0; ch < kInterChunks; ++ch) {
          if (ch + 1 < kInterChunks)
            Bf16RowFragments(p.act, ch + 1, warp, lane, b[(ch + 1) & 1]);
          RowProduct(acquire(), b[ch & 1], warp, lane, acc);
          release();
        }
        StoreAcc(red, warp, lane, acc);
        ConsumerSync();
        reduce_row(red, [&](int feature, float v) {
          const int at = u * 16 + feature;
          p.hidden[at] = __ldcg(p.hidden + at) + v;
        });
        ConsumerSync();
        publish(sync + kSyncHidden, 1u);
      }
      base = (base + kDownUnits) % ctas;
    }
  }
  // The final norm's fp32 output (kernels/generator_kernels.hip:91-108).
  if (cta == 0) {
    if (!WaitCount(c, sync + kSyncHidden,
                   2 * kOUnits * static_cast<unsigned>(p.layers)))
      return;
    const float4 v = __ldcg(reinterpret_cast<const float4*>(p.hidden) + tid);
    const float s = WarpAllSum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
    if (lane == 0)
      sums[warp] = s;
    ConsumerSync();
    float total = sums[0];
    for (int w = 1; w < kConsumerWarps; ++w)
      total += sums[w];
    const float r = rsqrtf(total / static_cast<float>(kHidden) + p.eps);
    const uint2 wb = __ldg(reinterpret_cast<const uint2*>(p.final_norm) + tid);
    reinterpret_cast<float4*>(p.output)[tid] =
        make_float4(v.x * r * Bf16ToFloat(static_cast<Bf16>(wb.x & 0xFFFFu)),
                    v.y * r * Bf16ToFloat(static_cast<Bf16>(wb.x >> 16)),
                    v.z * r * Bf16ToFloat(static_cast<Bf16>(wb.y & 0xFFFFu)),
                    v.w * r * Bf16ToFloat(static_cast<Bf16>(wb.y >> 16)));
  }
  publish(nullptr, 0u);
}

__global__ void __launch_bounds__(kThreads, 1)
    LmStackKernel(const LmStackParams p, unsigned* error_word) {
  extern __shared__ __align__(128) unsigned char smem[];
  std::uint64_t* full = reinterpret_cast<std::uint64_t*>(smem + kBarOffset);
  std::uint64_t* empty = full + kSlots;
  std::uint64_t* pub_full = empty + kSlots;
  std::uint64_t* pub_empty = pub_full + kPubSlots;
  volatile int* aborted = reinterpret_cast<volatile int*>(smem + kFlagOffset);
  const Control c{p.sync, error_word, aborted};
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      MbarInit(&full[s], 1);
      MbarInit(&empty[s], kConsumerWarps);
    }
    for (int s = 0; s < kPubSlots; ++s) {
      MbarInit(&pub_full[s], 1);
      MbarInit(&pub_empty[s], 1);
    }
    *aborted = 0;
    FenceMbarInit();
  }
  __syncthreads();
  if (threadIdx.x >= kConsumers) {
    if (threadIdx.x == kConsumers)
      Produce(p, smem, full, empty, c);
    else if (threadIdx.x == kConsumers + 32)
      Publish(reinterpret_cast<PubEntry*>(smem + kPubOffset), pub_full,
              pub_empty, c);
    return;
  }
  Consume(p, smem, c);
}

constexpr std::size_t Align256(std::size_t n) {
  return (n + 255) & ~std::size_t{255};
}

int LmCtas() {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64)
    return 0;
  static std::mutex mutex;
  static int ctas[64] = {};
  static bool probed[64] = {};
  std::lock_guard<std::mutex> lock(mutex);
  if (!probed[device]) {
    probed[device] = true;
    int cooperative = 0, sms = 0, blocks = 0;
    if (cudaDeviceGetAttribute(&cooperative, cudaDevAttrCooperativeLaunch,
                               device) != cudaSuccess ||
        cooperative == 0 ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) !=
            cudaSuccess ||
        cudaFuncSetAttribute(LmStackKernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemBytes) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, LmStackKernel,
                                                      kThreads, kSmemBytes) !=
            cudaSuccess ||
        blocks < 1)
      return 0;
    ctas[device] = sms >= kTasks ? sms : 0;
  }
  const int cap = PersistentMaxCtas();
  if (cap > 0 && ctas[device] > 0)
    return std::min(ctas[device], std::max(cap, kTasks));
  return ctas[device];
}

}  // namespace

std::size_t LmWorkBytes() {
  return Align256(kQkvWidth * 4) +
         Align256(std::size_t{kHeads} * kSplits * kPartFloats * 4) +
         Align256(kInter * 2) + Align256(kLmSyncWords * 4);
}

void LmWorkLayout(void* base, LmStackParams& params) {
  auto* at = static_cast<unsigned char*>(base);
  auto take = [&](std::size_t bytes) {
    unsigned char* p = at;
    at += Align256(bytes);
    return p;
  };
  params.qkv = reinterpret_cast<float*>(take(kQkvWidth * 4));
  params.att_parts =
      reinterpret_cast<float*>(take(std::size_t{kHeads} * kSplits * kPartFloats * 4));
  params.act = reinterpret_cast<std::uint16_t*>(take(kInter * 2));
  params.sync = reinterpret_cast<unsigned*>(take(kLmSyncWords * 4));
}

bool LmStackSupported() {
  const bool ok = LmCtas() > 0;
  (void)cudaGetLastError();
  return ok;
}

int LaunchLmStack(const LmStackParams& p, cudaStream_t stream) {
  if (p.layers < 1 || p.layer == nullptr || p.final_norm == nullptr ||
      p.position == nullptr || p.hidden == nullptr || p.output == nullptr ||
      p.qkv == nullptr || p.att_parts == nullptr || p.act == nullptr ||
      p.sync == nullptr || p.capacity < 1)
    return Fail(kInvalid, "persistent stack: missing argument");
  const int ctas = LmCtas();
  if (ctas == 0)
    return Fail(kUnsupported,
                "persistent stack: the device cannot hold one CTA per SM for "
                "128 attention tasks");
  unsigned* error_word = DeviceErrorWord();
  if (error_word == nullptr)
    return Fail(kCudaError, "persistent stack: device error word");
  if (cudaMemsetAsync(p.sync, 0, kLmSyncWords * sizeof(unsigned), stream) !=
      cudaSuccess)
    return Fail(kCudaError, "persistent stack: memset");
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(static_cast<unsigned>(ctas));
  config.blockDim = dim3(kThreads);
  config.dynamicSmemBytes = kSmemBytes;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeCooperative;
  attribute[0].val.cooperative = 1;
  config.attrs = attribute;
  config.numAttrs = PersistentCooperative() ? 1 : 0;
  return FromCuda(cudaLaunchKernelEx(&config, LmStackKernel, p, error_word),
                  "persistent stack launch");
}

}  // namespace vx
