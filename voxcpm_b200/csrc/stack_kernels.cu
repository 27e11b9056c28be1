// Stack and generation-step kernels on sm_100a (see stack_kernels.cuh).
//
// Semantics follow kernels/generator_kernels.hip (cited per kernel); the
// launch shapes are this library's own: vectorized 16-byte accesses, every
// kernel PDL-aware (it signals its dependents first, then waits for its
// predecessors before touching their outputs), and attention split over the
// keys inside a thread-block cluster whose CTAs merge their online-softmax
// partials through distributed shared memory in rank order (deterministic,
// no scratch).
#include "stack_kernels.cuh"
#include "vx_common.cuh"
#include "vx_launch.cuh"

#include <cmath>

namespace vx {
namespace {

constexpr int kThreads = 256;

__device__ inline void Prologue() {
  GridLaunchDependents();
  GridDependencyWait();
}

__device__ inline float WarpSum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

/// Block-wide sum in a fixed order (warp trees, then warps in order).
__device__ inline float BlockSum(float v, float* scratch) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps = (blockDim.x + 31) >> 5;
  v = WarpSum(v);
  __syncthreads();
  if (lane == 0)
    scratch[warp] = v;
  __syncthreads();
  float total = scratch[0];
  for (int i = 1; i < warps; ++i)
    total += scratch[i];
  return total;
}

unsigned Blocks(std::size_t count, int threads = kThreads) {
  return static_cast<unsigned>((count + threads - 1) / threads);
}

const dim3 kNoCluster(1, 1, 1);

__device__ inline uint2 PackBf16x4(float a, float b, float c, float d) {
  uint2 packed;
  packed.x = static_cast<unsigned>(FloatToBf16(a)) |
             (static_cast<unsigned>(FloatToBf16(b)) << 16);
  packed.y = static_cast<unsigned>(FloatToBf16(c)) |
             (static_cast<unsigned>(FloatToBf16(d)) << 16);
  return packed;
}

// ---------------------------------------------------------------- row plumbing

/// kernels/generator_kernels.hip:63-71
__global__ void EmbedKernel(const Bf16* table, const std::int32_t* ids,
                            const std::int32_t* text_mask, float* output,
                            int width, float scale) {
  Prologue();
  const std::size_t row = blockIdx.x;
  const bool text = text_mask[row] != 0;
  const Bf16* source = table + static_cast<std::size_t>(ids[row]) * width;
  for (int i = threadIdx.x; i < width; i += blockDim.x)
    output[row * width + i] = text ? Bf16ToFloat(source[i]) * scale : 0.0f;
}

/// kernels/generator_kernels.hip:73-79
__global__ void ScatterRowsKernel(const float* input,
                                  const std::int32_t* indices, float* output,
                                  int width) {
  Prologue();
  const std::size_t row = blockIdx.x;
  const std::size_t target = static_cast<std::size_t>(indices[row]);
  for (int i = threadIdx.x; i < width; i += blockDim.x)
    output[target * width + i] = input[row * width + i];
}

/// kernels/generator_kernels.hip:81-89
__global__ void GatherRowsKernel(const float* input,
                                 const std::int32_t* indices, float* output,
                                 int width) {
  Prologue();
  const std::size_t row = blockIdx.x;
  const std::size_t source = static_cast<std::size_t>(indices[row]);
  for (int i = threadIdx.x; i < width; i += blockDim.x)
    output[row * width + i] = input[source * width + i];
}

// ---------------------------------------------------------------- RMSNorm

/// bf16(w * x * rsqrt(mean(x^2) + eps)), optional fp32 copy
/// (kernels/generator_kernels.hip:91-108). One CTA per row.
__global__ void __launch_bounds__(kThreads)
    RmsNormKernel(const float* input, const Bf16* weight, Bf16* output,
                  float* output_f32, int width, float epsilon) {
  __shared__ float scratch[kThreads / 32];
  Prologue();
  const std::size_t row = blockIdx.x;
  const float* x = input + row * width;
  float sum = 0.0f;
  for (int i = threadIdx.x * 4; i < width; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(x + i);
    sum += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  sum = BlockSum(sum, scratch);
  const float inverse = rsqrtf(sum / static_cast<float>(width) + epsilon);
  for (int i = threadIdx.x * 4; i < width; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(x + i);
    const uint2 wb = *reinterpret_cast<const uint2*>(weight + i);
    const float o0 = v.x * inverse * Bf16ToFloat(static_cast<Bf16>(wb.x & 0xFFFFu));
    const float o1 = v.y * inverse * Bf16ToFloat(static_cast<Bf16>(wb.x >> 16));
    const float o2 = v.z * inverse * Bf16ToFloat(static_cast<Bf16>(wb.y & 0xFFFFu));
    const float o3 = v.w * inverse * Bf16ToFloat(static_cast<Bf16>(wb.y >> 16));
    *reinterpret_cast<uint2*>(output + row * width + i) =
        PackBf16x4(o0, o1, o2, o3);
    if (output_f32 != nullptr)
      *reinterpret_cast<float4*>(output_f32 + row * width + i) =
          make_float4(o0, o1, o2, o3);
  }
}

// ---------------------------------------------------------------- QKV + RoPE

template <typename CacheT>
__device__ inline void StoreCache(CacheT* p, float v);
template <>
__device__ inline void StoreCache<float>(float* p, float v) {
  *p = v;
}
template <>
__device__ inline void StoreCache<Bf16>(Bf16* p, float v) {
  *p = FloatToBf16(v);
}

/// Splits [q heads | k heads | v heads], rotates the (i, i + d/2) pairs of q
/// and k by the table row of the row's position, writes q [rows][heads][d]
/// and appends k, v to the cache at the row's cache row
/// (kernels/generator_kernels.hip:110-158).
template <typename CacheT>
__global__ void __launch_bounds__(kThreads)
    QkvRopeKernel(const float* qkv, const float* cos_sin,
                  const std::int32_t* positions,
                  const std::int32_t* cache_rows, float* q, CacheT* k_cache,
                  CacheT* v_cache, int heads, int kv_heads, int head_dim,
                  int capacity) {
  Prologue();
  const std::size_t row = blockIdx.x;
  const int half = head_dim / 2;
  const int width = (heads + 2 * kv_heads) * head_dim;
  const float* source = qkv + row * width;
  const float* table =
      cos_sin == nullptr
          ? nullptr
          : cos_sin + static_cast<std::size_t>(positions[row]) * head_dim;
  const std::size_t cache_row = static_cast<std::size_t>(cache_rows[row]);
  const int pairs = (heads + kv_heads) * half;
  for (int index = threadIdx.x; index < pairs; index += blockDim.x) {
    const int head = index / half;
    const int i = index % half;
    const float a = source[head * head_dim + i];
    const float b = source[head * head_dim + half + i];
    float first = a;
    float second = b;
    if (table != nullptr) {
      const float c = table[i];
      const float s = table[half + i];
      first = a * c - b * s;
      second = b * c + a * s;
    }
    if (head < heads) {
      float* target = q + (row * heads + head) * head_dim;
      target[i] = first;
      target[half + i] = second;
    } else {
      CacheT* target =
          k_cache +
          (static_cast<std::size_t>(head - heads) * capacity + cache_row) *
              head_dim;
      StoreCache(target + i, first);
      StoreCache(target + half + i, second);
    }
  }
  const float* v = source + (heads + kv_heads) * head_dim;
  for (int index = threadIdx.x; index < kv_heads * head_dim;
       index += blockDim.x) {
    const int head = index / head_dim;
    StoreCache(v_cache + (static_cast<std::size_t>(head) * capacity +
                          cache_row) *
                             head_dim +
                   index % head_dim,
               v[index]);
  }
}

// ---------------------------------------------------------------- attention

constexpr int kAttentionWarps = 4;
constexpr int kMaxKeySplits = 8;

template <typename CacheT>
__device__ inline float4 LoadKv(const CacheT* base, std::size_t key, int lane);
template <>
__device__ inline float4 LoadKv<float>(const float* base, std::size_t key,
                                       int lane) {
  return reinterpret_cast<const float4*>(base + key * 128)[lane];
}
template <>
__device__ inline float4 LoadKv<Bf16>(const Bf16* base, std::size_t key,
                                      int lane) {
  const uint2 v = reinterpret_cast<const uint2*>(base + key * 128)[lane];
  return make_float4(Bf16ToFloat(static_cast<Bf16>(v.x & 0xFFFFu)),
                     Bf16ToFloat(static_cast<Bf16>(v.x >> 16)),
                     Bf16ToFloat(static_cast<Bf16>(v.y & 0xFFFFu)),
                     Bf16ToFloat(static_cast<Bf16>(v.y >> 16)));
}

__device__ inline float LoadSharedCluster1(std::uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

struct AttentionArgs {
  const float* q;
  const void* k_cache;
  const void* v_cache;
  Bf16* output;
  const std::int32_t* past_device;
  int past_stride;  // 1: past_device holds one value per sequence
  const std::int32_t* first_keys;  // per sequence; null: sequence * keys_per_sequence
  int rows_per_sequence;
  int keys_per_sequence;
  int past;
  int causal;
  int heads;
  int kv_heads;
  int capacity;
  int splits;
  float scale;
};

/// Softmax attention of one (row, head) over `past` cached keys plus its
/// sequence's rows (up to itself when causal), head_dim 128, GQA, scale
/// 1/sqrt(128), bf16 output (kernels/generator_kernels.hip:160-241). The
/// keys are split over the `splits` CTAs of a cluster; four warps per CTA
/// take every fourth key with an online softmax (running max and sum); the
/// warps merge in shared memory, then CTA 0 merges the CTAs in rank order.
template <typename CacheT>
__global__ void __launch_bounds__(kAttentionWarps * 32)
    AttentionKernel(const AttentionArgs a) {
  __shared__ float warp_max[kAttentionWarps];
  __shared__ float warp_sum[kAttentionWarps];
  __shared__ float4 warp_out[kAttentionWarps][32];
  __shared__ float cta_max;
  __shared__ float cta_sum;
  __shared__ float4 cta_out[32];
  Prologue();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int row = static_cast<int>(blockIdx.x) / a.heads;
  const int head = static_cast<int>(blockIdx.x) % a.heads;
  const int split = static_cast<int>(blockIdx.y);
  const int sequence = row / a.rows_per_sequence;
  const int local = row % a.rows_per_sequence;
  const int past = a.past_device != nullptr
                       ? a.past_device[a.past_stride * sequence]
                       : a.past;
  const int count = past + (a.causal ? local + 1 : a.rows_per_sequence);
  const int per = (count + a.splits - 1) / a.splits;
  const int k0 = split * per;
  const int k1 = min(count, k0 + per);
  const std::size_t first_key =
      a.first_keys != nullptr
          ? static_cast<std::size_t>(a.first_keys[sequence])
          : static_cast<std::size_t>(sequence) * a.keys_per_sequence;
  const int kv_head = head / (a.heads / a.kv_heads);
  const CacheT* keys = static_cast<const CacheT*>(a.k_cache) +
                       (static_cast<std::size_t>(kv_head) * a.capacity +
                        first_key) *
                           128;
  const CacheT* values = static_cast<const CacheT*>(a.v_cache) +
                         (static_cast<std::size_t>(kv_head) * a.capacity +
                          first_key) *
                             128;
  float4 query = reinterpret_cast<const float4*>(
      a.q + (static_cast<std::size_t>(row) * a.heads + head) * 128)[lane];
  query.x *= a.scale;
  query.y *= a.scale;
  query.z *= a.scale;
  query.w *= a.scale;
  float maximum = -INFINITY;
  float sum = 0.0f;
  float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int key = k0 + warp; key < k1; key += kAttentionWarps) {
    const float4 k = LoadKv<CacheT>(keys, key, lane);
    const float4 v = LoadKv<CacheT>(values, key, lane);
    float score = query.x * k.x + query.y * k.y + query.z * k.z + query.w * k.w;
    score = WarpSum(score);
    const float next = fmaxf(maximum, score);
    const float decay = expf(maximum - next);
    const float weight = expf(score - next);
    sum = sum * decay + weight;
    out.x = out.x * decay + weight * v.x;
    out.y = out.y * decay + weight * v.y;
    out.z = out.z * decay + weight * v.z;
    out.w = out.w * decay + weight * v.w;
    maximum = next;
  }
  if (lane == 0) {
    warp_max[warp] = maximum;
    warp_sum[warp] = sum;
  }
  warp_out[warp][lane] = out;
  __syncthreads();
  if (warp == 0) {
    float m = warp_max[0];
    for (int w = 1; w < kAttentionWarps; ++w)
      m = fmaxf(m, warp_max[w]);
    float total = 0.0f;
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int w = 0; w < kAttentionWarps; ++w) {
      const float f = warp_max[w] == -INFINITY ? 0.0f : expf(warp_max[w] - m);
      total += warp_sum[w] * f;
      const float4 p = warp_out[w][lane];
      r.x += p.x * f;
      r.y += p.y * f;
      r.z += p.z * f;
      r.w += p.w * f;
    }
    cta_out[lane] = r;
    if (lane == 0) {
      cta_max = m;
      cta_sum = total;
    }
  }
  Bf16* target = a.output +
                 (static_cast<std::size_t>(row) * a.heads + head) * 128 +
                 lane * 4;
  if (a.splits > 1) {
    ClusterSync();
    if (split == 0 && warp == 0) {
      float peer_max[kMaxKeySplits];
      float m = -INFINITY;
      for (int r = 0; r < a.splits; ++r) {
        peer_max[r] =
            r == 0 ? cta_max : LoadSharedCluster1(MapShared(&cta_max, r));
        m = fmaxf(m, peer_max[r]);
      }
      float total = 0.0f;
      float4 result = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < a.splits; ++r) {
        const float s =
            r == 0 ? cta_sum : LoadSharedCluster1(MapShared(&cta_sum, r));
        const float4 p = r == 0 ? cta_out[lane]
                                : LoadSharedCluster4(MapShared(&cta_out[lane], r));
        const float f =
            peer_max[r] == -INFINITY ? 0.0f : expf(peer_max[r] - m);
        total += s * f;
        result.x += p.x * f;
        result.y += p.y * f;
        result.z += p.z * f;
        result.w += p.w * f;
      }
      const float inverse = 1.0f / total;
      *reinterpret_cast<uint2*>(target) =
          PackBf16x4(result.x * inverse, result.y * inverse,
                     result.z * inverse, result.w * inverse);
    }
    ClusterSync();  // peers keep their shared memory until CTA 0 read it
    return;
  }
  __syncthreads();
  if (warp == 0) {
    const float4 r = cta_out[lane];
    const float inverse = 1.0f / cta_sum;
    *reinterpret_cast<uint2*>(target) = PackBf16x4(
        r.x * inverse, r.y * inverse, r.z * inverse, r.w * inverse);
  }
}

/// The same attention for rows that see at most 32 keys (the DiT's 11-row
/// sequences, short prefills): one warp per (row, head), four per CTA, each
/// warp taking all of its keys in order with the online softmax, so no
/// cross-warp merge and a quarter of the CTAs (at 704 rows x 16 heads:
/// 2,816 CTAs instead of 11,264).
template <typename CacheT>
__global__ void __launch_bounds__(kAttentionWarps * 32)
    ShortAttentionKernel(const AttentionArgs a, int pairs) {
  Prologue();
  const int lane = threadIdx.x & 31;
  const int pair = static_cast<int>(blockIdx.x) * kAttentionWarps +
                   static_cast<int>(threadIdx.x >> 5);
  if (pair >= pairs)
    return;
  const int row = pair / a.heads;
  const int head = pair % a.heads;
  const int sequence = row / a.rows_per_sequence;
  const int local = row % a.rows_per_sequence;
  const int past = a.past_device != nullptr
                       ? a.past_device[a.past_stride * sequence]
                       : a.past;
  const int count = past + (a.causal ? local + 1 : a.rows_per_sequence);
  const std::size_t first_key =
      a.first_keys != nullptr
          ? static_cast<std::size_t>(a.first_keys[sequence])
          : static_cast<std::size_t>(sequence) * a.keys_per_sequence;
  const int kv_head = head / (a.heads / a.kv_heads);
  const CacheT* keys = static_cast<const CacheT*>(a.k_cache) +
                       (static_cast<std::size_t>(kv_head) * a.capacity +
                        first_key) *
                           128;
  const CacheT* values = static_cast<const CacheT*>(a.v_cache) +
                         (static_cast<std::size_t>(kv_head) * a.capacity +
                          first_key) *
                             128;
  float4 query = reinterpret_cast<const float4*>(
      a.q + (static_cast<std::size_t>(row) * a.heads + head) * 128)[lane];
  query.x *= a.scale;
  query.y *= a.scale;
  query.z *= a.scale;
  query.w *= a.scale;
  float maximum = -INFINITY;
  float sum = 0.0f;
  float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int key = 0; key < count; ++key) {
    const float4 k = LoadKv<CacheT>(keys, key, lane);
    const float4 v = LoadKv<CacheT>(values, key, lane);
    float score = query.x * k.x + query.y * k.y + query.z * k.z + query.w * k.w;
    score = WarpSum(score);
    const float next = fmaxf(maximum, score);
    const float decay = expf(maximum - next);
    const float weight = expf(score - next);
    sum = sum * decay + weight;
    out.x = out.x * decay + weight * v.x;
    out.y = out.y * decay + weight * v.y;
    out.z = out.z * decay + weight * v.z;
    out.w = out.w * decay + weight * v.w;
    maximum = next;
  }
  const float inverse = 1.0f / sum;
  *reinterpret_cast<uint2*>(a.output +
                            (static_cast<std::size_t>(row) * a.heads + head) *
                                128 +
                            lane * 4) =
      PackBf16x4(out.x * inverse, out.y * inverse, out.z * inverse,
                 out.w * inverse);
}

// ---------------------------------------------------------------- elementwise

/// bf16(silu(g) * u) (kernels/generator_kernels.hip:243-254).
__global__ void SwiGluKernel(const float* gate_up, Bf16* output, int rows,
                             int width) {
  Prologue();
  const std::size_t index =
      static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= static_cast<std::size_t>(rows) * width)
    return;
  const std::size_t row = index / width;
  const std::size_t i = index % width;
  const float gate = gate_up[row * 2 * width + i];
  const float up = gate_up[row * 2 * width + width + i];
  output[index] = FloatToBf16(gate / (1.0f + expf(-gate)) * up);
}

/// kernels/generator_kernels.hip:256-262
__global__ void AddBiasKernel(float* data, const Bf16* bias, int rows,
                              int width) {
  Prologue();
  const std::size_t index =
      static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index < static_cast<std::size_t>(rows) * width)
    data[index] += Bf16ToFloat(bias[index % width]);
}

/// kernels/generator_kernels.hip:264-274
__global__ void ToBf16Kernel(const float* input, Bf16* output,
                             std::size_t count, int silu) {
  Prologue();
  const std::size_t index =
      static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= count)
    return;
  float value = input[index];
  if (silu)
    value = value / (1.0f + expf(-value));
  output[index] = FloatToBf16(value);
}

/// kernels/generator_kernels.hip:276-289
__global__ void ConcatRowsKernel(const float* a, const float* a_scale,
                                 int a_width, const float* b,
                                 const float* b_scale, int b_width,
                                 Bf16* output) {
  Prologue();
  const std::size_t row = blockIdx.x;
  const int width = a_width + b_width;
  const float sa = a_scale == nullptr ? 1.0f : a_scale[row];
  const float sb = b_scale == nullptr ? 1.0f : b_scale[row];
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const float value = i < a_width ? a[row * a_width + i] * sa
                                    : b[row * b_width + i - a_width] * sb;
    output[row * width + i] = FloatToBf16(value);
  }
}

/// FSQ: bf16(rint(tanh(x) * scale) / scale), round half to even
/// (kernels/generator_kernels.hip:291-297).
__global__ void QuantizeKernel(const float* input, Bf16* output,
                               std::size_t count, float scale) {
  Prologue();
  const std::size_t index =
      static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index < count)
    output[index] = FloatToBf16(rintf(tanhf(input[index]) * scale) / scale);
}

/// kernels/generator_kernels.hip:299-306
__global__ void SelectRowsKernel(const float* quantized, const float* plain,
                                 const std::int32_t* mask, float* output,
                                 int width) {
  Prologue();
  const std::size_t row = blockIdx.x;
  const float* source = mask[row] != 0 ? quantized : plain;
  for (int i = threadIdx.x; i < width; i += blockDim.x)
    output[row * width + i] = source[row * width + i];
}

/// kernels/generator_kernels.hip:308-318
__global__ void PrependSpecialKernel(const float* rows_in, const Bf16* special,
                                     float* output, int patch_size,
                                     int width) {
  Prologue();
  const std::size_t patch = blockIdx.x;
  const std::size_t row = blockIdx.y;
  float* target = output + (patch * (patch_size + 1) + row) * width;
  const float* source =
      row == 0 ? nullptr : rows_in + (patch * patch_size + row - 1) * width;
  for (int i = threadIdx.x; i < width; i += blockDim.x)
    target[i] = source == nullptr ? Bf16ToFloat(special[i]) : source[i];
}

/// The DiT's CFG pair of sequences [mu_a, mu_b, time, cond x P, x x P]; the
/// unconditional one has zero mu (kernels/generator_kernels.hip:320-340).
__global__ void AssembleDitKernel(const float* mu, const float* time,
                                  const float* cond, const float* x,
                                  float* output, int patch_size, int width) {
  Prologue();
  const int sequence = blockIdx.x;
  const int row = blockIdx.y;
  const int length = 3 + 2 * patch_size;
  float* target =
      output + (static_cast<std::size_t>(sequence) * length + row) * width;
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    float value;
    if (row < 2)
      value = sequence == 0 ? mu[row * width + i] : 0.0f;
    else if (row == 2)
      value = time[i];
    else if (row < 3 + patch_size)
      value = cond[(row - 3) * width + i];
    else
      value = x[(row - 3 - patch_size) * width + i];
    target[i] = value;
  }
}

/// CFG-Zero*: s = <c,u> / (|u|^2 + 1e-8), v = u s + cfg (c - u s),
/// x -= dt v (kernels/generator_kernels.hip:342-360). One CTA.
__global__ void __launch_bounds__(kThreads)
    GuidedEulerKernel(const float* velocity, float* x, int count, float cfg,
                      float dt) {
  __shared__ float scratch[kThreads / 32];
  Prologue();
  const float* c = velocity;
  const float* u = velocity + count;
  float dot = 0.0f;
  float norm = 0.0f;
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    dot += c[i] * u[i];
    norm += u[i] * u[i];
  }
  dot = BlockSum(dot, scratch);
  norm = BlockSum(norm, scratch);
  const float s = dot / (norm + 1e-8f);
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    const float guided = u[i] * s + cfg * (c[i] - u[i] * s);
    x[i] -= dt * guided;
  }
}

__global__ void CopyFloatsKernel(const float* input, float* output,
                                 std::size_t count) {
  Prologue();
  const std::size_t index =
      static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index < count)
    output[index] = input[index];
}

__global__ void AdvancePositionKernel(std::int32_t* counter,
                                      std::int32_t* positions) {
  Prologue();
  if (threadIdx.x == 0) {
    const std::int32_t next = *counter + 1;
    *counter = next;
    positions[0] = next;
  }
}

/// output[(*position & 1) * count + i] = input[i]: the patch's latent into
/// the slot of its position's parity (one block).
__global__ void CopyToParitySlotKernel(const float* input, float* slots,
                                       std::size_t count,
                                       const std::int32_t* position) {
  Prologue();
  float* output = slots + static_cast<std::size_t>(*position & 1) * count;
  for (std::size_t i = threadIdx.x; i < count; i += blockDim.x)
    output[i] = input[i];
}

}  // namespace

int Embed(const std::uint16_t* table, const std::int32_t* ids,
          const std::int32_t* text_mask, float* output, std::size_t rows,
          std::size_t width, float scale, cudaStream_t stream) {
  if (rows == 0)
    return kOk;
  return LaunchKernel(EmbedKernel, dim3(rows), dim3(kThreads), 0, stream,
                      kNoCluster, table, ids, text_mask, output,
                      static_cast<int>(width), scale);
}

int ScatterRows(const float* input, const std::int32_t* indices, float* output,
                std::size_t rows, std::size_t width, cudaStream_t stream) {
  if (rows == 0)
    return kOk;
  return LaunchKernel(ScatterRowsKernel, dim3(rows), dim3(kThreads), 0, stream,
                      kNoCluster, input, indices, output,
                      static_cast<int>(width));
}

int GatherRows(const float* input, const std::int32_t* indices, float* output,
               std::size_t rows, std::size_t width, cudaStream_t stream) {
  if (rows == 0)
    return kOk;
  return LaunchKernel(GatherRowsKernel, dim3(rows), dim3(kThreads), 0, stream,
                      kNoCluster, input, indices, output,
                      static_cast<int>(width));
}

int RmsNorm(const float* input, const std::uint16_t* weight,
            std::uint16_t* output, float* output_f32, std::size_t rows,
            std::size_t width, float epsilon, cudaStream_t stream) {
  if (rows == 0)
    return kOk;
  if (width % 4 != 0)
    return kUnsupported;
  return LaunchKernel(RmsNormKernel, dim3(rows), dim3(kThreads), 0, stream,
                      kNoCluster, input, weight, output, output_f32,
                      static_cast<int>(width), epsilon);
}

int QkvRope(const float* qkv, const float* cos_sin,
            const std::int32_t* positions, const std::int32_t* cache_rows,
            float* q, void* k_cache, void* v_cache, CacheType cache_type,
            std::size_t rows, std::size_t heads, std::size_t kv_heads,
            std::size_t head_dim, std::size_t capacity, cudaStream_t stream) {
  if (rows == 0)
    return kOk;
  if (cache_type == CacheType::kF32)
    return LaunchKernel(QkvRopeKernel<float>, dim3(rows), dim3(kThreads), 0,
                        stream, kNoCluster, qkv, cos_sin, positions,
                        cache_rows, q, static_cast<float*>(k_cache),
                        static_cast<float*>(v_cache), static_cast<int>(heads),
                        static_cast<int>(kv_heads), static_cast<int>(head_dim),
                        static_cast<int>(capacity));
  return LaunchKernel(QkvRopeKernel<Bf16>, dim3(rows), dim3(kThreads), 0,
                      stream, kNoCluster, qkv, cos_sin, positions, cache_rows,
                      q, static_cast<Bf16*>(k_cache),
                      static_cast<Bf16*>(v_cache), static_cast<int>(heads),
                      static_cast<int>(kv_heads), static_cast<int>(head_dim),
                      static_cast<int>(capacity));
}

int Attention(const float* q, const void* k_cache, const void* v_cache,
              CacheType cache_type, std::uint16_t* output, std::size_t rows,
              std::size_t rows_per_sequence, std::size_t keys_per_sequence,
              std::size_t past, const std::int32_t* past_device, bool causal,
              std::size_t heads, std::size_t kv_heads, std::size_t head_dim,
              std::size_t capacity, std::size_t max_keys,
              cudaStream_t stream, bool past_per_sequence,
              const std::int32_t* first_keys) {
  if (rows == 0)
    return kOk;
  if (head_dim != 128 || kv_heads == 0 || heads % kv_heads != 0 ||
      rows_per_sequence == 0)
    return kUnsupported;
  // Keys a row may see: at most max_keys when the position lives on the
  // device, else known now. About 32 keys per CTA, at most 8 CTAs.
  const std::size_t keys =
      past_device != nullptr ? max_keys : past + rows_per_sequence;
  int splits = static_cast<int>((keys + 31) / 32);
  splits = splits < 1 ? 1 : (splits > kMaxKeySplits ? kMaxKeySplits : splits);
  AttentionArgs a;
  a.q = q;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.output = output;
  a.past_device = past_device;
  a.past_stride = past_per_sequence ? 1 : 0;
  a.first_keys = first_keys;
  a.rows_per_sequence = static_cast<int>(rows_per_sequence);
  a.keys_per_sequence = static_cast<int>(keys_per_sequence);
  a.past = static_cast<int>(past);
  a.causal = causal ? 1 : 0;
  a.heads = static_cast<int>(heads);
  a.kv_heads = static_cast<int>(kv_heads);
  a.capacity = static_cast<int>(capacity);
  a.splits = splits;
  a.scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
  if (keys <= 32) {
    const int pairs = static_cast<int>(rows * heads);
    const dim3 short_grid(
        static_cast<unsigned>((pairs + kAttentionWarps - 1) / kAttentionWarps));
    if (cache_type == CacheType::kF32)
      return LaunchKernel(ShortAttentionKernel<float>, short_grid,
                          dim3(kAttentionWarps * 32), 0, stream, kNoCluster, a,
                          pairs);
    return LaunchKernel(ShortAttentionKernel<Bf16>, short_grid,
                        dim3(kAttentionWarps * 32), 0, stream, kNoCluster, a,
                        pairs);
  }
  const dim3 grid(static_cast<unsigned>(rows * heads),
                  static_cast<unsigned>(splits));
  const dim3 cluster(1, static_cast<unsigned>(splits), 1);
  if (cache_type == CacheType::kF32)
    return LaunchKernel(AttentionKernel<float>, grid,
                        dim3(kAttentionWarps * 32), 0, stream, cluster, a);
  return LaunchKernel(AttentionKernel<Bf16>, grid, dim3(kAttentionWarps * 32),
                      0, stream, cluster, a);
}

int SwiGlu(const float* gate_up, std::uint16_t* output, std::size_t rows,
           std::size_t width, cudaStream_t stream) {
  if (rows * width == 0)
    return kOk;
  return LaunchKernel(SwiGluKernel, dim3(Blocks(rows * width)), dim3(kThreads),
                      0, stream, kNoCluster, gate_up, output,
                      static_cast<int>(rows), static_cast<int>(width));
}

int AddBias(float* data, const std::uint16_t* bias, std::size_t rows,
            std::size_t width, cudaStream_t stream) {
  if (rows * width == 0)
    return kOk;
  return LaunchKernel(AddBiasKernel, dim3(Blocks(rows * width)),
                      dim3(kThreads), 0, stream, kNoCluster, data, bias,
                      static_cast<int>(rows), static_cast<int>(width));
}

int ToBf16(const float* input, std::uint16_t* output, std::size_t count,
           bool silu, cudaStream_t stream) {
  if (count == 0)
    return kOk;
  return LaunchKernel(ToBf16Kernel, dim3(Blocks(count)), dim3(kThreads), 0,
                      stream, kNoCluster, input, output, count, silu ? 1 : 0);
}

int ConcatRows(const float* a, const float* a_scale, std::size_t a_width,
               const float* b, const float* b_scale, std::size_t b_width,
               std::uint16_t* output, std::size_t rows, cudaStream_t stream) {
  if (rows == 0)
    return kOk;
  return LaunchKernel(ConcatRowsKernel, dim3(rows), dim3(kThreads), 0, stream,
                      kNoCluster, a, a_scale, static_cast<int>(a_width), b,
                      b_scale, static_cast<int>(b_width), output);
}

int Quantize(const float* input, std::uint16_t* output, std::size_t count,
             float scale, cudaStream_t stream) {
  if (count == 0)
    return kOk;
  return LaunchKernel(QuantizeKernel, dim3(Blocks(count)), dim3(kThreads), 0,
                      stream, kNoCluster, input, output, count, scale);
}

int SelectRows(const float* quantized, const float* plain,
               const std::int32_t* mask, float* output, std::size_t rows,
               std::size_t width, cudaStream_t stream) {
  if (rows == 0)
    return kOk;
  return LaunchKernel(SelectRowsKernel, dim3(rows), dim3(kThreads), 0, stream,
                      kNoCluster, quantized, plain, mask, output,
                      static_cast<int>(width));
}

int PrependSpecial(const float* rows_in, const std::uint16_t* special,
                   float* output, std::size_t patches, std::size_t patch_size,
                   std::size_t width, cudaStream_t stream) {
  if (patches == 0)
    return kOk;
  return LaunchKernel(PrependSpecialKernel,
                      dim3(static_cast<unsigned>(patches),
                           static_cast<unsigned>(patch_size + 1)),
                      dim3(kThreads), 0, stream, kNoCluster, rows_in, special,
                      output, static_cast<int>(patch_size),
                      static_cast<int>(width));
}

int AssembleDit(const float* mu, const float* time, const float* cond,
                const float* x, float* output, std::size_t patch_size,
                std::size_t width, cudaStream_t stream) {
  return LaunchKernel(AssembleDitKernel,
                      dim3(2, static_cast<unsigned>(3 + 2 * patch_size)),
                      dim3(kThreads), 0, stream, kNoCluster, mu, time, cond, x,
                      output, static_cast<int>(patch_size),
                      static_cast<int>(width));
}

int GuidedEuler(const float* velocity, float* x, std::size_t count, float cfg,
                float dt, cudaStream_t stream) {
  return LaunchKernel(GuidedEulerKernel, dim3(1), dim3(kThreads), 0, stream,
                      kNoCluster, velocity, x, static_cast<int>(count), cfg,
                      dt);
}

int CopyFloats(const float* input, float* output, std::size_t count,
               cudaStream_t stream) {
  if (count == 0)
    return kOk;
  return LaunchKernel(CopyFloatsKernel, dim3(Blocks(count)), dim3(kThreads), 0,
                      stream, kNoCluster, input, output, count);
}

int CopyToParitySlot(const float* input, float* slots, std::size_t count,
                     const std::int32_t* position, cudaStream_t stream) {
  if (count == 0)
    return kOk;
  return LaunchKernel(CopyToParitySlotKernel, dim3(1), dim3(kThreads), 0,
                      stream, kNoCluster, input, slots, count, position);
}

int AdvancePosition(std::int32_t* counter, std::int32_t* positions,
                    cudaStream_t stream) {
  return LaunchKernel(AdvancePositionKernel, dim3(1), dim3(32), 0, stream,
                      kNoCluster, counter, positions);
}

}  // namespace vx
