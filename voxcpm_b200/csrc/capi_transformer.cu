// C ABI of transformer.hpp (include/voxcpm_b200.h): KvCache, ForwardStack
// and Project for callers that drive a MiniCPM4 stack themselves
// (transformer.hpp:17-76, transformer.cpp:47-100). They run the same
// kernels the generator's per-kernel path runs (model.cu).
#include "model.cuh"
#include "vx_status.h"

#include "../../include/voxcpm_b200.h"

#include <exception>
#include <string>
#include <vector>

struct vx_kv_cache {
  vx::KvCache cache;
  int layers = 0;
};

namespace {

vx::StackConfig StackFromC(const vx_stack_config& s) {
  vx::StackConfig c;
  c.hidden = s.hidden;
  c.intermediate = s.intermediate;
  c.layers = s.layers;
  c.heads = s.heads;
  c.kv_heads = s.kv_heads;
  c.head_dim = s.head_dim;
  c.rms_eps = s.rms_eps;
  c.rope = s.rope != 0;
  return c;
}

const char* BadConfig(const vx_stack_config& s) {
  if (s.hidden <= 0 || s.intermediate <= 0 || s.layers <= 0 || s.heads <= 0 ||
      s.kv_heads <= 0 || s.head_dim <= 0)
    return "sizes must be positive";
  if (s.head_dim != 128)
    return "the attention kernels take head_dim 128";
  if (s.heads % s.kv_heads != 0)
    return "heads must be a multiple of kv_heads";
  return nullptr;
}

bool ToProjection(const vx_projection& in, vx::Projection* out) {
  if (in.weight == nullptr || in.in == 0 || in.out == 0 ||
      (in.format != VX_WEIGHTS_BF16 && in.format != VX_WEIGHTS_BF16_TILES &&
       in.format != VX_WEIGHTS_Q8_TILES))
    return false;
  out->format = static_cast<vx::WeightFormat>(in.format);
  out->weight = in.weight;
  out->bias = in.bias;
  out->in = static_cast<int>(in.in);
  out->out = static_cast<int>(in.out);
  return true;
}

}  // namespace

extern "C" {

vx_status vx_stack_scratch_elements(const vx_stack_config* config, size_t rows,
                                    size_t counts[6]) {
  if (config == nullptr || counts == nullptr)
    return vx::Fail(vx::kInvalid, "vx_stack_scratch_elements: null argument");
  if (const char* why = BadConfig(*config))
    return vx::Fail(vx::kInvalid, std::string("vx_stack_scratch_elements: ") + why);
  const size_t q = static_cast<size_t>(config->heads) * config->head_dim;
  const size_t qkv =
      static_cast<size_t>(config->heads + 2 * config->kv_heads) * config->head_dim;
  counts[0] = rows * config->hidden;            // normed (bf16)
  counts[1] = rows * qkv;                       // qkv
  counts[2] = rows * q;                         // q
  counts[3] = rows * q;                         // attention (bf16)
  counts[4] = rows * 2 * config->intermediate;  // gate_up
  counts[5] = rows * config->intermediate;      // activation (bf16)
  return VX_OK;
}

vx_kv_cache* vx_kv_cache_create(const vx_stack_config* config, size_t capacity,
                                int cache_type) {
  if (config == nullptr || capacity == 0 || capacity > (1u << 30) ||
      (cache_type != VX_CACHE_F32 && cache_type != VX_CACHE_BF16)) {
    vx::Fail(vx::kInvalid, "vx_kv_cache_create: bad argument");
    return nullptr;
  }
  if (const char* why = BadConfig(*config)) {
    vx::Fail(vx::kInvalid, std::string("vx_kv_cache_create: ") + why);
    return nullptr;
  }
  try {
    auto* handle = new vx_kv_cache{
        vx::KvCache(StackFromC(*config), static_cast<int>(capacity),
                    static_cast<vx::CacheType>(cache_type)),
        config->layers};
    // Zeroed like a fresh cache of the reference's DeviceBuffer users
    // expect; rows never written must not hold stale memory.
    const size_t half = handle->cache.bytes() / 2;
    cudaError_t e = cudaMemset(handle->cache.keys(0), 0, half);
    if (e == cudaSuccess)
      e = cudaMemset(handle->cache.values(0), 0, half);
    if (e != cudaSuccess) {
      delete handle;
      vx::FromCuda(e, "vx_kv_cache_create");
      return nullptr;
    }
    return handle;
  } catch (const std::exception& error) {
    vx::Fail(vx::kCudaError, std::string("vx_kv_cache_create: ") + error.what());
    return nullptr;
  }
}

void vx_kv_cache_destroy(vx_kv_cache* cache) { delete cache; }

size_t vx_kv_cache_capacity(const vx_kv_cache* cache) {
  return cache != nullptr ? static_cast<size_t>(cache->cache.capacity()) : 0;
}

void* vx_kv_cache_keys(const vx_kv_cache* cache, size_t layer) {
  if (cache == nullptr || layer >= static_cast<size_t>(cache->layers))
    return nullptr;
  return cache->cache.keys(static_cast<int>(layer));
}

void* vx_kv_cache_values(const vx_kv_cache* cache, size_t layer) {
  if (cache == nullptr || layer >= static_cast<size_t>(cache->layers))
    return nullptr;
  return cache->cache.values(static_cast<int>(layer));
}

vx_status vx_forward_stack(const vx_stack_weights* stack, const float* rope,
                           const vx_attention_layout* layout,
                           vx_kv_cache* cache, float* hidden, float* output,
                           size_t rows, const vx_stack_scratch* scratch,
                           cudaStream_t stream) {
  if (stack == nullptr || layout == nullptr || cache == nullptr ||
      hidden == nullptr || output == nullptr || scratch == nullptr ||
      stack->layers == nullptr || stack->norm == nullptr)
    return vx::Fail(vx::kInvalid, "vx_forward_stack: null argument");
  if (const char* why = BadConfig(stack->config))
    return vx::Fail(vx::kInvalid, std::string("vx_forward_stack: ") + why);
  if (stack->config.layers > cache->layers)
    return vx::Fail(vx::kInvalid, "vx_forward_stack: the cache has fewer layers than the stack");
  if (rows == 0)
    return VX_OK;
  if (layout->positions == nullptr || layout->cache_rows == nullptr ||
      layout->rows_per_sequence == 0 || rows % layout->rows_per_sequence != 0)
    return vx::Fail(vx::kInvalid,
                    "vx_forward_stack: positions, cache_rows and a row count "
                    "that is a multiple of rows_per_sequence are required");
  vx::StackWeights w;
  w.config = StackFromC(stack->config);
  w.norm = stack->norm;
  w.layers.resize(static_cast<size_t>(stack->config.layers));
  for (int i = 0; i < stack->config.layers; ++i) {
    const vx_layer_weights& in = stack->layers[i];
    vx::LayerWeights& out = w.layers[static_cast<size_t>(i)];
    out.input_norm = in.input_norm;
    out.post_norm = in.post_norm;
    if (in.input_norm == nullptr || in.post_norm == nullptr ||
        !ToProjection(in.qkv, &out.qkv) || !ToProjection(in.o, &out.o) ||
        !ToProjection(in.gate_up, &out.gate_up) ||
        !ToProjection(in.down, &out.down))
      return vx::Fail(vx::kInvalid,
                      "vx_forward_stack: layer " + std::to_string(i) +
                          " has a null or malformed weight");
  }
  vx::AttentionLayout l;
  l.positions = layout->positions;
  l.cache_rows = layout->cache_rows;
  l.rows_per_sequence = static_cast<int>(layout->rows_per_sequence);
  l.keys_per_sequence = static_cast<int>(layout->keys_per_sequence);
  l.past = static_cast<int>(layout->past);
  l.max_keys = cache->cache.capacity();
  l.causal = layout->causal != 0;
  vx::StackScratch s;
  s.normed = scratch->normed;
  s.qkv = scratch->qkv;
  s.q = scratch->q;
  s.attention = scratch->attention;
  s.gate_up = scratch->gate_up;
  s.activation = scratch->activation;
  return vx::Checked(vx::ForwardStack(w, rope, l, cache->cache, hidden, output,
                                      static_cast<int>(rows), s, stream),
                     "vx_forward_stack");
}

vx_status vx_project(const vx_projection* projection, const uint16_t* x,
                     float* y, size_t rows, cudaStream_t stream) {
  vx::Projection p;
  if (projection == nullptr || x == nullptr || y == nullptr ||
      !ToProjection(*projection, &p))
    return vx::Fail(vx::kInvalid, "vx_project: null or malformed argument");
  if (rows == 0)
    return VX_OK;
  return vx::Checked(vx::Project(p, x, y, static_cast<int>(rows), stream),
                     "vx_project");
}

}  // extern "C"
