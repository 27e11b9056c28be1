// C ABI of the stack kernels and the host-side math of the generation step
// (include/voxcpm_b200.h).
#include "stack_kernels.cuh"
#include "vx_status.h"

#include "../../include/voxcpm_b200.h"

#include <cmath>
#include <vector>

namespace {

vx::CacheType ToCache(int cache_type) {
  return cache_type == VX_CACHE_BF16 ? vx::CacheType::kBf16
                                     : vx::CacheType::kF32;
}

bool ValidCache(int cache_type) {
  return cache_type == VX_CACHE_F32 || cache_type == VX_CACHE_BF16;
}

}  // namespace

extern "C" {

vx_status vx_embed(const uint16_t* table, const int32_t* ids,
                   const int32_t* text_mask, float* output, size_t rows,
                   size_t width, float scale, cudaStream_t stream) {
  return vx::Checked(
      vx::Embed(table, ids, text_mask, output, rows, width, scale, stream),
      "vx_embed");
}

vx_status vx_scatter_rows(const float* input, const int32_t* indices,
                          float* output, size_t rows, size_t width,
                          cudaStream_t stream) {
  return vx::Checked(
      vx::ScatterRows(input, indices, output, rows, width, stream),
      "vx_scatter_rows");
}

vx_status vx_gather_rows(const float* input, const int32_t* indices,
                         float* output, size_t rows, size_t width,
                         cudaStream_t stream) {
  return vx::Checked(vx::GatherRows(input, indices, output, rows, width, stream),
                     "vx_gather_rows");
}

vx_status vx_rms_norm(const float* input, const uint16_t* weight,
                      uint16_t* output, float* output_f32, size_t rows,
                      size_t width, float epsilon, cudaStream_t stream) {
  return vx::Checked(vx::RmsNorm(input, weight, output, output_f32, rows,
                                 width, epsilon, stream),
                     "vx_rms_norm");
}

vx_status vx_qkv_rope(const float* qkv, const float* cos_sin,
                      const int32_t* positions, const int32_t* cache_rows,
                      float* q, void* k_cache, void* v_cache, int cache_type,
                      size_t rows, size_t heads, size_t kv_heads,
                      size_t head_dim, size_t capacity, cudaStream_t stream) {
  if (!ValidCache(cache_type))
    return vx::Fail(vx::kInvalid, "vx_qkv_rope: unknown cache type");
  return vx::Checked(
      vx::QkvRope(qkv, cos_sin, positions, cache_rows, q, k_cache, v_cache,
                  ToCache(cache_type), rows, heads, kv_heads, head_dim,
                  capacity, stream),
      "vx_qkv_rope");
}

vx_status vx_attention(const float* q, const void* k_cache,
                       const void* v_cache, int cache_type, uint16_t* output,
                       size_t rows, size_t rows_per_sequence,
                       size_t keys_per_sequence, size_t past,
                       const int32_t* past_device, int causal, size_t heads,
                       size_t kv_heads, size_t head_dim, size_t capacity,
                       size_t max_keys, cudaStream_t stream) {
  if (!ValidCache(cache_type))
    return vx::Fail(vx::kInvalid, "vx_attention: unknown cache type");
  return vx::Checked(
      vx::Attention(q, k_cache, v_cache, ToCache(cache_type), output, rows,
                    rows_per_sequence, keys_per_sequence, past, past_device,
                    causal != 0, heads, kv_heads, head_dim, capacity, max_keys,
                    stream),
      "vx_attention");
}

vx_status vx_swiglu(const float* gate_up, uint16_t* output, size_t rows,
                    size_t width, cudaStream_t stream) {
  return vx::Checked(vx::SwiGlu(gate_up, output, rows, width, stream),
                     "vx_swiglu");
}

vx_status vx_add_bias(float* data, const uint16_t* bias, size_t rows,
                      size_t width, cudaStream_t stream) {
  return vx::Checked(vx::AddBias(data, bias, rows, width, stream),
                     "vx_add_bias");
}

vx_status vx_to_bf16(const float* input, uint16_t* output, size_t count,
                     int silu, cudaStream_t stream) {
  return vx::Checked(vx::ToBf16(input, output, count, silu != 0, stream),
                     "vx_to_bf16");
}

vx_status vx_concat_rows(const float* a, const float* a_scale, size_t a_width,
                         const float* b, const float* b_scale, size_t b_width,
                         uint16_t* output, size_t rows, cudaStream_t stream) {
  return vx::Checked(vx::ConcatRows(a, a_scale, a_width, b, b_scale, b_width,
                                    output, rows, stream),
                     "vx_concat_rows");
}

vx_status vx_quantize(const float* input, uint16_t* output, size_t count,
                      float scale, cudaStream_t stream) {
  return vx::Checked(vx::Quantize(input, output, count, scale, stream),
                     "vx_quantize");
}

vx_status vx_select_rows(const float* quantized, const float* plain,
                         const int32_t* mask, float* output, size_t rows,
                         size_t width, cudaStream_t stream) {
  return vx::Checked(
      vx::SelectRows(quantized, plain, mask, output, rows, width, stream),
      "vx_select_rows");
}

vx_status vx_prepend_special(const float* rows_in, const uint16_t* special,
                             float* output, size_t patches, size_t patch_size,
                             size_t width, cudaStream_t stream) {
  return vx::Checked(vx::PrependSpecial(rows_in, special, output, patches,
                                        patch_size, width, stream),
                     "vx_prepend_special");
}

vx_status vx_assemble_dit(const float* mu, const float* time,
                          const float* cond, const float* x, float* output,
                          size_t patch_size, size_t width,
                          cudaStream_t stream) {
  return vx::Checked(
      vx::AssembleDit(mu, time, cond, x, output, patch_size, width, stream),
      "vx_assemble_dit");
}

vx_status vx_guided_euler(const float* velocity, float* x, size_t count,
                          float cfg, float dt, cudaStream_t stream) {
  return vx::Checked(vx::GuidedEuler(velocity, x, count, cfg, dt, stream),
                     "vx_guided_euler");
}

// ---------------------------------------------------------------- host math

vx_status vx_rope_table(double theta, size_t dim, const double* factors,
                        double scaling, size_t positions, float* table) {
  // transformer.cpp:20-45: inv_freq = 1 / theta^(2i / dim), angle =
  // position / factor_i * inv_freq_i, cos and sin scaled, in float32.
  if (factors == nullptr || table == nullptr || dim == 0 || dim % 2 != 0)
    return vx::Fail(vx::kInvalid, "vx_rope_table: bad arguments");
  const std::size_t half = dim / 2;
  std::vector<float> inverse(half);
  std::vector<float> factor_inverse(half);
  const auto scale = static_cast<float>(scaling);
  for (std::size_t i = 0; i < half; ++i) {
    const float exponent = static_cast<float>(2 * i) / static_cast<float>(dim);
    inverse[i] = 1.0f / std::pow(static_cast<float>(theta), exponent);
    factor_inverse[i] = 1.0f / static_cast<float>(factors[i]);
  }
  for (std::size_t p = 0; p < positions; ++p) {
    for (std::size_t i = 0; i < half; ++i) {
      const float angle =
          static_cast<float>(p) * factor_inverse[i] * inverse[i];
      table[p * dim + i] = std::cos(angle) * scale;
      table[p * dim + half + i] = std::sin(angle) * scale;
    }
  }
  return VX_OK;
}

size_t vx_euler_schedule(size_t timesteps, float sway, float* t_out,
                         float* dt_out, int32_t* evaluate, size_t capacity) {
  // generator.cpp:21-37 (torch.linspace in float32, two-sided) and :63-80
  // (sway sampling; CFG-Zero* skips max(1, int(0.04 (n + 1))) steps).
  const std::size_t n = timesteps + 1;
  std::vector<float> span(n);
  if (n == 1) {
    span[0] = 1.0f;
  } else {
    const float step = (0.0f - 1.0f) / static_cast<float>(n - 1);
    const std::size_t halfway = n / 2;
    for (std::size_t i = 0; i < n; ++i)
      span[i] = i < halfway ? 1.0f + step * static_cast<float>(i)
                            : 0.0f - step * static_cast<float>(n - i - 1);
  }
  const auto quarter_turn = static_cast<float>(M_PI / 2.0);
  for (float& v : span)
    v = v + sway * (std::cos(quarter_turn * v) - 1.0f + v);
  std::size_t zero_steps =
      static_cast<std::size_t>(static_cast<double>(n) * 0.04);
  if (zero_steps < 1)
    zero_steps = 1;
  float t = span[0];
  float dt = n > 1 ? span[0] - span[1] : 0.0f;
  std::size_t count = 0;
  for (std::size_t step = 1; step < n; ++step) {
    if (count < capacity) {
      if (t_out != nullptr)
        t_out[count] = t;
      if (dt_out != nullptr)
        dt_out[count] = dt;
      if (evaluate != nullptr)
        evaluate[count] = step > zero_steps ? 1 : 0;
    }
    ++count;
    t = t - dt;
    if (step < n - 1)
      dt = t - span[step + 1];
  }
  return count;
}

vx_status vx_sinusoid(float t, size_t width, float* out) {
  // generator.cpp:39-53: SinusoidalPosEmb(width)(t) with scale 1000.
  if (out == nullptr || width < 4 || width % 2 != 0)
    return vx::Fail(vx::kInvalid, "vx_sinusoid: bad arguments");
  const std::size_t half = width / 2;
  const auto exponent =
      static_cast<float>(std::log(10000.0) / static_cast<double>(half - 1));
  const float scaled = 1000.0f * t;
  for (std::size_t i = 0; i < half; ++i) {
    const float frequency = std::exp(static_cast<float>(i) * -exponent);
    const float angle = scaled * frequency;
    out[i] = std::sin(angle);
    out[half + i] = std::cos(angle);
  }
  return VX_OK;
}

}  // extern "C"
