/*
 * vxoracle — CPU restatement of the reference's per-patch generation path.
 * TEST INFRASTRUCTURE ONLY (see vxoracle.h): the checker of the parity tests
 * and the timed CPU baseline, never part of the product.
 *
 * Built with -ffp-contract=off so that a * b + c rounds twice unless a
 * function calls fmaf explicitly, as the reference's kernels do where it
 * matters (kernels/wmma_products.hip:206).
 */
#include "vxoracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------ numerics */

static uint32_t float_bits(float v) {
  uint32_t b;
  memcpy(&b, &v, 4);
  return b;
}

static float bits_float(uint32_t b) {
  float v;
  memcpy(&v, &b, 4);
  return v;
}

/* kernels/device_math.hpp:12-19: RNE, NaN kept quiet. */
uint16_t vxo_bf16_bits(float value) {
  const uint32_t bits = float_bits(value);
  if ((bits & 0x7F800000u) == 0x7F800000u && (bits & 0x007FFFFFu) != 0)
    return (uint16_t)((bits >> 16) | 0x40u);
  const uint32_t rounding = 0x7FFFu + ((bits >> 16) & 1u);
  return (uint16_t)((bits + rounding) >> 16);
}

float vxo_bf16_value(uint16_t bits) { return bits_float((uint32_t)bits << 16); }

/* IEEE binary16 decode, as tests/products_test.cpp:48-60. */
float vxo_half_value(uint16_t bits) {
  const uint32_t sign = (bits >> 15) & 1u;
  const uint32_t exponent = (bits >> 10) & 0x1Fu;
  const uint32_t mantissa = bits & 0x3FFu;
  float value;
  if (exponent == 0x1Fu)
    value = mantissa ? NAN : INFINITY;
  else if (exponent == 0)
    value = ldexpf((float)mantissa, -24);
  else
    value = ldexpf((float)(mantissa | 0x400u), (int)exponent - 25);
  return sign ? -value : value;
}

/* float -> binary16, round to nearest even (finite inputs of the weight
 * generator; overflow saturates to infinity). */
uint16_t vxo_half_bits(float value) {
  const uint32_t bits = float_bits(value);
  const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  const uint32_t abs_bits = bits & 0x7FFFFFFFu;
  if (abs_bits >= 0x7F800000u)
    return (uint16_t)(sign | 0x7C00u | (abs_bits > 0x7F800000u ? 0x200u : 0));
  const float a = bits_float(abs_bits);
  if (a >= 65520.0f)
    return (uint16_t)(sign | 0x7C00u);
  if (a < 6.103515625e-05f) {
    /* subnormal: value / 2^-24 rounded to nearest even integer */
    const float scaled = a * 16777216.0f; /* exact (power of two) */
    float r = rintf(scaled);              /* default mode: nearest even */
    return (uint16_t)(sign | (uint16_t)r);
  }
  const int exponent = (int)((abs_bits >> 23) & 0xFFu) - 127 + 15;
  uint32_t mantissa = abs_bits & 0x7FFFFFu;
  uint32_t half = ((uint32_t)exponent << 10) | (mantissa >> 13);
  const uint32_t rest = mantissa & 0x1FFFu;
  if (rest > 0x1000u || (rest == 0x1000u && (half & 1u)))
    half += 1; /* carries into the exponent correctly */
  return (uint16_t)(sign | half);
}

void vxo_to_bf16_array(const float* in, uint16_t* out, size_t count) {
  for (size_t i = 0; i < count; ++i)
    out[i] = vxo_bf16_bits(in[i]);
}

/* ------------------------------------------------------------ weights */

static uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint64_t vxo_hash(uint64_t seed, uint64_t tensor, uint64_t index) {
  return mix64(mix64(seed ^ (tensor * 0xD1B54A32D192ED03ull)) ^ index);
}

/* An approximately normal integer: the sum of four 16-bit uniforms, centred
 * (Irwin-Hall, standard deviation 65536 / sqrt(3)). */
static int32_t centred_sum(uint64_t h) {
  int32_t s = 0;
  for (int i = 0; i < 4; ++i)
    s += (int32_t)((h >> (16 * i)) & 0xFFFFu);
  return s - 131070;
}

#define VXO_SUM_STD 37837.226f /* 65536 / sqrt(3) */

void vxo_random_q8_0(uint64_t seed, uint64_t tensor, size_t rows, size_t in,
                     float scale_std, uint8_t* blocks) {
  const size_t count = rows * (in / 32);
  const float factor = scale_std / VXO_SUM_STD;
#pragma omp parallel for schedule(static)
  for (long b = 0; b < (long)count; ++b) {
    uint8_t* target = blocks + (size_t)b * 34;
    const uint64_t hs = vxo_hash(seed, tensor, ((uint64_t)1 << 62) | (uint64_t)b);
    const float scale = fabsf((float)centred_sum(hs)) * factor;
    const uint16_t bits = vxo_half_bits(scale);
    target[0] = (uint8_t)(bits & 0xFFu);
    target[1] = (uint8_t)(bits >> 8);
    for (int i = 0; i < 32; ++i) {
      const uint64_t h = vxo_hash(seed, tensor, (uint64_t)b * 32 + (uint64_t)i);
      const int q = (int)(h % 255u) - 127;
      target[2 + i] = (uint8_t)(int8_t)q;
    }
  }
}

void vxo_random_bf16(uint64_t seed, uint64_t tensor, size_t count, float mean,
                     float std, uint16_t* out) {
  const float factor = std / VXO_SUM_STD;
#pragma omp parallel for schedule(static)
  for (long i = 0; i < (long)count; ++i) {
    const float v = (float)centred_sum(vxo_hash(seed, tensor, (uint64_t)i)) *
                    factor;
    out[i] = vxo_bf16_bits(mean + v);
  }
}

/* ------------------------------------------------------------ tiles */

void vxo_q8_0_to_tiles(const uint8_t* blocks, size_t rows, size_t in,
                       uint8_t* tiles) {
  const size_t per_row = in / 32;
  const size_t padded = (rows + 15) / 16 * 16;
  for (size_t row = 0; row < padded; ++row) {
    for (size_t block = 0; block < per_row; ++block) {
      uint8_t* tile = tiles + ((row / 16) * per_row + block) * 544;
      const size_t r = row % 16;
      const size_t slot = r < 8 ? 2 * r : 2 * (r - 8) + 1;
      if (row < rows) {
        const uint8_t* source = blocks + (row * per_row + block) * 34;
        tile[512 + 2 * slot] = source[0];
        tile[512 + 2 * slot + 1] = source[1];
        for (int i = 0; i < 32; ++i)
          tile[32 * r + i] = (uint8_t)(source[2 + i] ^ 0x80u);
      } else {
        tile[512 + 2 * slot] = 0;
        tile[512 + 2 * slot + 1] = 0;
        for (int i = 0; i < 32; ++i)
          tile[32 * r + i] = 0x80u;
      }
    }
  }
}

void vxo_bf16_to_tiles(const uint16_t* w, size_t rows, size_t in,
                       uint16_t* tiles) {
  const size_t per_row = in / 32;
  const size_t padded = (rows + 15) / 16 * 16;
  for (size_t row = 0; row < padded; ++row)
    for (size_t k = 0; k < in; ++k)
      tiles[((row / 16) * per_row + k / 32) * 512 + (row % 16) * 32 + k % 32] =
          row < rows ? w[row * in + k] : 0;
}

void vxo_q8_0_dequant(const uint8_t* blocks, size_t rows, size_t in,
                      double* values) {
  const size_t count = rows * in / 32;
  for (size_t b = 0; b < count; ++b) {
    const uint8_t* source = blocks + b * 34;
    const double scale =
        vxo_half_value((uint16_t)(source[0] | (source[1] << 8)));
    for (int i = 0; i < 32; ++i)
      values[b * 32 + i] = scale * (double)(int8_t)source[2 + i];
  }
}

/* ------------------------------------------------------------ products */

static void set_threads(int threads) {
#ifdef _OPENMP
  if (threads > 0)
    omp_set_num_threads(threads);
#else
  (void)threads;
#endif
}

void vxo_product_exact(const uint16_t* x, int format, const void* w,
                       const float* before, double* exact, double* magnitude,
                       size_t rows, size_t in, size_t out, int threads) {
  set_threads(threads);
#pragma omp parallel
  {
    double* row_w = (double*)malloc(in * sizeof(double));
#pragma omp for schedule(static)
    for (long n = 0; n < (long)out; ++n) {
      if (format == VXO_Q8_0) {
        const uint8_t* blocks = (const uint8_t*)w + (size_t)n * (in / 32) * 34;
        vxo_q8_0_dequant(blocks, 1, in, row_w);
      } else {
        const uint16_t* r = (const uint16_t*)w + (size_t)n * in;
        for (size_t k = 0; k < in; ++k)
          row_w[k] = vxo_bf16_value(r[k]);
      }
      for (size_t m = 0; m < rows; ++m) {
        double sum = before ? before[m * out + n] : 0.0;
        double mag = 0.0;
        for (size_t k = 0; k < in; ++k) {
          const double product = (double)vxo_bf16_value(x[m * in + k]) * row_w[k];
          sum += product;
          mag += fabs(product);
        }
        exact[m * out + n] = sum;
        if (magnitude)
          magnitude[m * out + n] = mag;
      }
    }
    free(row_w);
  }
}

void vxo_linear(const uint16_t* x, int format, const void* w, float* y,
                size_t rows, size_t in, size_t out, int accumulate,
                int threads) {
  set_threads(threads);
  float* xf = (float*)malloc(rows * in * sizeof(float));
  for (size_t i = 0; i < rows * in; ++i)
    xf[i] = vxo_bf16_value(x[i]);
  const size_t k_blocks = in / 32;
#pragma omp parallel
  {
    float* acc = (float*)malloc(rows * sizeof(float));
    float* row_w = (float*)malloc(in * sizeof(float));
#pragma omp for schedule(static)
    for (long n = 0; n < (long)out; ++n) {
      for (size_t m = 0; m < rows; ++m)
        acc[m] = 0.0f;
      if (format == VXO_Q8_0) {
        const uint8_t* blocks = (const uint8_t*)w + (size_t)n * k_blocks * 34;
        for (size_t b = 0; b < k_blocks; ++b) {
          const uint8_t* block = blocks + b * 34;
          const float scale =
              vxo_half_value((uint16_t)(block[0] | (block[1] << 8)));
          float q[32];
          for (int i = 0; i < 32; ++i)
            q[i] = (float)(int8_t)block[2 + i];
          for (size_t m = 0; m < rows; ++m) {
            const float* xr = xf + m * in + b * 32;
            float sum = 0.0f;
            for (int i = 0; i < 32; ++i)
              sum += xr[i] * q[i]; /* exact products, float32 sums */
            acc[m] = fmaf(scale, sum, acc[m]);
          }
        }
      } else {
        const uint16_t* r = (const uint16_t*)w + (size_t)n * in;
        for (size_t k = 0; k < in; ++k)
          row_w[k] = vxo_bf16_value(r[k]);
        for (size_t m = 0; m < rows; ++m) {
          const float* xr = xf + m * in;
          float sum = 0.0f;
          for (size_t k = 0; k < in; ++k)
            sum += xr[k] * row_w[k];
          acc[m] = sum;
        }
      }
      for (size_t m = 0; m < rows; ++m) {
        float* target = y + m * out + (size_t)n;
        *target = accumulate ? *target + acc[m] : acc[m];
      }
    }
    free(acc);
    free(row_w);
  }
  free(xf);
}

/* ------------------------------------------------------------ stack kernels */

/* kernels/generator_kernels.hip:91-108 */
void vxo_rms_norm(const float* input, const uint16_t* weight, uint16_t* out,
                  float* out_f32, size_t rows, size_t width, float eps) {
  for (size_t row = 0; row < rows; ++row) {
    const float* x = input + row * width;
    float sum = 0.0f;
    for (size_t i = 0; i < width; ++i)
      sum += x[i] * x[i];
    const float inverse = 1.0f / sqrtf(sum / (float)width + eps);
    for (size_t i = 0; i < width; ++i) {
      const float value = x[i] * inverse * vxo_bf16_value(weight[i]);
      out[row * width + i] = vxo_bf16_bits(value);
      if (out_f32)
        out_f32[row * width + i] = value;
    }
  }
}

/* transformer.cpp:20-45 (float32 pow / cos / sin). */
void vxo_rope_table(double theta, size_t dim, const double* factors,
                    double scaling, size_t positions, float* table) {
  const size_t half = dim / 2;
  float* inverse = (float*)malloc(half * sizeof(float));
  float* factor_inverse = (float*)malloc(half * sizeof(float));
  const float scale = (float)scaling;
  for (size_t i = 0; i < half; ++i) {
    const float exponent = (float)(2 * i) / (float)dim;
    inverse[i] = 1.0f / powf((float)theta, exponent);
    factor_inverse[i] = 1.0f / (float)factors[i];
  }
  for (size_t p = 0; p < positions; ++p) {
    for (size_t i = 0; i < half; ++i) {
      const float angle = (float)p * factor_inverse[i] * inverse[i];
      table[p * dim + i] = cosf(angle) * scale;
      table[p * dim + half + i] = sinf(angle) * scale;
    }
  }
  free(inverse);
  free(factor_inverse);
}

/* kernels/generator_kernels.hip:110-158 */
void vxo_qkv_rope(const float* qkv, const float* cos_sin,
                  const int32_t* positions, const int32_t* cache_rows,
                  float* q, float* k_cache, float* v_cache, size_t rows,
                  size_t heads, size_t kv_heads, size_t head_dim,
                  size_t capacity) {
  const size_t half = head_dim / 2;
  const size_t width = (heads + 2 * kv_heads) * head_dim;
  for (size_t row = 0; row < rows; ++row) {
    const float* source = qkv + row * width;
    const float* table =
        cos_sin ? cos_sin + (size_t)positions[row] * head_dim : NULL;
    const size_t cache_row = (size_t)cache_rows[row];
    for (size_t head = 0; head < heads + kv_heads; ++head) {
      for (size_t i = 0; i < half; ++i) {
        const float a = source[head * head_dim + i];
        const float b = source[head * head_dim + half + i];
        float first = a, second = b;
        if (table) {
          const float c = table[i];
          const float s = table[half + i];
          first = a * c - b * s;
          second = b * c + a * s;
        }
        float* target = head < heads
                            ? q + (row * heads + head) * head_dim
                            : k_cache + ((head - heads) * capacity + cache_row) *
                                            head_dim;
        target[i] = first;
        target[half + i] = second;
      }
    }
    const float* v = source + (heads + kv_heads) * head_dim;
    for (size_t index = 0; index < kv_heads * head_dim; ++index) {
      const size_t head = index / head_dim;
      v_cache[(head * capacity + cache_row) * head_dim + index % head_dim] =
          v[index];
    }
  }
}

/* kernels/generator_kernels.hip:160-241: softmax attention of each row over
 * `past` cached keys plus its sequence's rows (up to itself when causal),
 * scale 1 / sqrt(head_dim), bf16 output. The reference merges four online
 * softmax partials; the result is the same softmax. */
void vxo_attention(const float* q, const float* k_cache, const float* v_cache,
                   uint16_t* out, size_t rows, size_t rows_per_sequence,
                   size_t keys_per_sequence, size_t past, int causal,
                   size_t heads, size_t kv_heads, size_t head_dim,
                   size_t capacity) {
  const float scale = 1.0f / sqrtf((float)head_dim);
  const size_t group = heads / kv_heads;
#pragma omp parallel
  {
    float* scores = NULL;
    size_t scores_size = 0;
    float* acc = (float*)malloc(head_dim * sizeof(float));
    float* query = (float*)malloc(head_dim * sizeof(float));
#pragma omp for collapse(2) schedule(static)
    for (long row = 0; row < (long)rows; ++row) {
      for (long head = 0; head < (long)heads; ++head) {
        const size_t sequence = (size_t)row / rows_per_sequence;
        const size_t local = (size_t)row % rows_per_sequence;
        const size_t count = past + (causal ? local + 1 : rows_per_sequence);
        const size_t first_key = sequence * keys_per_sequence;
        const size_t kv_head = (size_t)head / group;
        const float* keys = k_cache + (kv_head * capacity + first_key) * head_dim;
        const float* values =
            v_cache + (kv_head * capacity + first_key) * head_dim;
        if (count > scores_size) {
          free(scores);
          scores = (float*)malloc(count * sizeof(float));
          scores_size = count;
        }
        const float* qr = q + ((size_t)row * heads + (size_t)head) * head_dim;
        for (size_t d = 0; d < head_dim; ++d)
          query[d] = qr[d] * scale;
        float maximum = -INFINITY;
        for (size_t key = 0; key < count; ++key) {
          float s = 0.0f;
          for (size_t d = 0; d < head_dim; ++d)
            s += query[d] * keys[key * head_dim + d];
          scores[key] = s;
          if (s > maximum)
            maximum = s;
        }
        float total = 0.0f;
        for (size_t d = 0; d < head_dim; ++d)
          acc[d] = 0.0f;
        for (size_t key = 0; key < count; ++key) {
          const float weight = expf(scores[key] - maximum);
          total += weight;
          for (size_t d = 0; d < head_dim; ++d)
            acc[d] += weight * values[key * head_dim + d];
        }
        const float inverse = 1.0f / total;
        uint16_t* target = out + ((size_t)row * heads + (size_t)head) * head_dim;
        for (size_t d = 0; d < head_dim; ++d)
          target[d] = vxo_bf16_bits(acc[d] * inverse);
      }
    }
    free(scores);
    free(acc);
    free(query);
  }
}

/* kernels/generator_kernels.hip:243-254 */
void vxo_swiglu(const float* gate_up, uint16_t* out, size_t rows,
                size_t width) {
  for (size_t row = 0; row < rows; ++row)
    for (size_t i = 0; i < width; ++i) {
      const float gate = gate_up[row * 2 * width + i];
      const float up = gate_up[row * 2 * width + width + i];
      out[row * width + i] = vxo_bf16_bits(gate / (1.0f + expf(-gate)) * up);
    }
}

/* kernels/generator_kernels.hip:256-262 */
void vxo_add_bias(float* data, const uint16_t* bias, size_t rows,
                  size_t width) {
  for (size_t i = 0; i < rows * width; ++i)
    data[i] += vxo_bf16_value(bias[i % width]);
}

/* kernels/generator_kernels.hip:264-274 */
void vxo_to_bf16(const float* in, uint16_t* out, size_t count, int silu) {
  for (size_t i = 0; i < count; ++i) {
    float value = in[i];
    if (silu)
      value = value / (1.0f + expf(-value));
    out[i] = vxo_bf16_bits(value);
  }
}

/* kernels/generator_kernels.hip:276-289 */
void vxo_concat_rows(const float* a, const float* a_scale, size_t a_width,
                     const float* b, const float* b_scale, size_t b_width,
                     uint16_t* out, size_t rows) {
  const size_t width = a_width + b_width;
  for (size_t row = 0; row < rows; ++row) {
    const float sa = a_scale ? a_scale[row] : 1.0f;
    const float sb = b_scale ? b_scale[row] : 1.0f;
    for (size_t i = 0; i < width; ++i) {
      const float value = i < a_width ? a[row * a_width + i] * sa
                                      : b[row * b_width + i - a_width] * sb;
      out[row * width + i] = vxo_bf16_bits(value);
    }
  }
}

/* kernels/generator_kernels.hip:291-297: round half to even (rintf). */
void vxo_quantize(const float* in, uint16_t* out, size_t count, float scale) {
  for (size_t i = 0; i < count; ++i)
    out[i] = vxo_bf16_bits(rintf(tanhf(in[i]) * scale) / scale);
}

/* kernels/generator_kernels.hip:308-318 */
void vxo_prepend_special(const float* rows_in, const uint16_t* special,
                         float* out, size_t patches, size_t patch_size,
                         size_t width) {
  for (size_t patch = 0; patch < patches; ++patch)
    for (size_t row = 0; row <= patch_size; ++row) {
      float* target = out + (patch * (patch_size + 1) + row) * width;
      for (size_t i = 0; i < width; ++i)
        target[i] = row == 0 ? vxo_bf16_value(special[i])
                             : rows_in[(patch * patch_size + row - 1) * width + i];
    }
}

/* kernels/generator_kernels.hip:320-340 */
void vxo_assemble_dit(const float* mu, const float* time, const float* cond,
                      const float* x, float* out, size_t patch_size,
                      size_t width) {
  const size_t length = 3 + 2 * patch_size;
  for (size_t sequence = 0; sequence < 2; ++sequence)
    for (size_t row = 0; row < length; ++row) {
      float* target = out + (sequence * length + row) * width;
      for (size_t i = 0; i < width; ++i) {
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
}

/* kernels/generator_kernels.hip:81-89 */
void vxo_gather_rows(const float* in, const int32_t* indices, float* out,
                     size_t rows, size_t width) {
  for (size_t row = 0; row < rows; ++row)
    memcpy(out + row * width, in + (size_t)indices[row] * width,
           width * sizeof(float));
}

/* kernels/generator_kernels.hip:342-360 (CFG-Zero*, Euler). */
void vxo_guided_euler(const float* velocity, float* x, size_t count,
                      float cfg, float dt) {
  const float* c = velocity;
  const float* u = velocity + count;
  float dot = 0.0f, norm = 0.0f;
  for (size_t i = 0; i < count; ++i) {
    dot += c[i] * u[i];
    norm += u[i] * u[i];
  }
  const float s = dot / (norm + 1e-8f);
  for (size_t i = 0; i < count; ++i) {
    const float guided = u[i] * s + cfg * (c[i] - u[i] * s);
    x[i] -= dt * guided;
  }
}

/* generator.cpp:21-37: torch.linspace in float32. */
void vxo_linspace(float start, float end, size_t steps, float* out) {
  if (steps == 1) {
    out[0] = start;
    return;
  }
  const float step = (end - start) / (float)(steps - 1);
  const size_t halfway = steps / 2;
  for (size_t i = 0; i < steps; ++i)
    out[i] = i < halfway ? start + step * (float)i
                         : end - step * (float)(steps - i - 1);
}

/* generator.cpp:63-80 */
size_t vxo_euler_schedule(size_t timesteps, float sway, float* t_out,
                          float* dt_out, int32_t* evaluate, size_t capacity) {
  const size_t n = timesteps + 1;
  float* span = (float*)malloc(n * sizeof(float));
  vxo_linspace(1.0f, 0.0f, n, span);
  const float quarter_turn = (float)(M_PI / 2.0);
  for (size_t i = 0; i < n; ++i)
    span[i] = span[i] + sway * (cosf(quarter_turn * span[i]) - 1.0f + span[i]);
  size_t zero_steps = (size_t)((double)n * 0.04);
  if (zero_steps < 1)
    zero_steps = 1;
  float t = span[0];
  float dt = span[0] - span[1];
  size_t count = 0;
  for (size_t step = 1; step < n; ++step) {
    if (count < capacity) {
      t_out[count] = t;
      dt_out[count] = dt;
      evaluate[count] = step > zero_steps;
    }
    ++count;
    t = t - dt;
    if (step < n - 1)
      dt = t - span[step + 1];
  }
  free(span);
  return count;
}

/* generator.cpp:39-53 */
void vxo_sinusoid(float t, size_t width, float* out) {
  const size_t half = width / 2;
  const float exponent = (float)(log(10000.0) / (double)(half - 1));
  const float scaled = 1000.0f * t;
  for (size_t i = 0; i < half; ++i) {
    const float frequency = expf((float)i * -exponent);
    const float angle = scaled * frequency;
    out[i] = sinf(angle);
    out[half + i] = cosf(angle);
  }
}
