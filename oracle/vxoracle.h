/*
 * vxoracle — CPU restatement of the reference's per-patch generation path.
 *
 * TEST INFRASTRUCTURE ONLY. The parity tests, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference legs call it as the checker; the
 * product (libvoxcpm_b200.so) never links or calls it.
 *
 * Every function restates the arithmetic of a reference file (paths are
 * relative to the gufo-extensions/voxcpm tree) in plain C: float32 where the
 * reference computes in float32, double where its test oracle does, bf16
 * rounding at the same points (round to nearest even, quiet NaN).
 *
 * Parity status: the reference's HIP kernels cannot be built or run here, and
 * its OpenBMB golden tensors (tests/fixtures/generator_golden.safetensors)
 * need the 4.58 GB checkpoint, which is absent, so parity with OpenBMB's
 * outputs is UNPINNED. The oracle is pinned on the weight-free pieces: the
 * products test's double-precision oracle and metric
 * (tests/products_test.cpp:115-145), torch's float32 linspace / round /
 * conversions that generator.cpp restates (golden vectors generated with
 * torch, tests/golden/make_golden.py), and the Euler schedule values.
 */
#ifndef VXORACLE_H_
#define VXORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- numerics: kernels/device_math.hpp:12-24 */
uint16_t vxo_bf16_bits(float value);
float vxo_bf16_value(uint16_t bits);
float vxo_half_value(uint16_t bits);
uint16_t vxo_half_bits(float value);
void vxo_to_bf16_array(const float* in, uint16_t* out, size_t count);

/* ---- seeded synthetic weights (restates the library's vx_random_*) */
uint64_t vxo_hash(uint64_t seed, uint64_t tensor, uint64_t index);
void vxo_random_q8_0(uint64_t seed, uint64_t tensor, size_t rows, size_t in,
                     float scale_std, uint8_t* blocks);
void vxo_random_bf16(uint64_t seed, uint64_t tensor, size_t count, float mean,
                     float std, uint16_t* out);

/* ---- tiles of the library's format (restates its repack; geometry of
 * kernels/wmma_products.hip:62-92) */
void vxo_q8_0_to_tiles(const uint8_t* blocks, size_t rows, size_t in,
                       uint8_t* tiles);
void vxo_bf16_to_tiles(const uint16_t* w, size_t rows, size_t in,
                       uint16_t* tiles);
void vxo_q8_0_dequant(const uint8_t* blocks, size_t rows, size_t in,
                      double* values);

/* ---- products */
#define VXO_BF16_ROWS 0
#define VXO_Q8_0 2
/* products_test.cpp:115-145: exact = before + sum bf16(x) * w in double,
 * magnitude = sum |bf16(x) * w|. `w` is GGML Q8_0 blocks or bf16 rows. */
void vxo_product_exact(const uint16_t* x, int format, const void* w,
                       const float* before, double* exact, double* magnitude,
                       size_t rows, size_t in, size_t out, int threads);
/* The fp32 transcription of the device products: Q8_0 sums each 32-column
 * block in float32 and adds scale * sum with fmaf
 * (kernels/wmma_products.hip:201-214); bf16 keeps one float32 running sum
 * (kernels/skinny_gemm.hip:42-113). y (+)= x W^T. */
void vxo_linear(const uint16_t* x, int format, const void* w, float* y,
                size_t rows, size_t in, size_t out, int accumulate,
                int threads);

/* ---- generator kernels: kernels/generator_kernels.hip */
void vxo_rms_norm(const float* input, const uint16_t* weight, uint16_t* out,
                  float* out_f32, size_t rows, size_t width, float eps);
void vxo_rope_table(double theta, size_t dim, const double* factors,
                    double scaling, size_t positions, float* table);
void vxo_qkv_rope(const float* qkv, const float* cos_sin,
                  const int32_t* positions, const int32_t* cache_rows,
                  float* q, float* k_cache, float* v_cache, size_t rows,
                  size_t heads, size_t kv_heads, size_t head_dim,
                  size_t capacity);
void vxo_attention(const float* q, const float* k_cache, const float* v_cache,
                   uint16_t* out, size_t rows, size_t rows_per_sequence,
                   size_t keys_per_sequence, size_t past, int causal,
                   size_t heads, size_t kv_heads, size_t head_dim,
                   size_t capacity);
void vxo_swiglu(const float* gate_up, uint16_t* out, size_t rows,
                size_t width);
void vxo_add_bias(float* data, const uint16_t* bias, size_t rows,
                  size_t width);
void vxo_to_bf16(const float* in, uint16_t* out, size_t count, int silu);
void vxo_concat_rows(const float* a, const float* a_scale, size_t a_width,
                     const float* b, const float* b_scale, size_t b_width,
                     uint16_t* out, size_t rows);
void vxo_quantize(const float* in, uint16_t* out, size_t count, float scale);
void vxo_prepend_special(const float* rows_in, const uint16_t* special,
                         float* out, size_t patches, size_t patch_size,
                         size_t width);
void vxo_assemble_dit(const float* mu, const float* time, const float* cond,
                      const float* x, float* out, size_t patch_size,
                      size_t width);
void vxo_gather_rows(const float* in, const int32_t* indices, float* out,
                     size_t rows, size_t width);
void vxo_guided_euler(const float* velocity, float* x, size_t count,
                      float cfg, float dt);
/* generator.cpp:21-37, :63-80. Writes up to `capacity` steps; returns the
 * step count. */
size_t vxo_euler_schedule(size_t timesteps, float sway, float* t, float* dt,
                          int32_t* evaluate, size_t capacity);
void vxo_linspace(float start, float end, size_t steps, float* out);
/* generator.cpp:39-53 */
void vxo_sinusoid(float t, size_t width, float* out);

#ifdef __cplusplus
}
#endif

#endif /* VXORACLE_H_ */
