/*
 * voxcpm_b200 — the C ABI of a B200-native (sm_100a) VoxCPM2 per-patch
 * generation path: skinny Q8_0 / bf16 products, the MiniCPM4 stack kernels,
 * the local-DiT Euler/CFG sampler and the generation step.
 *
 * Every entry point replaces a function of the reference
 * (gufo-extensions/voxcpm); the comment above each one names the reference
 * interface it stands in for (file:line). Conventions:
 *  - Pointers are device pointers unless a comment says "host".
 *  - The caller owns every buffer it passes; handles own what they allocate.
 *  - bf16 values travel as uint16_t bit patterns.
 *  - Functions return a vx_status: VX_OK, VX_UNSUPPORTED (the reference's
 *    launchers returning false: the shape does not suit the kernels and
 *    nothing was launched), VX_INVALID (bad argument), VX_CUDA_ERROR (the
 *    reference throws GpuError there) or VX_DEVICE_TIMEOUT. vx_last_error()
 *    gives the calling thread's last message.
 *  - Work is enqueued on the given stream; nothing synchronizes unless a
 *    comment says so.
 */
#ifndef VOXCPM_B200_H_
#define VOXCPM_B200_H_

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define VX_API __attribute__((visibility("default")))
#else
#define VX_API
#endif

typedef int vx_status;
#define VX_OK 0
#define VX_UNSUPPORTED 1
#define VX_INVALID 2
#define VX_CUDA_ERROR 3
#define VX_DEVICE_TIMEOUT 4

/* Weight storage, matrix.hpp:9-13 (WeightFormat, same values). */
#define VX_WEIGHTS_BF16 0       /* bf16 [out][in], row-major */
#define VX_WEIGHTS_BF16_TILES 1 /* bf16 tiles of 16 rows x 32 columns */
#define VX_WEIGHTS_Q8_TILES 2   /* Q8_0 tiles: 16x32 int8 + 16 fp16 scales */

/* Output element type of a product. */
#define VX_OUT_F32 0
#define VX_OUT_BF16 1

/* The calling thread's last error message ("" if none). Replaces the text of
 * GpuError (device.hpp:16-30). */
VX_API const char* vx_last_error(void);

/* Reads and clears the device error bits set by a kernel whose bounded wait
 * expired (0: none). Synchronizes the device. No reference counterpart: the
 * reference's kernels have no bounded waits. */
VX_API vx_status vx_device_error(unsigned* bits);

/* Library version string. */
VX_API const char* vx_version(void);

/* ------------------------------------------------------------ tiles */

/* Bytes of Q8_0 / bf16 tiles of a [rows][in] matrix, rows padded to 16.
 * Replace Q8TilesBytes / Bf16TilesBytes (kernels/wmma_products.hpp:29-38). */
VX_API size_t vx_q8_tiles_bytes(size_t rows, size_t in);
VX_API size_t vx_bf16_tiles_bytes(size_t rows, size_t in);

/* GGML Q8_0 blocks ([rows][in/32] of {fp16 d, int8 q[32]}, 34 bytes) ->
 * Q8 tiles; padding rows are written too. Replaces Q8_0ToTiles
 * (kernels/wmma_products.hpp:55-59). */
VX_API vx_status vx_q8_0_to_tiles(const uint8_t* blocks, size_t rows, size_t in,
                           uint8_t* tiles, cudaStream_t stream);
/* bf16 [rows][in] -> bf16 tiles. Replaces Bf16ToTiles
 * (kernels/wmma_products.hpp:61-63). */
VX_API vx_status vx_bf16_to_tiles(const uint16_t* weights, size_t rows, size_t in,
                           uint16_t* tiles, cudaStream_t stream);
/* Q8 tiles -> bf16(scale * q) rows. Replaces Q8TilesToBf16
 * (kernels/wmma_products.hpp:65-68). */
VX_API vx_status vx_q8_tiles_to_bf16(const uint8_t* tiles, size_t rows, size_t in,
                              uint16_t* out, cudaStream_t stream);
/* bf16 tiles -> bf16 rows. Replaces Bf16TilesToRows
 * (kernels/wmma_products.hpp:70-72). */
VX_API vx_status vx_bf16_tiles_to_rows(const uint16_t* tiles, size_t rows, size_t in,
                                uint16_t* out, cudaStream_t stream);

/* ------------------------------------------------------------ products */

/* How a product is split. Replaces WmmaPlan (kernels/wmma_products.hpp:
 * 74-81). For the cluster plans (vx_plan_wmma) `splits` CTAs of one
 * thread-block cluster share each panel of weight rows and reduce on chip,
 * so partial_floats and counters are 0 (no scratch). For a spread plan
 * (variant VX_SPREAD_VARIANT, vx_plan_spread) `splits` is the CTA count,
 * `blocks_per_split` the longest run of (panel, block) units of one CTA, and
 * partial_floats / counters the split scratch the launch needs.
 * `variant` selects the kernel shape. */
typedef struct vx_wmma_plan {
  size_t splits;
  size_t blocks_per_split;
  size_t partial_floats;
  size_t counters;
  int variant;
} vx_wmma_plan;

/* Replaces SplitScratch (kernels/wmma_products.hpp:62-68): fp32 partial
 * sums and one counter per 128-row panel, owned by the caller. The counters
 * must be zero before the first launch that uses them; every launch leaves
 * them zero. Launches that share one scratch must be ordered on one stream
 * (the reference's rule). Cluster plans ignore it (may be all zero). */
typedef struct vx_split_scratch {
  float* partials;
  size_t partial_floats;
  unsigned* counters;
  size_t counter_count;
} vx_split_scratch;

/* The split of a product of `rows` rows over about `target_waves` CTAs
 * (0: the planner's choice). Replaces PlanWmma
 * (kernels/wmma_products.hpp:83-85). Returns a plan with splits 0 for a
 * shape the kernels do not serve. */
VX_API vx_wmma_plan vx_plan_wmma(size_t rows, size_t in, size_t out,
                          size_t target_waves);

/* The spread plan of a product of `rows` (at most 32) rows in the weight
 * format `format`: the product's (128-row panel, 32-column block) units cut
 * evenly over at most one CTA per SM, panels cut between CTAs added in part
 * order by the CTA that finishes last, through split scratch of
 * `partial_floats` floats and `counters` counters. splits 0 when the shape is
 * not served. Extends PlanWmma (kernels/wmma_products.hpp:83-85). */
#define VX_SPREAD_VARIANT 102
VX_API vx_wmma_plan vx_plan_spread(int format, size_t rows, size_t in,
                                   size_t out);
/* Whether products launched without a plan, with split scratch at hand
 * (vx_gemm_linear, or vx_wmma_q8 / vx_wmma_bf16 given scratch), take the
 * spread kernel (default off: in dependent chains it measured slower than
 * the planner's whole-reduction plans). No reference counterpart. */
VX_API void vx_set_spread_products(int enabled);
VX_API int vx_spread_products(void);

/* y[rows][out] (+)= x[rows][in] * W^T for bf16 x and Q8 tiles W, at most
 * 128 rows (the reference's kernel takes 32 per launch; 33..128 run in one
 * launch here), `in` a multiple of 32 (at most 8192). `plan` may be null
 * (the planner's choice: with `scratch` given and large enough, the spread
 * plan for up to 32 rows; else a cluster plan); `scratch` may be null except
 * for a spread plan. Replaces WmmaQ8 (kernels/wmma_products.hpp:87-93). */
VX_API vx_status vx_wmma_q8(const uint16_t* x, const uint8_t* w, float* y,
                     size_t rows, size_t in, size_t out, int accumulate,
                     const vx_wmma_plan* plan, const vx_split_scratch* scratch,
                     cudaStream_t stream);
/* The same for bf16 tiles. Replaces WmmaBf16
 * (kernels/wmma_products.hpp:95-99). */
VX_API vx_status vx_wmma_bf16(const uint16_t* x, const uint16_t* w, float* y,
                       size_t rows, size_t in, size_t out, int accumulate,
                       const vx_wmma_plan* plan,
                       const vx_split_scratch* scratch, cudaStream_t stream);
/* y (+)= x * W^T for bf16 rows W ([out][in]), at most 32 rows, `in` a
 * multiple of 8 and at most 8192 (the reference's SkinnyGemm contract);
 * other shapes return VX_UNSUPPORTED. Multiples of 32 run on the skinny
 * product kernels, other multiples of 8 on the general product (vx_matmul).
 * Replaces SkinnyGemm (kernels/skinny_gemm.hpp:18-24). */
VX_API vx_status vx_skinny_gemm(const uint16_t* x, const uint16_t* w, float* y,
                         size_t rows, size_t in, size_t out, int accumulate,
                         cudaStream_t stream);
/* SkinnyGemm with an explicit kernel shape (benchmarks): `vec` selects the
 * plan variant (negative: planner). Replaces SkinnyGemmWith
 * (kernels/skinny_gemm.hpp:26-30). */
VX_API vx_status vx_skinny_gemm_with(int vec, const uint16_t* x, const uint16_t* w,
                              float* y, size_t rows, size_t in, size_t out,
                              int accumulate, cudaStream_t stream);
/* Reads `pieces` 16-byte values with `blocks` CTAs (bandwidth probe).
 * Replaces ReadProbe (kernels/skinny_gemm.hpp:32-34). */
VX_API vx_status vx_read_probe(const void* data, size_t pieces, unsigned blocks,
                        unsigned* sink, cudaStream_t stream);

/* The general product: any weight format, fp32 or bf16 output
 * (`out_dtype`), at most 128 rows per launch. Extends WmmaQ8/WmmaBf16/
 * SkinnyGemm (kernels/wmma_products.hpp:87-99, kernels/skinny_gemm.hpp:
 * 18-24) with the bf16-output epilogue. */
VX_API vx_status vx_product(int format, const uint16_t* x, const void* w, void* y,
                     int out_dtype, size_t rows, size_t in, size_t out,
                     int accumulate, const vx_wmma_plan* plan,
                     cudaStream_t stream);

/* Flags of vx_product_ex. */
#define VX_PRODUCT_ACCUMULATE 1u
/* The launch reads nothing that earlier kernels on the stream write (x, w
 * and, when accumulating, y are ready before it is enqueued): it may overlap
 * them instead of waiting for their completion. With a null plan it takes
 * the library's measured plan for such streams where it has one. That plan
 * (config 0's shape) does its tile math in fp16 over rows scaled by a power
 * of two: bit-equal to the bf16 math for activations within 2^31 of their
 * row's largest magnitude; smaller ones are rounded to fp16 there, which can
 * change the last bits of a sum (within the products' 1e-5 limit). */
#define VX_PRODUCT_INDEPENDENT 2u

/* vx_product with flags (VX_PRODUCT_ACCUMULATE, VX_PRODUCT_INDEPENDENT).
 * Extends WmmaQ8/WmmaBf16/SkinnyGemm (kernels/wmma_products.hpp:87-99,
 * kernels/skinny_gemm.hpp:18-24). */
VX_API vx_status vx_product_ex(int format, const uint16_t* x, const void* w,
                               void* y, int out_dtype, size_t rows, size_t in,
                               size_t out, unsigned flags,
                               const vx_wmma_plan* plan, cudaStream_t stream);

/* A product whose activations and output live in page-locked host memory
 * (cudaHostAlloc, or cudaHostRegister'd: reachable from the device at the
 * same address): x_host [rows][in] bf16, y_host [rows][out] of out_dtype.
 * Three launches on `stream`: x_host is staged into x_dev (rows * in bf16 of
 * device memory), the product writes y_dev (rows * out of out_dtype, device
 * memory; read first when accumulating), and y_dev is staged into y_host.
 * The staging launches move 16-byte pieces with SM loads and stores over
 * PCIe, not the copy engines (faster for transfers of a few hundred KB; see
 * vx_stage). y_host holds the result once the stream has reached this
 * point. Flags: VX_PRODUCT_ACCUMULATE only (VX_PRODUCT_INDEPENDENT is
 * VX_INVALID: the product reads what the first launch wrote). Replaces the
 * upload, Linear and download a caller of the reference's products makes
 * (tests/products_test.cpp:100-110 around kernels/wmma_products.hpp:87-99). */
VX_API vx_status vx_product_host(int format, const uint16_t* x_host,
                                 uint16_t* x_dev, const void* w, void* y_dev,
                                 void* y_host, int out_dtype, size_t rows,
                                 size_t in, size_t out, unsigned flags,
                                 const vx_wmma_plan* plan, cudaStream_t stream);
/* Copies `bytes` from `src` to `dst`, either of which may be page-locked
 * host memory, with one launch of SM loads and stores (16-byte pieces where
 * both addresses and the size are multiples of 16). Ordered on `stream`
 * like a kernel. Replaces hipMemcpy (tests/products_test.cpp:100-110) for
 * transfers where the copy engines' per-copy cost dominates. */
VX_API vx_status vx_stage(void* dst, const void* src, size_t bytes,
                          cudaStream_t stream);

/* Programmatic dependent launch for every kernel of the library (default on).
 * No reference counterpart (HIP has none). */
VX_API void vx_set_programmatic_launch(int enabled);
/* Dependent product launches (the default) with more CTAs than a
 * same-shaped launch leaves SMs free start their first CTAs while the
 * previous product runs; with this on (default 1) those CTAs prefetch the
 * other CTAs' weights into L2. No reference counterpart. */
VX_API void vx_set_product_l2_prefetch(int enabled);
/* Whether the planner gives Q8_0 products of 9..32 rows to the tensor-core
 * (tcgen05) kernel, plan variant VX_TENSOR_CORE_VARIANT, or (default) to the
 * mma.sync kernels. A plan with that variant runs it either way. No reference counterpart (the reference has one
 * WMMA kernel, kernels/wmma_products.hip:139-296). */
#define VX_TENSOR_CORE_VARIANT 100
VX_API void vx_set_tensor_core_products(int enabled);
VX_API int vx_tensor_core_products(void);
/* Q8_0 products of 33..128 rows on the tcgen05 kernel for many rows: one
 * 128 x N MMA per K step (N = rows rounded up to 64, 96 or 128), every weight
 * byte read once, per-block fp32 sums scaled in block order. A plan with
 * variant VX_TENSOR_CORE_WIDE_VARIANT runs it for one call. With the switch
 * on (default), products launched without a plan take it where it measured
 * faster than the mma.sync kernels: more than 64 rows, in <= 1024 and
 * out >= 3072 (the DiT's gate/up products of batched slots). No reference
 * counterpart (the reference takes 32 rows per launch, wmma_products.hip). */
#define VX_TENSOR_CORE_WIDE_VARIANT 101
VX_API void vx_set_wide_tensor_core_products(int enabled);
VX_API int vx_wide_tensor_core_products(void);
/* Number of product kernel shapes and the shape of one (benchmarks). */
VX_API int vx_product_variants(void);
VX_API void vx_product_variant_shape(int variant, int* warps, int* groups,
                              int* stage, int* depth);

/* ------------------------------------------------------------ stack kernels */

/* KV cache element type: float32 (the reference's, transformer.hpp:17-36)
 * or bf16. Caches are [kv_head][capacity][head_dim] per layer. */
#define VX_CACHE_F32 0
#define VX_CACHE_BF16 1

/* Text rows take embedding[ids[row]] * scale, others zero. Replaces Embed
 * (kernels/generator_kernels.hpp:18-22). */
VX_API vx_status vx_embed(const uint16_t* table, const int32_t* ids,
                          const int32_t* text_mask, float* output, size_t rows,
                          size_t width, float scale, cudaStream_t stream);
/* output[indices[i]] = input[i]. Replaces ScatterRows
 * (kernels/generator_kernels.hpp:24-26). */
VX_API vx_status vx_scatter_rows(const float* input, const int32_t* indices,
                                 float* output, size_t rows, size_t width,
                                 cudaStream_t stream);
/* output[i] = input[indices[i]]. Replaces GatherRows
 * (kernels/generator_kernels.hpp:28-30). */
VX_API vx_status vx_gather_rows(const float* input, const int32_t* indices,
                                float* output, size_t rows, size_t width,
                                cudaStream_t stream);
/* bf16(weight * x * rsqrt(mean(x^2) + eps)) per row, optional fp32 copy.
 * Replaces RmsNorm (kernels/generator_kernels.hpp:32-36). */
VX_API vx_status vx_rms_norm(const float* input, const uint16_t* weight,
                             uint16_t* output, float* output_f32, size_t rows,
                             size_t width, float epsilon, cudaStream_t stream);
/* Splits [q | k | v] heads, rotates q and k by the cos/sin table row
 * positions[row] (no rotation when cos_sin is null), writes q
 * [rows][heads][head_dim] and appends k, v at cache_rows[row]. Replaces
 * QkvRope (kernels/generator_kernels.hpp:38-47). */
VX_API vx_status vx_qkv_rope(const float* qkv, const float* cos_sin,
                             const int32_t* positions,
                             const int32_t* cache_rows, float* q,
                             void* k_cache, void* v_cache, int cache_type,
                             size_t rows, size_t heads, size_t kv_heads,
                             size_t head_dim, size_t capacity,
                             cudaStream_t stream);
/* Softmax attention (head_dim 128, GQA) of each row over `past` cached keys
 * plus its sequence's rows (up to itself when causal); bf16 output
 * [rows][heads * 128]. With `past_device` non-null the kernel reads `past`
 * from device memory (graph replays) and `max_keys` bounds the keys per row.
 * Replaces Attention (kernels/generator_kernels.hpp:49-58). */
VX_API vx_status vx_attention(const float* q, const void* k_cache,
                              const void* v_cache, int cache_type,
                              uint16_t* output, size_t rows,
                              size_t rows_per_sequence,
                              size_t keys_per_sequence, size_t past,
                              const int32_t* past_device, int causal,
                              size_t heads, size_t kv_heads, size_t head_dim,
                              size_t capacity, size_t max_keys,
                              cudaStream_t stream);
/* bf16(silu(g) * u) of [rows][gate | up]. Replaces SwiGlu
 * (kernels/generator_kernels.hpp:60-62). */
VX_API vx_status vx_swiglu(const float* gate_up, uint16_t* output, size_t rows,
                           size_t width, cudaStream_t stream);
/* data[row][i] += bias[i]. Replaces AddBias
 * (kernels/generator_kernels.hpp:64-66). */
VX_API vx_status vx_add_bias(float* data, const uint16_t* bias, size_t rows,
                             size_t width, cudaStream_t stream);
/* bf16(x) or bf16(silu(x)). Replaces ToBf16
 * (kernels/generator_kernels.hpp:68-70). */
VX_API vx_status vx_to_bf16(const float* input, uint16_t* output, size_t count,
                            int silu, cudaStream_t stream);
/* bf16 rows [a * a_scale | b * b_scale] (null scales are 1). Replaces
 * ConcatRows (kernels/generator_kernels.hpp:72-76). */
VX_API vx_status vx_concat_rows(const float* a, const float* a_scale,
                                size_t a_width, const float* b,
                                const float* b_scale, size_t b_width,
                                uint16_t* output, size_t rows,
                                cudaStream_t stream);
/* FSQ: bf16(rint(tanh(x) * scale) / scale). Replaces Quantize
 * (kernels/generator_kernels.hpp:78-81). */
VX_API vx_status vx_quantize(const float* input, uint16_t* output, size_t count,
                             float scale, cudaStream_t stream);
/* mask ? quantized : plain, per row. Replaces SelectRows
 * (kernels/generator_kernels.hpp:83-86). */
VX_API vx_status vx_select_rows(const float* quantized, const float* plain,
                                const int32_t* mask, float* output,
                                size_t rows, size_t width,
                                cudaStream_t stream);
/* The local encoder's input: per patch a special row, then the projected
 * rows. Replaces PrependSpecial (kernels/generator_kernels.hpp:88-92). */
VX_API vx_status vx_prepend_special(const float* rows_in,
                                    const uint16_t* special, float* output,
                                    size_t patches, size_t patch_size,
                                    size_t width, cudaStream_t stream);
/* The DiT's CFG pair [mu_a, mu_b, time, cond x P, x x P] (unconditional mu
 * zero). Replaces AssembleDit (kernels/generator_kernels.hpp:94-99). */
VX_API vx_status vx_assemble_dit(const float* mu, const float* time,
                                 const float* cond, const float* x,
                                 float* output, size_t patch_size,
                                 size_t width, cudaStream_t stream);
/* CFG-Zero* guidance and the Euler step. Replaces GuidedEuler
 * (kernels/generator_kernels.hpp:101-107). */
VX_API vx_status vx_guided_euler(const float* velocity, float* x,
                                 size_t count, float cfg, float dt,
                                 cudaStream_t stream);

/* Host: the LongRoPE cos/sin table [positions][cos dim/2 | sin dim/2] in
 * float32. Replaces RopeTable (transformer.hpp:63-66, transformer.cpp:20-45). */
VX_API vx_status vx_rope_table(double theta, size_t dim, const double* factors,
                               double scaling, size_t positions, float* table);
/* Host: the Euler steps (t, dt, evaluate) of `timesteps` sway-sampled steps;
 * writes at most `capacity`, returns the count. Replaces EulerSchedule
 * (generator.hpp:43-44, generator.cpp:63-80). */
VX_API size_t vx_euler_schedule(size_t timesteps, float sway, float* t,
                                float* dt, int32_t* evaluate, size_t capacity);
/* Host: SinusoidalPosEmb(width)(t), scale 1000 (generator.cpp:39-53). */
VX_API vx_status vx_sinusoid(float t, size_t width, float* out);

/* ------------------------------------------------------------ generator */

/* One MiniCPM4 stack (config.hpp:15-31). */
typedef struct vx_stack_config {
  int hidden;
  int intermediate;
  int layers;
  int heads;
  int kv_heads;
  int head_dim; /* 128: the attention kernels need it (config.cpp:302-306) */
  float rms_eps;
  int rope;
} vx_stack_config;

/* ------------------------------------------------------------ transformer */

/* A linear layer y = x W^T (+ b): `format` one of VX_WEIGHTS_*, `weight` in
 * that layout, `bias` bf16 [out] or null. Replaces Projection
 * (weights.hpp:20-26). */
typedef struct vx_projection {
  int format;
  const void* weight;
  const uint16_t* bias;
  size_t in, out;
} vx_projection;
/* One pre-norm layer: bf16 norm weights, fused [q | k | v] and [gate | up].
 * Replaces LayerWeights (weights.hpp:28-36). */
typedef struct vx_layer_weights {
  const uint16_t* input_norm;
  vx_projection qkv, o;
  const uint16_t* post_norm;
  vx_projection gate_up, down;
} vx_layer_weights;
/* `config.layers` layers (host array) and the final norm. Replaces
 * StackWeights (weights.hpp:38-42). */
typedef struct vx_stack_weights {
  vx_stack_config config;
  const vx_layer_weights* layers;
  const uint16_t* norm;
} vx_stack_weights;
/* Which keys each row attends to; `positions` (rotary table rows) and
 * `cache_rows` are device arrays of one entry per row. Replaces
 * AttentionLayout (transformer.hpp:38-48). */
typedef struct vx_attention_layout {
  const int32_t* positions;
  const int32_t* cache_rows;
  size_t rows_per_sequence;
  size_t keys_per_sequence;
  size_t past;
  int causal;
} vx_attention_layout;
/* Device work buffers of ForwardStack, sized by vx_stack_scratch_elements.
 * Replaces StackScratch (transformer.hpp:50-58). */
typedef struct vx_stack_scratch {
  uint16_t* normed;
  float* qkv;
  float* q;
  uint16_t* attention;
  float* gate_up;
  uint16_t* activation;
} vx_stack_scratch;
/* Elements each vx_stack_scratch buffer needs for `rows` rows of `config`,
 * in field order (normed, qkv, q, attention, gate_up, activation). */
VX_API vx_status vx_stack_scratch_elements(const vx_stack_config* config,
                                           size_t rows, size_t counts[6]);

/* Keys and values of one stack, [layer][kv_head][capacity][head_dim] each,
 * float32 (VX_CACHE_F32) or bf16 (VX_CACHE_BF16); zeroed at creation.
 * Replaces KvCache (transformer.hpp:17-36). Null on failure
 * (vx_last_error). */
typedef struct vx_kv_cache vx_kv_cache;
VX_API vx_kv_cache* vx_kv_cache_create(const vx_stack_config* config,
                                       size_t capacity, int cache_type);
VX_API void vx_kv_cache_destroy(vx_kv_cache* cache);
VX_API size_t vx_kv_cache_capacity(const vx_kv_cache* cache);
/* Layer `layer`'s keys / values (null for a layer out of range). */
VX_API void* vx_kv_cache_keys(const vx_kv_cache* cache, size_t layer);
VX_API void* vx_kv_cache_values(const vx_kv_cache* cache, size_t layer);

/* One MiniCPM4 stack over `rows` rows of the float32 residual stream
 * `hidden` (updated in place); the final norm's float32 output goes to
 * `output`. `rope` is the device rotary table ([position][cos | sin]), null
 * for a stack without rotary embedding. Replaces ForwardStack
 * (transformer.hpp:68-71, transformer.cpp:55-100). */
VX_API vx_status vx_forward_stack(const vx_stack_weights* stack,
                                  const float* rope,
                                  const vx_attention_layout* layout,
                                  vx_kv_cache* cache, float* hidden,
                                  float* output, size_t rows,
                                  const vx_stack_scratch* scratch,
                                  cudaStream_t stream);
/* y[rows][out] = x[rows][in] W^T + b for bf16 x. Replaces Project
 * (transformer.hpp:73-76, transformer.cpp:47-53). */
VX_API vx_status vx_project(const vx_projection* projection,
                            const uint16_t* x, float* y, size_t rows,
                            cudaStream_t stream);

/* The generator's configuration (config.hpp:78-92). */
typedef struct vx_model_config {
  vx_stack_config lm, residual_lm, encoder, dit;
  double rope_theta;
  double rope_scaling;
  double rope_factors[64]; /* head_dim / 2 LongRoPE factors */
  int patch_size;
  int feat_dim;
  int fsq_latent_dim;
  float fsq_scale;
  int max_length; /* positions of each LM cache */
  int vocab;      /* embedding rows (0: no embedding table, prefill of audio
                     rows only) */
} vx_model_config;

/* Matrix formats of a seeded checkpoint: like a GGUF Q8_0 one (every matrix
 * Q8 tiles) or like the HF bf16 one (the DiT in bf16 tiles, the rest bf16
 * rows) (weights.cpp:138-144, :281-282). */
#define VX_CHECKPOINT_Q8 0
#define VX_CHECKPOINT_BF16 1

/* The released checkpoint's shapes (tests/config_test.cpp:36-67); LongRoPE
 * factors 1 and vocab 0 (set them for real use). */
VX_API void vx_model_config_released(vx_model_config* config);

/* VoxCPM2's generator on the current device with seeded weights (benchmarks
 * and parity tests; vx_generator_create_from_files reads checkpoint files).
 * Generator::Create (generator.hpp:60-62, generator.cpp:82-174) with a
 * seeded weight source. Returns null on failure (vx_last_error). */
typedef struct vx_generator vx_generator;
VX_API vx_generator* vx_generator_create(const vx_model_config* config,
                                         uint64_t seed, int checkpoint,
                                         int cache_type);
VX_API void vx_generator_destroy(vx_generator* generator);
/* Host arrays: tokens, masks [rows], feats [rows][patch][feat]. Replaces
 * Generator::Prefill (generator.hpp:73-74, generator.cpp:326-422). */
VX_API vx_status vx_generator_prefill(vx_generator* generator,
                                      const int32_t* tokens,
                                      const int32_t* text_mask,
                                      const int32_t* audio_mask,
                                      const float* feats, size_t rows);
/* Host noise [patch][feat]; writes the stop logits [2] of the state before
 * the patch and (when not null) its latent [patch][feat], then advances
 * both LMs. One CUDA graph per patch when graphs are on (default).
 * Synchronizes. Replaces Generator::Step (generator.hpp:76-86,
 * generator.cpp:424-513). */
VX_API vx_status vx_generator_step(vx_generator* generator, const float* noise,
                                   size_t timesteps, float cfg, float* latent,
                                   float* stop_logits);
/* Host arrays: mu [2 * dit hidden], cond and x [patch][feat]; writes the
 * CFG pair of velocities [2][patch][feat]. Replaces Generator::Velocity
 * (generator.hpp:88-91, generator.cpp:515-538). */
VX_API vx_status vx_generator_velocity(vx_generator* generator,
                                       const float* mu, const float* cond,
                                       const float* x, float t,
                                       float* velocity);
/* The DiT part of a step with the conditioning given (host mu, prefix cond,
 * noise): dit_cond, then the Euler/CFG steps (generator.cpp:448-463);
 * writes the latent when `latent` is not null (synchronizing; then
 * VX_DEVICE_TIMEOUT when the persistent kernel's launch aborted). */
VX_API vx_status vx_generator_dit_patch(vx_generator* generator,
                                        const float* mu, const float* cond,
                                        const float* noise, size_t timesteps,
                                        float cfg, float* latent);
/* The DiT patch of vx_generator_dit_patch for callers that must not allocate
 * device memory while generating: a host that sized all of its GPU memory at
 * start-up, or a real-time audio loop that cannot wait on the driver's
 * allocator. No reference counterpart. All arrays are DEVICE pointers: mu
 * [2][dit hidden], cond and noise [patch][feat] in, latent [patch][feat] out.
 * The persistent kernel's work buffers live in a fixed 1 MiB device array of
 * the library instead of the generator's own allocation; the call allocates
 * nothing. Needs the persistent kernel (a generator whose DiT has another
 * shape gets VX_INVALID) and a schedule prepared by an earlier
 * vx_generator_dit_patch or vx_generator_step with the same `timesteps`
 * (else VX_INVALID). The first call on a device looks the array's address up
 * (make that first call before any stream capture). Calls that overlap on
 * the GPU, from any generator, share the array and race. The inputs are
 * copied on the generator's own stream, which is not ordered after the
 * caller's streams: mu, cond and noise must be completely written before the
 * call (synchronize the stream that produced them). Synchronizes the
 * generator's stream. Returns VX_DEVICE_TIMEOUT (the latent is not valid)
 * when one of the kernel's bounded waits gave up and the launch aborted. */
VX_API vx_status vx_generator_dit_patch_static(vx_generator* generator,
                                               const float* mu,
                                               const float* cond,
                                               const float* noise,
                                               size_t timesteps, float cfg,
                                               float* latent);
/* Test hook: every later persistent DiT launch of this process first makes
 * one thread wait for a device word that nothing sets, for at most
 * `limit_ns` nanoseconds, then abort the launch as a real time-out would, so
 * tests can check that the entries report VX_DEVICE_TIMEOUT without a GPU
 * fault (0: off, the default). No reference counterpart. */
VX_API void vx_set_dit_stall_for_tests(uint64_t limit_ns);
/* Replays the last DiT patch (its captured graph) on the generator's stream
 * without synchronizing (benchmarks). */
VX_API vx_status vx_generator_replay_dit_patch(vx_generator* generator);
/* Host copies of internal state (tests, benchmarks): names "lm_hidden",
 * "residual_hidden", "prefix_cond", "x", "mu", "stop", "embed", "cond_rows",
 * "velocity", "delta_time", "lm_output" (the LM's last row before FSQ), and
 * the LM caches "base_cache_k", "base_cache_v", "residual_cache_k",
 * "residual_cache_v" ([layer][kv_head][capacity][head_dim] as float, bf16
 * caches widened); set_state takes "lm_hidden", "residual_hidden",
 * "prefix_cond", "mu" and "position" (one value). Stands in for
 * Generator::set_trace (generator.hpp:93-94). */
VX_API vx_status vx_generator_state(vx_generator* generator, const char* name,
                                    float* out, size_t count);
VX_API vx_status vx_generator_set_state(vx_generator* generator,
                                        const char* name, const float* in,
                                        size_t count);
/* CUDA graphs for Step and the DiT patch (default on). */
VX_API vx_status vx_generator_set_graphs(vx_generator* generator, int enabled);
/* The DiT patch as one persistent cooperative kernel (default on when the
 * DiT has VoxCPM2's shape: hidden 1024, FFN 4096, 16/2 heads of 128, patch
 * 4 x 64) or as the per-kernel sequence (generator.cpp:297-324, :457-463).
 * Enabling it for another DiT shape returns VX_UNSUPPORTED. No reference
 * counterpart: the reference always runs the per-kernel sequence. */
VX_API vx_status vx_generator_set_persistent(vx_generator* generator,
                                             int enabled);
/* 1 when the DiT patch runs as the persistent kernel. */
VX_API int vx_generator_persistent(const vx_generator* generator);
/* Caps the CTAs of the persistent DiT and stack kernels launched from now on
 * (0: no cap, the default: as many as the occupancy query says co-reside;
 * below a kernel's minimum of 128 CTAs the minimum). Graphs captured before
 * keep their grids. For tuning and for profilers that hold back resources.
 * No reference counterpart. */
VX_API void vx_set_persistent_max_ctas(size_t ctas);
/* Whether the persistent kernels launch with the cooperative attribute
 * (default 1). With 0 their CTAs' co-residency rests on the grid fitting
 * an idle GPU (one CTA per SM); when it does not, the kernels' bounded waits
 * end the step with VX_DEVICE_TIMEOUT instead of waiting for good. For
 * profilers that cannot replay cooperative launches with thread-block
 * clusters. No reference counterpart. */
VX_API void vx_set_persistent_cooperative(int enabled);
/* Rows in the caches (Generator::position, generator.hpp:69-70). */
VX_API size_t vx_generator_position(const vx_generator* generator);
/* The last patch's latent [patch][feat] in device memory, valid until the
 * step after next (two slots alternate), ready once the event of
 * vx_generator_latent_event completes; null before the first step of a
 * sequence. Replaces Generator::latent (generator.hpp:78-84). */
VX_API const float* vx_generator_latent(const vx_generator* generator);
/* The event recorded on the generator's stream after the last step's
 * launches. Replaces Generator::latent_event (generator.hpp:84). */
VX_API cudaEvent_t vx_generator_latent_event(const vx_generator* generator);
VX_API size_t vx_generator_weight_bytes(const vx_generator* generator);
VX_API cudaStream_t vx_generator_stream(const vx_generator* generator);

/* ------------------------------------------------------------ batched slots */

typedef struct vx_model_files vx_model_files; /* checkpoint files, below */

/* Several requests generated together on the current device: `slots`
 * generators that share one set of weights and one stream, each with its own
 * caches and state. A step advances every active slot by one patch: their
 * DiT passes run as one pass of 22 rows per slot (the DiT's weights are read
 * once per Euler evaluation for all of them) and their local encoder as one
 * call; each slot's LMs advance on its own caches. No reference counterpart:
 * it batches the per-request loop of synthesizer.cpp:283-307 (one
 * Generator::Step per request). Seeded weights, or the files' with
 * _from_files. Null on failure. */
typedef struct vx_generator_batch vx_generator_batch;
VX_API vx_generator_batch* vx_generator_batch_create(
    const vx_model_config* config, uint64_t seed, int checkpoint,
    int cache_type, size_t slots);
VX_API vx_generator_batch* vx_generator_batch_create_from_files(
    const vx_model_config* config, const vx_model_files* files,
    int cache_type, size_t slots);
VX_API void vx_generator_batch_destroy(vx_generator_batch* batch);
VX_API size_t vx_generator_batch_slots(const vx_generator_batch* batch);
/* A new request in `slot` (Generator::Prefill; the other slots keep their
 * state). Synchronizes. */
VX_API vx_status vx_generator_batch_prefill(vx_generator_batch* batch,
                                            size_t slot, const int32_t* tokens,
                                            const int32_t* text_mask,
                                            const int32_t* audio_mask,
                                            const float* feats, size_t rows);
/* One patch for every slot with active[slot] != 0 (host arrays: active
 * [slots], noise [slots][patch][feat]); writes those slots' latents
 * [slots][patch][feat] (when not null) and stop logits [slots][2]. One CUDA
 * graph per set of active slots. Synchronizes once. VX_INVALID when an
 * active slot has no prefilled request or no room. */
VX_API vx_status vx_generator_batch_step(vx_generator_batch* batch,
                                         const int32_t* active,
                                         const float* noise, size_t timesteps,
                                         float cfg, float* latents,
                                         float* stop_logits);
VX_API size_t vx_generator_batch_position(const vx_generator_batch* batch,
                                          size_t slot);
/* vx_generator_state of one slot. */
VX_API vx_status vx_generator_batch_state(vx_generator_batch* batch,
                                          size_t slot, const char* name,
                                          float* out, size_t count);
VX_API vx_status vx_generator_batch_set_graphs(vx_generator_batch* batch,
                                               int enabled);
VX_API cudaStream_t vx_generator_batch_stream(const vx_generator_batch* batch);

/* ------------------------------------------------------------ AudioVAE */

/* The decoder fields of AudioVaeConfig (config.hpp:53-72): latent frames of
 * `latent_dim` to mono audio at `out_sample_rate`, through one block per
 * decoder rate (each halves the channels and multiplies the frames by its
 * rate), conditioned on the rate's bucket among `sr_bin_boundaries`. */
typedef struct vx_vae_config {
  size_t latent_dim;
  size_t decoder_dim;
  size_t decoder_rates[8];
  size_t decoder_rate_count;
  size_t out_sample_rate;
  size_t sr_bin_boundaries[8];
  size_t sr_bin_boundary_count;
} vx_vae_config;
/* The released AudioVAE V2: latent 64, decoder 2048, rates 8 6 5 2 2 2,
 * 48 kHz out, boundaries 20000 30000 40000. */
VX_API void vx_vae_config_default(vx_vae_config* config);

/* The AudioVAE V2 decoder in float32 on its own stream, chunk by chunk with
 * the state of every causal convolution carried between calls (decoding a
 * stream in chunks gives the samples of decoding it at once, up to float32
 * rounding; the same chunks give the same samples bit for bit). Weights are
 * the seeded AudioVAE checkpoint of `seed` (bf16 values of the seeded
 * hash, tensor ids FNV-1a of "audio_vae." + name), packed as the decoder
 * reads them. Replaces AudioVae (vae.hpp:25-79) for decoding; null on
 * failure (vx_last_error). */
typedef struct vx_audio_vae vx_audio_vae;
VX_API vx_audio_vae* vx_audio_vae_create(const vx_vae_config* config,
                                         uint64_t seed);
VX_API void vx_audio_vae_destroy(vx_audio_vae* vae);
/* Output samples per latent frame (AudioVaeConfig::decode_hop). */
VX_API size_t vx_audio_vae_decode_hop(const vx_audio_vae* vae);
VX_API cudaStream_t vx_audio_vae_stream(const vx_audio_vae* vae);
/* A new stream: zero history (AudioVae::Reset, vae.cpp:363-368). */
VX_API vx_status vx_audio_vae_reset(vx_audio_vae* vae);
/* Decodes `frames` host latent frames [frames][latent_dim] into
 * frames * decode_hop host samples (AudioVae::Decode, vae.cpp:382-393).
 * VX_INVALID while an enqueued decoding is pending. */
VX_API vx_status vx_audio_vae_decode(vx_audio_vae* vae, const float* latents,
                                     size_t frames, float* audio);
/* Queues the decoding of `frames` device latent frames on the AudioVAE's
 * stream once `ready` (may be null; e.g. vx_generator_latent_event) has
 * completed; the latents are copied before anything else, so the generator
 * may overwrite them afterwards. One decoding may be pending: VX_INVALID
 * while one is (the reference would overwrite it). AudioVae::Enqueue
 * (vae.cpp:395-407). */
VX_API vx_status vx_audio_vae_enqueue(vx_audio_vae* vae, const float* latents,
                                      size_t frames, cudaEvent_t ready);
/* Waits for the pending decoding and copies its samples (frames *
 * decode_hop, 0 when none is pending) into `audio`; `*samples` is how many.
 * VX_INVALID when `capacity` is smaller. AudioVae::Collect (vae.cpp:409-
 * 413). */
VX_API vx_status vx_audio_vae_collect(vx_audio_vae* vae, float* audio,
                                      size_t capacity, size_t* samples);

/* ------------------------------------------------------------ model files */

/* Tensor element types (safetensors.hpp:18, same order). Q8_0 is GGML's
 * 34-byte block: an fp16 scale, then 32 int8 values. */
#define VX_DTYPE_F32 0
#define VX_DTYPE_BF16 1
#define VX_DTYPE_F16 2
#define VX_DTYPE_I64 3
#define VX_DTYPE_I32 4
#define VX_DTYPE_U8 5
#define VX_DTYPE_Q8_0 6

/* Components of the files: the generator's tensors (model.safetensors names)
 * and the AudioVAE's (read from a GGUF only; not used by the generator). */
#define VX_COMPONENT_MODEL 0
#define VX_COMPONENT_VAE 1

/* One tensor (safetensors.hpp:23-34). `name` and `data` stay valid while
 * the files are open; `data` is host memory in the mapped file; `shape` is
 * outermost first; `offset` is the tensor's byte position in its file. */
typedef struct vx_tensor_info {
  const char* name;
  int dtype;
  int rank;
  uint64_t shape[8];
  const void* data;
  uint64_t bytes;
  uint64_t offset;
} vx_tensor_info;

/* The checkpoint files: a Hugging Face directory (config.json,
 * model.safetensors, tokenizer.json when present) or an audio.cpp VoxCPM2
 * GGUF file (GGUF v2/v3, config and tokenizer embedded, abbreviated tensor
 * names resolved). Host only. Replaces ModelFiles::Open
 * (model_files.hpp:45-51, model_files.cpp:111-180); null on failure
 * (vx_last_error names the file and the problem). */
VX_API vx_model_files* vx_model_files_open(const char* path);
VX_API void vx_model_files_close(vx_model_files* files);
/* ModelFiles::IsVoxCpm2Gguf (model_files.hpp:49-51): a .gguf file whose
 * header names audio.cpp's VoxCPM2 layout. */
VX_API int vx_model_files_is_voxcpm2_gguf(const char* path);
VX_API int vx_model_files_is_gguf(const vx_model_files* files);
/* config.json / tokenizer.json text (ModelFiles::config, ::tokenizer; the
 * tokenizer is empty when a directory has none). */
VX_API const char* vx_model_files_config(const vx_model_files* files);
VX_API const char* vx_model_files_tokenizer(const vx_model_files* files);
VX_API size_t vx_model_files_count(const vx_model_files* files, int component);
VX_API vx_status vx_model_files_tensor(const vx_model_files* files,
                                       int component, size_t index,
                                       vx_tensor_info* info);
/* ModelFiles::Model / ::Vae (model_files.hpp:60-63); VX_INVALID when
 * absent. */
VX_API vx_status vx_model_files_find(const vx_model_files* files,
                                     int component, const char* name,
                                     vx_tensor_info* info);

/* Parses config.json text into the generator's configuration and checks
 * that the kernels serve it. Replaces ParseConfig + IsSupported
 * (config.hpp:89-98, config.cpp:144-323). `max_length` is config.json's
 * max_length; the LongRoPE factors and scale are those the reference
 * applies. VX_INVALID with the key named on failure. */
VX_API vx_status vx_parse_config(const char* json, size_t length,
                                 vx_model_config* config);

/* The generator with the files' weights (Generator::Create(config, files),
 * generator.hpp:60-62): every model tensor must be one the generator takes,
 * with the expected shape (weights.cpp:187-197, :316-318). Matrices become
 * Q8 tiles when Q8_0, bf16 tiles in the DiT and bf16 rows elsewhere
 * (weights.cpp:44-144); F16/F32/Q8_0 vectors are converted to bf16 on the
 * device. The files may be closed afterwards. Null on failure. */
VX_API vx_generator* vx_generator_create_from_files(
    const vx_model_config* config, const vx_model_files* files,
    int cache_type);

/* Device conversions to bf16, round to nearest even with NaN kept quiet
 * (kernels/convert_kernels.hpp:12-23). Device arrays; `count` values (a
 * multiple of 32 for Q8_0). */
VX_API vx_status vx_half_to_bf16(const uint16_t* input, uint16_t* output,
                                 size_t count, cudaStream_t stream);
VX_API vx_status vx_float_to_bf16(const float* input, uint16_t* output,
                                  size_t count, cudaStream_t stream);
VX_API vx_status vx_q8_0_to_bf16(const uint8_t* blocks, uint16_t* output,
                                 size_t count, cudaStream_t stream);

/* ------------------------------------------------------------ synthetic weights */

/* Host: GGML Q8_0 blocks [rows][in/32] of seeded random weights, a pure
 * function of (seed, tensor, index): q uniform in [-127, 127], one fp16
 * scale |N(0, scale_std)| per 32 values. The seeded checkpoint of
 * vx_generator_create (no released checkpoint is available here). */
VX_API vx_status vx_random_q8_0(uint64_t seed, uint64_t tensor, size_t rows,
                         size_t in, float scale_std, uint8_t* blocks);
/* Host: `count` seeded bf16 values bf16(mean + N(0, std)). */
VX_API vx_status vx_random_bf16(uint64_t seed, uint64_t tensor, size_t count,
                         float mean, float std, uint16_t* out);

/* ------------------------------------------------------------ Bf16Gemm */

/* Product dispatch by weight format and row count. Replaces Bf16Gemm
 * (gemm.hpp:49-72); one instance per stream. */
typedef struct vx_gemm vx_gemm;
VX_API vx_gemm* vx_gemm_create(cudaStream_t stream);
/* Synchronizes the gemm's stream (launches may still use its scratch), so
 * the stream must outlive the gemm. */
VX_API void vx_gemm_destroy(vx_gemm* gemm);
/* y[rows][out] (+)= x[rows][in] * w[out][in]^T, float32 y. Up to 128 rows
 * run in one launch on the planner's plan (the spread product through the
 * gemm's own split scratch when vx_set_spread_products is on), more in
 * chunks of 128.
 * bf16 rows with `in` not a multiple of 32 run on the general product, as
 * the reference's LinearRows falls back to Matmul. Replaces Bf16Gemm::Linear
 * (gemm.hpp:51-58, gemm.cpp:259-336). vx_gemm_create allocates the scratch
 * (about 5 MB); where it cannot (no device), the gemm serves every shape on
 * the cluster plans, which need none. */
VX_API vx_status vx_gemm_linear(vx_gemm* gemm, const uint16_t* x, int format,
                         const void* w, float* y, size_t rows, size_t in,
                         size_t out, int accumulate);

/* vx_gemm_linear with the output type `out_dtype` (VX_OUT_F32 or
 * VX_OUT_BF16: bf16 of the fp32 sum, BASELINE config 0's epilogue) and
 * flags (VX_PRODUCT_ACCUMULATE). bf16 output needs `in` a multiple of 32.
 * Extends Bf16Gemm::Linear (gemm.hpp:51-58). */
VX_API vx_status vx_gemm_linear_ex(vx_gemm* gemm, const uint16_t* x, int format,
                                   const void* w, void* y, int out_dtype,
                                   size_t rows, size_t in, size_t out,
                                   unsigned flags);

/* vx_gemm_linear_ex with activations and output in page-locked host memory
 * (as vx_product_host): x_host is staged into x_dev (rows * in bf16 of
 * device memory), the product writes y_dev (read first when accumulating)
 * and y_dev is staged into y_host, all on the gemm's stream by SM loads and
 * stores. Replaces the upload, Bf16Gemm::Linear and download a caller of the
 * reference's products makes (tests/products_test.cpp:100-110 around
 * gemm.hpp:51-58). */
VX_API vx_status vx_gemm_linear_host(vx_gemm* gemm, const uint16_t* x_host,
                                     uint16_t* x_dev, int format, const void* w,
                                     void* y_dev, void* y_host, int out_dtype,
                                     size_t rows, size_t in, size_t out,
                                     unsigned flags);

/* A column-major (BLAS) product C[m][n] (+)= op(A)[m][k] * op(B)[k][n],
 * optionally strided-batched (strides in elements, batch b at a + b *
 * stride_a, ...). Replaces MatmulShape (gemm.hpp:16-38). */
typedef struct vx_matmul_shape {
  int transpose_a;
  int transpose_b;
  size_t m, n, k;
  size_t lda, ldb, ldc;
  int64_t stride_a, stride_b, stride_c;
  size_t batch;
  int accumulate;
} vx_matmul_shape;
/* bf16 A and B, float32 C and sums. `representative` (the shape a tuned
 * algorithm is shared with) may be null: one kernel serves every shape.
 * VX_INVALID for leading dimensions below the stored column heights, sizes
 * above 2^30 or more than 65535 batches; nothing is launched for m, n or
 * batch 0. Replaces Bf16Gemm::Matmul (gemm.hpp:62-63, gemm.cpp:338-361). */
VX_API vx_status vx_matmul(const vx_matmul_shape* shape,
                           const vx_matmul_shape* representative,
                           const uint16_t* a, const uint16_t* b, float* c,
                           cudaStream_t stream);
/* vx_matmul on the gemm's stream. */
VX_API vx_status vx_gemm_matmul(vx_gemm* gemm, const vx_matmul_shape* shape,
                                const vx_matmul_shape* representative,
                                const uint16_t* a, const uint16_t* b, float* c);
/* Rounds up to a multiple of 128, the bucket size of shared shapes.
 * Replaces TuningBucket (gemm.hpp:74-77). */
static inline size_t vx_tuning_bucket(size_t size) {
  return (size + 127) / 128 * 128;
}

#ifdef __cplusplus
}
#endif

#endif /* VOXCPM_B200_H_ */
