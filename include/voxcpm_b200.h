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
 * 74-81). `splits` CTAs of one thread-block cluster share each panel of
 * weight rows and reduce on chip, so partial_floats and counters are always
 * 0 (no scratch). `variant` selects the kernel shape. */
typedef struct vx_wmma_plan {
  size_t splits;
  size_t blocks_per_split;
  size_t partial_floats;
  size_t counters;
  int variant;
} vx_wmma_plan;

/* Replaces SplitScratch (kernels/wmma_products.hpp:62-68); accepted for
 * interface parity and not used (may be all zero). */
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

/* y[rows][out] (+)= x[rows][in] * W^T for bf16 x and Q8 tiles W, at most 32
 * rows, `in` a multiple of 32 (at most 8192). `plan` may be null (planner's
 * choice), `scratch` may be null. Replaces WmmaQ8
 * (kernels/wmma_products.hpp:87-93). */
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
 * multiple of 8 (the kernels need a multiple of 32; other sizes return
 * VX_UNSUPPORTED). Replaces SkinnyGemm (kernels/skinny_gemm.hpp:18-24). */
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
 * (`out_dtype`), at most 32 rows per launch. Extends WmmaQ8/WmmaBf16/
 * SkinnyGemm (kernels/wmma_products.hpp:87-99, kernels/skinny_gemm.hpp:
 * 18-24) with the bf16-output epilogue. */
VX_API vx_status vx_product(int format, const uint16_t* x, const void* w, void* y,
                     int out_dtype, size_t rows, size_t in, size_t out,
                     int accumulate, const vx_wmma_plan* plan,
                     cudaStream_t stream);

/* Programmatic dependent launch for every kernel of the library (default on).
 * No reference counterpart (HIP has none). */
VX_API void vx_set_programmatic_launch(int enabled);
/* Number of product kernel shapes and the shape of one (benchmarks). */
VX_API int vx_product_variants(void);
VX_API void vx_product_variant_shape(int variant, int* warps, int* groups,
                              int* stage, int* depth);

/* ------------------------------------------------------------ synthetic weights */

/* Host: GGML Q8_0 blocks [rows][in/32] of seeded random weights, a pure
 * function of (seed, tensor, index): q uniform in [-127, 127], one fp16
 * scale |N(0, scale_std)| per 32 values. Stands in for the checkpoint reader
 * (weights.cpp:26-327, out of scope: no checkpoint is available). */
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
VX_API void vx_gemm_destroy(vx_gemm* gemm);
/* y[rows][out] (+)= x[rows][in] * w[out][in]^T, float32 y. Rows beyond 32
 * run in chunks of 32 (every chunk re-reads W). Replaces Bf16Gemm::Linear
 * (gemm.hpp:51-58, gemm.cpp:259-313). */
VX_API vx_status vx_gemm_linear(vx_gemm* gemm, const uint16_t* x, int format,
                         const void* w, float* y, size_t rows, size_t in,
                         size_t out, int accumulate);

#ifdef __cplusplus
}
#endif

#endif /* VOXCPM_B200_H_ */
