// C ABI of the product layer (include/voxcpm_b200.h): status codes, the
// thread-local error message and the Bf16Gemm dispatch (gemm.cpp:259-313).
#include "products.cuh"
#include "vx_common.cuh"
#include "vx_status.h"

#include "../../include/voxcpm_b200.h"

#include <string>

namespace vx {

namespace {
thread_local std::string g_last_error;
}

int Fail(int status, const std::string& message) {
  g_last_error = message;
  return status;
}

int FromCuda(cudaError_t error, const char* what) {
  if (error == cudaSuccess)
    return kOk;
  return Fail(kCudaError, std::string(what) + ": " + cudaGetErrorString(error));
}

int Checked(int status, const char* what) {
  switch (status) {
    case kOk:
      return kOk;
    case kUnsupported:
      return Fail(status, std::string(what) + ": shape not served by the kernels");
    case kInvalid:
      return Fail(status, std::string(what) + ": invalid argument");
    case kCudaError: {
      const cudaError_t error = cudaGetLastError();
      return Fail(status, std::string(what) + ": " + cudaGetErrorString(error));
    }
    default:
      return Fail(status, std::string(what) + ": failed");
  }
}

const char* LastError() { return g_last_error.c_str(); }

}  // namespace vx

namespace {

vx::ProductPlan ToPlan(const vx_wmma_plan* plan) {
  vx::ProductPlan p;
  if (plan != nullptr && plan->splits > 0) {
    p.variant = plan->variant;
    p.splits = static_cast<int>(plan->splits);
    p.blocks_per_split = static_cast<int>(plan->blocks_per_split);
  }
  return p;
}

vx::SplitScratch ToScratch(const vx_split_scratch& s) {
  vx::SplitScratch out;
  out.partials = s.partials;
  out.partial_floats = s.partial_floats;
  out.counters = s.counters;
  out.counter_count = s.counter_count;
  return out;
}

vx_status Product(int format, const uint16_t* x, const void* w, void* y,
                  int out_dtype, size_t rows, size_t in, size_t out,
                  int accumulate, const vx_wmma_plan* plan,
                  cudaStream_t stream, const char* what,
                  bool independent = false,
                  const vx::SplitScratch* scratch = nullptr) {
  if (out_dtype != VX_OUT_F32 && out_dtype != VX_OUT_BF16)
    return vx::Fail(vx::kInvalid, std::string(what) + ": unknown out_dtype");
  const vx::ProductPlan p = ToPlan(plan);
  if (p.variant == vx::kSpreadVariant && scratch == nullptr)
    return vx::Fail(vx::kInvalid,
                    std::string(what) +
                        ": a spread plan needs split scratch (partials and "
                        "counters, sized by vx_plan_spread)");
  const int status = vx::LaunchProduct(
      static_cast<vx::WeightFormat>(format), x, w,
      out_dtype == VX_OUT_F32 ? static_cast<float*>(y) : nullptr,
      out_dtype == VX_OUT_BF16 ? static_cast<uint16_t*>(y) : nullptr, rows,
      in, out, accumulate != 0, plan != nullptr && plan->splits > 0 ? &p : nullptr,
      stream, independent, scratch);
  if (status == vx::kInvalid && p.variant == vx::kSpreadVariant)
    return vx::Fail(status, std::string(what) +
                                ": split scratch smaller than the spread plan "
                                "needs (vx_plan_spread)");
  return vx::Checked(status, what);
}

/// y (+)= x * w^T for bf16 rows through the general column-major product
/// (the reference's LinearRows fallback, gemm.cpp:315-336): C = W^T-major
/// [out][rows] with A = w ([out][in] row-major, transposed) and B = x.
vx_status RowsByMatmul(const uint16_t* x, const uint16_t* w, float* y,
                       size_t rows, size_t in, size_t out, int accumulate,
                       cudaStream_t stream) {
  vx_matmul_shape shape = {};
  shape.transpose_a = 1;
  shape.transpose_b = 0;
  shape.m = out;
  shape.n = rows;
  shape.k = in;
  shape.lda = in;
  shape.ldb = in;
  shape.ldc = out;
  shape.batch = 1;
  shape.accumulate = accumulate;
  return vx_matmul(&shape, nullptr, w, x, y, stream);
}

}  // namespace

extern "C" {

const char* vx_last_error(void) { return vx::LastError(); }

const char* vx_version(void) { return "voxcpm_b200 0.1.0 (sm_100a)"; }

vx_status vx_device_error(unsigned* bits) {
  if (bits == nullptr)
    return vx::Fail(vx::kInvalid, "vx_device_error: null output");
  if (vx::ReadDeviceError(bits) != vx::kOk)
    return vx::FromCuda(cudaGetLastError(), "vx_device_error");
  return VX_OK;
}

size_t vx_q8_tiles_bytes(size_t rows, size_t in) {
  return vx::Q8TilesBytes(rows, in);
}
size_t vx_bf16_tiles_bytes(size_t rows, size_t in) {
  return vx::Bf16TilesBytes(rows, in);
}

vx_status vx_q8_0_to_tiles(const uint8_t* blocks, size_t rows, size_t in,
                           uint8_t* tiles, cudaStream_t stream) {
  return vx::Checked(vx::Q8_0ToTiles(blocks, rows, in, tiles, stream),
                     "vx_q8_0_to_tiles");
}
vx_status vx_bf16_to_tiles(const uint16_t* weights, size_t rows, size_t in,
                           uint16_t* tiles, cudaStream_t stream) {
  return vx::Checked(vx::Bf16ToTiles(weights, rows, in, tiles, stream),
                     "vx_bf16_to_tiles");
}
vx_status vx_q8_tiles_to_bf16(const uint8_t* tiles, size_t rows, size_t in,
                              uint16_t* out, cudaStream_t stream) {
  return vx::Checked(vx::Q8TilesToBf16(tiles, rows, in, out, stream),
                     "vx_q8_tiles_to_bf16");
}
vx_status vx_bf16_tiles_to_rows(const uint16_t* tiles, size_t rows, size_t in,
                                uint16_t* out, cudaStream_t stream) {
  return vx::Checked(vx::Bf16TilesToRows(tiles, rows, in, out, stream),
                     "vx_bf16_tiles_to_rows");
}

vx_wmma_plan vx_plan_wmma(size_t rows, size_t in, size_t out,
                          size_t target_waves) {
  vx_wmma_plan plan = {0, 0, 0, 0, -1};
  const vx::ProductPlan p = vx::PlanProduct(
      vx::WeightFormat::kQ8Tiles, rows, in, out, target_waves);
  if (p.variant < 0)
    return plan;
  plan.splits = static_cast<size_t>(p.splits);
  plan.blocks_per_split = static_cast<size_t>(p.blocks_per_split);
  plan.variant = p.variant;
  return plan;
}

vx_wmma_plan vx_plan_spread(int format, size_t rows, size_t in, size_t out) {
  vx_wmma_plan plan = {0, 0, 0, 0, -1};
  if (format < VX_WEIGHTS_BF16 || format > VX_WEIGHTS_Q8_TILES)
    return plan;
  const vx::SpreadNeeds needs = vx::SpreadScratchNeeds(
      static_cast<vx::WeightFormat>(format), rows, in, out);
  if (!needs.ok)
    return plan;
  plan.splits = static_cast<size_t>(needs.ctas);
  plan.blocks_per_split = static_cast<size_t>(needs.run);
  plan.partial_floats = needs.partial_floats;
  plan.counters = needs.counters;
  plan.variant = vx::kSpreadVariant;
  return plan;
}

void vx_set_spread_products(int enabled) {
  vx::SetSpreadProducts(enabled != 0);
}

int vx_spread_products(void) { return vx::SpreadProducts() ? 1 : 0; }

vx_status vx_wmma_q8(const uint16_t* x, const uint8_t* w, float* y,
                     size_t rows, size_t in, size_t out, int accumulate,
                     const vx_wmma_plan* plan, const vx_split_scratch* scratch,
                     cudaStream_t stream) {
  const vx::SplitScratch s =
      scratch != nullptr ? ToScratch(*scratch) : vx::SplitScratch();
  return Product(VX_WEIGHTS_Q8_TILES, x, w, y, VX_OUT_F32, rows, in, out,
                 accumulate, plan, stream, "vx_wmma_q8", false,
                 scratch != nullptr ? &s : nullptr);
}

vx_status vx_wmma_bf16(const uint16_t* x, const uint16_t* w, float* y,
                       size_t rows, size_t in, size_t out, int accumulate,
                       const vx_wmma_plan* plan,
                       const vx_split_scratch* scratch, cudaStream_t stream) {
  const vx::SplitScratch s =
      scratch != nullptr ? ToScratch(*scratch) : vx::SplitScratch();
  return Product(VX_WEIGHTS_BF16_TILES, x, w, y, VX_OUT_F32, rows, in, out,
                 accumulate, plan, stream, "vx_wmma_bf16", false,
                 scratch != nullptr ? &s : nullptr);
}

vx_status vx_skinny_gemm(const uint16_t* x, const uint16_t* w, float* y,
                         size_t rows, size_t in, size_t out, int accumulate,
                         cudaStream_t stream) {
  // The reference's contract (kernels/skinny_gemm.hip:360-389): at most 32
  // rows, `in` a multiple of 8 and at most 8192.
  if (in > 8192)
    return vx::Fail(vx::kUnsupported, "vx_skinny_gemm: in > 8192");
  if (rows > 32)
    return vx::Fail(vx::kUnsupported, "vx_skinny_gemm: more than 32 rows");
  if (in % 8 != 0)
    return vx::Fail(vx::kUnsupported, "vx_skinny_gemm: in is not a multiple of 8");
  if (rows == 0 || out == 0)
    return VX_OK;
  if (in % vx::kTileColumns != 0) {
    // The skinny kernels stream 32-column blocks; other multiples of 8 run
    // on the library's general product, which reads every weight once too.
    if (x == nullptr || w == nullptr || y == nullptr)
      return vx::Fail(vx::kInvalid, "vx_skinny_gemm: null operand");
    return RowsByMatmul(x, w, y, rows, in, out, accumulate, stream);
  }
  return Product(VX_WEIGHTS_BF16, x, w, y, VX_OUT_F32, rows, in, out,
                 accumulate, nullptr, stream, "vx_skinny_gemm");
}

vx_status vx_skinny_gemm_with(int vec, const uint16_t* x, const uint16_t* w,
                              float* y, size_t rows, size_t in, size_t out,
                              int accumulate, cudaStream_t stream) {
  if (vec < 0)
    return vx_skinny_gemm(x, w, y, rows, in, out, accumulate, stream);
  if (vec >= vx::NumProductVariants())
    return vx::Fail(vx::kInvalid, "vx_skinny_gemm_with: unknown variant");
  // The planner's split for the requested variant.
  vx::ProductPlan best = vx::PlanProduct(vx::WeightFormat::kBf16, rows, in,
                                         out, 0);
  if (best.variant < 0)
    return vx::Fail(vx::kUnsupported, "vx_skinny_gemm_with: shape");
  vx_wmma_plan plan = {static_cast<size_t>(best.splits),
                       static_cast<size_t>(best.blocks_per_split), 0, 0, vec};
  return Product(VX_WEIGHTS_BF16, x, w, y, VX_OUT_F32, rows, in, out,
                 accumulate, &plan, stream, "vx_skinny_gemm_with");
}

vx_status vx_read_probe(const void* data, size_t pieces, unsigned blocks,
                        unsigned* sink, cudaStream_t stream) {
  return vx::Checked(vx::ReadProbe(data, pieces, blocks, sink, stream),
                     "vx_read_probe");
}

vx_status vx_product(int format, const uint16_t* x, const void* w, void* y,
                     int out_dtype, size_t rows, size_t in, size_t out,
                     int accumulate, const vx_wmma_plan* plan,
                     cudaStream_t stream) {
  return Product(format, x, w, y, out_dtype, rows, in, out, accumulate, plan,
                 stream, "vx_product");
}

vx_status vx_product_ex(int format, const uint16_t* x, const void* w, void* y,
                        int out_dtype, size_t rows, size_t in, size_t out,
                        unsigned flags, const vx_wmma_plan* plan,
                        cudaStream_t stream) {
  if ((flags & ~(VX_PRODUCT_ACCUMULATE | VX_PRODUCT_INDEPENDENT)) != 0)
    return vx::Fail(vx::kInvalid, "vx_product_ex: unknown flags");
  return Product(format, x, w, y, out_dtype, rows, in, out,
                 (flags & VX_PRODUCT_ACCUMULATE) != 0 ? 1 : 0, plan, stream,
                 "vx_product_ex", (flags & VX_PRODUCT_INDEPENDENT) != 0);
}

vx_status vx_product_host(int format, const uint16_t* x_host, uint16_t* x_dev,
                          const void* w, void* y_dev, void* y_host,
                          int out_dtype, size_t rows, size_t in, size_t out,
                          unsigned flags, const vx_wmma_plan* plan,
                          cudaStream_t stream) {
  if ((flags & ~VX_PRODUCT_ACCUMULATE) != 0)
    return vx::Fail(vx::kInvalid,
                    "vx_product_host: only VX_PRODUCT_ACCUMULATE applies");
  if (x_host == nullptr || x_dev == nullptr || y_dev == nullptr ||
      y_host == nullptr)
    return vx::Fail(vx::kInvalid, "vx_product_host: null buffer");
  if (out_dtype != VX_OUT_F32 && out_dtype != VX_OUT_BF16)
    return vx::Fail(vx::kInvalid, "vx_product_host: unknown out_dtype");
  if (rows == 0)
    return VX_OK;
  const size_t y_bytes = rows * out * (out_dtype == VX_OUT_F32 ? 4 : 2);
  vx_status status = vx::Checked(
      vx::StageBytes(x_dev, x_host, rows * in * sizeof(uint16_t), stream),
      "vx_product_host");
  if (status != VX_OK)
    return status;
  status = Product(format, x_dev, w, y_dev, out_dtype, rows, in, out,
                   (flags & VX_PRODUCT_ACCUMULATE) != 0 ? 1 : 0, plan, stream,
                   "vx_product_host");
  if (status != VX_OK)
    return status;
  return vx::Checked(vx::StageBytes(y_host, y_dev, y_bytes, stream),
                     "vx_product_host");
}

vx_status vx_stage(void* dst, const void* src, size_t bytes,
                   cudaStream_t stream) {
  return vx::Checked(vx::StageBytes(dst, src, bytes, stream), "vx_stage");
}

void vx_set_programmatic_launch(int enabled) {
  vx::SetProgrammaticLaunch(enabled != 0);
}

void vx_set_product_l2_prefetch(int enabled) {
  vx::SetProductL2Prefetch(enabled != 0);
}

void vx_set_tensor_core_products(int enabled) {
  vx::SetTensorCoreProducts(enabled != 0);
}

int vx_tensor_core_products(void) { return vx::TensorCoreProducts() ? 1 : 0; }

void vx_set_wide_tensor_core_products(int enabled) {
  vx::SetWideTensorCoreProducts(enabled != 0);
}

int vx_wide_tensor_core_products(void) {
  return vx::WideTensorCoreProducts() ? 1 : 0;
}

int vx_product_variants(void) { return vx::NumProductVariants(); }

void vx_product_variant_shape(int variant, int* warps, int* groups,
                              int* stage, int* depth) {
  if (variant < 0 || variant >= vx::NumProductVariants())
    return;
  vx::ProductVariantShape(variant, warps, groups, stage, depth);
}

// ------------------------------------------------------------ Bf16Gemm

struct vx_gemm {
  cudaStream_t stream;
  // Split scratch of the spread products, sized for every shape at one CTA
  // per SM (the reference's Bf16Gemm keeps its partials and counters the
  // same way, gemm.cpp:270-290); the counters start at zero and every launch
  // leaves them zero. One gemm per stream, so its launches are ordered.
  vx::SplitScratch scratch;
};

vx_gemm* vx_gemm_create(cudaStream_t stream) {
  vx_gemm* gemm = new vx_gemm{stream, {}};
  const std::size_t floats = vx::SpreadScratchFloatsFor(vx::MaxSpreadCtas());
  const std::size_t counters = vx::kSpreadMaxPanels;
  void* partials = nullptr;
  void* count_words = nullptr;
  if (cudaMalloc(&partials, floats * sizeof(float)) != cudaSuccess ||
      cudaMalloc(&count_words, counters * sizeof(unsigned)) != cudaSuccess ||
      cudaMemsetAsync(count_words, 0, counters * sizeof(unsigned), stream) !=
          cudaSuccess) {
    // No scratch (no device, or no memory): the gemm still serves every
    // shape on the cluster plans, which need none.
    (void)cudaGetLastError();
    cudaFree(partials);
    cudaFree(count_words);
    (void)cudaGetLastError();
    return gemm;
  }
  gemm->scratch.partials = static_cast<float*>(partials);
  gemm->scratch.partial_floats = floats;
  gemm->scratch.counters = static_cast<unsigned*>(count_words);
  gemm->scratch.counter_count = counters;
  return gemm;
}

void vx_gemm_destroy(vx_gemm* gemm) {
  if (gemm == nullptr)
    return;
  if (gemm->scratch.partials != nullptr) {
    // Launches on the gemm's stream may still use the scratch.
    cudaStreamSynchronize(gemm->stream);
    cudaFree(gemm->scratch.partials);
    cudaFree(gemm->scratch.counters);
  }
  delete gemm;
}

vx_status vx_gemm_linear(vx_gemm* gemm, const uint16_t* x, int format,
                         const void* w, float* y, size_t rows, size_t in,
                         size_t out, int accumulate) {
  if (gemm == nullptr)
    return vx::Fail(vx::kInvalid, "vx_gemm_linear: null gemm");
  if (rows == 0 || out == 0)
    return vx::kOk;
  if (format == VX_WEIGHTS_BF16 && in % vx::kTileColumns != 0) {
    // bf16 rows the skinny kernels refuse: the general product, as
    // Bf16Gemm::LinearRows falls back to Matmul (gemm.cpp:315-336).
    if (x == nullptr || w == nullptr || y == nullptr)
      return vx::Fail(vx::kInvalid, "vx_gemm_linear: null operand");
    return RowsByMatmul(x, static_cast<const uint16_t*>(w), y, rows, in, out,
                        accumulate, gemm->stream);
  }
  // Chunks of up to 128 rows, one launch each (gemm.cpp:270-303 chunks the
  // reference's matrix-core products by 32 rows).
  for (size_t first = 0; first < rows; first += vx::kMaxProductRows) {
    const size_t count =
        rows - first < static_cast<size_t>(vx::kMaxProductRows)
            ? rows - first
            : static_cast<size_t>(vx::kMaxProductRows);
    const vx_status status = Product(format, x + first * in, w, y + first * out,
                                     VX_OUT_F32, count, in, out, accumulate,
                                     nullptr, gemm->stream, "vx_gemm_linear",
                                     false, &gemm->scratch);
    if (status != VX_OK)
      return status;
  }
  return VX_OK;
}

vx_status vx_gemm_linear_ex(vx_gemm* gemm, const uint16_t* x, int format,
                            const void* w, void* y, int out_dtype, size_t rows,
                            size_t in, size_t out, unsigned flags) {
  if (gemm == nullptr)
    return vx::Fail(vx::kInvalid, "vx_gemm_linear_ex: null gemm");
  if ((flags & ~VX_PRODUCT_ACCUMULATE) != 0)
    return vx::Fail(vx::kInvalid,
                    "vx_gemm_linear_ex: only VX_PRODUCT_ACCUMULATE applies");
  const int accumulate = (flags & VX_PRODUCT_ACCUMULATE) != 0 ? 1 : 0;
  if (out_dtype == VX_OUT_F32)
    return vx_gemm_linear(gemm, x, format, w, static_cast<float*>(y), rows,
                          in, out, accumulate);
  if (out_dtype != VX_OUT_BF16)
    return vx::Fail(vx::kInvalid, "vx_gemm_linear_ex: unknown out_dtype");
  if (rows == 0 || out == 0)
    return vx::kOk;
  const size_t element = 2;
  for (size_t first = 0; first < rows; first += vx::kMaxProductRows) {
    const size_t count =
        rows - first < static_cast<size_t>(vx::kMaxProductRows)
            ? rows - first
            : static_cast<size_t>(vx::kMaxProductRows);
    const vx_status status = Product(
        format, x + first * in, w,
        static_cast<unsigned char*>(y) + first * out * element, VX_OUT_BF16,
        count, in, out, accumulate, nullptr, gemm->stream,
        "vx_gemm_linear_ex", false, &gemm->scratch);
    if (status != VX_OK)
      return status;
  }
  return VX_OK;
}

vx_status vx_gemm_linear_host(vx_gemm* gemm, const uint16_t* x_host,
                              uint16_t* x_dev, int format, const void* w,
                              void* y_dev, void* y_host, int out_dtype,
                              size_t rows, size_t in, size_t out,
                              unsigned flags) {
  if (gemm == nullptr)
    return vx::Fail(vx::kInvalid, "vx_gemm_linear_host: null gemm");
  if (x_host == nullptr || x_dev == nullptr || y_dev == nullptr ||
      y_host == nullptr)
    return vx::Fail(vx::kInvalid, "vx_gemm_linear_host: null buffer");
  if (out_dtype != VX_OUT_F32 && out_dtype != VX_OUT_BF16)
    return vx::Fail(vx::kInvalid, "vx_gemm_linear_host: unknown out_dtype");
  if (rows == 0 || out == 0)
    return VX_OK;
  vx_status status = vx::Checked(
      vx::StageBytes(x_dev, x_host, rows * in * sizeof(uint16_t), gemm->stream),
      "vx_gemm_linear_host");
  if (status != VX_OK)
    return status;
  status = vx_gemm_linear_ex(gemm, x_dev, format, w, y_dev, out_dtype, rows,
                             in, out, flags);
  if (status != VX_OK)
    return status;
  const size_t y_bytes = rows * out * (out_dtype == VX_OUT_F32 ? 4 : 2);
  return vx::Checked(vx::StageBytes(y_host, y_dev, y_bytes, gemm->stream),
                     "vx_gemm_linear_host");
}

vx_status vx_gemm_matmul(vx_gemm* gemm, const vx_matmul_shape* shape,
                         const vx_matmul_shape* representative,
                         const uint16_t* a, const uint16_t* b, float* c) {
  if (gemm == nullptr)
    return vx::Fail(vx::kInvalid, "vx_gemm_matmul: null gemm");
  return vx_matmul(shape, representative, a, b, c, gemm->stream);
}

}  // extern "C"
