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

vx_status Product(int format, const uint16_t* x, const void* w, void* y,
                  int out_dtype, size_t rows, size_t in, size_t out,
                  int accumulate, const vx_wmma_plan* plan,
                  cudaStream_t stream, const char* what,
                  bool independent = false) {
  if (out_dtype != VX_OUT_F32 && out_dtype != VX_OUT_BF16)
    return vx::Fail(vx::kInvalid, std::string(what) + ": unknown out_dtype");
  const vx::ProductPlan p = ToPlan(plan);
  const int status = vx::LaunchProduct(
      static_cast<vx::WeightFormat>(format), x, w,
      out_dtype == VX_OUT_F32 ? static_cast<float*>(y) : nullptr,
      out_dtype == VX_OUT_BF16 ? static_cast<uint16_t*>(y) : nullptr, rows,
      in, out, accumulate != 0, plan != nullptr && plan->splits > 0 ? &p : nullptr,
      stream, independent);
  return vx::Checked(status, what);
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

vx_status vx_wmma_q8(const uint16_t* x, const uint8_t* w, float* y,
                     size_t rows, size_t in, size_t out, int accumulate,
                     const vx_wmma_plan* plan, const vx_split_scratch* scratch,
                     cudaStream_t stream) {
  (void)scratch;
  return Product(VX_WEIGHTS_Q8_TILES, x, w, y, VX_OUT_F32, rows, in, out,
                 accumulate, plan, stream, "vx_wmma_q8");
}

vx_status vx_wmma_bf16(const uint16_t* x, const uint16_t* w, float* y,
                       size_t rows, size_t in, size_t out, int accumulate,
                       const vx_wmma_plan* plan,
                       const vx_split_scratch* scratch, cudaStream_t stream) {
  (void)scratch;
  return Product(VX_WEIGHTS_BF16_TILES, x, w, y, VX_OUT_F32, rows, in, out,
                 accumulate, plan, stream, "vx_wmma_bf16");
}

vx_status vx_skinny_gemm(const uint16_t* x, const uint16_t* w, float* y,
                         size_t rows, size_t in, size_t out, int accumulate,
                         cudaStream_t stream) {
  if (in > 8192)
    return vx::Fail(vx::kUnsupported, "vx_skinny_gemm: in > 8192");
  if (rows > 32)
    return vx::Fail(vx::kUnsupported, "vx_skinny_gemm: more than 32 rows");
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
};

vx_gemm* vx_gemm_create(cudaStream_t stream) {
  return new vx_gemm{stream};
}

void vx_gemm_destroy(vx_gemm* gemm) { delete gemm; }

vx_status vx_gemm_linear(vx_gemm* gemm, const uint16_t* x, int format,
                         const void* w, float* y, size_t rows, size_t in,
                         size_t out, int accumulate) {
  if (gemm == nullptr)
    return vx::Fail(vx::kInvalid, "vx_gemm_linear: null gemm");
  if (rows == 0)
    return vx::kOk;
  // Chunks of up to 128 rows, one launch each (gemm.cpp:270-303 chunks the
  // reference's matrix-core products by 32 rows).
  for (size_t first = 0; first < rows; first += vx::kMaxProductRows) {
    const size_t count =
        rows - first < static_cast<size_t>(vx::kMaxProductRows)
            ? rows - first
            : static_cast<size_t>(vx::kMaxProductRows);
    const vx_status status = Product(format, x + first * in, w, y + first * out,
                                     VX_OUT_F32, count, in, out, accumulate,
                                     nullptr, gemm->stream, "vx_gemm_linear");
    if (status != VX_OK)
      return status;
  }
  return VX_OK;
}

vx_status vx_gemm_matmul(vx_gemm* gemm, const vx_matmul_shape* shape,
                         const vx_matmul_shape* representative,
                         const uint16_t* a, const uint16_t* b, float* c) {
  if (gemm == nullptr)
    return vx::Fail(vx::kInvalid, "vx_gemm_matmul: null gemm");
  return vx_matmul(shape, representative, a, b, c, gemm->stream);
}

}  // extern "C"
