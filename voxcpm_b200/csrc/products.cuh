// Skinny products y[rows][out] (+)= x[rows][in] * W[out][in]^T on sm_100a:
// bf16 activations, weights as Q8_0 tiles, bf16 tiles or bf16 rows, fp32
// accumulation, fp32 or bf16 output.
//
// Replaces the reference's product kernels: kernels/wmma_products.hip
// (WmmaQ8 / WmmaBf16, :139-296, :386-400), kernels/skinny_gemm.hip
// (SkinnyGemm, :42-253, :360-389) and their repack kernels
// (kernels/wmma_products.hip:62-126).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace vx {

/// Weight storage, matrix.hpp:9-13 (same order).
enum class WeightFormat : int {
  kBf16 = 0,       // bfloat16 [out][in], row-major
  kBf16Tiles = 1,  // bfloat16 tiles of 16 rows x 32 columns
  kQ8Tiles = 2,    // Q8_0 tiles of 16 rows x 32 columns plus 16 fp16 scales
};

constexpr int kTileRows = 16;
constexpr int kTileColumns = 32;
constexpr int kQ8TileBytes = 16 * 32 + 16 * 2;
constexpr int kBf16TileBytes = 16 * 32 * 2;
/// Most activation rows one launch takes (up to 16 MMA column tiles of 8;
/// 33..128 rows on the small CTA shapes only).
constexpr int kMaxProductRows = 128;
/// Most activation rows the tensor-core kernel takes.
constexpr int kTensorCoreMaxRows = 32;
/// Longest reduction slice one CTA holds in shared memory (explicit plans).
constexpr int kMaxSliceColumns = 2048;
/// Longest slice the planner's cost model gives one CTA.
constexpr int kPlannedSliceColumns = 1024;

inline std::size_t Q8TilesBytes(std::size_t rows, std::size_t in) {
  return (rows + kTileRows - 1) / kTileRows * (in / kTileColumns) *
         kQ8TileBytes;
}
inline std::size_t Bf16TilesBytes(std::size_t rows, std::size_t in) {
  return (rows + kTileRows - 1) / kTileRows * (in / kTileColumns) *
         kBf16TileBytes;
}

/// How one product launch is cut: `splits` CTAs (one thread-block
/// cluster) share each panel of weight rows, each taking
/// `blocks_per_split` 32-column blocks of the reduction; `variant` picks
/// the kernel shape (warps per CTA, row groups per warp, pipeline).
struct ProductPlan {
  int variant = -1;
  int splits = 1;
  int blocks_per_split = 0;
};

/// Plan variant of the tensor-core (tcgen05) kernel for Q8_0 tiles
/// (products_tc.cu): 128 weight rows per CTA, at most
/// kTensorCoreMaxBlocks 32-column blocks of the reduction per split.
constexpr int kTensorCoreVariant = 100;  // above every mma.sync variant
constexpr int kTensorCoreMaxBlocks = 24;
/// Fewest activation rows the planner gives to the tensor-core kernel.
constexpr int kTensorCoreMinRows = 9;

/// The tensor-core plan for Q8_0 tiles: about one CTA per SM (`sms`).
ProductPlan PlanTensorCoreProduct(std::size_t rows, std::size_t in,
                                  std::size_t out, int sms);
/// Launches the tensor-core kernel with `plan` (variant
/// kTensorCoreVariant). Returns kOk, kUnsupported or kCudaError.
int LaunchTensorCoreProduct(const std::uint16_t* x, const void* w, float* y,
                            std::uint16_t* y_bf16, std::size_t rows,
                            std::size_t in, std::size_t out, bool accumulate,
                            const ProductPlan& plan, cudaStream_t stream,
                            bool independent, bool programmatic);

/// The plan for a product (target_ctas 0: the planner's choice; otherwise
/// about that many CTAs).
ProductPlan PlanProduct(WeightFormat format, std::size_t rows, std::size_t in,
                        std::size_t out, std::size_t target_ctas = 0);

/// Caller-owned scratch of products whose panels are cut between CTAs (the
/// reference's SplitScratch, kernels/wmma_products.hpp:62-68): fp32 partial
/// sums, and one counter per 128-row panel that must be zero before the
/// first launch; every launch leaves the counters zero again. Launches that
/// share a scratch must be ordered (one stream), as in the reference.
struct SplitScratch {
  float* partials = nullptr;
  std::size_t partial_floats = 0;
  unsigned* counters = nullptr;
  std::size_t counter_count = 0;
};

/// Plan variant of the spread product (products_spread.cu): the product's
/// (128-row panel, 32-column block) units cut evenly over at most one CTA
/// per SM, panels cut between CTAs added in part order through a
/// SplitScratch. Plans carry the CTA count in `splits` and the longest run
/// of units in `blocks_per_split`.
constexpr int kSpreadVariant = 102;
constexpr int kSpreadMaxRows = 32;
constexpr int kSpreadMaxPanels = 1024;

struct SpreadNeeds {
  bool ok = false;
  int ctas = 0;
  int run = 0;
  std::size_t partial_floats = 0;
  std::size_t counters = 0;
};
/// Whether the spread kernel serves this shape, and the scratch it needs.
SpreadNeeds SpreadScratchNeeds(WeightFormat format, std::size_t rows,
                               std::size_t in, std::size_t out);
/// Scratch floats that serve every spread shape of at most `ctas` CTAs.
std::size_t SpreadScratchFloatsFor(int ctas);
/// CTAs of the widest spread launch on the current device (its SM count).
int MaxSpreadCtas();
/// Whether products launched without a plan may take the spread kernel
/// (default off: it measured slower than the whole-reduction plans).
void SetSpreadProducts(bool enabled);
bool SpreadProducts();
/// Whether a product launched without a plan takes the spread kernel when
/// the caller gave scratch (the shapes where it measured faster).
bool SpreadProductPays(WeightFormat format, std::size_t rows, std::size_t in,
                       std::size_t out);
/// Launches the spread kernel. Returns kOk, kUnsupported (shape not served),
/// kInvalid (scratch missing or too small) or kCudaError.
int LaunchSpreadProduct(WeightFormat format, const std::uint16_t* x,
                        const void* w, float* y, std::uint16_t* y_bf16,
                        std::size_t rows, std::size_t in, std::size_t out,
                        bool accumulate, const SplitScratch& scratch,
                        cudaStream_t stream, bool independent,
                        bool programmatic);

/// Launches one product of at most kMaxProductRows rows. Returns kOk,
/// kUnsupported (nothing launched) or kInvalid / kCudaError.
/// `independent`: the launch reads nothing that the kernels before it on
/// the stream write, so it skips the programmatic-launch wait and may overlap
/// them (streams of independent products); with no plan it takes the
/// measured stream plan for its shape where there is one.
/// `scratch` (may be null): split scratch the launch may use; with no plan,
/// shapes where SpreadProductPays take the spread kernel through it.
int LaunchProduct(WeightFormat format, const std::uint16_t* x, const void* w,
                  float* y, std::uint16_t* y_bf16, std::size_t rows,
                  std::size_t in, std::size_t out, bool accumulate,
                  const ProductPlan* plan, cudaStream_t stream,
                  bool independent = false,
                  const SplitScratch* scratch = nullptr);

/// Whether kernels are launched with programmatic dependent launch.
void SetProgrammaticLaunch(bool enabled);
/// Whether dependent product launches whose first CTAs start early have them
/// prefetch the later CTAs' weights into L2 (default on).
void SetProductL2Prefetch(bool enabled);
bool ProductL2Prefetch();
bool ProgrammaticLaunch();
/// Whether the planner gives Q8_0 products of 9..32 rows to the
/// tensor-core kernel or (default) to the mma.sync kernels.
void SetTensorCoreProducts(bool enabled);
bool TensorCoreProducts();

/// The tensor-core product for 33..128 rows of Q8_0 tiles
/// (products_tc_wide.cu): one 128 x N MMA per K step (N = rows rounded up to
/// 64, 96 or 128), weights streamed once through a two-stage ring, per-block
/// fp32 sums scaled in block order. Plans carry kTensorCoreWideVariant.
constexpr int kTensorCoreWideVariant = 101;
constexpr int kWideMinRows = 33;
constexpr int kWideMaxRows = 128;
ProductPlan PlanWideProduct(std::size_t rows, std::size_t in, std::size_t out,
                            int sms);
int LaunchWideProduct(const std::uint16_t* x, const void* w, float* y,
                      std::uint16_t* y_bf16, std::size_t rows, std::size_t in,
                      std::size_t out, bool accumulate, const ProductPlan& plan,
                      cudaStream_t stream, bool independent, bool programmatic);
/// Whether Q8_0 products launched without a plan take the wide tensor-core
/// kernel where WideProductPays (default on); else the mma.sync planner, or
/// launches of 32 rows.
void SetWideTensorCoreProducts(bool enabled);
bool WideTensorCoreProducts();
/// The shapes where the wide kernel measured faster than the mma.sync path.
bool WideProductPays(std::size_t rows, std::size_t in, std::size_t out);

int NumProductVariants();
/// Warps, row groups per warp, blocks per stage, stages of a variant.
void ProductVariantShape(int variant, int* warps, int* groups, int* stage,
                         int* depth);

// Repacks (load time).
int Q8_0ToTiles(const std::uint8_t* blocks, std::size_t rows, std::size_t in,
                std::uint8_t* tiles, cudaStream_t stream);
int Bf16ToTiles(const std::uint16_t* w, std::size_t rows, std::size_t in,
                std::uint16_t* tiles, cudaStream_t stream);
int Q8TilesToBf16(const std::uint8_t* tiles, std::size_t rows, std::size_t in,
                  std::uint16_t* out, cudaStream_t stream);
int Bf16TilesToRows(const std::uint16_t* tiles, std::size_t rows,
                    std::size_t in, std::uint16_t* out, cudaStream_t stream);
int ReadProbe(const void* data, std::size_t pieces, unsigned blocks,
              unsigned* sink, cudaStream_t stream);
// Copies `bytes` from `src` to `dst` with SM loads and stores (staging.cu):
// either side may be page-locked host memory. 16- or 4-byte pieces where
// both addresses and the size allow, else bytes.
int StageBytes(void* dst, const void* src, std::size_t bytes,
               cudaStream_t stream);

}  // namespace vx
