// Bf16Gemm::Matmul (gemm.hpp:16-38, 62-63; gemm.cpp:338-361): a column-major
// (BLAS) product C[m][n] (+)= op(A)[m][k] * op(B)[k][n] of bf16 operands with
// float32 accumulation and float32 C, optionally strided-batched.
//
// The reference sends this shape to hipBLASLt (hipBLAS as the fallback) and
// uses it for products of more than 128 activation rows. Linear here runs
// every row count on the exact products, so Matmul is the library's general
// GEMM for callers that use it directly. `representative` names the shape a
// tuned algorithm is shared with; one kernel serves every shape, so it is
// accepted and unused.
//
// The reduction-contiguous layout (below) has its own pipelined kernel. For
// the rest, one CTA computes a 64 x 64 tile of C with four warps (2 x 2, 32 x 32 each)
// on m16n8k16 bf16 MMAs. Each 32-column step of the reduction is gathered
// from global memory by element loads that follow the operand's contiguous
// dimension (any transpose, any leading dimension), held in registers while
// the previous step's tile is multiplied, then stored to shared memory with
// the reduction index contiguous. Sums are fp32; C = sums + beta * C.
#include "products.cuh"
#include "product_math.cuh"
#include "vx_common.cuh"
#include "vx_status.h"

#include "../../include/voxcpm_b200.h"

#include <cstdint>
#include <string>

namespace {

constexpr int kTileM = 64;
constexpr int kTileN = 64;
constexpr int kStepK = 32;
constexpr int kThreads = 128;
// Row pitch of the shared tiles in bf16: 40 (80 bytes) puts the eight
// fragment rows a warp reads at distinct banks.
constexpr int kPitch = kStepK + 8;
constexpr int kLoadsA = kTileM * kStepK / kThreads;  // 16
constexpr int kLoadsB = kTileN * kStepK / kThreads;  // 16

struct MatmulArgs {
  const std::uint16_t* a;
  const std::uint16_t* b;
  float* c;
  int m, n, k;
  long long lda, ldb, ldc;
  long long stride_a, stride_b, stride_c;
  int transpose_a, transpose_b;
  float beta;
};

/// Gathers op(A)[i0 .. i0+63][l0 .. l0+31] into `v` (zeros outside).
/// Without transpose A is column-major m x k (element (i, l) at
/// a[i + l * lda]), so lanes walk i; transposed, A is column-major k x m
/// (element (i, l) at a[l + i * lda]), so lanes walk l.
__device__ __forceinline__ void GatherA(const MatmulArgs& p,
                                        const std::uint16_t* a, int i0, int l0,
                                        std::uint16_t (&v)[kLoadsA]) {
#pragma unroll
  for (int t = 0; t < kLoadsA; ++t) {
    const int idx = static_cast<int>(threadIdx.x) + t * kThreads;
    int i, l;
    if (p.transpose_a) {
      l = idx % kStepK;
      i = idx / kStepK;
    } else {
      i = idx % kTileM;
      l = idx / kTileM;
    }
    const int gi = i0 + i, gl = l0 + l;
    std::uint16_t value = 0;
    if (gi < p.m && gl < p.k)
      value = p.transpose_a ? a[gl + static_cast<long long>(gi) * p.lda]
                            : a[gi + static_cast<long long>(gl) * p.lda];
    v[t] = value;
  }
}

/// Gathers op(B)[l0 .. l0+31][j0 .. j0+63]. Without transpose B is
/// column-major k x n (element (l, j) at b[l + j * ldb]); transposed, B is
/// column-major n x k (element (l, j) at b[j + l * ldb]).
__device__ __forceinline__ void GatherB(const MatmulArgs& p,
                                        const std::uint16_t* b, int j0, int l0,
                                        std::uint16_t (&v)[kLoadsB]) {
#pragma unroll
  for (int t = 0; t < kLoadsB; ++t) {
    const int idx = static_cast<int>(threadIdx.x) + t * kThreads;
    int j, l;
    if (p.transpose_b) {
      j = idx % kTileN;
      l = idx / kTileN;
    } else {
      l = idx % kStepK;
      j = idx / kStepK;
    }
    const int gj = j0 + j, gl = l0 + l;
    std::uint16_t value = 0;
    if (gj < p.n && gl < p.k)
      value = p.transpose_b ? b[gj + static_cast<long long>(gl) * p.ldb]
                            : b[gl + static_cast<long long>(gj) * p.ldb];
    v[t] = value;
  }
}

__global__ void __launch_bounds__(kThreads) MatmulKernel(const MatmulArgs p) {
  // Tiles with the reduction index contiguous: as[i][l], bs[j][l].
  __shared__ __align__(16) std::uint16_t as[kTileM * kPitch];
  __shared__ __align__(16) std::uint16_t bs[kTileN * kPitch];

  const int batch = static_cast<int>(blockIdx.z);
  const std::uint16_t* a = p.a + batch * p.stride_a;
  const std::uint16_t* b = p.b + batch * p.stride_b;
  float* c = p.c + batch * p.stride_c;
  const int i0 = static_cast<int>(blockIdx.x) * kTileM;
  const int j0 = static_cast<int>(blockIdx.y) * kTileN;

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int gid = lane >> 2;
  const int tig = lane & 3;
  const int wm = (warp & 1) * 32;   // warp's first row in the tile
  const int wn = (warp >> 1) * 32;  // warp's first column in the tile

  float acc[2][4][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        acc[mt][nt][e] = 0.0f;

  std::uint16_t va[kLoadsA], vb[kLoadsB];
  GatherA(p, a, i0, 0, va);
  GatherB(p, b, j0, 0, vb);

  for (int l0 = 0; l0 < p.k; l0 += kStepK) {
    __syncthreads();  // the previous step's fragments have been read
#pragma unroll
    for (int t = 0; t < kLoadsA; ++t) {
      const int idx = static_cast<int>(threadIdx.x) + t * kThreads;
      const int i = p.transpose_a ? idx / kStepK : idx % kTileM;
      const int l = p.transpose_a ? idx % kStepK : idx / kTileM;
      as[i * kPitch + l] = va[t];
    }
#pragma unroll
    for (int t = 0; t < kLoadsB; ++t) {
      const int idx = static_cast<int>(threadIdx.x) + t * kThreads;
      const int j = p.transpose_b ? idx % kTileN : idx / kStepK;
      const int l = p.transpose_b ? idx / kTileN : idx % kStepK;
      bs[j * kPitch + l] = vb[t];
    }
    __syncthreads();
    // The next step's elements load while this step's MMAs run.
    if (l0 + kStepK < p.k) {
      GatherA(p, a, i0, l0 + kStepK, va);
      GatherB(p, b, j0, l0 + kStepK, vb);
    }
#pragma unroll
    for (int kk = 0; kk < kStepK; kk += 16) {
      std::uint32_t fa[2][4], fb[4][2];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const std::uint16_t* r0 = as + (wm + mt * 16 + gid) * kPitch + kk + 2 * tig;
        const std::uint16_t* r8 = r0 + 8 * kPitch;
        fa[mt][0] = *reinterpret_cast<const std::uint32_t*>(r0);
        fa[mt][1] = *reinterpret_cast<const std::uint32_t*>(r8);
        fa[mt][2] = *reinterpret_cast<const std::uint32_t*>(r0 + 8);
        fa[mt][3] = *reinterpret_cast<const std::uint32_t*>(r8 + 8);
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const std::uint16_t* col = bs + (wn + nt * 8 + gid) * kPitch + kk + 2 * tig;
        fb[nt][0] = *reinterpret_cast<const std::uint32_t*>(col);
        fb[nt][1] = *reinterpret_cast<const std::uint32_t*>(col + 8);
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
          vx::Mma16816(acc[mt][nt], fa[mt][0], fa[mt][1], fa[mt][2], fa[mt][3],
                       fb[nt][0], fb[nt][1], acc[mt][nt]);
    }
  }

  // C is column-major: element (i, j) at c[i + j * ldc].
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = i0 + wm + mt * 16 + gid + (e >= 2 ? 8 : 0);
        const int j = j0 + wn + nt * 8 + 2 * tig + (e & 1);
        if (i < p.m && j < p.n) {
          float* out = c + i + static_cast<long long>(j) * p.ldc;
          *out = p.beta != 0.0f ? acc[mt][nt][e] + p.beta * *out
                                : acc[mt][nt][e];
        }
      }
}

// ------------------------------------------------- reduction-contiguous path
//
// Both operands contiguous along the reduction (transposed A, B as is: the
// layout of y = x W^T with row-major x and W, gemm.cpp:324-335), leading
// dimensions and batch strides multiples of 8 elements, 16-byte aligned
// bases. 128 x 128 tiles of C per CTA, eight warps of 64 x 32, a three-stage
// ring of 32-column steps filled by 16-byte cp.async copies (zero-filled past
// m, n and k), fragments read with ldmatrix.

constexpr int kFastTile = 128;
constexpr int kFastThreads = 256;
constexpr int kFastStages = 3;
// Row pitch 40 bf16 (80 bytes): 16-byte aligned rows, and the eight rows of
// one ldmatrix phase land on distinct bank quads.
constexpr int kFastStageElems = kFastTile * kPitch;  // per operand
constexpr std::size_t kFastSmem =
    sizeof(std::uint16_t) * 2 * kFastStages * kFastStageElems;

__device__ __forceinline__ void CpAsync16(void* dst, const void* src,
                                          int bytes) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d),
               "l"(src), "r"(bytes));
}

__device__ __forceinline__ void LdMatrixX4(std::uint32_t (&r)[4],
                                           const void* row) {
  const unsigned a = static_cast<unsigned>(__cvta_generic_to_shared(row));
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(a));
}

/// One 32-column step of a 128-row operand (row r at base + r * ld, the
/// step's columns from l0) into a shared stage [128][kPitch]. Rows at or
/// past `rows` and columns at or past `k` are zero-filled.
__device__ __forceinline__ void LoadFastStage(std::uint16_t* stage,
                                              const std::uint16_t* base,
                                              long long ld, int row0, int rows,
                                              int l0, int k) {
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int chunk = static_cast<int>(threadIdx.x) + t * kFastThreads;
    const int r = chunk >> 2;        // 4 chunks of 8 columns per row
    const int col = (chunk & 3) * 8;
    const int gr = row0 + r, gl = l0 + col;
    const bool inside = gr < rows && gl < k;
    const std::uint16_t* src =
        inside ? base + static_cast<long long>(gr) * ld + gl : base;
    CpAsync16(stage + r * kPitch + col, src, inside ? 16 : 0);
  }
}

__global__ void __launch_bounds__(kFastThreads)
    MatmulRowsKernel(const MatmulArgs p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  std::uint16_t* as = reinterpret_cast<std::uint16_t*>(smem_raw);
  std::uint16_t* bs = as + kFastStages * kFastStageElems;

  const int batch = static_cast<int>(blockIdx.z);
  const std::uint16_t* a = p.a + batch * p.stride_a;
  const std::uint16_t* b = p.b + batch * p.stride_b;
  float* c = p.c + batch * p.stride_c;
  const int i0 = static_cast<int>(blockIdx.x) * kFastTile;
  const int j0 = static_cast<int>(blockIdx.y) * kFastTile;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int gid = lane >> 2;
  const int tig = lane & 3;
  const int wm = (warp & 1) * 64;   // warp's rows in the tile
  const int wn = (warp >> 1) * 32;  // warp's columns in the tile

  float acc[4][4][4];
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        acc[mt][nt][e] = 0.0f;

  const int steps = (p.k + kStepK - 1) / kStepK;
#pragma unroll
  for (int s = 0; s < kFastStages - 1; ++s) {
    if (s < steps) {
      LoadFastStage(as + s * kFastStageElems, a, p.lda, i0, p.m, s * kStepK, p.k);
      LoadFastStage(bs + s * kFastStageElems, b, p.ldb, j0, p.n, s * kStepK, p.k);
    }
    asm volatile("cp.async.commit_group;\n" ::);
  }

  // ldmatrix row addresses: A tiles take rows lane % 16 at column
  // (lane / 16) * 8; B pairs of n8 tiles take row (lane % 8) + (lane / 16) * 8
  // at column ((lane / 8) % 2) * 8.
  const int a_row = lane & 15, a_col = (lane >> 4) * 8;
  const int b_row = (lane & 7) + (lane >> 4) * 8, b_col = ((lane >> 3) & 1) * 8;

  for (int step = 0; step < steps; ++step) {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(kFastStages - 2));
    __syncthreads();  // stage `step` landed; stage step - 1 is free
    const int next = step + kFastStages - 1;
    if (next < steps) {
      const int slot = next % kFastStages;
      LoadFastStage(as + slot * kFastStageElems, a, p.lda, i0, p.m, next * kStepK, p.k);
      LoadFastStage(bs + slot * kFastStageElems, b, p.ldb, j0, p.n, next * kStepK, p.k);
    }
    asm volatile("cp.async.commit_group;\n" ::);

    const std::uint16_t* sa = as + (step % kFastStages) * kFastStageElems;
    const std::uint16_t* sb = bs + (step % kFastStages) * kFastStageElems;
#pragma unroll
    for (int kk = 0; kk < kStepK; kk += 16) {
      std::uint32_t fa[4][4], fb[2][4];
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
        LdMatrixX4(fa[mt], sa + (wm + mt * 16 + a_row) * kPitch + kk + a_col);
#pragma unroll
      for (int np = 0; np < 2; ++np)
        LdMatrixX4(fb[np], sb + (wn + np * 16 + b_row) * kPitch + kk + b_col);
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
          vx::Mma16816(acc[mt][nt], fa[mt][0], fa[mt][1], fa[mt][2], fa[mt][3],
                       fb[nt >> 1][(nt & 1) * 2], fb[nt >> 1][(nt & 1) * 2 + 1],
                       acc[mt][nt]);
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::);

#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = i0 + wm + mt * 16 + gid + (e >= 2 ? 8 : 0);
        const int j = j0 + wn + nt * 8 + 2 * tig + (e & 1);
        if (i < p.m && j < p.n) {
          float* out = c + i + static_cast<long long>(j) * p.ldc;
          *out = p.beta != 0.0f ? acc[mt][nt][e] + p.beta * *out
                                : acc[mt][nt][e];
        }
      }
}

bool RowsLayout(const vx_matmul_shape& s, const std::uint16_t* a,
                const std::uint16_t* b) {
  const auto aligned = [](const void* ptr) {
    return reinterpret_cast<std::uintptr_t>(ptr) % 16 == 0;
  };
  return s.transpose_a && !s.transpose_b && s.k % 8 == 0 && s.lda % 8 == 0 &&
         s.ldb % 8 == 0 && (s.batch <= 1 || (s.stride_a % 8 == 0 &&
                                             s.stride_b % 8 == 0)) &&
         aligned(a) && aligned(b);
}

bool ValidShape(const vx_matmul_shape& s, const char** why) {
  constexpr std::size_t kMaxDim = 1u << 30;
  if (s.m > kMaxDim || s.n > kMaxDim || s.k > kMaxDim) {
    *why = "m, n and k must be at most 2^30";
    return false;
  }
  if (s.ldc < s.m || s.lda < (s.transpose_a ? s.k : s.m) ||
      s.ldb < (s.transpose_b ? s.n : s.k)) {
    *why = "a leading dimension is smaller than its operand's column";
    return false;
  }
  if (s.lda == 0 || s.ldb == 0 || s.ldc == 0) {
    *why = "leading dimensions must be positive";
    return false;
  }
  if (s.batch > 65535) {
    *why = "at most 65535 batches";
    return false;
  }
  if (s.batch > 1 && (s.stride_a < 0 || s.stride_b < 0 || s.stride_c < 0)) {
    *why = "negative batch stride";
    return false;
  }
  return true;
}

}  // namespace

extern "C" {

vx_status vx_matmul(const vx_matmul_shape* shape,
                    const vx_matmul_shape* representative, const uint16_t* a,
                    const uint16_t* b, float* c, cudaStream_t stream) {
  if (shape == nullptr)
    return vx::Fail(vx::kInvalid, "vx_matmul: null shape");
  const vx_matmul_shape& s = *shape;
  const char* why = nullptr;
  if (!ValidShape(s, &why))
    return vx::Fail(vx::kInvalid, std::string("vx_matmul: ") + why);
  (void)representative;  // one kernel for every shape: nothing to tune
  if (s.m == 0 || s.n == 0 || s.batch == 0)
    return vx::kOk;
  if (c == nullptr || (s.k > 0 && (a == nullptr || b == nullptr)))
    return vx::Fail(vx::kInvalid, "vx_matmul: null operand");
  MatmulArgs p;
  p.a = a;
  p.b = b;
  p.c = c;
  p.m = static_cast<int>(s.m);
  p.n = static_cast<int>(s.n);
  p.k = static_cast<int>(s.k);
  p.lda = static_cast<long long>(s.lda);
  p.ldb = static_cast<long long>(s.ldb);
  p.ldc = static_cast<long long>(s.ldc);
  p.stride_a = s.stride_a;
  p.stride_b = s.stride_b;
  p.stride_c = s.stride_c;
  p.transpose_a = s.transpose_a ? 1 : 0;
  p.transpose_b = s.transpose_b ? 1 : 0;
  p.beta = s.accumulate ? 1.0f : 0.0f;
  if (s.k > 0 && RowsLayout(s, a, b)) {
    const dim3 grid(static_cast<unsigned>((s.m + kFastTile - 1) / kFastTile),
                    static_cast<unsigned>((s.n + kFastTile - 1) / kFastTile),
                    static_cast<unsigned>(s.batch));
    if (grid.y > 65535)
      return vx::Fail(vx::kInvalid, "vx_matmul: n above 65535 * 128");
    const cudaError_t set = cudaFuncSetAttribute(
        MatmulRowsKernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
        static_cast<int>(kFastSmem));
    if (set != cudaSuccess)
      return vx::FromCuda(set, "vx_matmul");
    MatmulRowsKernel<<<grid, kFastThreads, kFastSmem, stream>>>(p);
    return vx::FromCuda(cudaGetLastError(), "vx_matmul");
  }
  const dim3 grid(static_cast<unsigned>((s.m + kTileM - 1) / kTileM),
                  static_cast<unsigned>((s.n + kTileN - 1) / kTileN),
                  static_cast<unsigned>(s.batch));
  if (grid.y > 65535)
    return vx::Fail(vx::kInvalid, "vx_matmul: n above 65535 * 64");
  MatmulKernel<<<grid, kThreads, 0, stream>>>(p);
  return vx::FromCuda(cudaGetLastError(), "vx_matmul");
}

}  // extern "C"
