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
// One CTA computes a 64 x 64 tile of C with four warps (2 x 2, 32 x 32 each)
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
  const dim3 grid(static_cast<unsigned>((s.m + kTileM - 1) / kTileM),
                  static_cast<unsigned>((s.n + kTileN - 1) / kTileN),
                  static_cast<unsigned>(s.batch));
  if (grid.y > 65535)
    return vx::Fail(vx::kInvalid, "vx_matmul: n above 65535 * 64");
  MatmulKernel<<<grid, kThreads, 0, stream>>>(p);
  return vx::FromCuda(cudaGetLastError(), "vx_matmul");
}

}  // extern "C"
