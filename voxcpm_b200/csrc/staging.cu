// Host <-> device staging by SM loads and stores: moves a buffer between
// two device-accessible addresses, one of them typically page-locked host
// memory (cudaHostAlloc / cudaHostRegister, reachable at the same address
// under unified addressing) read or written over PCIe.
//
// Why not cudaMemcpyAsync: for the product's per-call transfers (90 KB of
// activations in, 270 KB of bf16 output back at M = 22, K = 2048,
// N = 6144) the copy engines moved one call's pair in 11.1 us on B200,
// where a grid of SM threads issuing 16-byte PCIe reads and writes took
// 6.5 us (two launches) over 16 streams. Mixing the two (one direction on a
// copy engine, the other on SMs) was slower than either.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "products.cuh"
#include "vx_common.cuh"
#include "vx_launch.cuh"

namespace vx {
namespace {

constexpr int kStageThreads = 256;
// Enough CTAs for the PCIe round trips of a few hundred KB to overlap; more
// measured no faster (16 to 148 CTAs within 1 % for 270 KB).
constexpr int kMaxStageCtas = 296;

template <typename Piece>
__global__ void StageKernel(const Piece* __restrict__ src,
                            Piece* __restrict__ dst, std::size_t pieces) {
  // The destination may be read by the next kernel, and the source written
  // by the previous one: wait for the predecessor, let the successor start
  // its prologue (it waits for this grid before reading).
  GridLaunchDependents();
  GridDependencyWait();
  const std::size_t stride =
      static_cast<std::size_t>(gridDim.x) * blockDim.x;
  for (std::size_t i =
           static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < pieces; i += stride)
    dst[i] = src[i];
}

template <typename Piece>
int LaunchStage(const void* src, void* dst, std::size_t bytes,
                cudaStream_t stream) {
  const std::size_t pieces = bytes / sizeof(Piece);
  const int ctas = static_cast<int>(std::min<std::size_t>(
      kMaxStageCtas, (pieces + kStageThreads - 1) / kStageThreads));
  return LaunchKernel(StageKernel<Piece>, dim3(ctas), dim3(kStageThreads), 0,
                      stream, dim3(1, 1, 1), static_cast<const Piece*>(src),
                      static_cast<Piece*>(dst), pieces);
}

}  // namespace

int StageBytes(void* dst, const void* src, std::size_t bytes,
               cudaStream_t stream) {
  if (bytes == 0)
    return kOk;
  if (dst == nullptr || src == nullptr)
    return kInvalid;
  const std::uintptr_t a = reinterpret_cast<std::uintptr_t>(dst);
  const std::uintptr_t b = reinterpret_cast<std::uintptr_t>(src);
  // The widest piece both addresses and the size allow.
  if ((a | b | bytes) % 16 == 0)
    return LaunchStage<uint4>(src, dst, bytes, stream);
  if ((a | b | bytes) % 4 == 0)
    return LaunchStage<std::uint32_t>(src, dst, bytes, stream);
  return LaunchStage<unsigned char>(src, dst, bytes, stream);
}

}  // namespace vx
