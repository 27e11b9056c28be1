// Kernel launch helper: every launch of the library carries the
// programmatic-dependent-launch attribute (when enabled), so a kernel's
// prologue overlaps its predecessor's tail inside streams and CUDA graphs,
// and optionally a thread-block cluster shape.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <utility>

#include "products.cuh"
#include "vx_status.h"

namespace vx {

template <typename... Params, typename... Args>
int LaunchKernel(void (*kernel)(Params...), dim3 grid, dim3 block,
                 std::size_t smem, cudaStream_t stream, dim3 cluster,
                 Args&&... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attributes[2];
  int count = 0;
  if (cluster.x * cluster.y * cluster.z > 1) {
    attributes[count].id = cudaLaunchAttributeClusterDimension;
    attributes[count].val.clusterDim.x = cluster.x;
    attributes[count].val.clusterDim.y = cluster.y;
    attributes[count].val.clusterDim.z = cluster.z;
    ++count;
  }
  if (ProgrammaticLaunch()) {
    attributes[count].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attributes[count].val.programmaticStreamSerializationAllowed = 1;
    ++count;
  }
  config.attrs = attributes;
  config.numAttrs = count;
  return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...) ==
                 cudaSuccess
             ? kOk
             : kCudaError;
}

}  // namespace vx
