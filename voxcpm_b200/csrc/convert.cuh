// Load-time conversions of checkpoint tensors to bf16 (convert.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace vx {

/// output[i] = bf16(input[i]) for fp16 input (device arrays).
int HalfToBf16(const std::uint16_t* input, std::uint16_t* output,
               std::size_t count, cudaStream_t stream);
/// output[i] = bf16(input[i]) for fp32 input.
int FloatToBf16(const float* input, std::uint16_t* output, std::size_t count,
                cudaStream_t stream);
/// GGML Q8_0 blocks (fp16 scale, 32 int8) to bf16(scale * q); `count` values,
/// a multiple of 32.
int Q8_0ToBf16(const std::uint8_t* blocks, std::uint16_t* output,
               std::size_t count, cudaStream_t stream);

}  // namespace vx
