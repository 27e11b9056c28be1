// Load-time conversion of checkpoint tensors to the bf16 the kernels read
// (kernels/convert_kernels.hpp:9-24): fp16 -> bf16, fp32 -> bf16 and GGML
// Q8_0 -> bf16 (bf16(scale * q)), each rounded to nearest even with NaN
// kept quiet and the top bits of its payload kept. HBM-bound byte work:
// grid-stride loops over eight values (fp16, fp32) or one 32-value block
// (Q8_0) per thread, with 16-byte loads and stores where the pointers allow,
// on a grid of a few CTAs per SM.
#include "convert.cuh"
#include "vx_common.cuh"
#include "vx_status.h"

#include <cstdint>

namespace vx {

namespace {

constexpr int kThreads = 256;

unsigned GridFor(std::size_t work) {
  int device = 0;
  int sms = 148;
  if (cudaGetDevice(&device) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const std::size_t wanted = (work + kThreads - 1) / kThreads;
  const std::size_t cap = static_cast<std::size_t>(sms) * 8;
  return static_cast<unsigned>(wanted < cap ? (wanted == 0 ? 1 : wanted) : cap);
}

bool Aligned16(const void* p) {
  return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0;
}

/// IEEE 754 binary16 -> binary32 from the bit layout, exact, with NaN
/// payloads kept (the reference widens with a plain _Float16 conversion,
/// kernels/device_math.hpp:22-24, which keeps them; __half2float returns a
/// canonical NaN).
__device__ inline float HalfToFloatExact(std::uint16_t h) {
  const std::uint32_t sign = static_cast<std::uint32_t>(h & 0x8000u) << 16;
  const std::uint32_t exponent = (h >> 10) & 0x1Fu;
  const std::uint32_t mantissa = h & 0x3FFu;
  if (exponent == 0x1Fu)
    return __uint_as_float(sign | 0x7F800000u | (mantissa << 13));
  if (exponent != 0)
    return __uint_as_float(sign | ((exponent + 112u) << 23) | (mantissa << 13));
  // Zero or subnormal: mantissa * 2^-24, exact in binary32.
  const float magnitude = static_cast<float>(mantissa) * 5.9604644775390625e-8f;
  return sign != 0 ? -magnitude : magnitude;
}

__device__ inline std::uint32_t Pack(Bf16 lo, Bf16 hi) {
  return static_cast<std::uint32_t>(lo) | (static_cast<std::uint32_t>(hi) << 16);
}

/// Eight values per thread per step; `vector` when both pointers are 16-byte
/// aligned (the tail past the last whole group of eight runs scalar).
template <bool kHalf>
__global__ void ToBf16Kernel(const void* input, Bf16* output, std::size_t count,
                             bool vector) {
  const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
  const std::size_t first = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const std::size_t groups = vector ? count / 8 : 0;
  for (std::size_t g = first; g < groups; g += stride) {
    float v[8];
    if constexpr (kHalf) {
      const uint4 raw = reinterpret_cast<const uint4*>(input)[g];
      const std::uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = HalfToFloatExact(static_cast<std::uint16_t>(w[i] & 0xFFFFu));
        v[2 * i + 1] = HalfToFloatExact(static_cast<std::uint16_t>(w[i] >> 16));
      }
    } else {
      const float4 a = reinterpret_cast<const float4*>(input)[2 * g];
      const float4 b = reinterpret_cast<const float4*>(input)[2 * g + 1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    uint4 out;
    out.x = Pack(FloatToBf16(v[0]), FloatToBf16(v[1]));
    out.y = Pack(FloatToBf16(v[2]), FloatToBf16(v[3]));
    out.z = Pack(FloatToBf16(v[4]), FloatToBf16(v[5]));
    out.w = Pack(FloatToBf16(v[6]), FloatToBf16(v[7]));
    reinterpret_cast<uint4*>(output)[g] = out;
  }
  for (std::size_t i = groups * 8 + first; i < count; i += stride) {
    const float v = kHalf ? HalfToFloatExact(static_cast<const std::uint16_t*>(input)[i])
                          : static_cast<const float*>(input)[i];
    output[i] = FloatToBf16(v);
  }
}

/// One 34-byte block (fp16 scale, 32 int8) per thread per step: 64 bytes of
/// bf16 out, as four 16-byte stores when the output is aligned.
__global__ void Q8_0ToBf16Kernel(const std::uint8_t* blocks, Bf16* output,
                                 std::size_t count_blocks, bool vector) {
  const std::size_t stride = static_cast<std::size_t>(gridDim.x) * blockDim.x;
  for (std::size_t b = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       b < count_blocks; b += stride) {
    const std::uint8_t* block = blocks + b * 34;
    const float scale = HalfToFloatExact(
        static_cast<std::uint16_t>(block[0] | (block[1] << 8)));
    // A NaN scale propagates with its payload (IEEE multiply), which the
    // GPU's multiply would replace by its canonical NaN.
    const bool nan_scale = scale != scale;
    Bf16 out[32];
    for (int i = 0; i < 32; ++i)
      out[i] = FloatToBf16(nan_scale ? scale
                                     : scale * static_cast<float>(static_cast<std::int8_t>(block[2 + i])));
    Bf16* target = output + b * 32;
    if (vector) {
      for (int i = 0; i < 4; ++i) {
        uint4 v;
        v.x = Pack(out[8 * i], out[8 * i + 1]);
        v.y = Pack(out[8 * i + 2], out[8 * i + 3]);
        v.z = Pack(out[8 * i + 4], out[8 * i + 5]);
        v.w = Pack(out[8 * i + 6], out[8 * i + 7]);
        reinterpret_cast<uint4*>(target)[i] = v;
      }
    } else {
      for (int i = 0; i < 32; ++i)
        target[i] = out[i];
    }
  }
}

int Launched() { return cudaGetLastError() == cudaSuccess ? kOk : kCudaError; }

}  // namespace

int HalfToBf16(const std::uint16_t* input, std::uint16_t* output,
               std::size_t count, cudaStream_t stream) {
  if (count == 0)
    return kOk;
  if (input == nullptr || output == nullptr)
    return kInvalid;
  ToBf16Kernel<true><<<GridFor((count + 7) / 8), kThreads, 0, stream>>>(
      input, output, count, Aligned16(input) && Aligned16(output));
  return Launched();
}

int FloatToBf16(const float* input, std::uint16_t* output, std::size_t count,
                cudaStream_t stream) {
  if (count == 0)
    return kOk;
  if (input == nullptr || output == nullptr)
    return kInvalid;
  ToBf16Kernel<false><<<GridFor((count + 7) / 8), kThreads, 0, stream>>>(
      input, output, count, Aligned16(input) && Aligned16(output));
  return Launched();
}

int Q8_0ToBf16(const std::uint8_t* blocks, std::uint16_t* output,
               std::size_t count, cudaStream_t stream) {
  if (count == 0)
    return kOk;
  if (blocks == nullptr || output == nullptr || count % 32 != 0)
    return kInvalid;
  Q8_0ToBf16Kernel<<<GridFor(count / 32), kThreads, 0, stream>>>(
      blocks, output, count / 32, Aligned16(output));
  return Launched();
}

}  // namespace vx
