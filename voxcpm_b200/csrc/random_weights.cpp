// Seeded synthetic weights on the host (random-init checkpoints for the
// benchmarks and parity tests; the reference reads real checkpoints,
// weights.cpp:26-327, which are out of scope here).
//
// Values are a pure function of (seed, tensor id, index), computed with
// integer arithmetic plus one float multiply and one round-to-nearest-even
// conversion, so any implementation reproduces them bit for bit:
//   h      = mix(mix(seed ^ tensor * 0xD1B54A32D192ED03) ^ index)   (splitmix64)
//   normal ~ (sum of the four 16-bit words of h - 131070) / (65536 / sqrt 3)
//   Q8_0   : q = h % 255 - 127 (uniform in [-127, 127]); per 32 values one
//            fp16 scale |normal| * std (the BASELINE distribution
//            |N(0, 0.02)| / 127 with std = 0.02 / 127)
//   bf16   : bf16(mean + normal * std)
#include "vx_status.h"

#include "../../include/voxcpm_b200.h"

#include <cmath>
#include <cstdint>
#include <cstring>
#include <algorithm>
#include <thread>
#include <vector>

namespace {

std::uint64_t Mix64(std::uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

std::uint64_t Hash(std::uint64_t seed, std::uint64_t tensor,
                   std::uint64_t index) {
  return Mix64(Mix64(seed ^ (tensor * 0xD1B54A32D192ED03ull)) ^ index);
}

std::int32_t CentredSum(std::uint64_t h) {
  std::int32_t s = 0;
  for (int i = 0; i < 4; ++i)
    s += static_cast<std::int32_t>((h >> (16 * i)) & 0xFFFFu);
  return s - 131070;
}

constexpr float kSumStd = 37837.226f;  // 65536 / sqrt(3)

std::uint32_t Bits(float v) {
  std::uint32_t b;
  std::memcpy(&b, &v, 4);
  return b;
}

float FromBits(std::uint32_t b) {
  float v;
  std::memcpy(&v, &b, 4);
  return v;
}

std::uint16_t Bf16Bits(float value) {
  const std::uint32_t bits = Bits(value);
  if ((bits & 0x7F800000u) == 0x7F800000u && (bits & 0x007FFFFFu) != 0)
    return static_cast<std::uint16_t>((bits >> 16) | 0x40u);
  const std::uint32_t rounding = 0x7FFFu + ((bits >> 16) & 1u);
  return static_cast<std::uint16_t>((bits + rounding) >> 16);
}

/// float -> binary16 bits, round to nearest even.
std::uint16_t HalfBits(float value) {
  const std::uint32_t bits = Bits(value);
  const auto sign = static_cast<std::uint16_t>((bits >> 16) & 0x8000u);
  const std::uint32_t magnitude = bits & 0x7FFFFFFFu;
  if (magnitude >= 0x7F800000u)
    return static_cast<std::uint16_t>(sign | 0x7C00u |
                                      (magnitude > 0x7F800000u ? 0x200u : 0));
  const float a = FromBits(magnitude);
  if (a >= 65520.0f)
    return static_cast<std::uint16_t>(sign | 0x7C00u);
  if (a < 6.103515625e-05f) {
    const float r = std::nearbyint(a * 16777216.0f);
    return static_cast<std::uint16_t>(sign | static_cast<std::uint16_t>(r));
  }
  const int exponent = static_cast<int>((magnitude >> 23) & 0xFFu) - 112;
  const std::uint32_t mantissa = magnitude & 0x7FFFFFu;
  std::uint32_t half = (static_cast<std::uint32_t>(exponent) << 10) |
                       (mantissa >> 13);
  const std::uint32_t rest = mantissa & 0x1FFFu;
  if (rest > 0x1000u || (rest == 0x1000u && (half & 1u)))
    half += 1;
  return static_cast<std::uint16_t>(sign | half);
}

template <typename F>
void Parallel(std::size_t count, F&& body) {
  unsigned threads = std::thread::hardware_concurrency();
  if (threads == 0)
    threads = 1;
  if (count < 65536 || threads == 1) {
    body(0, count);
    return;
  }
  threads = std::min<unsigned>(threads, 64);
  std::vector<std::thread> pool;
  const std::size_t chunk = (count + threads - 1) / threads;
  for (unsigned t = 0; t < threads; ++t) {
    const std::size_t begin = t * chunk;
    const std::size_t end = std::min(count, begin + chunk);
    if (begin >= end)
      break;
    pool.emplace_back([&body, begin, end] { body(begin, end); });
  }
  for (auto& thread : pool)
    thread.join();
}

}  // namespace

extern "C" {

/* Host: GGML Q8_0 blocks [rows][in/32] of seeded weights. */
vx_status vx_random_q8_0(uint64_t seed, uint64_t tensor, size_t rows,
                         size_t in, float scale_std, uint8_t* blocks) {
  if (blocks == nullptr || in % 32 != 0)
    return vx::Fail(vx::kInvalid, "vx_random_q8_0: bad arguments");
  const float factor = scale_std / kSumStd;
  Parallel(rows * (in / 32), [&](std::size_t begin, std::size_t end) {
    for (std::size_t b = begin; b < end; ++b) {
      std::uint8_t* target = blocks + b * 34;
      const std::uint64_t hs = Hash(seed, tensor, (std::uint64_t{1} << 62) | b);
      const float scale =
          std::fabs(static_cast<float>(CentredSum(hs))) * factor;
      const std::uint16_t bits = HalfBits(scale);
      target[0] = static_cast<std::uint8_t>(bits & 0xFFu);
      target[1] = static_cast<std::uint8_t>(bits >> 8);
      for (int i = 0; i < 32; ++i) {
        const std::uint64_t h = Hash(seed, tensor, b * 32 + i);
        const int q = static_cast<int>(h % 255u) - 127;
        target[2 + i] = static_cast<std::uint8_t>(static_cast<std::int8_t>(q));
      }
    }
  });
  return VX_OK;
}

/* Host: `count` seeded bf16 values bf16(mean + N(0, std)). */
vx_status vx_random_bf16(uint64_t seed, uint64_t tensor, size_t count,
                         float mean, float std, uint16_t* out) {
  if (out == nullptr)
    return vx::Fail(vx::kInvalid, "vx_random_bf16: null output");
  const float factor = std / kSumStd;
  Parallel(count, [&](std::size_t begin, std::size_t end) {
    for (std::size_t i = begin; i < end; ++i) {
      const float v =
          static_cast<float>(CentredSum(Hash(seed, tensor, i))) * factor;
      out[i] = Bf16Bits(mean + v);
    }
  });
  return VX_OK;
}

}  // extern "C"
