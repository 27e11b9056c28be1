// Device pieces of the skinny products shared by the product kernel
// (products.cu) and the persistent DiT kernel (persistent_dit.cu): the
// m16n8k16 MMA, the exact biased-int8 -> bf16 conversion and one
// 32-column block of one 16-row weight group.
#pragma once

#include <cstdint>

#include "products.cuh"
#include "vx_common.cuh"

namespace vx {

__device__ inline void Mma16816(float (&d)[4], std::uint32_t a0,
                                std::uint32_t a1, std::uint32_t a2,
                                std::uint32_t a3, std::uint32_t b0,
                                std::uint32_t b1, const float (&c)[4]) {
  // Not volatile: the MMA has no side effects, so the compiler may
  // interleave the independent MMAs of neighbouring tiles.
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, "
      "{%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]),
        "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

/// The same MMA on fp16 operands (both A and B fp16).
__device__ inline void Mma16816Half(float (&d)[4], std::uint32_t a0,
                                    std::uint32_t a1, std::uint32_t a2,
                                    std::uint32_t a3, std::uint32_t b0,
                                    std::uint32_t b1, const float (&c)[4]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, "
      "{%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]),
        "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

/// Four biased int8 values (q + 128) -> two fp16 pairs (bytes 0,1 and 2,3),
/// exactly: 0x64uu is 1024 + u as an fp16 (ten mantissa bits hold u), and
/// one packed subtraction of 1152 leaves q. Two instructions per pair,
/// against four for the bf16 route below.
__device__ inline void DequantWordHalf(std::uint32_t w, std::uint32_t& pair01,
                                       std::uint32_t& pair23) {
  const std::uint32_t bias = 0x64806480u;  // fp16 1152 in both halves
  const std::uint32_t a = Prmt(w, 0x64646464u, 0x5140u);
  const std::uint32_t b = Prmt(w, 0x64646464u, 0x5342u);
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(pair01) : "r"(a), "r"(bias));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(pair23) : "r"(b), "r"(bias));
}

/// Four biased int8 values (q + 128) -> two bf16 pairs (bytes 0,1 and 2,3),
/// exactly: 0x4B0000uu is 2^23 + u as a float; subtracting 2^23 + 128
/// leaves q, whose float has at most 8 significant bits, so its upper half
/// is its bf16.
__device__ inline void DequantWord(std::uint32_t w, std::uint32_t& pair01,
                                   std::uint32_t& pair23) {
  const float f0 = __uint_as_float(Prmt(w, 0x4B000000u, 0x7540u));
  const float f1 = __uint_as_float(Prmt(w, 0x4B000000u, 0x7541u));
  const float f2 = __uint_as_float(Prmt(w, 0x4B000000u, 0x7542u));
  const float f3 = __uint_as_float(Prmt(w, 0x4B000000u, 0x7543u));
  const float2 bias = make_float2(-8388736.0f, -8388736.0f);
  const float2 a = Add2(make_float2(f0, f1), bias);
  const float2 b = Add2(make_float2(f2, f3), bias);
  pair01 = Prmt(__float_as_uint(a.x), __float_as_uint(a.y), 0x7632u);
  pair23 = Prmt(__float_as_uint(b.x), __float_as_uint(b.y), 0x7632u);
}

/// One 32-column block of one 16-row group: the block's partial sums for
/// every activation tile, added into `acc` (Q8: scaled; bf16: directly).
/// kHalf (Q8 only): the activation fragments `b` hold fp16 and the weights
/// are dequantized to fp16 (the products and fp32 sums are the same).
template <int kFormat, int kNTiles, int kRowStride, bool kHalf = false>
__device__ __forceinline__ void BlockProduct(const unsigned char* base, int kb,
                                             int gid, int tig,
                                             const uint4 (&b)[kNTiles],
                                             float (&acc)[kNTiles][4]) {
  constexpr bool kQ8 = kFormat == static_cast<int>(WeightFormat::kQ8Tiles);
  constexpr bool kRows = kFormat == static_cast<int>(WeightFormat::kBf16);
  if constexpr (kQ8) {
    const unsigned char* tile = base + kb * kQ8TileBytes;
    const uint2 lo = *reinterpret_cast<const uint2*>(tile + gid * 32 + 8 * tig);
    const uint2 hi =
        *reinterpret_cast<const uint2*>(tile + (gid + 8) * 32 + 8 * tig);
    const std::uint32_t sc =
        *reinterpret_cast<const std::uint32_t*>(tile + 512 + 4 * gid);
    const float s_lo =
        HalfBitsToFloat(static_cast<std::uint16_t>(sc & 0xFFFFu));
    const float s_hi = HalfBitsToFloat(static_cast<std::uint16_t>(sc >> 16));
    std::uint32_t a00, a02, a01, a03, a10, a12, a11, a13;
    if constexpr (kHalf) {
      DequantWordHalf(lo.x, a00, a02);
      DequantWordHalf(hi.x, a01, a03);
      DequantWordHalf(lo.y, a10, a12);
      DequantWordHalf(hi.y, a11, a13);
    } else {
      DequantWord(lo.x, a00, a02);
      DequantWord(hi.x, a01, a03);
      DequantWord(lo.y, a10, a12);
      DequantWord(hi.y, a11, a13);
    }
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < kNTiles; ++j) {
      float part[4];
      if constexpr (kHalf) {
        Mma16816Half(part, a00, a01, a02, a03, b[j].x, b[j].y, zero);
        Mma16816Half(part, a10, a11, a12, a13, b[j].z, b[j].w, part);
      } else {
        Mma16816(part, a00, a01, a02, a03, b[j].x, b[j].y, zero);
        Mma16816(part, a10, a11, a12, a13, b[j].z, b[j].w, part);
      }
      const float2 lo2 =
          Fma2(make_float2(s_lo, s_lo), make_float2(part[0], part[1]),
               make_float2(acc[j][0], acc[j][1]));
      const float2 hi2 =
          Fma2(make_float2(s_hi, s_hi), make_float2(part[2], part[3]),
               make_float2(acc[j][2], acc[j][3]));
      acc[j][0] = lo2.x;
      acc[j][1] = lo2.y;
      acc[j][2] = hi2.x;
      acc[j][3] = hi2.y;
    }
  } else {
    const unsigned char* row_lo;
    const unsigned char* row_hi;
    if constexpr (kRows) {
      row_lo = base + gid * kRowStride + kb * 64;
      row_hi = base + (gid + 8) * kRowStride + kb * 64;
    } else {
      const unsigned char* tile = base + kb * kBf16TileBytes;
      row_lo = tile + gid * 64;
      row_hi = tile + (gid + 8) * 64;
    }
    const uint4 lo = *reinterpret_cast<const uint4*>(row_lo + 16 * tig);
    const uint4 hi = *reinterpret_cast<const uint4*>(row_hi + 16 * tig);
#pragma unroll
    for (int j = 0; j < kNTiles; ++j) {
      Mma16816(acc[j], lo.x, hi.x, lo.y, hi.y, b[j].x, b[j].y, acc[j]);
      Mma16816(acc[j], lo.z, hi.z, lo.w, hi.w, b[j].z, b[j].w, acc[j]);
    }
  }
}

}  // namespace vx
