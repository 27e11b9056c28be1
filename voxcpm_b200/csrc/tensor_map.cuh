// Host-side encoding of TMA tensor maps (cuTensorMapEncodeTiled, reached
// through the runtime's driver entry point, so the library does not link
// against the driver library).
#pragma once

#include <cuda.h>

#include <cstdint>

namespace vx {

/// Encodes a tiled tensor map of `rank` dimensions over `base` (bf16
/// elements): `dims` innermost first, `strides` the byte strides of
/// dimensions 1..rank-1, `box` the box extent per dimension. Loads past the
/// tensor's extent read zeros. Returns false when the driver refuses it.
bool EncodeBf16TensorMap(CUtensorMap* map, const void* base, int rank,
                         const std::uint64_t* dims,
                         const std::uint64_t* strides,
                         const std::uint32_t* box, CUtensorMapSwizzle swizzle);

}  // namespace vx
