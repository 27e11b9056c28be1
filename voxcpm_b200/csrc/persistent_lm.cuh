// The persistent one-row decoder stack: every layer of a MiniCPM4 stack
// (the 28-layer LM or the 8-layer residual LM) for the one new row of a
// generation step, as ONE cooperative kernel with one CTA per SM. It
// replaces ForwardStack at one row (transformer.cpp:55-100) with the decode
// attention over the KV cache and the cache append
// (kernels/generator_kernels.hip:91-254).
//
// Work split: every product is cut into units of one 16-row weight group
// over the whole reduction (two to six 32-tile slots of the tile layout), so
// the unit's CTA owns its outputs and adds them into the residual row
// itself. A producer warp streams the CTA's units for all layers into a
// ring of 17.4 KB slots with 1-D TMA bulk copies; sixteen consumer warps own
// 64 reduction columns each and hold the row as register fragments.
// Attention runs as 16 heads x 8 key chunks: each task writes an online-
// softmax partial, and the O phase's warps merge the partials of their own
// head. Phases wait on monotone counters published by a publisher warp.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "products.cuh"

namespace vx {

/// The stack shape the kernel is built for (VoxCPM2's LM and residual LM).
struct LmShape {
  static constexpr int kHidden = 2048;
  static constexpr int kIntermediate = 6144;
  static constexpr int kHeads = 16;
  static constexpr int kKvHeads = 2;
  static constexpr int kHeadDim = 128;
  static constexpr int kKeySplits = 8;  // key chunks per head
};

/// One layer: Q8_0 tiles, norms and this layer's KV cache
/// ([kv head][capacity][128], fp32 or bf16).
struct LmLayer {
  const unsigned char* qkv = nullptr;      // [q 2048 | k 256 | v 256][2048]
  const unsigned char* o = nullptr;        // [2048][2048]
  const unsigned char* gate_up = nullptr;  // [gate 6144 | up 6144][2048]
  const unsigned char* down = nullptr;     // [2048][6144]
  const std::uint16_t* input_norm = nullptr;
  const std::uint16_t* post_norm = nullptr;
  void* keys = nullptr;
  void* values = nullptr;
};

constexpr int kLmSyncWords = 64;

struct LmStackParams {
  int layers = 0;
  int bf16_kv = 0;
  int capacity = 0;
  float eps = 1e-5f;
  float attention_scale = 0.0f;
  const LmLayer* layer = nullptr;          // device array [layers]
  const std::uint16_t* final_norm = nullptr;
  const float* rope = nullptr;             // [position][cos 64 | sin 64] or null
  const std::int32_t* position = nullptr;  // device: rows already cached
  float* hidden = nullptr;                 // [2048] residual row, in and out
  float* output = nullptr;                 // [2048] final norm (fp32)
  // Work buffers (device), laid out by LmWorkLayout.
  float* qkv = nullptr;        // [2560]
  float* att_parts = nullptr;  // [16][8][132]: o[128], max, sum
  std::uint16_t* act = nullptr;  // [6144]
  unsigned* sync = nullptr;      // [kLmSyncWords]
};

std::size_t LmWorkBytes();
void LmWorkLayout(void* base, LmStackParams& params);

/// Whether the current device can run the persistent stack.
bool LmStackSupported();

/// Enqueues the stack on `stream`: a memset of the sync words, then the
/// cooperative kernel. `hidden` is read and updated, `output` written, the
/// new row's keys and values appended at row *position of each layer's
/// cache. Returns a Status.
int LaunchLmStack(const LmStackParams& params, cudaStream_t stream);

}  // namespace vx
