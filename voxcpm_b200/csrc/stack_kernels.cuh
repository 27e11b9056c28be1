// Kernels of the MiniCPM4 stacks and the generation step on sm_100a
// (replace kernels/generator_kernels.hpp:18-107). The residual stream,
// norms, attention and elementwise steps run in fp32; outputs feeding a
// product are rounded to bf16 (RNE) at the reference's points.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace vx {

/// Element type of a KV cache: fp32 (the reference's, transformer.hpp:17-36)
/// or bf16 (half the bytes per decode step).
enum class CacheType : int { kF32 = 0, kBf16 = 1 };

int Embed(const std::uint16_t* table, const std::int32_t* ids,
          const std::int32_t* text_mask, float* output, std::size_t rows,
          std::size_t width, float scale, cudaStream_t stream);
int ScatterRows(const float* input, const std::int32_t* indices, float* output,
                std::size_t rows, std::size_t width, cudaStream_t stream);
int GatherRows(const float* input, const std::int32_t* indices, float* output,
               std::size_t rows, std::size_t width, cudaStream_t stream);
int RmsNorm(const float* input, const std::uint16_t* weight,
            std::uint16_t* output, float* output_f32, std::size_t rows,
            std::size_t width, float epsilon, cudaStream_t stream);
/// Positions and cache rows are device arrays of one entry per row.
int QkvRope(const float* qkv, const float* cos_sin,
            const std::int32_t* positions, const std::int32_t* cache_rows,
            float* q, void* k_cache, void* v_cache, CacheType cache_type,
            std::size_t rows, std::size_t heads, std::size_t kv_heads,
            std::size_t head_dim, std::size_t capacity, cudaStream_t stream);
/// `past` keys before each sequence's rows; when `past_device` is not null
/// the kernel reads `past` from it (graph replays with a moving position),
/// one value per sequence with `past_per_sequence`, and `max_keys` bounds the
/// keys a row may see. A sequence's keys start at cache row
/// sequence * keys_per_sequence, or at first_keys[sequence] when given.
int Attention(const float* q, const void* k_cache, const void* v_cache,
              CacheType cache_type, std::uint16_t* output, std::size_t rows,
              std::size_t rows_per_sequence, std::size_t keys_per_sequence,
              std::size_t past, const std::int32_t* past_device, bool causal,
              std::size_t heads, std::size_t kv_heads, std::size_t head_dim,
              std::size_t capacity, std::size_t max_keys, cudaStream_t stream,
              bool past_per_sequence = false,
              const std::int32_t* first_keys = nullptr);
int SwiGlu(const float* gate_up, std::uint16_t* output, std::size_t rows,
           std::size_t width, cudaStream_t stream);
int AddBias(float* data, const std::uint16_t* bias, std::size_t rows,
            std::size_t width, cudaStream_t stream);
int ToBf16(const float* input, std::uint16_t* output, std::size_t count,
           bool silu, cudaStream_t stream);
int ConcatRows(const float* a, const float* a_scale, std::size_t a_width,
               const float* b, const float* b_scale, std::size_t b_width,
               std::uint16_t* output, std::size_t rows, cudaStream_t stream);
int Quantize(const float* input, std::uint16_t* output, std::size_t count,
             float scale, cudaStream_t stream);
int SelectRows(const float* quantized, const float* plain,
               const std::int32_t* mask, float* output, std::size_t rows,
               std::size_t width, cudaStream_t stream);
int PrependSpecial(const float* rows_in, const std::uint16_t* special,
                   float* output, std::size_t patches, std::size_t patch_size,
                   std::size_t width, cudaStream_t stream);
int AssembleDit(const float* mu, const float* time, const float* cond,
                const float* x, float* output, std::size_t patch_size,
                std::size_t width, cudaStream_t stream);
int GuidedEuler(const float* velocity, float* x, std::size_t count, float cfg,
                float dt, cudaStream_t stream);
/// Copies `count` floats (a device-side copy kernel that takes part in
/// programmatic dependent launch).
int CopyFloats(const float* input, float* output, std::size_t count,
               cudaStream_t stream);
/// Copies `count` floats into slot (*position & 1) of `slots` ([2][count]):
/// a two-slot ring indexed by the device-held decode position, graph-safe.
int CopyToParitySlot(const float* input, float* slots, std::size_t count,
                     const std::int32_t* position, cudaStream_t stream);
/// *counter += 1 and positions[0] = *counter (the decode step's moving
/// position, graph-safe).
int AdvancePosition(std::int32_t* counter, std::int32_t* positions,
                    cudaStream_t stream);

}  // namespace vx
