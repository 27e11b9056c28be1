// The persistent DiT patch: the whole Euler/CFG loop of one patch (every
// DiT evaluation of the local DiT, its in/out projections and the CFG-Zero*
// Euler updates) as ONE cooperative kernel with one CTA per SM. It replaces
// the per-kernel sequence of Generator::EvaluateDit / GuidedEuler
// (generator.cpp:297-324, :457-463) and ForwardStack (transformer.cpp:55-100)
// for VoxCPM2's DiT shape.
//
// Work split: every product is cut into units of one 16-row weight group
// times 1024 reduction columns (32 tiles, one contiguous run of the tile
// layout). A producer warp per CTA streams its units for the whole patch
// into a ring of unit-sized shared-memory slots with 1-D TMA bulk copies,
// running ahead across layers; sixteen consumer warps take two tiles each
// and reduce in a fixed order. There is no grid barrier: each phase (QKV,
// O, gate/up, down, the patch boundary) waits only on monotone ready
// counters of the data it reads, published with release semantics (by a
// publisher warp, so compute warps never stall on a fence). Attention runs
// as 32 (head, sequence) tasks on CTAs that hold a single QKV unit. The
// split reductions of O (two 1024-column parts) and down (four) live on a
// CTA pair (a cluster of two): rank 1 sends its reduced parts through
// distributed shared memory and rank 0 adds them into the residual stream
// in a fixed part order, so results are deterministic.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "products.cuh"

namespace vx {

/// The DiT shape the persistent kernel is built for (VoxCPM2's local DiT).
struct DitShape {
  static constexpr int kHidden = 1024;
  static constexpr int kIntermediate = 4096;
  static constexpr int kHeads = 16;
  static constexpr int kKvHeads = 2;
  static constexpr int kHeadDim = 128;
  static constexpr int kPatch = 4;
  static constexpr int kFeat = 64;
  static constexpr int kSequence = 3 + 2 * kPatch;  // mu, mu, time, cond, x
  static constexpr int kRows = 2 * kSequence;       // CFG pair
};

/// One DiT layer's device weights (Q8 tiles or bf16 tiles) and norms.
struct DitLayer {
  const unsigned char* qkv = nullptr;      // [q 2048 | k 256 | v 256][1024]
  const unsigned char* o = nullptr;        // [1024][2048]
  const unsigned char* gate_up = nullptr;  // [gate 4096 | up 4096][1024]
  const unsigned char* down = nullptr;     // [1024][4096]
  const std::uint16_t* input_norm = nullptr;
  const std::uint16_t* post_norm = nullptr;
};

/// Words of the per-launch synchronization block (zeroed by the launcher).
constexpr int kDitSyncWords = 256;

/// Everything the persistent patch reads and writes.
struct DitPatchParams {
  WeightFormat format = WeightFormat::kQ8Tiles;  // kQ8Tiles or kBf16Tiles
  int layers = 0;
  int evaluations = 0;      // Euler steps that evaluate the DiT
  int bf16_kv = 0;          // round keys and values to bf16 (bf16 KV cache)
  float eps = 1e-5f;
  float cfg = 2.0f;
  float attention_scale = 0.0f;
  const DitLayer* layer = nullptr;  // device array [layers]
  const std::uint16_t* final_norm = nullptr;
  const unsigned char* dit_in = nullptr;  // tiles [1024][64]
  const std::uint16_t* dit_in_bias = nullptr;
  const unsigned char* dit_out = nullptr;  // tiles [64][1024]
  const std::uint16_t* dit_out_bias = nullptr;
  const float* rope = nullptr;       // [position][cos 64 | sin 64] or null
  const float* mu = nullptr;         // [2][1024]
  const float* cond_rows = nullptr;  // [4][1024]
  const float* const* time_vectors = nullptr;  // device [evaluations] -> [1024]
  const float* dts = nullptr;                  // device [evaluations]
  float* x = nullptr;                // [4][64]: noise in, latent out
  // Work buffers (device).
  float* hidden = nullptr;      // [22][1024] residual stream
  float* qkv = nullptr;         // [22][2560]
  std::uint16_t* att = nullptr; // [22][2048]
  std::uint16_t* act = nullptr; // [22][4096]
  unsigned* sync = nullptr;     // [kDitSyncWords]
  // Test hook (0: off): CTA 0 first waits for a sync word that no CTA ever
  // sets, gives up after this many nanoseconds and aborts the launch, so a
  // test can run the bounded-wait error path without a GPU fault.
  std::uint64_t stall_limit_ns = 0;
};

/// The test hook above for every later launch of this process (0: off).
void SetDitStall(std::uint64_t limit_ns);
/// The CTA cap and the cooperative attribute of the persistent kernels
/// (persistent_common.cuh).
void SetPersistentMaxCtas(int ctas);
void SetPersistentCooperative(bool enabled);
/// Whether the last launch that used `params.sync` aborted (sync word 0 set
/// by a CTA whose bounded wait gave up); clears the word. Synchronizes
/// `stream` first.
int DitLaunchAborted(const DitPatchParams& params, cudaStream_t stream,
                     bool* aborted);
/// The same for the allocation-free launch's sync words.
int DitStaticLaunchAborted(cudaStream_t stream, bool* aborted);

/// Device bytes of the work buffers above (hidden .. sync), laid out
/// in that order with 256-byte alignment by DitWorkLayout.
std::size_t DitWorkBytes();
/// Points the work-buffer fields of `params` into `base` (DitWorkBytes()).
void DitWorkLayout(void* base, DitPatchParams& params);

/// Whether the current device can run the persistent patch for `format`
/// (cooperative launch of co-resident CTA pairs, at least one pair per
/// 16-column residual group).
bool DitPatchSupported(WeightFormat format);

/// Enqueues the persistent patch on `stream`: a memset of the sync words,
/// then the cooperative kernel (CTA pairs as clusters of two, one CTA per
/// SM). Returns a Status.
int LaunchDitPatch(const DitPatchParams& params, cudaStream_t stream);

/// LaunchDitPatch with the work buffers (and sync words) placed in a fixed
/// 1 MiB device array of this library instead of `params`' buffers: nothing
/// is allocated. The first call on a device looks the array's address up
/// (make it before any stream capture). Launches overlapping on the GPU
/// share the array and race.
int LaunchDitPatchStatic(const DitPatchParams& params, cudaStream_t stream);

}  // namespace vx
