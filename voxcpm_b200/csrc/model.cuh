// The generator's model layer on sm_100a: configuration, device weights,
// KV caches, the MiniCPM4 stack loop and the per-patch generation step.
// Replaces transformer.hpp (KvCache, AttentionLayout, StackScratch,
// RopeTable, ForwardStack, Project), weights.hpp (Projection, LayerWeights,
// StackWeights, GeneratorWeights, DeviceWeights) and generator.hpp
// (Generator, EulerStep, EulerSchedule).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <map>
#include <tuple>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "persistent_dit.cuh"
#include "persistent_lm.cuh"
#include "products.cuh"
#include "stack_kernels.cuh"

namespace vx {

/// One MiniCPM4 stack (config.hpp:15-31).
struct StackConfig {
  int hidden = 0;
  int intermediate = 0;
  int layers = 0;
  int heads = 0;
  int kv_heads = 0;
  int head_dim = 0;
  float rms_eps = 1e-5f;
  bool rope = true;
};

/// The generator's configuration (config.hpp:78-92).
struct ModelConfig {
  StackConfig lm, residual_lm, encoder, dit;
  double rope_theta = 10000.0;
  double rope_scaling = 1.0;
  std::vector<double> rope_factors;  // head_dim / 2 LongRoPE factors
  int patch_size = 4;
  int feat_dim = 64;
  int fsq_latent_dim = 512;
  float fsq_scale = 9.0f;
  int max_length = 8192;
  int vocab = 0;
};

/// A linear layer y = x W^T (+ b) (weights.hpp:20-26).
struct Projection {
  WeightFormat format = WeightFormat::kBf16;
  const void* weight = nullptr;
  const std::uint16_t* bias = nullptr;
  int in = 0;
  int out = 0;
};

struct LayerWeights {
  const std::uint16_t* input_norm = nullptr;
  Projection qkv;  // [q heads | k heads | v heads]
  Projection o;
  const std::uint16_t* post_norm = nullptr;
  Projection gate_up;  // [gate | up]
  Projection down;
};

struct StackWeights {
  StackConfig config;
  std::vector<LayerWeights> layers;
  const std::uint16_t* norm = nullptr;
};

struct GeneratorWeights {
  StackWeights base_lm, residual_lm, encoder, dit;
  const std::uint16_t* embed = nullptr;
  const std::uint16_t* special = nullptr;
  Projection encoder_in, enc_to_lm, lm_to_dit, res_to_dit, fusion, fsq_in,
      fsq_out, stop_proj, stop_head, dit_in, dit_cond, dit_out, time_1, time_2,
      delta_time_1, delta_time_2;
};

/// Which matrix formats a seeded checkpoint uses: like a GGUF Q8_0
/// checkpoint (every matrix Q8 tiles) or like the HF bf16 one (the DiT in
/// bf16 tiles, everything else bf16 rows) (weights.cpp:138-144, :281-282).
enum class CheckpointKind : int { kQ8 = 0, kBf16 = 1 };

/// Keys and values of one stack: [layer][kv_head][capacity][head_dim] each
/// (transformer.hpp:17-36).
class KvCache {
 public:
  KvCache() = default;
  /// [layer][kv_head][capacity][head_dim] keys and values; with `slots` > 1,
  /// [layer][slot][kv_head][capacity][head_dim]: one cache per slot, each a
  /// view (Slot) that the one-sequence kernels read as usual, while a kernel
  /// given slot 0's pointers reaches slot s at s * kv_heads * capacity rows.
  KvCache(const StackConfig& config, int capacity, CacheType type,
          int slots = 1);
  ~KvCache();
  KvCache(const KvCache&) = delete;
  KvCache& operator=(const KvCache&) = delete;
  KvCache(KvCache&& other) noexcept;
  KvCache& operator=(KvCache&& other) noexcept;

  int capacity() const { return capacity_; }
  CacheType type() const { return type_; }
  void* keys(int layer) const;
  void* values(int layer) const;
  std::size_t bytes() const { return bytes_; }
  /// A non-owning view of slot `slot` (valid while this cache lives).
  KvCache Slot(int slot) const;

 private:
  void Release();
  unsigned char* keys_ = nullptr;
  unsigned char* values_ = nullptr;
  bool owns_ = true;
  std::size_t slot_bytes_ = 0;
  std::size_t layer_bytes_ = 0;
  std::size_t bytes_ = 0;
  int capacity_ = 0;
  CacheType type_ = CacheType::kF32;
};

/// Which keys each row attends to (transformer.hpp:38-48). `past_device`,
/// when set, holds `past` on the device (graph replays) and `max_keys`
/// bounds the keys a row may see.
struct AttentionLayout {
  const std::int32_t* positions = nullptr;
  const std::int32_t* cache_rows = nullptr;
  int rows_per_sequence = 0;
  int keys_per_sequence = 0;
  int past = 0;
  const std::int32_t* past_device = nullptr;
  int max_keys = 0;
  bool causal = true;
  bool past_per_sequence = false;  // past_device holds one value per sequence
  const std::int32_t* first_keys = nullptr;  // device: each sequence's first key row
};

/// Scratch shared by the stacks of one generator (transformer.hpp:50-58).
struct StackScratch {
  std::uint16_t* normed = nullptr;
  float* qkv = nullptr;
  float* q = nullptr;
  std::uint16_t* attention = nullptr;
  float* gate_up = nullptr;
  std::uint16_t* activation = nullptr;
};

/// y[rows][out] = x W^T (+ y when accumulating) (+ b), chunks of 32 rows
/// (gemm.cpp:259-313; transformer.cpp:47-53 adds the bias).
int Linear(const std::uint16_t* x, const Projection& p, float* y, int rows,
           bool accumulate, cudaStream_t stream);
int Project(const Projection& p, const std::uint16_t* x, float* y, int rows,
            cudaStream_t stream);

/// One MiniCPM4 stack over `rows` rows of the fp32 residual stream `hidden`
/// (updated in place); the final norm's fp32 output goes to `output`
/// (transformer.cpp:55-100).
int ForwardStack(const StackWeights& stack, const float* rope,
                 const AttentionLayout& layout, KvCache& cache, float* hidden,
                 float* output, int rows, StackScratch& scratch,
                 cudaStream_t stream);

class DeviceArena;
class ModelFiles;

/// A persistent kernel's bounded wait gave up and the launch aborted: its
/// outputs are not valid (the C ABI returns VX_DEVICE_TIMEOUT).
class DeviceTimeout : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

/// The LM caches of one GeneratorBatch slot: slot `slot` of slot-major caches
/// (KvCache with slots) that outlive the generator.
struct SlotCaches {
  const KvCache* base = nullptr;
  const KvCache* residual = nullptr;
  int slot = 0;
};

/// VoxCPM2's generator on one GPU (generator.hpp:58-179): one sequence at a
/// time on its own stream.
class Generator {
 public:
  /// Seeded weights when `files` is null, else the files' tensors (`seed`
  /// and `kind` unused; generator.cpp:82-174, weights.cpp:308-327).
  ///
  /// With `share`, the weights are `share`'s (same configuration; nothing is
  /// uploaded). With `stream`, the generator runs on that stream and does
  /// not own it; with `lm_caches`, its LM caches are views of those (the
  /// slots of a GeneratorBatch).
  static std::unique_ptr<Generator> Create(const ModelConfig& config,
                                           std::uint64_t seed,
                                           CheckpointKind kind,
                                           CacheType cache_type,
                                           std::string* error,
                                           const ModelFiles* files = nullptr,
                                           const Generator* share = nullptr,
                                           cudaStream_t stream = nullptr,
                                           const SlotCaches* lm_caches = nullptr);
  ~Generator();

  const ModelConfig& config() const { return config_; }
  cudaStream_t stream() const { return stream_; }
  int capacity() const { return config_.max_length; }
  int position() const { return position_; }
  std::size_t weight_bytes() const;

  /// generator.cpp:326-422 (host arrays; feats [rows][patch][feat]).
  void Prefill(const std::int32_t* tokens, const std::int32_t* text_mask,
               const std::int32_t* audio_mask, const float* feats, int rows);
  /// generator.cpp:424-513 (noise [patch][feat], host). Runs as one CUDA
  /// graph when graphs are enabled.
  void Step(const float* noise, int timesteps, float cfg, float* latent,
            float* stop_logits);
  /// generator.hpp:83-84: the last patch's latent [patch][feat] on the
  /// device, valid until the step after next (two slots alternate by
  /// position), ready once latent_event() completes; null before the first
  /// step of a sequence.
  const float* latent() const;
  cudaEvent_t latent_event() const { return latent_event_; }
  /// generator.cpp:515-538: one DiT evaluation's velocity pair.
  void Velocity(const float* mu, const float* cond, const float* x, float t,
                float* velocity);
  /// The DiT part of Step with the conditioning given (mu [2][dit hidden],
  /// prefix cond and noise [patch][feat]): dit_cond, then the Euler steps.
  void DitPatch(const float* mu, const float* cond, const float* noise,
                int timesteps, float cfg, float* latent);
  /// Replays the last captured DiT patch (inputs already on the device).
  void ReplayDitPatch();
  /// DitPatch from device arrays with the persistent kernel's work buffers
  /// in the library's static scratch; allocates nothing. Needs the
  /// persistent kernel and a schedule prepared by an earlier DitPatch or
  /// Step with the same `timesteps`. Synchronizes the generator's stream.
  void DitPatchStatic(const float* mu, const float* cond, const float* noise,
                      int timesteps, float cfg, float* latent);
  /// Downloads an internal state vector (tests).
  void State(const std::string& name, float* out, std::size_t count);
  /// Uploads an internal state vector (tests and benchmarks).
  void SetState(const std::string& name, const float* in, std::size_t count);
  void set_graphs(bool enabled) { graphs_ = enabled; }
  bool graphs() const { return graphs_; }
  /// Whether the DiT patch runs as the persistent kernel (default when the
  /// DiT has VoxCPM2's shape). Returns false when asked to enable it for a
  /// DiT of another shape.
  bool set_persistent(bool enabled);
  bool persistent() const { return persistent_; }
  /// Device buffers of the DiT patch's inputs and output (benchmarks).
  float* device_mu() const { return mu_; }
  float* device_prefix() const { return prefix_cond_; }
  float* device_x() const { return x_; }

 private:
  friend class GeneratorBatch;
  Generator() = default;
  void Check(int status, const char* what);
  /// Reads and clears the device error word and throws DeviceTimeout.
  [[noreturn]] void ThrowAborted(const char* what);
  /// StepBody's parts: the stop logits, mu and the DiT conditioning from
  /// the LM states, and the patch's noise into x (generator.cpp:424-447);
  /// the latent, stop logits and next prefix out (:465-476); both LMs
  /// advanced by the patch's embedding in embed_ (:478-513).
  void PreDit();
  void PatchOutputs();
  void AdvanceLms();
  void CheckCuda(cudaError_t error, const char* what);
  const float* TimeVector(float t);
  void EvaluateDit(const float* x, float t, float* velocity);
  void Encode(const float* latents, int patches, float* embeds);
  void EnsureEncoder(int patches);
  void Fsq(const float* input, float* output, int rows);
  void DitCond();
  void EulerLoop(int timesteps, float cfg);
  void StepBody(int timesteps, float cfg);
  void PrepareTimes(int timesteps);
  void EnsureRows(int rows);
  void DestroyGraphs();
  void SetupPersistent();
  void SetupPersistentLm();
  /// One of the two one-row stacks of a step (0: LM, 1: residual LM):
  /// the persistent kernel when enabled, else ForwardStack.
  void StepStack(int which, const AttentionLayout& layout, float* hidden,
                 float* output);

  ModelConfig config_;
  cudaStream_t stream_ = nullptr;
  std::shared_ptr<DeviceArena> arena_;  // the weights (shared by batch slots)
  std::unique_ptr<DeviceArena> work_;
  bool owns_stream_ = true;
  // Counts DestroyGraphs calls: every reallocation of a buffer that graphs
  // capture goes through it, so a GeneratorBatch re-captures when it moves.
  std::uint64_t buffers_epoch_ = 0;
  GeneratorWeights w_;
  float* rope_ = nullptr;
  KvCache base_cache_, residual_cache_, encoder_cache_, dit_cache_;
  StackScratch scratch_;
  int scratch_rows_ = 0;
  // Prefill work buffers, grown to the largest prompt seen (reused, so a
  // prefill allocates nothing once the block is large enough).
  unsigned char* prefill_block_ = nullptr;
  std::size_t prefill_bytes_ = 0;
  int position_ = 0;
  bool graphs_ = true;
  // Latents of the last two patches ([2][patch][feat], slot = position & 1)
  // and the event after the last step's launches.
  float* latent_slots_ = nullptr;
  cudaEvent_t latent_event_ = nullptr;
  bool latent_ready_ = false;

  // Sequence state.
  float* lm_hidden_ = nullptr;
  float* residual_hidden_ = nullptr;
  float* prefix_cond_ = nullptr;
  float* x_ = nullptr;
  float* velocity_ = nullptr;
  float* mu_ = nullptr;
  float* cond_rows_ = nullptr;
  float* stop_ = nullptr;
  float* delta_time_ = nullptr;
  float* embed_ = nullptr;
  std::int32_t* position_counter_ = nullptr;  // device: rows in the caches
  std::int32_t* step_positions_ = nullptr;    // device: [position]
  std::map<float, float*> time_vectors_;

  // Index arrays.
  std::int32_t* dit_positions_ = nullptr;
  std::int32_t* dit_rows_ = nullptr;
  std::int32_t* dit_outputs_ = nullptr;
  std::int32_t* local_positions_ = nullptr;
  std::int32_t* local_rows_ = nullptr;
  std::int32_t* local_firsts_ = nullptr;
  int local_capacity_ = 0;  // patches the encoder's buffers hold

  // Working buffers.
  std::uint16_t* step_bf16_ = nullptr;
  float* step_a_ = nullptr;
  float* step_b_ = nullptr;
  std::uint16_t* dit_bf16_ = nullptr;
  float* x_rows_ = nullptr;
  float* dit_hidden_ = nullptr;
  float* dit_output_ = nullptr;
  std::uint16_t* encoder_bf16_ = nullptr;
  float* encoder_a_ = nullptr;
  float* encoder_b_ = nullptr;
  float* encoder_c_ = nullptr;
  std::uint16_t* fsq_bf16_ = nullptr;
  float* fsq_latent_ = nullptr;

  // Pinned staging and graphs.
  float* pinned_noise_ = nullptr;
  float* pinned_latent_ = nullptr;
  float* pinned_stop_ = nullptr;
  cudaGraphExec_t step_graph_ = nullptr;
  int step_graph_timesteps_ = -1;
  float step_graph_cfg_ = 0.0f;
  cudaGraphExec_t patch_graph_ = nullptr;
  int patch_graph_timesteps_ = -1;
  float patch_graph_cfg_ = 0.0f;
  std::vector<float> schedule_t_, schedule_dt_;
  std::vector<int> schedule_eval_;

  // The persistent DiT patch.
  bool persistent_ok_ = false;
  bool persistent_ = false;
  DitPatchParams dit_params_;
  DitLayer* dit_layers_ = nullptr;
  void* dit_work_ = nullptr;
  unsigned char* dit_io_tiles_ = nullptr;  // bf16 rows of dit_in/out as tiles
  const float** dit_times_ = nullptr;      // device: time vector per evaluation
  float* dit_dts_ = nullptr;               // device: dt per evaluation
  int dit_schedule_capacity_ = 0;
  int dit_schedule_timesteps_ = -1;
  int dit_evaluations_ = 0;

  // The persistent one-row stacks (LM, residual LM).
  bool lm_persistent_ok_ = false;
  LmLayer* lm_layers_ = nullptr;  // [LM layers | residual layers]
  void* lm_work_ = nullptr;
  LmStackParams lm_params_[2];
};

/// Several requests generated together on one GPU: the loop of
/// synthesizer.cpp:283-307 over `slots` requests at once (no reference
/// counterpart; the reference serves one sequence per generator). The slots
/// are Generators that share one set of weights and one stream, each with its
/// own caches and states. A step runs, for the active slots:
/// - each slot's stop logits and DiT conditioning;
/// - one DiT pass of 22 rows per slot (two CFG sequences of 11 per slot,
///   attention block-diagonal per sequence) for every Euler evaluation, so
///   the DiT's weights are read once per evaluation for all of them;
/// - the local encoder over all their patches at once;
/// - each slot's LM and residual LM on its own caches.
/// A slot takes a new request through its Prefill while the others keep
/// their state. One CUDA graph per set of active slots (and timesteps, cfg).
class GeneratorBatch {
 public:
  static std::unique_ptr<GeneratorBatch> Create(const ModelConfig& config,
                                                std::uint64_t seed,
                                                CheckpointKind kind,
                                                CacheType cache_type,
                                                int slots, std::string* error,
                                                const ModelFiles* files = nullptr);
  ~GeneratorBatch();

  int slots() const { return static_cast<int>(slots_.size()); }
  Generator& slot(int index) { return *slots_.at(index); }
  cudaStream_t stream() const { return stream_; }
  void set_graphs(bool enabled) { graphs_enabled_ = enabled; }
  /// One patch for every slot with active[i] != 0: noise [slots][patch][feat]
  /// in; latents [slots][patch][feat] (may be null) and stop logits
  /// [slots][2] out for those slots. Synchronizes once.
  void Step(const std::int32_t* active, const float* noise, int timesteps,
            float cfg, float* latents, float* stop_logits);

 private:
  GeneratorBatch() = default;
  void Body(const std::vector<int>& members, int timesteps, float cfg);
  void EvaluateDit(int count, float t);
  void AdvanceLms(const std::vector<int>& members);
  void DestroyGraphs();

  // The slots' LM caches, slot-major (declared before the slots, released
  // after them).
  KvCache base_caches_;
  KvCache residual_caches_;
  std::vector<std::unique_ptr<Generator>> slots_;
  cudaStream_t stream_ = nullptr;
  KvCache dit_cache_;
  unsigned char* block_ = nullptr;
  float* mu_ = nullptr;        // [slots][2][dit hidden]
  float* cond_ = nullptr;      // [slots][patch][dit hidden]
  float* x_ = nullptr;         // [slots][patch][feat]
  float* velocity_ = nullptr;  // [slots][2][patch][feat]
  float* x_rows_ = nullptr;    // [slots][patch][dit hidden]
  float* hidden_ = nullptr;    // [slots * dit rows][dit hidden]
  float* output_ = nullptr;    // [slots * dit rows][dit hidden]
  std::uint16_t* bf16_ = nullptr;
  float* embed_ = nullptr;     // [slots][lm hidden]
  float* lm_a_ = nullptr;      // [slots][lm hidden] LM step rows
  float* lm_b_ = nullptr;
  float* lm_hidden_ = nullptr;       // [slots][lm hidden] after FSQ
  float* residual_hidden_ = nullptr; // [slots][lm hidden]
  float* fsq_ = nullptr;       // [slots][fsq latent]
  std::int32_t* past_ = nullptr;        // [slots] each active slot's position
  std::int32_t* cache_rows_ = nullptr;  // [slots] its cache row (slot-major)
  std::int32_t* first_keys_ = nullptr;  // [slots] its first key row
  std::int32_t* positions_ = nullptr;
  std::int32_t* rows_ = nullptr;
  std::int32_t* outputs_ = nullptr;
  bool graphs_enabled_ = true;
  std::map<std::tuple<std::uint64_t, int, float>, cudaGraphExec_t> graphs_;
  std::vector<std::uint64_t> epochs_;  // the slots' buffers_epoch_ at capture
};

/// The reference's released shapes (tests/config_test.cpp:36-67): LM 28 x
/// 2048 (FFN 6144), residual LM 8 x 2048 without RoPE, encoder and DiT
/// 12 x 1024 (FFN 4096), 16 query / 2 KV heads of 128, eps 1e-5, patch 4 x
/// 64, FSQ 512 at scale 9, 8192 positions. LongRoPE factors default to 1.
ModelConfig ReleasedConfig();

/// The FNV-1a hash of a tensor name: the tensor id of its seeded values.
std::uint64_t TensorId(const std::string& name);

}  // namespace vx
