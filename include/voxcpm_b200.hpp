// voxcpm_b200.hpp — header-only C++ mirror of the reference's interfaces
// over the C ABI (voxcpm_b200.h): the names, argument meanings and error
// behaviour of gemm.hpp, matrix.hpp, kernels/wmma_products.hpp,
// kernels/skinny_gemm.hpp, kernels/generator_kernels.hpp, transformer.hpp
// (RopeTable), generator.hpp (Prompt, EulerStep, EulerSchedule, Generator),
// model_files.hpp / safetensors.hpp (ModelFiles, Tensor) and config.hpp
// (ParseConfig), so that code written against the reference keeps
// compiling.
//
// Error behaviour: launchers that return bool in the reference return false
// when the shape does not suit the kernels (VX_UNSUPPORTED, nothing
// launched); every other failure throws GpuError (device.hpp:16-30). Link
// with -lvoxcpm_b200 (the shared library builds in voxcpm_b200/).
#ifndef VOXCPM_B200_HPP_
#define VOXCPM_B200_HPP_

#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "voxcpm_b200.h"

namespace voxcpm_b200 {

/// device.hpp:16-19
class GpuError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

inline void Check(vx_status status, const char* what) {
  if (status != VX_OK)
    throw GpuError(std::string(what) + ": " + vx_last_error());
}

/// false for VX_UNSUPPORTED, throws on other failures.
inline bool Launched(vx_status status, const char* what) {
  if (status == VX_UNSUPPORTED)
    return false;
  Check(status, what);
  return true;
}

using Bf16 = std::uint16_t;

/// matrix.hpp:9-19
enum class WeightFormat : std::uint8_t { kBf16 = 0, kBf16Tiles = 1, kQ8Tiles = 2 };
struct Matrix {
  WeightFormat format = WeightFormat::kBf16;
  const void* data = nullptr;
};

namespace kernels {

inline constexpr std::size_t kTileRows = 16;
inline constexpr std::size_t kTileColumns = 32;
inline constexpr std::size_t kQ8TileBytes = 16 * 32 + 16 * 2;
inline constexpr std::size_t kBf16TileBytes = 16 * 32 * 2;
inline constexpr std::size_t kSkinnyRows = 32;

inline std::size_t Q8TilesBytes(std::size_t rows, std::size_t in) {
  return vx_q8_tiles_bytes(rows, in);
}
inline std::size_t Bf16TilesBytes(std::size_t rows, std::size_t in) {
  return vx_bf16_tiles_bytes(rows, in);
}
inline void Q8_0ToTiles(const std::uint8_t* blocks, std::size_t rows,
                        std::size_t in, std::uint8_t* output,
                        cudaStream_t stream) {
  Check(vx_q8_0_to_tiles(blocks, rows, in, output, stream), "Q8_0ToTiles");
}
inline void Bf16ToTiles(const Bf16* weights, std::size_t rows, std::size_t in,
                        Bf16* output, cudaStream_t stream) {
  Check(vx_bf16_to_tiles(weights, rows, in, output, stream), "Bf16ToTiles");
}
inline void Q8TilesToBf16(const std::uint8_t* tiles, std::size_t rows,
                          std::size_t in, Bf16* output, cudaStream_t stream) {
  Check(vx_q8_tiles_to_bf16(tiles, rows, in, output, stream), "Q8TilesToBf16");
}
inline void Bf16TilesToRows(const Bf16* tiles, std::size_t rows,
                            std::size_t in, Bf16* output,
                            cudaStream_t stream) {
  Check(vx_bf16_tiles_to_rows(tiles, rows, in, output, stream),
        "Bf16TilesToRows");
}

/// kernels/wmma_products.hpp:62-81 (no scratch is needed: splits reduce on
/// chip, so partial_floats and counters stay 0).
struct SplitScratch {
  float* partials = nullptr;
  std::size_t partial_floats = 0;
  unsigned* counters = nullptr;
  std::size_t counter_count = 0;
};
using WmmaPlan = vx_wmma_plan;

inline WmmaPlan PlanWmma(std::size_t rows, std::size_t in, std::size_t out,
                         std::size_t target_waves = 0) {
  return vx_plan_wmma(rows, in, out, target_waves);
}
inline bool WmmaQ8(const Bf16* x, const std::uint8_t* w, float* y,
                   std::size_t rows, std::size_t in, std::size_t out,
                   bool accumulate, const WmmaPlan& plan,
                   const SplitScratch& scratch, cudaStream_t stream) {
  const vx_split_scratch s{scratch.partials, scratch.partial_floats,
                           scratch.counters, scratch.counter_count};
  return Launched(vx_wmma_q8(x, w, y, rows, in, out, accumulate ? 1 : 0, &plan,
                             &s, stream),
                  "WmmaQ8");
}
inline bool WmmaBf16(const Bf16* x, const Bf16* w, float* y, std::size_t rows,
                     std::size_t in, std::size_t out, bool accumulate,
                     const WmmaPlan& plan, const SplitScratch& scratch,
                     cudaStream_t stream) {
  const vx_split_scratch s{scratch.partials, scratch.partial_floats,
                           scratch.counters, scratch.counter_count};
  return Launched(vx_wmma_bf16(x, w, y, rows, in, out, accumulate ? 1 : 0,
                               &plan, &s, stream),
                  "WmmaBf16");
}
/// kernels/skinny_gemm.hpp:18-34
inline bool SkinnyGemm(const Bf16* x, const Bf16* w, float* y,
                       std::size_t rows, std::size_t in, std::size_t out,
                       bool accumulate, cudaStream_t stream) {
  return Launched(
      vx_skinny_gemm(x, w, y, rows, in, out, accumulate ? 1 : 0, stream),
      "SkinnyGemm");
}
inline bool SkinnyGemmWith(int vec, const Bf16* x, const Bf16* w, float* y,
                           std::size_t rows, std::size_t in, std::size_t out,
                           bool accumulate, cudaStream_t stream) {
  return Launched(vx_skinny_gemm_with(vec, x, w, y, rows, in, out,
                                      accumulate ? 1 : 0, stream),
                  "SkinnyGemmWith");
}
inline void ReadProbe(const Bf16* data, std::size_t pieces, unsigned blocks,
                      unsigned* sink, cudaStream_t stream) {
  Check(vx_read_probe(data, pieces, blocks, sink, stream), "ReadProbe");
}

/// kernels/generator_kernels.hpp:18-107 (fp32 KV caches, as the
/// reference's; the C ABI also takes bf16 caches).
inline void Embed(const Bf16* table, const std::int32_t* ids,
                  const std::int32_t* text_mask, float* output,
                  std::size_t rows, std::size_t width, float scale,
                  cudaStream_t stream) {
  Check(vx_embed(table, ids, text_mask, output, rows, width, scale, stream),
        "Embed");
}
inline void ScatterRows(const float* input, const std::int32_t* indices,
                        float* output, std::size_t rows, std::size_t width,
                        cudaStream_t stream) {
  Check(vx_scatter_rows(input, indices, output, rows, width, stream),
        "ScatterRows");
}
inline void GatherRows(const float* input, const std::int32_t* indices,
                       float* output, std::size_t rows, std::size_t width,
                       cudaStream_t stream) {
  Check(vx_gather_rows(input, indices, output, rows, width, stream),
        "GatherRows");
}
inline void RmsNorm(const float* input, const Bf16* weight, Bf16* output,
                    float* output_f32, std::size_t rows, std::size_t width,
                    float epsilon, cudaStream_t stream) {
  Check(vx_rms_norm(input, weight, output, output_f32, rows, width, epsilon,
                    stream),
        "RmsNorm");
}
inline void QkvRope(const float* qkv, const float* cos_sin,
                    const std::int32_t* positions,
                    const std::int32_t* cache_rows, float* q, float* k_cache,
                    float* v_cache, std::size_t rows, std::size_t heads,
                    std::size_t kv_heads, std::size_t head_dim,
                    std::size_t capacity, cudaStream_t stream) {
  Check(vx_qkv_rope(qkv, cos_sin, positions, cache_rows, q, k_cache, v_cache,
                    VX_CACHE_F32, rows, heads, kv_heads, head_dim, capacity,
                    stream),
        "QkvRope");
}
inline void Attention(const float* q, const float* k_cache,
                      const float* v_cache, Bf16* output, std::size_t rows,
                      std::size_t rows_per_sequence,
                      std::size_t keys_per_sequence, std::size_t past,
                      bool causal, std::size_t heads, std::size_t kv_heads,
                      std::size_t head_dim, std::size_t capacity,
                      cudaStream_t stream) {
  Check(vx_attention(q, k_cache, v_cache, VX_CACHE_F32, output, rows,
                     rows_per_sequence, keys_per_sequence, past, nullptr,
                     causal ? 1 : 0, heads, kv_heads, head_dim, capacity, 0,
                     stream),
        "Attention");
}
inline void SwiGlu(const float* gate_up, Bf16* output, std::size_t rows,
                   std::size_t width, cudaStream_t stream) {
  Check(vx_swiglu(gate_up, output, rows, width, stream), "SwiGlu");
}
inline void AddBias(float* data, const Bf16* bias, std::size_t rows,
                    std::size_t width, cudaStream_t stream) {
  Check(vx_add_bias(data, bias, rows, width, stream), "AddBias");
}
inline void ToBf16(const float* input, Bf16* output, std::size_t count,
                   bool silu, cudaStream_t stream) {
  Check(vx_to_bf16(input, output, count, silu ? 1 : 0, stream), "ToBf16");
}
inline void ConcatRows(const float* a, const float* a_scale,
                       std::size_t a_width, const float* b,
                       const float* b_scale, std::size_t b_width, Bf16* output,
                       std::size_t rows, cudaStream_t stream) {
  Check(vx_concat_rows(a, a_scale, a_width, b, b_scale, b_width, output, rows,
                       stream),
        "ConcatRows");
}
inline void Quantize(const float* input, Bf16* output, std::size_t count,
                     float scale, cudaStream_t stream) {
  Check(vx_quantize(input, output, count, scale, stream), "Quantize");
}
inline void SelectRows(const float* quantized, const float* plain,
                       const std::int32_t* mask, float* output,
                       std::size_t rows, std::size_t width,
                       cudaStream_t stream) {
  Check(vx_select_rows(quantized, plain, mask, output, rows, width, stream),
        "SelectRows");
}
inline void PrependSpecial(const float* rows_in, const Bf16* special,
                           float* output, std::size_t patches,
                           std::size_t patch_size, std::size_t width,
                           cudaStream_t stream) {
  Check(vx_prepend_special(rows_in, special, output, patches, patch_size,
                           width, stream),
        "PrependSpecial");
}
inline void AssembleDit(const float* mu, const float* time, const float* cond,
                        const float* x, float* output, std::size_t patch_size,
                        std::size_t width, cudaStream_t stream) {
  Check(vx_assemble_dit(mu, time, cond, x, output, patch_size, width, stream),
        "AssembleDit");
}
inline void GuidedEuler(const float* velocity, float* x, std::size_t count,
                        float cfg, float dt, cudaStream_t stream) {
  Check(vx_guided_euler(velocity, x, count, cfg, dt, stream), "GuidedEuler");
}

}  // namespace kernels

/// gemm.hpp:16-38: a column-major (BLAS) product C[m][n] (+)= op(A)[m][k] *
/// op(B)[k][n], optionally strided-batched.
struct MatmulShape {
  bool transpose_a = false;
  bool transpose_b = false;
  std::size_t m = 0;
  std::size_t n = 0;
  std::size_t k = 0;
  std::size_t lda = 0;
  std::size_t ldb = 0;
  std::size_t ldc = 0;
  std::int64_t stride_a = 0;
  std::int64_t stride_b = 0;
  std::int64_t stride_c = 0;
  std::size_t batch = 1;
  bool accumulate = false;

  [[nodiscard]] vx_matmul_shape ToC() const {
    return vx_matmul_shape{transpose_a ? 1 : 0, transpose_b ? 1 : 0, m, n, k,
                           lda, ldb, ldc, stride_a, stride_b, stride_c, batch,
                           accumulate ? 1 : 0};
  }
};

/// gemm.hpp:74-77
[[nodiscard]] constexpr std::size_t TuningBucket(std::size_t size) {
  return (size + 127) / 128 * 128;
}

/// gemm.hpp:49-72. The reference's constructor also takes a hipBLAS handle
/// for its library fallback; these products need none.
class Bf16Gemm {
 public:
  explicit Bf16Gemm(cudaStream_t stream) : gemm_(vx_gemm_create(stream)) {
    if (gemm_ == nullptr)
      throw GpuError("vx_gemm_create failed");
  }
  ~Bf16Gemm() { vx_gemm_destroy(gemm_); }
  Bf16Gemm(const Bf16Gemm&) = delete;
  Bf16Gemm& operator=(const Bf16Gemm&) = delete;

  void Linear(const void* x, const Matrix& w, float* y, std::size_t rows,
              std::size_t in, std::size_t out, bool accumulate) {
    Check(vx_gemm_linear(gemm_, static_cast<const std::uint16_t*>(x),
                         static_cast<int>(w.format), w.data, y, rows, in, out,
                         accumulate ? 1 : 0),
          "Bf16Gemm::Linear");
  }

  /// gemm.hpp:60-63: bf16 a and b, float32 c. One kernel serves every
  /// shape, so `representative` is not used for tuning.
  void Matmul(const MatmulShape& shape, const MatmulShape& representative,
              const void* a, const void* b, float* c) {
    const vx_matmul_shape s = shape.ToC();
    const vx_matmul_shape r = representative.ToC();
    Check(vx_gemm_matmul(gemm_, &s, &r, static_cast<const std::uint16_t*>(a),
                         static_cast<const std::uint16_t*>(b), c),
          "Bf16Gemm::Matmul");
  }

 private:
  vx_gemm* gemm_;
};

/// transformer.hpp:17-36: keys and values of one stack, zeroed.
class KvCache {
 public:
  KvCache(const vx_stack_config& config, std::size_t capacity,
          int cache_type = VX_CACHE_F32)
      : cache_(vx_kv_cache_create(&config, capacity, cache_type)) {
    if (cache_ == nullptr)
      throw GpuError(std::string("KvCache: ") + vx_last_error());
  }
  ~KvCache() { vx_kv_cache_destroy(cache_); }
  KvCache(const KvCache&) = delete;
  KvCache& operator=(const KvCache&) = delete;

  std::size_t capacity() const { return vx_kv_cache_capacity(cache_); }
  void* keys(std::size_t layer) const { return vx_kv_cache_keys(cache_, layer); }
  void* values(std::size_t layer) const {
    return vx_kv_cache_values(cache_, layer);
  }
  vx_kv_cache* get() const { return cache_; }

 private:
  vx_kv_cache* cache_;
};

/// transformer.hpp:68-71. The products run on the library's own kernels, so
/// no Bf16Gemm is passed.
inline void ForwardStack(const vx_stack_weights& stack, const float* rope,
                         const vx_attention_layout& layout, KvCache& cache,
                         float* hidden, float* output, std::size_t rows,
                         const vx_stack_scratch& scratch,
                         cudaStream_t stream) {
  Check(vx_forward_stack(&stack, rope, &layout, cache.get(), hidden, output,
                         rows, &scratch, stream),
        "ForwardStack");
}

/// transformer.hpp:73-76
inline void Project(const vx_projection& projection, const Bf16* x, float* y,
                    std::size_t rows, cudaStream_t stream) {
  Check(vx_project(&projection, x, y, rows, stream), "Project");
}

/// transformer.hpp:63-66 (factors per frequency; the reference derives them
/// from its RopeConfig).
inline std::vector<float> RopeTable(double theta, std::size_t dim,
                                    const std::vector<double>& factors,
                                    double scaling, std::size_t positions) {
  std::vector<float> table(positions * dim);
  Check(vx_rope_table(theta, dim, factors.data(), scaling, positions,
                      table.data()),
        "RopeTable");
  return table;
}

/// generator.hpp:24-44
struct Prompt {
  std::vector<std::int32_t> tokens;
  std::vector<std::int32_t> text_mask;
  std::vector<std::int32_t> audio_mask;
  std::vector<float> feats;  // [rows][patch_size][feat_dim]
};

struct EulerStep {
  float t = 0.0f;
  float dt = 0.0f;
  bool evaluate = true;
};

inline std::vector<EulerStep> EulerSchedule(std::size_t timesteps,
                                            float sway = 1.0f) {
  std::vector<float> t(timesteps), dt(timesteps);
  std::vector<std::int32_t> evaluate(timesteps);
  const std::size_t n = vx_euler_schedule(timesteps, sway, t.data(), dt.data(),
                                          evaluate.data(), timesteps);
  std::vector<EulerStep> steps;
  for (std::size_t i = 0; i < n && i < timesteps; ++i)
    steps.push_back({t[i], dt[i], evaluate[i] != 0});
  return steps;
}

/// safetensors.hpp:18-34: one tensor of the checkpoint files; `data` is
/// host memory in the mapped file, valid while the files are open.
enum class DType : int { kF32 = 0, kBF16, kF16, kI64, kI32, kU8, kQ8_0 };

struct Tensor {
  std::string name;
  DType dtype = DType::kF32;
  std::vector<std::size_t> shape;
  const std::byte* data = nullptr;
  std::size_t bytes = 0;
  std::uint64_t offset = 0;

  std::size_t Elements() const {
    std::size_t n = 1;
    for (const std::size_t d : shape)
      n *= d;
    return n;
  }
};

/// model_files.hpp:45-83: a Hugging Face directory or an audio.cpp VoxCPM2
/// GGUF file.
class ModelFiles {
 public:
  static std::unique_ptr<ModelFiles> Open(const std::string& path,
                                          std::string* error = nullptr) {
    vx_model_files* f = vx_model_files_open(path.c_str());
    if (f == nullptr) {
      if (error != nullptr)
        *error = vx_last_error();
      return nullptr;
    }
    return std::unique_ptr<ModelFiles>(new ModelFiles(f));
  }
  static bool IsVoxCpm2Gguf(const std::string& path) {
    return vx_model_files_is_voxcpm2_gguf(path.c_str()) != 0;
  }
  ~ModelFiles() { vx_model_files_close(f_); }
  ModelFiles(const ModelFiles&) = delete;
  ModelFiles& operator=(const ModelFiles&) = delete;

  std::string config() const { return vx_model_files_config(f_); }
  std::string tokenizer() const { return vx_model_files_tokenizer(f_); }
  bool gguf() const { return vx_model_files_is_gguf(f_) != 0; }
  const Tensor* Model(const std::string& name) const { return Find(model_, name); }
  const Tensor* Vae(const std::string& name) const { return Find(vae_, name); }
  const std::vector<Tensor>& model_tensors() const { return model_; }
  const vx_model_files* handle() const { return f_; }

 private:
  explicit ModelFiles(vx_model_files* f) : f_(f) {
    for (int component : {VX_COMPONENT_MODEL, VX_COMPONENT_VAE}) {
      std::vector<Tensor>& out = component == VX_COMPONENT_MODEL ? model_ : vae_;
      const std::size_t count = vx_model_files_count(f_, component);
      for (std::size_t i = 0; i < count; ++i) {
        vx_tensor_info info;
        Check(vx_model_files_tensor(f_, component, i, &info), "ModelFiles");
        Tensor t;
        t.name = info.name;
        t.dtype = static_cast<DType>(info.dtype);
        t.shape.assign(info.shape, info.shape + info.rank);
        t.data = static_cast<const std::byte*>(info.data);
        t.bytes = static_cast<std::size_t>(info.bytes);
        t.offset = info.offset;
        out.push_back(std::move(t));
      }
    }
  }
  static const Tensor* Find(const std::vector<Tensor>& tensors,
                            const std::string& name) {
    for (const Tensor& t : tensors)
      if (t.name == name)
        return &t;
    return nullptr;
  }
  vx_model_files* f_;
  std::vector<Tensor> model_;
  std::vector<Tensor> vae_;
};

/// config.hpp:92-98: config.json text -> the generator's configuration,
/// false (and `error`) for a malformed or unsupported one (ParseConfig and
/// IsSupported in one).
inline bool ParseConfig(const std::string& text, vx_model_config* config,
                        std::string* error = nullptr) {
  if (vx_parse_config(text.data(), text.size(), config) != VX_OK) {
    if (error != nullptr)
      *error = vx_last_error();
    return false;
  }
  return true;
}

/// generator.hpp:58-179: weights from checkpoint files (Create with
/// ModelFiles) or seeded (Create with a seed, for benchmarks and tests).
class Generator {
 public:
  static std::unique_ptr<Generator> Create(const vx_model_config& config,
                                           std::uint64_t seed, int checkpoint,
                                           int cache_type,
                                           std::string* error = nullptr) {
    vx_generator* g = vx_generator_create(&config, seed, checkpoint, cache_type);
    if (g == nullptr) {
      if (error != nullptr)
        *error = vx_last_error();
      return nullptr;
    }
    return std::unique_ptr<Generator>(new Generator(g, config));
  }
  static std::unique_ptr<Generator> Create(const vx_model_config& config,
                                           const ModelFiles& files,
                                           std::string* error = nullptr,
                                           int cache_type = VX_CACHE_F32) {
    vx_generator* g =
        vx_generator_create_from_files(&config, files.handle(), cache_type);
    if (g == nullptr) {
      if (error != nullptr)
        *error = vx_last_error();
      return nullptr;
    }
    return std::unique_ptr<Generator>(new Generator(g, config));
  }
  ~Generator() { vx_generator_destroy(g_); }
  Generator(const Generator&) = delete;
  Generator& operator=(const Generator&) = delete;

  std::size_t capacity() const { return static_cast<std::size_t>(config_.max_length); }
  std::size_t position() const { return vx_generator_position(g_); }
  /// generator.hpp:83-84
  const float* latent() const { return vx_generator_latent(g_); }
  cudaEvent_t latent_event() const { return vx_generator_latent_event(g_); }

  void Prefill(const Prompt& prompt) {
    Check(vx_generator_prefill(g_, prompt.tokens.data(),
                               prompt.text_mask.data(),
                               prompt.audio_mask.data(), prompt.feats.data(),
                               prompt.tokens.size()),
          "Generator::Prefill");
  }
  void Step(const float* noise, std::size_t timesteps, float cfg,
            float* latent, float* stop_logits) {
    Check(vx_generator_step(g_, noise, timesteps, cfg, latent, stop_logits),
          "Generator::Step");
  }
  void Velocity(const float* mu, const float* cond, const float* x, float t,
                float* velocity) {
    Check(vx_generator_velocity(g_, mu, cond, x, t, velocity),
          "Generator::Velocity");
  }

 private:
  Generator(vx_generator* g, const vx_model_config& config)
      : g_(g), config_(config) {}
  vx_generator* g_;
  vx_model_config config_;
};

/// vae.hpp:25-79, decoding: the AudioVAE V2 decoder on its own stream, with
/// the seeded AudioVAE checkpoint of `seed` (no audiovae.pth reader).
class AudioVae {
 public:
  static std::unique_ptr<AudioVae> Create(const vx_vae_config& config,
                                          std::uint64_t seed,
                                          std::string* error = nullptr) {
    vx_audio_vae* v = vx_audio_vae_create(&config, seed);
    if (v == nullptr) {
      if (error != nullptr)
        *error = vx_last_error();
      return nullptr;
    }
    return std::unique_ptr<AudioVae>(new AudioVae(v, config));
  }
  ~AudioVae() { vx_audio_vae_destroy(v_); }
  AudioVae(const AudioVae&) = delete;
  AudioVae& operator=(const AudioVae&) = delete;

  /// vae.hpp:39-52
  void Reset() { Check(vx_audio_vae_reset(v_), "AudioVae::Reset"); }
  void Decode(const float* latents, std::size_t frames,
              std::vector<float>* audio) {
    const std::size_t at = audio->size();
    audio->resize(at + frames * decode_hop());
    Check(vx_audio_vae_decode(v_, latents, frames, audio->data() + at),
          "AudioVae::Decode");
  }
  void Enqueue(const float* latents, std::size_t frames, cudaEvent_t ready) {
    Check(vx_audio_vae_enqueue(v_, latents, frames, ready),
          "AudioVae::Enqueue");
    pending_ = frames * decode_hop();
  }
  void Collect(std::vector<float>* audio) {
    const std::size_t at = audio->size();
    audio->resize(at + pending_);
    std::size_t samples = 0;
    Check(vx_audio_vae_collect(v_, audio->data() + at, pending_, &samples),
          "AudioVae::Collect");
    audio->resize(at + samples);
    pending_ = 0;
  }
  std::size_t output_rate() const { return config_.out_sample_rate; }
  std::size_t decode_hop() const { return vx_audio_vae_decode_hop(v_); }
  cudaStream_t stream() const { return vx_audio_vae_stream(v_); }

 private:
  AudioVae(vx_audio_vae* v, const vx_vae_config& config)
      : v_(v), config_(config) {}
  vx_audio_vae* v_;
  vx_vae_config config_;
  std::size_t pending_ = 0;
};

}  // namespace voxcpm_b200

#endif  // VOXCPM_B200_HPP_
