// The generator's model layer (see model.cuh): seeded device weights,
// KV caches, ForwardStack, Project and the per-patch Generator.
//
// Control flow follows the reference (transformer.cpp:47-100,
// generator.cpp:82-538) with B200-first changes:
// - the per-step host synchronizations are gone: the time vectors of the
//   Euler schedule are computed before the loop, the decode position lives
//   on the device (QkvRope reads it, Attention reads `past` from it and a
//   kernel advances it), so a whole Step (and a DiT patch) is captured once
//   as a CUDA graph and replayed per patch;
// - every kernel is launched with programmatic dependent launch, so the
//   products' weight streams start while the previous kernel drains.
#include "model.cuh"
#include "convert.cuh"
#include "model_files.h"
#include "vx_common.cuh"
#include "vx_status.h"

#include "../../include/voxcpm_b200.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <stdexcept>

namespace vx {

// ------------------------------------------------------------ arena

/// One device allocation handed out in 256-byte aligned pieces; a null
/// base only counts bytes.
class DeviceArena {
 public:
  DeviceArena() = default;
  explicit DeviceArena(std::size_t bytes) {
    if (bytes > 0 &&
        cudaMalloc(reinterpret_cast<void**>(&base_), bytes) != cudaSuccess)
      throw std::runtime_error("cudaMalloc of " + std::to_string(bytes) +
                               " bytes failed");
    capacity_ = bytes;
  }
  ~DeviceArena() {
    if (base_ != nullptr)
      cudaFree(base_);
  }
  DeviceArena(const DeviceArena&) = delete;
  DeviceArena& operator=(const DeviceArena&) = delete;

  void* Take(std::size_t bytes) {
    used_ = (used_ + 255) / 256 * 256;
    void* p = nullptr;
    if (base_ != nullptr) {
      if (used_ + bytes > capacity_)
        throw std::runtime_error("device arena exhausted");
      p = base_ + used_;
    }
    used_ += bytes;
    return p;
  }
  template <typename T>
  T* Take(std::size_t count) {
    return static_cast<T*>(Take(count * sizeof(T)));
  }
  std::size_t used() const { return used_; }

 private:
  unsigned char* base_ = nullptr;
  std::size_t capacity_ = 0;
  std::size_t used_ = 0;
};

namespace {

void ThrowCuda(cudaError_t error, const std::string& what) {
  if (error != cudaSuccess)
    throw std::runtime_error(what + ": " + cudaGetErrorString(error));
}

void ThrowStatus(int status, const std::string& what) {
  if (status == kOk)
    return;
  const cudaError_t error = cudaGetLastError();
  throw std::runtime_error(what + ": status " + std::to_string(status) +
                           (error != cudaSuccess
                                ? std::string(" (") + cudaGetErrorString(error) +
                                      ")"
                                : std::string()));
}

// ------------------------------------------------------------ seeded upload

constexpr float kQ8ScaleStd = 0.02f / 127.0f;  // |N(0, 0.02)| / 127
constexpr float kMatrixStd = 0.02f;

/// Takes every tensor of the generator in the reference's order
/// (weights.cpp:268-304), from a seeded checkpoint or from checkpoint files;
/// without an arena it only counts bytes.
///
/// Files follow the reference's format rule (weights.cpp:47-144): a matrix
/// of Q8_0 blocks becomes Q8 tiles; other matrices become bf16 tiles in the
/// DiT stack and bf16 rows elsewhere; fused parts (qkv, gate_up) keep tiles
/// only when every part is Q8_0 (for Q8 tiles) and fills whole 16-row tiles;
/// a reduction that is not a multiple of 32 keeps bf16 rows. Vectors and the
/// embedding table become bf16. F16, F32 and Q8_0 sources are converted on
/// the device after the raw bytes are copied in.
class Uploader {
 public:
  Uploader(std::uint64_t seed, CheckpointKind kind, const ModelFiles* files,
           DeviceArena* arena, cudaStream_t stream)
      : seed_(seed), kind_(kind), files_(files), arena_(arena),
        stream_(stream) {}
  ~Uploader() {
    cudaStreamSynchronize(stream_);
    if (pinned_ != nullptr)
      cudaFreeHost(pinned_);
    for (int i = 0; i < 2; ++i) {
      if (bounce_[i] != nullptr)
        cudaFreeHost(bounce_[i]);
      if (bounce_done_[i] != nullptr)
        cudaEventDestroy(bounce_done_[i]);
    }
    if (staging_ != nullptr)
      cudaFree(staging_);
    if (rows_ != nullptr)
      cudaFree(rows_);
  }

  /// A vector (or the embedding table) as bf16; seeded values are
  /// bf16(mean + N(0, std)).
  const std::uint16_t* Vector(const std::string& name,
                              std::initializer_list<std::size_t> shape,
                              float mean, float std) {
    std::size_t count = 1;
    for (const std::size_t d : shape)
      count *= d;
    const Tensor* tensor = files_ != nullptr ? &Find(name, shape) : nullptr;
    auto* target = arena_->Take<std::uint16_t>(count);
    if (target == nullptr)
      return nullptr;
    if (tensor != nullptr) {
      ToBf16(*tensor, target);
    } else {
      auto* host = static_cast<std::uint16_t*>(Pinned(count * 2));
      ThrowStatus(vx_random_bf16(seed_, TensorId(name), count, mean, std, host),
                  "seeded " + name);
      ThrowCuda(cudaMemcpyAsync(target, host, count * 2,
                                cudaMemcpyHostToDevice, stream_),
                "upload " + name);
    }
    ThrowCuda(cudaStreamSynchronize(stream_), "upload " + name);
    return target;
  }

  /// `names` ([outs[i]][in] each) side by side as one matrix. A seeded
  /// checkpoint uses Q8 tiles for kQ8, bf16 tiles for the DiT of kBf16 and
  /// bf16 rows otherwise. `fused` applies the whole-tile rule of fused
  /// matrices to files (weights.cpp:57-86); single matrices follow
  /// TakeMatrix (:44-54).
  Projection Fused(const std::vector<std::string>& names,
                   const std::vector<int>& outs, int in, bool dit,
                   bool fused = true) {
    Projection p;
    std::vector<const Tensor*> tensors;
    if (files_ != nullptr) {
      bool q8 = true;
      bool whole = true;
      for (std::size_t i = 0; i < names.size(); ++i) {
        tensors.push_back(&Find(names[i], {static_cast<std::size_t>(outs[i]),
                                           static_cast<std::size_t>(in)}));
        q8 = q8 && tensors.back()->dtype == DType::kQ8_0;
        whole = whole && (!fused || outs[i] % 16 == 0);
      }
      p.format = in % 32 != 0 ? WeightFormat::kBf16
                 : q8 && whole ? WeightFormat::kQ8Tiles
                 : dit && whole ? WeightFormat::kBf16Tiles
                                : WeightFormat::kBf16;
    } else {
      p.format = kind_ == CheckpointKind::kQ8
                     ? WeightFormat::kQ8Tiles
                     : (dit ? WeightFormat::kBf16Tiles : WeightFormat::kBf16);
    }
    p.in = in;
    p.out = std::accumulate(outs.begin(), outs.end(), 0);
    std::size_t total = 0;
    for (const int out : outs)
      total += Bytes(p.format, out, in);
    auto* target = static_cast<unsigned char*>(arena_->Take(total));
    p.weight = target;
    if (target == nullptr)
      return p;
    for (std::size_t i = 0; i < names.size(); ++i) {
      if (files_ != nullptr)
        WriteFile(*tensors[i], p.format, outs[i], in, target);
      else
        Write(names[i], p.format, outs[i], in, target);
      ThrowCuda(cudaStreamSynchronize(stream_), "upload " + names[i]);
      target += Bytes(p.format, outs[i], in);
    }
    return p;
  }

  Projection Linear(const std::string& prefix, int in, int out, bool bias,
                    bool dit = false) {
    Projection p = Fused({prefix + ".weight"}, {out}, in, dit, false);
    if (bias)
      p.bias = Vector(prefix + ".bias", {static_cast<std::size_t>(out)}, 0.0f,
                      kMatrixStd);
    return p;
  }

  StackWeights Stack(const std::string& prefix, const StackConfig& config,
                     bool dit) {
    StackWeights stack;
    stack.config = config;
    const int hidden = config.hidden;
    const std::size_t h = static_cast<std::size_t>(hidden);
    const int q = config.heads * config.head_dim;
    const int kv = config.kv_heads * config.head_dim;
    for (int index = 0; index < config.layers; ++index) {
      const std::string layer = prefix + ".layers." + std::to_string(index);
      LayerWeights w;
      w.input_norm = Vector(layer + ".input_layernorm.weight", {h}, 1.0f, 0.05f);
      const std::string attn = layer + ".self_attn.";
      w.qkv = Fused({attn + "q_proj.weight", attn + "k_proj.weight",
                     attn + "v_proj.weight"},
                    {q, kv, kv}, hidden, dit);
      w.o = Linear(attn + "o_proj", q, hidden, false, dit);
      w.post_norm =
          Vector(layer + ".post_attention_layernorm.weight", {h}, 1.0f, 0.05f);
      w.gate_up = Fused(
          {layer + ".mlp.gate_proj.weight", layer + ".mlp.up_proj.weight"},
          {config.intermediate, config.intermediate}, hidden, dit);
      w.down = Linear(layer + ".mlp.down_proj", config.intermediate, hidden,
                      false, dit);
      stack.layers.push_back(w);
    }
    stack.norm = Vector(prefix + ".norm.weight", {h}, 1.0f, 0.05f);
    return stack;
  }

  /// Tensors taken from the files so far.
  std::size_t taken() const { return taken_; }

 private:
  static std::size_t Bytes(WeightFormat format, int out, int in) {
    switch (format) {
      case WeightFormat::kQ8Tiles:
        return Q8TilesBytes(out, in);
      case WeightFormat::kBf16Tiles:
        return Bf16TilesBytes(out, in);
      case WeightFormat::kBf16:
        break;
    }
    return static_cast<std::size_t>(out) * in * 2;
  }

  /// The named tensor of the files with the expected shape
  /// (weights.cpp:187-197).
  const Tensor& Find(const std::string& name,
                     std::initializer_list<std::size_t> shape) {
    const Tensor* tensor = files_->Model(name);
    if (tensor == nullptr)
      throw std::runtime_error("the checkpoint lacks " + name);
    if (!std::equal(tensor->shape.begin(), tensor->shape.end(), shape.begin(),
                    shape.end()))
      throw std::runtime_error(name + " has an unexpected shape");
    ++taken_;
    return *tensor;
  }

  void* Pinned(std::size_t bytes) {
    if (bytes > pinned_bytes_) {
      if (pinned_ != nullptr) {
        ThrowCuda(cudaStreamSynchronize(stream_), "upload");
        cudaFreeHost(pinned_);
        pinned_ = nullptr;
      }
      ThrowCuda(cudaMallocHost(&pinned_, bytes), "cudaMallocHost");
      pinned_bytes_ = bytes;
    }
    return pinned_;
  }

  static void* Grow(void*& buffer, std::size_t& size, std::size_t bytes,
                    cudaStream_t stream) {
    if (bytes > size) {
      if (buffer != nullptr) {
        ThrowCuda(cudaStreamSynchronize(stream), "upload");
        cudaFree(buffer);
        buffer = nullptr;
      }
      ThrowCuda(cudaMalloc(&buffer, bytes), "cudaMalloc staging");
      size = bytes;
    }
    return buffer;
  }
  void* Staging(std::size_t bytes) {
    return Grow(staging_, staging_bytes_, bytes, stream_);
  }
  void* Rows(std::size_t bytes) {
    return Grow(rows_, rows_bytes_, bytes, stream_);
  }

  /// Copies `bytes` of (pageable, possibly mapped) host memory to the device
  /// through two pinned bounce buffers: the memcpy into one overlaps the DMA
  /// out of the other.
  void CopyIn(const void* host, std::size_t bytes, void* device) {
    constexpr std::size_t kChunk = 32u << 20;
    const auto* from = static_cast<const unsigned char*>(host);
    auto* to = static_cast<unsigned char*>(device);
    for (std::size_t done = 0, chunk = 0; done < bytes; done += kChunk, ++chunk) {
      const int b = static_cast<int>(chunk % 2);
      if (bounce_[b] == nullptr) {
        ThrowCuda(cudaMallocHost(&bounce_[b], kChunk), "cudaMallocHost");
        ThrowCuda(cudaEventCreateWithFlags(&bounce_done_[b],
                                           cudaEventDisableTiming),
                  "cudaEventCreate");
      } else {
        ThrowCuda(cudaEventSynchronize(bounce_done_[b]), "upload");
      }
      const std::size_t n = std::min(kChunk, bytes - done);
      std::memcpy(bounce_[b], from + done, n);
      ThrowCuda(cudaMemcpyAsync(to + done, bounce_[b], n,
                                cudaMemcpyHostToDevice, stream_),
                "upload");
      ThrowCuda(cudaEventRecord(bounce_done_[b], stream_), "upload");
    }
  }

  static void CheckQ8(const Tensor& tensor) {
    const std::size_t elements = tensor.Elements();
    if (elements % 32 != 0 || tensor.bytes != elements / 32 * 34)
      throw std::runtime_error(tensor.name + " is not whole Q8_0 blocks");
  }

  /// bf16 of a file tensor at `target` (weights.cpp:215-246).
  void ToBf16(const Tensor& tensor, std::uint16_t* target) {
    const std::size_t elements = tensor.Elements();
    switch (tensor.dtype) {
      case DType::kBF16:
        CopyIn(tensor.data, tensor.bytes, target);
        return;
      case DType::kF16:
      case DType::kF32:
      case DType::kQ8_0: {
        if (tensor.dtype == DType::kQ8_0)
          CheckQ8(tensor);
        void* raw = Staging(tensor.bytes);
        CopyIn(tensor.data, tensor.bytes, raw);
        int status = kOk;
        if (tensor.dtype == DType::kF16)
          status = HalfToBf16(static_cast<const std::uint16_t*>(raw), target,
                              elements, stream_);
        else if (tensor.dtype == DType::kF32)
          status = FloatToBf16(static_cast<const float*>(raw), target,
                               elements, stream_);
        else
          status = Q8_0ToBf16(static_cast<const std::uint8_t*>(raw), target,
                              elements, stream_);
        ThrowStatus(status, "convert " + tensor.name);
        return;
      }
      default:
        throw std::runtime_error(tensor.name + " has an unsupported type " +
                                 DTypeName(tensor.dtype));
    }
  }

  /// A file tensor [out][in] in `format` at `target` (weights.cpp:159-185).
  void WriteFile(const Tensor& tensor, WeightFormat format, int out, int in,
                 unsigned char* target) {
    switch (format) {
      case WeightFormat::kBf16:
        ToBf16(tensor, reinterpret_cast<std::uint16_t*>(target));
        return;
      case WeightFormat::kBf16Tiles: {
        auto* rows = static_cast<std::uint16_t*>(
            Rows(static_cast<std::size_t>(out) * in * 2));
        ToBf16(tensor, rows);
        ThrowStatus(Bf16ToTiles(rows, out, in,
                                reinterpret_cast<std::uint16_t*>(target),
                                stream_),
                    "tiles " + tensor.name);
        return;
      }
      case WeightFormat::kQ8Tiles: {
        CheckQ8(tensor);
        void* raw = Staging(tensor.bytes);
        CopyIn(tensor.data, tensor.bytes, raw);
        ThrowStatus(Q8_0ToTiles(static_cast<const std::uint8_t*>(raw), out, in,
                                target, stream_),
                    "tiles " + tensor.name);
        return;
      }
    }
  }

  void Write(const std::string& name, WeightFormat format, int out, int in,
             unsigned char* target) {
    const std::uint64_t id = TensorId(name);
    if (format == WeightFormat::kQ8Tiles) {
      const std::size_t bytes = static_cast<std::size_t>(out) * (in / 32) * 34;
      auto* host = static_cast<std::uint8_t*>(Pinned(bytes));
      ThrowStatus(vx_random_q8_0(seed_, id, out, in, kQ8ScaleStd, host),
                  "seeded " + name);
      void* stage = Staging(bytes);
      ThrowCuda(cudaMemcpyAsync(stage, host, bytes, cudaMemcpyHostToDevice,
                                stream_),
                "upload " + name);
      ThrowStatus(Q8_0ToTiles(static_cast<const std::uint8_t*>(stage), out,
                              in, target, stream_),
                  "tiles " + name);
    } else {
      const std::size_t count = static_cast<std::size_t>(out) * in;
      auto* host = static_cast<std::uint16_t*>(Pinned(count * 2));
      ThrowStatus(vx_random_bf16(seed_, id, count, 0.0f, kMatrixStd, host),
                  "seeded " + name);
      if (format == WeightFormat::kBf16) {
        ThrowCuda(cudaMemcpyAsync(target, host, count * 2,
                                  cudaMemcpyHostToDevice, stream_),
                  "upload " + name);
      } else {
        void* stage = Staging(count * 2);
        ThrowCuda(cudaMemcpyAsync(stage, host, count * 2,
                                  cudaMemcpyHostToDevice, stream_),
                  "upload " + name);
        ThrowStatus(Bf16ToTiles(static_cast<const std::uint16_t*>(stage), out,
                                in, reinterpret_cast<std::uint16_t*>(target),
                                stream_),
                    "tiles " + name);
      }
    }
    ThrowCuda(cudaStreamSynchronize(stream_), "upload " + name);
  }

  std::uint64_t seed_;
  CheckpointKind kind_;
  const ModelFiles* files_;
  DeviceArena* arena_;
  cudaStream_t stream_;
  std::size_t taken_ = 0;
  void* pinned_ = nullptr;
  std::size_t pinned_bytes_ = 0;
  void* bounce_[2] = {nullptr, nullptr};
  cudaEvent_t bounce_done_[2] = {nullptr, nullptr};
  void* staging_ = nullptr;
  std::size_t staging_bytes_ = 0;
  void* rows_ = nullptr;
  std::size_t rows_bytes_ = 0;
};

GeneratorWeights TakeAll(Uploader& take, const ModelConfig& c) {
  GeneratorWeights w;
  const int hidden = c.lm.hidden;
  const int local = c.encoder.hidden;
  const int dit = c.dit.hidden;
  const int feat = c.feat_dim;
  if (c.vocab > 0)
    w.embed = take.Vector("base_lm.embed_tokens.weight",
                          {static_cast<std::size_t>(c.vocab),
                           static_cast<std::size_t>(hidden)},
                          0.0f, 0.5f);
  w.base_lm = take.Stack("base_lm", c.lm, false);
  w.residual_lm = take.Stack("residual_lm", c.residual_lm, false);
  w.encoder = take.Stack("feat_encoder.encoder", c.encoder, false);
  w.special = take.Vector("feat_encoder.special_token",
                          {1, 1, 1, static_cast<std::size_t>(local)}, 0.0f,
                          1.0f);
  w.encoder_in = take.Linear("feat_encoder.in_proj", feat, local, true);
  w.dit = take.Stack("feat_decoder.estimator.decoder", c.dit, true);
  const std::string estimator = "feat_decoder.estimator.";
  w.dit_in = take.Linear(estimator + "in_proj", feat, dit, true);
  w.dit_cond = take.Linear(estimator + "cond_proj", feat, dit, true);
  w.dit_out = take.Linear(estimator + "out_proj", dit, feat, true);
  w.time_1 = take.Linear(estimator + "time_mlp.linear_1", dit, dit, true);
  w.time_2 = take.Linear(estimator + "time_mlp.linear_2", dit, dit, true);
  w.delta_time_1 =
      take.Linear(estimator + "delta_time_mlp.linear_1", dit, dit, true);
  w.delta_time_2 =
      take.Linear(estimator + "delta_time_mlp.linear_2", dit, dit, true);
  w.enc_to_lm = take.Linear("enc_to_lm_proj", local, hidden, true);
  w.lm_to_dit = take.Linear("lm_to_dit_proj", hidden, dit, true);
  w.res_to_dit = take.Linear("res_to_dit_proj", hidden, dit, true);
  w.fusion = take.Linear("fusion_concat_proj", 2 * hidden, hidden, true);
  w.fsq_in = take.Linear("fsq_layer.in_proj", hidden, c.fsq_latent_dim, true);
  w.fsq_out = take.Linear("fsq_layer.out_proj", c.fsq_latent_dim, hidden, true);
  w.stop_proj = take.Linear("stop_proj", hidden, hidden, true);
  w.stop_head = take.Linear("stop_head", hidden, 2, false);
  return w;
}

std::size_t CacheElementBytes(CacheType type) {
  return type == CacheType::kF32 ? 4 : 2;
}

}  // namespace

std::uint64_t TensorId(const std::string& name) {
  std::uint64_t h = 0xCBF29CE484222325ull;
  for (const unsigned char c : name) {
    h ^= c;
    h *= 0x100000001B3ull;
  }
  return h;
}

ModelConfig ReleasedConfig() {
  ModelConfig c;
  c.lm = {2048, 6144, 28, 16, 2, 128, 1e-5f, true};
  c.residual_lm = {2048, 6144, 8, 16, 2, 128, 1e-5f, false};
  c.encoder = {1024, 4096, 12, 16, 2, 128, 1e-5f, true};
  c.dit = {1024, 4096, 12, 16, 2, 128, 1e-5f, true};
  c.rope_factors.assign(64, 1.0);
  return c;
}

// ------------------------------------------------------------ KvCache

KvCache::KvCache(const StackConfig& config, int capacity, CacheType type,
                 int slots)
    : capacity_(capacity), type_(type) {
  slot_bytes_ = static_cast<std::size_t>(config.kv_heads) * capacity *
                config.head_dim * CacheElementBytes(type);
  layer_bytes_ = slot_bytes_ * static_cast<std::size_t>(std::max(slots, 1));
  bytes_ = layer_bytes_ * config.layers;
  ThrowCuda(cudaMalloc(reinterpret_cast<void**>(&keys_), bytes_),
            "cudaMalloc keys");
  if (cudaMalloc(reinterpret_cast<void**>(&values_), bytes_) != cudaSuccess) {
    cudaFree(keys_);
    keys_ = nullptr;
    throw std::runtime_error("cudaMalloc values failed");
  }
  bytes_ *= 2;
}

KvCache::~KvCache() { Release(); }

KvCache::KvCache(KvCache&& other) noexcept { *this = std::move(other); }

KvCache& KvCache::operator=(KvCache&& other) noexcept {
  if (this != &other) {
    Release();
    keys_ = other.keys_;
    values_ = other.values_;
    owns_ = other.owns_;
    slot_bytes_ = other.slot_bytes_;
    layer_bytes_ = other.layer_bytes_;
    bytes_ = other.bytes_;
    capacity_ = other.capacity_;
    type_ = other.type_;
    other.keys_ = other.values_ = nullptr;
    other.bytes_ = 0;
    other.capacity_ = 0;
  }
  return *this;
}

void KvCache::Release() {
  if (owns_) {
    if (keys_ != nullptr)
      cudaFree(keys_);
    if (values_ != nullptr)
      cudaFree(values_);
  }
  keys_ = values_ = nullptr;
}

void* KvCache::keys(int layer) const { return keys_ + layer * layer_bytes_; }
void* KvCache::values(int layer) const {
  return values_ + layer * layer_bytes_;
}

KvCache KvCache::Slot(int slot) const {
  KvCache view;
  view.keys_ = keys_ + static_cast<std::size_t>(slot) * slot_bytes_;
  view.values_ = values_ + static_cast<std::size_t>(slot) * slot_bytes_;
  view.owns_ = false;
  view.slot_bytes_ = slot_bytes_;
  view.layer_bytes_ = layer_bytes_;
  view.bytes_ = 0;
  view.capacity_ = capacity_;
  view.type_ = type_;
  return view;
}

// ------------------------------------------------------------ stack loop

int Linear(const std::uint16_t* x, const Projection& p, float* y, int rows,
           bool accumulate, cudaStream_t stream) {
  for (int first = 0; first < rows; first += kMaxProductRows) {
    const int count = std::min(kMaxProductRows, rows - first);
    const int status = LaunchProduct(
        p.format, x + static_cast<std::size_t>(first) * p.in, p.weight,
        y + static_cast<std::size_t>(first) * p.out, nullptr, count, p.in,
        p.out, accumulate, nullptr, stream);
    if (status != kOk)
      return status;
  }
  return kOk;
}

int Project(const Projection& p, const std::uint16_t* x, float* y, int rows,
            cudaStream_t stream) {
  int status = Linear(x, p, y, rows, false, stream);
  if (status == kOk && p.bias != nullptr)
    status = AddBias(y, p.bias, rows, p.out, stream);
  return status;
}

int ForwardStack(const StackWeights& stack, const float* rope,
                 const AttentionLayout& layout, KvCache& cache, float* hidden,
                 float* output, int rows, StackScratch& s,
                 cudaStream_t stream) {
  const StackConfig& c = stack.config;
  const int width = c.hidden;
  const int q_width = c.heads * c.head_dim;
  int status = kOk;
  auto run = [&](int st) {
    if (status == kOk)
      status = st;
  };
  for (int index = 0; index < c.layers && status == kOk; ++index) {
    const LayerWeights& layer = stack.layers[index];
    run(RmsNorm(hidden, layer.input_norm, s.normed, nullptr, rows, width,
                c.rms_eps, stream));
    run(Linear(s.normed, layer.qkv, s.qkv, rows, false, stream));
    run(QkvRope(s.qkv, c.rope ? rope : nullptr, layout.positions,
                layout.cache_rows, s.q, cache.keys(index), cache.values(index),
                cache.type(), rows, c.heads, c.kv_heads, c.head_dim,
                cache.capacity(), stream));
    run(Attention(s.q, cache.keys(index), cache.values(index), cache.type(),
                  s.attention, rows, layout.rows_per_sequence,
                  layout.keys_per_sequence, layout.past, layout.past_device,
                  layout.causal, c.heads, c.kv_heads, c.head_dim,
                  cache.capacity(), layout.max_keys, stream,
                  layout.past_per_sequence, layout.first_keys));
    run(Linear(s.attention, layer.o, hidden, rows, true, stream));
    run(RmsNorm(hidden, layer.post_norm, s.normed, nullptr, rows, width,
                c.rms_eps, stream));
    run(Linear(s.normed, layer.gate_up, s.gate_up, rows, false, stream));
    run(SwiGlu(s.gate_up, s.activation, rows, c.intermediate, stream));
    run(Linear(s.activation, layer.down, hidden, rows, true, stream));
  }
  run(RmsNorm(hidden, stack.norm, s.normed, output, rows, width, c.rms_eps,
              stream));
  return status;
}

// ------------------------------------------------------------ Generator

std::unique_ptr<Generator> Generator::Create(const ModelConfig& config,
                                             std::uint64_t seed,
                                             CheckpointKind kind,
                                             CacheType cache_type,
                                             std::string* error,
                                             const ModelFiles* files,
                                             const Generator* share,
                                             cudaStream_t stream,
                                             const SlotCaches* lm_caches) {
  std::unique_ptr<Generator> g(new Generator());
  try {
    const ModelConfig& c = config;
    for (const StackConfig* s : {&c.lm, &c.residual_lm, &c.encoder, &c.dit}) {
      if (s->head_dim != 128)
        throw std::runtime_error("the attention kernels need a head size of 128");
      if (s->kv_heads <= 0 || s->heads % s->kv_heads != 0)
        throw std::runtime_error("attention heads must be a multiple of the KV heads");
      if (s->hidden % 32 != 0 || s->intermediate % 32 != 0)
        throw std::runtime_error("stack widths must be multiples of 32");
    }
    if (c.lm.hidden != c.residual_lm.hidden ||
        static_cast<int>(c.rope_factors.size()) * 2 != c.lm.head_dim ||
        c.feat_dim % 32 != 0 || c.patch_size < 1 || c.max_length < 2)
      throw std::runtime_error("unsupported configuration");
    g->config_ = config;
    if (stream != nullptr) {
      g->stream_ = stream;
      g->owns_stream_ = false;
    } else {
      ThrowCuda(cudaStreamCreateWithFlags(&g->stream_, cudaStreamNonBlocking),
                "cudaStreamCreate");
    }

    // Count, allocate, upload (weights.cpp:308-327).
    if (share != nullptr) {
      g->arena_ = share->arena_;
      g->w_ = share->w_;
    } else {
      DeviceArena counter;
      Uploader count(seed, kind, files, &counter, g->stream_);
      (void)TakeAll(count, c);
      if (files != nullptr && count.taken() != files->model_tensors().size())
        throw std::runtime_error(
            "the checkpoint holds tensors VoxCPM2 does not use");
      g->arena_ = std::make_unique<DeviceArena>(counter.used());
      Uploader take(seed, kind, files, g->arena_.get(), g->stream_);
      g->w_ = TakeAll(take, c);
    }
    if (files != nullptr)
      files->ReleasePages();

    const int patch_values = c.patch_size * c.feat_dim;
    const int dit_rows = 2 * (3 + 2 * c.patch_size);
    const int positions = std::max(c.max_length, 64);
    const int max_hidden = std::max(c.lm.hidden, c.dit.hidden);
    // Work buffers in one allocation (counted first).
    auto plan = [&](DeviceArena& a) {
      g->rope_ = a.Take<float>(static_cast<std::size_t>(positions) * 128);
      g->lm_hidden_ = a.Take<float>(c.lm.hidden);
      g->residual_hidden_ = a.Take<float>(c.lm.hidden);
      g->prefix_cond_ = a.Take<float>(patch_values);
      g->x_ = a.Take<float>(2 * patch_values);  // x and the patch's noise
      g->latent_slots_ = a.Take<float>(2 * patch_values);
      g->velocity_ = a.Take<float>(2 * patch_values);
      g->mu_ = a.Take<float>(2 * c.dit.hidden);
      g->cond_rows_ = a.Take<float>(static_cast<std::size_t>(c.patch_size) * c.dit.hidden);
      g->stop_ = a.Take<float>(2);
      g->delta_time_ = a.Take<float>(c.dit.hidden);
      g->embed_ = a.Take<float>(c.lm.hidden);
      g->position_counter_ = a.Take<std::int32_t>(1);
      g->step_positions_ = a.Take<std::int32_t>(1);
      g->dit_positions_ = a.Take<std::int32_t>(dit_rows);
      g->dit_rows_ = a.Take<std::int32_t>(dit_rows);
      g->dit_outputs_ = a.Take<std::int32_t>(2 * c.patch_size);
      g->step_bf16_ = a.Take<std::uint16_t>(2 * static_cast<std::size_t>(c.lm.hidden));
      g->step_a_ = a.Take<float>(c.lm.hidden);
      g->step_b_ = a.Take<float>(c.lm.hidden);
      g->dit_bf16_ = a.Take<std::uint16_t>(static_cast<std::size_t>(dit_rows) * c.dit.hidden);
      g->x_rows_ = a.Take<float>(static_cast<std::size_t>(c.patch_size) * c.dit.hidden);
      g->dit_hidden_ = a.Take<float>(static_cast<std::size_t>(dit_rows) * c.dit.hidden);
      g->dit_output_ = a.Take<float>(static_cast<std::size_t>(dit_rows) * c.dit.hidden);
      g->fsq_bf16_ = a.Take<std::uint16_t>(static_cast<std::size_t>(std::max(c.lm.hidden, c.fsq_latent_dim)));
      g->fsq_latent_ = a.Take<float>(c.fsq_latent_dim);
      (void)max_hidden;
    };
    {
      DeviceArena counter;
      plan(counter);
      g->work_ = std::make_unique<DeviceArena>(counter.used());
      plan(*g->work_);
    }
    // Rotary table (transformer.cpp:20-45).
    {
      std::vector<float> table(static_cast<std::size_t>(positions) * 128);
      ThrowStatus(vx_rope_table(c.rope_theta, 128, c.rope_factors.data(),
                                c.rope_scaling, positions, table.data()),
                  "rope table");
      ThrowCuda(cudaMemcpy(g->rope_, table.data(), table.size() * 4,
                           cudaMemcpyHostToDevice),
                "upload rope");
    }
    if (lm_caches != nullptr) {
      g->base_cache_ = lm_caches->base->Slot(lm_caches->slot);
      g->residual_cache_ = lm_caches->residual->Slot(lm_caches->slot);
    } else {
      g->base_cache_ = KvCache(c.lm, c.max_length, cache_type);
      g->residual_cache_ = KvCache(c.residual_lm, c.max_length, cache_type);
    }
    g->dit_cache_ = KvCache(c.dit, dit_rows, cache_type);
    g->encoder_cache_ = KvCache(c.encoder, 64, cache_type);
    g->EnsureRows(std::max(dit_rows, c.patch_size + 1));

    // The DiT's rows: two sequences of 3 + 2P positions; outputs are the
    // last P rows of each (generator.cpp:109-124).
    {
      const int length = dit_rows / 2;
      std::vector<std::int32_t> pos(dit_rows), rows(dit_rows), outs;
      for (int r = 0; r < dit_rows; ++r) {
        pos[r] = r % length;
        rows[r] = r;
      }
      for (int s = 0; s < 2; ++s)
        for (int i = 0; i < c.patch_size; ++i)
          outs.push_back(s * length + 3 + c.patch_size + i);
      ThrowCuda(cudaMemcpy(g->dit_positions_, pos.data(), dit_rows * 4,
                           cudaMemcpyHostToDevice), "upload indices");
      ThrowCuda(cudaMemcpy(g->dit_rows_, rows.data(), dit_rows * 4,
                           cudaMemcpyHostToDevice), "upload indices");
      ThrowCuda(cudaMemcpy(g->dit_outputs_, outs.data(), outs.size() * 4,
                           cudaMemcpyHostToDevice), "upload indices");
    }
    ThrowCuda(cudaMemset(g->position_counter_, 0, 4), "cudaMemset");
    ThrowCuda(cudaMemset(g->step_positions_, 0, 4), "cudaMemset");
    ThrowCuda(cudaEventCreateWithFlags(&g->latent_event_, cudaEventDisableTiming),
              "cudaEventCreate");
    ThrowCuda(cudaMallocHost(reinterpret_cast<void**>(&g->pinned_noise_),
                             patch_values * sizeof(float)), "cudaMallocHost");
    ThrowCuda(cudaMallocHost(reinterpret_cast<void**>(&g->pinned_latent_),
                             patch_values * sizeof(float)), "cudaMallocHost");
    ThrowCuda(cudaMallocHost(reinterpret_cast<void**>(&g->pinned_stop_),
                             2 * sizeof(float)), "cudaMallocHost");

    // delta_time_mlp(sinusoid(0)) (generator.cpp:150-166).
    {
      const int width = c.dit.hidden;
      std::vector<float> zero(width);
      ThrowStatus(vx_sinusoid(0.0f, width, zero.data()), "sinusoid");
      float* input = g->dit_hidden_;
      float* middle = g->dit_output_;
      ThrowCuda(cudaMemcpyAsync(input, zero.data(), width * 4,
                                cudaMemcpyHostToDevice, g->stream_), "upload");
      g->Check(ToBf16(input, g->dit_bf16_, width, false, g->stream_), "ToBf16");
      g->Check(Project(g->w_.delta_time_1, g->dit_bf16_, middle, 1, g->stream_),
               "delta_time_1");
      g->Check(ToBf16(middle, g->dit_bf16_, width, true, g->stream_), "ToBf16");
      g->Check(Project(g->w_.delta_time_2, g->dit_bf16_, g->delta_time_, 1,
                       g->stream_),
               "delta_time_2");
      g->CheckCuda(cudaStreamSynchronize(g->stream_), "create");
    }
    g->SetupPersistent();
    g->SetupPersistentLm();
  } catch (const std::exception& failure) {
    if (error != nullptr)
      *error = failure.what();
    return nullptr;
  }
  return g;
}

Generator::~Generator() {
  if (stream_ != nullptr)
    cudaStreamSynchronize(stream_);
  DestroyGraphs();
  for (auto& kv : time_vectors_)
    cudaFree(kv.second);
  auto free = [](auto*& p) {
    if (p != nullptr)
      cudaFree(p);
    p = nullptr;
  };
  free(prefill_block_);
  free(scratch_.normed);
  free(scratch_.qkv);
  free(scratch_.q);
  free(scratch_.attention);
  free(scratch_.gate_up);
  free(scratch_.activation);
  free(local_positions_);
  free(local_rows_);
  free(local_firsts_);
  free(encoder_bf16_);
  free(encoder_a_);
  free(encoder_b_);
  free(encoder_c_);
  free(dit_layers_);
  free(dit_work_);
  free(dit_io_tiles_);
  free(dit_times_);
  free(dit_dts_);
  free(lm_layers_);
  free(lm_work_);
  if (pinned_noise_ != nullptr)
    cudaFreeHost(pinned_noise_);
  if (pinned_latent_ != nullptr)
    cudaFreeHost(pinned_latent_);
  if (pinned_stop_ != nullptr)
    cudaFreeHost(pinned_stop_);
  if (latent_event_ != nullptr)
    cudaEventDestroy(latent_event_);
  arena_.reset();
  work_.reset();
  if (stream_ != nullptr && owns_stream_)
    cudaStreamDestroy(stream_);
}

std::size_t Generator::weight_bytes() const {
  return arena_ ? arena_->used() : 0;
}

void Generator::Check(int status, const char* what) { ThrowStatus(status, what); }

void Generator::CheckCuda(cudaError_t error, const char* what) {
  ThrowCuda(error, what);
}

void Generator::DestroyGraphs() {
  ++buffers_epoch_;
  if (step_graph_ != nullptr)
    cudaGraphExecDestroy(step_graph_);
  if (patch_graph_ != nullptr)
    cudaGraphExecDestroy(patch_graph_);
  step_graph_ = nullptr;
  patch_graph_ = nullptr;
}

void Generator::EnsureRows(int rows) {
  if (rows <= scratch_rows_)
    return;
  CheckCuda(cudaStreamSynchronize(stream_), "sync");
  DestroyGraphs();  // graphs hold the old scratch pointers
  const ModelConfig& c = config_;
  int hidden = 0, qkv = 0, q = 0, inter = 0;
  for (const StackConfig* s : {&c.lm, &c.residual_lm, &c.encoder, &c.dit}) {
    hidden = std::max(hidden, s->hidden);
    qkv = std::max(qkv, (s->heads + 2 * s->kv_heads) * s->head_dim);
    q = std::max(q, s->heads * s->head_dim);
    inter = std::max(inter, s->intermediate);
  }
  auto realloc = [&](auto*& p, std::size_t count) {
    using T = std::remove_reference_t<decltype(*p)>;
    if (p != nullptr)
      cudaFree(p);
    p = nullptr;
    CheckCuda(cudaMalloc(reinterpret_cast<void**>(&p), count * sizeof(T)),
              "cudaMalloc scratch");
  };
  const std::size_t r = rows;
  realloc(scratch_.normed, r * hidden);
  realloc(scratch_.qkv, r * qkv);
  realloc(scratch_.q, r * q);
  realloc(scratch_.attention, r * q);
  realloc(scratch_.gate_up, r * 2 * inter);
  realloc(scratch_.activation, r * inter);
  scratch_rows_ = rows;
}

void Generator::PrepareTimes(int timesteps) {
  if (static_cast<int>(schedule_t_.size()) != timesteps) {
    schedule_t_.assign(timesteps, 0.0f);
    schedule_dt_.assign(timesteps, 0.0f);
    std::vector<std::int32_t> evaluate(timesteps);
    vx_euler_schedule(timesteps, 1.0f, schedule_t_.data(), schedule_dt_.data(),
                      evaluate.data(), timesteps);
    schedule_eval_.assign(evaluate.begin(), evaluate.end());
  }
  std::vector<const float*> times;
  std::vector<float> dts;
  for (int i = 0; i < timesteps; ++i)
    if (schedule_eval_[i]) {
      times.push_back(TimeVector(schedule_t_[i]));
      dts.push_back(schedule_dt_[i]);
    }
  if (!persistent_ok_ || dit_schedule_timesteps_ == timesteps)
    return;
  // The persistent kernel's per-evaluation schedule, on the device.
  const int count = static_cast<int>(times.size());
  CheckCuda(cudaStreamSynchronize(stream_), "sync");
  if (count > dit_schedule_capacity_) {
    DestroyGraphs();  // graphs hold the old schedule pointers
    for (void* p : {static_cast<void*>(dit_times_), static_cast<void*>(dit_dts_)})
      if (p != nullptr)
        cudaFree(p);
    dit_times_ = nullptr;
    dit_dts_ = nullptr;
    dit_schedule_capacity_ = 0;
    const std::size_t capacity = std::max(count, 16);
    CheckCuda(cudaMalloc(reinterpret_cast<void**>(&dit_times_),
                         capacity * sizeof(float*)), "cudaMalloc schedule");
    CheckCuda(cudaMalloc(reinterpret_cast<void**>(&dit_dts_),
                         capacity * sizeof(float)), "cudaMalloc schedule");
    dit_schedule_capacity_ = static_cast<int>(capacity);
  }
  if (count > 0) {
    CheckCuda(cudaMemcpy(dit_times_, times.data(), count * sizeof(float*),
                         cudaMemcpyHostToDevice), "upload schedule");
    CheckCuda(cudaMemcpy(dit_dts_, dts.data(), count * sizeof(float),
                         cudaMemcpyHostToDevice), "upload schedule");
  }
  dit_evaluations_ = count;
  dit_schedule_timesteps_ = timesteps;
}

void Generator::SetupPersistent() {
  // The persistent patch serves VoxCPM2's DiT shape with tiled layer
  // weights (both checkpoint kinds store the DiT stack as tiles).
  const ModelConfig& c = config_;
  const StackConfig& d = c.dit;
  using Shape = DitShape;
  if (d.hidden != Shape::kHidden || d.intermediate != Shape::kIntermediate ||
      d.heads != Shape::kHeads || d.kv_heads != Shape::kKvHeads ||
      d.head_dim != Shape::kHeadDim || c.patch_size != Shape::kPatch ||
      c.feat_dim != Shape::kFeat || d.layers < 1)
    return;
  const WeightFormat format = w_.dit.layers[0].qkv.format;
  if (!DitPatchSupported(format))
    return;
  // The kernel streams every layer in one format; checkpoint files may mix
  // formats, and those run the per-kernel sequence.
  for (const LayerWeights& layer : w_.dit.layers)
    for (const Projection* m : {&layer.qkv, &layer.o, &layer.gate_up, &layer.down})
      if (m->format != format)
        return;
  std::vector<DitLayer> layers(d.layers);
  for (int i = 0; i < d.layers; ++i) {
    const LayerWeights& w = w_.dit.layers[i];
    layers[i].qkv = static_cast<const unsigned char*>(w.qkv.weight);
    layers[i].o = static_cast<const unsigned char*>(w.o.weight);
    layers[i].gate_up = static_cast<const unsigned char*>(w.gate_up.weight);
    layers[i].down = static_cast<const unsigned char*>(w.down.weight);
    layers[i].input_norm = w.input_norm;
    layers[i].post_norm = w.post_norm;
  }
  CheckCuda(cudaMalloc(reinterpret_cast<void**>(&dit_layers_),
                       layers.size() * sizeof(DitLayer)), "cudaMalloc layers");
  CheckCuda(cudaMemcpy(dit_layers_, layers.data(),
                       layers.size() * sizeof(DitLayer), cudaMemcpyHostToDevice),
            "upload layers");
  CheckCuda(cudaMalloc(&dit_work_, DitWorkBytes()), "cudaMalloc DiT work");
  DitPatchParams& p = dit_params_;
  DitWorkLayout(dit_work_, p);
  p.format = format;
  p.layers = d.layers;
  p.bf16_kv = dit_cache_.type() == CacheType::kBf16 ? 1 : 0;
  p.eps = d.rms_eps;
  p.attention_scale = 1.0f / std::sqrt(static_cast<float>(d.head_dim));
  p.layer = dit_layers_;
  p.final_norm = w_.dit.norm;
  p.rope = d.rope ? rope_ : nullptr;
  p.mu = mu_;
  p.cond_rows = cond_rows_;
  p.x = x_;
  p.dit_in_bias = w_.dit_in.bias;
  p.dit_out_bias = w_.dit_out.bias;
  if (w_.dit_in.format == format && w_.dit_out.format == format) {
    p.dit_in = static_cast<const unsigned char*>(w_.dit_in.weight);
    p.dit_out = static_cast<const unsigned char*>(w_.dit_out.weight);
  } else if (format == WeightFormat::kBf16Tiles &&
             w_.dit_in.format == WeightFormat::kBf16 &&
             w_.dit_out.format == WeightFormat::kBf16) {
    // The bf16 checkpoint keeps the DiT's in/out projections as rows; the
    // persistent kernel streams them as tiles.
    const std::size_t in_bytes = Bf16TilesBytes(w_.dit_in.out, w_.dit_in.in);
    const std::size_t out_bytes = Bf16TilesBytes(w_.dit_out.out, w_.dit_out.in);
    CheckCuda(cudaMalloc(reinterpret_cast<void**>(&dit_io_tiles_),
                         in_bytes + out_bytes), "cudaMalloc tiles");
    Check(Bf16ToTiles(static_cast<const std::uint16_t*>(w_.dit_in.weight),
                      w_.dit_in.out, w_.dit_in.in,
                      reinterpret_cast<std::uint16_t*>(dit_io_tiles_), stream_),
          "dit_in tiles");
    Check(Bf16ToTiles(static_cast<const std::uint16_t*>(w_.dit_out.weight),
                      w_.dit_out.out, w_.dit_out.in,
                      reinterpret_cast<std::uint16_t*>(dit_io_tiles_ + in_bytes),
                      stream_),
          "dit_out tiles");
    CheckCuda(cudaStreamSynchronize(stream_), "tiles");
    p.dit_in = dit_io_tiles_;
    p.dit_out = dit_io_tiles_ + in_bytes;
  } else {
    return;
  }
  persistent_ok_ = true;
  persistent_ = true;
}

void Generator::SetupPersistentLm() {
  // The persistent one-row stacks serve VoxCPM2's LM shape with Q8 tiles.
  const ModelConfig& c = config_;
  for (const StackConfig* stack : {&c.lm, &c.residual_lm})
    if (stack->hidden != LmShape::kHidden ||
        stack->intermediate != LmShape::kIntermediate ||
        stack->heads != LmShape::kHeads || stack->kv_heads != LmShape::kKvHeads ||
        stack->head_dim != LmShape::kHeadDim || stack->layers < 1)
      return;
  for (const StackWeights* stack : {&w_.base_lm, &w_.residual_lm})
    for (const LayerWeights& layer : stack->layers)
      for (const Projection* m : {&layer.qkv, &layer.o, &layer.gate_up, &layer.down})
        if (m->format != WeightFormat::kQ8Tiles)
          return;
  if (!LmStackSupported())
    return;
  const StackWeights* stacks[2] = {&w_.base_lm, &w_.residual_lm};
  KvCache* caches[2] = {&base_cache_, &residual_cache_};
  std::vector<LmLayer> layers;
  for (int k = 0; k < 2; ++k)
    for (int i = 0; i < stacks[k]->config.layers; ++i) {
      const LayerWeights& w = stacks[k]->layers[i];
      LmLayer l;
      l.qkv = static_cast<const unsigned char*>(w.qkv.weight);
      l.o = static_cast<const unsigned char*>(w.o.weight);
      l.gate_up = static_cast<const unsigned char*>(w.gate_up.weight);
      l.down = static_cast<const unsigned char*>(w.down.weight);
      l.input_norm = w.input_norm;
      l.post_norm = w.post_norm;
      l.keys = caches[k]->keys(i);
      l.values = caches[k]->values(i);
      layers.push_back(l);
    }
  CheckCuda(cudaMalloc(reinterpret_cast<void**>(&lm_layers_),
                       layers.size() * sizeof(LmLayer)), "cudaMalloc layers");
  CheckCuda(cudaMemcpy(lm_layers_, layers.data(), layers.size() * sizeof(LmLayer),
                       cudaMemcpyHostToDevice), "upload layers");
  CheckCuda(cudaMalloc(&lm_work_, LmWorkBytes()), "cudaMalloc stack work");
  int offset = 0;
  for (int k = 0; k < 2; ++k) {
    LmStackParams& p = lm_params_[k];
    LmWorkLayout(lm_work_, p);
    const StackConfig& sc = stacks[k]->config;
    p.layers = sc.layers;
    p.bf16_kv = caches[k]->type() == CacheType::kBf16 ? 1 : 0;
    p.capacity = caches[k]->capacity();
    p.eps = sc.rms_eps;
    p.attention_scale = 1.0f / std::sqrt(static_cast<float>(sc.head_dim));
    p.layer = lm_layers_ + offset;
    p.final_norm = stacks[k]->norm;
    p.rope = sc.rope ? rope_ : nullptr;
    p.position = position_counter_;
    offset += sc.layers;
  }
  lm_persistent_ok_ = true;
}

void Generator::StepStack(int which, const AttentionLayout& layout,
                          float* hidden, float* output) {
  if (persistent_ && lm_persistent_ok_) {
    LmStackParams p = lm_params_[which];
    p.hidden = hidden;
    p.output = output;
    Check(LaunchLmStack(p, stream_), which == 0 ? "persistent lm" : "persistent residual lm");
    return;
  }
  if (which == 0)
    Check(ForwardStack(w_.base_lm, rope_, layout, base_cache_, hidden, output,
                       1, scratch_, stream_),
          "base lm");
  else
    Check(ForwardStack(w_.residual_lm, nullptr, layout, residual_cache_, hidden,
                       output, 1, scratch_, stream_),
          "residual lm");
}

bool Generator::set_persistent(bool enabled) {
  if (enabled && !persistent_ok_)
    return false;
  if (enabled != persistent_) {
    CheckCuda(cudaStreamSynchronize(stream_), "sync");
    DestroyGraphs();
    persistent_ = enabled;
  }
  return true;
}

const float* Generator::TimeVector(float t) {
  // time_mlp(sinusoid(t)) + delta_time_mlp(sinusoid(0)), computed once per t
  // (generator.cpp:212-237).
  const auto found = time_vectors_.find(t);
  if (found != time_vectors_.end())
    return found->second;
  const int width = config_.dit.hidden;
  std::vector<float> sinusoid(width);
  ThrowStatus(vx_sinusoid(t, width, sinusoid.data()), "sinusoid");
  float* vector = nullptr;
  CheckCuda(cudaMalloc(reinterpret_cast<void**>(&vector), width * 4),
            "cudaMalloc time vector");
  float* input = dit_hidden_;
  float* middle = dit_output_;
  CheckCuda(cudaMemcpyAsync(input, sinusoid.data(), width * 4,
                            cudaMemcpyHostToDevice, stream_), "upload");
  Check(ToBf16(input, dit_bf16_, width, false, stream_), "ToBf16");
  Check(Project(w_.time_1, dit_bf16_, middle, 1, stream_), "time_1");
  Check(ToBf16(middle, dit_bf16_, width, true, stream_), "ToBf16");
  Check(CopyFloats(delta_time_, vector, width, stream_), "copy");
  Check(Linear(dit_bf16_, w_.time_2, vector, 1, true, stream_), "time_2");
  Check(AddBias(vector, w_.time_2.bias, 1, width, stream_), "bias");
  CheckCuda(cudaStreamSynchronize(stream_), "time vector");
  time_vectors_.emplace(t, vector);
  return vector;
}

void Generator::EvaluateDit(const float* x, float t, float* velocity) {
  // generator.cpp:297-324
  const ModelConfig& c = config_;
  const int patch = c.patch_size;
  const int width = c.dit.hidden;
  const int rows = 2 * (3 + 2 * patch);
  const float* time = TimeVector(t);
  Check(ToBf16(x, dit_bf16_, patch * c.feat_dim, false, stream_), "ToBf16");
  Check(Project(w_.dit_in, dit_bf16_, x_rows_, patch, stream_), "dit_in");
  Check(AssembleDit(mu_, time, cond_rows_, x_rows_, dit_hidden_, patch, width,
                    stream_),
        "AssembleDit");
  AttentionLayout layout;
  layout.positions = dit_positions_;
  layout.cache_rows = dit_rows_;
  layout.rows_per_sequence = rows / 2;
  layout.keys_per_sequence = rows / 2;
  layout.causal = false;
  Check(ForwardStack(w_.dit, rope_, layout, dit_cache_, dit_hidden_,
                     dit_output_, rows, scratch_, stream_),
        "dit stack");
  Check(GatherRows(dit_output_, dit_outputs_, dit_hidden_, 2 * patch, width,
                   stream_),
        "GatherRows");
  Check(ToBf16(dit_hidden_, dit_bf16_, 2 * patch * width, false, stream_),
        "ToBf16");
  Check(Project(w_.dit_out, dit_bf16_, velocity, 2 * patch, stream_),
        "dit_out");
}

void Generator::EnsureEncoder(int patches) {
  // Buffers, index arrays and the cache of the local encoder for `patches`
  // patches (sized outside any graph capture).
  const ModelConfig& c = config_;
  const int patch = c.patch_size;
  const int width = c.encoder.hidden;
  const int rows = patches * (patch + 1);
  if (encoder_cache_.capacity() < rows) {
    CheckCuda(cudaStreamSynchronize(stream_), "sync");
    DestroyGraphs();
    encoder_cache_ = KvCache(c.encoder, std::max(rows, 64), encoder_cache_.type());
  }
  EnsureRows(rows);
  if (local_capacity_ >= patches)
    return;
  CheckCuda(cudaStreamSynchronize(stream_), "sync");
  DestroyGraphs();
  for (auto** p : {&local_positions_, &local_rows_, &local_firsts_})
    if (*p != nullptr)
      cudaFree(*p);
  for (auto** p : {&encoder_a_, &encoder_b_, &encoder_c_})
    if (*p != nullptr)
      cudaFree(*p);
  if (encoder_bf16_ != nullptr)
    cudaFree(encoder_bf16_);
  const std::size_t r = rows;
  CheckCuda(cudaMalloc(reinterpret_cast<void**>(&local_positions_), r * 4), "cudaMalloc");
  CheckCuda(cudaMalloc(reinterpret_cast<void**>(&local_rows_), r * 4), "cudaMalloc");
  CheckCuda(cudaMalloc(reinterpret_cast<void**>(&local_firsts_), patches * 4), "cudaMalloc");
  CheckCuda(cudaMalloc(reinterpret_cast<void**>(&encoder_a_), r * width * 4), "cudaMalloc");
  CheckCuda(cudaMalloc(reinterpret_cast<void**>(&encoder_b_), r * width * 4), "cudaMalloc");
  CheckCuda(cudaMalloc(reinterpret_cast<void**>(&encoder_c_), r * width * 4), "cudaMalloc");
  CheckCuda(cudaMalloc(reinterpret_cast<void**>(&encoder_bf16_),
                       r * std::max(width, c.feat_dim) * 2), "cudaMalloc");
  std::vector<std::int32_t> pos(rows), iota(rows), firsts(patches);
  for (int i = 0; i < rows; ++i) {
    pos[i] = i % (patch + 1);
    iota[i] = i;
  }
  for (int i = 0; i < patches; ++i)
    firsts[i] = i * (patch + 1);
  CheckCuda(cudaMemcpy(local_positions_, pos.data(), rows * 4, cudaMemcpyHostToDevice), "upload");
  CheckCuda(cudaMemcpy(local_rows_, iota.data(), rows * 4, cudaMemcpyHostToDevice), "upload");
  CheckCuda(cudaMemcpy(local_firsts_, firsts.data(), patches * 4, cudaMemcpyHostToDevice), "upload");
  local_capacity_ = patches;
}

void Generator::Encode(const float* latents, int patches, float* embeds) {
  // generator.cpp:252-295
  const ModelConfig& c = config_;
  const int patch = c.patch_size;
  const int width = c.encoder.hidden;
  const int rows = patches * (patch + 1);
  EnsureEncoder(patches);
  Check(ToBf16(latents, encoder_bf16_, patches * patch * c.feat_dim, false,
               stream_),
        "ToBf16");
  Check(Project(w_.encoder_in, encoder_bf16_, encoder_a_, patches * patch,
                stream_),
        "encoder_in");
  Check(PrependSpecial(encoder_a_, w_.special, encoder_b_, patches, patch,
                       width, stream_),
        "PrependSpecial");
  AttentionLayout layout;
  layout.positions = local_positions_;
  layout.cache_rows = local_rows_;
  layout.rows_per_sequence = patch + 1;
  layout.keys_per_sequence = patch + 1;
  layout.causal = false;
  Check(ForwardStack(w_.encoder, rope_, layout, encoder_cache_, encoder_b_,
                     encoder_c_, rows, scratch_, stream_),
        "encoder stack");
  Check(GatherRows(encoder_c_, local_firsts_, encoder_a_, patches, width,
                   stream_),
        "GatherRows");
  Check(ToBf16(encoder_a_, encoder_bf16_, patches * width, false, stream_),
        "ToBf16");
  Check(Project(w_.enc_to_lm, encoder_bf16_, embeds, patches, stream_),
        "enc_to_lm");
}

void Generator::Fsq(const float* input, float* output, int rows) {
  // generator.cpp:239-250 (single rows on the step path; prefill uses its
  // own buffers through the same kernels).
  const ModelConfig& c = config_;
  Check(ToBf16(input, fsq_bf16_, rows * c.lm.hidden, false, stream_), "ToBf16");
  Check(Project(w_.fsq_in, fsq_bf16_, fsq_latent_, rows, stream_), "fsq_in");
  Check(Quantize(fsq_latent_, fsq_bf16_, rows * c.fsq_latent_dim, c.fsq_scale,
                 stream_),
        "Quantize");
  Check(Project(w_.fsq_out, fsq_bf16_, output, rows, stream_), "fsq_out");
}

void Generator::DitCond() {
  const ModelConfig& c = config_;
  Check(ToBf16(prefix_cond_, step_bf16_, c.patch_size * c.feat_dim, false,
               stream_),
        "ToBf16");
  Check(Project(w_.dit_cond, step_bf16_, cond_rows_, c.patch_size, stream_),
        "dit_cond");
}

void Generator::EulerLoop(int timesteps, float cfg) {
  const int values = config_.patch_size * config_.feat_dim;
  if (persistent_) {
    // PrepareTimes(timesteps) uploaded this schedule beforehand.
    if (dit_schedule_timesteps_ != timesteps)
      throw std::logic_error("DiT schedule not prepared");
    if (dit_evaluations_ == 0)
      return;
    DitPatchParams p = dit_params_;
    p.cfg = cfg;
    p.evaluations = dit_evaluations_;
    p.time_vectors = dit_times_;
    p.dts = dit_dts_;
    Check(LaunchDitPatch(p, stream_), "persistent DiT patch");
    return;
  }
  for (int i = 0; i < timesteps; ++i) {
    if (!schedule_eval_[i])
      continue;  // zero velocity (CFG-Zero*)
    EvaluateDit(x_, schedule_t_[i], velocity_);
    Check(GuidedEuler(velocity_, x_, values, cfg, schedule_dt_[i], stream_),
          "GuidedEuler");
  }
}

void Generator::PreDit() {
  const ModelConfig& c = config_;
  const int hidden = c.lm.hidden;
  const int dit = c.dit.hidden;
  const int values = c.patch_size * c.feat_dim;
  Check(ToBf16(lm_hidden_, step_bf16_, hidden, false, stream_), "ToBf16");
  Check(Project(w_.lm_to_dit, step_bf16_, mu_, 1, stream_), "lm_to_dit");
  Check(Project(w_.stop_proj, step_bf16_, step_a_, 1, stream_), "stop_proj");
  Check(ToBf16(step_a_, step_bf16_, hidden, true, stream_), "ToBf16");
  Check(Project(w_.stop_head, step_bf16_, stop_, 1, stream_), "stop_head");
  Check(ToBf16(residual_hidden_, step_bf16_, hidden, false, stream_), "ToBf16");
  Check(Project(w_.res_to_dit, step_bf16_, mu_ + dit, 1, stream_), "res_to_dit");
  DitCond();
  CheckCuda(cudaMemcpyAsync(x_, pinned_noise_, values * sizeof(float),
                            cudaMemcpyHostToDevice, stream_),
            "noise");
}

void Generator::PatchOutputs() {
  const int values = config_.patch_size * config_.feat_dim;
  CheckCuda(cudaMemcpyAsync(pinned_latent_, x_, values * sizeof(float),
                            cudaMemcpyDeviceToHost, stream_),
            "latent");
  // The device copy behind latent(): the slot of this patch's position
  // (the device counter still holds it; the LMs advance it afterwards).
  Check(CopyToParitySlot(x_, latent_slots_, values, position_counter_, stream_),
        "latent slot");
  Check(CopyFloats(x_, prefix_cond_, values, stream_), "prefix");
  CheckCuda(cudaMemcpyAsync(pinned_stop_, stop_, 2 * sizeof(float),
                            cudaMemcpyDeviceToHost, stream_),
            "stop");
}

void Generator::AdvanceLms() {
  // One row at the device-held position (its rotary row and cache row
  // coincide).
  const int hidden = config_.lm.hidden;
  AttentionLayout layout;
  layout.positions = step_positions_;
  layout.cache_rows = step_positions_;
  layout.rows_per_sequence = 1;
  layout.past_device = position_counter_;
  layout.max_keys = capacity();
  layout.causal = true;
  Check(CopyFloats(embed_, step_a_, hidden, stream_), "copy");
  StepStack(0, layout, step_a_, step_b_);
  Fsq(step_b_, lm_hidden_, 1);
  Check(ConcatRows(lm_hidden_, nullptr, hidden, embed_, nullptr, hidden,
                   step_bf16_, 1, stream_),
        "ConcatRows");
  Check(Project(w_.fusion, step_bf16_, step_a_, 1, stream_), "fusion");
  StepStack(1, layout, step_a_, residual_hidden_);
  Check(AdvancePosition(position_counter_, step_positions_, stream_),
        "advance");
}

void Generator::StepBody(int timesteps, float cfg) {
  // generator.cpp:424-513, with the host syncs replaced by device state.
  PreDit();
  EulerLoop(timesteps, cfg);
  PatchOutputs();
  // The patch's embedding advances both LMs.
  Encode(x_, 1, embed_);
  AdvanceLms();
}

void Generator::Step(const float* noise, int timesteps, float cfg,
                     float* latent, float* stop_logits) {
  if (position_ <= 0 || position_ >= capacity())
    throw std::logic_error("the generator has no room for a patch");
  const int values = config_.patch_size * config_.feat_dim;
  PrepareTimes(timesteps);
  EnsureEncoder(1);  // sizes the encoder's buffers outside any capture
  std::memcpy(pinned_noise_, noise, values * sizeof(float));
  if (!graphs_) {
    StepBody(timesteps, cfg);
  } else {
    if (step_graph_ == nullptr || step_graph_timesteps_ != timesteps ||
        step_graph_cfg_ != cfg) {
      if (step_graph_ != nullptr) {
        cudaGraphExecDestroy(step_graph_);
        step_graph_ = nullptr;
      }
      cudaGraph_t graph = nullptr;
      CheckCuda(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeRelaxed),
                "capture");
      try {
        StepBody(timesteps, cfg);
      } catch (...) {
        cudaStreamEndCapture(stream_, &graph);
        if (graph != nullptr)
          cudaGraphDestroy(graph);
        throw;
      }
      CheckCuda(cudaStreamEndCapture(stream_, &graph), "end capture");
      const cudaError_t made = cudaGraphInstantiate(&step_graph_, graph, 0);
      cudaGraphDestroy(graph);
      CheckCuda(made, "instantiate step graph");
      step_graph_timesteps_ = timesteps;
      step_graph_cfg_ = cfg;
    }
    CheckCuda(cudaGraphLaunch(step_graph_, stream_), "step graph");
  }
  CheckCuda(cudaEventRecord(latent_event_, stream_), "latent event");
  CheckCuda(cudaStreamSynchronize(stream_), "step");
  if (latent != nullptr)
    std::memcpy(latent, pinned_latent_, values * sizeof(float));
  if (stop_logits != nullptr)
    std::memcpy(stop_logits, pinned_stop_, 2 * sizeof(float));
  ++position_;
  latent_ready_ = true;
}

const float* Generator::latent() const {
  if (!latent_ready_ || position_ < 1)
    return nullptr;
  const int values = config_.patch_size * config_.feat_dim;
  return latent_slots_ + static_cast<std::size_t>((position_ - 1) & 1) * values;
}

void Generator::Velocity(const float* mu, const float* cond, const float* x,
                         float t, float* velocity) {
  // generator.cpp:515-538
  const ModelConfig& c = config_;
  const int values = c.patch_size * c.feat_dim;
  CheckCuda(cudaMemcpyAsync(mu_, mu, 2 * c.dit.hidden * sizeof(float),
                            cudaMemcpyHostToDevice, stream_), "mu");
  CheckCuda(cudaMemcpyAsync(prefix_cond_, cond, values * sizeof(float),
                            cudaMemcpyHostToDevice, stream_), "cond");
  CheckCuda(cudaMemcpyAsync(x_, x, values * sizeof(float),
                            cudaMemcpyHostToDevice, stream_), "x");
  (void)TimeVector(t);
  DitCond();
  EvaluateDit(x_, t, velocity_);
  CheckCuda(cudaMemcpyAsync(velocity, velocity_, 2 * values * sizeof(float),
                            cudaMemcpyDeviceToHost, stream_), "velocity");
  CheckCuda(cudaStreamSynchronize(stream_), "velocity");
}

void Generator::DitPatch(const float* mu, const float* cond,
                         const float* noise, int timesteps, float cfg,
                         float* latent) {
  const ModelConfig& c = config_;
  const int values = c.patch_size * c.feat_dim;
  float* noise_dev = x_ + values;
  CheckCuda(cudaMemcpyAsync(mu_, mu, 2 * c.dit.hidden * sizeof(float),
                            cudaMemcpyHostToDevice, stream_), "mu");
  CheckCuda(cudaMemcpyAsync(prefix_cond_, cond, values * sizeof(float),
                            cudaMemcpyHostToDevice, stream_), "cond");
  CheckCuda(cudaMemcpyAsync(noise_dev, noise, values * sizeof(float),
                            cudaMemcpyHostToDevice, stream_), "noise");
  PrepareTimes(timesteps);
  auto body = [&]() {
    Check(CopyFloats(noise_dev, x_, values, stream_), "copy");
    DitCond();
    EulerLoop(timesteps, cfg);
  };
  if (!graphs_) {
    body();
  } else {
    if (patch_graph_ == nullptr || patch_graph_timesteps_ != timesteps ||
        patch_graph_cfg_ != cfg) {
      if (patch_graph_ != nullptr) {
        cudaGraphExecDestroy(patch_graph_);
        patch_graph_ = nullptr;
      }
      CheckCuda(cudaStreamSynchronize(stream_), "sync");
      cudaGraph_t graph = nullptr;
      CheckCuda(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeRelaxed),
                "capture");
      try {
        body();
      } catch (...) {
        cudaStreamEndCapture(stream_, &graph);
        if (graph != nullptr)
          cudaGraphDestroy(graph);
        throw;
      }
      CheckCuda(cudaStreamEndCapture(stream_, &graph), "end capture");
      const cudaError_t made = cudaGraphInstantiate(&patch_graph_, graph, 0);
      cudaGraphDestroy(graph);
      CheckCuda(made, "instantiate patch graph");
      patch_graph_timesteps_ = timesteps;
      patch_graph_cfg_ = cfg;
    }
    CheckCuda(cudaGraphLaunch(patch_graph_, stream_), "patch graph");
  }
  if (latent != nullptr) {
    CheckCuda(cudaMemcpyAsync(latent, x_, values * sizeof(float),
                              cudaMemcpyDeviceToHost, stream_), "latent");
    CheckCuda(cudaStreamSynchronize(stream_), "patch");
    if (persistent_ && dit_evaluations_ > 0) {
      bool aborted = false;
      Check(DitLaunchAborted(dit_params_, stream_, &aborted),
            "persistent DiT patch");
      if (aborted)
        ThrowAborted("persistent DiT patch");
    }
  }
}

void Generator::DitPatchStatic(const float* mu, const float* cond,
                               const float* noise, int timesteps, float cfg,
                               float* latent) {
  if (!persistent_ok_)
    throw std::logic_error(
        "the allocation-free DiT patch needs the persistent kernel (VoxCPM2's "
        "DiT shape)");
  if (dit_schedule_timesteps_ != timesteps)
    throw std::logic_error(
        "no prepared schedule for these timesteps: run DitPatch or Step once "
        "with them first");
  const ModelConfig& c = config_;
  const int values = c.patch_size * c.feat_dim;
  CheckCuda(cudaMemcpyAsync(mu_, mu, 2 * c.dit.hidden * sizeof(float),
                            cudaMemcpyDeviceToDevice, stream_), "mu");
  CheckCuda(cudaMemcpyAsync(prefix_cond_, cond, values * sizeof(float),
                            cudaMemcpyDeviceToDevice, stream_), "cond");
  CheckCuda(cudaMemcpyAsync(x_, noise, values * sizeof(float),
                            cudaMemcpyDeviceToDevice, stream_), "noise");
  DitCond();
  if (dit_evaluations_ > 0) {
    DitPatchParams p = dit_params_;
    p.cfg = cfg;
    p.evaluations = dit_evaluations_;
    p.time_vectors = dit_times_;
    p.dts = dit_dts_;
    Check(LaunchDitPatchStatic(p, stream_), "allocation-free DiT patch");
  }
  CheckCuda(cudaMemcpyAsync(latent, x_, values * sizeof(float),
                            cudaMemcpyDeviceToDevice, stream_), "latent");
  CheckCuda(cudaStreamSynchronize(stream_), "patch");
  if (dit_evaluations_ > 0) {
    bool aborted = false;
    Check(DitStaticLaunchAborted(stream_, &aborted),
          "allocation-free DiT patch");
    if (aborted)
      ThrowAborted("allocation-free DiT patch");
  }
}

void Generator::ThrowAborted(const char* what) {
  unsigned bits = 0;
  (void)ReadDeviceError(&bits);  // reads and clears the device error word
  throw DeviceTimeout(std::string(what) +
                      ": a bounded device wait gave up and the launch "
                      "aborted (device error bits " +
                      std::to_string(bits) + "); the latent is not valid");
}

void Generator::ReplayDitPatch() {
  if (patch_graph_ == nullptr)
    throw std::logic_error("no captured DiT patch (call DitPatch first)");
  CheckCuda(cudaGraphLaunch(patch_graph_, stream_), "patch graph");
}

void Generator::Prefill(const std::int32_t* tokens,
                        const std::int32_t* text_mask,
                        const std::int32_t* audio_mask, const float* feats,
                        int rows) {
  // generator.cpp:326-422
  const ModelConfig& c = config_;
  const int hidden = c.lm.hidden;
  const int patch_values = c.patch_size * c.feat_dim;
  if (rows <= 0 || rows >= capacity() || tokens == nullptr ||
      text_mask == nullptr || audio_mask == nullptr || feats == nullptr)
    throw std::invalid_argument("malformed VoxCPM2 prompt");
  for (int r = 0; r < rows; ++r)
    if (text_mask[r] != 0 && (tokens[r] < 0 || tokens[r] >= c.vocab))
      throw std::invalid_argument("token outside the vocabulary");
  CheckCuda(cudaStreamSynchronize(stream_), "sync");
  EnsureRows(std::max(rows, scratch_rows_));
  // Work buffers from one grow-only block: an upper bound for this prompt
  // (every row an audio row), then bump allocation.
  auto rounded = [](std::size_t bytes) { return (std::max<std::size_t>(bytes, 4) + 255) / 256 * 256; };
  {
    const std::size_t r = rows;
    const std::size_t bound = 5 * rounded(r * 4) + 5 * rounded(r * hidden * 4) +
                              rounded(r * 2 * hidden * 2) +
                              rounded(r * c.fsq_latent_dim * 4) +
                              rounded(r * patch_values * 4);
    if (bound > prefill_bytes_) {
      if (prefill_block_ != nullptr)
        cudaFree(prefill_block_);
      prefill_block_ = nullptr;
      prefill_bytes_ = 0;
      CheckCuda(cudaMalloc(reinterpret_cast<void**>(&prefill_block_), bound),
                "cudaMalloc prefill");
      prefill_bytes_ = bound;
    }
  }
  std::size_t used = 0;
  auto temp = [&](std::size_t bytes) {
    const std::size_t size = rounded(bytes);
    if (used + size > prefill_bytes_)
      throw std::logic_error("prefill work buffers exceed their bound");
    void* p = prefill_block_ + used;
    used += size;
    return p;
  };
  try {
    const std::size_t r = rows;
    auto* ids = static_cast<std::int32_t*>(temp(r * 4));
    auto* tmask = static_cast<std::int32_t*>(temp(r * 4));
    auto* amask = static_cast<std::int32_t*>(temp(r * 4));
    auto* positions = static_cast<std::int32_t*>(temp(r * 4));
    auto* a = static_cast<float*>(temp(r * hidden * 4));
    auto* b = static_cast<float*>(temp(r * hidden * 4));
    auto* cbuf = static_cast<float*>(temp(r * hidden * 4));
    auto* d = static_cast<float*>(temp(r * hidden * 4));
    auto* bf16 = static_cast<std::uint16_t*>(temp(r * 2 * hidden * 2));
    auto* fsq_latent = static_cast<float*>(temp(r * c.fsq_latent_dim * 4));
    CheckCuda(cudaMemcpy(ids, tokens, r * 4, cudaMemcpyHostToDevice), "upload");
    CheckCuda(cudaMemcpy(tmask, text_mask, r * 4, cudaMemcpyHostToDevice), "upload");
    CheckCuda(cudaMemcpy(amask, audio_mask, r * 4, cudaMemcpyHostToDevice), "upload");
    std::vector<std::int32_t> iota(rows);
    std::iota(iota.begin(), iota.end(), 0);
    CheckCuda(cudaMemcpy(positions, iota.data(), r * 4, cudaMemcpyHostToDevice), "upload");
    if (c.vocab > 0)
      Check(Embed(w_.embed, ids, tmask, a, rows, hidden, 1.0f, stream_), "Embed");
    else
      CheckCuda(cudaMemsetAsync(a, 0, r * hidden * 4, stream_), "memset");
    CheckCuda(cudaMemsetAsync(b, 0, r * hidden * 4, stream_), "memset");
    std::vector<std::int32_t> audio_rows;
    std::vector<float> latents;
    for (int row = 0; row < rows; ++row) {
      if (audio_mask[row] == 0)
        continue;
      audio_rows.push_back(row);
      latents.insert(latents.end(), feats + static_cast<std::size_t>(row) * patch_values,
                     feats + static_cast<std::size_t>(row + 1) * patch_values);
    }
    if (!audio_rows.empty()) {
      const int count = static_cast<int>(audio_rows.size());
      auto* arows = static_cast<std::int32_t*>(temp(count * 4));
      auto* lat = static_cast<float*>(temp(latents.size() * 4));
      auto* emb = static_cast<float*>(temp(static_cast<std::size_t>(count) * hidden * 4));
      CheckCuda(cudaMemcpy(arows, audio_rows.data(), count * 4, cudaMemcpyHostToDevice), "upload");
      CheckCuda(cudaMemcpy(lat, latents.data(), latents.size() * 4, cudaMemcpyHostToDevice), "upload");
      Encode(lat, count, emb);
      Check(ScatterRows(emb, arows, a, count, hidden, stream_), "ScatterRows");
      Check(ScatterRows(emb, arows, b, count, hidden, stream_), "ScatterRows");
    }
    AttentionLayout layout;
    layout.positions = positions;
    layout.cache_rows = positions;
    layout.rows_per_sequence = rows;
    layout.causal = true;
    Check(ForwardStack(w_.base_lm, rope_, layout, base_cache_, a, cbuf, rows,
                       scratch_, stream_),
          "base lm prefill");
    // FSQ of every row, then the audio rows take the quantized values.
    Check(ToBf16(cbuf, bf16, r * hidden, false, stream_), "ToBf16");
    Check(Project(w_.fsq_in, bf16, fsq_latent, rows, stream_), "fsq_in");
    Check(Quantize(fsq_latent, bf16, r * c.fsq_latent_dim, c.fsq_scale, stream_), "Quantize");
    Check(Project(w_.fsq_out, bf16, a, rows, stream_), "fsq_out");
    Check(SelectRows(a, cbuf, amask, d, rows, hidden, stream_), "SelectRows");
    Check(CopyFloats(d + (r - 1) * hidden, lm_hidden_, hidden, stream_), "copy");
    Check(CopyFloats(cbuf + (r - 1) * hidden, step_b_, hidden, stream_), "copy");
    Check(ConcatRows(d, nullptr, hidden, b, nullptr, hidden, bf16, rows, stream_),
          "ConcatRows");
    Check(Project(w_.fusion, bf16, a, rows, stream_), "fusion");
    Check(ForwardStack(w_.residual_lm, nullptr, layout, residual_cache_, a, cbuf,
                       rows, scratch_, stream_),
          "residual lm prefill");
    Check(CopyFloats(cbuf + (r - 1) * hidden, residual_hidden_, hidden, stream_),
          "copy");
    CheckCuda(cudaMemcpyAsync(prefix_cond_, feats + (r - 1) * patch_values,
                              patch_values * 4, cudaMemcpyHostToDevice, stream_),
              "prefix");
    const std::int32_t next = rows;
    CheckCuda(cudaMemcpyAsync(position_counter_, &next, 4, cudaMemcpyHostToDevice, stream_),
              "position");
    CheckCuda(cudaMemcpyAsync(step_positions_, &next, 4, cudaMemcpyHostToDevice, stream_),
              "position");
    CheckCuda(cudaStreamSynchronize(stream_), "prefill");
  } catch (...) {
    cudaStreamSynchronize(stream_);
    throw;
  }
  position_ = rows;
  latent_ready_ = false;
}

namespace {

struct StateBuffer {
  float* data;
  std::size_t count;
};

}  // namespace

void Generator::State(const std::string& name, float* out, std::size_t count) {
  const ModelConfig& c = config_;
  // The LM caches: [layer][kv_head][capacity][head_dim], bf16 widened.
  const KvCache* cache = name == "base_cache_k" || name == "base_cache_v"
                             ? &base_cache_
                             : (name == "residual_cache_k" ||
                                        name == "residual_cache_v"
                                    ? &residual_cache_
                                    : nullptr);
  if (cache != nullptr) {
    const StackConfig& s = cache == &base_cache_ ? c.lm : c.residual_lm;
    const bool keys = name.back() == 'k';
    const std::size_t per_layer = static_cast<std::size_t>(s.kv_heads) *
                                  cache->capacity() * s.head_dim;
    if (count > per_layer * s.layers)
      throw std::invalid_argument("count too large: " + name);
    CheckCuda(cudaStreamSynchronize(stream_), "sync");
    const bool bf16 = cache->type() == CacheType::kBf16;
    std::vector<std::uint16_t> bits(bf16 ? per_layer : 0);
    for (int layer = 0; layer < s.layers && count > 0; ++layer) {
      const std::size_t n = std::min(count, per_layer);
      const void* src = keys ? cache->keys(layer) : cache->values(layer);
      if (bf16) {
        CheckCuda(cudaMemcpy(bits.data(), src, n * 2, cudaMemcpyDeviceToHost),
                  "state");
        for (std::size_t i = 0; i < n; ++i) {
          const std::uint32_t word = static_cast<std::uint32_t>(bits[i]) << 16;
          std::memcpy(out + i, &word, 4);
        }
      } else {
        CheckCuda(cudaMemcpy(out, src, n * 4, cudaMemcpyDeviceToHost), "state");
      }
      out += n;
      count -= n;
    }
    return;
  }
  const std::map<std::string, StateBuffer> buffers = {
      {"lm_hidden", {lm_hidden_, static_cast<std::size_t>(c.lm.hidden)}},
      {"residual_hidden", {residual_hidden_, static_cast<std::size_t>(c.lm.hidden)}},
      {"prefix_cond", {prefix_cond_, static_cast<std::size_t>(c.patch_size * c.feat_dim)}},
      {"x", {x_, static_cast<std::size_t>(c.patch_size * c.feat_dim)}},
      {"mu", {mu_, static_cast<std::size_t>(2 * c.dit.hidden)}},
      {"stop", {stop_, 2}},
      {"embed", {embed_, static_cast<std::size_t>(c.lm.hidden)}},
      {"lm_output", {step_b_, static_cast<std::size_t>(c.lm.hidden)}},
      {"cond_rows", {cond_rows_, static_cast<std::size_t>(c.patch_size * c.dit.hidden)}},
      {"velocity", {velocity_, static_cast<std::size_t>(2 * c.patch_size * c.feat_dim)}},
      {"delta_time", {delta_time_, static_cast<std::size_t>(c.dit.hidden)}},
  };
  const auto it = buffers.find(name);
  if (it == buffers.end() || count > it->second.count)
    throw std::invalid_argument("unknown state or count too large: " + name);
  CheckCuda(cudaStreamSynchronize(stream_), "sync");
  CheckCuda(cudaMemcpy(out, it->second.data, count * 4, cudaMemcpyDeviceToHost),
            "state");
}

void Generator::SetState(const std::string& name, const float* in,
                         std::size_t count) {
  const ModelConfig& c = config_;
  if (name == "position") {
    const auto p = static_cast<std::int32_t>(in[0]);
    if (p < 0 || p >= capacity())
      throw std::invalid_argument("position outside the caches");
    CheckCuda(cudaStreamSynchronize(stream_), "sync");
    CheckCuda(cudaMemcpy(position_counter_, &p, 4, cudaMemcpyHostToDevice), "position");
    CheckCuda(cudaMemcpy(step_positions_, &p, 4, cudaMemcpyHostToDevice), "position");
    position_ = p;
    return;
  }
  const std::map<std::string, StateBuffer> buffers = {
      {"lm_hidden", {lm_hidden_, static_cast<std::size_t>(c.lm.hidden)}},
      {"residual_hidden", {residual_hidden_, static_cast<std::size_t>(c.lm.hidden)}},
      {"prefix_cond", {prefix_cond_, static_cast<std::size_t>(c.patch_size * c.feat_dim)}},
      {"mu", {mu_, static_cast<std::size_t>(2 * c.dit.hidden)}},
  };
  const auto it = buffers.find(name);
  if (it == buffers.end() || count > it->second.count)
    throw std::invalid_argument("unknown state or count too large: " + name);
  CheckCuda(cudaStreamSynchronize(stream_), "sync");
  CheckCuda(cudaMemcpy(it->second.data, in, count * 4, cudaMemcpyHostToDevice),
            "state");
}

}  // namespace vx
