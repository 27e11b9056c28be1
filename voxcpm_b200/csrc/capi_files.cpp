// C ABI of the checkpoint files (include/voxcpm_b200.h): ModelFiles, the
// config.json parser and the load-time bf16 conversions.
#include "convert.cuh"
#include "json.h"
#include "model_files.h"
#include "vx_status.h"

#include "../../include/voxcpm_b200.h"

#include <cmath>
#include <cstring>
#include <limits>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

struct vx_model_files {
  std::unique_ptr<vx::ModelFiles> impl;
};

namespace {

class ConfigError : public std::runtime_error {
 public:
  explicit ConfigError(const std::string& what)
      : std::runtime_error("config.json: " + what) {}
};

// ------------------------------------------------------------ config.json
//
// The generator's view of an openbmb VoxCPM2 config.json is a table: one row
// per field it reads, with the field's dotted path from the document root,
// the kind of value it must hold and what stands in when the field is absent
// or null. One loop applies the table; a second stage derives the stacks and
// checks the combinations this library serves. The keys and defaults are the
// checkpoint format's (the reference's config.cpp reads the same ones).

enum class Kind { kObject, kCount, kReal, kFlag, kText, kReals };

/// Where a field's value lands.
enum Slot : int {
  kArchitecture, kLm, kLmHidden, kLmFfn, kLmLayers, kLmHeads, kLmKvHeads,
  kLmHeadDim, kVocab, kEps, kNoRope, kUseMup, kScaleEmb, kScaleDepth,
  kScaling, kTheta, kMaxPositions, kOriginalPositions, kShortFactors,
  kLongFactors, kResidualLayers, kResidualNoRope, kEncoder, kEncHidden,
  kEncFfn, kEncHeads, kEncLayers, kEncHeadDim, kDit, kDitHidden, kDitFfn,
  kDitHeads, kDitLayers, kDitHeadDim, kDitMeanMode, kPatch, kFeat, kFsqDim,
  kFsqScale, kMaxLength, kDtype, kVae, kVaeLatent, kSlots
};

/// `fallback` applies when the field is absent or null; a NaN fallback
/// means the field is required; `derived` marks a count whose default is
/// computed from other fields afterwards (left unset here).
struct Row {
  Slot slot;
  const char* path;
  Kind kind;
  double fallback;
  const char* text_fallback = "";
  bool derived = false;
};

constexpr double kRequired = std::numeric_limits<double>::quiet_NaN();

const Row kRows[] = {
    {kArchitecture, "architecture", Kind::kText, 0, ""},
    {kLm, "lm_config", Kind::kObject, kRequired},
    {kLmHidden, "lm_config.hidden_size", Kind::kCount, kRequired},
    {kLmFfn, "lm_config.intermediate_size", Kind::kCount, kRequired},
    {kLmLayers, "lm_config.num_hidden_layers", Kind::kCount, kRequired},
    {kLmHeads, "lm_config.num_attention_heads", Kind::kCount, kRequired},
    {kLmKvHeads, "lm_config.num_key_value_heads", Kind::kCount, kRequired},
    {kLmHeadDim, "lm_config.kv_channels", Kind::kCount, 0, "", true},
    {kVocab, "lm_config.vocab_size", Kind::kCount, kRequired},
    {kEps, "lm_config.rms_norm_eps", Kind::kReal, kRequired},
    {kNoRope, "lm_config.no_rope", Kind::kFlag, 0},
    {kUseMup, "lm_config.use_mup", Kind::kFlag, 1},
    {kScaleEmb, "lm_config.scale_emb", Kind::kReal, kRequired},
    {kScaleDepth, "lm_config.scale_depth", Kind::kReal, kRequired},
    {kScaling, "lm_config.rope_scaling", Kind::kObject, kRequired},
    {kTheta, "lm_config.rope_theta", Kind::kReal, kRequired},
    {kMaxPositions, "lm_config.max_position_embeddings", Kind::kCount,
     kRequired},
    {kOriginalPositions,
     "lm_config.rope_scaling.original_max_position_embeddings", Kind::kCount,
     kRequired},
    {kShortFactors, "lm_config.rope_scaling.short_factor", Kind::kReals,
     kRequired},
    {kLongFactors, "lm_config.rope_scaling.long_factor", Kind::kReals,
     kRequired},
    {kResidualLayers, "residual_lm_num_layers", Kind::kCount, 8},
    {kResidualNoRope, "residual_lm_no_rope", Kind::kFlag, 0},
    {kEncoder, "encoder_config", Kind::kObject, kRequired},
    {kEncHidden, "encoder_config.hidden_dim", Kind::kCount, 1024},
    {kEncFfn, "encoder_config.ffn_dim", Kind::kCount, 4096},
    {kEncHeads, "encoder_config.num_heads", Kind::kCount, 16},
    {kEncLayers, "encoder_config.num_layers", Kind::kCount, 4},
    {kEncHeadDim, "encoder_config.kv_channels", Kind::kCount, 0, "", true},
    {kDit, "dit_config", Kind::kObject, kRequired},
    {kDitHidden, "dit_config.hidden_dim", Kind::kCount, 1024},
    {kDitFfn, "dit_config.ffn_dim", Kind::kCount, 4096},
    {kDitHeads, "dit_config.num_heads", Kind::kCount, 16},
    {kDitLayers, "dit_config.num_layers", Kind::kCount, 4},
    {kDitHeadDim, "dit_config.kv_channels", Kind::kCount, 0, "", true},
    {kDitMeanMode, "dit_config.dit_mean_mode", Kind::kFlag, 0},
    {kPatch, "patch_size", Kind::kCount, 4},
    {kFeat, "feat_dim", Kind::kCount, 64},
    {kFsqDim, "scalar_quantization_latent_dim", Kind::kCount, 512},
    {kFsqScale, "scalar_quantization_scale", Kind::kReal, 9},
    {kMaxLength, "max_length", Kind::kCount, 8192},
    {kDtype, "dtype", Kind::kText, 0, "bfloat16"},
    // Of the AudioVAE's settings only its latent size meets the generator.
    {kVae, "audio_vae_config", Kind::kObject, 0},
    {kVaeLatent, "audio_vae_config.latent_dim", Kind::kCount, 64},
};

/// The table's values after the loop: numbers (counts, reals and flags),
/// texts, lists of reals, and whether a derived count was given.
struct Values {
  double number[kSlots] = {};
  bool given[kSlots] = {};
  std::string text[kSlots];
  std::vector<double> reals[kSlots];
};

const char* Describe(Kind kind) {
  switch (kind) {
    case Kind::kObject: return "an object";
    case Kind::kCount: return "a whole number from 1 to 2^30";
    case Kind::kReal: return "a finite number";
    case Kind::kFlag: return "true or false";
    case Kind::kText: return "a string";
    case Kind::kReals: return "a list of one or more finite numbers";
  }
  return "?";
}

/// The value at the dotted `path`, or null when it (or an object on the way)
/// is absent or null.
const vx::json::Value* Lookup(const vx::json::Value& root,
                              const std::string& path) {
  const vx::json::Value* node = &root;
  std::size_t at = 0;
  while (node != nullptr) {
    const std::size_t dot = path.find('.', at);
    const std::string key = path.substr(at, dot - at);
    node = node->is_object() ? node->find(key) : nullptr;
    if (node != nullptr && node->is_null())
      node = nullptr;
    if (dot == std::string::npos)
      break;
    at = dot + 1;
  }
  return node;
}

/// Applies one row: checks the value's kind and stores it, or stores the
/// fallback.
void Apply(const Row& row, const vx::json::Value* v, Values& out) {
  const std::string path = row.path;
  if (v == nullptr) {
    if (std::isnan(row.fallback))
      throw ConfigError(path + " is missing (it has no default)");
    out.number[row.slot] = row.fallback;
    out.text[row.slot] = row.text_fallback;
    return;
  }
  auto wrong = [&]() {
    return ConfigError(path + " must be " + Describe(row.kind));
  };
  out.given[row.slot] = true;
  switch (row.kind) {
    case Kind::kObject:
      if (!v->is_object())
        throw wrong();
      return;
    case Kind::kCount: {
      std::uint64_t n = 0;
      if (!v->as_unsigned(&n) || n == 0 || n > (1u << 30))
        throw wrong();
      out.number[row.slot] = static_cast<double>(n);
      return;
    }
    case Kind::kReal:
      if (!v->is_number() || !std::isfinite(v->as_double()))
        throw wrong();
      out.number[row.slot] = v->as_double();
      return;
    case Kind::kFlag:
      if (!v->is_bool())
        throw wrong();
      out.number[row.slot] = v->as_bool() ? 1 : 0;
      return;
    case Kind::kText:
      if (!v->is_string())
        throw wrong();
      out.text[row.slot] = v->str();
      return;
    case Kind::kReals:
      if (!v->is_array() || v->items().empty())
        throw wrong();
      for (const vx::json::Value& item : v->items()) {
        if (!item.is_number() || !std::isfinite(item.as_double()))
          throw wrong();
        out.reals[row.slot].push_back(item.as_double());
      }
      return;
  }
}

/// One stack from its hidden, FFN, head, layer and head-size slots; the KV
/// heads, norm epsilon and rotary flag are the LM's (the derived stacks
/// share them); an absent head size is hidden / heads.
vx_stack_config StackOf(const Values& v, Slot hidden, Slot ffn, Slot heads,
                        Slot layers, Slot head_dim) {
  vx_stack_config s = {};
  auto count = [&](Slot slot) { return static_cast<int>(v.number[slot]); };
  s.hidden = count(hidden);
  s.intermediate = count(ffn);
  s.heads = count(heads);
  s.layers = count(layers);
  s.head_dim = v.given[head_dim] ? count(head_dim) : s.hidden / s.heads;
  s.kv_heads = count(kLmKvHeads);
  s.rms_eps = static_cast<float>(v.number[kEps]);
  s.rope = v.number[kNoRope] != 0 ? 0 : 1;
  return s;
}

/// openbmb config.json -> the generator's configuration (the fields the
/// reference's config.cpp:149-236 reads, and the checks of its
/// IsSupported, :265-301, for what this library serves).
void ParseConfig(std::string_view document, vx_model_config* out) {
  vx::json::Value root;
  try {
    root = vx::json::Parse(document);
  } catch (const vx::json::Error& failure) {
    throw ConfigError(std::string("not valid JSON (") + failure.what() + ")");
  }
  if (!root.is_object())
    throw ConfigError("the document must be a JSON object");
  Values v;
  for (const Row& row : kRows)
    Apply(row, Lookup(root, row.path), v);

  if (v.text[kArchitecture] != "voxcpm2")
    throw ConfigError("architecture is \"" + v.text[kArchitecture] +
                      "\"; this library loads \"voxcpm2\" checkpoints");
  vx_model_config c;
  std::memset(&c, 0, sizeof(c));
  c.lm = StackOf(v, kLmHidden, kLmFfn, kLmHeads, kLmLayers, kLmHeadDim);
  c.residual_lm = c.lm;
  c.residual_lm.layers = static_cast<int>(v.number[kResidualLayers]);
  c.residual_lm.rope = v.number[kResidualNoRope] != 0 ? 0 : 1;
  c.encoder =
      StackOf(v, kEncHidden, kEncFfn, kEncHeads, kEncLayers, kEncHeadDim);
  c.dit = StackOf(v, kDitHidden, kDitFfn, kDitHeads, kDitLayers, kDitHeadDim);
  c.vocab = static_cast<int>(v.number[kVocab]);
  c.patch_size = static_cast<int>(v.number[kPatch]);
  c.feat_dim = static_cast<int>(v.number[kFeat]);
  c.fsq_latent_dim = static_cast<int>(v.number[kFsqDim]);
  c.fsq_scale = static_cast<float>(v.number[kFsqScale]);
  c.max_length = static_cast<int>(v.number[kMaxLength]);
  c.rope_theta = v.number[kTheta];
  // LongRoPE: the long factors once the trained length exceeds the original
  // one, and the cos/sin magnitude sqrt(1 + ln(scale) / ln(original))
  // (config.hpp:34-50, config.cpp:238-243).
  const double trained = v.number[kMaxPositions];
  const double original = v.number[kOriginalPositions];
  const std::vector<double>& factors =
      trained > original ? v.reals[kLongFactors] : v.reals[kShortFactors];
  c.rope_scaling =
      std::sqrt(1.0 + std::log(trained / original) / std::log(original));

  // What the kernels and the generator serve.
  if (v.number[kDitMeanMode] != 0)
    throw ConfigError(
        "dit_config.dit_mean_mode is set; the DiT's mean mode is not "
        "implemented");
  for (const vx_stack_config* s : {&c.lm, &c.residual_lm, &c.encoder, &c.dit}) {
    if (s->head_dim != 128)
      throw ConfigError(
          "every stack needs attention heads of 128 values (head size of "
          "128, the attention kernels' width); got " +
          std::to_string(s->head_dim));
    if (s->heads % s->kv_heads != 0)
      throw ConfigError(
          "the query heads must split into equal groups per KV head (a "
          "multiple of the KV heads)");
  }
  if (v.number[kUseMup] != 0)
    throw ConfigError(
        "lm_config.use_mup is on (or absent); muP-scaled checkpoints are not "
        "supported");
  const std::size_t pairs = static_cast<std::size_t>(c.lm.head_dim) / 2;
  if (v.reals[kShortFactors].size() != pairs ||
      v.reals[kLongFactors].size() != pairs)
    throw ConfigError(
        "rope_scaling needs one LongRoPE factor per rotary pair (head size / "
        "2 of them)");
  if (c.feat_dim != static_cast<int>(v.number[kVaeLatent]))
    throw ConfigError(
        "feat_dim must equal the AudioVAE's latent_dim (its latent size)");
  if (v.text[kDtype] != "bfloat16")
    throw ConfigError("dtype is \"" + v.text[kDtype] +
                      "\"; only bfloat16 checkpoints are supported");
  for (std::size_t i = 0; i < 64; ++i)
    c.rope_factors[i] = i < factors.size() ? factors[i] : 1.0;
  *out = c;
}

bool Fill(const vx::Tensor& t, vx_tensor_info* info) {
  if (t.shape.size() > 8)
    return false;
  std::memset(info, 0, sizeof(*info));
  info->name = t.name.c_str();
  info->dtype = static_cast<int>(t.dtype);
  info->rank = static_cast<int>(t.shape.size());
  for (std::size_t i = 0; i < t.shape.size(); ++i)
    info->shape[i] = t.shape[i];
  info->data = t.data;
  info->bytes = t.bytes;
  info->offset = t.offset;
  return true;
}

const std::vector<vx::Tensor>* Component(const vx_model_files* files,
                                         int component) {
  if (files == nullptr || !files->impl)
    return nullptr;
  if (component == VX_COMPONENT_MODEL)
    return &files->impl->model_tensors();
  if (component == VX_COMPONENT_VAE)
    return &files->impl->vae_tensors();
  return nullptr;
}

}  // namespace

extern "C" {

vx_model_files* vx_model_files_open(const char* path) {
  if (path == nullptr) {
    vx::Fail(vx::kInvalid, "vx_model_files_open: null path");
    return nullptr;
  }
  std::string error;
  auto impl = vx::ModelFiles::Open(path, &error);
  if (!impl) {
    vx::Fail(vx::kInvalid, "vx_model_files_open: " + error);
    return nullptr;
  }
  return new vx_model_files{std::move(impl)};
}

void vx_model_files_close(vx_model_files* files) { delete files; }

int vx_model_files_is_voxcpm2_gguf(const char* path) {
  return path != nullptr && vx::ModelFiles::IsVoxCpm2Gguf(path) ? 1 : 0;
}

int vx_model_files_is_gguf(const vx_model_files* files) {
  return files != nullptr && files->impl && files->impl->gguf() ? 1 : 0;
}

const char* vx_model_files_config(const vx_model_files* files) {
  return files != nullptr && files->impl ? files->impl->config().c_str() : nullptr;
}

const char* vx_model_files_tokenizer(const vx_model_files* files) {
  return files != nullptr && files->impl ? files->impl->tokenizer().c_str()
                                         : nullptr;
}

size_t vx_model_files_count(const vx_model_files* files, int component) {
  const auto* tensors = Component(files, component);
  return tensors == nullptr ? 0 : tensors->size();
}

vx_status vx_model_files_tensor(const vx_model_files* files, int component,
                                size_t index, vx_tensor_info* info) {
  const auto* tensors = Component(files, component);
  if (tensors == nullptr || info == nullptr || index >= tensors->size())
    return vx::Fail(vx::kInvalid, "vx_model_files_tensor: bad arguments");
  if (!Fill((*tensors)[index], info))
    return vx::Fail(vx::kUnsupported, "vx_model_files_tensor: rank above 8");
  return vx::kOk;
}

vx_status vx_model_files_find(const vx_model_files* files, int component,
                              const char* name, vx_tensor_info* info) {
  if (Component(files, component) == nullptr || name == nullptr ||
      info == nullptr)
    return vx::Fail(vx::kInvalid, "vx_model_files_find: bad arguments");
  const vx::Tensor* t = component == VX_COMPONENT_MODEL
                            ? files->impl->Model(name)
                            : files->impl->Vae(name);
  if (t == nullptr)
    return vx::Fail(vx::kInvalid,
                    std::string("vx_model_files_find: no tensor ") + name);
  if (!Fill(*t, info))
    return vx::Fail(vx::kUnsupported, "vx_model_files_find: rank above 8");
  return vx::kOk;
}

vx_status vx_parse_config(const char* json, size_t length,
                          vx_model_config* config) {
  if (json == nullptr || config == nullptr)
    return vx::Fail(vx::kInvalid, "vx_parse_config: null argument");
  try {
    ParseConfig(std::string_view(json, length), config);
  } catch (const std::exception& failure) {
    return vx::Fail(vx::kInvalid, std::string("vx_parse_config: ") +
                                      failure.what());
  }
  return vx::kOk;
}

vx_status vx_half_to_bf16(const uint16_t* input, uint16_t* output,
                          size_t count, cudaStream_t stream) {
  return vx::Checked(vx::HalfToBf16(input, output, count, stream),
                     "vx_half_to_bf16");
}

vx_status vx_float_to_bf16(const float* input, uint16_t* output, size_t count,
                           cudaStream_t stream) {
  return vx::Checked(vx::FloatToBf16(input, output, count, stream),
                     "vx_float_to_bf16");
}

vx_status vx_q8_0_to_bf16(const uint8_t* blocks, uint16_t* output,
                          size_t count, cudaStream_t stream) {
  return vx::Checked(vx::Q8_0ToBf16(blocks, output, count, stream),
                     "vx_q8_0_to_bf16");
}

}  // extern "C"

namespace vx {

const ModelFiles* FilesOf(const vx_model_files* files) {
  return files != nullptr ? files->impl.get() : nullptr;
}

}  // namespace vx
