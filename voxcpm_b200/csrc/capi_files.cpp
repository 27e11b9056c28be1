// C ABI of the checkpoint files (include/voxcpm_b200.h): ModelFiles, the
// config.json parser and the load-time bf16 conversions.
#include "convert.cuh"
#include "json.h"
#include "model_files.h"
#include "vx_status.h"

#include "../../include/voxcpm_b200.h"

#include <cmath>
#include <cstring>
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
  using std::runtime_error::runtime_error;
};

/// Typed, named access to one object of config.json; an absent or null key
/// takes the given default (the reference's pydantic defaults,
/// config.cpp:26-133).
class Fields {
 public:
  Fields(const vx::json::Value& object, std::string where)
      : object_(object), where_(std::move(where)) {
    if (!object_.is_object())
      throw ConfigError(where_ + " is not a JSON object");
  }

  const vx::json::Value* Find(const std::string& key) const {
    const vx::json::Value* v = object_.find(key);
    return v == nullptr || v->is_null() ? nullptr : v;
  }
  const vx::json::Value& Get(const std::string& key) const {
    const vx::json::Value* v = Find(key);
    if (v == nullptr)
      throw ConfigError(where_ + " lacks \"" + key + "\"");
    return *v;
  }
  int Size(const std::string& key) const {
    std::uint64_t v = 0;
    if (!Get(key).as_unsigned(&v) || v == 0 || v > (1u << 30))
      throw ConfigError(where_ + "." + key + " is not a positive integer");
    return static_cast<int>(v);
  }
  int Size(const std::string& key, int fallback) const {
    return Find(key) == nullptr ? fallback : Size(key);
  }
  double Number(const std::string& key) const {
    const vx::json::Value& v = Get(key);
    if (!v.is_number() || !std::isfinite(v.as_double()))
      throw ConfigError(where_ + "." + key + " is not a number");
    return v.as_double();
  }
  double Number(const std::string& key, double fallback) const {
    return Find(key) == nullptr ? fallback : Number(key);
  }
  bool Bool(const std::string& key, bool fallback) const {
    const vx::json::Value* v = Find(key);
    if (v == nullptr)
      return fallback;
    if (!v->is_bool())
      throw ConfigError(where_ + "." + key + " is not a boolean");
    return v->as_bool();
  }
  std::string String(const std::string& key, const std::string& fallback) const {
    const vx::json::Value* v = Find(key);
    if (v == nullptr)
      return fallback;
    if (!v->is_string())
      throw ConfigError(where_ + "." + key + " is not a string");
    return v->str();
  }
  std::vector<double> Numbers(const std::string& key) const {
    const vx::json::Value& v = Get(key);
    if (!v.is_array() || v.items().empty())
      throw ConfigError(where_ + "." + key + " is not a non-empty array");
    std::vector<double> out;
    for (const vx::json::Value& item : v.items()) {
      if (!item.is_number() || !std::isfinite(item.as_double()))
        throw ConfigError(where_ + "." + key + " holds a non-number");
      out.push_back(item.as_double());
    }
    return out;
  }
  Fields Object(const std::string& key) const {
    return Fields(Get(key), where_ + "." + key);
  }
  bool Has(const std::string& key) const { return Find(key) != nullptr; }

 private:
  const vx::json::Value& object_;
  std::string where_;
};

/// An encoder / DiT stack: lm_config with the sizes of `fields`
/// (config.cpp:135-147; kv_channels falls back to hidden / heads).
vx_stack_config Derive(const vx_stack_config& lm, const Fields& fields) {
  vx_stack_config s = lm;
  s.hidden = fields.Size("hidden_dim", 1024);
  s.intermediate = fields.Size("ffn_dim", 4096);
  s.heads = fields.Size("num_heads", 16);
  s.layers = fields.Size("num_layers", 4);
  s.head_dim = fields.Size("kv_channels", s.hidden / s.heads);
  return s;
}

/// config.cpp:149-236 (generator fields) and :265-301 (IsSupported).
void ParseConfig(std::string_view text, vx_model_config* out) {
  vx::json::Value root;
  try {
    root = vx::json::Parse(text);
  } catch (const vx::json::Error& failure) {
    throw ConfigError(std::string("config.json: ") + failure.what());
  }
  const Fields config(root, "config.json");
  const std::string architecture = config.String("architecture", "");
  if (architecture != "voxcpm2")
    throw ConfigError("config.json names architecture \"" + architecture +
                      "\", expected \"voxcpm2\"");
  vx_model_config c;
  std::memset(&c, 0, sizeof(c));
  const Fields lm = config.Object("lm_config");
  vx_stack_config& base = c.lm;
  base.hidden = lm.Size("hidden_size");
  base.intermediate = lm.Size("intermediate_size");
  base.layers = lm.Size("num_hidden_layers");
  base.heads = lm.Size("num_attention_heads");
  base.kv_heads = lm.Size("num_key_value_heads");
  base.head_dim = lm.Size("kv_channels", base.hidden / base.heads);
  c.vocab = lm.Size("vocab_size");
  base.rms_eps = static_cast<float>(lm.Number("rms_norm_eps"));
  base.rope = lm.Bool("no_rope", false) ? 0 : 1;
  const bool use_mup = lm.Bool("use_mup", true);
  (void)lm.Number("scale_emb");
  (void)lm.Number("scale_depth");

  const Fields scaling = lm.Object("rope_scaling");
  c.rope_theta = lm.Number("rope_theta");
  const double max_positions = lm.Size("max_position_embeddings");
  const double original = scaling.Size("original_max_position_embeddings");
  const std::vector<double> short_factor = scaling.Numbers("short_factor");
  const std::vector<double> long_factor = scaling.Numbers("long_factor");
  // The factors the reference applies, and the cos/sin magnitude
  // (config.hpp:34-50, config.cpp:238-243).
  const std::vector<double>& factors =
      max_positions > original ? long_factor : short_factor;
  c.rope_scaling =
      std::sqrt(1.0 + std::log(max_positions / original) / std::log(original));

  c.residual_lm = base;
  c.residual_lm.layers = config.Size("residual_lm_num_layers", 8);
  c.residual_lm.rope = config.Bool("residual_lm_no_rope", false) ? 0 : 1;
  c.encoder = Derive(base, config.Object("encoder_config"));
  const Fields dit = config.Object("dit_config");
  c.dit = Derive(base, dit);
  if (dit.Bool("dit_mean_mode", false))
    throw ConfigError("config.json: dit_mean_mode is not supported");
  c.patch_size = config.Size("patch_size", 4);
  c.feat_dim = config.Size("feat_dim", 64);
  c.fsq_latent_dim = config.Size("scalar_quantization_latent_dim", 512);
  c.fsq_scale =
      static_cast<float>(config.Number("scalar_quantization_scale", 9));
  c.max_length = config.Size("max_length", 8192);
  const std::string dtype = config.String("dtype", "bfloat16");
  // Of the AudioVAE's settings only its latent size meets the generator.
  int latent_dim = 64;
  if (config.Has("audio_vae_config"))
    latent_dim = config.Object("audio_vae_config").Size("latent_dim", 64);

  for (const vx_stack_config* s : {&c.lm, &c.residual_lm, &c.encoder, &c.dit}) {
    if (s->head_dim != 128)
      throw ConfigError("the attention kernels need a head size of 128");
    if (s->heads % s->kv_heads != 0)
      throw ConfigError("attention heads must be a multiple of the KV heads");
  }
  if (use_mup)
    throw ConfigError("muP-scaled checkpoints are not supported");
  if (short_factor.size() * 2 != static_cast<std::size_t>(base.head_dim) ||
      long_factor.size() * 2 != static_cast<std::size_t>(base.head_dim))
    throw ConfigError("the LongRoPE factors do not match the head size");
  if (c.feat_dim != latent_dim)
    throw ConfigError("feat_dim differs from the AudioVAE latent size");
  if (dtype != "bfloat16")
    throw ConfigError("only bfloat16 checkpoints are supported");
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
