// C ABI of the generator (include/voxcpm_b200.h): configuration, creation,
// prefill, step, the DiT patch and state access. Exceptions of the model
// layer become status codes with the thread's last error message.
#include "model.cuh"
#include "model_files.h"
#include "vx_status.h"

#include "../../include/voxcpm_b200.h"

#include <exception>
#include <stdexcept>
#include <string>

struct vx_generator {
  std::unique_ptr<vx::Generator> impl;
};

struct vx_generator_batch {
  std::unique_ptr<vx::GeneratorBatch> impl;
};

namespace {

vx::StackConfig FromC(const vx_stack_config& s) {
  vx::StackConfig c;
  c.hidden = s.hidden;
  c.intermediate = s.intermediate;
  c.layers = s.layers;
  c.heads = s.heads;
  c.kv_heads = s.kv_heads;
  c.head_dim = s.head_dim;
  c.rms_eps = s.rms_eps;
  c.rope = s.rope != 0;
  return c;
}

vx_stack_config ToC(const vx::StackConfig& c) {
  vx_stack_config s;
  s.hidden = c.hidden;
  s.intermediate = c.intermediate;
  s.layers = c.layers;
  s.heads = c.heads;
  s.kv_heads = c.kv_heads;
  s.head_dim = c.head_dim;
  s.rms_eps = c.rms_eps;
  s.rope = c.rope ? 1 : 0;
  return s;
}

template <typename F>
vx_status Guard(vx_generator* g, const char* what, F&& body) {
  if (g == nullptr || !g->impl)
    return vx::Fail(vx::kInvalid, std::string(what) + ": null generator");
  try {
    body(*g->impl);
  } catch (const vx::DeviceTimeout& e) {
    return vx::Fail(vx::kDeviceTimeout, std::string(what) + ": " + e.what());
  } catch (const std::invalid_argument& e) {
    return vx::Fail(vx::kInvalid, std::string(what) + ": " + e.what());
  } catch (const std::logic_error& e) {
    return vx::Fail(vx::kInvalid, std::string(what) + ": " + e.what());
  } catch (const std::exception& e) {
    return vx::Fail(vx::kCudaError, std::string(what) + ": " + e.what());
  }
  return vx::kOk;
}

}  // namespace

namespace {

/// The C configuration as the model layer's; false (with the thread's error
/// set) when the head size is out of range.
bool ToModelConfig(const vx_model_config& config, vx::ModelConfig* out,
                   const char* what) {
  vx::ModelConfig c;
  c.lm = FromC(config.lm);
  c.residual_lm = FromC(config.residual_lm);
  c.encoder = FromC(config.encoder);
  c.dit = FromC(config.dit);
  c.rope_theta = config.rope_theta;
  c.rope_scaling = config.rope_scaling;
  const int half = config.lm.head_dim / 2;
  if (half <= 0 || half > 64) {
    vx::Fail(vx::kInvalid, std::string(what) + ": head_dim must be in 2..128");
    return false;
  }
  c.rope_factors.assign(config.rope_factors, config.rope_factors + half);
  c.patch_size = config.patch_size;
  c.feat_dim = config.feat_dim;
  c.fsq_latent_dim = config.fsq_latent_dim;
  c.fsq_scale = config.fsq_scale;
  c.max_length = config.max_length;
  c.vocab = config.vocab;
  *out = std::move(c);
  return true;
}

template <typename F>
vx_status BatchGuard(vx_generator_batch* b, const char* what, F&& body) {
  if (b == nullptr || !b->impl)
    return vx::Fail(vx::kInvalid, std::string(what) + ": null batch");
  try {
    body(*b->impl);
  } catch (const std::logic_error& e) {
    return vx::Fail(vx::kInvalid, std::string(what) + ": " + e.what());
  } catch (const std::exception& e) {
    return vx::Fail(vx::kCudaError, std::string(what) + ": " + e.what());
  }
  return vx::kOk;
}

vx_generator_batch* CreateBatch(const vx_model_config* config, uint64_t seed,
                                int checkpoint, int cache_type, size_t slots,
                                const vx_model_files* files, const char* what) {
  if (config == nullptr || slots == 0 || slots > 64 ||
      (checkpoint != VX_CHECKPOINT_Q8 && checkpoint != VX_CHECKPOINT_BF16) ||
      (cache_type != VX_CACHE_F32 && cache_type != VX_CACHE_BF16)) {
    vx::Fail(vx::kInvalid, std::string(what) + ": bad arguments");
    return nullptr;
  }
  vx::ModelConfig c;
  if (!ToModelConfig(*config, &c, what))
    return nullptr;
  std::string error;
  auto impl = vx::GeneratorBatch::Create(
      c, seed, static_cast<vx::CheckpointKind>(checkpoint),
      cache_type == VX_CACHE_BF16 ? vx::CacheType::kBf16 : vx::CacheType::kF32,
      static_cast<int>(slots), &error, vx::FilesOf(files));
  if (!impl) {
    vx::Fail(vx::kCudaError, std::string(what) + ": " + error);
    return nullptr;
  }
  return new vx_generator_batch{std::move(impl)};
}

vx_generator* Create(const vx_model_config* config, uint64_t seed,
                     int checkpoint, int cache_type,
                     const vx_model_files* files, const char* what) {
  if (config == nullptr ||
      (checkpoint != VX_CHECKPOINT_Q8 && checkpoint != VX_CHECKPOINT_BF16) ||
      (cache_type != VX_CACHE_F32 && cache_type != VX_CACHE_BF16)) {
    vx::Fail(vx::kInvalid, std::string(what) + ": bad arguments");
    return nullptr;
  }
  vx::ModelConfig c;
  if (!ToModelConfig(*config, &c, what))
    return nullptr;
  std::string error;
  auto impl = vx::Generator::Create(
      c, seed, static_cast<vx::CheckpointKind>(checkpoint),
      cache_type == VX_CACHE_BF16 ? vx::CacheType::kBf16 : vx::CacheType::kF32,
      &error, vx::FilesOf(files));
  if (!impl) {
    vx::Fail(vx::kCudaError, std::string(what) + ": " + error);
    return nullptr;
  }
  return new vx_generator{std::move(impl)};
}

}  // namespace

extern "C" {

void vx_model_config_released(vx_model_config* config) {
  if (config == nullptr)
    return;
  const vx::ModelConfig c = vx::ReleasedConfig();
  config->lm = ToC(c.lm);
  config->residual_lm = ToC(c.residual_lm);
  config->encoder = ToC(c.encoder);
  config->dit = ToC(c.dit);
  config->rope_theta = c.rope_theta;
  config->rope_scaling = c.rope_scaling;
  for (int i = 0; i < 64; ++i)
    config->rope_factors[i] = i < static_cast<int>(c.rope_factors.size())
                                  ? c.rope_factors[i]
                                  : 1.0;
  config->patch_size = c.patch_size;
  config->feat_dim = c.feat_dim;
  config->fsq_latent_dim = c.fsq_latent_dim;
  config->fsq_scale = c.fsq_scale;
  config->max_length = c.max_length;
  config->vocab = c.vocab;
}

vx_generator* vx_generator_create(const vx_model_config* config, uint64_t seed,
                                  int checkpoint, int cache_type) {
  return Create(config, seed, checkpoint, cache_type, nullptr,
                "vx_generator_create");
}

vx_generator* vx_generator_create_from_files(const vx_model_config* config,
                                             const vx_model_files* files,
                                             int cache_type) {
  if (vx::FilesOf(files) == nullptr) {
    vx::Fail(vx::kInvalid, "vx_generator_create_from_files: null files");
    return nullptr;
  }
  return Create(config, 0, VX_CHECKPOINT_Q8, cache_type, files,
                "vx_generator_create_from_files");
}

void vx_generator_destroy(vx_generator* generator) { delete generator; }

vx_status vx_generator_prefill(vx_generator* generator, const int32_t* tokens,
                               const int32_t* text_mask,
                               const int32_t* audio_mask, const float* feats,
                               size_t rows) {
  return Guard(generator, "vx_generator_prefill", [&](vx::Generator& g) {
    g.Prefill(tokens, text_mask, audio_mask, feats, static_cast<int>(rows));
  });
}

vx_status vx_generator_step(vx_generator* generator, const float* noise,
                            size_t timesteps, float cfg, float* latent,
                            float* stop_logits) {
  return Guard(generator, "vx_generator_step", [&](vx::Generator& g) {
    if (noise == nullptr || timesteps == 0)
      throw std::invalid_argument("noise and timesteps are required");
    g.Step(noise, static_cast<int>(timesteps), cfg, latent, stop_logits);
  });
}

vx_status vx_generator_velocity(vx_generator* generator, const float* mu,
                                const float* cond, const float* x, float t,
                                float* velocity) {
  return Guard(generator, "vx_generator_velocity", [&](vx::Generator& g) {
    if (mu == nullptr || cond == nullptr || x == nullptr || velocity == nullptr)
      throw std::invalid_argument("null array");
    g.Velocity(mu, cond, x, t, velocity);
  });
}

vx_status vx_generator_dit_patch(vx_generator* generator, const float* mu,
                                 const float* cond, const float* noise,
                                 size_t timesteps, float cfg, float* latent) {
  return Guard(generator, "vx_generator_dit_patch", [&](vx::Generator& g) {
    if (mu == nullptr || cond == nullptr || noise == nullptr || timesteps == 0)
      throw std::invalid_argument("null array or no timesteps");
    g.DitPatch(mu, cond, noise, static_cast<int>(timesteps), cfg, latent);
  });
}

vx_status vx_generator_dit_patch_static(vx_generator* generator,
                                        const float* mu, const float* cond,
                                        const float* noise, size_t timesteps,
                                        float cfg, float* latent) {
  return Guard(generator, "vx_generator_dit_patch_static",
               [&](vx::Generator& g) {
                 if (mu == nullptr || cond == nullptr || noise == nullptr ||
                     latent == nullptr || timesteps == 0)
                   throw std::invalid_argument("null array or no timesteps");
                 g.DitPatchStatic(mu, cond, noise, static_cast<int>(timesteps),
                                  cfg, latent);
               });
}

void vx_set_dit_stall_for_tests(uint64_t limit_ns) {
  vx::SetDitStall(limit_ns);
}

void vx_set_persistent_max_ctas(size_t ctas) {
  vx::SetPersistentMaxCtas(ctas > 4096 ? 4096 : static_cast<int>(ctas));
}

void vx_set_persistent_cooperative(int enabled) {
  vx::SetPersistentCooperative(enabled != 0);
}

vx_status vx_generator_replay_dit_patch(vx_generator* generator) {
  return Guard(generator, "vx_generator_replay_dit_patch",
               [&](vx::Generator& g) { g.ReplayDitPatch(); });
}

vx_status vx_generator_state(vx_generator* generator, const char* name,
                             float* out, size_t count) {
  return Guard(generator, "vx_generator_state", [&](vx::Generator& g) {
    if (name == nullptr || out == nullptr)
      throw std::invalid_argument("null argument");
    g.State(name, out, count);
  });
}

vx_status vx_generator_set_state(vx_generator* generator, const char* name,
                                 const float* in, size_t count) {
  return Guard(generator, "vx_generator_set_state", [&](vx::Generator& g) {
    if (name == nullptr || in == nullptr)
      throw std::invalid_argument("null argument");
    g.SetState(name, in, count);
  });
}

vx_status vx_generator_set_graphs(vx_generator* generator, int enabled) {
  return Guard(generator, "vx_generator_set_graphs",
               [&](vx::Generator& g) { g.set_graphs(enabled != 0); });
}

vx_status vx_generator_set_persistent(vx_generator* generator, int enabled) {
  bool served = true;
  const vx_status status =
      Guard(generator, "vx_generator_set_persistent",
            [&](vx::Generator& g) { served = g.set_persistent(enabled != 0); });
  if (status == vx::kOk && !served)
    return vx::Fail(vx::kUnsupported,
                    "vx_generator_set_persistent: the DiT does not have the "
                    "shape the persistent kernel serves");
  return status;
}

int vx_generator_persistent(const vx_generator* generator) {
  return generator != nullptr && generator->impl &&
                 generator->impl->persistent()
             ? 1
             : 0;
}

size_t vx_generator_position(const vx_generator* generator) {
  return generator != nullptr && generator->impl
             ? static_cast<size_t>(generator->impl->position())
             : 0;
}

const float* vx_generator_latent(const vx_generator* generator) {
  return generator != nullptr && generator->impl ? generator->impl->latent()
                                                 : nullptr;
}

cudaEvent_t vx_generator_latent_event(const vx_generator* generator) {
  return generator != nullptr && generator->impl
             ? generator->impl->latent_event()
             : nullptr;
}

size_t vx_generator_weight_bytes(const vx_generator* generator) {
  return generator != nullptr && generator->impl
             ? generator->impl->weight_bytes()
             : 0;
}

cudaStream_t vx_generator_stream(const vx_generator* generator) {
  return generator != nullptr && generator->impl ? generator->impl->stream()
                                                 : nullptr;
}

vx_generator_batch* vx_generator_batch_create(const vx_model_config* config,
                                              uint64_t seed, int checkpoint,
                                              int cache_type, size_t slots) {
  return CreateBatch(config, seed, checkpoint, cache_type, slots, nullptr,
                     "vx_generator_batch_create");
}

vx_generator_batch* vx_generator_batch_create_from_files(
    const vx_model_config* config, const vx_model_files* files, int cache_type,
    size_t slots) {
  if (vx::FilesOf(files) == nullptr) {
    vx::Fail(vx::kInvalid, "vx_generator_batch_create_from_files: null files");
    return nullptr;
  }
  return CreateBatch(config, 0, VX_CHECKPOINT_Q8, cache_type, slots, files,
                     "vx_generator_batch_create_from_files");
}

void vx_generator_batch_destroy(vx_generator_batch* batch) { delete batch; }

size_t vx_generator_batch_slots(const vx_generator_batch* batch) {
  return batch != nullptr && batch->impl ? batch->impl->slots() : 0;
}

vx_status vx_generator_batch_prefill(vx_generator_batch* batch, size_t slot,
                                     const int32_t* tokens,
                                     const int32_t* text_mask,
                                     const int32_t* audio_mask,
                                     const float* feats, size_t rows) {
  return BatchGuard(batch, "vx_generator_batch_prefill", [&](vx::GeneratorBatch& b) {
    if (slot >= static_cast<size_t>(b.slots()))
      throw std::invalid_argument("no such slot");
    b.slot(static_cast<int>(slot)).Prefill(tokens, text_mask, audio_mask, feats,
                                           static_cast<int>(rows));
  });
}

vx_status vx_generator_batch_step(vx_generator_batch* batch,
                                  const int32_t* active, const float* noise,
                                  size_t timesteps, float cfg, float* latents,
                                  float* stop_logits) {
  return BatchGuard(batch, "vx_generator_batch_step", [&](vx::GeneratorBatch& b) {
    b.Step(active, noise, static_cast<int>(timesteps), cfg, latents, stop_logits);
  });
}

size_t vx_generator_batch_position(const vx_generator_batch* batch,
                                   size_t slot) {
  if (batch == nullptr || !batch->impl ||
      slot >= static_cast<size_t>(batch->impl->slots()))
    return 0;
  return static_cast<size_t>(batch->impl->slot(static_cast<int>(slot)).position());
}

vx_status vx_generator_batch_state(vx_generator_batch* batch, size_t slot,
                                   const char* name, float* out, size_t count) {
  return BatchGuard(batch, "vx_generator_batch_state", [&](vx::GeneratorBatch& b) {
    if (slot >= static_cast<size_t>(b.slots()) || name == nullptr || out == nullptr)
      throw std::invalid_argument("bad argument");
    b.slot(static_cast<int>(slot)).State(name, out, count);
  });
}

vx_status vx_generator_batch_set_graphs(vx_generator_batch* batch, int enabled) {
  return BatchGuard(batch, "vx_generator_batch_set_graphs", [&](vx::GeneratorBatch& b) {
    b.set_graphs(enabled != 0);
  });
}

cudaStream_t vx_generator_batch_stream(const vx_generator_batch* batch) {
  return batch != nullptr && batch->impl ? batch->impl->stream() : nullptr;
}

}  // extern "C"
