// GeneratorBatch (model.cuh): several requests per GPU sharing one set of
// weights, with the DiT of all active requests run as one pass per Euler
// evaluation and their local encoder as one call.
//
// Per step, for n active slots (the reference runs this once per request,
// generator.cpp:424-513):
//   each slot: stop logits, mu, DiT conditioning, noise (Generator::PreDit)
//   gather mu, cond and x of the n slots into the batch's rows
//   per evaluation: dit_in over 4n rows, AssembleDit per slot into 22n rows,
//     the DiT stack over 22n rows (2n sequences of 11, non-causal),
//     the 8n output rows, dit_out, GuidedEuler per slot
//   scatter the latents; each slot's outputs (Generator::PatchOutputs)
//   the local encoder over the n patches (5n rows, n sequences)
//   both LMs advanced for all n slots as one pass of n rows: the slots' LM
//   caches are slot-major ([layer][slot][kv_head][position][128]), so row i
//   writes and reads slot s_i's cache through a cache row of
//   s_i * kv_heads * positions + position and a first key row of
//   s_i * kv_heads * positions, with its own past length
// The products of 22n rows read each DiT weight once per evaluation for all
// n requests (rows beyond 128 in chunks of 32), and the LM's weights are read
// once per step for all n requests.
#include "model.cuh"
#include "vx_status.h"

#include <algorithm>
#include <cstring>
#include <stdexcept>

namespace vx {

namespace {

void Cuda(cudaError_t error, const char* what) {
  if (error != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(error));
}

void Ok(int status, const char* what) {
  if (status != kOk) {
    const cudaError_t error = cudaGetLastError();
    throw std::runtime_error(std::string(what) + ": status " +
                             std::to_string(status) +
                             (error != cudaSuccess
                                  ? std::string(" (") + cudaGetErrorString(error) + ")"
                                  : std::string()));
  }
}

/// The active slots of a step: their position counters and slot indices
/// (kernel arguments, so a captured graph keeps its own list).
struct SlotPositions {
  int count;
  int stride;  // cache rows per slot: kv_heads * positions
  const std::int32_t* counter[64];
  int slot[64];
};

__global__ void GatherPositionsKernel(const SlotPositions a,
                                      std::int32_t* past,
                                      std::int32_t* cache_rows,
                                      std::int32_t* first_keys) {
  const int i = static_cast<int>(threadIdx.x);
  if (i < a.count) {
    const std::int32_t position = *a.counter[i];
    past[i] = position;
    first_keys[i] = a.slot[i] * a.stride;
    cache_rows[i] = a.slot[i] * a.stride + position;
  }
}

}  // namespace

std::unique_ptr<GeneratorBatch> GeneratorBatch::Create(
    const ModelConfig& config, std::uint64_t seed, CheckpointKind kind,
    CacheType cache_type, int slots, std::string* error,
    const ModelFiles* files) {
  std::unique_ptr<GeneratorBatch> b(new GeneratorBatch());
  try {
    if (slots < 1 || slots > 64)
      throw std::invalid_argument("a batch holds 1 to 64 slots");
    std::string failure;
    b->base_caches_ = KvCache(config.lm, config.max_length, cache_type, slots);
    b->residual_caches_ =
        KvCache(config.residual_lm, config.max_length, cache_type, slots);
    SlotCaches caches{&b->base_caches_, &b->residual_caches_, 0};
    auto first = Generator::Create(config, seed, kind, cache_type, &failure,
                                   files, nullptr, nullptr, &caches);
    if (!first)
      throw std::runtime_error(failure);
    b->stream_ = first->stream_;
    b->slots_.push_back(std::move(first));
    for (int i = 1; i < slots; ++i) {
      caches.slot = i;
      auto g = Generator::Create(config, seed, kind, cache_type, &failure,
                                 nullptr, b->slots_[0].get(), b->stream_,
                                 &caches);
      if (!g)
        throw std::runtime_error(failure);
      b->slots_.push_back(std::move(g));
    }
    const ModelConfig& c = config;
    const int patch = c.patch_size;
    const int values = patch * c.feat_dim;
    const int dit = c.dit.hidden;
    const int dit_rows = 2 * (3 + 2 * patch);
    const std::size_t n = static_cast<std::size_t>(slots);
    b->dit_cache_ = KvCache(c.dit, dit_rows * slots, cache_type);
    // One block for the batch's rows (256-byte aligned pieces).
    std::size_t used = 0;
    auto take = [&](std::size_t bytes) {
      const std::size_t at = used;
      used = (used + bytes + 255) / 256 * 256;
      return at;
    };
    const std::size_t mu_at = take(n * 2 * dit * 4);
    const std::size_t cond_at = take(n * patch * dit * 4);
    const std::size_t x_at = take(n * values * 4);
    const std::size_t velocity_at = take(n * 2 * values * 4);
    const std::size_t x_rows_at = take(n * patch * dit * 4);
    const std::size_t hidden_at = take(n * dit_rows * dit * 4);
    const std::size_t output_at = take(n * dit_rows * dit * 4);
    const std::size_t bf16_at = take(
        n * std::max<std::size_t>(dit_rows * std::max(dit, c.feat_dim),
                                  2 * c.lm.hidden) * 2);
    const std::size_t embed_at = take(n * c.lm.hidden * 4);
    const std::size_t lm_a_at = take(n * c.lm.hidden * 4);
    const std::size_t lm_b_at = take(n * c.lm.hidden * 4);
    const std::size_t lm_hidden_at = take(n * c.lm.hidden * 4);
    const std::size_t residual_at = take(n * c.lm.hidden * 4);
    const std::size_t fsq_at = take(n * c.fsq_latent_dim * 4);
    const std::size_t past_at = take(n * 4);
    const std::size_t cache_rows_at = take(n * 4);
    const std::size_t first_keys_at = take(n * 4);
    const std::size_t positions_at = take(n * dit_rows * 4);
    const std::size_t rows_at = take(n * dit_rows * 4);
    const std::size_t outputs_at = take(n * 2 * patch * 4);
    Cuda(cudaMalloc(reinterpret_cast<void**>(&b->block_), used), "cudaMalloc batch");
    unsigned char* base = b->block_;
    b->mu_ = reinterpret_cast<float*>(base + mu_at);
    b->cond_ = reinterpret_cast<float*>(base + cond_at);
    b->x_ = reinterpret_cast<float*>(base + x_at);
    b->velocity_ = reinterpret_cast<float*>(base + velocity_at);
    b->x_rows_ = reinterpret_cast<float*>(base + x_rows_at);
    b->hidden_ = reinterpret_cast<float*>(base + hidden_at);
    b->output_ = reinterpret_cast<float*>(base + output_at);
    b->bf16_ = reinterpret_cast<std::uint16_t*>(base + bf16_at);
    b->embed_ = reinterpret_cast<float*>(base + embed_at);
    b->lm_a_ = reinterpret_cast<float*>(base + lm_a_at);
    b->lm_b_ = reinterpret_cast<float*>(base + lm_b_at);
    b->lm_hidden_ = reinterpret_cast<float*>(base + lm_hidden_at);
    b->residual_hidden_ = reinterpret_cast<float*>(base + residual_at);
    b->fsq_ = reinterpret_cast<float*>(base + fsq_at);
    b->past_ = reinterpret_cast<std::int32_t*>(base + past_at);
    b->cache_rows_ = reinterpret_cast<std::int32_t*>(base + cache_rows_at);
    b->first_keys_ = reinterpret_cast<std::int32_t*>(base + first_keys_at);
    b->positions_ = reinterpret_cast<std::int32_t*>(base + positions_at);
    b->rows_ = reinterpret_cast<std::int32_t*>(base + rows_at);
    b->outputs_ = reinterpret_cast<std::int32_t*>(base + outputs_at);
    // Slot s's rows: positions 0..10 in each of its two sequences, cache
    // rows 22s.., outputs the last P rows of each sequence
    // (generator.cpp:109-124).
    const int length = dit_rows / 2;
    std::vector<std::int32_t> pos(n * dit_rows), rows(n * dit_rows), outs;
    for (std::size_t r = 0; r < n * dit_rows; ++r) {
      pos[r] = static_cast<std::int32_t>(r % length);
      rows[r] = static_cast<std::int32_t>(r);
    }
    for (std::size_t s = 0; s < n; ++s)
      for (int q = 0; q < 2; ++q)
        for (int i = 0; i < patch; ++i)
          outs.push_back(static_cast<std::int32_t>(s * dit_rows + q * length + 3 + patch + i));
    Cuda(cudaMemcpy(b->positions_, pos.data(), pos.size() * 4, cudaMemcpyHostToDevice), "upload");
    Cuda(cudaMemcpy(b->rows_, rows.data(), rows.size() * 4, cudaMemcpyHostToDevice), "upload");
    Cuda(cudaMemcpy(b->outputs_, outs.data(), outs.size() * 4, cudaMemcpyHostToDevice), "upload");
    // The shared work buffers of slot 0 serve the batch's stack passes.
    Generator& g0 = *b->slots_[0];
    g0.EnsureRows(std::max(dit_rows * slots, slots * (patch + 1)));
    g0.EnsureEncoder(slots);
  } catch (const std::exception& failure) {
    if (error != nullptr)
      *error = failure.what();
    return nullptr;
  }
  return b;
}

GeneratorBatch::~GeneratorBatch() {
  if (stream_ != nullptr)
    cudaStreamSynchronize(stream_);
  DestroyGraphs();
  if (block_ != nullptr)
    cudaFree(block_);
  // Slot 0 owns the stream and the weights: release it last.
  while (slots_.size() > 1)
    slots_.pop_back();
  slots_.clear();
}

void GeneratorBatch::DestroyGraphs() {
  for (auto& kv : graphs_)
    cudaGraphExecDestroy(kv.second);
  graphs_.clear();
}

void GeneratorBatch::EvaluateDit(int count, float t) {
  // generator.cpp:297-324 over `count` slots' rows.
  Generator& g0 = *slots_[0];
  const ModelConfig& c = g0.config_;
  const GeneratorWeights& w = g0.w_;
  const int patch = c.patch_size;
  const int values = patch * c.feat_dim;
  const int width = c.dit.hidden;
  const int rows = 2 * (3 + 2 * patch);
  const float* time = g0.TimeVector(t);  // prepared before capture
  Ok(ToBf16(x_, bf16_, static_cast<std::size_t>(count) * values, false, stream_), "ToBf16");
  Ok(Project(w.dit_in, bf16_, x_rows_, count * patch, stream_), "dit_in");
  for (int s = 0; s < count; ++s)
    Ok(AssembleDit(mu_ + static_cast<std::size_t>(s) * 2 * width, time,
                   cond_ + static_cast<std::size_t>(s) * patch * width,
                   x_rows_ + static_cast<std::size_t>(s) * patch * width,
                   hidden_ + static_cast<std::size_t>(s) * rows * width, patch,
                   width, stream_),
       "AssembleDit");
  AttentionLayout layout;
  layout.positions = positions_;
  layout.cache_rows = rows_;
  layout.rows_per_sequence = rows / 2;
  layout.keys_per_sequence = rows / 2;
  layout.causal = false;
  Ok(ForwardStack(w.dit, g0.rope_, layout, dit_cache_, hidden_, output_,
                  count * rows, g0.scratch_, stream_),
     "dit stack");
  Ok(GatherRows(output_, outputs_, hidden_, static_cast<std::size_t>(count) * 2 * patch,
                width, stream_),
     "GatherRows");
  Ok(ToBf16(hidden_, bf16_, static_cast<std::size_t>(count) * 2 * patch * width, false,
            stream_),
     "ToBf16");
  Ok(Project(w.dit_out, bf16_, velocity_, count * 2 * patch, stream_), "dit_out");
}

void GeneratorBatch::Body(const std::vector<int>& members, int timesteps,
                          float cfg) {
  Generator& g0 = *slots_[0];
  const ModelConfig& c = g0.config_;
  const int patch = c.patch_size;
  const int values = patch * c.feat_dim;
  const int dit = c.dit.hidden;
  const int hidden = c.lm.hidden;
  const int count = static_cast<int>(members.size());
  for (int i = 0; i < count; ++i) {
    Generator& g = *slots_[members[i]];
    g.PreDit();
    Ok(CopyFloats(g.mu_, mu_ + static_cast<std::size_t>(i) * 2 * dit, 2 * dit, stream_), "copy");
    Ok(CopyFloats(g.cond_rows_, cond_ + static_cast<std::size_t>(i) * patch * dit,
                  static_cast<std::size_t>(patch) * dit, stream_),
       "copy");
    Ok(CopyFloats(g.x_, x_ + static_cast<std::size_t>(i) * values, values, stream_), "copy");
  }
  for (int step = 0; step < timesteps; ++step) {
    if (!g0.schedule_eval_[step])
      continue;  // zero velocity (CFG-Zero*)
    EvaluateDit(count, g0.schedule_t_[step]);
    for (int i = 0; i < count; ++i)
      Ok(GuidedEuler(velocity_ + static_cast<std::size_t>(i) * 2 * values,
                     x_ + static_cast<std::size_t>(i) * values, values, cfg,
                     g0.schedule_dt_[step], stream_),
         "GuidedEuler");
  }
  for (int i = 0; i < count; ++i) {
    Generator& g = *slots_[members[i]];
    Ok(CopyFloats(x_ + static_cast<std::size_t>(i) * values, g.x_, values, stream_), "copy");
    g.PatchOutputs();
  }
  g0.Encode(x_, count, embed_);
  AdvanceLms(members);
}

void GeneratorBatch::AdvanceLms(const std::vector<int>& members) {
  // Generator::AdvanceLms (generator.cpp:478-513) for every active slot as
  // one pass of `count` rows over the slot-major caches.
  Generator& g0 = *slots_[0];
  const ModelConfig& c = g0.config_;
  const GeneratorWeights& w = g0.w_;
  const int hidden = c.lm.hidden;
  const int count = static_cast<int>(members.size());
  const int capacity = g0.capacity();
  SlotPositions positions{};
  positions.count = count;
  positions.stride = c.lm.kv_heads * capacity;
  for (int i = 0; i < count; ++i) {
    positions.counter[i] = slots_[members[i]]->position_counter_;
    positions.slot[i] = members[i];
  }
  GatherPositionsKernel<<<1, 64, 0, stream_>>>(positions, past_, cache_rows_,
                                                first_keys_);
  Cuda(cudaGetLastError(), "gather positions");
  AttentionLayout layout;
  layout.positions = past_;      // the rotary row is the position
  layout.cache_rows = cache_rows_;
  layout.rows_per_sequence = 1;
  layout.keys_per_sequence = positions.stride;
  layout.first_keys = first_keys_;  // row i reads slot members[i]
  layout.past_device = past_;
  layout.past_per_sequence = true;
  layout.max_keys = capacity;
  layout.causal = true;
  const std::size_t rows_h = static_cast<std::size_t>(count) * hidden;
  Ok(CopyFloats(embed_, lm_a_, rows_h, stream_), "copy");
  Ok(ForwardStack(w.base_lm, g0.rope_, layout, base_caches_, lm_a_, lm_b_,
                  count, g0.scratch_, stream_),
     "base lm");
  // FSQ (generator.cpp:239-250) over the rows.
  Ok(ToBf16(lm_b_, bf16_, rows_h, false, stream_), "ToBf16");
  Ok(Project(w.fsq_in, bf16_, fsq_, count, stream_), "fsq_in");
  Ok(Quantize(fsq_, bf16_, static_cast<std::size_t>(count) * c.fsq_latent_dim,
              c.fsq_scale, stream_),
     "Quantize");
  Ok(Project(w.fsq_out, bf16_, lm_hidden_, count, stream_), "fsq_out");
  Ok(ConcatRows(lm_hidden_, nullptr, hidden, embed_, nullptr, hidden, bf16_,
                count, stream_),
     "ConcatRows");
  Ok(Project(w.fusion, bf16_, lm_a_, count, stream_), "fusion");
  Ok(ForwardStack(w.residual_lm, nullptr, layout, residual_caches_, lm_a_,
                  residual_hidden_, count, g0.scratch_, stream_),
     "residual lm");
  for (int i = 0; i < count; ++i) {
    Generator& g = *slots_[members[i]];
    const std::size_t row = static_cast<std::size_t>(i) * hidden;
    Ok(CopyFloats(lm_hidden_ + row, g.lm_hidden_, hidden, stream_), "copy");
    Ok(CopyFloats(residual_hidden_ + row, g.residual_hidden_, hidden, stream_),
       "copy");
    Ok(AdvancePosition(g.position_counter_, g.step_positions_, stream_),
       "advance");
  }
}

void GeneratorBatch::Step(const std::int32_t* active, const float* noise,
                          int timesteps, float cfg, float* latents,
                          float* stop_logits) {
  if (active == nullptr || noise == nullptr || timesteps <= 0)
    throw std::invalid_argument("active, noise and timesteps are required");
  Generator& g0 = *slots_[0];
  const int values = g0.config_.patch_size * g0.config_.feat_dim;
  std::vector<int> members;
  std::uint64_t mask = 0;
  for (int s = 0; s < slots(); ++s) {
    if (active[s] == 0)
      continue;
    Generator& g = *slots_[s];
    if (g.position_ <= 0 || g.position_ >= g.capacity())
      throw std::logic_error("slot " + std::to_string(s) + " has no room for a patch");
    members.push_back(s);
    mask |= 1ull << s;
  }
  if (members.empty())
    return;
  g0.PrepareTimes(timesteps);
  // Graphs hold the slots' buffer pointers: re-capture once any moved.
  std::vector<std::uint64_t> epochs;
  for (const auto& g : slots_)
    epochs.push_back(g->buffers_epoch_);
  if (epochs != epochs_) {
    Cuda(cudaStreamSynchronize(stream_), "sync");
    DestroyGraphs();
    epochs_ = epochs;
  }
  for (const int s : members)
    std::memcpy(slots_[s]->pinned_noise_, noise + static_cast<std::size_t>(s) * values,
                values * sizeof(float));
  if (!graphs_enabled_) {
    Body(members, timesteps, cfg);
  } else {
    const auto key = std::make_tuple(mask, timesteps, cfg);
    auto found = graphs_.find(key);
    if (found == graphs_.end()) {
      cudaGraph_t graph = nullptr;
      Cuda(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeRelaxed), "capture");
      try {
        Body(members, timesteps, cfg);
      } catch (...) {
        cudaStreamEndCapture(stream_, &graph);
        if (graph != nullptr)
          cudaGraphDestroy(graph);
        throw;
      }
      Cuda(cudaStreamEndCapture(stream_, &graph), "end capture");
      cudaGraphExec_t exec = nullptr;
      const cudaError_t made = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      Cuda(made, "instantiate batch graph");
      found = graphs_.emplace(key, exec).first;
    }
    Cuda(cudaGraphLaunch(found->second, stream_), "batch graph");
  }
  for (const int s : members)
    Cuda(cudaEventRecord(slots_[s]->latent_event_, stream_), "latent event");
  Cuda(cudaStreamSynchronize(stream_), "batch step");
  for (const int s : members) {
    Generator& g = *slots_[s];
    if (latents != nullptr)
      std::memcpy(latents + static_cast<std::size_t>(s) * values, g.pinned_latent_,
                  values * sizeof(float));
    if (stop_logits != nullptr)
      std::memcpy(stop_logits + 2 * static_cast<std::size_t>(s), g.pinned_stop_,
                  2 * sizeof(float));
    ++g.position_;
    g.latent_ready_ = true;
  }
}

}  // namespace vx
