// Device use of the C++ mirror header, as a caller of the reference's
// gemm.hpp and generator.hpp writes it (tests/products_test.cpp,
// synthesizer.cpp:262,290): Bf16Gemm::Linear on Q8_0 tiles and on bf16 rows,
// then a seeded Generator's Prefill and Steps, then the AudioVae decoding the
// last latent. Inputs come from raw files
// the Python test writes into <dir>; outputs go back there for it to check
// against the oracle.
//
//   shim_device <dir>
//
// <dir>/dims.txt: rows in out steps prompt_rows; x.u16 [rows][in] bf16 bits;
// blocks.u8 [out][in/32] GGML Q8_0 blocks; w.u16 [out][in] bf16 bits;
// config.json; tokens.i32, text.i32, audio.i32 [prompt_rows];
// feats.f32 [prompt_rows][patch * feat]; noise.f32 [steps][patch * feat].
// Writes y_q8.f32, y_bf16.f32 [rows][out], latents.f32 [steps][patch * feat],
// stops.f32 [steps][2], and the last latent decoded by a seeded AudioVae
// (latent = feat, decoder 64, rates 2 3, seed 11) from the device latent after
// the step's event (vae_enqueued.f32) and from the host (vae_decoded.f32).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>
#include <string>
#include <vector>

#include "voxcpm_b200.hpp"

namespace vb = voxcpm_b200;

template <typename T>
std::vector<T> Read(const std::string& path) {
  std::ifstream in(path, std::ios::binary);
  std::vector<char> bytes((std::istreambuf_iterator<char>(in)),
                          std::istreambuf_iterator<char>());
  std::vector<T> out(bytes.size() / sizeof(T));
  std::memcpy(out.data(), bytes.data(), out.size() * sizeof(T));
  return out;
}

template <typename T>
void Write(const std::string& path, const std::vector<T>& values) {
  std::ofstream out(path, std::ios::binary);
  out.write(reinterpret_cast<const char*>(values.data()),
            static_cast<std::streamsize>(values.size() * sizeof(T)));
}

void Cuda(cudaError_t error, const char* what) {
  if (error != cudaSuccess)
    throw vb::GpuError(std::string(what) + ": " + cudaGetErrorString(error));
}

template <typename T>
T* Upload(const std::vector<T>& host) {
  void* device = nullptr;
  Cuda(cudaMalloc(&device, host.size() * sizeof(T) + 16), "cudaMalloc");
  Cuda(cudaMemcpy(device, host.data(), host.size() * sizeof(T),
                  cudaMemcpyHostToDevice),
       "upload");
  return static_cast<T*>(device);
}

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: shim_device <dir>\n");
    return 2;
  }
  const std::string dir = argv[1];
  try {
    std::size_t rows = 0, in = 0, out = 0, steps = 0, prompt_rows = 0;
    {
      std::ifstream dims(dir + "/dims.txt");
      dims >> rows >> in >> out >> steps >> prompt_rows;
    }
    cudaStream_t stream = nullptr;
    Cuda(cudaStreamCreate(&stream), "stream");

    // Bf16Gemm::Linear (gemm.hpp:51-58) on Q8_0 tiles and on bf16 rows.
    const auto x_host = Read<std::uint16_t>(dir + "/x.u16");
    const auto blocks = Read<std::uint8_t>(dir + "/blocks.u8");
    const auto w_host = Read<std::uint16_t>(dir + "/w.u16");
    std::uint16_t* x = Upload(x_host);
    std::uint8_t* block_dev = Upload(blocks);
    std::uint16_t* w = Upload(w_host);
    void* tiles = nullptr;
    Cuda(cudaMalloc(&tiles, vb::kernels::Q8TilesBytes(out, in)), "tiles");
    vb::kernels::Q8_0ToTiles(block_dev, out, in,
                             static_cast<std::uint8_t*>(tiles), stream);
    float* y = nullptr;
    Cuda(cudaMalloc(&y, rows * out * sizeof(float)), "y");
    {
    // The gemm synchronizes its stream when destroyed: it goes first.
    vb::Bf16Gemm gemm(stream);
    std::vector<float> y_host(rows * out);
    const struct {
      vb::Matrix w;
      const char* file;
    } runs[] = {{{vb::WeightFormat::kQ8Tiles, tiles}, "/y_q8.f32"},
                {{vb::WeightFormat::kBf16, w}, "/y_bf16.f32"}};
    for (const auto& run : runs) {
      gemm.Linear(x, run.w, y, rows, in, out, false);
      Cuda(cudaStreamSynchronize(stream), "sync");
      Cuda(cudaMemcpy(y_host.data(), y, y_host.size() * sizeof(float),
                      cudaMemcpyDeviceToHost),
           "download");
      Write(dir + run.file, y_host);
    }
    }

    // A seeded Generator: Prefill, then Steps (generator.hpp:58-94).
    std::string text;
    {
      std::ifstream config(dir + "/config.json");
      text.assign(std::istreambuf_iterator<char>(config),
                  std::istreambuf_iterator<char>());
    }
    vx_model_config config;
    std::string error;
    if (!vb::ParseConfig(text, &config, &error))
      throw vb::GpuError("ParseConfig: " + error);
    const auto generator =
        vb::Generator::Create(config, 7, VX_CHECKPOINT_Q8, VX_CACHE_F32, &error);
    if (generator == nullptr)
      throw vb::GpuError("Generator::Create: " + error);
    vb::Prompt prompt;
    prompt.tokens = Read<std::int32_t>(dir + "/tokens.i32");
    prompt.text_mask = Read<std::int32_t>(dir + "/text.i32");
    prompt.audio_mask = Read<std::int32_t>(dir + "/audio.i32");
    prompt.feats = Read<float>(dir + "/feats.f32");
    generator->Prefill(prompt);
    const auto noise = Read<float>(dir + "/noise.f32");
    const std::size_t values = noise.size() / steps;
    std::vector<float> latents(steps * values);
    std::vector<float> stops(steps * 2);
    for (std::size_t s = 0; s < steps; ++s)
      generator->Step(noise.data() + s * values, 10, 2.0F,
                      latents.data() + s * values, stops.data() + 2 * s);
    Write(dir + "/latents.f32", latents);
    Write(dir + "/stops.f32", stops);
    std::printf("positions %zu\n", generator->position());

    // AudioVae (vae.hpp:25-79): the last step's device latent decoded on the
    // AudioVAE's stream after the step's event, and the same latent from the
    // host, each from a new stream.
    vx_vae_config vae_config;
    vx_vae_config_default(&vae_config);
    vae_config.latent_dim = config.feat_dim;
    vae_config.decoder_dim = 64;
    vae_config.decoder_rate_count = 2;
    vae_config.decoder_rates[0] = 2;
    vae_config.decoder_rates[1] = 3;
    const auto streamed = vb::AudioVae::Create(vae_config, 11, &error);
    const auto host = vb::AudioVae::Create(vae_config, 11, &error);
    if (streamed == nullptr || host == nullptr)
      throw vb::GpuError("AudioVae::Create: " + error);
    std::vector<float> enqueued, decoded;
    streamed->Enqueue(generator->latent(), config.patch_size,
                      generator->latent_event());
    streamed->Collect(&enqueued);
    host->Decode(latents.data() + (steps - 1) * values, config.patch_size,
                 &decoded);
    Write(dir + "/vae_enqueued.f32", enqueued);
    Write(dir + "/vae_decoded.f32", decoded);
    cudaFree(x);
    cudaFree(block_dev);
    cudaFree(w);
    cudaFree(tiles);
    cudaFree(y);
    cudaStreamDestroy(stream);
  } catch (const std::exception& failure) {
    std::fprintf(stderr, "shim_device: %s\n", failure.what());
    return 1;
  }
  return 0;
}
