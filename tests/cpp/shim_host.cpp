// Host-only use of the C++ mirror header (no GPU calls): compiles against
// include/voxcpm_b200.hpp, links libvoxcpm_b200.so and prints the Euler
// schedule, a product plan and tile sizes for the Python test to check.
#include <cstdio>
#include <string>

#include "voxcpm_b200.hpp"

int main(int argc, char** argv) {
  namespace vb = voxcpm_b200;
  if (argc > 1) {
    // Checkpoint files: open, list, parse the embedded config.
    std::string error;
    const auto files = vb::ModelFiles::Open(argv[1], &error);
    if (files == nullptr) {
      std::printf("files error %s\n", error.c_str());
      return 0;
    }
    std::printf("files %zu %d\n", files->model_tensors().size(), files->gguf() ? 1 : 0);
    const vb::Tensor* t = files->Model("stop_head.weight");
    if (t != nullptr)
      std::printf("tensor %d %zu %zu %zu\n", static_cast<int>(t->dtype), t->shape[0], t->shape[1], t->bytes);
    vx_model_config config;
    if (vb::ParseConfig(files->config(), &config, &error))
      std::printf("config %d %d %d %d\n", config.lm.hidden, config.dit.layers, config.vocab, config.max_length);
    else
      std::printf("config error %s\n", error.c_str());
    return 0;
  }
  for (const vb::EulerStep& s : vb::EulerSchedule(10))
    std::printf("step %.9g %.9g %d\n", s.t, s.dt, s.evaluate ? 1 : 0);
  const vb::kernels::WmmaPlan plan = vb::kernels::PlanWmma(22, 2048, 6144);
  std::printf("plan %zu %zu %zu %zu\n", plan.splits, plan.blocks_per_split,
              plan.partial_floats, plan.counters);
  std::printf("tiles %zu %zu\n", vb::kernels::Q8TilesBytes(6144, 2048),
              vb::kernels::Bf16TilesBytes(72, 1024));
  const std::vector<float> table = vb::RopeTable(10000.0, 128, std::vector<double>(64, 1.0), 1.0, 4);
  std::printf("rope %.9g %.9g\n", table[128 + 1], table[3 * 128 + 64 + 5]);
  std::printf("bucket %zu %zu\n", vb::TuningBucket(129), vb::TuningBucket(128));
  {
    // Bf16Gemm::Matmul rejects a leading dimension below m before launching.
    vb::Bf16Gemm gemm(nullptr);
    vb::MatmulShape shape;
    shape.m = 64;
    shape.n = 8;
    shape.k = 32;
    shape.lda = 63;
    shape.ldb = 32;
    shape.ldc = 64;
    try {
      gemm.Matmul(shape, shape, nullptr, nullptr, nullptr);
    } catch (const vb::GpuError& e) {
      std::printf("matmul rejects ok\n");
    }
  }
  try {
    vb::Check(VX_INVALID, "forced");
  } catch (const vb::GpuError& e) {
    std::printf("error ok\n");
  }
  return 0;
}
