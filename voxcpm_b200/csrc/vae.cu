// AudioVAE V2 decoder on sm_100a: latents -> audio on the AudioVAE's own
// stream, fed by the generator's latent event (the reference's AudioVae,
// vae.hpp:25-79, vae.cpp:382-572; kernels/vae_kernels.hip:19-100).
//
// The decoder is causal and runs chunk by chunk: every causal convolution
// keeps the last frames of its input as state for the next call, so
// decoding a stream in chunks equals decoding it at once (up to float32
// rounding: a product may take another kernel at another row count).
// Time-major float32 throughout ([frames][channels]), as the reference
// computes it.
//
// Layout of the work (B200-first, this library's own design):
// - Every product is one launch with its bias (and, for the residual units,
//   the residual add) in the epilogue: for at most 8 rows, where the
//   weight stream is the work, a warp per two output columns with the lanes
//   splitting the reduction (VaeSkinnyKernel); for more rows, float32 tiles
//   staged by asynchronous copies (VaeProductKernel), the tile and a split
//   of the reduction over a thread-block cluster chosen so that the launch
//   fills the SMs (the cluster's sums meet in distributed shared memory).
// - A transposed convolution (kernel 2s, stride s) is ONE product: its input
//   rows are windows of two adjacent frames (the previous and the current)
//   read in place from the state-prefixed window (row stride = one frame,
//   row length = two), against weights packed as [s * out][2 * in].
// - Each causal convolution's history lives in a two-half state: a decoding
//   reads one half and writes the other, so no copies move history around.
//   A residual unit's Snake, depthwise convolution and second Snake are one
//   kernel that forms the window on the fly (VaeWindowDepthwiseKernel).
// - A decoding is one CUDA graph per chunk size and state half (52 kernels
//   for the released decoder, then the copy of the samples to pinned host
//   memory), replayed on the AudioVAE's own stream.
// Weights are the seeded checkpoint (SeededVaeWeights): bf16 values of the
// library's seeded hash, widened to float32, in the packed layouts.
#include "model.cuh"
#include "vx_common.cuh"
#include "vx_launch.cuh"
#include "vx_status.h"

#include "../../include/voxcpm_b200.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace vx {
namespace {

constexpr int kVaeKernel = 7;
constexpr int kDilations[3] = {1, 3, 9};
constexpr int kMaxRates = 8;
constexpr int kSms = 148;  // B200

void CudaCheck(cudaError_t error, const char* what) {
  if (error != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " +
                             cudaGetErrorString(error));
}

// ------------------------------------------------------------ kernels

constexpr int kThreads = 256;
constexpr int kDepth = 32;          // reduction values per stage
constexpr int kPitch = kDepth + 4;  // floats per staged row (16-byte rows)
constexpr int kStages = 4;          // stages in flight

template <int kTileRows, int kTileCols>
constexpr int ProductSmem() {
  return kStages * (kTileRows + kTileCols) * kPitch * 4;
}

__device__ __forceinline__ void CopyChunk(float* dst, const float* src,
                                          bool valid) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  // A chunk outside the matrix reads nothing and fills zeros.
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d),
               "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void CommitChunks() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int kPending>
__device__ __forceinline__ void WaitChunks() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(kPending) : "memory");
}

/// A weight vector read once: through the non-coherent path without
/// allocating in L1 (the activations stay there).
__device__ __forceinline__ float4 LoadStreamed(const float4* at) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(at));
  return v;
}

__device__ __forceinline__ float Dot4(float acc, float4 a, float4 b) {
  acc = fmaf(a.x, b.x, acc);
  acc = fmaf(a.y, b.y, acc);
  acc = fmaf(a.z, b.z, acc);
  return fmaf(a.w, b.w, acc);
}

/// y[rows][out] = (accumulate ? y : 0) + x[rows][k] w[out][k]^T + bias[out]
/// (bias may be null) for a few rows (at most kRows), where the weight
/// stream is the work: each warp takes kCols output columns and its lanes
/// split the reduction (lane l sums the 4-value groups l, l + 32, ...; the
/// lanes' sums meet in a butterfly). x rows are `ldx` floats apart and may
/// overlap; k, ldx and the pointers are multiples of 4 floats.
template <int kRows, int kCols>
__global__ void __launch_bounds__(128)
    VaeSkinnyKernel(const float* __restrict__ x, int ldx,
                    const float* __restrict__ w, const float* __restrict__ bias,
                    float* y, int rows, int k, int out, int accumulate) {
  const int lane = threadIdx.x % 32;
  const int col0 = (blockIdx.x * 4 + threadIdx.x / 32) * kCols;
  if (col0 >= out)
    return;
  const float4* wr[kCols];
#pragma unroll
  for (int c = 0; c < kCols; ++c)
    wr[c] = reinterpret_cast<const float4*>(
        w + static_cast<long long>(min(col0 + c, out - 1)) * k);
  float acc[kRows][kCols];
#pragma unroll
  for (int r = 0; r < kRows; ++r)
#pragma unroll
    for (int c = 0; c < kCols; ++c)
      acc[r][c] = 0.0f;
  const int groups = k / 4;
  // The first weights are in flight before the wait for the previous
  // launch (they do not depend on it).
  float4 wv[kCols];
  if (lane < groups) {
#pragma unroll
    for (int c = 0; c < kCols; ++c)
      wv[c] = LoadStreamed(wr[c] + lane);
  }
  GridDependencyWait();
#pragma unroll 1
  for (int g = lane; g < groups; g += 32) {
    if (g != lane) {
#pragma unroll
      for (int c = 0; c < kCols; ++c)
        wv[c] = LoadStreamed(wr[c] + g);
    }
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      if (r < rows) {
        const float4 xv = __ldg(reinterpret_cast<const float4*>(
                                    x + static_cast<long long>(r) * ldx) +
                                g);
#pragma unroll
        for (int c = 0; c < kCols; ++c)
          acc[r][c] = Dot4(acc[r][c], xv, wv[c]);
      }
    }
  }
  GridLaunchDependents();
#pragma unroll
  for (int r = 0; r < kRows; ++r)
#pragma unroll
    for (int c = 0; c < kCols; ++c)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
        acc[r][c] += __shfl_xor_sync(0xFFFFFFFFu, acc[r][c], o);
#pragma unroll
  for (int r = 0; r < kRows; ++r)
#pragma unroll
    for (int c = 0; c < kCols; ++c) {
      const int col = col0 + c;
      if (lane == (r * kCols + c) % 32 && r < rows && col < out) {
        float v = acc[r][c];
        if (bias != nullptr)
          v += bias[col];
        float* at = y + static_cast<long long>(r) * out + col;
        *at = accumulate ? *at + v : v;
      }
    }
}

/// The same product for more rows: tiles of kTileRows x kTileCols outputs,
/// kStages stages of 32 reduction values copied asynchronously into shared
/// memory, (kTileRows / 16) x (kTileCols / 16) outputs per thread. The
/// reduction may be split over the gridDim.z CTAs of a thread-block cluster
/// (`k_split` values each, a multiple of 32): each sums its range in order,
/// and the cluster's first CTA adds the others' sums in rank order from
/// their shared memory, so the result does not depend on timing.
template <int kTileRows, int kTileCols>
__global__ void __launch_bounds__(kThreads)
    VaeProductKernel(const float* __restrict__ x, int ldx,
                     const float* __restrict__ w, const float* __restrict__ bias,
                     float* y, int rows, int k, int out, int accumulate,
                     int k_split) {
  constexpr int kRowsPerThread = kTileRows / 16;
  constexpr int kColsPerThread = kTileCols / 16;
  constexpr int kOutputs = kRowsPerThread * kColsPerThread;
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;                                 // [stage][row][kPitch]
  float* ws = smem + kStages * kTileRows * kPitch;  // [stage][col][kPitch]
  const int tid = threadIdx.x;
  const int tx = tid % 16;  // columns tx + 16 j
  const int ty = tid / 16;  // rows ty + 16 i
  const int row0 = blockIdx.y * kTileRows;
  const int col0 = blockIdx.x * kTileCols;
  const int splits = gridDim.z;
  const int k_begin = blockIdx.z * k_split;
  const int k_end = min(k, k_begin + k_split);
  const int stages_total = max(0, (k_end - k_begin + kDepth - 1) / kDepth);

  // 8 chunks of 4 floats per staged row.
  auto load_x = [&](int stage, int index) {
    const int k0 = k_begin + index * kDepth;
    for (int c = tid; c < kTileRows * 8; c += kThreads) {
      const int r = c / 8, kk = k0 + (c % 8) * 4;
      const bool valid = row0 + r < rows && kk < k_end;
      CopyChunk(xs + (stage * kTileRows + r) * kPitch + (c % 8) * 4,
                valid ? x + static_cast<long long>(row0 + r) * ldx + kk : x,
                valid);
    }
  };
  auto load_w = [&](int stage, int index) {
    const int k0 = k_begin + index * kDepth;
    for (int c = tid; c < kTileCols * 8; c += kThreads) {
      const int r = c / 8, kk = k0 + (c % 8) * 4;
      const bool valid = col0 + r < out && kk < k_end;
      CopyChunk(ws + (stage * kTileCols + r) * kPitch + (c % 8) * 4,
                valid ? w + static_cast<long long>(col0 + r) * k + kk : w,
                valid);
    }
  };

  float acc[kRowsPerThread][kColsPerThread] = {};
  // The first stages' weights are copied before the wait for the previous
  // launch (they do not depend on it; they join the first copy group), the
  // activations after it.
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s)
    if (s < stages_total)
      load_w(s, s);
  GridDependencyWait();
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < stages_total)
      load_x(s, s);
    CommitChunks();
  }
  for (int index = 0; index < stages_total; ++index) {
    WaitChunks<kStages - 2>();
    __syncthreads();  // stage `index` landed; stage index - 1 is free
    if (index + kStages - 1 < stages_total) {
      load_x((index + kStages - 1) % kStages, index + kStages - 1);
      load_w((index + kStages - 1) % kStages, index + kStages - 1);
    }
    CommitChunks();
    const int stage = index % kStages;
    const float* xt = xs + stage * kTileRows * kPitch;
    const float* wt = ws + stage * kTileCols * kPitch;
#pragma unroll
    for (int kk = 0; kk < kDepth; kk += 4) {
      float4 a[kRowsPerThread], b[kColsPerThread];
#pragma unroll
      for (int i = 0; i < kRowsPerThread; ++i)
        a[i] = *reinterpret_cast<const float4*>(xt + (ty + 16 * i) * kPitch + kk);
#pragma unroll
      for (int j = 0; j < kColsPerThread; ++j)
        b[j] = *reinterpret_cast<const float4*>(wt + (tx + 16 * j) * kPitch + kk);
#pragma unroll
      for (int i = 0; i < kRowsPerThread; ++i)
#pragma unroll
        for (int j = 0; j < kColsPerThread; ++j)
          acc[i][j] = Dot4(acc[i][j], a[i], b[j]);
    }
  }
  WaitChunks<0>();
  GridLaunchDependents();
  if (splits > 1) {
    // The partial sums, 4 at a time, interleaved by thread.
    float4* part = reinterpret_cast<float4*>(smem);
    __syncthreads();  // the staging buffers are read
#pragma unroll
    for (int q = 0; q < kOutputs / 4; ++q)
      part[q * kThreads + tid] =
          make_float4(acc[(4 * q + 0) / kColsPerThread][(4 * q + 0) % kColsPerThread],
                      acc[(4 * q + 1) / kColsPerThread][(4 * q + 1) % kColsPerThread],
                      acc[(4 * q + 2) / kColsPerThread][(4 * q + 2) % kColsPerThread],
                      acc[(4 * q + 3) / kColsPerThread][(4 * q + 3) % kColsPerThread]);
    ClusterSync();
    if (blockIdx.z == 0) {
      for (int r = 1; r < splits; ++r) {
#pragma unroll
        for (int q = 0; q < kOutputs / 4; ++q) {
          const float4 v = LoadSharedCluster4(
              MapShared(part + q * kThreads + tid, static_cast<unsigned>(r)));
          acc[(4 * q + 0) / kColsPerThread][(4 * q + 0) % kColsPerThread] += v.x;
          acc[(4 * q + 1) / kColsPerThread][(4 * q + 1) % kColsPerThread] += v.y;
          acc[(4 * q + 2) / kColsPerThread][(4 * q + 2) % kColsPerThread] += v.z;
          acc[(4 * q + 3) / kColsPerThread][(4 * q + 3) % kColsPerThread] += v.w;
        }
      }
    }
    ClusterSync();  // the others' sums stay in place until they are read
    if (blockIdx.z != 0)
      return;
  }
#pragma unroll
  for (int i = 0; i < kRowsPerThread; ++i) {
    const int r = row0 + ty + 16 * i;
    if (r >= rows)
      continue;
#pragma unroll
    for (int j = 0; j < kColsPerThread; ++j) {
      const int c = col0 + tx + 16 * j;
      if (c >= out)
        continue;
      float v = acc[i][j];
      if (bias != nullptr)
        v += bias[c];
      float* at = y + static_cast<long long>(r) * out + c;
      *at = accumulate ? *at + v : v;
    }
  }
}

/// Snake (DAC, kernels/vae_kernels.hip:19-33): y + sin(alpha y)^2 /
/// (alpha + 1e-9).
__device__ __forceinline__ float SnakeOf(float y, float alpha) {
  const float s = sinf(alpha * y);
  return y + (1.0f / (alpha + 1e-9f)) * (s * s);
}

__device__ __forceinline__ float4 SnakeOf(float4 y, float4 a) {
  return make_float4(SnakeOf(y.x, a.x), SnakeOf(y.y, a.y), SnakeOf(y.z, a.z),
                     SnakeOf(y.w, a.w));
}

/// Row `row` of a causal convolution's window [state_old (rows frames) |
/// f(in)]: f is Snake of (in * scale + bias) (scale may be null), or the
/// identity when alpha is null. Four channels (group c) at a time.
__device__ __forceinline__ float4 WindowRow(const float4* in,
                                           const float4* state_old, int row,
                                           int rows, int c, int channels4,
                                           const float4* alpha,
                                           const float4* scale,
                                           const float4* bias) {
  if (row < rows)
    return state_old[static_cast<long long>(row) * channels4 + c];
  float4 v = in[static_cast<long long>(row - rows) * channels4 + c];
  if (scale != nullptr) {
    const float4 s = scale[c], b = bias[c];
    v = make_float4(v.x * s.x + b.x, v.y * s.y + b.y, v.z * s.z + b.z,
                    v.w * s.w + b.w);
  }
  return alpha != nullptr ? SnakeOf(v, alpha[c]) : v;
}

/// The window of a causal convolution written out: work = [state_old |
/// f(in)] (rows + t frames), and state_new = its last `rows` frames (the
/// next call's history). state_old and state_new are the two halves of one
/// state. Four channels per thread.
__global__ void VaeWindowKernel(const float4* __restrict__ in,
                                const float4* __restrict__ state_old,
                                float4* __restrict__ work,
                                float4* __restrict__ state_new, int t,
                                int rows, int channels4, const float4* alpha,
                                const float4* scale, const float4* bias) {
  GridDependencyWait();
  const long long i =
      static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(rows + t) * channels4)
    return;
  const int row = static_cast<int>(i / channels4);
  const int c = static_cast<int>(i % channels4);
  const float4 v =
      WindowRow(in, state_old, row, rows, c, channels4, alpha, scale, bias);
  work[i] = v;
  if (row >= t)
    state_new[static_cast<long long>(row - t) * channels4 + c] = v;
}

/// Channel groups (of four) of one VaeWindowDepthwiseKernel CTA.
__host__ __device__ constexpr int DepthwiseGroups(int channels4) {
  return channels4 < 32 ? channels4 : 32;
}

/// A causal depthwise convolution (kernel 7, `dilation` d) over the window
/// [state_old | f(in)] (kernels/vae_kernels.hip:35-50): out[f][c] = bias[c]
/// + sum_j w[c][j] window[f + j d][c], then Snake with alpha_out when it is
/// not null. A CTA takes `frames` frames of up to 32 channel groups: it
/// forms their window rows (frames + 6 d) once in shared memory, then each
/// thread sums the taps of its outputs there. The CTAs of the last grid
/// column write state_new instead, the window's last `rows` frames.
__global__ void __launch_bounds__(kThreads) VaeWindowDepthwiseKernel(
    const float4* __restrict__ in, const float4* __restrict__ state_old,
    float4* __restrict__ state_new, float4* __restrict__ out, int t, int rows,
    int channels4, int dilation, int frames, const float4* alpha_in,
    const float* __restrict__ w, const float* __restrict__ bias,
    const float4* alpha_out) {
  extern __shared__ float4 window[];  // [frames + 6 d][groups]
  GridDependencyWait();
  const int groups = DepthwiseGroups(channels4);
  const int c0 = blockIdx.y * groups;
  const int tid = threadIdx.x;
  if (blockIdx.x == gridDim.x - 1) {
    for (int e = tid; e < rows * groups; e += kThreads) {
      const int j = e / groups, c = c0 + e % groups;
      if (c < channels4)
        state_new[static_cast<long long>(j) * channels4 + c] =
            WindowRow(in, state_old, t + j, rows, c, channels4, alpha_in,
                      nullptr, nullptr);
    }
    return;
  }
  const int f0 = blockIdx.x * frames;
  const int span = frames + (kVaeKernel - 1) * dilation;
  for (int e = tid; e < span * groups; e += kThreads) {
    const int row = f0 + e / groups, c = c0 + e % groups;
    window[e] = c < channels4 && row < rows + t
                    ? WindowRow(in, state_old, row, rows, c, channels4,
                                alpha_in, nullptr, nullptr)
                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  __syncthreads();
  const int per_pass = kThreads / groups;
  const int cg = tid % groups, fg = tid / groups;
  const int c = c0 + cg;
  if (fg >= per_pass || c >= channels4)
    return;
  float taps[4][kVaeKernel];
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int j = 0; j < kVaeKernel; ++j)
      taps[q][j] = w[(4 * c + q) * kVaeKernel + j];
  const float4 b = reinterpret_cast<const float4*>(bias)[c];
  for (int f = fg; f < frames && f0 + f < t; f += per_pass) {
    float sum[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int j = 0; j < kVaeKernel; ++j) {
      const float4 v = window[(f + j * dilation) * groups + cg];
      sum[0] += taps[0][j] * v.x;
      sum[1] += taps[1][j] * v.y;
      sum[2] += taps[2][j] * v.z;
      sum[3] += taps[3][j] * v.w;
    }
    float4 v = make_float4(sum[0], sum[1], sum[2], sum[3]);
    if (alpha_out != nullptr)
      v = SnakeOf(v, alpha_out[c]);
    out[static_cast<long long>(f0 + f) * channels4 + c] = v;
  }
}

/// samples[t] = tanh(bias + sum_{c, j} w[c][j] in[t + j][c]); one warp per
/// output frame.
__global__ void VaeToMonoKernel(const float* in, const float* w, float bias,
                                float* samples, int frames, int channels) {
  GridDependencyWait();
  const int warp = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) / 32);
  const int lane = threadIdx.x % 32;
  if (warp >= frames)
    return;
  float sum = 0.0f;
  for (int c = lane; c < channels; c += 32)
#pragma unroll
    for (int j = 0; j < kVaeKernel; ++j)
      sum += w[c * kVaeKernel + j] *
             in[static_cast<long long>(warp + j) * channels + c];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
  if (lane == 0)
    samples[warp] = tanhf(sum + bias);
}

constexpr int kDepthwiseSmemMax = 64 << 10;

int DepthwiseSmem(int frames, int dilation, int groups) {
  return (frames + (kVaeKernel - 1) * dilation) * groups * 16;
}

void Launched(int status, const char* what) {
  if (status != kOk)
    CudaCheck(cudaGetLastError(), what);
}

unsigned BlocksOf(long long count, int threads = kThreads) {
  return static_cast<unsigned>((count + threads - 1) / threads);
}

// ------------------------------------------------------------ weights

struct VaeUnit {
  int dilation = 1;
  std::size_t alpha_in = 0, depthwise = 0, depthwise_bias = 0;
  std::size_t alpha_out = 0, pointwise = 0, pointwise_bias = 0;
};

struct VaeBlock {
  int stride = 0, in = 0, out = 0;
  std::size_t scale = 0, bias = 0, alpha = 0;
  std::size_t up = 0;       // [stride * out][2 * in]: previous frame, then current
  std::size_t up_bias = 0;  // [stride * out]
  VaeUnit units[3];
};

/// Offsets of every tensor in the packed float32 weights, and the host
/// copy they are built in.
struct VaeLayout {
  std::size_t in_depthwise = 0, in_depthwise_bias = 0;
  std::size_t in_pointwise = 0, in_pointwise_bias = 0;
  std::vector<VaeBlock> blocks;
  int out_channels = 0;
  std::size_t out_alpha = 0, out_conv = 0;
  float out_bias = 0.01f;
  std::vector<float> host;
};

/// The seeded AudioVAE checkpoint: every tensor bf16(mean + N(0, std)) of
/// the library's seeded hash (tensor id = FNV-1a of "audio_vae." + name),
/// widened to float32, drawn in the checkpoint's layouts and packed as the
/// decoder reads them (the reference packs at load, vae.cpp:222-291).
VaeLayout SeededVaeWeights(const vx_vae_config& c, std::uint64_t seed) {
  VaeLayout l;
  std::vector<std::uint16_t> bits;
  auto tensor = [&](const std::string& name, std::size_t count, float mean,
                    float std) {
    bits.resize(count);
    if (vx_random_bf16(seed, TensorId("audio_vae." + name), count, mean, std,
                       bits.data()) != VX_OK)
      throw std::runtime_error(std::string("seeded AudioVAE weights: ") +
                               vx_last_error());
    // Every tensor starts on a 16-byte boundary (vector loads).
    const std::size_t at = (l.host.size() + 3) / 4 * 4;
    l.host.resize(at + count);
    for (std::size_t i = 0; i < count; ++i) {
      const std::uint32_t wide = static_cast<std::uint32_t>(bits[i]) << 16;
      std::memcpy(&l.host[at + i], &wide, 4);
    }
    return at;
  };
  const int latent = static_cast<int>(c.latent_dim);
  const int width = static_cast<int>(c.decoder_dim);
  const std::size_t buckets = c.sr_bin_boundary_count + 1;
  std::size_t bucket = 0;  // torch.bucketize, right=False (config.cpp:269-275)
  while (bucket < c.sr_bin_boundary_count &&
         c.sr_bin_boundaries[bucket] < c.out_sample_rate)
    ++bucket;
  l.in_depthwise = tensor("in.depthwise", latent * kVaeKernel, 0.0f, 0.3f);
  l.in_depthwise_bias = tensor("in.depthwise_bias", latent, 0.0f, 0.02f);
  l.in_pointwise = tensor("in.pointwise", static_cast<std::size_t>(width) * latent,
                          0.0f, 1.0f / std::sqrt(static_cast<float>(latent)));
  l.in_pointwise_bias = tensor("in.pointwise_bias", width, 0.0f, 0.02f);
  int channels = width;
  for (std::size_t b = 0; b < c.decoder_rate_count; ++b) {
    VaeBlock block;
    block.stride = static_cast<int>(c.decoder_rates[b]);
    block.in = channels;
    block.out = channels / 2;
    const std::string p = "block" + std::to_string(b) + ".";
    // The rate conditioning: the output rate's bucket selects one row of
    // each [buckets][in] embedding table (vae.cpp:250-261).
    const std::size_t scale = tensor(p + "scale_embed", buckets * channels, 1.0f, 0.05f);
    const std::size_t bias = tensor(p + "bias_embed", buckets * channels, 0.0f, 0.05f);
    block.scale = scale + bucket * channels;
    block.bias = bias + bucket * channels;
    block.alpha = tensor(p + "alpha", channels, 1.0f, 0.1f);
    // ConvTranspose1d weight [in][out][2s] (vae.cpp:263-275), packed for
    // one product over frame pairs: row r * out + o is [taps r + s of the
    // previous frame | taps r of the current frame].
    const int s = block.stride, in = block.in, o_count = block.out;
    const std::size_t taps =
        tensor(p + "up", static_cast<std::size_t>(in) * o_count * 2 * s, 0.0f,
               1.0f / std::sqrt(2.0f * in));
    const std::vector<float> up(l.host.begin() + taps,
                                l.host.begin() + taps +
                                    static_cast<std::size_t>(in) * o_count * 2 * s);
    l.host.resize(taps);  // the packed matrix replaces the checkpoint layout
    block.up = taps;
    l.host.resize(taps + static_cast<std::size_t>(s) * o_count * 2 * in);
    for (int i = 0; i < in; ++i)
      for (int o = 0; o < o_count; ++o)
        for (int r = 0; r < s; ++r) {
          const float* tap = up.data() + (static_cast<std::size_t>(i) * o_count + o) * 2 * s;
          float* row = l.host.data() + taps +
                       (static_cast<std::size_t>(r) * o_count + o) * 2 * in;
          row[i] = tap[r + s];
          row[in + i] = tap[r];
        }
    // The bias per output channel, repeated for each of the stride's frames.
    const std::size_t one = tensor(p + "up_bias", block.out, 0.0f, 0.02f);
    const std::vector<float> per_channel(l.host.begin() + one,
                                         l.host.begin() + one + block.out);
    block.up_bias = (l.host.size() + 3) / 4 * 4;
    l.host.resize(block.up_bias);
    for (int r = 0; r < block.stride; ++r)
      l.host.insert(l.host.end(), per_channel.begin(), per_channel.end());
    for (int u = 0; u < 3; ++u) {
      VaeUnit& unit = block.units[u];
      const std::string q = p + "unit" + std::to_string(u) + ".";
      const int o = block.out;
      unit.dilation = kDilations[u];
      unit.alpha_in = tensor(q + "alpha_in", o, 1.0f, 0.1f);
      unit.depthwise = tensor(q + "depthwise", o * kVaeKernel, 0.0f, 0.3f);
      unit.depthwise_bias = tensor(q + "depthwise_bias", o, 0.0f, 0.02f);
      unit.alpha_out = tensor(q + "alpha_out", o, 1.0f, 0.1f);
      unit.pointwise = tensor(q + "pointwise", static_cast<std::size_t>(o) * o,
                              0.0f, 0.5f / std::sqrt(static_cast<float>(o)));
      unit.pointwise_bias = tensor(q + "pointwise_bias", o, 0.0f, 0.02f);
    }
    l.blocks.push_back(block);
    channels = block.out;
  }
  l.out_channels = channels;
  l.out_alpha = tensor("out.alpha", channels, 1.0f, 0.1f);
  l.out_conv = tensor("out.conv", static_cast<std::size_t>(channels) * kVaeKernel,
                      0.0f, 1.0f / std::sqrt(static_cast<float>(kVaeKernel * channels)));
  return l;
}

}  // namespace

// ------------------------------------------------------------ AudioVae

class AudioVae {
 public:
  AudioVae(const vx_vae_config& config, std::uint64_t seed) : config_(config) {
    if (config.latent_dim == 0 || config.latent_dim % 4 != 0 ||
        config.decoder_dim == 0 || config.decoder_rate_count == 0 ||
        config.decoder_rate_count > kMaxRates ||
        config.sr_bin_boundary_count > kMaxRates)
      throw std::invalid_argument("AudioVAE configuration out of range");
    hop_ = 1;
    std::size_t channels = config.decoder_dim;
    for (std::size_t b = 0; b < config.decoder_rate_count; ++b) {
      if (config.decoder_rates[b] == 0 || channels % 8 != 0)
        throw std::invalid_argument(
            "AudioVAE decoder: every block halves its channels, which must "
            "stay multiples of 4");
      hop_ *= config.decoder_rates[b];
      channels /= 2;
    }
    layout_ = SeededVaeWeights(config, seed);
    CudaCheck(cudaFuncSetAttribute(VaeWindowDepthwiseKernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kDepthwiseSmemMax),
              "AudioVAE depthwise");
    SetSmem(VaeProductKernel<64, 64>, ProductSmem<64, 64>());
    SetSmem(VaeProductKernel<64, 32>, ProductSmem<64, 32>());
    SetSmem(VaeProductKernel<32, 64>, ProductSmem<32, 64>());
    SetSmem(VaeProductKernel<32, 32>, ProductSmem<32, 32>());
    CudaCheck(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking),
              "AudioVAE stream");
    CudaCheck(cudaMalloc(&weights_, layout_.host.size() * sizeof(float)),
              "AudioVAE weights");
    CudaCheck(cudaMemcpy(weights_, layout_.host.data(),
                         layout_.host.size() * sizeof(float),
                         cudaMemcpyHostToDevice),
              "AudioVAE weights");
    layout_.host.clear();
    layout_.host.shrink_to_fit();
    // States in decoding order (vae.cpp:334-342): the input convolution's
    // 6 frames of latents, per block the last post-Snake frame before the
    // transposed convolution and each residual unit's 6 x dilation frames,
    // then the output convolution's 6 frames. Each has two halves: a
    // decoding reads one and writes the other.
    auto state = [&](std::size_t rows, std::size_t width) {
      State s{{nullptr, nullptr}, rows, width};
      CudaCheck(cudaMalloc(&s.data[0], 2 * rows * width * sizeof(float)),
                "AudioVAE state");
      s.data[1] = s.data[0] + rows * width;
      states_.push_back(s);
    };
    state(kVaeKernel - 1, config.latent_dim);
    for (const VaeBlock& block : layout_.blocks) {
      state(1, block.in);
      for (const VaeUnit& unit : block.units)
        state(static_cast<std::size_t>(kVaeKernel - 1) * unit.dilation,
              block.out);
    }
    state(kVaeKernel - 1, layout_.out_channels);
    Reset();
  }

  ~AudioVae() {
    if (stream_ != nullptr)
      cudaStreamSynchronize(stream_);
    DropGraphs();
    for (const State& s : states_)
      cudaFree(s.data[0]);
    cudaFree(weights_);
    cudaFree(latents_);
    cudaFree(work_);
    cudaFree(hidden_);
    cudaFree(scratch_);
    cudaFree(samples_);
    if (pinned_ != nullptr)
      cudaFreeHost(pinned_);
    if (stream_ != nullptr)
      cudaStreamDestroy(stream_);
  }

  std::size_t hop() const { return hop_; }
  cudaStream_t stream() const { return stream_; }

  /// vae.cpp:363-368: a new stream (zero history).
  void Reset() {
    for (const State& s : states_)
      CudaCheck(cudaMemsetAsync(s.data[0], 0,
                                2 * s.rows * s.width * sizeof(float), stream_),
                "AudioVAE reset");
    CudaCheck(cudaStreamSynchronize(stream_), "AudioVAE reset");
    phase_ = 0;
    pending_ = 0;
  }

  /// vae.cpp:382-393: host latents [frames][latent] -> host audio.
  void Decode(const float* latents, std::size_t frames, float* audio) {
    if (frames == 0)
      return;
    if (pending_ != 0)
      throw std::logic_error(
          "AudioVAE: a decoding is pending (Collect it first)");
    Reserve(frames);
    CudaCheck(cudaMemcpyAsync(latents_, latents,
                              frames * config_.latent_dim * sizeof(float),
                              cudaMemcpyHostToDevice, stream_),
              "AudioVAE latents");
    Run(frames);
    Collect(audio, frames * hop_);
  }

  /// vae.cpp:395-407: device latents, once `ready` completed, on the
  /// AudioVAE's own stream; the latents are copied before anything else.
  void Enqueue(const float* latents, std::size_t frames, cudaEvent_t ready) {
    if (frames == 0)
      return;
    if (pending_ != 0)
      throw std::logic_error(
          "AudioVAE: a decoding is pending (Collect it first)");
    Reserve(frames);
    if (ready != nullptr)
      CudaCheck(cudaStreamWaitEvent(stream_, ready, 0), "AudioVAE wait");
    CudaCheck(cudaMemcpyAsync(latents_, latents,
                              frames * config_.latent_dim * sizeof(float),
                              cudaMemcpyDeviceToDevice, stream_),
              "AudioVAE latents");
    Run(frames);
  }

  /// vae.cpp:409-413: waits for the pending decoding and copies its
  /// samples out; returns how many.
  std::size_t Collect(float* audio, std::size_t capacity) {
    CudaCheck(cudaStreamSynchronize(stream_), "AudioVAE collect");
    const std::size_t n = pending_;
    if (n > capacity)
      throw std::invalid_argument("AudioVAE collect: buffer too small");
    if (n != 0)
      std::memcpy(audio, pinned_, n * sizeof(float));
    pending_ = 0;
    return n;
  }

 private:
  using ProductFn = void (*)(const float*, int, const float*, const float*,
                            float*, int, int, int, int, int);

  static void SetSmem(ProductFn kernel, int bytes) {
    CudaCheck(cudaFuncSetAttribute(kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   bytes),
              "AudioVAE product");
  }

  struct State {
    float* data[2];
    std::size_t rows;
    std::size_t width;
  };

  const float* at(std::size_t offset) const { return weights_ + offset; }

  void DropGraphs() {
    for (auto& g : graphs_)
      if (g.exec != nullptr)
        cudaGraphExecDestroy(g.exec);
    graphs_.clear();
  }

  /// Grow-only work buffers for `frames` latent frames (vae.cpp:418-437);
  /// growing drops the captured decodings, which hold the old buffers.
  void Reserve(std::size_t frames) {
    if (frames <= reserved_)
      return;
    std::size_t widest =
        frames * std::max(config_.latent_dim, config_.decoder_dim);
    std::size_t length = frames;
    for (const VaeBlock& block : layout_.blocks) {
      widest = std::max(widest, length * block.in);
      length *= block.stride;
      widest = std::max(widest, length * block.out);
    }
    const std::size_t history =
        static_cast<std::size_t>(kVaeKernel - 1) * kDilations[2] *
        std::max(config_.latent_dim, config_.decoder_dim);
    CudaCheck(cudaStreamSynchronize(stream_), "AudioVAE reserve");
    DropGraphs();
    auto grow = [](float*& p, std::size_t floats) {
      cudaFree(p);
      p = nullptr;
      CudaCheck(cudaMalloc(&p, floats * sizeof(float)), "AudioVAE buffer");
    };
    grow(latents_, frames * config_.latent_dim);
    grow(work_, widest + history);
    grow(hidden_, widest);
    grow(scratch_, widest);
    grow(samples_, length);
    if (pinned_ != nullptr)
      cudaFreeHost(pinned_);
    pinned_ = nullptr;
    CudaCheck(cudaMallocHost(&pinned_, length * sizeof(float)),
              "AudioVAE pinned");
    reserved_ = frames;
  }

  /// y = (accumulate ? y : 0) + x w^T + bias: VaeSkinnyKernel for at most
  /// 8 rows (the weight stream is the work); else VaeProductKernel on the
  /// largest tile that, with the reduction split over a cluster of up to 8
  /// CTAs (each at least 128 values of it), fills the SMs.
  void Product(const float* x, int ldx, std::size_t weight,
               std::size_t bias, float* y, int rows, int k, int out,
               bool accumulate) {
    if (k % 4 != 0 || ldx % 4 != 0 ||
        reinterpret_cast<std::uintptr_t>(x) % 16 != 0)
      throw std::invalid_argument("AudioVAE product: unaligned rows");
    const float* w = at(weight);
    const float* b = at(bias);
    const int acc = accumulate ? 1 : 0;
    if (rows <= 8) {
      const dim3 ctas((out + 7) / 8);  // 4 warps of 2 columns
      Launched(LaunchKernel(rows <= 4 ? VaeSkinnyKernel<4, 2>
                                      : VaeSkinnyKernel<8, 2>,
                            ctas, dim3(128), 0, stream_, dim3(1), x, ldx, w, b,
                            y, rows, k, out, acc),
               "AudioVAE product");
      return;
    }
    struct Tile {
      int rows, cols, smem;
      ProductFn kernel;
    };
    const Tile tiles[] = {
        {64, 64, ProductSmem<64, 64>(), VaeProductKernel<64, 64>},
        {64, 32, ProductSmem<64, 32>(), VaeProductKernel<64, 32>},
        {32, 64, ProductSmem<32, 64>(), VaeProductKernel<32, 64>},
        {32, 32, ProductSmem<32, 32>(), VaeProductKernel<32, 32>}};
    const Tile* pick = nullptr;
    int splits = 1;
    for (const Tile& tile : tiles) {
      if ((tile.cols > 32 && out <= 32) || (tile.rows > 32 && rows <= 32))
        continue;
      const long long base =
          static_cast<long long>((rows + tile.rows - 1) / tile.rows) *
          ((out + tile.cols - 1) / tile.cols);
      pick = &tile;  // the smallest tile, if none fills the SMs
      splits = 1;
      while (base * splits < kSms && splits < 8 && k / (2 * splits) >= 128)
        splits *= 2;
      if (base * splits >= kSms)
        break;
    }
    const int k_split = (k / splits + kDepth - 1) / kDepth * kDepth;
    Launched(LaunchKernel(pick->kernel,
                          dim3((out + pick->cols - 1) / pick->cols,
                               (rows + pick->rows - 1) / pick->rows, splits),
                          dim3(kThreads), pick->smem, stream_,
                          dim3(1, 1, splits), x, ldx, w, b, y, rows, k, out,
                          acc, k_split),
             "AudioVAE product");
  }

  /// The block's window (Snake of the rate-conditioned input after one
  /// frame of history) written to work_.
  void Window(int& state, const float* in, int t, int width,
              const float* alpha, const float* scale, const float* bias) {
    const State& s = states_[state++];
    const int rows = static_cast<int>(s.rows);
    const long long count4 = static_cast<long long>(rows + t) * width / 4;
    Launched(LaunchKernel(
        VaeWindowKernel, dim3(BlocksOf(count4)), dim3(kThreads), 0, stream_,
        dim3(1), reinterpret_cast<const float4*>(in),
        reinterpret_cast<const float4*>(s.data[phase_]),
        reinterpret_cast<float4*>(work_),
        reinterpret_cast<float4*>(s.data[phase_ ^ 1]), t, rows, width / 4,
        reinterpret_cast<const float4*>(alpha),
        reinterpret_cast<const float4*>(scale),
        reinterpret_cast<const float4*>(bias)),
             "AudioVAE window");
  }

  /// A depthwise convolution over its window, formed on the fly from the
  /// state and `in` (Snake with alpha_in when not null), Snake with
  /// alpha_out after it when not null; into scratch_.
  void WindowDepthwise(int& state, const float* in, int t, int width,
                       int dilation, const float* alpha_in,
                       std::size_t weight, std::size_t bias,
                       const float* alpha_out) {
    const State& s = states_[state++];
    const int rows = static_cast<int>(s.rows);
    const int channels4 = width / 4;
    const int groups = DepthwiseGroups(channels4);
    const int per_pass = kThreads / groups;
    const int channel_tiles = (channels4 + groups - 1) / groups;
    // Frames per CTA: as many passes as keep the launch at a wave or more,
    // within the shared memory of the window.
    int frames = per_pass;
    while (frames < 64 &&
           static_cast<long long>((t + 2 * frames - 1) / (2 * frames)) *
                   channel_tiles >= kSms &&
           DepthwiseSmem(2 * frames, dilation, groups) <= kDepthwiseSmemMax)
      frames *= 2;
    const dim3 grid((t + frames - 1) / frames + 1, channel_tiles);
    Launched(LaunchKernel(
        VaeWindowDepthwiseKernel, grid, dim3(kThreads),
        DepthwiseSmem(frames, dilation, groups), stream_, dim3(1),
        reinterpret_cast<const float4*>(in),
        reinterpret_cast<const float4*>(s.data[phase_]),
        reinterpret_cast<float4*>(s.data[phase_ ^ 1]),
        reinterpret_cast<float4*>(scratch_), t, rows, channels4, dilation,
        frames, reinterpret_cast<const float4*>(alpha_in), at(weight),
        at(bias), reinterpret_cast<const float4*>(alpha_out)),
             "AudioVAE depthwise");
  }

  /// vae.cpp:415-516 (Run): latents_ -> samples_ -> pinned_, as launches on
  /// the stream (captured once per frame count and state half).
  void Launches(int frames) {
    const int latent = static_cast<int>(config_.latent_dim);
    const int width = static_cast<int>(config_.decoder_dim);
    int state = 0;
    // Input: depthwise k = 7 over the latents, then pointwise to the width.
    WindowDepthwise(state, latents_, frames, latent, 1, nullptr,
                    layout_.in_depthwise, layout_.in_depthwise_bias, nullptr);
    Product(scratch_, latent, layout_.in_pointwise, layout_.in_pointwise_bias,
            hidden_, frames, latent, width, false);
    int t = frames;
    for (const VaeBlock& block : layout_.blocks) {
      // Snake of the rate-conditioned input after one frame of history,
      // then the transposed convolution as one product over frame pairs.
      Window(state, hidden_, t, block.in, at(block.alpha), at(block.scale),
             at(block.bias));
      Product(work_, block.in, block.up, block.up_bias, hidden_, t,
              2 * block.in, block.stride * block.out, false);
      t *= block.stride;
      const int c = block.out;
      for (const VaeUnit& unit : block.units) {
        WindowDepthwise(state, hidden_, t, c, unit.dilation, at(unit.alpha_in),
                        unit.depthwise, unit.depthwise_bias,
                        at(unit.alpha_out));
        Product(scratch_, c, unit.pointwise, unit.pointwise_bias, hidden_, t,
                c, c, true);
      }
    }
    const int c = layout_.out_channels;
    Window(state, hidden_, t, c, at(layout_.out_alpha), nullptr, nullptr);
    Launched(LaunchKernel(VaeToMonoKernel,
                          dim3(BlocksOf(static_cast<long long>(t) * 32)),
                          dim3(kThreads), 0, stream_, dim3(1),
                          static_cast<const float*>(work_),
                          at(layout_.out_conv), layout_.out_bias, samples_, t,
                          c),
             "AudioVAE output");
    CudaCheck(cudaMemcpyAsync(pinned_, samples_, t * sizeof(float),
                              cudaMemcpyDeviceToHost, stream_),
              "AudioVAE samples");
  }

  /// Replays (capturing on first use) the decoding of `frames` frames from
  /// the current state half, then flips the halves.
  void Run(std::size_t frames_in) {
    const int frames = static_cast<int>(frames_in);
    Graph* graph = nullptr;
    for (Graph& g : graphs_)
      if (g.frames == frames && g.phase == phase_)
        graph = &g;
    if (graph == nullptr) {
      cudaGraph_t captured = nullptr;
      CudaCheck(cudaStreamBeginCapture(stream_,
                                       cudaStreamCaptureModeThreadLocal),
                "AudioVAE capture");
      try {
        Launches(frames);
        CudaCheck(cudaGetLastError(), "AudioVAE launch");
      } catch (...) {
        cudaStreamEndCapture(stream_, &captured);
        if (captured != nullptr)
          cudaGraphDestroy(captured);
        throw;
      }
      CudaCheck(cudaStreamEndCapture(stream_, &captured), "AudioVAE capture");
      cudaGraphExec_t exec = nullptr;
      const cudaError_t made = cudaGraphInstantiate(&exec, captured, 0);
      cudaGraphDestroy(captured);
      CudaCheck(made, "AudioVAE graph");
      graphs_.push_back({frames, phase_, exec});
      graph = &graphs_.back();
    }
    CudaCheck(cudaGraphLaunch(graph->exec, stream_), "AudioVAE replay");
    phase_ ^= 1;
    pending_ = frames_in * hop_;
  }

  struct Graph {
    int frames;
    int phase;
    cudaGraphExec_t exec;
  };

  vx_vae_config config_;
  VaeLayout layout_;
  std::size_t hop_ = 1;
  cudaStream_t stream_ = nullptr;
  float* weights_ = nullptr;
  std::vector<State> states_;
  int phase_ = 0;  // the state half the next decoding reads
  std::vector<Graph> graphs_;
  std::size_t reserved_ = 0;
  float* latents_ = nullptr;
  float* work_ = nullptr;
  float* hidden_ = nullptr;
  float* scratch_ = nullptr;
  float* samples_ = nullptr;
  float* pinned_ = nullptr;
  std::size_t pending_ = 0;
};

}  // namespace vx

struct vx_audio_vae {
  std::unique_ptr<vx::AudioVae> impl;
};

namespace {

template <typename F>
vx_status VaeGuard(vx_audio_vae* vae, const char* what, F&& body) {
  if (vae == nullptr || !vae->impl)
    return vx::Fail(vx::kInvalid, std::string(what) + ": null AudioVAE");
  try {
    body(*vae->impl);
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

extern "C" {

void vx_vae_config_default(vx_vae_config* c) {
  if (c == nullptr)
    return;
  std::memset(c, 0, sizeof(*c));
  c->latent_dim = 64;
  c->decoder_dim = 2048;
  const std::size_t rates[] = {8, 6, 5, 2, 2, 2};
  for (std::size_t i = 0; i < 6; ++i)
    c->decoder_rates[i] = rates[i];
  c->decoder_rate_count = 6;
  c->out_sample_rate = 48000;
  const std::size_t bounds[] = {20000, 30000, 40000};
  for (std::size_t i = 0; i < 3; ++i)
    c->sr_bin_boundaries[i] = bounds[i];
  c->sr_bin_boundary_count = 3;
}

vx_audio_vae* vx_audio_vae_create(const vx_vae_config* config, uint64_t seed) {
  if (config == nullptr) {
    vx::Fail(vx::kInvalid, "vx_audio_vae_create: null config");
    return nullptr;
  }
  try {
    return new vx_audio_vae{std::make_unique<vx::AudioVae>(*config, seed)};
  } catch (const std::exception& e) {
    vx::Fail(vx::kInvalid, std::string("vx_audio_vae_create: ") + e.what());
    return nullptr;
  }
}

void vx_audio_vae_destroy(vx_audio_vae* vae) { delete vae; }

size_t vx_audio_vae_decode_hop(const vx_audio_vae* vae) {
  return vae != nullptr && vae->impl ? vae->impl->hop() : 0;
}

cudaStream_t vx_audio_vae_stream(const vx_audio_vae* vae) {
  return vae != nullptr && vae->impl ? vae->impl->stream() : nullptr;
}

vx_status vx_audio_vae_reset(vx_audio_vae* vae) {
  return VaeGuard(vae, "vx_audio_vae_reset", [](vx::AudioVae& v) { v.Reset(); });
}

vx_status vx_audio_vae_decode(vx_audio_vae* vae, const float* latents,
                              size_t frames, float* audio) {
  return VaeGuard(vae, "vx_audio_vae_decode", [&](vx::AudioVae& v) {
    if (frames != 0 && (latents == nullptr || audio == nullptr))
      throw std::invalid_argument("null buffer");
    v.Decode(latents, frames, audio);
  });
}

vx_status vx_audio_vae_enqueue(vx_audio_vae* vae, const float* latents,
                               size_t frames, cudaEvent_t ready) {
  return VaeGuard(vae, "vx_audio_vae_enqueue", [&](vx::AudioVae& v) {
    if (frames != 0 && latents == nullptr)
      throw std::invalid_argument("null latents");
    v.Enqueue(latents, frames, ready);
  });
}

vx_status vx_audio_vae_collect(vx_audio_vae* vae, float* audio,
                               size_t capacity, size_t* samples) {
  return VaeGuard(vae, "vx_audio_vae_collect", [&](vx::AudioVae& v) {
    if (samples == nullptr || (capacity != 0 && audio == nullptr))
      throw std::invalid_argument("null buffer");
    *samples = v.Collect(audio, capacity);
  });
}

}  // extern "C"
