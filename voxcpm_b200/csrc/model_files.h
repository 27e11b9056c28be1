// The generator's checkpoint files on the host (model_files.hpp:45-83,
// safetensors.hpp:18-60): a Hugging Face directory (config.json,
// model.safetensors, optional tokenizer.json) or one audio.cpp GGUF file
// (GGUF v2/v3 with the config and tokenizer embedded). Files are mapped
// read-only; tensors point into the mapping.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

struct vx_model_files;  // the C ABI's handle (include/voxcpm_b200.h)

namespace vx {

/// Element types of a checkpoint tensor (safetensors.hpp:18). Q8_0 is GGML's
/// block of 32: an fp16 scale, then 32 int8 values (34 bytes).
enum class DType : int { kF32 = 0, kBF16, kF16, kI64, kI32, kU8, kQ8_0 };

const char* DTypeName(DType dtype);

struct Tensor {
  std::string name;
  DType dtype = DType::kF32;
  std::vector<std::size_t> shape;  // outermost first
  const unsigned char* data = nullptr;
  std::size_t bytes = 0;
  std::uint64_t offset = 0;  // byte position in its file

  std::size_t Elements() const;
};

/// A read-only mapping of a whole file.
class MappedFile {
 public:
  MappedFile() = default;
  ~MappedFile();
  MappedFile(const MappedFile&) = delete;
  MappedFile& operator=(const MappedFile&) = delete;

  /// Maps `path`; throws std::runtime_error naming the file.
  void Open(const std::string& path);
  const unsigned char* data() const { return data_; }
  std::size_t size() const { return size_; }
  /// Drops the resident pages (the mapping stays valid).
  void ReleasePages() const;

 private:
  unsigned char* data_ = nullptr;
  std::size_t size_ = 0;
};

/// A safetensors file: an 8-byte little-endian header length, a JSON header
/// of {name: {dtype, shape, data_offsets}}, then the payload. Tensors come
/// back sorted by name. Throws std::runtime_error on a malformed file
/// (safetensors.cpp:160-222).
std::vector<Tensor> ReadSafetensors(const MappedFile& file);

class GgufFile;

class ModelFiles {
 public:
  /// A directory or a GGUF file; null (and `error`) on failure
  /// (model_files.cpp:111-180).
  static std::unique_ptr<ModelFiles> Open(const std::string& path,
                                          std::string* error);
  /// Whether `path` is a GGUF file of audio.cpp's VoxCPM2 layout
  /// (model_files.cpp:102-109).
  static bool IsVoxCpm2Gguf(const std::string& path);
  ~ModelFiles();

  const std::string& config() const { return config_; }
  const std::string& tokenizer() const { return tokenizer_; }
  bool gguf() const { return gguf_ != nullptr; }
  const Tensor* Model(std::string_view name) const;
  const Tensor* Vae(std::string_view name) const;
  const std::vector<Tensor>& model_tensors() const { return model_; }
  const std::vector<Tensor>& vae_tensors() const { return vae_; }
  void ReleasePages() const;

 private:
  ModelFiles();

  std::string config_;
  std::string tokenizer_;
  std::unique_ptr<MappedFile> safetensors_;
  std::unique_ptr<GgufFile> gguf_;
  std::vector<Tensor> model_;
  std::vector<Tensor> vae_;
  std::unordered_map<std::string, std::size_t> model_index_;
  std::unordered_map<std::string, std::size_t> vae_index_;
};

/// The files behind a C ABI handle (null for a null handle).
const ModelFiles* FilesOf(const vx_model_files* files);

}  // namespace vx
