// Checkpoint files on the host (model_files.h): the mapped file, the
// safetensors reader, the GGUF reader and the audio.cpp VoxCPM2 layout.
//
// GGUF follows the published ggml GGUF specification (versions 2 and 3,
// little-endian): magic "GGUF", version, tensor count, metadata count, the
// metadata key/value pairs, the tensor infos (name, dims innermost first,
// ggml type, offset from the data section), then the data section at the
// next multiple of `general.alignment` (32 when absent). The reference reads
// GGUF through the Gufo SDK's core::GgufReader, which is not part of the
// reference tree; this reader restates the format from the specification.
//
// audio.cpp's layout on top (model_files.cpp:17-180): general.architecture
// "audiocpp" with audiocpp.model_spec.family "voxcpm2"; tensor names under
// "weights/" (the generator) or "audiovae_weights/" (the AudioVAE); a name
// "_audiocpp.<i>" stands for the i-th entry of the string array
// audiocpp.tensor_names; config.json and tokenizer.json are embedded as
// audiocpp.embedded_files.{names, offsets, data} (data holds one byte per
// array element, offsets one more entry than names).
#include "model_files.h"

#include "json.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <fstream>
#include <iterator>
#include <optional>
#include <stdexcept>

namespace vx {

namespace {

class FormatError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

std::size_t DTypeSize(DType dtype) {
  switch (dtype) {
    case DType::kF32:
    case DType::kI32:
      return 4;
    case DType::kBF16:
    case DType::kF16:
      return 2;
    case DType::kI64:
      return 8;
    case DType::kU8:
      return 1;
    case DType::kQ8_0:
      return 34;  // per block of 32
  }
  return 0;
}

/// a * b, or false on overflow.
bool Multiply(std::size_t a, std::size_t b, std::size_t* out) {
  if (a != 0 && b > SIZE_MAX / a)
    return false;
  *out = a * b;
  return true;
}

std::string ReadText(const std::string& path) {
  std::ifstream stream(path, std::ios::binary);
  if (!stream)
    throw FormatError("cannot read " + path);
  return {std::istreambuf_iterator<char>(stream),
          std::istreambuf_iterator<char>()};
}

bool IsFile(const std::string& path) {
  struct stat info {};
  return ::stat(path.c_str(), &info) == 0 && S_ISREG(info.st_mode);
}

bool IsDirectory(const std::string& path) {
  struct stat info {};
  return ::stat(path.c_str(), &info) == 0 && S_ISDIR(info.st_mode);
}

/// No two tensors may share a byte of the file (checked in file order).
void CheckOverlap(const std::vector<Tensor>& tensors) {
  std::vector<const Tensor*> order;
  for (const Tensor& t : tensors)
    order.push_back(&t);
  std::sort(order.begin(), order.end(), [](const Tensor* a, const Tensor* b) {
    return a->offset < b->offset;
  });
  for (std::size_t i = 1; i < order.size(); ++i)
    if (order[i - 1]->offset + order[i - 1]->bytes > order[i]->offset)
      throw FormatError("tensors " + order[i - 1]->name + " and " +
                        order[i]->name + " share bytes of the file");
}

}  // namespace

const char* DTypeName(DType dtype) {
  switch (dtype) {
    case DType::kF32: return "F32";
    case DType::kBF16: return "BF16";
    case DType::kF16: return "F16";
    case DType::kI64: return "I64";
    case DType::kI32: return "I32";
    case DType::kU8: return "U8";
    case DType::kQ8_0: return "Q8_0";
  }
  return "?";
}

std::size_t Tensor::Elements() const {
  std::size_t elements = 1;
  for (const std::size_t size : shape)
    elements *= size;
  return elements;
}

// ------------------------------------------------------------ MappedFile

MappedFile::~MappedFile() {
  if (data_ != nullptr)
    ::munmap(data_, size_);
}

void MappedFile::Open(const std::string& path) {
  const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0)
    throw FormatError("cannot open " + path + ": " + std::strerror(errno));
  struct stat info {};
  if (::fstat(fd, &info) != 0 || !S_ISREG(info.st_mode)) {
    ::close(fd);
    throw FormatError(path + " is not a regular file");
  }
  if (info.st_size == 0) {
    ::close(fd);
    throw FormatError(path + " is empty");
  }
  void* map = ::mmap(nullptr, static_cast<std::size_t>(info.st_size),
                     PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map == MAP_FAILED)
    throw FormatError("cannot map " + path + ": " + std::strerror(errno));
  data_ = static_cast<unsigned char*>(map);
  size_ = static_cast<std::size_t>(info.st_size);
}

void MappedFile::ReleasePages() const {
  if (data_ != nullptr)
    ::madvise(data_, size_, MADV_DONTNEED);
}

// ------------------------------------------------------------ safetensors
//
// The safetensors layout (huggingface/safetensors, the format's README):
//   u64 little-endian N | N bytes of UTF-8 JSON | the data buffer.
// The JSON is an object: "__metadata__" (optional, a string map) and one
// entry per tensor, {"dtype": "F32" | ..., "shape": [d0, d1, ...],
// "data_offsets": [begin, end]} with the offsets relative to the data
// buffer. The format caps N at 100,000,000 bytes.
//
// Reading happens in two passes: the header's entries become declarations
// (name, element type, dimensions, byte range) with each entry checked on
// its own; then the declarations are checked against each other and the
// buffer (ranges inside it, sizes that match, no shared bytes, no repeated
// name) before any becomes a Tensor.

namespace {

constexpr std::uint64_t kSafetensorsHeaderCap = 100'000'000;

/// The element types this library reads from safetensors files.
struct SafetensorsType {
  const char* code;
  DType dtype;
};
constexpr SafetensorsType kSafetensorsTypes[] = {
    {"BF16", DType::kBF16}, {"F16", DType::kF16}, {"F32", DType::kF32},
    {"I32", DType::kI32},   {"I64", DType::kI64}, {"U8", DType::kU8},
};

struct Declared {
  std::string name;
  DType dtype = DType::kU8;
  std::vector<std::size_t> dims;
  std::uint64_t begin = 0;
  std::uint64_t end = 0;
};

[[noreturn]] void BadEntry(const std::string& name, const std::string& why) {
  throw FormatError("safetensors entry \"" + name + "\" " + why);
}

Declared Declare(const std::string& name, const json::Value& entry) {
  if (!entry.is_object())
    BadEntry(name, "must be an object");
  const json::Value* code = entry.find("dtype");
  const json::Value* dims = entry.find("shape");
  const json::Value* range = entry.find("data_offsets");
  if (code == nullptr || dims == nullptr || range == nullptr)
    BadEntry(name, "needs all of dtype, shape and data_offsets");
  Declared d;
  d.name = name;
  const SafetensorsType* type = nullptr;
  if (code->is_string())
    for (const SafetensorsType& t : kSafetensorsTypes)
      if (code->str() == t.code)
        type = &t;
  if (type == nullptr)
    BadEntry(name, "stores elements of type " +
                       (code->is_string() ? code->str() : std::string("?")) +
                       ", which this library does not read");
  d.dtype = type->dtype;
  if (!dims->is_array())
    BadEntry(name, "has a shape that is not a list of sizes");
  for (const json::Value& dim : dims->items()) {
    std::uint64_t extent = 0;
    if (!dim.as_unsigned(&extent))
      BadEntry(name, "has a shape that is not a list of sizes");
    d.dims.push_back(static_cast<std::size_t>(extent));
  }
  if (!range->is_array() || range->items().size() != 2 ||
      !range->items()[0].as_unsigned(&d.begin) ||
      !range->items()[1].as_unsigned(&d.end))
    BadEntry(name, "needs data_offsets of two byte positions");
  return d;
}

/// Bytes a declaration's dimensions and element type take, or false on
/// overflow.
bool DeclaredBytes(const Declared& d, std::size_t* bytes) {
  std::size_t count = 1;
  for (const std::size_t extent : d.dims)
    if (!Multiply(count, extent, &count))
      return false;
  return Multiply(count, DTypeSize(d.dtype), bytes);
}

}  // namespace

std::vector<Tensor> ReadSafetensors(const MappedFile& file) {
  const unsigned char* bytes = file.data();
  const std::size_t size = file.size();
  if (size < 8)
    throw FormatError("safetensors file of " + std::to_string(size) +
                      " bytes is shorter than its 8-byte header length");
  std::uint64_t json_bytes = 0;
  for (int i = 0; i < 8; ++i)
    json_bytes |= static_cast<std::uint64_t>(bytes[i]) << (8 * i);
  if (json_bytes == 0 || json_bytes > kSafetensorsHeaderCap ||
      json_bytes > size - 8)
    throw FormatError("safetensors header length " +
                      std::to_string(json_bytes) +
                      " is implausible: it must be 1..100,000,000 and fit "
                      "in the file");
  json::Value header;
  try {
    header = json::Parse(std::string_view(
        reinterpret_cast<const char*>(bytes + 8), json_bytes));
  } catch (const json::Error& failure) {
    throw FormatError(std::string("safetensors header is not valid JSON (") +
                      failure.what() + ")");
  }
  if (!header.is_object())
    throw FormatError("safetensors header must be a JSON object");
  const std::uint64_t buffer_at = 8 + json_bytes;
  const std::uint64_t buffer_bytes = size - buffer_at;

  // Pass 1: each entry on its own.
  std::vector<Declared> declared;
  for (const auto& [name, entry] : header.members())
    if (name != "__metadata__")
      declared.push_back(Declare(name, entry));
  if (declared.empty())
    throw FormatError("safetensors header declares no tensors");

  // Pass 2: against the buffer and each other, in byte order.
  std::sort(declared.begin(), declared.end(),
            [](const Declared& a, const Declared& b) {
              return a.begin != b.begin ? a.begin < b.begin : a.end < b.end;
            });
  std::vector<Tensor> tensors;
  tensors.reserve(declared.size());
  for (std::size_t i = 0; i < declared.size(); ++i) {
    const Declared& d = declared[i];
    if (d.begin > d.end || d.end > buffer_bytes)
      BadEntry(d.name, "spans bytes " + std::to_string(d.begin) + ".." +
                           std::to_string(d.end) + ", outside the payload of " +
                           std::to_string(buffer_bytes) + " bytes");
    std::size_t need = 0;
    if (!DeclaredBytes(d, &need))
      BadEntry(d.name, "has a shape too large to address");
    if (need != d.end - d.begin)
      BadEntry(d.name, "spans " + std::to_string(d.end - d.begin) +
                           " bytes, but its shape and dtype need " +
                           std::to_string(need));
    if (i > 0 && declared[i - 1].end > d.begin)
      throw FormatError("safetensors entries \"" + declared[i - 1].name +
                        "\" and \"" + d.name + "\" share bytes (their ranges "
                        "overlap)");
    Tensor t;
    t.name = d.name;
    t.dtype = d.dtype;
    t.shape = d.dims;
    t.data = bytes + buffer_at + d.begin;
    t.bytes = need;
    t.offset = buffer_at + d.begin;
    tensors.push_back(std::move(t));
  }
  std::sort(tensors.begin(), tensors.end(),
            [](const Tensor& a, const Tensor& b) { return a.name < b.name; });
  for (std::size_t i = 1; i < tensors.size(); ++i)
    if (tensors[i - 1].name == tensors[i].name)
      BadEntry(tensors[i].name, "appears twice in the header");
  return tensors;
}

// ------------------------------------------------------------ GGUF

namespace {

// GGUF metadata value types.
enum GgufType : std::uint32_t {
  kGgufU8 = 0, kGgufI8 = 1, kGgufU16 = 2, kGgufI16 = 3, kGgufU32 = 4,
  kGgufI32 = 5, kGgufF32 = 6, kGgufBool = 7, kGgufString = 8,
  kGgufArray = 9, kGgufU64 = 10, kGgufI64 = 11, kGgufF64 = 12,
};

std::size_t GgufScalarBytes(std::uint32_t type) {
  switch (type) {
    case kGgufU8: case kGgufI8: case kGgufBool: return 1;
    case kGgufU16: case kGgufI16: return 2;
    case kGgufU32: case kGgufI32: case kGgufF32: return 4;
    case kGgufU64: case kGgufI64: case kGgufF64: return 8;
    default: return 0;
  }
}

bool GgufInteger(std::uint32_t type) {
  return type != kGgufF32 && type != kGgufF64 && type != kGgufBool &&
         GgufScalarBytes(type) != 0;
}

/// ggml tensor types the generator reads: {dtype, values per block, bytes
/// per block}.
struct GgmlType {
  DType dtype;
  std::size_t block;
  std::size_t bytes;
};

std::optional<GgmlType> FromGgml(std::uint32_t type) {
  switch (type) {
    case 0: return GgmlType{DType::kF32, 1, 4};
    case 1: return GgmlType{DType::kF16, 1, 2};
    case 8: return GgmlType{DType::kQ8_0, 32, 34};
    case 26: return GgmlType{DType::kI32, 1, 4};
    case 30: return GgmlType{DType::kBF16, 1, 2};
    default: return std::nullopt;
  }
}

/// Bounds-checked little-endian reads over the mapped file.
class Cursor {
 public:
  Cursor(const unsigned char* data, std::size_t size) : data_(data), size_(size) {}

  template <typename T>
  T Read() {
    Need(sizeof(T));
    T value;
    std::memcpy(&value, data_ + at_, sizeof(T));
    at_ += sizeof(T);
    return value;
  }
  std::string_view String() {
    const std::uint64_t length = Read<std::uint64_t>();
    Need(length);
    std::string_view text(reinterpret_cast<const char*>(data_ + at_), length);
    at_ += length;
    return text;
  }
  const unsigned char* Skip(std::uint64_t bytes) {
    Need(bytes);
    const unsigned char* start = data_ + at_;
    at_ += bytes;
    return start;
  }
  std::size_t at() const { return at_; }
  std::size_t left() const { return size_ - at_; }

 private:
  void Need(std::uint64_t bytes) const {
    if (bytes > size_ - at_)
      throw FormatError("GGUF header runs past the end of the file");
  }
  const unsigned char* data_;
  std::size_t size_;
  std::size_t at_ = 0;
};

}  // namespace

/// One GGUF file: metadata and tensor infos, data pointing into the map.
class GgufFile {
 public:
  struct Meta {
    std::uint32_t type = 0;
    const unsigned char* scalar = nullptr;  // scalar types
    std::string_view text;                  // kGgufString
    std::uint32_t element_type = 0;         // kGgufArray
    std::uint64_t count = 0;
    const unsigned char* elements = nullptr;  // numeric arrays
    std::vector<std::string_view> strings;    // string arrays
  };
  struct Info {
    std::string name;
    std::uint32_t type = 0;
    std::vector<std::uint64_t> dims;  // innermost first
    std::uint64_t offset = 0;
    const unsigned char* data = nullptr;
    std::size_t bytes = 0;
  };

  explicit GgufFile(const std::string& path) {
    file_.Open(path);
    Parse();
  }

  const Meta* Find(std::string_view key) const {
    const auto found = meta_.find(std::string(key));
    return found == meta_.end() ? nullptr : &found->second;
  }
  std::optional<std::string_view> String(std::string_view key) const {
    const Meta* m = Find(key);
    if (m == nullptr || m->type != kGgufString)
      return std::nullopt;
    return m->text;
  }
  std::vector<std::string_view> Strings(std::string_view key) const {
    const Meta* m = Find(key);
    if (m == nullptr || m->type != kGgufArray || m->element_type != kGgufString)
      throw FormatError("GGUF lacks the string array " + std::string(key));
    return m->strings;
  }
  /// Element `index` of an integer array as a signed 64-bit value.
  static std::int64_t Element(const Meta& m, std::uint64_t index) {
    const unsigned char* p = m.elements + index * GgufScalarBytes(m.element_type);
    switch (m.element_type) {
      case kGgufU8: return *p;
      case kGgufI8: return static_cast<std::int8_t>(*p);
      case kGgufU16: { std::uint16_t v; std::memcpy(&v, p, 2); return v; }
      case kGgufI16: { std::int16_t v; std::memcpy(&v, p, 2); return v; }
      case kGgufU32: { std::uint32_t v; std::memcpy(&v, p, 4); return v; }
      case kGgufI32: { std::int32_t v; std::memcpy(&v, p, 4); return v; }
      case kGgufU64: { std::uint64_t v; std::memcpy(&v, p, 8); return static_cast<std::int64_t>(v); }
      default: { std::int64_t v; std::memcpy(&v, p, 8); return v; }
    }
  }
  const Meta& IntegerArray(std::string_view key) const {
    const Meta* m = Find(key);
    if (m == nullptr)
      throw FormatError("GGUF lacks " + std::string(key));
    if (m->type != kGgufArray || !GgufInteger(m->element_type))
      throw FormatError("GGUF " + std::string(key) + " is not an integer array");
    return *m;
  }
  const std::vector<Info>& tensors() const { return tensors_; }
  std::uint32_t version() const { return version_; }

 private:
  void Value(Cursor& c, std::uint32_t type, Meta* out, int depth) {
    if (depth > 8)
      throw FormatError("GGUF metadata nests too deeply");
    if (type == kGgufString) {
      const std::string_view text = c.String();
      if (out != nullptr)
        out->text = text;
    } else if (type == kGgufArray) {
      const std::uint32_t element = c.Read<std::uint32_t>();
      const std::uint64_t count = c.Read<std::uint64_t>();
      if (out != nullptr) {
        out->element_type = element;
        out->count = count;
      }
      const std::size_t scalar = GgufScalarBytes(element);
      if (scalar != 0) {
        if (count > c.left() / scalar)
          throw FormatError("GGUF array runs past the end of the file");
        const unsigned char* first = c.Skip(count * scalar);
        if (out != nullptr)
          out->elements = first;
      } else if (element == kGgufString || element == kGgufArray) {
        // Each element takes at least 8 bytes.
        if (count > c.left() / 8)
          throw FormatError("GGUF array runs past the end of the file");
        for (std::uint64_t i = 0; i < count; ++i) {
          if (element == kGgufString) {
            const std::string_view text = c.String();
            if (out != nullptr)
              out->strings.push_back(text);
          } else {
            Value(c, kGgufArray, nullptr, depth + 1);
          }
        }
      } else {
        throw FormatError("GGUF array has the unknown type " +
                          std::to_string(element));
      }
    } else {
      const std::size_t scalar = GgufScalarBytes(type);
      if (scalar == 0)
        throw FormatError("GGUF metadata has the unknown type " +
                          std::to_string(type));
      const unsigned char* p = c.Skip(scalar);
      if (out != nullptr)
        out->scalar = p;
    }
  }

  void Parse() {
    Cursor c(file_.data(), file_.size());
    if (file_.size() < 24 || std::memcmp(file_.data(), "GGUF", 4) != 0)
      throw FormatError("not a GGUF file");
    c.Skip(4);
    version_ = c.Read<std::uint32_t>();
    if (version_ != 2 && version_ != 3)
      throw FormatError("unsupported GGUF version " + std::to_string(version_) +
                        " (little-endian 2 and 3 are read)");
    const std::uint64_t tensor_count = c.Read<std::uint64_t>();
    const std::uint64_t meta_count = c.Read<std::uint64_t>();
    // A key/value pair takes at least 13 bytes, a tensor info 24.
    if (meta_count > c.left() / 13 || tensor_count > c.left() / 24)
      throw FormatError("GGUF counts exceed the file");
    for (std::uint64_t i = 0; i < meta_count; ++i) {
      std::string key(c.String());
      Meta m;
      m.type = c.Read<std::uint32_t>();
      Value(c, m.type, &m, 0);
      meta_[key] = std::move(m);
    }
    std::uint64_t alignment = 32;
    if (const Meta* a = Find("general.alignment")) {
      if (a->scalar == nullptr || !GgufInteger(a->type))
        throw FormatError("GGUF general.alignment is not an integer");
      std::uint64_t v = 0;
      std::memcpy(&v, a->scalar, GgufScalarBytes(a->type));
      alignment = v;
      if (alignment == 0 || alignment > (1u << 20))
        throw FormatError("GGUF general.alignment is implausible");
    }
    for (std::uint64_t i = 0; i < tensor_count; ++i) {
      Info info;
      info.name = std::string(c.String());
      const std::uint32_t dims = c.Read<std::uint32_t>();
      if (dims > 4)
        throw FormatError("GGUF tensor " + info.name + " has " +
                          std::to_string(dims) + " dimensions");
      for (std::uint32_t d = 0; d < dims; ++d)
        info.dims.push_back(c.Read<std::uint64_t>());
      info.type = c.Read<std::uint32_t>();
      info.offset = c.Read<std::uint64_t>();
      tensors_.push_back(std::move(info));
    }
    const std::size_t data_at = (c.at() + alignment - 1) / alignment * alignment;
    if (data_at > file_.size())
      throw FormatError("GGUF data section starts past the end of the file");
    const std::size_t data_bytes = file_.size() - data_at;
    std::vector<Tensor> spans;
    for (Info& info : tensors_) {
      const auto type = FromGgml(info.type);
      if (!type.has_value())
        throw FormatError("GGUF tensor " + info.name +
                          " has an unsupported type " + std::to_string(info.type));
      std::size_t elements = 1;
      for (const std::uint64_t d : info.dims)
        if (!Multiply(elements, d, &elements))
          throw FormatError("GGUF tensor " + info.name + " is too large");
      if (!info.dims.empty() && info.dims[0] % type->block != 0)
        throw FormatError("GGUF tensor " + info.name +
                          " does not fill whole blocks");
      if (!Multiply(elements / type->block, type->bytes, &info.bytes))
        throw FormatError("GGUF tensor " + info.name + " is too large");
      if (info.offset % alignment != 0 || info.offset > data_bytes ||
          info.bytes > data_bytes - info.offset)
        throw FormatError("GGUF tensor " + info.name +
                          " lies outside the data section");
      info.data = file_.data() + data_at + info.offset;
      Tensor span;
      span.name = info.name;
      span.offset = info.offset;
      span.bytes = info.bytes;
      spans.push_back(std::move(span));
    }
    CheckOverlap(spans);
    for (Info& info : tensors_)
      info.offset += data_at;
  }

  MappedFile file_;
  std::uint32_t version_ = 0;
  std::unordered_map<std::string, Meta> meta_;
  std::vector<Info> tensors_;

 public:
  void ReleasePages() const { file_.ReleasePages(); }
};

// ------------------------------------------------------------ ModelFiles

namespace {

constexpr std::string_view kModelPrefix = "weights/";
constexpr std::string_view kVaePrefix = "audiovae_weights/";
constexpr std::string_view kAbbreviated = "_audiocpp.";

bool IsVoxCpm2(const GgufFile& gguf) {
  return gguf.String("general.architecture") ==
             std::optional<std::string_view>("audiocpp") &&
         gguf.String("audiocpp.model_spec.family") ==
             std::optional<std::string_view>("voxcpm2");
}

/// An embedded file of an audio.cpp GGUF (model_files.cpp:71-93).
std::string Embedded(const GgufFile& gguf, std::string_view name) {
  const std::vector<std::string_view> names =
      gguf.Strings("audiocpp.embedded_files.names");
  const GgufFile::Meta& offsets =
      gguf.IntegerArray("audiocpp.embedded_files.offsets");
  const GgufFile::Meta& data = gguf.IntegerArray("audiocpp.embedded_files.data");
  for (std::size_t index = 0; index < names.size(); ++index) {
    if (names[index] != name)
      continue;
    if (index + 1 >= offsets.count)
      throw FormatError("GGUF embedded file table is malformed");
    const std::int64_t begin = GgufFile::Element(offsets, index);
    const std::int64_t end = GgufFile::Element(offsets, index + 1);
    if (begin < 0 || begin > end || static_cast<std::uint64_t>(end) > data.count)
      throw FormatError("GGUF embedded file table is malformed");
    std::string text;
    text.reserve(static_cast<std::size_t>(end - begin));
    if (GgufScalarBytes(data.element_type) == 1) {
      text.assign(reinterpret_cast<const char*>(data.elements) + begin,
                  static_cast<std::size_t>(end - begin));
    } else {
      for (std::int64_t at = begin; at < end; ++at)
        text.push_back(static_cast<char>(GgufFile::Element(data, at)));
    }
    return text;
  }
  throw FormatError("GGUF lacks the embedded " + std::string(name));
}

}  // namespace

ModelFiles::ModelFiles() = default;
ModelFiles::~ModelFiles() = default;

bool ModelFiles::IsVoxCpm2Gguf(const std::string& path) {
  if (!IsFile(path) || path.size() < 5 ||
      path.compare(path.size() - 5, 5, ".gguf") != 0)
    return false;
  try {
    return IsVoxCpm2(GgufFile(path));
  } catch (const std::exception&) {
    return false;
  }
}

std::unique_ptr<ModelFiles> ModelFiles::Open(const std::string& path,
                                             std::string* error) {
  std::unique_ptr<ModelFiles> files(new ModelFiles());
  try {
    if (IsDirectory(path)) {
      // The AudioVAE's audiovae.pth is not read: the AudioVAE is not part
      // of the generator.
      files->config_ = ReadText(path + "/config.json");
      if (IsFile(path + "/tokenizer.json"))
        files->tokenizer_ = ReadText(path + "/tokenizer.json");
      const std::string weights = path + "/model.safetensors";
      files->safetensors_ = std::make_unique<MappedFile>();
      files->safetensors_->Open(weights);
      try {
        files->model_ = ReadSafetensors(*files->safetensors_);
      } catch (const std::exception& failure) {
        throw FormatError(weights + ": " + failure.what());
      }
    } else {
      try {
        files->gguf_ = std::make_unique<GgufFile>(path);
      } catch (const std::exception& failure) {
        throw FormatError(path + ": " + failure.what());
      }
      const GgufFile& gguf = *files->gguf_;
      if (!IsVoxCpm2(gguf))
        throw FormatError(path + " is not an audio.cpp VoxCPM2 GGUF");
      files->config_ = Embedded(gguf, "config.json");
      files->tokenizer_ = Embedded(gguf, "tokenizer.json");
      const std::vector<std::string_view> names =
          gguf.Find("audiocpp.tensor_names") != nullptr
              ? gguf.Strings("audiocpp.tensor_names")
              : std::vector<std::string_view>();
      for (const GgufFile::Info& info : gguf.tensors()) {
        std::string name = info.name;
        if (name.compare(0, kAbbreviated.size(), kAbbreviated) == 0) {
          const std::string digits = name.substr(kAbbreviated.size());
          if (digits.empty() || digits.size() > 18 ||
              digits.find_first_not_of("0123456789") != std::string::npos)
            throw FormatError("GGUF tensor " + name + " has a malformed index");
          const std::size_t index = std::stoull(digits);
          if (index >= names.size())
            throw FormatError("GGUF tensor " + name + " has no listed name");
          name = std::string(names[index]);
        }
        Tensor tensor;
        tensor.dtype = FromGgml(info.type)->dtype;
        for (auto it = info.dims.rbegin(); it != info.dims.rend(); ++it)
          tensor.shape.push_back(static_cast<std::size_t>(*it));
        tensor.data = info.data;
        tensor.bytes = info.bytes;
        tensor.offset = info.offset;
        if (name.compare(0, kModelPrefix.size(), kModelPrefix) == 0) {
          tensor.name = name.substr(kModelPrefix.size());
          files->model_.push_back(std::move(tensor));
        } else if (name.compare(0, kVaePrefix.size(), kVaePrefix) == 0) {
          tensor.name = name.substr(kVaePrefix.size());
          files->vae_.push_back(std::move(tensor));
        } else {
          throw FormatError("GGUF tensor " + name + " belongs to no component");
        }
      }
    }
    for (std::size_t i = 0; i < files->model_.size(); ++i)
      if (!files->model_index_.emplace(files->model_[i].name, i).second)
        throw FormatError("the checkpoint names " + files->model_[i].name +
                          " twice");
    for (std::size_t i = 0; i < files->vae_.size(); ++i)
      if (!files->vae_index_.emplace(files->vae_[i].name, i).second)
        throw FormatError("the checkpoint names " + files->vae_[i].name +
                          " twice");
  } catch (const std::exception& failure) {
    if (error != nullptr)
      *error = failure.what();
    return nullptr;
  }
  return files;
}

const Tensor* ModelFiles::Model(std::string_view name) const {
  const auto found = model_index_.find(std::string(name));
  return found == model_index_.end() ? nullptr : &model_[found->second];
}

const Tensor* ModelFiles::Vae(std::string_view name) const {
  const auto found = vae_index_.find(std::string(name));
  return found == vae_index_.end() ? nullptr : &vae_[found->second];
}

void ModelFiles::ReleasePages() const {
  if (safetensors_ != nullptr)
    safetensors_->ReleasePages();
  if (gguf_ != nullptr)
    gguf_->ReleasePages();
}

}  // namespace vx
