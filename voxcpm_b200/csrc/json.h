// A small JSON reader for the model files' text parts: safetensors headers
// and config.json (RFC 8259). Objects keep their members in file order;
// numbers keep the exact unsigned value when written as a plain integer, so
// byte offsets above 2^53 stay exact.
#pragma once

#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

namespace vx::json {

class Error : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

class Value {
 public:
  enum class Kind { kNull, kBool, kNumber, kString, kArray, kObject };

  Kind kind() const { return kind_; }
  bool is_null() const { return kind_ == Kind::kNull; }
  bool is_bool() const { return kind_ == Kind::kBool; }
  bool is_number() const { return kind_ == Kind::kNumber; }
  bool is_string() const { return kind_ == Kind::kString; }
  bool is_array() const { return kind_ == Kind::kArray; }
  bool is_object() const { return kind_ == Kind::kObject; }

  bool as_bool() const { return boolean_; }
  double as_double() const { return number_; }
  /// The value as a non-negative integer, when it was written as one.
  bool as_unsigned(std::uint64_t* out) const {
    if (!is_number() || !integral_)
      return false;
    *out = unsigned_;
    return true;
  }
  const std::string& str() const { return text_; }
  const std::vector<Value>& items() const { return items_; }
  const std::vector<std::pair<std::string, Value>>& members() const {
    return members_;
  }
  /// The member named `key` (the last one when repeated), or null.
  const Value* find(std::string_view key) const;

 private:
  friend class Parser;
  Kind kind_ = Kind::kNull;
  bool boolean_ = false;
  bool integral_ = false;
  double number_ = 0.0;
  std::uint64_t unsigned_ = 0;
  std::string text_;
  std::vector<Value> items_;
  std::vector<std::pair<std::string, Value>> members_;
};

/// Parses one JSON document (surrounding white space allowed). Throws Error
/// with the byte position of the first problem.
Value Parse(std::string_view text);

}  // namespace vx::json
