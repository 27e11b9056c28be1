// JSON reader (json.h): recursive descent over RFC 8259 with a nesting
// limit, \u escapes (surrogate pairs included) decoded to UTF-8.
#include "json.h"

#include <cerrno>
#include <cstdlib>
#include <cstring>

namespace vx::json {

namespace {
constexpr int kMaxDepth = 256;
}  // namespace

const Value* Value::find(std::string_view key) const {
  const Value* found = nullptr;
  for (const auto& member : members_)
    if (member.first == key)
      found = &member.second;
  return found;
}

class Parser {
 public:
  explicit Parser(std::string_view text) : text_(text) {}

  Value Document() {
    Value value = Any(0);
    Space();
    if (at_ != text_.size())
      Fail("trailing characters");
    return value;
  }

 private:
  [[noreturn]] void Fail(const std::string& what) const {
    throw Error("JSON " + what + " at byte " + std::to_string(at_));
  }

  void Space() {
    while (at_ < text_.size() && (text_[at_] == ' ' || text_[at_] == '\t' ||
                                  text_[at_] == '\n' || text_[at_] == '\r'))
      ++at_;
  }

  char Peek() {
    Space();
    if (at_ >= text_.size())
      Fail("ends early");
    return text_[at_];
  }

  void Expect(char c) {
    if (Peek() != c)
      Fail(std::string("expects '") + c + "'");
    ++at_;
  }

  void Word(std::string_view word) {
    if (text_.substr(at_, word.size()) != word)
      Fail("has an unknown literal");
    at_ += word.size();
  }

  Value Any(int depth) {
    if (depth > kMaxDepth)
      Fail("nests too deeply");
    Value value;
    switch (Peek()) {
      case '{':
        value.kind_ = Value::Kind::kObject;
        ++at_;
        if (Peek() == '}') {
          ++at_;
          return value;
        }
        for (;;) {
          if (Peek() != '"')
            Fail("expects a member name");
          std::string key = String();
          Expect(':');
          value.members_.emplace_back(std::move(key), Any(depth + 1));
          const char c = Peek();
          ++at_;
          if (c == '}')
            return value;
          if (c != ',')
            Fail("expects ',' or '}'");
        }
      case '[':
        value.kind_ = Value::Kind::kArray;
        ++at_;
        if (Peek() == ']') {
          ++at_;
          return value;
        }
        for (;;) {
          value.items_.push_back(Any(depth + 1));
          const char c = Peek();
          ++at_;
          if (c == ']')
            return value;
          if (c != ',')
            Fail("expects ',' or ']'");
        }
      case '"':
        value.kind_ = Value::Kind::kString;
        value.text_ = String();
        return value;
      case 't':
        Word("true");
        value.kind_ = Value::Kind::kBool;
        value.boolean_ = true;
        return value;
      case 'f':
        Word("false");
        value.kind_ = Value::Kind::kBool;
        return value;
      case 'n':
        Word("null");
        return value;
      default:
        return Number();
    }
  }

  Value Number() {
    const std::size_t start = at_;
    bool integral = true;
    if (at_ < text_.size() && text_[at_] == '-') {
      integral = false;
      ++at_;
    }
    const std::size_t digits = at_;
    while (at_ < text_.size() && text_[at_] >= '0' && text_[at_] <= '9')
      ++at_;
    if (at_ == digits)
      Fail("has a malformed number");
    if (text_[digits] == '0' && at_ - digits > 1)
      Fail("has a number with a leading zero");
    if (at_ < text_.size() && text_[at_] == '.') {
      integral = false;
      const std::size_t fraction = ++at_;
      while (at_ < text_.size() && text_[at_] >= '0' && text_[at_] <= '9')
        ++at_;
      if (at_ == fraction)
        Fail("has a malformed fraction");
    }
    if (at_ < text_.size() && (text_[at_] == 'e' || text_[at_] == 'E')) {
      integral = false;
      ++at_;
      if (at_ < text_.size() && (text_[at_] == '+' || text_[at_] == '-'))
        ++at_;
      const std::size_t exponent = at_;
      while (at_ < text_.size() && text_[at_] >= '0' && text_[at_] <= '9')
        ++at_;
      if (at_ == exponent)
        Fail("has a malformed exponent");
    }
    const std::string token(text_.substr(start, at_ - start));
    Value value;
    value.kind_ = Value::Kind::kNumber;
    value.number_ = std::strtod(token.c_str(), nullptr);
    if (integral) {
      errno = 0;
      const unsigned long long u = std::strtoull(token.c_str(), nullptr, 10);
      value.integral_ = errno == 0;
      value.unsigned_ = u;
    }
    return value;
  }

  unsigned Hex4() {
    if (at_ + 4 > text_.size())
      Fail("has a short \\u escape");
    unsigned code = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = text_[at_++];
      code <<= 4;
      if (c >= '0' && c <= '9')
        code |= static_cast<unsigned>(c - '0');
      else if (c >= 'a' && c <= 'f')
        code |= static_cast<unsigned>(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F')
        code |= static_cast<unsigned>(c - 'A' + 10);
      else
        Fail("has a bad \\u escape");
    }
    return code;
  }

  static void Utf8(unsigned code, std::string& out) {
    if (code < 0x80) {
      out.push_back(static_cast<char>(code));
    } else if (code < 0x800) {
      out.push_back(static_cast<char>(0xC0 | (code >> 6)));
      out.push_back(static_cast<char>(0x80 | (code & 0x3F)));
    } else if (code < 0x10000) {
      out.push_back(static_cast<char>(0xE0 | (code >> 12)));
      out.push_back(static_cast<char>(0x80 | ((code >> 6) & 0x3F)));
      out.push_back(static_cast<char>(0x80 | (code & 0x3F)));
    } else {
      out.push_back(static_cast<char>(0xF0 | (code >> 18)));
      out.push_back(static_cast<char>(0x80 | ((code >> 12) & 0x3F)));
      out.push_back(static_cast<char>(0x80 | ((code >> 6) & 0x3F)));
      out.push_back(static_cast<char>(0x80 | (code & 0x3F)));
    }
  }

  std::string String() {
    ++at_;  // the opening quote
    std::string out;
    for (;;) {
      if (at_ >= text_.size())
        Fail("has an unterminated string");
      const char c = text_[at_++];
      if (c == '"')
        return out;
      if (static_cast<unsigned char>(c) < 0x20)
        Fail("has a control character in a string");
      if (c != '\\') {
        out.push_back(c);
        continue;
      }
      if (at_ >= text_.size())
        Fail("has an unterminated escape");
      const char e = text_[at_++];
      switch (e) {
        case '"': out.push_back('"'); break;
        case '\\': out.push_back('\\'); break;
        case '/': out.push_back('/'); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': {
          unsigned code = Hex4();
          if (code >= 0xD800 && code < 0xDC00) {
            if (text_.substr(at_, 2) != "\\u")
              Fail("has an unpaired surrogate");
            at_ += 2;
            const unsigned low = Hex4();
            if (low < 0xDC00 || low >= 0xE000)
              Fail("has an unpaired surrogate");
            code = 0x10000 + ((code - 0xD800) << 10) + (low - 0xDC00);
          } else if (code >= 0xDC00 && code < 0xE000) {
            Fail("has an unpaired surrogate");
          }
          Utf8(code, out);
          break;
        }
        default:
          Fail("has an unknown escape");
      }
    }
  }

  std::string_view text_;
  std::size_t at_ = 0;
};

Value Parse(std::string_view text) { return Parser(text).Document(); }

}  // namespace vx::json
