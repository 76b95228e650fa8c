// Minimal JSON DOM reader for AtlasIR documents.
//
// AtlasIR carries every model float as a hex string, so JSON numbers only hold
// integers (counts, indices, ticks, seeds) and SI dimension exponents.  Numbers
// therefore keep their source text: integers are decoded exactly as u64/i64 and
// the rare real number through strtod (correctly rounded in glibc).
#pragma once

#include <cerrno>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace b2json {

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

class Value {
 public:
  enum class Type : uint8_t { Null, Bool, Number, String, Array, Object };

  Value() = default;
  Type type() const { return type_; }
  bool is_null() const { return type_ == Type::Null; }
  bool is_string() const { return type_ == Type::String; }
  bool is_array() const { return type_ == Type::Array; }
  bool is_object() const { return type_ == Type::Object; }
  bool is_number() const { return type_ == Type::Number; }
  bool is_bool() const { return type_ == Type::Bool; }

  const std::string& str() const {
    if (type_ != Type::String) throw Error("JSON value is not a string");
    return text_;
  }
  bool boolean() const {
    if (type_ != Type::Bool) throw Error("JSON value is not a bool");
    return bool_;
  }
  uint64_t u64() const {
    if (type_ != Type::Number || text_.empty() || text_[0] == '-')
      throw Error("JSON value is not an unsigned integer");
    for (char c : text_)
      if (c < '0' || c > '9') throw Error("JSON value is not an unsigned integer");
    errno = 0;
    unsigned long long v = std::strtoull(text_.c_str(), nullptr, 10);
    if (errno) throw Error("JSON integer out of range");
    return v;
  }
  int64_t i64() const {
    if (type_ != Type::Number) throw Error("JSON value is not an integer");
    size_t start = (!text_.empty() && text_[0] == '-') ? 1 : 0;
    if (start == text_.size()) throw Error("JSON value is not an integer");
    for (size_t i = start; i < text_.size(); ++i)
      if (text_[i] < '0' || text_[i] > '9') throw Error("JSON value is not an integer");
    errno = 0;
    long long v = std::strtoll(text_.c_str(), nullptr, 10);
    if (errno) throw Error("JSON integer out of range");
    return v;
  }
  double real() const {
    if (type_ != Type::Number) throw Error("JSON value is not a number");
    return std::strtod(text_.c_str(), nullptr);
  }
  const std::string& number_text() const { return text_; }

  const std::vector<Value>& arr() const {
    if (type_ != Type::Array) throw Error("JSON value is not an array");
    return items_;
  }
  const std::vector<std::pair<std::string, Value>>& obj() const {
    if (type_ != Type::Object) throw Error("JSON value is not an object");
    return members_;
  }
  // Object member lookup; nullptr when absent.
  const Value* find(const char* key) const {
    if (type_ != Type::Object) throw Error("JSON value is not an object");
    for (const auto& kv : members_)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
  const Value& at(const char* key) const {
    const Value* v = find(key);
    if (!v) throw Error(std::string("missing JSON field '") + key + "'");
    return *v;
  }
  // True when the key is absent or explicitly null.
  bool absent(const char* key) const {
    const Value* v = find(key);
    return !v || v->is_null();
  }

  // ---- editing (schema migrations rewrite a parsed document in place)
  static Value string(std::string s) {
    Value v;
    v.type_ = Type::String;
    v.text_ = std::move(s);
    return v;
  }
  static Value array() {
    Value v;
    v.type_ = Type::Array;
    return v;
  }
  static Value object() {
    Value v;
    v.type_ = Type::Object;
    return v;
  }
  std::vector<Value>& arr_mut() {
    if (type_ != Type::Array) throw Error("JSON value is not an array");
    return items_;
  }
  Value* find_mut(const char* key) {
    if (type_ != Type::Object) throw Error("JSON value is not an object");
    for (auto& kv : members_)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
  // Replace the member's value, or append the member.
  void set(const char* key, Value v) {
    if (Value* old = find_mut(key)) *old = std::move(v);
    else members_.emplace_back(key, std::move(v));
  }

 private:
  friend class Parser;
  Type type_ = Type::Null;
  bool bool_ = false;
  std::string text_;
  std::vector<Value> items_;
  std::vector<std::pair<std::string, Value>> members_;
};

class Parser {
 public:
  Parser(const char* data, size_t size) : p_(data), end_(data + size) {}

  Value parse_document() {
    Value v;
    skip_ws();
    parse_value(v, 0);
    skip_ws();
    if (p_ != end_) fail("trailing characters after JSON document");
    return v;
  }

 private:
  const char* p_;
  const char* end_;

  [[noreturn]] void fail(const char* what) { throw Error(std::string("JSON parse error: ") + what); }

  void skip_ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }

  void expect(char c) {
    if (p_ >= end_ || *p_ != c) fail("unexpected character");
    ++p_;
  }

  void parse_value(Value& out, int depth) {
    if (depth > 512) fail("nesting too deep");
    if (p_ >= end_) fail("unexpected end of input");
    switch (*p_) {
      case '{': parse_object(out, depth); return;
      case '[': parse_array(out, depth); return;
      case '"': out.type_ = Value::Type::String; parse_string(out.text_); return;
      case 't': literal("true"); out.type_ = Value::Type::Bool; out.bool_ = true; return;
      case 'f': literal("false"); out.type_ = Value::Type::Bool; out.bool_ = false; return;
      case 'n': literal("null"); out.type_ = Value::Type::Null; return;
      default: parse_number(out); return;
    }
  }

  void literal(const char* word) {
    size_t n = std::strlen(word);
    if (size_t(end_ - p_) < n || std::memcmp(p_, word, n) != 0) fail("invalid literal");
    p_ += n;
  }

  void parse_number(Value& out) {
    const char* start = p_;
    if (p_ < end_ && *p_ == '-') ++p_;
    if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) fail("invalid number");
    while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                         *p_ == '+' || *p_ == '-'))
      ++p_;
    out.type_ = Value::Type::Number;
    out.text_.assign(start, p_);
  }

  static void put_utf8(std::string& s, uint32_t cp) {
    if (cp < 0x80) {
      s.push_back(char(cp));
    } else if (cp < 0x800) {
      s.push_back(char(0xC0 | (cp >> 6)));
      s.push_back(char(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
      s.push_back(char(0xE0 | (cp >> 12)));
      s.push_back(char(0x80 | ((cp >> 6) & 0x3F)));
      s.push_back(char(0x80 | (cp & 0x3F)));
    } else {
      s.push_back(char(0xF0 | (cp >> 18)));
      s.push_back(char(0x80 | ((cp >> 12) & 0x3F)));
      s.push_back(char(0x80 | ((cp >> 6) & 0x3F)));
      s.push_back(char(0x80 | (cp & 0x3F)));
    }
  }

  uint32_t hex4() {
    if (end_ - p_ < 4) fail("short unicode escape");
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) {
      char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= uint32_t(c - '0');
      else if (c >= 'a' && c <= 'f') v |= uint32_t(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= uint32_t(c - 'A' + 10);
      else fail("invalid unicode escape");
    }
    return v;
  }

  void parse_string(std::string& out) {
    expect('"');
    const char* run = p_;
    while (true) {
      if (p_ >= end_) fail("unterminated string");
      char c = *p_;
      if (c == '"') {
        out.append(run, p_);
        ++p_;
        return;
      }
      if (c == '\\') {
        out.append(run, p_);
        ++p_;
        if (p_ >= end_) fail("unterminated escape");
        char e = *p_++;
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
            uint32_t cp = hex4();
            if (cp >= 0xD800 && cp < 0xDC00) {
              if (end_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') fail("unpaired surrogate");
              p_ += 2;
              uint32_t lo = hex4();
              if (lo < 0xDC00 || lo >= 0xE000) fail("invalid surrogate pair");
              cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            }
            put_utf8(out, cp);
            break;
          }
          default: fail("invalid escape");
        }
        run = p_;
        continue;
      }
      if (static_cast<unsigned char>(c) < 0x20) fail("control character in string");
      ++p_;
    }
  }

  void parse_array(Value& out, int depth) {
    expect('[');
    out.type_ = Value::Type::Array;
    skip_ws();
    if (p_ < end_ && *p_ == ']') {
      ++p_;
      return;
    }
    while (true) {
      skip_ws();
      out.items_.emplace_back();
      parse_value(out.items_.back(), depth + 1);
      skip_ws();
      if (p_ < end_ && *p_ == ',') {
        ++p_;
        continue;
      }
      expect(']');
      return;
    }
  }

  void parse_object(Value& out, int depth) {
    expect('{');
    out.type_ = Value::Type::Object;
    skip_ws();
    if (p_ < end_ && *p_ == '}') {
      ++p_;
      return;
    }
    while (true) {
      skip_ws();
      std::string key;
      parse_string(key);
      skip_ws();
      expect(':');
      skip_ws();
      out.members_.emplace_back(std::move(key), Value());
      parse_value(out.members_.back().second, depth + 1);
      skip_ws();
      if (p_ < end_ && *p_ == ',') {
        ++p_;
        continue;
      }
      expect('}');
      return;
    }
  }
};

inline Value parse(const char* data, size_t size) { return Parser(data, size).parse_document(); }
inline Value parse(const std::string& s) { return parse(s.data(), s.size()); }

}  // namespace b2json
