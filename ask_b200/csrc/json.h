// Minimal JSON reader for plan recipes (objects, arrays, strings, numbers,
// true/false/null).  Integers are kept exactly as int64 alongside their double
// value so element counts and constant bit patterns survive unchanged.
#pragma once

#include <stdint.h>

#include <cerrno>
#include <cstdlib>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace askb {
namespace json {

struct Value {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  int64_t integer = 0;
  bool is_integer = false;
  bool negative = false;  // the literal had a minus sign (integer may hold a u64 above INT64_MAX)
  std::string str;
  std::vector<Value> items;
  std::vector<std::pair<std::string, Value>> fields;

  const Value* get(const std::string& key) const {
    for (const auto& f : fields)
      if (f.first == key) return &f.second;
    return nullptr;
  }
  const Value& at(const std::string& key) const {
    const Value* v = get(key);
    if (!v) throw std::runtime_error("recipe field '" + key + "' is missing");
    return *v;
  }
  int64_t as_int(const char* what) const {
    if (kind != Number || !is_integer) throw std::runtime_error(std::string(what) + " must be an integer");
    return integer;
  }
  const std::string& as_str(const char* what) const {
    if (kind != String) throw std::runtime_error(std::string(what) + " must be a string");
    return str;
  }
  const std::vector<Value>& as_array(const char* what) const {
    if (kind != Array) throw std::runtime_error(std::string(what) + " must be an array");
    return items;
  }
};

class Parser {
 public:
  explicit Parser(const char* text) : p_(text) {}
  Value parse() {
    Value v = value();
    ws();
    if (*p_) fail("trailing characters");
    return v;
  }

 private:
  const char* p_;
  int depth_ = 0;

  [[noreturn]] void fail(const char* why) { throw std::runtime_error(std::string("recipe JSON: ") + why); }
  void ws() {
    while (*p_ == ' ' || *p_ == '\n' || *p_ == '\t' || *p_ == '\r') ++p_;
  }
  bool lit(const char* s) {
    size_t n = 0;
    while (s[n]) ++n;
    for (size_t i = 0; i < n; ++i)
      if (p_[i] != s[i]) return false;
    p_ += n;
    return true;
  }
  Value value() {
    if (++depth_ > 64) fail("nesting too deep");
    ws();
    Value v;
    if (*p_ == '{') {
      ++p_;
      v.kind = Value::Object;
      ws();
      if (*p_ == '}') { ++p_; --depth_; return v; }
      for (;;) {
        ws();
        if (*p_ != '"') fail("expected key");
        std::string key = string();
        ws();
        if (*p_ != ':') fail("expected ':'");
        ++p_;
        v.fields.emplace_back(std::move(key), value());
        ws();
        if (*p_ == ',') { ++p_; continue; }
        if (*p_ == '}') { ++p_; break; }
        fail("expected ',' or '}'");
      }
    } else if (*p_ == '[') {
      ++p_;
      v.kind = Value::Array;
      ws();
      if (*p_ == ']') { ++p_; --depth_; return v; }
      for (;;) {
        v.items.push_back(value());
        ws();
        if (*p_ == ',') { ++p_; continue; }
        if (*p_ == ']') { ++p_; break; }
        fail("expected ',' or ']'");
      }
    } else if (*p_ == '"') {
      v.kind = Value::String;
      v.str = string();
    } else if (lit("true")) {
      v.kind = Value::Bool; v.b = true;
    } else if (lit("false")) {
      v.kind = Value::Bool; v.b = false;
    } else if (lit("null")) {
      v.kind = Value::Null;
    } else {
      number(v);
    }
    --depth_;
    return v;
  }
  std::string string() {
    ++p_;  // opening quote
    std::string out;
    while (*p_ && *p_ != '"') {
      if (*p_ == '\\') {
        ++p_;
        switch (*p_) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          default: fail("unsupported escape");
        }
        ++p_;
      } else {
        out += *p_++;
      }
    }
    if (*p_ != '"') fail("unterminated string");
    ++p_;
    return out;
  }
  void number(Value& v) {
    const char* start = p_;
    if (*p_ == '-') ++p_;
    if (!(*p_ >= '0' && *p_ <= '9')) fail("unexpected character");
    bool integral = true;
    while ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '+' || *p_ == '-') {
      if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') integral = false;
      ++p_;
    }
    std::string text(start, p_);
    v.kind = Value::Number;
    v.negative = text[0] == '-';
    v.num = std::strtod(text.c_str(), nullptr);
    if (integral) {
      errno = 0;
      char* end = nullptr;
      const long long parsed = std::strtoll(text.c_str(), &end, 10);
      if (errno == 0 && end && *end == '\0') { v.integer = parsed; v.is_integer = true; }
      else {
        // Non-negative values above INT64_MAX (e.g. u64 bit patterns).
        errno = 0;
        const unsigned long long u = std::strtoull(text.c_str(), &end, 10);
        if (errno == 0 && end && *end == '\0' && text[0] != '-') { v.integer = int64_t(u); v.is_integer = true; }
      }
    }
  }
};

inline Value parse(const char* text) { return Parser(text).parse(); }

}  // namespace json
}  // namespace askb
