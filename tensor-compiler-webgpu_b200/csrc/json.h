// json.h -- a small JSON value, reader and writer for the library's graph interchange.
//
// Graphs arrive as the reference's Graph.toJSON form ({"nodes": [{op, inputs, attrs, shape}]},
// src/ir/graph.js:48-50); launch records leave as JSON.  Numbers keep their source text's value as a
// double plus whether the text was an integer, so integer attributes (shapes, axes, perms, ids) round
// trip exactly and float constants are read with strtod's correct rounding.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace tcb_json {

struct Value {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  bool integral = false;
  std::string str;
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;   // insertion order kept

  bool is_null() const { return kind == Null; }
  bool is_number() const { return kind == Number; }
  bool is_array() const { return kind == Array; }
  bool is_object() const { return kind == Object; }
  bool is_string() const { return kind == String; }
  const Value* find(const std::string& key) const {
    for (auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
  const Value& at(const std::string& key) const {
    const Value* v = find(key);
    if (!v) throw std::runtime_error("JSON: missing key '" + key + "'");
    return *v;
  }
  int64_t as_int() const {
    if (kind != Number) throw std::runtime_error("JSON: expected a number");
    return (int64_t)num;
  }
  double as_double() const {
    if (kind != Number) throw std::runtime_error("JSON: expected a number");
    return num;
  }
  const std::string& as_string() const {
    if (kind != String) throw std::runtime_error("JSON: expected a string");
    return str;
  }
  bool truthy() const { return kind == Bool ? b : (kind == Number ? num != 0 : kind != Null); }
};

class Reader {
 public:
  explicit Reader(const char* s) : p_(s) {}
  Value parse() {
    Value v = value();
    ws();
    if (*p_) fail("trailing text");
    return v;
  }

 private:
  const char* p_;
  [[noreturn]] void fail(const char* what) { throw std::runtime_error(std::string("JSON: ") + what); }
  void ws() {
    while (*p_ == ' ' || *p_ == '\n' || *p_ == '\t' || *p_ == '\r') ++p_;
  }
  Value value() {
    ws();
    Value v;
    switch (*p_) {
      case '{': {
        v.kind = Value::Object;
        ++p_;
        ws();
        if (*p_ == '}') { ++p_; return v; }
        for (;;) {
          ws();
          if (*p_ != '"') fail("expected a key");
          std::string k = string();
          ws();
          if (*p_ != ':') fail("expected ':'");
          ++p_;
          v.obj.emplace_back(std::move(k), value());
          ws();
          if (*p_ == ',') { ++p_; continue; }
          if (*p_ == '}') { ++p_; return v; }
          fail("expected ',' or '}'");
        }
      }
      case '[': {
        v.kind = Value::Array;
        ++p_;
        ws();
        if (*p_ == ']') { ++p_; return v; }
        for (;;) {
          v.arr.push_back(value());
          ws();
          if (*p_ == ',') { ++p_; continue; }
          if (*p_ == ']') { ++p_; return v; }
          fail("expected ',' or ']'");
        }
      }
      case '"':
        v.kind = Value::String;
        v.str = string();
        return v;
      case 't':
        if (std::string(p_, 4) != "true") fail("bad literal");
        p_ += 4; v.kind = Value::Bool; v.b = true; return v;
      case 'f':
        if (std::string(p_, 5) != "false") fail("bad literal");
        p_ += 5; v.kind = Value::Bool; v.b = false; return v;
      case 'n':
        if (std::string(p_, 4) != "null") fail("bad literal");
        p_ += 4; return v;
      default: {
        const char* s = p_;
        bool integral = true;
        if (*p_ == '-') ++p_;
        if (!(*p_ >= '0' && *p_ <= '9')) fail("bad value");
        while (*p_ >= '0' && *p_ <= '9') ++p_;
        if (*p_ == '.') { integral = false; ++p_; while (*p_ >= '0' && *p_ <= '9') ++p_; }
        if (*p_ == 'e' || *p_ == 'E') {
          integral = false;
          ++p_;
          if (*p_ == '+' || *p_ == '-') ++p_;
          while (*p_ >= '0' && *p_ <= '9') ++p_;
        }
        v.kind = Value::Number;
        v.num = std::strtod(std::string(s, p_).c_str(), nullptr);
        v.integral = integral;
        return v;
      }
    }
  }
  std::string string() {
    std::string out;
    ++p_;  // opening quote
    while (*p_ && *p_ != '"') {
      if (*p_ == '\\') {
        ++p_;
        switch (*p_) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            unsigned cp = (unsigned)std::stoul(std::string(p_ + 1, 4), nullptr, 16);
            p_ += 4;
            if (cp < 0x80) out += (char)cp;
            else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3F)); }
            else { out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F)); }
            break;
          }
          default: out += *p_; break;
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
};

inline Value parse(const char* text) { return Reader(text).parse(); }

// ---- writing: a minimal streaming writer ----
inline std::string quote(const std::string& s) {
  std::string o = "\"";
  for (char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\t': o += "\\t"; break;
      case '\r': o += "\\r"; break;
      default:
        if ((unsigned char)c < 0x20) {
          char buf[8];
          snprintf(buf, sizeof buf, "\\u%04x", (unsigned char)c);
          o += buf;
        } else {
          o += c;
        }
    }
  }
  return o + "\"";
}

}  // namespace tcb_json
