// json.hpp -- the small JSON reader the host layer needs for safetensors headers and
// config.json (objects, arrays, strings with escapes, numbers, true / false / null).
//
// The reference scans config.json for individual keys by hand (server/src/model.cpp:31-99)
// and leaves safetensors headers to MLX's loader; this reader parses the whole document
// once, so nested keys ("quantization": {"bits", "group_size"}) and per-tensor records
// ({"dtype", "shape", "data_offsets"}) are plain lookups.
#pragma once

#include <cctype>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace flashmoe {
namespace json {

struct Value {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Value> arr;
  std::map<std::string, Value> obj;

  bool is_object() const { return kind == Object; }
  bool has(const std::string& k) const { return kind == Object && obj.count(k) != 0; }
  const Value* find(const std::string& k) const {
    if (kind != Object) return nullptr;
    auto it = obj.find(k);
    return it == obj.end() ? nullptr : &it->second;
  }
  // obj[k] as a number, `def` when absent or null; a present value of another kind is an error
  double number_or(const std::string& k, double def) const {
    const Value* v = find(k);
    if (!v || v->kind == Null) return def;
    if (v->kind == Bool) return v->b ? 1.0 : 0.0;
    if (v->kind != Number) throw std::runtime_error("json: \"" + k + "\" is not a number");
    return v->num;
  }
  bool bool_or(const std::string& k, bool def) const {
    const Value* v = find(k);
    if (!v || v->kind == Null) return def;
    if (v->kind == Bool) return v->b;
    if (v->kind == Number) return v->num != 0.0;
    throw std::runtime_error("json: \"" + k + "\" is not a boolean");
  }
  std::string string_or(const std::string& k, const std::string& def) const {
    const Value* v = find(k);
    if (!v || v->kind == Null) return def;
    if (v->kind != String) throw std::runtime_error("json: \"" + k + "\" is not a string");
    return v->str;
  }
};

class Parser {
 public:
  Parser(const char* p, size_t n) : p_(p), end_(p + n) {}

  Value parse_document() {
    Value v = parse_value(0);
    skip_ws();
    if (p_ != end_) fail("trailing characters");
    return v;
  }

 private:
  const char* p_;
  const char* end_;

  [[noreturn]] void fail(const char* what) const { throw std::runtime_error(std::string("json: ") + what); }

  void skip_ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool consume(char c) {
    skip_ws();
    if (p_ < end_ && *p_ == c) {
      ++p_;
      return true;
    }
    return false;
  }
  void expect(char c) {
    if (!consume(c)) fail("unexpected character");
  }
  bool literal(const char* s) {
    const char* q = p_;
    for (; *s; ++s, ++q)
      if (q >= end_ || *q != *s) return false;
    p_ = q;
    return true;
  }

  static void put_utf8(std::string& out, uint32_t cp) {
    if (cp < 0x80) {
      out += static_cast<char>(cp);
    } else if (cp < 0x800) {
      out += static_cast<char>(0xC0 | (cp >> 6));
      out += static_cast<char>(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      out += static_cast<char>(0xE0 | (cp >> 12));
      out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
      out += static_cast<char>(0x80 | (cp & 0x3F));
    } else {
      out += static_cast<char>(0xF0 | (cp >> 18));
      out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
      out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
      out += static_cast<char>(0x80 | (cp & 0x3F));
    }
  }
  uint32_t hex4() {
    if (end_ - p_ < 4) fail("short \\u escape");
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad \\u escape");
    }
    return v;
  }
  std::string parse_string() {
    skip_ws();
    if (p_ >= end_ || *p_ != '"') fail("expected a string");
    ++p_;
    std::string out;
    while (true) {
      if (p_ >= end_) fail("unterminated string");
      const char c = *p_++;
      if (c == '"') break;
      if (c != '\\') {
        out += c;
        continue;
      }
      if (p_ >= end_) fail("unterminated escape");
      const char e = *p_++;
      switch (e) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00 && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
            p_ += 2;
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo > 0xDFFF) fail("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(out, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
    return out;
  }
  Value parse_value(int depth) {
    if (depth > 64) fail("nesting too deep");
    skip_ws();
    if (p_ >= end_) fail("unexpected end");
    Value v;
    const char c = *p_;
    if (c == '{') {
      ++p_;
      v.kind = Value::Object;
      if (consume('}')) return v;
      do {
        std::string k = parse_string();
        expect(':');
        v.obj[k] = parse_value(depth + 1);  // a repeated key keeps the last value
      } while (consume(','));
      expect('}');
    } else if (c == '[') {
      ++p_;
      v.kind = Value::Array;
      if (consume(']')) return v;
      do v.arr.push_back(parse_value(depth + 1));
      while (consume(','));
      expect(']');
    } else if (c == '"') {
      v.kind = Value::String;
      v.str = parse_string();
    } else if (literal("true")) {
      v.kind = Value::Bool;
      v.b = true;
    } else if (literal("false")) {
      v.kind = Value::Bool;
    } else if (literal("null")) {
      v.kind = Value::Null;
    } else {
      // number: strtod on a bounded copy (the buffer need not be NUL-terminated)
      const char* q = p_;
      while (q < end_ && (std::isdigit(static_cast<unsigned char>(*q)) || *q == '-' || *q == '+' || *q == '.' ||
                          *q == 'e' || *q == 'E'))
        ++q;
      if (q == p_) fail("unexpected character");
      const std::string s(p_, q);
      char* stop = nullptr;
      v.kind = Value::Number;
      v.num = std::strtod(s.c_str(), &stop);
      if (stop != s.c_str() + s.size()) fail("bad number");
      p_ = q;
    }
    return v;
  }
};

inline Value parse(const std::string& s) { return Parser(s.data(), s.size()).parse_document(); }
inline Value parse(const char* p, size_t n) { return Parser(p, n).parse_document(); }

}  // namespace json
}  // namespace flashmoe
