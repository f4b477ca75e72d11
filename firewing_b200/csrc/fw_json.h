// fw_json.h -- a small JSON reader (RFC 8259 values; non-negative integers
// kept exact) for safetensors headers, checkpoint indexes and codec
// manifests (host code).
#pragma once

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

namespace fw {
namespace json {

struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  bool is_uint = false;  // a non-negative integer literal that fits in 64 bits
  uint64_t u = 0;
  double d = 0.0;
  std::string s;
  std::vector<Json> items;                          // Array
  std::vector<std::pair<std::string, Json>> members;  // Object, in order
};

class JsonReader {
 public:
  JsonReader(const char* p, size_t n) : p_(p), end_(p + n) {}

  bool parse(Json* out, std::string* err) {
    if (!value(out, 0)) {
      *err = err_.empty() ? "malformed JSON" : err_;
      return false;
    }
    ws();
    if (p_ != end_) {
      *err = "trailing bytes after JSON value";
      return false;
    }
    return true;
  }

 private:
  const char* p_;
  const char* end_;
  std::string err_;

  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool lit(const char* w) {
    const size_t n = std::strlen(w);
    if (static_cast<size_t>(end_ - p_) < n || std::memcmp(p_, w, n) != 0) return false;
    p_ += n;
    return true;
  }
  static void utf8(uint32_t c, std::string* s) {
    if (c < 0x80) {
      s->push_back(static_cast<char>(c));
    } else if (c < 0x800) {
      s->push_back(static_cast<char>(0xc0 | (c >> 6)));
      s->push_back(static_cast<char>(0x80 | (c & 0x3f)));
    } else if (c < 0x10000) {
      s->push_back(static_cast<char>(0xe0 | (c >> 12)));
      s->push_back(static_cast<char>(0x80 | ((c >> 6) & 0x3f)));
      s->push_back(static_cast<char>(0x80 | (c & 0x3f)));
    } else {
      s->push_back(static_cast<char>(0xf0 | (c >> 18)));
      s->push_back(static_cast<char>(0x80 | ((c >> 12) & 0x3f)));
      s->push_back(static_cast<char>(0x80 | ((c >> 6) & 0x3f)));
      s->push_back(static_cast<char>(0x80 | (c & 0x3f)));
    }
  }
  bool hex4(uint32_t* v) {
    if (end_ - p_ < 4) return false;
    uint32_t r = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p_++;
      r <<= 4;
      if (c >= '0' && c <= '9') r |= c - '0';
      else if (c >= 'a' && c <= 'f') r |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') r |= c - 'A' + 10;
      else return false;
    }
    *v = r;
    return true;
  }
  bool str(std::string* s) {
    if (p_ >= end_ || *p_ != '"') return false;
    ++p_;
    while (p_ < end_) {
      const unsigned char c = static_cast<unsigned char>(*p_++);
      if (c == '"') return true;
      if (c < 0x20) return false;
      if (c != '\\') {
        s->push_back(static_cast<char>(c));
        continue;
      }
      if (p_ >= end_) return false;
      const char e = *p_++;
      switch (e) {
        case '"': s->push_back('"'); break;
        case '\\': s->push_back('\\'); break;
        case '/': s->push_back('/'); break;
        case 'b': s->push_back('\b'); break;
        case 'f': s->push_back('\f'); break;
        case 'n': s->push_back('\n'); break;
        case 'r': s->push_back('\r'); break;
        case 't': s->push_back('\t'); break;
        case 'u': {
          uint32_t c1;
          if (!hex4(&c1)) return false;
          if (c1 >= 0xd800 && c1 < 0xdc00) {  // surrogate pair
            uint32_t c2;
            if (!lit("\\u") || !hex4(&c2) || c2 < 0xdc00 || c2 >= 0xe000) return false;
            c1 = 0x10000 + ((c1 - 0xd800) << 10) + (c2 - 0xdc00);
          } else if (c1 >= 0xdc00 && c1 < 0xe000) {
            return false;
          }
          utf8(c1, s);
          break;
        }
        default: return false;
      }
    }
    return false;
  }
  bool number(Json* v) {
    const char* s = p_;
    if (p_ < end_ && *p_ == '-') ++p_;
    if (p_ >= end_ || *p_ < '0' || *p_ > '9') return false;
    if (*p_ == '0') ++p_;
    else while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    bool integral = true;
    if (p_ < end_ && *p_ == '.') {
      integral = false;
      ++p_;
      if (p_ >= end_ || *p_ < '0' || *p_ > '9') return false;
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
      integral = false;
      ++p_;
      if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (p_ >= end_ || *p_ < '0' || *p_ > '9') return false;
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    v->kind = Json::Number;
    const std::string text(s, p_);
    v->d = std::strtod(text.c_str(), nullptr);
    if (integral && text[0] != '-') {
      uint64_t u = 0;
      bool fits = true;
      for (char c : text) {
        const uint64_t digit = static_cast<uint64_t>(c - '0');
        if (u > (UINT64_MAX - digit) / 10) {
          fits = false;
          break;
        }
        u = u * 10 + digit;
      }
      v->is_uint = fits;
      v->u = u;
    }
    return true;
  }
  bool value(Json* v, int depth) {
    if (depth > 64) {
      err_ = "JSON nested too deeply";
      return false;
    }
    ws();
    if (p_ >= end_) return false;
    const char c = *p_;
    if (c == '{') {
      ++p_;
      v->kind = Json::Object;
      ws();
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        return true;
      }
      for (;;) {
        ws();
        std::string key;
        if (!str(&key)) return false;
        ws();
        if (p_ >= end_ || *p_ != ':') return false;
        ++p_;
        Json item;
        if (!value(&item, depth + 1)) return false;
        v->members.emplace_back(std::move(key), std::move(item));
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == '}') {
          ++p_;
          return true;
        }
        return false;
      }
    }
    if (c == '[') {
      ++p_;
      v->kind = Json::Array;
      ws();
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        return true;
      }
      for (;;) {
        Json item;
        if (!value(&item, depth + 1)) return false;
        v->items.push_back(std::move(item));
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == ']') {
          ++p_;
          return true;
        }
        return false;
      }
    }
    if (c == '"') {
      v->kind = Json::String;
      return str(&v->s);
    }
    if (lit("true")) {
      v->kind = Json::Bool;
      v->b = true;
      return true;
    }
    if (lit("false")) {
      v->kind = Json::Bool;
      return true;
    }
    if (lit("null")) return true;
    return number(v);
  }
};

inline const Json* member(const Json& o, const char* key) {
  for (const auto& m : o.members)
    if (m.first == key) return &m.second;
  return nullptr;
}

}  // namespace json
}  // namespace fw
