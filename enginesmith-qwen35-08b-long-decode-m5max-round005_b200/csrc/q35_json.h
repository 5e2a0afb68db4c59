// Minimal JSON DOM for the safetensors header, config.json and the engine's
// JSON-lines protocol. Integers are kept exactly (int64 / uint64) next to the
// double value so that token ids round-trip.
#pragma once
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace q35json {

struct Value {
  enum Type { Null, Bool, Number, String, Array, Object } type = Null;
  bool b = false;
  double num = 0.0;
  bool is_int = false;     // number had no fraction/exponent
  bool neg = false;
  uint64_t u = 0;          // magnitude when is_int
  std::string str;
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;

  const Value* get(const std::string& k) const {
    if (type != Object) return nullptr;
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
  bool as_u64(uint64_t& out) const {
    if (type != Number || !is_int || neg) return false;
    out = u;
    return true;
  }
};

class Parser {
 public:
  Parser(const char* s, size_t n) : p_(s), e_(s + n) {}
  bool parse(Value& v, std::string& err) {
    ws();
    if (!value(v, 0)) {
      err = err_.empty() ? "invalid JSON" : err_;
      return false;
    }
    ws();
    if (p_ != e_) {
      err = "trailing characters after JSON value";
      return false;
    }
    return true;
  }

 private:
  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool fail(const char* m) {
    if (err_.empty()) err_ = m;
    return false;
  }
  bool value(Value& v, int depth) {
    if (depth > 64) return fail("JSON nesting too deep");
    if (p_ >= e_) return fail("unexpected end of JSON");
    switch (*p_) {
      case '{': return object(v, depth);
      case '[': return array(v, depth);
      case '"': v.type = Value::String; return string(v.str);
      case 't': return lit("true", v, Value::Bool, true);
      case 'f': return lit("false", v, Value::Bool, false);
      case 'n': return lit("null", v, Value::Null, false);
      default: return number(v);
    }
  }
  bool lit(const char* w, Value& v, Value::Type t, bool b) {
    size_t n = std::strlen(w);
    if (size_t(e_ - p_) < n || std::memcmp(p_, w, n) != 0) return fail("invalid literal");
    p_ += n;
    v.type = t;
    v.b = b;
    return true;
  }
  bool number(Value& v) {
    const char* s = p_;
    bool neg = false;
    if (p_ < e_ && *p_ == '-') {
      neg = true;
      ++p_;
    }
    if (p_ >= e_ || *p_ < '0' || *p_ > '9') return fail("invalid number");
    uint64_t u = 0;
    bool overflow = false;
    while (p_ < e_ && *p_ >= '0' && *p_ <= '9') {
      uint64_t d = uint64_t(*p_ - '0');
      if (u > (UINT64_MAX - d) / 10) overflow = true;
      u = u * 10 + d;
      ++p_;
    }
    bool frac = false;
    if (p_ < e_ && *p_ == '.') {
      frac = true;
      ++p_;
      while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < e_ && (*p_ == 'e' || *p_ == 'E')) {
      frac = true;
      ++p_;
      if (p_ < e_ && (*p_ == '+' || *p_ == '-')) ++p_;
      while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    v.type = Value::Number;
    v.is_int = !frac && !overflow;
    v.neg = neg;
    v.u = u;
    v.num = std::strtod(std::string(s, size_t(p_ - s)).c_str(), nullptr);
    return true;
  }
  bool string(std::string& out) {
    ++p_;
    out.clear();
    while (p_ < e_ && *p_ != '"') {
      char c = *p_++;
      if (c == '\\') {
        if (p_ >= e_) return fail("bad escape");
        char x = *p_++;
        switch (x) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {
            if (e_ - p_ < 4) return fail("bad \\u escape");
            unsigned cp = unsigned(std::strtoul(std::string(p_, 4).c_str(), nullptr, 16));
            p_ += 4;
            if (cp < 0x80) out += char(cp);
            else if (cp < 0x800) {
              out += char(0xC0 | (cp >> 6));
              out += char(0x80 | (cp & 0x3F));
            } else {
              out += char(0xE0 | (cp >> 12));
              out += char(0x80 | ((cp >> 6) & 0x3F));
              out += char(0x80 | (cp & 0x3F));
            }
            break;
          }
          default: return fail("bad escape");
        }
      } else {
        out += c;
      }
    }
    if (p_ >= e_) return fail("unterminated string");
    ++p_;
    return true;
  }
  bool array(Value& v, int depth) {
    ++p_;
    v.type = Value::Array;
    ws();
    if (p_ < e_ && *p_ == ']') {
      ++p_;
      return true;
    }
    for (;;) {
      ws();
      v.arr.emplace_back();
      if (!value(v.arr.back(), depth + 1)) return false;
      ws();
      if (p_ < e_ && *p_ == ',') {
        ++p_;
        continue;
      }
      if (p_ < e_ && *p_ == ']') {
        ++p_;
        return true;
      }
      return fail("expected , or ] in array");
    }
  }
  bool object(Value& v, int depth) {
    ++p_;
    v.type = Value::Object;
    ws();
    if (p_ < e_ && *p_ == '}') {
      ++p_;
      return true;
    }
    for (;;) {
      ws();
      if (p_ >= e_ || *p_ != '"') return fail("expected key string");
      std::string k;
      if (!string(k)) return false;
      ws();
      if (p_ >= e_ || *p_ != ':') return fail("expected :");
      ++p_;
      ws();
      v.obj.emplace_back(k, Value());
      if (!value(v.obj.back().second, depth + 1)) return false;
      ws();
      if (p_ < e_ && *p_ == ',') {
        ++p_;
        continue;
      }
      if (p_ < e_ && *p_ == '}') {
        ++p_;
        return true;
      }
      return fail("expected , or } in object");
    }
  }
  const char* p_;
  const char* e_;
  std::string err_;
};

inline bool parse(const std::string& s, Value& v, std::string& err) {
  return Parser(s.data(), s.size()).parse(v, err);
}

inline void escape(const std::string& s, std::string& out) {
  out += '"';
  for (unsigned char c : s) {
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (c < 0x20) {
          char b[8];
          std::snprintf(b, sizeof b, "\\u%04x", c);
          out += b;
        } else {
          out += char(c);
        }
    }
  }
  out += '"';
}

// Serialise a value (used to echo request ids verbatim).
inline void dump(const Value& v, std::string& out) {
  switch (v.type) {
    case Value::Null: out += "null"; break;
    case Value::Bool: out += v.b ? "true" : "false"; break;
    case Value::Number:
      if (v.is_int) {
        if (v.neg) out += '-';
        out += std::to_string(v.u);
      } else {
        char b[40];
        std::snprintf(b, sizeof b, "%.17g", v.num);
        out += b;
      }
      break;
    case Value::String: escape(v.str, out); break;
    case Value::Array:
      out += '[';
      for (size_t i = 0; i < v.arr.size(); ++i) {
        if (i) out += ',';
        dump(v.arr[i], out);
      }
      out += ']';
      break;
    case Value::Object:
      out += '{';
      for (size_t i = 0; i < v.obj.size(); ++i) {
        if (i) out += ',';
        escape(v.obj[i].first, out);
        out += ':';
        dump(v.obj[i].second, out);
      }
      out += '}';
      break;
  }
}

}  // namespace q35json
