#include "json.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>

namespace spc {

struct JsonParser {
  const std::string& s;
  size_t i = 0;
  int depth = 0;

  [[noreturn]] void err(const char* what) {
    fail(Status::ParseError, std::string("json: ") + what + " at byte " + std::to_string(i));
  }
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\t' || s[i] == '\n' || s[i] == '\r')) ++i;
  }
  bool lit(const char* w) {
    size_t n = 0;
    while (w[n]) ++n;
    if (s.compare(i, n, w) == 0) { i += n; return true; }
    return false;
  }
  static void utf8(std::string& out, uint32_t cp) {
    if (cp < 0x80) out += char(cp);
    else if (cp < 0x800) { out += char(0xC0 | (cp >> 6)); out += char(0x80 | (cp & 0x3F)); }
    else if (cp < 0x10000) {
      out += char(0xE0 | (cp >> 12)); out += char(0x80 | ((cp >> 6) & 0x3F)); out += char(0x80 | (cp & 0x3F));
    } else {
      out += char(0xF0 | (cp >> 18)); out += char(0x80 | ((cp >> 12) & 0x3F));
      out += char(0x80 | ((cp >> 6) & 0x3F)); out += char(0x80 | (cp & 0x3F));
    }
  }
  uint32_t hex4() {
    if (i + 4 > s.size()) err("short \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = s[i++];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else err("bad hex digit");
    }
    return v;
  }
  std::string string() {
    if (s[i] != '"') err("expected string");
    ++i;
    std::string out;
    while (true) {
      if (i >= s.size()) err("unterminated string");
      const char c = s[i++];
      if (c == '"') break;
      if (static_cast<unsigned char>(c) < 0x20) err("control character in string");
      if (c != '\\') { out += c; continue; }
      if (i >= s.size()) err("bad escape");
      const char e = s[i++];
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
          if (cp >= 0xD800 && cp < 0xDC00) {
            if (i + 6 <= s.size() && s[i] == '\\' && s[i + 1] == 'u') {
              i += 2;
              const uint32_t lo = hex4();
              if (lo < 0xDC00 || lo > 0xDFFF) err("bad low surrogate");
              cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            } else {
              err("lone high surrogate");
            }
          }
          utf8(out, cp);
          break;
        }
        default: err("bad escape");
      }
    }
    return out;
  }
  Json value() {
    if (++depth > 512) err("nesting too deep");
    ws();
    if (i >= s.size()) err("unexpected end");
    Json v;
    const char c = s[i];
    if (c == '{') {
      ++i;
      v.type_ = Json::Type::Object;
      ws();
      if (i < s.size() && s[i] == '}') { ++i; --depth; return v; }
      while (true) {
        ws();
        std::string k = string();
        ws();
        if (i >= s.size() || s[i] != ':') err("expected ':'");
        ++i;
        Json x = value();
        v.o_.emplace_back(std::move(k), std::move(x));
        ws();
        if (i < s.size() && s[i] == ',') { ++i; continue; }
        if (i < s.size() && s[i] == '}') { ++i; break; }
        err("expected ',' or '}'");
      }
    } else if (c == '[') {
      ++i;
      v.type_ = Json::Type::Array;
      ws();
      if (i < s.size() && s[i] == ']') { ++i; --depth; return v; }
      while (true) {
        v.a_.push_back(value());
        ws();
        if (i < s.size() && s[i] == ',') { ++i; continue; }
        if (i < s.size() && s[i] == ']') { ++i; break; }
        err("expected ',' or ']'");
      }
    } else if (c == '"') {
      v.type_ = Json::Type::String;
      v.s_ = string();
    } else if (lit("true")) {
      v.type_ = Json::Type::Bool;
      v.b_ = true;
    } else if (lit("false")) {
      v.type_ = Json::Type::Bool;
    } else if (lit("null")) {
    } else if (c == '-' || (c >= '0' && c <= '9')) {
      const size_t st = i;
      bool integral = true;
      if (s[i] == '-') ++i;
      while (i < s.size() && ((s[i] >= '0' && s[i] <= '9') || s[i] == '.' || s[i] == 'e' || s[i] == 'E' ||
                              s[i] == '+' || s[i] == '-')) {
        if (s[i] == '.' || s[i] == 'e' || s[i] == 'E') integral = false;
        ++i;
      }
      const std::string num = s.substr(st, i - st);
      char* end = nullptr;
      v.type_ = Json::Type::Number;
      v.d_ = std::strtod(num.c_str(), &end);
      if (!end || *end) err("bad number");
      if (integral) {
        v.is_int_ = true;
        v.i_ = std::strtoll(num.c_str(), nullptr, 10);
      }
    } else {
      err("unexpected character");
    }
    --depth;
    return v;
  }
};

Json Json::parse(const std::string& text) {
  JsonParser p{text};
  Json v = p.value();
  p.ws();
  if (p.i != text.size()) p.err("trailing characters");
  return v;
}

std::string json_escape(const std::string& s) {
  std::string o;
  o.reserve(s.size() + 2);
  for (unsigned char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      case '\b': o += "\\b"; break;
      case '\f': o += "\\f"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof buf, "\\u%04x", c);
          o += buf;
        } else {
          o += char(c);
        }
    }
  }
  return o;
}

std::string Json::dump() const {
  switch (type_) {
    case Type::Null: return "null";
    case Type::Bool: return b_ ? "true" : "false";
    case Type::Number: {
      if (is_int_) return std::to_string(i_);
      if (!std::isfinite(d_)) return "null";
      char buf[40];
      std::snprintf(buf, sizeof buf, "%.17g", d_);
      return buf;
    }
    case Type::String: return "\"" + json_escape(s_) + "\"";
    case Type::Array: {
      std::string o = "[";
      for (size_t k = 0; k < a_.size(); ++k) {
        if (k) o += ",";
        o += a_[k].dump();
      }
      return o + "]";
    }
    case Type::Object: {
      std::string o = "{";
      for (size_t k = 0; k < o_.size(); ++k) {
        if (k) o += ",";
        o += "\"" + json_escape(o_[k].first) + "\":" + o_[k].second.dump();
      }
      return o + "}";
    }
  }
  return "null";
}

const std::string& Json::str() const {
  if (type_ != Type::String) fail(Status::SchemaError, "json: expected a string");
  return s_;
}
double Json::num() const {
  if (type_ != Type::Number) fail(Status::SchemaError, "json: expected a number");
  return d_;
}
int64_t Json::int64() const {
  if (type_ != Type::Number) fail(Status::SchemaError, "json: expected a number");
  return is_int_ ? i_ : int64_t(d_);
}
bool Json::boolean() const {
  if (type_ != Type::Bool) fail(Status::SchemaError, "json: expected a boolean");
  return b_;
}
const std::vector<Json>& Json::arr() const {
  if (type_ != Type::Array) fail(Status::SchemaError, "json: expected an array");
  return a_;
}
const std::vector<std::pair<std::string, Json>>& Json::obj() const {
  if (type_ != Type::Object) fail(Status::SchemaError, "json: expected an object");
  return o_;
}
const Json* Json::get(const std::string& key) const {
  if (type_ != Type::Object) return nullptr;
  for (const auto& kv : o_)
    if (kv.first == key) return &kv.second;
  return nullptr;
}
const Json& Json::at(const std::string& key) const {
  const Json* v = get(key);
  if (!v) fail(Status::SchemaError, "json: missing key '" + key + "'");
  return *v;
}
size_t Json::size() const {
  if (type_ == Type::Array) return a_.size();
  if (type_ == Type::Object) return o_.size();
  return 0;
}
Json Json::make_bool(bool b) { Json j; j.type_ = Type::Bool; j.b_ = b; return j; }
Json Json::make_number(double v) { Json j; j.type_ = Type::Number; j.d_ = v; return j; }
Json Json::make_int(int64_t v) {
  Json j;
  j.type_ = Type::Number;
  j.i_ = v;
  j.d_ = double(v);
  j.is_int_ = true;
  return j;
}
Json Json::make_string(std::string s) { Json j; j.type_ = Type::String; j.s_ = std::move(s); return j; }
Json Json::make_array(std::vector<Json> a) { Json j; j.type_ = Type::Array; j.a_ = std::move(a); return j; }
Json Json::make_object() { Json j; j.type_ = Type::Object; return j; }
void Json::push(Json v) {
  if (type_ != Type::Array) fail(Status::InvalidArgument, "json: push on a non-array");
  a_.push_back(std::move(v));
}
void Json::set(const std::string& k, Json v) {
  if (type_ != Type::Object) fail(Status::InvalidArgument, "json: set on a non-object");
  for (auto& kv : o_)
    if (kv.first == k) { kv.second = std::move(v); return; }
  o_.emplace_back(k, std::move(v));
}

}  // namespace spc
