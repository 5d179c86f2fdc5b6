// JSON parser / canonical serialiser; see json.h.
#include "json.h"

#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>

namespace hk {

namespace {
const Json kNull;

struct Parser {
  const char* p;
  const char* e;
  [[noreturn]] void fail(const char* what) const {
    throw std::runtime_error(std::string("json: ") + what + " at offset " + std::to_string((long)(e - p)) + " from end");
  }
  void ws() {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool lit(const char* s) {
    size_t n = std::strlen(s);
    if ((size_t)(e - p) >= n && std::memcmp(p, s, n) == 0) { p += n; return true; }
    return false;
  }
  static void put_utf8(std::string& o, uint32_t c) {
    if (c < 0x80) o.push_back((char)c);
    else if (c < 0x800) { o.push_back((char)(0xC0 | (c >> 6))); o.push_back((char)(0x80 | (c & 0x3F))); }
    else if (c < 0x10000) {
      o.push_back((char)(0xE0 | (c >> 12)));
      o.push_back((char)(0x80 | ((c >> 6) & 0x3F)));
      o.push_back((char)(0x80 | (c & 0x3F)));
    } else {
      o.push_back((char)(0xF0 | (c >> 18)));
      o.push_back((char)(0x80 | ((c >> 12) & 0x3F)));
      o.push_back((char)(0x80 | ((c >> 6) & 0x3F)));
      o.push_back((char)(0x80 | (c & 0x3F)));
    }
  }
  uint32_t hex4() {
    if (e - p < 4) fail("short \\u escape");
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) {
      char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad hex digit");
    }
    return v;
  }
  std::string str() {
    if (p >= e || *p != '"') fail("expected string");
    ++p;
    std::string o;
    while (true) {
      if (p >= e) fail("unterminated string");
      char c = *p++;
      if (c == '"') break;
      if ((unsigned char)c < 0x20) fail("control character in string");
      if (c != '\\') { o.push_back(c); continue; }
      if (p >= e) fail("bad escape");
      char x = *p++;
      switch (x) {
        case '"': o.push_back('"'); break;
        case '\\': o.push_back('\\'); break;
        case '/': o.push_back('/'); break;
        case 'b': o.push_back('\b'); break;
        case 'f': o.push_back('\f'); break;
        case 'n': o.push_back('\n'); break;
        case 'r': o.push_back('\r'); break;
        case 't': o.push_back('\t'); break;
        case 'u': {
          uint32_t c1 = hex4();
          if (c1 >= 0xD800 && c1 < 0xDC00) {
            if (!lit("\\u")) fail("lone surrogate");
            uint32_t c2 = hex4();
            c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
          }
          put_utf8(o, c1);
          break;
        }
        default: fail("bad escape");
      }
    }
    return o;
  }
  Json num() {
    const char* s = p;
    bool neg = false, is_float = false;
    if (p < e && *p == '-') { neg = true; ++p; }
    while (p < e && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '+' || *p == '-')) {
      if (*p == '.' || *p == 'e' || *p == 'E') is_float = true;
      ++p;
    }
    std::string t(s, p);
    if (t.empty() || t == "-") fail("bad number");
    if (!is_float) {
      errno = 0;
      if (neg) {
        long long v = std::strtoll(t.c_str(), nullptr, 10);
        if (errno == 0) return Json::integer(v);
      } else {
        unsigned long long v = std::strtoull(t.c_str(), nullptr, 10);
        if (errno == 0) return v <= (unsigned long long)INT64_MAX ? Json::integer((int64_t)v) : Json::uinteger(v);
      }
    }
    return Json::number(std::strtod(t.c_str(), nullptr));
  }
  Json value(int depth) {
    if (depth > 256) fail("nesting too deep");
    ws();
    if (p >= e) fail("unexpected end");
    char c = *p;
    if (c == '{') {
      ++p;
      Json o = Json::object();
      ws();
      if (p < e && *p == '}') { ++p; return o; }
      while (true) {
        ws();
        std::string k = str();
        ws();
        if (p >= e || *p != ':') fail("expected ':'");
        ++p;
        o.set(k, value(depth + 1));
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == '}') { ++p; break; }
        fail("expected ',' or '}'");
      }
      return o;
    }
    if (c == '[') {
      ++p;
      Json a = Json::array();
      ws();
      if (p < e && *p == ']') { ++p; return a; }
      while (true) {
        a.push(value(depth + 1));
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == ']') { ++p; break; }
        fail("expected ',' or ']'");
      }
      return a;
    }
    if (c == '"') return Json::string(str());
    if (lit("true")) return Json::boolean(true);
    if (lit("false")) return Json::boolean(false);
    if (lit("null")) return Json::null();
    return num();
  }
};

void dump_to(const Json& j, std::string& o) {
  switch (j.type()) {
    case Json::Type::Null: o += "null"; break;
    case Json::Type::Bool: o += j.as_bool() ? "true" : "false"; break;
    case Json::Type::Int: o += std::to_string(j.as_int()); break;
    case Json::Type::UInt: o += std::to_string(j.as_uint()); break;
    case Json::Type::Float: o += json_number(j.as_double()); break;
    case Json::Type::String: o += json_escape(j.as_string()); break;
    case Json::Type::Array: {
      o.push_back('[');
      bool first = true;
      for (const auto& v : j.items()) {
        if (!first) o.push_back(',');
        first = false;
        dump_to(v, o);
      }
      o.push_back(']');
      break;
    }
    case Json::Type::Object: {
      o.push_back('{');
      bool first = true;
      for (const auto& kv : j.members()) {
        if (!first) o.push_back(',');
        first = false;
        o += json_escape(kv.first);
        o.push_back(':');
        dump_to(kv.second, o);
      }
      o.push_back('}');
      break;
    }
  }
}
}  // namespace

int64_t Json::as_int() const {
  if (t_ == Type::Int) return i_;
  if (t_ == Type::UInt) return (int64_t)u_;
  if (t_ == Type::Float) return (int64_t)f_;
  throw std::runtime_error("json: not a number");
}
uint64_t Json::as_uint() const {
  if (t_ == Type::UInt) return u_;
  if (t_ == Type::Int) return (uint64_t)i_;
  if (t_ == Type::Float) return (uint64_t)f_;
  throw std::runtime_error("json: not a number");
}
double Json::as_double() const {
  if (t_ == Type::Float) return f_;
  if (t_ == Type::Int) return (double)i_;
  if (t_ == Type::UInt) return (double)u_;
  throw std::runtime_error("json: not a number");
}
const Json& Json::operator[](const std::string& k) const {
  auto it = obj_.find(k);
  return it == obj_.end() ? kNull : it->second;
}
const Json& Json::pointer(const std::string& path) const {
  const Json* cur = this;
  size_t i = 0;
  while (i < path.size()) {
    if (path[i] != '/') return kNull;
    size_t j = path.find('/', i + 1);
    std::string key = path.substr(i + 1, j == std::string::npos ? std::string::npos : j - i - 1);
    if (cur->is_object()) cur = &(*cur)[key];
    else if (cur->is_array()) {
      size_t idx = std::strtoull(key.c_str(), nullptr, 10);
      if (idx >= cur->arr_.size()) return kNull;
      cur = &cur->arr_[idx];
    } else return kNull;
    if (j == std::string::npos) break;
    i = j;
  }
  return *cur;
}
Json Json::parse(const std::string& text) { return parse(text.data(), text.size()); }
Json Json::parse(const char* p, size_t n) {
  Parser ps{p, p + n};
  Json v = ps.value(0);
  ps.ws();
  if (ps.p != ps.e) ps.fail("trailing characters");
  return v;
}
std::string Json::dump() const {
  std::string o;
  dump_to(*this, o);
  return o;
}

std::string json_escape(const std::string& s) {
  std::string o = "\"";
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
          o.push_back((char)c);
        }
    }
  }
  o.push_back('"');
  return o;
}

// Shortest round-trip decimal digits of v (by increasing %e precision), placed like ryu:
// integers keep ".0", decimal notation for exponents in (-5, 16], scientific otherwise.
std::string json_number(double v) {
  if (!std::isfinite(v)) return "null";
  if (v == 0) return std::signbit(v) ? "-0.0" : "0.0";
  char buf[64];
  int prec = 1;
  for (; prec <= 17; ++prec) {
    std::snprintf(buf, sizeof buf, "%.*e", prec - 1, v);
    if (std::strtod(buf, nullptr) == v) break;
  }
  // buf = [-]d.ddde[+-]XX
  std::string t(buf);
  bool neg = t[0] == '-';
  if (neg) t = t.substr(1);
  size_t epos = t.find('e');
  int exp10 = std::atoi(t.c_str() + epos + 1);
  std::string digits;
  for (size_t i = 0; i < epos; ++i)
    if (t[i] != '.') digits.push_back(t[i]);
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  const int n = (int)digits.size();
  const int kk = exp10 + 1;  // decimal point position relative to the digit string
  std::string o;
  if (n <= kk && kk <= 16) {
    o = digits + std::string(kk - n, '0') + ".0";
  } else if (0 < kk && kk <= 16) {
    o = digits.substr(0, kk) + "." + digits.substr(kk);
  } else if (-5 < kk && kk <= 0) {
    o = "0." + std::string(-kk, '0') + digits;
  } else if (n == 1) {
    o = digits + "e" + std::to_string(kk - 1);
  } else {
    o = digits.substr(0, 1) + "." + digits.substr(1) + "e" + std::to_string(kk - 1);
  }
  return neg ? "-" + o : o;
}

}  // namespace hk
