// Minimal JSON value, parser and serialisers (compact and canonical).
//
// Canonical form (the `.gravity` header encoding): object keys sorted bytewise, no whitespace,
// strings escaped like serde_json (\" \\ \n \r \t \b \f, other control characters as \u00XX,
// non-ASCII kept as UTF-8), integers in decimal, finite floats in shortest round-trip digits
// with ryu-style placement (e.g. 1.0, 0.25, 1e-7, 1.5e16). Parity: crates/hawking-core/src/artifact.rs:73-112.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace hk {

class Json {
 public:
  enum class Type { Null, Bool, Int, UInt, Float, String, Array, Object };

  Json() = default;
  static Json null() { return Json(); }
  static Json boolean(bool b) { Json j; j.t_ = Type::Bool; j.b_ = b; return j; }
  static Json integer(int64_t v) { Json j; j.t_ = Type::Int; j.i_ = v; return j; }
  static Json uinteger(uint64_t v) { Json j; j.t_ = Type::UInt; j.u_ = v; return j; }
  static Json number(double v) { Json j; j.t_ = Type::Float; j.f_ = v; return j; }
  static Json string(std::string s) { Json j; j.t_ = Type::String; j.s_ = std::move(s); return j; }
  static Json array() { Json j; j.t_ = Type::Array; return j; }
  static Json object() { Json j; j.t_ = Type::Object; return j; }

  Type type() const { return t_; }
  bool is_null() const { return t_ == Type::Null; }
  bool is_object() const { return t_ == Type::Object; }
  bool is_array() const { return t_ == Type::Array; }
  bool is_string() const { return t_ == Type::String; }
  bool is_number() const { return t_ == Type::Int || t_ == Type::UInt || t_ == Type::Float; }

  bool as_bool() const { return b_; }
  int64_t as_int() const;
  uint64_t as_uint() const;
  double as_double() const;
  const std::string& as_string() const { return s_; }

  // arrays
  size_t size() const { return t_ == Type::Array ? arr_.size() : obj_.size(); }
  const Json& at(size_t i) const { return arr_.at(i); }
  Json& push(Json v) { arr_.push_back(std::move(v)); return arr_.back(); }
  const std::vector<Json>& items() const { return arr_; }
  // objects
  bool has(const std::string& k) const { return obj_.count(k) != 0; }
  const Json& operator[](const std::string& k) const;
  Json& set(const std::string& k, Json v) { return obj_[k] = std::move(v); }
  void erase(const std::string& k) { obj_.erase(k); }
  const std::map<std::string, Json>& members() const { return obj_; }
  // JSON pointer lookup ("/integrity/body_sha256"); returns null when absent.
  const Json& pointer(const std::string& path) const;

  static Json parse(const std::string& text);
  static Json parse(const char* p, size_t n);
  std::string dump() const;            // compact, keys sorted (std::map order == bytewise)
  std::string canonical() const { return dump(); }

 private:
  Type t_ = Type::Null;
  bool b_ = false;
  int64_t i_ = 0;
  uint64_t u_ = 0;
  double f_ = 0;
  std::string s_;
  std::vector<Json> arr_;
  std::map<std::string, Json> obj_;
};

std::string json_escape(const std::string& s);
std::string json_number(double v);

}  // namespace hk
