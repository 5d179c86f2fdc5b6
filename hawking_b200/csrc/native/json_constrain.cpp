#include "json_constrain.h"

#include <algorithm>
#include <cmath>
#include <limits>
#include <numeric>

#include "tokenizer.h"

namespace hk {

// Number sub-states (num_): 1 after '-', 2 after a leading '0', 3 integer digits, 4 after '.',
// 5 fraction digits, 6 after 'e', 7 after the exponent sign, 8 exponent digits. A number may end
// in 2, 3, 5 and 8.
namespace {
bool ws(uint8_t c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }
bool digit(uint8_t c) { return c >= '0' && c <= '9'; }
bool hex(uint8_t c) { return digit(c) || (c >= 'a' && c <= 'f') || (c >= 'A' && c <= 'F'); }
}  // namespace

bool JsonConstraint::end_number() {
  if (num_ != 2 && num_ != 3 && num_ != 5 && num_ != 8) return false;
  num_ = 0;
  mode_ = Mode::After;
  return true;
}

bool JsonConstraint::step(uint8_t c) {
  if (!lenient_ && mode_ != Mode::Str && mode_ != Mode::Num && ws(c)) {
    if (mode_ == Mode::Start || ws_run_ >= 1) return false;  // progress: no leading / repeated whitespace
    ++ws_run_;
  } else if (mode_ != Mode::Num || !ws(c)) {
    ws_run_ = 0;
  }
  auto after_close = [&] { mode_ = stack_.empty() ? Mode::Done : Mode::After; };
  auto begin_value = [&](uint8_t ch) -> bool {
    switch (ch) {
      case '{': stack_.push_back('{'); mode_ = Mode::ObjKeyOrEnd; return true;
      case '[': stack_.push_back('['); mode_ = Mode::ArrValueOrEnd; return true;
      case '"': key_ = false; esc_ = 0; mode_ = Mode::Str; return true;
      case '-': num_ = 1; mode_ = Mode::Num; return true;
      case '0': num_ = 2; mode_ = Mode::Num; return true;
      case 't': lit_ = "rue"; mode_ = Mode::Lit; return true;
      case 'f': lit_ = "alse"; mode_ = Mode::Lit; return true;
      case 'n': lit_ = "ull"; mode_ = Mode::Lit; return true;
      default:
        if (ch >= '1' && ch <= '9') { num_ = 3; mode_ = Mode::Num; return true; }
        return false;
    }
  };
  switch (mode_) {
    case Mode::Start:
      if (ws(c)) return true;
      if (c != '{') return false;  // a JSON object at the top level
      stack_.push_back('{');
      mode_ = Mode::ObjKeyOrEnd;
      return true;
    case Mode::Value:
      return ws(c) || begin_value(c);
    case Mode::ArrValueOrEnd:
      if (ws(c)) return true;
      if (c == ']') { stack_.pop_back(); after_close(); return true; }
      return begin_value(c);
    case Mode::ObjKeyOrEnd:
      if (ws(c)) return true;
      if (c == '}') { stack_.pop_back(); after_close(); return true; }
      if (c == '"') { key_ = true; esc_ = 0; mode_ = Mode::Str; return true; }
      return false;
    case Mode::ObjKey:
      if (ws(c)) return true;
      if (c == '"') { key_ = true; esc_ = 0; mode_ = Mode::Str; return true; }
      return false;
    case Mode::Colon:
      if (ws(c)) return true;
      if (c == ':') { mode_ = Mode::Value; return true; }
      return false;
    case Mode::After:
      if (ws(c)) return true;
      if (c == ',') { mode_ = stack_.back() == '{' ? Mode::ObjKey : Mode::Value; return true; }
      if ((c == '}' && stack_.back() == '{') || (c == ']' && stack_.back() == '[')) {
        stack_.pop_back();
        after_close();
        return true;
      }
      return false;
    case Mode::Str:
      if (esc_ == 1) {
        if (c == 'u') { esc_ = 5; return true; }
        if (c == '"' || c == '\\' || c == '/' || c == 'b' || c == 'f' || c == 'n' || c == 'r' || c == 't') {
          esc_ = 0;
          return true;
        }
        return false;
      }
      if (esc_ >= 2) {
        if (!hex(c)) return false;
        esc_ = esc_ == 2 ? 0 : esc_ - 1;
        return true;
      }
      if (c == '\\') { esc_ = 1; return true; }
      if (c == '"') { mode_ = key_ ? Mode::Colon : Mode::After; return true; }
      return c >= 0x20;  // raw control characters are not allowed inside strings
    case Mode::Num:
      switch (num_) {
        case 1:
          if (c == '0') { num_ = 2; return true; }
          if (c >= '1' && c <= '9') { num_ = 3; return true; }
          return false;
        case 2:
        case 3:
          if (num_ == 3 && digit(c)) return true;
          if (c == '.') { num_ = 4; return true; }
          if (c == 'e' || c == 'E') { num_ = 6; return true; }
          break;
        case 4:
          if (digit(c)) { num_ = 5; return true; }
          return false;
        case 5:
          if (digit(c)) return true;
          if (c == 'e' || c == 'E') { num_ = 6; return true; }
          break;
        case 6:
          if (c == '+' || c == '-') { num_ = 7; return true; }
          if (digit(c)) { num_ = 8; return true; }
          return false;
        case 7:
          if (digit(c)) { num_ = 8; return true; }
          return false;
        case 8:
          if (digit(c)) return true;
          break;
      }
      // the number ends here; the byte belongs to what follows it
      return end_number() && step(c);
    case Mode::Lit:
      if (lit_.empty() || (uint8_t)lit_[0] != c) return false;
      lit_.erase(0, 1);
      if (lit_.empty()) mode_ = Mode::After;
      return true;
    case Mode::Done:
      return ws(c);
  }
  return false;
}

bool JsonConstraint::accepts(const std::string& bytes) const {
  if (bytes.empty()) return false;  // no progress (control / empty tokens)
  JsonConstraint t = *this;
  for (unsigned char c : bytes)
    if (!t.step(c)) return false;
  return true;
}

bool JsonConstraint::advance(const std::string& bytes) {
  JsonConstraint t = *this;
  for (unsigned char c : bytes)
    if (!t.step(c)) return false;
  *this = std::move(t);
  return true;
}

int32_t JsonConstraint::pick(const Tokenizer& tok, const float* logits, int64_t n) const {
  std::vector<int32_t> order((size_t)n);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int32_t x, int32_t y) { return logits[x] > logits[y]; });
  for (int32_t id : order) {
    if (!std::isfinite(logits[id])) break;
    if (tok.is_eog(id)) {
      if (done()) return id;
      continue;
    }
    if (tok.is_special(id)) continue;
    if (accepts(tok.token_bytes(id))) return id;
  }
  return -1;
}

void JsonConstraint::mask(const Tokenizer& tok, float* logits, int64_t n) const {
  const float ninf = -std::numeric_limits<float>::infinity();
  for (int64_t id = 0; id < n; ++id) {
    bool ok;
    if (tok.is_eog((int32_t)id)) ok = done();
    else ok = !tok.is_special((int32_t)id) && accepts(tok.token_bytes((int32_t)id));
    if (!ok) logits[id] = ninf;
  }
}

bool JsonConstraint::validate(const std::string& text) {
  JsonConstraint c(true);
  for (unsigned char ch : text)
    if (!c.step(ch)) return false;
  return c.done();
}

}  // namespace hk
