// JSON-mode constrained sampling: a byte-level pushdown automaton over RFC 8259 JSON that tells
// which tokens can continue the text generated so far, so the sampler only draws tokens that keep
// the output a prefix of one JSON object (OpenAI `response_format: {"type": "json_object"}`).
//
// The state is the container stack plus the position inside the current token class (string with
// escape / \u digits, number sub-states, literal remainder). A candidate token is accepted when
// every byte of its text is a valid continuation; end-of-generation tokens are accepted only once
// the top-level object is complete. For generation (the default) the output must start with '{'
// and whitespace comes at most one byte at a time outside strings, so every accepted token makes
// progress (an unconstrained model could otherwise emit whitespace forever); `lenient_whitespace`
// accepts any whitespace JSON allows (validation of complete texts).
//
// Parity: crates/hawking-core/src/json_constrain.rs (JsonConstraint::{advance, mask_logits,
// is_done, validate}, JsonVocabIndex).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace hk {

class Tokenizer;

class JsonConstraint {
 public:
  explicit JsonConstraint(bool lenient_whitespace = false) : lenient_(lenient_whitespace) {}
  // Whether `bytes` (a token's text) can follow the current state.
  bool accepts(const std::string& bytes) const;
  // Consume `bytes` (must be accepted); returns false (state unchanged) when it is not.
  bool advance(const std::string& bytes);
  // The top-level object is closed (only whitespace may follow).
  bool done() const { return mode_ == Mode::Done; }
  // Highest-scoring allowed token among logits[0..n) (end-of-generation only when done), or -1.
  int32_t pick(const Tokenizer& tok, const float* logits, int64_t n) const;
  // Sets every token that cannot follow to -inf.
  void mask(const Tokenizer& tok, float* logits, int64_t n) const;
  // Whether `text` as a whole is one complete JSON object (surrounding whitespace allowed).
  static bool validate(const std::string& text);

 private:
  enum class Mode : uint8_t { Start, Value, ObjKeyOrEnd, ObjKey, Colon, After, ArrValueOrEnd, Str, Num, Lit, Done };
  bool step(uint8_t c);
  bool end_number();  // a number ends: continue in After
  Mode mode_ = Mode::Start;
  std::vector<char> stack_;  // '{' or '['
  bool key_ = false;          // the current string is an object key
  uint8_t esc_ = 0;           // 0 none, 1 after '\', 2..5 hex digits of \uXXXX left + 1
  uint8_t num_ = 0;           // number sub-state (see json_constrain.cpp)
  std::string lit_;           // remaining bytes of true / false / null
  bool lenient_ = false;
  uint8_t ws_run_ = 0;        // consecutive whitespace bytes outside strings
};

}  // namespace hk
