// Tokenizer built from the vocabulary embedded in a GGUF file, or from a Hugging Face tokenizer.json.
//
// Two GGUF vocabulary kinds are supported:
//   * byte-level BPE (`tokenizer.ggml.model` = "gpt2", or "llama" with merges): text is split
//     into pre-tokens (GPT-2 / Llama-3 / Qwen2 splitting rules, picked by `tokenizer.ggml.pre`),
//     every byte is mapped through the GPT-2 printable-byte alphabet, then merges are applied
//     lowest rank first;
//   * SentencePiece with scores (`tokenizer.ggml.model` = "llama" and no merges): spaces become
//     U+2581, a leading space is added, adjacent symbols are merged highest score first, and
//     pieces missing from the vocabulary fall back to <0xXX> byte tokens.
// Control tokens (`<|...|>` family, <s>, </s>, ... and GGUF token_type 3/4) are matched atomically
// in the input text. End-of-generation ids are the declared eos plus the turn terminators.
//
// Parity: crates/hawking-core/src/tokenizer.rs:156 (from_gguf), :241 (encode), :266 (decode),
// :281 (decode_one), :309 (is_eog), :68-115 (special / end-of-generation sets), :362
// (add_bos default for "llama-bpe"), :417-548 (SentencePiece bigram merge with byte fallback), :131
// (Tokenizer::from_file, tokenizer.json).
#pragma once
#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace hk {

class GgufFile;

struct TokenizerSpec {
  std::string model = "gpt2";   // "gpt2" | "llama"
  std::string pre = "default";  // "default" (GPT-2) | "llama-bpe" | "qwen2" | ...
  std::vector<std::string> tokens;
  std::vector<std::string> merges;  // "left right"
  std::vector<float> scores;
  std::vector<int32_t> token_types;  // optional (1 normal, 2 unknown, 3 control, 4 user, 6 byte)
  int32_t bos = -1, eos = -1, unk = -1, pad = -1;
  int add_bos = -1;  // -1: default for the vocabulary kind
  bool add_eos = false;
};

class Tokenizer {
 public:
  static std::unique_ptr<Tokenizer> from_spec(const TokenizerSpec& spec);
  static std::unique_ptr<Tokenizer> from_gguf(const GgufFile& f);
  // Hugging Face `tokenizer.json` (+ the `tokenizer_config.json` beside it, when present, for the
  // bos / eos tokens and add_bos): model BPE with a ByteLevel pre-tokenizer (its split regex
  // mapped to the GPT-2 / Llama-3 / Qwen2 rules), BPE with byte fallback (SentencePiece-style:
  // merge ranks become scores), or Unigram (SentencePiece with its scores). Added tokens are
  // control tokens when marked special.
  static std::unique_ptr<Tokenizer> from_json(const std::string& tokenizer_json, const std::string& config_json = "");

  std::vector<int32_t> encode(const std::string& text, bool add_special = true) const;
  std::string decode(const std::vector<int32_t>& ids, bool skip_special = true) const;
  // Raw bytes of one token (may be an incomplete UTF-8 sequence for byte-level vocabularies).
  std::string token_bytes(int32_t id) const;

  bool is_special(int32_t id) const { return special_.count(id) != 0; }
  bool is_eog(int32_t id) const { return eog_.count(id) != 0; }
  std::vector<int32_t> eog_ids() const { return std::vector<int32_t>(eog_.begin(), eog_.end()); }
  int32_t bos() const { return bos_; }
  int32_t eos() const { return eos_; }
  int32_t pad() const { return pad_; }
  bool add_bos() const { return add_bos_; }
  size_t vocab_size() const { return tokens_.size(); }
  const std::string& token(int32_t id) const { return tokens_.at(id); }
  int32_t find(const std::string& piece) const;
  bool is_spm() const { return spm_; }

 private:
  void encode_bpe_piece(const std::string& utf8, std::vector<int32_t>& out) const;
  void encode_bpe_text(const std::string& text, std::vector<int32_t>& out) const;
  void encode_spm_text(const std::string& text, std::vector<int32_t>& out) const;
  void spm_emit(const std::string& piece, std::vector<int32_t>& out) const;

  bool spm_ = false;
  std::string pre_;
  std::vector<std::string> tokens_;
  std::vector<float> scores_;
  std::unordered_map<std::string, int32_t> index_;
  std::unordered_map<std::string, int32_t> merge_rank_;  // "left\x01right" -> rank
  std::vector<std::string> specials_by_len_;               // control strings, longest first
  std::unordered_set<int32_t> special_, eog_;
  int32_t bos_ = -1, eos_ = -1, unk_ = -1, pad_ = -1;
  bool add_bos_ = false, add_eos_ = false;
  std::vector<std::string> byte_to_unicode_;  // 256 UTF-8 strings
  std::unordered_map<uint32_t, uint8_t> unicode_to_byte_;
  mutable std::unordered_map<std::string, std::vector<int32_t>> cache_;  // pre-token -> ids
};

// Incremental detokeniser for streaming: returns only complete UTF-8 text, holding back the
// bytes of a partial character until the next token completes it.
class StreamDecoder {
 public:
  explicit StreamDecoder(const Tokenizer* t, bool skip_special = true) : t_(t), skip_(skip_special) {}
  std::string push(int32_t id);
  std::string flush();

 private:
  const Tokenizer* t_;
  bool skip_;
  bool first_ = true;
  std::string pending_;
};

// Pre-tokenizer splitting (exposed for tests): returns the pre-token strings of `text`.
std::vector<std::string> pretokenize(const std::string& text, const std::string& pre);

}  // namespace hk
