// GGUF-vocabulary tokenizer; see tokenizer.h.
#include "tokenizer.h"

#include <cstdio>

#include "json.h"

#include <algorithm>
#include <climits>
#include <cstdint>
#include <cstdio>
#include <queue>
#include <stdexcept>

#include "gguf.h"

namespace hk {

namespace {

// ---- UTF-8 ---------------------------------------------------------------------------------
std::vector<uint32_t> utf8_decode(const std::string& s, std::vector<size_t>* offsets = nullptr) {
  std::vector<uint32_t> cps;
  size_t i = 0;
  while (i < s.size()) {
    const uint8_t c = (uint8_t)s[i];
    uint32_t cp = c;
    size_t n = 1;
    if (c >= 0xF0) {
      n = 4;
      cp = c & 0x07;
    } else if (c >= 0xE0) {
      n = 3;
      cp = c & 0x0F;
    } else if (c >= 0xC0) {
      n = 2;
      cp = c & 0x1F;
    }
    if (n > 1) {
      if (i + n > s.size()) { n = 1; cp = c; }
      else {
        for (size_t k = 1; k < n; ++k) {
          const uint8_t cc = (uint8_t)s[i + k];
          if ((cc & 0xC0) != 0x80) { n = 1; cp = c; break; }
          cp = (cp << 6) | (cc & 0x3F);
        }
      }
    }
    if (offsets) offsets->push_back(i);
    cps.push_back(cp);
    i += n;
  }
  if (offsets) offsets->push_back(s.size());
  return cps;
}

std::string utf8_encode(uint32_t cp) {
  std::string o;
  if (cp < 0x80) o += (char)cp;
  else if (cp < 0x800) { o += (char)(0xC0 | (cp >> 6)); o += (char)(0x80 | (cp & 0x3F)); }
  else if (cp < 0x10000) {
    o += (char)(0xE0 | (cp >> 12)); o += (char)(0x80 | ((cp >> 6) & 0x3F)); o += (char)(0x80 | (cp & 0x3F));
  } else {
    o += (char)(0xF0 | (cp >> 18)); o += (char)(0x80 | ((cp >> 12) & 0x3F));
    o += (char)(0x80 | ((cp >> 6) & 0x3F)); o += (char)(0x80 | (cp & 0x3F));
  }
  return o;
}

// Length of the complete-UTF-8 prefix of s (an incomplete trailing sequence is held back).
size_t utf8_complete_prefix(const std::string& s) {
  size_t n = s.size();
  for (size_t back = 1; back <= 3 && back <= n; ++back) {
    const uint8_t c = (uint8_t)s[n - back];
    if ((c & 0xC0) == 0x80) continue;  // continuation byte: keep looking for the lead
    size_t need = c >= 0xF0 ? 4 : c >= 0xE0 ? 3 : c >= 0xC0 ? 2 : 1;
    return need > back ? n - back : n;
  }
  return n;
}

// ---- Unicode classes used by the pre-tokenizer --------------------------------------------
// Approximations of \s, \p{N} and \p{L} over the scripts that LLM vocabularies cover; code points
// outside the listed ranges are classed as "other" (punctuation / symbols).
bool is_space(uint32_t c) {
  return c == ' ' || (c >= 0x09 && c <= 0x0D) || c == 0x85 || c == 0xA0 || c == 0x1680 ||
         (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F || c == 0x205F || c == 0x3000;
}
bool is_number(uint32_t c) {
  return (c >= '0' && c <= '9') || c == 0xB2 || c == 0xB3 || c == 0xB9 || (c >= 0xBC && c <= 0xBE) ||
         (c >= 0x660 && c <= 0x669) || (c >= 0x6F0 && c <= 0x6F9) || (c >= 0x966 && c <= 0x96F) ||
         (c >= 0x2070 && c <= 0x2079) || (c >= 0x2080 && c <= 0x2089) || (c >= 0x2150 && c <= 0x2189) ||
         (c >= 0x2460 && c <= 0x249B) || (c >= 0xFF10 && c <= 0xFF19);
}
bool is_letter(uint32_t c) {
  if (c < 0x80) return (c >= 'A' && c <= 'Z') || (c >= 'a' && c <= 'z');
  if (is_number(c) || is_space(c)) return false;
  return c == 0xAA || c == 0xB5 || c == 0xBA || (c >= 0xC0 && c <= 0xD6) || (c >= 0xD8 && c <= 0xF6) ||
         (c >= 0xF8 && c <= 0x2FF) || (c >= 0x370 && c <= 0x3FF && c != 0x37E && c != 0x387) ||
         (c >= 0x400 && c <= 0x52F) || (c >= 0x531 && c <= 0x587) || (c >= 0x5D0 && c <= 0x5F2) ||
         (c >= 0x620 && c <= 0x64A) || (c >= 0x671 && c <= 0x6D3) || (c >= 0x900 && c <= 0xDFF) ||
         (c >= 0xE01 && c <= 0xE30) || (c >= 0xE40 && c <= 0xE4E) || (c >= 0x10A0 && c <= 0x10FF) ||
         (c >= 0x1100 && c <= 0x11FF) || (c >= 0x1E00 && c <= 0x1FFF) || (c >= 0x3040 && c <= 0x30FF) ||
         (c >= 0x3105 && c <= 0x312F) || (c >= 0x3131 && c <= 0x318E) || (c >= 0x3400 && c <= 0x4DBF) ||
         (c >= 0x4E00 && c <= 0x9FFF) || (c >= 0xA000 && c <= 0xA48C) || (c >= 0xAC00 && c <= 0xD7A3) ||
         (c >= 0xF900 && c <= 0xFAFF) || (c >= 0xFF21 && c <= 0xFF3A) || (c >= 0xFF41 && c <= 0xFF5A) ||
         (c >= 0xFF66 && c <= 0xFFDC) || (c >= 0x20000 && c <= 0x2FFFF);
}
bool is_other(uint32_t c) { return !is_space(c) && !is_letter(c) && !is_number(c); }
bool is_nl(uint32_t c) { return c == '\r' || c == '\n'; }
uint32_t lower(uint32_t c) { return (c >= 'A' && c <= 'Z') ? c + 32 : c; }

// English contractions 's 't 're 've 'm 'll 'd at i; returns the match length or 0.
size_t contraction(const std::vector<uint32_t>& cp, size_t i, bool icase) {
  if (cp[i] != '\'' || i + 1 >= cp.size()) return 0;
  auto at = [&](size_t k) { return i + k < cp.size() ? (icase ? lower(cp[i + k]) : cp[i + k]) : 0u; };
  const uint32_t a = at(1), b = at(2);
  if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
  if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
  return 0;
}

// Whitespace handling shared by both rule sets: \s+(?!\S) then \s+.
size_t space_run(const std::vector<uint32_t>& cp, size_t i) {
  size_t e = i;
  while (e < cp.size() && is_space(cp[e])) ++e;
  if (e == i) return 0;
  if (e == cp.size() || e - i == 1) return e - i;
  return e - i - 1;  // leave the last space to prefix the next word
}

}  // namespace

// ---- pre-tokenizer -----------------------------------------------------------------------------
// "default": GPT-2 rules   's|'t|'re|'ve|'m|'ll|'d| ?L+| ?N+| ?O+|\s+(?!\S)|\s+
// "llama-bpe" / "qwen2" / others: Llama-3 rules (case-insensitive contractions, an optional
//   non-letter prefix before letters, digit groups of at most 3 (1 for qwen2), punctuation runs
//   followed by newlines, newline-terminated whitespace runs).
std::vector<std::string> pretokenize(const std::string& text, const std::string& pre) {
  std::vector<size_t> off;
  const std::vector<uint32_t> cp = utf8_decode(text, &off);
  std::vector<std::string> out;
  const bool gpt2 = pre == "default" || pre == "gpt2" || pre.empty();
  const size_t max_digits = (pre == "qwen2" || pre == "deepseek-llm") ? 1 : 3;
  size_t i = 0;
  const size_t n = cp.size();
  while (i < n) {
    size_t len = 0;
    if (gpt2) {
      len = contraction(cp, i, false);
      if (!len) {
        size_t j = i + (cp[i] == ' ' && i + 1 < n ? 1 : 0);
        auto run = [&](bool (*cls)(uint32_t)) {
          size_t e = j;
          while (e < n && cls(cp[e])) ++e;
          return e > j ? e - i : 0;
        };
        if (j < n && is_letter(cp[j])) len = run(is_letter);
        else if (j < n && is_number(cp[j])) len = run(is_number);
        else if (j < n && is_other(cp[j])) len = run(is_other);
      }
      if (!len) len = space_run(cp, i);
    } else {
      len = contraction(cp, i, true);
      if (!len) {  // [^\r\n\p{L}\p{N}]?\p{L}+
        size_t j = i;
        if (!is_letter(cp[j]) && !is_number(cp[j]) && !is_nl(cp[j]) && j + 1 < n && is_letter(cp[j + 1])) ++j;
        if (is_letter(cp[j])) {
          size_t e = j;
          while (e < n && is_letter(cp[e])) ++e;
          len = e - i;
        }
      }
      if (!len && is_number(cp[i])) {  // \p{N}{1,max}
        size_t e = i;
        while (e < n && e - i < max_digits && is_number(cp[e])) ++e;
        len = e - i;
      }
      if (!len) {  //  ?[^\s\p{L}\p{N}]+[\r\n]*
        size_t j = i + (cp[i] == ' ' ? 1 : 0);
        if (j < n && is_other(cp[j])) {
          size_t e = j;
          while (e < n && is_other(cp[e])) ++e;
          while (e < n && is_nl(cp[e])) ++e;
          len = e - i;
        }
      }
      if (!len && is_space(cp[i])) {  // \s*[\r\n]+
        size_t e = i, last_nl = SIZE_MAX;
        while (e < n && is_space(cp[e])) {
          if (is_nl(cp[e])) last_nl = e;
          ++e;
        }
        if (last_nl != SIZE_MAX) len = last_nl + 1 - i;
      }
      if (!len) len = space_run(cp, i);
    }
    if (!len) len = 1;
    out.push_back(text.substr(off[i], off[i + len] - off[i]));
    i += len;
  }
  return out;
}

// ---- construction ------------------------------------------------------------------------------
namespace {
bool special_shape(const std::string& s) {
  if (s.size() >= 4 && s.compare(0, 2, "<|") == 0 && s.compare(s.size() - 2, 2, "|>") == 0) return true;
  static const char* kNames[] = {"<s>", "</s>", "<unk>", "<pad>", "<mask>", "<bos>", "<eos>",
                                 "<start_of_turn>", "<end_of_turn>"};
  for (const char* k : kNames)
    if (s == k) return true;
  return false;
}
const char* kEog[] = {"<|im_end|>", "<|endoftext|>", "<|eot_id|>", "<|end|>", "<|end_of_text|>",
                      "<end_of_turn>", "</s>", "<eos>"};
}  // namespace

std::unique_ptr<Tokenizer> Tokenizer::from_spec(const TokenizerSpec& sp) {
  std::unique_ptr<Tokenizer> t(new Tokenizer());
  if (sp.tokens.empty()) throw std::runtime_error("tokenizer: empty vocabulary");
  t->tokens_ = sp.tokens;
  t->pre_ = sp.pre;
  t->spm_ = sp.model == "llama" && sp.merges.empty();
  if (!t->spm_ && sp.model != "gpt2" && sp.model != "llama")
    throw std::runtime_error("tokenizer: unsupported tokenizer.ggml.model '" + sp.model + "'");
  if (t->spm_) {
    if (sp.scores.size() != sp.tokens.size())
      throw std::runtime_error("tokenizer: SentencePiece vocabulary needs one score per token");
    t->scores_ = sp.scores;
  }
  for (size_t i = 0; i < t->tokens_.size(); ++i) t->index_.emplace(t->tokens_[i], (int32_t)i);
  for (size_t r = 0; r < sp.merges.size(); ++r) {
    const std::string& m = sp.merges[r];
    const size_t sp_pos = m.find(' ');
    if (sp_pos == std::string::npos) continue;
    t->merge_rank_.emplace(m.substr(0, sp_pos) + '\x01' + m.substr(sp_pos + 1), (int32_t)r);
  }
  t->bos_ = sp.bos;
  t->eos_ = sp.eos;
  t->unk_ = sp.unk;
  t->pad_ = sp.pad;
  t->add_bos_ = sp.add_bos >= 0 ? sp.add_bos != 0 : (t->spm_ || sp.pre == "llama-bpe");
  t->add_eos_ = sp.add_eos;
  for (int32_t id : {sp.bos, sp.eos, sp.pad, sp.unk})
    if (id >= 0) t->special_.insert(id);
  if (sp.eos >= 0) t->eog_.insert(sp.eos);
  for (size_t i = 0; i < t->tokens_.size(); ++i) {
    const std::string& s = t->tokens_[i];
    const int tt = i < sp.token_types.size() ? sp.token_types[i] : 1;
    const bool control = tt == 3 || tt == 4 || special_shape(s);
    if (control) {
      t->special_.insert((int32_t)i);
      if (!s.empty()) t->specials_by_len_.push_back(s);
    }
    for (const char* e : kEog)
      if (s == e) { t->eog_.insert((int32_t)i); t->special_.insert((int32_t)i); }
  }
  std::sort(t->specials_by_len_.begin(), t->specials_by_len_.end(),
            [](const std::string& a, const std::string& b) { return a.size() > b.size(); });
  // GPT-2 printable-byte alphabet: printable Latin-1 bytes map to themselves, the other 68 bytes
  // to U+0100.. in byte order.
  t->byte_to_unicode_.resize(256);
  int extra = 0;
  for (int b = 0; b < 256; ++b) {
    const bool keep = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
    const uint32_t cp = keep ? (uint32_t)b : 256u + (uint32_t)extra++;
    t->byte_to_unicode_[b] = utf8_encode(cp);
    t->unicode_to_byte_[cp] = (uint8_t)b;
  }
  return t;
}

std::unique_ptr<Tokenizer> Tokenizer::from_gguf(const GgufFile& f) {
  const auto& kv = f.metadata();
  auto str = [&](const char* k, const std::string& d) {
    auto it = kv.find(k);
    return it == kv.end() ? d : it->second.s;
  };
  auto integer = [&](const char* k, int64_t d) {
    auto it = kv.find(k);
    return it == kv.end() ? d : it->second.i;
  };
  auto strs = [&](const char* k) {
    std::vector<std::string> v;
    auto it = kv.find(k);
    if (it != kv.end() && it->second.arr)
      for (const auto& e : *it->second.arr) v.push_back(e.s);
    return v;
  };
  TokenizerSpec sp;
  sp.model = str("tokenizer.ggml.model", "");
  if (sp.model.empty()) throw std::runtime_error("tokenizer: gguf has no tokenizer.ggml.model");
  sp.pre = str("tokenizer.ggml.pre", "default");
  sp.tokens = strs("tokenizer.ggml.tokens");
  sp.merges = strs("tokenizer.ggml.merges");
  auto it = kv.find("tokenizer.ggml.scores");
  if (it != kv.end() && it->second.arr)
    for (const auto& e : *it->second.arr) sp.scores.push_back((float)e.f);
  it = kv.find("tokenizer.ggml.token_type");
  if (it != kv.end() && it->second.arr)
    for (const auto& e : *it->second.arr) sp.token_types.push_back((int32_t)e.i);
  sp.bos = (int32_t)integer("tokenizer.ggml.bos_token_id", -1);
  sp.eos = (int32_t)integer("tokenizer.ggml.eos_token_id", -1);
  sp.unk = (int32_t)integer("tokenizer.ggml.unknown_token_id", -1);
  sp.pad = (int32_t)integer("tokenizer.ggml.padding_token_id", -1);
  it = kv.find("tokenizer.ggml.add_bos_token");
  if (it != kv.end()) sp.add_bos = it->second.i != 0;
  it = kv.find("tokenizer.ggml.add_eos_token");
  if (it != kv.end()) sp.add_eos = it->second.i != 0;
  return from_spec(sp);
}

namespace {
// The pre-tokenizer rule set named by a Split regex of a tokenizer.json.
std::string pre_from_regex(const std::string& re) {
  const bool three_digits = re.find("\\p{N}{1,3}") != std::string::npos;
  const bool single_digit = re.find("|\\p{N}|") != std::string::npos || re.find("\\p{N}|") != std::string::npos;
  const bool ci_contractions = re.find("(?i:'s|'t|'re|'ve|'m|'ll|'d)") != std::string::npos;
  if (three_digits && ci_contractions) return "llama-bpe";
  if (ci_contractions && single_digit) return "qwen2";
  return "default";
}
void find_split_regex(const Json& pt, std::string* re, bool* byte_level) {
  if (!pt.is_object()) return;
  const std::string type = pt.has("type") ? pt["type"].as_string() : "";
  if (type == "ByteLevel") *byte_level = true;
  if (type == "Split" && pt.has("pattern") && pt["pattern"].is_object()) {
    const Json& pat = pt["pattern"];
    if (pat.has("Regex")) *re = pat["Regex"].as_string();
  }
  if (type == "Sequence" && pt.has("pretokenizers"))
    for (const auto& sub : pt["pretokenizers"].items()) find_split_regex(sub, re, byte_level);
}
std::string read_file(const std::string& path) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) throw std::runtime_error("tokenizer: cannot open " + path);
  std::string s;
  char buf[1 << 16];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) s.append(buf, n);
  std::fclose(f);
  return s;
}
std::string token_text(const Json& v) {  // "bos_token": "<s>" or {"content": "<s>", ...}
  if (v.is_string()) return v.as_string();
  if (v.is_object() && v.has("content")) return v["content"].as_string();
  return "";
}
}  // namespace

std::unique_ptr<Tokenizer> Tokenizer::from_json(const std::string& tokenizer_json, const std::string& config_json) {
  const Json j = Json::parse(read_file(tokenizer_json));
  const Json& model = j["model"];
  if (!model.is_object()) throw std::runtime_error("tokenizer.json: no model");
  const std::string type = model.has("type") ? model["type"].as_string() : "BPE";
  TokenizerSpec sp;
  std::vector<std::string> tokens;
  std::vector<float> scores;
  auto put = [&](int64_t id, const std::string& s, float score) {
    if (id < 0) throw std::runtime_error("tokenizer.json: negative id");
    if ((size_t)id >= tokens.size()) {
      tokens.resize((size_t)id + 1);
      scores.resize((size_t)id + 1, -1e9f);
    }
    tokens[(size_t)id] = s;
    scores[(size_t)id] = score;
  };
  std::unordered_map<std::string, int64_t> rank_of;  // merged token -> merge rank (byte fallback)
  if (type == "BPE") {
    for (const auto& kv : model["vocab"].members()) put(kv.second.as_int(), kv.first, 0.f);
    const Json& merges = model["merges"];
    int64_t r = 0;
    for (const auto& m : merges.items()) {
      std::string a, b;
      if (m.is_string()) {
        const std::string& t = m.as_string();
        const size_t sp_pos = t.find(' ');
        if (sp_pos == std::string::npos) continue;
        a = t.substr(0, sp_pos);
        b = t.substr(sp_pos + 1);
      } else if (m.is_array() && m.size() == 2) {
        a = m.at(0).as_string();
        b = m.at(1).as_string();
      } else {
        continue;
      }
      sp.merges.push_back(a + " " + b);
      rank_of.emplace(a + b, r++);
    }
  } else if (type == "Unigram") {
    int64_t id = 0;
    for (const auto& e : model["vocab"].items()) put(id++, e.at(0).as_string(), (float)e.at(1).as_double());
    if (model.has("unk_id") && model["unk_id"].is_number()) sp.unk = (int32_t)model["unk_id"].as_int();
  } else {
    throw std::runtime_error("tokenizer.json: model type '" + type + "' not supported");
  }
  std::vector<int32_t> types;
  if (j.has("added_tokens"))
    for (const auto& t : j["added_tokens"].items()) {
      const int64_t id = t["id"].as_int();
      put(id, t["content"].as_string(), 0.f);
      if (types.size() < tokens.size()) types.resize(tokens.size(), 1);
      types[(size_t)id] = t.has("special") && t["special"].as_bool() ? 3 : 4;
    }
  types.resize(tokens.size(), 1);
  for (size_t i = 0; i < tokens.size(); ++i)
    if (tokens[i].empty()) {
      tokens[i] = "[UNUSED_" + std::to_string(i) + "]";
      types[i] = 3;
    }
  const bool byte_fallback = type == "BPE" && model.has("byte_fallback") && model["byte_fallback"].as_bool();
  if (type == "Unigram" || byte_fallback) {
    // SentencePiece: highest score merges first; a BPE vocabulary's merge order becomes the score
    sp.model = "llama";
    if (byte_fallback) {
      for (size_t i = 0; i < tokens.size(); ++i) {
        auto it = rank_of.find(tokens[i]);
        scores[i] = it == rank_of.end() ? -1e9f : -(float)it->second;
      }
      sp.merges.clear();
    }
    sp.scores = scores;
  } else {
    sp.model = "gpt2";
    std::string re;
    bool byte_level = false;
    find_split_regex(j["pre_tokenizer"], &re, &byte_level);
    if (!byte_level) throw std::runtime_error("tokenizer.json: BPE without a ByteLevel pre-tokenizer");
    sp.pre = re.empty() ? "default" : pre_from_regex(re);
  }
  sp.tokens = tokens;
  sp.token_types = types;
  auto id_of = [&](const std::string& s) -> int32_t {
    for (size_t i = 0; i < tokens.size(); ++i)
      if (tokens[i] == s) return (int32_t)i;
    return -1;
  };
  if (!config_json.empty()) {
    const Json c = Json::parse(read_file(config_json));
    if (c.has("bos_token")) sp.bos = id_of(token_text(c["bos_token"]));
    if (c.has("eos_token")) sp.eos = id_of(token_text(c["eos_token"]));
    if (c.has("unk_token")) sp.unk = id_of(token_text(c["unk_token"]));
    if (c.has("pad_token")) sp.pad = id_of(token_text(c["pad_token"]));
    if (c.has("add_bos_token") && !c["add_bos_token"].is_null()) sp.add_bos = c["add_bos_token"].as_bool() ? 1 : 0;
    if (c.has("add_eos_token") && !c["add_eos_token"].is_null()) sp.add_eos = c["add_eos_token"].as_bool();
  }
  return from_spec(sp);
}

int32_t Tokenizer::find(const std::string& piece) const {
  auto it = index_.find(piece);
  return it == index_.end() ? -1 : it->second;
}

// ---- encode ------------------------------------------------------------------------------------
std::vector<int32_t> Tokenizer::encode(const std::string& text, bool add_special) const {
  std::vector<int32_t> out;
  if (add_special && add_bos_ && bos_ >= 0) out.push_back(bos_);
  // split out control-token strings (matched atomically, longest first at each position)
  size_t pos = 0, seg = 0;
  std::string plain;
  auto flush = [&](size_t end) {
    if (end > seg) {
      const std::string part = text.substr(seg, end - seg);
      if (spm_) encode_spm_text(part, out);
      else encode_bpe_text(part, out);
    }
  };
  while (pos < text.size()) {
    bool hit = false;
    if (!specials_by_len_.empty() && text[pos] == '<') {
      for (const auto& s : specials_by_len_) {
        if (text.compare(pos, s.size(), s) == 0) {
          flush(pos);
          out.push_back(index_.at(s));
          pos += s.size();
          seg = pos;
          hit = true;
          break;
        }
      }
    }
    if (!hit) ++pos;
  }
  flush(text.size());
  if (add_special && add_eos_ && eos_ >= 0) out.push_back(eos_);
  return out;
}

void Tokenizer::encode_bpe_text(const std::string& text, std::vector<int32_t>& out) const {
  for (const std::string& p : pretokenize(text, pre_)) encode_bpe_piece(p, out);
}

void Tokenizer::encode_bpe_piece(const std::string& piece, std::vector<int32_t>& out) const {
  auto hit = cache_.find(piece);
  if (hit != cache_.end()) {
    out.insert(out.end(), hit->second.begin(), hit->second.end());
    return;
  }
  std::vector<std::string> sym;
  for (unsigned char b : piece) sym.push_back(byte_to_unicode_[b]);
  // GPT-2 merge loop: repeatedly merge every occurrence of the lowest-ranked adjacent pair.
  while (sym.size() > 1) {
    int32_t best = INT32_MAX;
    for (size_t i = 0; i + 1 < sym.size(); ++i) {
      auto it = merge_rank_.find(sym[i] + '\x01' + sym[i + 1]);
      if (it != merge_rank_.end() && it->second < best) best = it->second;
    }
    if (best == INT32_MAX) break;
    std::vector<std::string> nxt;
    for (size_t i = 0; i < sym.size();) {
      if (i + 1 < sym.size()) {
        auto it = merge_rank_.find(sym[i] + '\x01' + sym[i + 1]);
        if (it != merge_rank_.end() && it->second == best) {
          nxt.push_back(sym[i] + sym[i + 1]);
          i += 2;
          continue;
        }
      }
      nxt.push_back(sym[i]);
      ++i;
    }
    sym.swap(nxt);
  }
  std::vector<int32_t> ids;
  for (const auto& s : sym) {
    auto it = index_.find(s);
    if (it != index_.end()) { ids.push_back(it->second); continue; }
    // not in the vocabulary: fall back to its single-byte symbols
    for (uint32_t cp : utf8_decode(s)) {
      auto jt = index_.find(utf8_encode(cp));
      if (jt != index_.end()) ids.push_back(jt->second);
      else if (unk_ >= 0) ids.push_back(unk_);
    }
  }
  if (cache_.size() < 65536) cache_.emplace(piece, ids);
  out.insert(out.end(), ids.begin(), ids.end());
}

void Tokenizer::spm_emit(const std::string& piece, std::vector<int32_t>& out) const {
  auto it = index_.find(piece);
  if (it != index_.end()) { out.push_back(it->second); return; }
  for (unsigned char b : piece) {
    char buf[8];
    snprintf(buf, sizeof buf, "<0x%02X>", b);
    auto jt = index_.find(buf);
    if (jt != index_.end()) out.push_back(jt->second);
    else if (unk_ >= 0) out.push_back(unk_);
    else throw std::runtime_error("tokenizer: piece has no byte fallback");
  }
}

void Tokenizer::encode_spm_text(const std::string& text, std::vector<int32_t>& out) const {
  if (text.empty()) return;
  std::string esc;
  const std::string kSpace = "\xE2\x96\x81";  // U+2581
  esc += kSpace;  // leading-space prefix
  for (char c : text) {
    if (c == ' ') esc += kSpace;
    else esc += c;
  }
  struct Sym { int prev, next; size_t start, len; };
  std::vector<size_t> off;
  const auto cps = utf8_decode(esc, &off);
  std::vector<Sym> sym(cps.size());
  for (size_t i = 0; i < cps.size(); ++i)
    sym[i] = Sym{(int)i - 1, i + 1 < cps.size() ? (int)i + 1 : -1, off[i], off[i + 1] - off[i]};
  struct Big { float score; int left, right; size_t size; };
  auto cmp = [](const Big& a, const Big& b) {
    return a.score != b.score ? a.score < b.score : a.left > b.left;  // higher score, then leftmost
  };
  std::priority_queue<Big, std::vector<Big>, decltype(cmp)> q(cmp);
  auto try_add = [&](int l, int r) {
    if (l < 0 || r < 0 || sym[l].len == 0 || sym[r].len == 0) return;
    const size_t size = sym[l].len + sym[r].len;
    auto it = index_.find(esc.substr(sym[l].start, size));
    if (it != index_.end()) q.push(Big{scores_[it->second], l, r, size});
  };
  for (size_t i = 1; i < sym.size(); ++i) try_add((int)i - 1, (int)i);
  while (!q.empty()) {
    const Big b = q.top();
    q.pop();
    if (sym[b.left].next != b.right || sym[b.left].len == 0 || sym[b.right].len == 0 ||
        sym[b.left].len + sym[b.right].len != b.size)
      continue;
    sym[b.left].len = b.size;
    sym[b.right].len = 0;
    sym[b.left].next = sym[b.right].next;
    if (sym[b.right].next >= 0) sym[sym[b.right].next].prev = b.left;
    try_add(sym[b.left].prev, b.left);
    try_add(b.left, sym[b.left].next);
  }
  for (int i = sym.empty() ? -1 : 0; i >= 0; i = sym[i].next)
    if (sym[i].len) spm_emit(esc.substr(sym[i].start, sym[i].len), out);
}

// ---- decode ------------------------------------------------------------------------------------
std::string Tokenizer::token_bytes(int32_t id) const {
  if (id < 0 || (size_t)id >= tokens_.size()) return std::string();
  const std::string& s = tokens_[id];
  if (special_.count(id)) return s;
  if (spm_) {
    if (s.size() == 6 && s.compare(0, 3, "<0x") == 0 && s[5] == '>')
      return std::string(1, (char)std::stoi(s.substr(3, 2), nullptr, 16));
    std::string o;
    for (size_t i = 0; i < s.size();) {
      if (s.compare(i, 3, "\xE2\x96\x81") == 0) { o += ' '; i += 3; }
      else o += s[i++];
    }
    return o;
  }
  std::string o;
  for (uint32_t cp : utf8_decode(s)) {
    auto it = unicode_to_byte_.find(cp);
    if (it != unicode_to_byte_.end()) o += (char)it->second;
    else o += utf8_encode(cp);
  }
  return o;
}

std::string Tokenizer::decode(const std::vector<int32_t>& ids, bool skip_special) const {
  std::string o;
  for (int32_t id : ids) {
    if (skip_special && is_special(id)) continue;
    o += token_bytes(id);
  }
  if (spm_ && !o.empty() && o[0] == ' ') o.erase(0, 1);  // the encoder's leading-space prefix
  return o;
}

std::string StreamDecoder::push(int32_t id) {
  if (skip_ && t_->is_special(id)) return std::string();
  std::string b = t_->token_bytes(id);
  if (first_ && t_->is_spm() && !b.empty() && b[0] == ' ') b.erase(0, 1);
  first_ = false;
  pending_ += b;
  const size_t n = utf8_complete_prefix(pending_);
  std::string out = pending_.substr(0, n);
  pending_.erase(0, n);
  return out;
}

std::string StreamDecoder::flush() {
  std::string o;
  o.swap(pending_);
  return o;
}

}  // namespace hk
