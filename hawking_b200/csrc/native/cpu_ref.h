// CPU reference: elementwise/norm/rope/attention/MoE/sampling ops and a full Llama-family
// forward (llama, mistral, mixtral, qwen2, qwen2moe/qwen3moe) that runs straight from GGUF
// blocks. It is the numerics oracle for the GPU kernels and the timed CPU baseline.
//
// Parity: crates/hawking-core/src/kernels/mod.rs:8-342 (rmsnorm, silu_mul, softmax, rope
// variants, embed, gemv, argmax, topk_softmax), crates/hawking-core/src/attn.rs:23 (GQA decode),
// crates/hawking-core/src/moe.rs:24-117 (top-k gate, expert FFN, shared experts),
// crates/hawking-core/src/sample.rs:39-98 (sampler order), crates/hawking-core/src/model/llama.rs:1-20
// (GQA + SwiGLU + RMSNorm + RoPE, llama3 frequency scaling).
#pragma once
#include <cstdint>
#include <memory>
#include <random>
#include <string>
#include <vector>

#include "gguf.h"

namespace hk {

// ---- ops -------------------------------------------------------------------------------------
void ref_rmsnorm(const float* x, const float* w, float* y, int n, float eps);
void ref_silu_mul(const float* g, const float* u, float* y, int n);
void ref_softmax(float* x, int n);
// RoPE in place on one head vector. style 0 = adjacent pairs (GGUF llama "norm"), 1 = neox
// halves. freq_factors (may be null) divides each pair's frequency (llama3 rope_freqs).
void ref_rope(float* x, int head_dim, int rot_dim, int pos, float theta, int style,
              const float* freq_factors);
// GQA decode for one query token: q [n_heads, hd]; k,v [n_ctx, n_kv, hd]; out [n_heads, hd].
void ref_attention_decode(const float* q, const float* k, const float* v, float* out, int n_heads,
                          int n_kv, int hd, int n_ctx, float scale);
// Softmax top-k gate with lowest-index tie break; returns (ids, weights).
void ref_topk_gate(const float* logits, int n_experts, int top_k, bool renorm, int* ids, float* w);
int ref_argmax(const float* x, int n);
// Round-trip through q8 activation blocks (in place), n a multiple of 32.
void ref_q8_roundtrip(float* x, int n);

// PCG64-MCG-style 128-bit multiplicative generator used by the sampler.
class Pcg64 {
 public:
  explicit Pcg64(uint64_t seed);
  uint64_t next_u64();
  float next_f32();  // uniform in [0, 1)
 private:
  unsigned __int128 state_;
};

struct SamplingParams {
  float temperature = 0.f;
  int top_k = 0;
  float top_p = 1.f;
  float repetition_penalty = 1.f;
  uint64_t seed = 42;
};

class Sampler {
 public:
  explicit Sampler(uint64_t seed, int rep_window = 64) : rng_(seed), window_(rep_window) {}
  void record(int token);
  int sample(std::vector<float>& logits, const SamplingParams& p);
  const std::vector<int>& recent() const { return recent_; }
 private:
  Pcg64 rng_;
  int window_;
  std::vector<int> recent_;
};

// ---- model -----------------------------------------------------------------------------------
struct RefModelConfig {
  std::string arch;  // llama / qwen2 / qwen2moe / qwen3moe / mixtral (llama with experts)
  int vocab = 0, hidden = 0, layers = 0, n_heads = 0, n_kv_heads = 0, head_dim = 0, ffn = 0;
  int rot_dim = 0, rope_style = 0;
  float eps = 1e-5f, theta = 10000.f;
  int n_experts = 0, top_k = 0, expert_ffn = 0, shared_ffn = 0;
  bool norm_topk = true;
  int max_ctx = 4096;
};

RefModelConfig ref_config_from_gguf(const GgufFile& f);

class CpuLlama {
 public:
  // act_q8: round every matmul input to q8 activation blocks (int8 per 32, scale amax/127) and
  // bf16_kv: store K/V rounded to bf16 — together they reproduce the device path's W4A8 numerics.
  CpuLlama(std::shared_ptr<GgufFile> file, int max_ctx, int threads, bool act_q8 = false, bool bf16_kv = false);
  const RefModelConfig& config() const { return cfg_; }
  // Forward one token at position pos (positions must be fed in order). Returns logits.
  std::vector<float> forward(int token, int pos);
  void reset() { n_past_ = 0; }
  int n_past() const { return n_past_; }
  // Greedy: feed prompt, then decode n tokens; returns the generated ids.
  std::vector<int> generate_greedy(const std::vector<int>& prompt, int n_new);
  std::vector<int> generate(const std::vector<int>& prompt, int n_new, const SamplingParams& p);
  // Final hidden state (after output norm) of the last forward, for embeddings.
  const std::vector<float>& last_hidden() const { return last_hidden_; }

 private:
  struct Lin { const uint8_t* data = nullptr; uint32_t type = 0; int rows = 0, cols = 0; };
  Lin lin(const std::string& name, bool required = true) const;
  void matvec(const Lin& w, const float* x, float* y, size_t row_offset = 0, int rows = -1) const;
  std::vector<float> vec_f32(const std::string& name, bool required = true) const;
  void ffn_dense(int l, const float* xn, float* out);
  void ffn_moe(int l, const float* xn, float* out);

  std::shared_ptr<GgufFile> file_;
  RefModelConfig cfg_;
  int threads_;
  bool act_q8_ = false, bf16_kv_ = false;
  int n_past_ = 0;
  std::vector<std::vector<float>> kc_, vc_;  // per layer [max_ctx, n_kv, hd]
  std::vector<float> freq_factors_;
  std::vector<float> last_hidden_;
};

}  // namespace hk
