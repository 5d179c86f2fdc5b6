// CPU reference ops and Llama-family forward; see cpu_ref.h.
#include "cpu_ref.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <stdexcept>

#include "ggml_quant.h"
#include "thread_pool.h"

namespace hk {

void ref_rmsnorm(const float* x, const float* w, float* y, int n, float eps) {
  double ss = 0;
  for (int i = 0; i < n; ++i) ss += (double)x[i] * x[i];
  float r = 1.f / std::sqrt((float)(ss / n) + eps);
  for (int i = 0; i < n; ++i) y[i] = x[i] * r * (w ? w[i] : 1.f);
}

void ref_silu_mul(const float* g, const float* u, float* y, int n) {
  for (int i = 0; i < n; ++i) y[i] = g[i] / (1.f + std::exp(-g[i])) * u[i];
}

void ref_softmax(float* x, int n) {
  float m = -INFINITY;
  for (int i = 0; i < n; ++i) m = std::max(m, x[i]);
  double s = 0;
  for (int i = 0; i < n; ++i) { x[i] = std::exp(x[i] - m); s += x[i]; }
  float inv = s > 0 ? (float)(1.0 / s) : 0.f;
  for (int i = 0; i < n; ++i) x[i] *= inv;
}

void ref_rope(float* x, int head_dim, int rot_dim, int pos, float theta, int style, const float* ff) {
  int half = rot_dim / 2;
  for (int i = 0; i < half; ++i) {
    double freq = std::pow((double)theta, -2.0 * i / rot_dim);
    if (ff) freq /= ff[i];
    double ang = pos * freq;
    float c = (float)std::cos(ang), s = (float)std::sin(ang);
    int a = style == 0 ? 2 * i : i;
    int b = style == 0 ? 2 * i + 1 : i + half;
    float x0 = x[a], x1 = x[b];
    x[a] = x0 * c - x1 * s;
    x[b] = x0 * s + x1 * c;
  }
  (void)head_dim;
}

void ref_attention_decode(const float* q, const float* k, const float* v, float* out, int n_heads,
                          int n_kv, int hd, int n_ctx, float scale) {
  int group = n_heads / n_kv;
  std::vector<float> sc(n_ctx);
  for (int h = 0; h < n_heads; ++h) {
    int kh = h / group;
    const float* qh = q + (size_t)h * hd;
    for (int t = 0; t < n_ctx; ++t) {
      const float* kt = k + ((size_t)t * n_kv + kh) * hd;
      double s = 0;
      for (int d = 0; d < hd; ++d) s += (double)qh[d] * kt[d];
      sc[t] = (float)s * scale;
    }
    ref_softmax(sc.data(), n_ctx);
    float* o = out + (size_t)h * hd;
    for (int d = 0; d < hd; ++d) o[d] = 0;
    for (int t = 0; t < n_ctx; ++t) {
      const float* vt = v + ((size_t)t * n_kv + kh) * hd;
      for (int d = 0; d < hd; ++d) o[d] += sc[t] * vt[d];
    }
  }
}

void ref_topk_gate(const float* logits, int n, int top_k, bool renorm, int* ids, float* w) {
  std::vector<float> p(logits, logits + n);
  ref_softmax(p.data(), n);
  std::vector<int> idx(n);
  std::iota(idx.begin(), idx.end(), 0);
  std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return p[a] > p[b]; });
  float s = 0;
  for (int k = 0; k < top_k; ++k) { ids[k] = idx[k]; w[k] = p[idx[k]]; s += w[k]; }
  if (renorm && s > 0)
    for (int k = 0; k < top_k; ++k) w[k] /= s;
}

void ref_q8_roundtrip(float* x, int n) {
  for (int b = 0; b + 32 <= n; b += 32) {
    float amax = 0;
    for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(x[b + i]));
    float d = amax / 127.f;
    for (int i = 0; i < 32; ++i) x[b + i] = amax > 0 ? (float)(int)std::nearbyint(x[b + i] / d) * d : 0.f;
  }
}

int ref_argmax(const float* x, int n) {
  int best = 0;
  float bv = -INFINITY;
  for (int i = 0; i < n; ++i)
    if (x[i] > bv) { bv = x[i]; best = i; }
  return best;
}

// ---- sampler ---------------------------------------------------------------------------------
namespace {
const unsigned __int128 kPcgMult =
    ((unsigned __int128)0x2360ED051FC65DA4ull << 64) | (unsigned __int128)0x4385DF649FCCF645ull;
}

Pcg64::Pcg64(uint64_t seed) : state_(((unsigned __int128)seed) | 3) {}

uint64_t Pcg64::next_u64() {
  state_ *= kPcgMult;
  uint64_t hi = (uint64_t)(state_ >> 64), lo = (uint64_t)state_;
  unsigned rot = (unsigned)(state_ >> 122);
  uint64_t x = hi ^ lo;
  return (x >> rot) | (x << ((64 - rot) & 63));
}

float Pcg64::next_f32() {
  uint32_t v = (uint32_t)next_u64();
  return (float)(v >> 8) * (1.0f / 16777216.0f);
}

void Sampler::record(int token) {
  recent_.push_back(token);
  if ((int)recent_.size() > window_) recent_.erase(recent_.begin(), recent_.end() - window_);
}

int Sampler::sample(std::vector<float>& logits, const SamplingParams& p) {
  int n = (int)logits.size();
  if (p.repetition_penalty != 1.f)
    for (int t : recent_)
      if (t >= 0 && t < n) {
        float v = logits[t];
        logits[t] = v >= 0 ? v / p.repetition_penalty : v * p.repetition_penalty;
      }
  if (p.temperature <= 0.f) return ref_argmax(logits.data(), n);
  for (auto& v : logits) v /= p.temperature;
  std::vector<float> probs(logits);
  ref_softmax(probs.data(), n);
  std::vector<int> idx(n);
  std::iota(idx.begin(), idx.end(), 0);
  std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return probs[a] > probs[b]; });
  size_t keep = idx.size();
  if (p.top_k > 0 && p.top_k < n) keep = p.top_k;
  if (p.top_p > 0.f && p.top_p < 1.f) {
    float cum = 0;
    for (size_t k = 0; k < keep; ++k) {
      cum += probs[idx[k]];
      if (cum >= p.top_p) { keep = k + 1; break; }
    }
  }
  float total = 0;
  for (size_t k = 0; k < keep; ++k) total += probs[idx[k]];
  float r = rng_.next_f32() * total, acc = 0;
  for (size_t k = 0; k < keep; ++k) {
    acc += probs[idx[k]];
    if (r <= acc) return idx[k];
  }
  return keep ? idx[keep - 1] : 0;
}

// ---- model -----------------------------------------------------------------------------------
namespace {
int64_t meta_int(const GgufFile& f, const std::string& key, int64_t dflt, bool required = false) {
  auto it = f.metadata().find(key);
  if (it == f.metadata().end()) {
    if (required) throw std::runtime_error("gguf: missing metadata " + key);
    return dflt;
  }
  if (it->second.kind == GgufKind::ARRAY)  // per-layer arrays: take the first entry
    return it->second.arr && !it->second.arr->empty() ? (*it->second.arr)[0].i : dflt;
  return it->second.kind == GgufKind::F32 || it->second.kind == GgufKind::F64 ? (int64_t)it->second.f
                                                                              : it->second.i;
}
double meta_f(const GgufFile& f, const std::string& key, double dflt) {
  auto it = f.metadata().find(key);
  if (it == f.metadata().end()) return dflt;
  return it->second.kind == GgufKind::F32 || it->second.kind == GgufKind::F64 ? it->second.f
                                                                              : (double)it->second.i;
}
std::string meta_s(const GgufFile& f, const std::string& key) {
  auto it = f.metadata().find(key);
  if (it == f.metadata().end()) throw std::runtime_error("gguf: missing metadata " + key);
  return it->second.s;
}
ThreadPool& pool(int n) {
  static thread_local std::unique_ptr<ThreadPool> p;
  if (!p || p->size() != n) p.reset(new ThreadPool(n));
  return *p;
}
}  // namespace

RefModelConfig ref_config_from_gguf(const GgufFile& f) {
  RefModelConfig c;
  c.arch = meta_s(f, "general.architecture");
  const std::string a = c.arch;
  if (a != "llama" && a != "mistral" && a != "qwen2" && a != "qwen2moe" && a != "qwen3" &&
      a != "qwen3moe")
    throw std::runtime_error("cpu reference: unsupported architecture " + a);
  c.hidden = (int)meta_int(f, a + ".embedding_length", 0, true);
  c.layers = (int)meta_int(f, a + ".block_count", 0, true);
  c.n_heads = (int)meta_int(f, a + ".attention.head_count", 0, true);
  c.n_kv_heads = (int)meta_int(f, a + ".attention.head_count_kv", c.n_heads);
  c.head_dim = (int)meta_int(f, a + ".attention.key_length", c.hidden / c.n_heads);
  c.ffn = (int)meta_int(f, a + ".feed_forward_length", 0);
  c.rot_dim = (int)meta_int(f, a + ".rope.dimension_count", c.head_dim);
  c.eps = (float)meta_f(f, a + ".attention.layer_norm_rms_epsilon", 1e-5);
  c.theta = (float)meta_f(f, a + ".rope.freq_base", 10000.0);
  c.n_experts = (int)meta_int(f, a + ".expert_count", 0);
  c.top_k = (int)meta_int(f, a + ".expert_used_count", 0);
  c.expert_ffn = (int)meta_int(f, a + ".expert_feed_forward_length", c.ffn);
  c.shared_ffn = (int)meta_int(f, a + ".expert_shared_feed_forward_length", 0);
  c.rope_style = (a == "llama" || a == "mistral") ? 0 : 1;
  c.norm_topk = a != "qwen2moe";
  const auto* emb = f.find("token_embd.weight");
  if (!emb) throw std::runtime_error("gguf: missing token_embd.weight");
  c.vocab = (int)meta_int(f, a + ".vocab_size", (int64_t)emb->dims[1]);
  return c;
}

CpuLlama::CpuLlama(std::shared_ptr<GgufFile> file, int max_ctx, int threads, bool act_q8, bool bf16_kv)
    : file_(std::move(file)), threads_(std::max(1, threads)), act_q8_(act_q8), bf16_kv_(bf16_kv) {
  cfg_ = ref_config_from_gguf(*file_);
  cfg_.max_ctx = max_ctx;
  size_t per = (size_t)max_ctx * cfg_.n_kv_heads * cfg_.head_dim;
  kc_.assign(cfg_.layers, std::vector<float>(per));
  vc_.assign(cfg_.layers, std::vector<float>(per));
  if (file_->find("rope_freqs.weight")) freq_factors_ = vec_f32("rope_freqs.weight");
}

CpuLlama::Lin CpuLlama::lin(const std::string& name, bool required) const {
  const auto* t = file_->find(name);
  if (!t) {
    if (required) throw std::runtime_error("cpu reference: missing tensor " + name);
    return Lin{};
  }
  Lin l;
  l.data = file_->tensor_data(*t);
  l.type = t->type;
  l.cols = (int)t->dims[0];
  l.rows = (int)(t->n_elements() / t->dims[0]);
  return l;
}

std::vector<float> CpuLlama::vec_f32(const std::string& name, bool required) const {
  const auto* t = file_->find(name);
  if (!t) {
    if (required) throw std::runtime_error("cpu reference: missing tensor " + name);
    return {};
  }
  std::vector<float> v(t->n_elements());
  dequantize(t->type, file_->tensor_data(*t), v.data(), v.size());
  return v;
}

void CpuLlama::matvec(const Lin& w, const float* x, float* y, size_t row_offset, int rows) const {
  if (rows < 0) rows = w.rows;
  size_t rb = type_nbytes(w.type, w.cols);
  const uint8_t* base = w.data + row_offset * rb;
  int cols = w.cols;
  uint32_t type = w.type;
  pool(threads_).parallel_for((size_t)rows, [&](size_t a, size_t e) {
    std::vector<float> tmp(cols);
    for (size_t r = a; r < e; ++r) {
      dequantize(type, base + r * rb, tmp.data(), cols);
      double s = 0;
      for (int c = 0; c < cols; ++c) s += (double)tmp[c] * x[c];
      y[r] = (float)s;
    }
  });
}

void CpuLlama::ffn_dense(int l, const float* xn, float* out) {
  std::string p = "blk." + std::to_string(l) + ".";
  Lin g = lin(p + "ffn_gate.weight"), u = lin(p + "ffn_up.weight"), d = lin(p + "ffn_down.weight");
  std::vector<float> gv(g.rows), uv(u.rows), h(g.rows);
  matvec(g, xn, gv.data());
  matvec(u, xn, uv.data());
  ref_silu_mul(gv.data(), uv.data(), h.data(), g.rows);
  if (act_q8_) ref_q8_roundtrip(h.data(), g.rows);
  matvec(d, h.data(), out);
}

void CpuLlama::ffn_moe(int l, const float* xn, float* out) {
  std::string p = "blk." + std::to_string(l) + ".";
  const int H = cfg_.hidden, E = cfg_.n_experts, F = cfg_.expert_ffn;
  Lin r = lin(p + "ffn_gate_inp.weight");
  std::vector<float> logits(E);
  matvec(r, xn, logits.data());
  std::vector<int> ids(cfg_.top_k);
  std::vector<float> w(cfg_.top_k);
  ref_topk_gate(logits.data(), E, cfg_.top_k, cfg_.norm_topk, ids.data(), w.data());
  Lin ge = lin(p + "ffn_gate_exps.weight"), ue = lin(p + "ffn_up_exps.weight"),
      de = lin(p + "ffn_down_exps.weight");
  std::fill(out, out + H, 0.f);
  std::vector<float> gv(F), uv(F), h(F), o(H);
  for (int k = 0; k < cfg_.top_k; ++k) {
    int e = ids[k];
    matvec(ge, xn, gv.data(), (size_t)e * F, F);
    matvec(ue, xn, uv.data(), (size_t)e * F, F);
    ref_silu_mul(gv.data(), uv.data(), h.data(), F);
    if (act_q8_) ref_q8_roundtrip(h.data(), F);
    Lin dd = de;
    dd.cols = F;
    matvec(dd, h.data(), o.data(), (size_t)e * H, H);
    for (int i = 0; i < H; ++i) out[i] += w[k] * o[i];
  }
  Lin gs = lin(p + "ffn_gate_shexp.weight", false);
  if (gs.data) {
    Lin us = lin(p + "ffn_up_shexp.weight"), ds = lin(p + "ffn_down_shexp.weight");
    std::vector<float> g2(gs.rows), u2(gs.rows), h2(gs.rows), o2(H);
    matvec(gs, xn, g2.data());
    matvec(us, xn, u2.data());
    ref_silu_mul(g2.data(), u2.data(), h2.data(), gs.rows);
    if (act_q8_) ref_q8_roundtrip(h2.data(), gs.rows);
    matvec(ds, h2.data(), o2.data());
    float gate = 1.f;
    Lin sg = lin(p + "ffn_gate_inp_shexp.weight", false);
    if (sg.data) {
      float z;
      matvec(sg, xn, &z);
      gate = 1.f / (1.f + std::exp(-z));
    }
    for (int i = 0; i < H; ++i) out[i] += gate * o2[i];
  }
}

std::vector<float> CpuLlama::forward(int token, int pos) {
  const auto& c = cfg_;
  if (pos >= c.max_ctx) throw std::runtime_error("cpu reference: context overflow");
  if (token < 0 || token >= c.vocab) throw std::runtime_error("cpu reference: token out of range");
  const int H = c.hidden, hd = c.head_dim, nh = c.n_heads, nkv = c.n_kv_heads;
  std::vector<float> x(H), xn(H), q(nh * hd), k(nkv * hd), v(nkv * hd), att(nh * hd), o(H);
  {
    const auto* t = file_->find("token_embd.weight");
    size_t rb = type_nbytes(t->type, H);
    dequantize(t->type, file_->tensor_data(*t) + (size_t)token * rb, x.data(), H);
  }
  const float* ff = freq_factors_.empty() ? nullptr : freq_factors_.data();
  for (int l = 0; l < c.layers; ++l) {
    std::string p = "blk." + std::to_string(l) + ".";
    auto an = vec_f32(p + "attn_norm.weight");
    ref_rmsnorm(x.data(), an.data(), xn.data(), H, c.eps);
    if (act_q8_) ref_q8_roundtrip(xn.data(), H);
    matvec(lin(p + "attn_q.weight"), xn.data(), q.data());
    matvec(lin(p + "attn_k.weight"), xn.data(), k.data());
    matvec(lin(p + "attn_v.weight"), xn.data(), v.data());
    auto bq = vec_f32(p + "attn_q.bias", false), bk = vec_f32(p + "attn_k.bias", false),
         bv = vec_f32(p + "attn_v.bias", false);
    for (size_t i = 0; i < bq.size(); ++i) q[i] += bq[i];
    for (size_t i = 0; i < bk.size(); ++i) k[i] += bk[i];
    for (size_t i = 0; i < bv.size(); ++i) v[i] += bv[i];
    auto qn = vec_f32(p + "attn_q_norm.weight", false), kn = vec_f32(p + "attn_k_norm.weight", false);
    for (int h = 0; h < nh; ++h) {
      if (!qn.empty()) ref_rmsnorm(&q[h * hd], qn.data(), &q[h * hd], hd, c.eps);
      ref_rope(&q[h * hd], hd, c.rot_dim, pos, c.theta, c.rope_style, ff);
    }
    for (int h = 0; h < nkv; ++h) {
      if (!kn.empty()) ref_rmsnorm(&k[h * hd], kn.data(), &k[h * hd], hd, c.eps);
      ref_rope(&k[h * hd], hd, c.rot_dim, pos, c.theta, c.rope_style, ff);
    }
    if (bf16_kv_)
      for (int i = 0; i < nkv * hd; ++i) { k[i] = bf16_to_f32(f32_to_bf16(k[i])); v[i] = bf16_to_f32(f32_to_bf16(v[i])); }
    std::memcpy(&kc_[l][(size_t)pos * nkv * hd], k.data(), sizeof(float) * nkv * hd);
    std::memcpy(&vc_[l][(size_t)pos * nkv * hd], v.data(), sizeof(float) * nkv * hd);
    ref_attention_decode(q.data(), kc_[l].data(), vc_[l].data(), att.data(), nh, nkv, hd, pos + 1,
                         1.f / std::sqrt((float)hd));
    if (act_q8_) ref_q8_roundtrip(att.data(), nh * hd);
    matvec(lin(p + "attn_output.weight"), att.data(), o.data());
    for (int i = 0; i < H; ++i) x[i] += o[i];
    auto fn = vec_f32(p + "ffn_norm.weight");
    ref_rmsnorm(x.data(), fn.data(), xn.data(), H, c.eps);
    if (act_q8_) ref_q8_roundtrip(xn.data(), H);
    if (c.n_experts > 0) ffn_moe(l, xn.data(), o.data());
    else ffn_dense(l, xn.data(), o.data());
    for (int i = 0; i < H; ++i) x[i] += o[i];
  }
  auto on = vec_f32("output_norm.weight");
  ref_rmsnorm(x.data(), on.data(), xn.data(), H, c.eps);
  last_hidden_ = xn;
  if (act_q8_) ref_q8_roundtrip(xn.data(), H);
  Lin out = file_->find("output.weight") ? lin("output.weight") : lin("token_embd.weight");
  std::vector<float> logits(out.rows);
  matvec(out, xn.data(), logits.data());
  n_past_ = pos + 1;
  return logits;
}

std::vector<int> CpuLlama::generate_greedy(const std::vector<int>& prompt, int n_new) {
  SamplingParams p;
  p.temperature = 0;
  return generate(prompt, n_new, p);
}

std::vector<int> CpuLlama::generate(const std::vector<int>& prompt, int n_new, const SamplingParams& sp) {
  if (prompt.empty()) throw std::runtime_error("cpu reference: empty prompt");
  reset();
  Sampler s(sp.seed);
  std::vector<float> logits;
  for (size_t i = 0; i < prompt.size(); ++i) { logits = forward(prompt[i], (int)i); s.record(prompt[i]); }
  std::vector<int> out;
  int pos = (int)prompt.size();
  for (int i = 0; i < n_new; ++i) {
    int t = s.sample(logits, sp);
    out.push_back(t);
    s.record(t);
    if (i + 1 < n_new) logits = forward(t, pos++);
  }
  return out;
}

}  // namespace hk
