// Mixture-of-experts decode kernels (K3 router + the single-GPU part of K4):
//
//   router_logits   logits[t, e] = W_r[e, :] . x_t with fp32 router weights and q8 activations
//   moe_topk        softmax (Mixtral/Qwen) or sigmoid + learned bias with group-limited selection
//                   (DeepSeek-V3 noaux_tc), top-k with lowest-index tie break, optional renormalise
//                   and routed scale -> ids [T, k], weights [T, k]
//   moe_align       counting sort of the T*k (token, slot) pairs by expert: per-expert counts and
//                   offsets, the sorted pair list, and the q8 activations gathered in sorted order
//   moe_gemv        grouped expert GEMV over the stacked [E * N, K] weight: one grid row per expert,
//                   each CTA streams its rows once per chunk of <= 8 routed pairs. Epilogues:
//                   SwiGLU -> q8 (gate/up, sorted order) and weighted atomic add into the fp32
//                   residual of each pair's token (down).
//
// Parity: crates/hawking-core/shaders/moe.metal moe_topk_gate (softmax + top-k, lexicographic
// tie break, :148-200), moe_batched_gemm_*_indexed(_gu), moe_route_accumulate(_add);
// crates/hawking-core/src/moe.rs:24-117 (topk_gate, expert_ffn, moe_forward_token, shared experts);
// qwen80_postnorm_router_top10 / qwen80_all_ten_routed_expert_wave (512-way expert table).
#include "api.h"
#include "qformats.cuh"
#include "tp.cuh"

namespace hk {

// ---- router logits ----------------------------------------------------------------------------
// One warp per (token, expert); lanes stride K.
__global__ void __launch_bounds__(256) router_logits_kernel(const float* __restrict__ w, int E, int K,
                                                             const int8_t* xq, const float* xd, int64_t xs_q,
                                                             int64_t xs_d, float* logits, int T) {
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T * E) return;
  const int t = warp / E, e = warp % E;
  const float* wr = w + (int64_t)e * K;
  const int8_t* q = xq + (int64_t)t * xs_q;
  const float* d = xd + (int64_t)t * xs_d;
  float acc = 0.f;
  for (int k = lane * 4; k < K; k += 128) {
    const float4 wv = *reinterpret_cast<const float4*>(wr + k);
    const char4 qv = *reinterpret_cast<const char4*>(q + k);
    const float dk = d[k >> 5];
    acc += (wv.x * qv.x + wv.y * qv.y + wv.z * qv.z + wv.w * qv.w) * dk;
  }
  acc = warp_sum(acc);
  if (lane == 0) logits[(int64_t)t * E + e] = acc;
  pdl_launch();
}

void router_logits_launch(const float* w, int E, int K, const int8_t* xq, const float* xd, int64_t xs_q,
                          int64_t xs_d, float* logits, int T, cudaStream_t s, bool pdl) {
  if (K % 128) throw std::runtime_error("router: K must be a multiple of 128");
  const int warps = T * E;
  launch(router_logits_kernel, dim3((warps * 32 + 255) / 256), dim3(256), 0, s, pdl, w, E, K, xq, xd, xs_q, xs_d,
         logits, T);
}

// ---- top-k ------------------------------------------------------------------------------------
__device__ __forceinline__ void lex_merge(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}
__device__ __forceinline__ void block_argmax(float& v, int& i, float* sv, int* si) {
  for (int o = 16; o > 0; o >>= 1) {
    float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    int i2 = __shfl_xor_sync(0xffffffffu, i, o);
    lex_merge(v, i, v2, i2);
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) { sv[w] = v; si[w] = i; }
  __syncthreads();
  v = lane < nw ? sv[lane] : -INFINITY;
  i = lane < nw ? si[lane] : 0x7fffffff;
  for (int o = 16; o > 0; o >>= 1) {
    float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    int i2 = __shfl_xor_sync(0xffffffffu, i, o);
    lex_merge(v, i, v2, i2);
  }
}

// Top-k of token t by one CTA of 256 threads; E <= 1024. Logits are read with .cg loads (the
// fused router writes them from other CTAs of the same launch).
struct TopkSmem {
  float score[1024], sel[1024];
  float sv[32];
  int si[32];
  float gscore[64];
  int keep_group[64];
  float red[32];
  int ids[32];
  float ws[32];
};
__device__ void topk_token(const MoeTopkArgs& a, int t, TopkSmem& sm) {
  float* score = sm.score;
  float* sel = sm.sel;
  float* sv = sm.sv;
  int* si = sm.si;
  float* gscore = sm.gscore;
  int* keep_group = sm.keep_group;
  float* red = sm.red;
  const int E = a.E, tid = threadIdx.x;
  const float* l = a.logits + (int64_t)t * E;
  // scores
  if (a.scoring == 0) {  // softmax
    float m = -INFINITY;
    for (int e = tid; e < E; e += blockDim.x) m = fmaxf(m, __ldcg(l + e));
    m = block_max(m, red);
    float z = 0.f;
    for (int e = tid; e < E; e += blockDim.x) z += __expf(__ldcg(l + e) - m);
    z = block_sum(z, red);
    for (int e = tid; e < E; e += blockDim.x) {
      score[e] = __expf(__ldcg(l + e) - m) / z;
      sel[e] = score[e];
    }
  } else {  // sigmoid; selection adds the learned bias
    for (int e = tid; e < E; e += blockDim.x) {
      score[e] = 1.f / (1.f + __expf(-__ldcg(l + e)));
      sel[e] = score[e] + (a.bias ? a.bias[e] : 0.f);
    }
  }
  __syncthreads();
  // group-limited routing: keep the top `topk_groups` groups by (sum of top-2 selection scores)
  if (a.n_groups > 1) {
    const int gsz = E / a.n_groups;
    if (tid < a.n_groups) {
      float b1 = -INFINITY, b2 = -INFINITY;
      for (int e = tid * gsz; e < (tid + 1) * gsz; ++e) {
        const float v = sel[e];
        if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) b2 = v;
      }
      gscore[tid] = b1 + b2;
      keep_group[tid] = 0;
    }
    __syncthreads();
    if (tid == 0) {
      for (int k = 0; k < a.topk_groups; ++k) {
        int best = -1;
        float bv = -INFINITY;
        for (int g = 0; g < a.n_groups; ++g)
          if (!keep_group[g] && gscore[g] > bv) { bv = gscore[g]; best = g; }
        if (best >= 0) keep_group[best] = 1;
      }
    }
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x)
      if (!keep_group[e / gsz]) sel[e] = -INFINITY;
    __syncthreads();
  }
  float wsum = 0.f;
  int* ids = sm.ids;
  float* ws = sm.ws;
  for (int k = 0; k < a.k; ++k) {
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int e = tid; e < E; e += blockDim.x) lex_merge(v, i, sel[e], e);
    block_argmax(v, i, sv, si);
    if (tid == 0) {
      ids[k] = i;
      ws[k] = score[i];
      wsum += score[i];
      sel[i] = -INFINITY;
    }
    __syncthreads();
  }
  if (tid < a.k) {
    float w = ws[tid];
    if (a.renorm) {
      float s = 0.f;
      for (int k = 0; k < a.k; ++k) s += ws[k];
      w = s > 0.f ? w / s : w;
    }
    a.ids[(int64_t)t * a.k + tid] = ids[tid];
    a.weights[(int64_t)t * a.k + tid] = w * a.scale;
  }
  (void)wsum;
  __syncthreads();
}

__global__ void __launch_bounds__(256) moe_topk_kernel(MoeTopkArgs a) {
  __shared__ TopkSmem sm;
  pdl_wait();
  topk_token(a, blockIdx.x, sm);
  pdl_launch();
}

void moe_topk_launch(const MoeTopkArgs& a, cudaStream_t s, bool pdl) {
  if (a.E > 1024 || a.k > 32) throw std::runtime_error("moe_topk: E <= 1024 and k <= 32");
  if (a.n_groups > 64 || (a.n_groups > 1 && a.E % a.n_groups)) throw std::runtime_error("moe_topk: bad groups");
  launch(moe_topk_kernel, dim3(a.T), dim3(256), 0, s, pdl, a);
}

// ---- fused routing (decode): router GEMV + top-k + counting sort + active list, one launch --------
// Every CTA computes router logits for its experts (4 warps per expert, each a quarter of K,
// joined in shared memory). The CTA whose arrival completes the grid (device-scope counter, reset
// by it afterwards) then runs top-k for every token, the counting sort of the (token, slot) pairs
// by expert (plus one shared-expert pair per token as expert E), and the compact list of experts
// with pairs. No activation gather: the expert kernels read each pair's token row directly.
constexpr int kRouteExpertsPerCta = 2;
__global__ void __launch_bounds__(256) moe_route_kernel(MoeRouteArgs a) {
  __shared__ TopkSmem sm;
  __shared__ float part[kRouteExpertsPerCta][8][4];
  __shared__ int cnt[1025], off[1026];
  __shared__ bool last;
  pdl_wait();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = a.T, E = a.E, K = a.K;
  {  // logits of experts e0 .. e0 + 1 for every token: warp = (expert slot, quarter)
    const int es = warp >> 2, qt = warp & 3;
    const int e = blockIdx.x * kRouteExpertsPerCta + es;
    const int kq = K / 4;
    if (e < E) {
      const float* wr = a.router + (int64_t)e * K + qt * kq;
      for (int t = 0; t < T; ++t) {
        const int8_t* xq = a.xq + (int64_t)t * a.x_stride_q + qt * kq;
        const float* xd = a.xd + (int64_t)t * a.x_stride_s + (qt * kq >> 5);
        float acc = 0.f;
        for (int k = lane * 4; k < kq; k += 128) {
          const float4 wv = *reinterpret_cast<const float4*>(wr + k);
          const char4 qv = *reinterpret_cast<const char4*>(xq + k);
          acc += (wv.x * qv.x + wv.y * qv.y + wv.z * qv.z + wv.w * qv.w) * xd[k >> 5];
        }
        acc = warp_sum(acc);
        if (lane == 0) part[es][t][qt] = acc;
      }
    }
    __syncthreads();
    if (tid < kRouteExpertsPerCta * T) {
      const int es2 = tid / T, t = tid % T;
      const int e2 = blockIdx.x * kRouteExpertsPerCta + es2;
      if (e2 < E) a.logits[(int64_t)t * E + e2] = part[es2][t][0] + part[es2][t][1] + part[es2][t][2] + part[es2][t][3];
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(a.counter, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!last) {
    pdl_launch();
    return;
  }
  __threadfence();
  MoeTopkArgs ta{};
  ta.logits = a.logits;
  ta.bias = a.bias;
  ta.T = T;
  ta.E = E;
  ta.k = a.k;
  ta.scoring = a.scoring;
  ta.n_groups = a.n_groups;
  ta.topk_groups = a.topk_groups;
  ta.renorm = a.renorm;
  ta.scale = a.scale;
  ta.ids = a.ids;
  ta.weights = a.weights;
  for (int t = 0; t < T; ++t) topk_token(ta, t, sm);
  // counting sort of the pairs by expert (ids written above by this CTA)
  const int P = T * a.k, E1 = E + (a.shared ? 1 : 0);
  for (int e = tid; e < E1; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int p = tid; p < P; p += blockDim.x) atomicAdd(&cnt[a.ids[p]], 1);
  if (a.shared && tid == 0) cnt[E] = T;
  __syncthreads();
  if (tid == 0) {
    off[0] = 0;
    int n = 0;
    const int lo = a.e_lo, hi = a.e_hi > 0 ? a.e_hi : E;
    for (int e = 0; e < E1; ++e) {
      off[e + 1] = off[e] + cnt[e];
      // expert parallelism: only this rank's experts (and the shared one, when appended) run here
      if (cnt[e] > 0 && ((e >= lo && e < hi) || e == E)) a.active[n++] = e;
    }
    *a.n_active = n;
    *a.counter = 0;  // ready for the next launch
  }
  __syncthreads();
  for (int e = tid; e < E1; e += blockDim.x) {
    a.counts[e] = cnt[e];
    a.offsets[e] = off[e];
  }
  for (int e = tid; e < E; e += blockDim.x) {  // stable: the pairs of one expert keep token order
    int pos = off[e];
    for (int p = 0; p < P; ++p)
      if (a.ids[p] == e) a.sorted[pos++] = p;
  }
  if (a.shared)
    for (int t = tid; t < T; t += blockDim.x) a.sorted[P + t] = P + t;
  pdl_launch();
}

void moe_route_launch(const MoeRouteArgs& a, cudaStream_t s, bool pdl) {
  if (a.E + (a.shared ? 1 : 0) > 1024 || a.k > 32) throw std::runtime_error("moe_route: E <= 1023 and k <= 32");
  if (a.T > 8) throw std::runtime_error("moe_route: at most 8 tokens (decode)");
  if (a.K % 512) throw std::runtime_error("moe_route: hidden must be a multiple of 512");
  if (a.n_groups > 64 || (a.n_groups > 1 && a.E % a.n_groups)) throw std::runtime_error("moe_route: bad groups");
  const int ctas = (a.E + kRouteExpertsPerCta - 1) / kRouteExpertsPerCta;
  launch(moe_route_kernel, dim3(ctas), dim3(256), 0, s, pdl, a);
}

// ---- align (counting sort by expert) + gather ---------------------------------------------------
// One CTA. counts/offsets [E], sorted pairs [T*k] (pair = t*k + j), and the q8 activations of
// each pair's token gathered in sorted order (gq [T*k, K], gd/gs [T*k, K/32]).
__global__ void __launch_bounds__(1024) moe_align_kernel(MoeAlignArgs a) {
  __shared__ int cnt[1025], off[1026];
  pdl_wait();
  const int tid = threadIdx.x, P = a.T * a.k;
  const int E1 = a.E + (a.shared ? 1 : 0), PS = P + (a.shared ? a.T : 0);
  for (int e = tid; e < E1; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int p = tid; p < P; p += blockDim.x) atomicAdd(&cnt[a.ids[p]], 1);
  if (a.shared && tid == 0) cnt[a.E] = a.T;
  __syncthreads();
  if (tid == 0) {
    off[0] = 0;
    for (int e = 0; e < E1; ++e) off[e + 1] = off[e] + cnt[e];
  }
  __syncthreads();
  for (int e = tid; e < E1; e += blockDim.x) {
    a.counts[e] = cnt[e];
    a.offsets[e] = off[e];
  }
  // Stable placement: pairs of one expert keep token order (serial per expert bucket).
  for (int e = tid; e < a.E; e += blockDim.x) {
    int pos = off[e];
    for (int p = 0; p < P; ++p)
      if (a.ids[p] == e) a.sorted[pos++] = p;
  }
  for (int t = tid; t < PS - P; t += blockDim.x) a.sorted[P + t] = P + t;  // shared bucket is last
  __syncthreads();
  // Gather q8 activations in sorted order (unless the caller gathers its own rows).
  const int K = a.K;
  if (!a.gq) {
    pdl_launch();
    return;
  }
  for (int idx = tid; idx < PS * (K / 16); idx += blockDim.x) {
    const int sp = idx / (K / 16), c = idx % (K / 16);
    const int pr = a.sorted[sp], tok = pr < P ? pr / a.k : pr - P;
    reinterpret_cast<int4*>(a.gq + (int64_t)sp * K)[c] = reinterpret_cast<const int4*>(a.xq + (int64_t)tok * a.x_stride_q)[c];
  }
  for (int idx = tid; idx < PS * (K / 32); idx += blockDim.x) {
    const int sp = idx / (K / 32), c = idx % (K / 32);
    const int pr = a.sorted[sp], tok = pr < P ? pr / a.k : pr - P;
    a.gd[(int64_t)sp * (K / 32) + c] = a.xd[(int64_t)tok * a.x_stride_s + c];
    a.gs[(int64_t)sp * (K / 32) + c] = a.xs[(int64_t)tok * a.x_stride_s + c];
  }
  pdl_launch();
}

void moe_align_launch(const MoeAlignArgs& a, cudaStream_t s, bool pdl) {
  if (a.E + (a.shared ? 1 : 0) > 1024) throw std::runtime_error("moe_align: E <= 1024 (1023 with a shared expert)");
  if (a.K % 32) throw std::runtime_error("moe_align: K must be a multiple of 32");
  launch(moe_align_kernel, dim3(1), dim3(1024), 0, s, pdl, a);
}

// ---- grouped expert GEMV -----------------------------------------------------------------------
template <int FMT> struct MUnit;
template <> struct MUnit<WF_Q4_K> { using T = UnitQ4K; };
template <> struct MUnit<WF_Q4_0> { using T = UnitQ4_0; };
template <> struct MUnit<WF_Q8_0> { using T = UnitQ8_0; };
template <> struct MUnit<WF_Q6_K> { using T = UnitQ6K; };

template <int FMT>
__device__ __forceinline__ void m_load(const WPlanes& w, int64_t row, int u, typename MUnit<FMT>::T& r) {
  if constexpr (FMT == WF_Q4_K) load_unit_q4k(w, row, u, r);
  else if constexpr (FMT == WF_Q4_0) load_unit_q4_0(w, row, u, r);
  else if constexpr (FMT == WF_Q8_0) load_unit_q8_0(w, row, u, r);
  else load_unit_q6k(w, row, u, r);
}
template <int FMT>
__device__ __forceinline__ float m_dot(const typename MUnit<FMT>::T& r, int u, const int8_t* q, const float* d,
                                       const float* s) {
  if constexpr (FMT == WF_Q4_K) return dot_unit_q4k(r, u, q, d, s);
  else if constexpr (FMT == WF_Q4_0) return dot_unit_q4_0(r, u, q, d, s);
  else if constexpr (FMT == WF_Q8_0) return dot_unit_q8_0(r, u, q, d, s);
  else return dot_unit_q6k(r, u, q, d, s);
}

// NB columns (pairs) of one expert, one weight row per warp.
template <int FMT, int NB>
__device__ __forceinline__ void m_row_dot(const WPlanes& w, int64_t row, int n_units, const int8_t* q,
                                          const float* d, const float* s, int K, float (&acc)[NB]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = 0.f;
#pragma unroll 2
  for (int u = lane; u < n_units; u += 32) {
    typename MUnit<FMT>::T r;
    m_load<FMT>(w, row, u, r);
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] += m_dot<FMT>(r, u, q + (int64_t)b * K, d + (int64_t)b * (K / 32), s + (int64_t)b * (K / 32));
  }
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = warp_sum(acc[b]);
}

// Per chunk of NB pairs: gate/up (SwiGLU -> q8) or down (weighted atomic residual add).
template <int FMT, int NB, int EPI>
__device__ __forceinline__ void m_chunk(const MoeGemvArgs& a, int e, int p0, float (*hbuf)[32]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_units = a.K / 128;
  const int8_t* q = a.xq + (int64_t)p0 * a.K;
  const float* d = a.xd + (int64_t)p0 * (a.K / 32);
  const float* s = a.xs + (int64_t)p0 * (a.K / 32);
  if constexpr (EPI == 0) {
    // 32 rows per CTA: 8 warps x 4 rows; gate rows from w0, up rows from w1 (both of expert e)
#pragma unroll 1
    for (int r = 0; r < 4; ++r) {
      const int n = blockIdx.x * 32 + warp * 4 + r;
      float g[NB], u[NB];
      const int64_t row = (int64_t)(e - a.e_lo) * a.N + n;
      m_row_dot<FMT, NB>(a.w0, row, n_units, q, d, s, a.K, g);
      m_row_dot<FMT, NB>(a.w1, row, n_units, q, d, s, a.K, u);
      if (lane == 0)
#pragma unroll
        for (int b = 0; b < NB; ++b) hbuf[b][warp * 4 + r] = g[b] / (1.f + __expf(-g[b])) * u[b];
    }
    __syncthreads();
    for (int b = warp; b < NB; b += 8) {
      const int n = blockIdx.x * 32 + lane;
      const float v = hbuf[b][lane];
      const float amax = warp_max(fabsf(v));
      const float dd = amax / 127.f;
      const int qv = amax > 0.f ? __float2int_rn(v / dd) : 0;
      const float qs = warp_sum((float)qv);
      const int64_t sp = p0 + b;
      a.oq[sp * a.N + n] = (int8_t)qv;
      if (lane == 0) {
        a.od[sp * (a.N / 32) + (n >> 5)] = dd;
        a.os[sp * (a.N / 32) + (n >> 5)] = dd * qs;
      }
    }
    __syncthreads();
  } else {
    const int n = blockIdx.x * 8 + warp;
    float acc[NB];
    m_row_dot<FMT, NB>(a.w0, (int64_t)(e - a.e_lo) * a.N + n, n_units, q, d, s, a.K, acc);
    if (lane < NB) {
      float v = acc[0];
#pragma unroll
      for (int b = 1; b < NB; ++b)
        if (lane == b) v = acc[b];
      const int pair = a.sorted[p0 + lane];
      const int tok = pair / a.k;
      atomicAdd(a.y + (int64_t)tok * a.y_stride + n, a.route_w[pair] * v);
    }
  }
}

template <int FMT, int EPI>
__global__ void __launch_bounds__(256) moe_gemv_kernel(MoeGemvArgs a) {
  __shared__ float hbuf[8][32];
  pdl_wait();
  const int e = a.e_lo + (int)blockIdx.y;  // global expert id (weights stacked from e_lo)
  const int c = a.counts[e];
  if (c == 0) { pdl_launch(); return; }
  const int off = a.offsets[e];
  for (int done = 0; done < c; done += 8) {
    const int nb = min(8, c - done);
    switch (nb) {
      case 1: m_chunk<FMT, 1, EPI>(a, e, off + done, hbuf); break;
      case 2: m_chunk<FMT, 2, EPI>(a, e, off + done, hbuf); break;
      case 3: m_chunk<FMT, 3, EPI>(a, e, off + done, hbuf); break;
      case 4: m_chunk<FMT, 4, EPI>(a, e, off + done, hbuf); break;
      case 5: m_chunk<FMT, 5, EPI>(a, e, off + done, hbuf); break;
      case 6: m_chunk<FMT, 6, EPI>(a, e, off + done, hbuf); break;
      case 7: m_chunk<FMT, 7, EPI>(a, e, off + done, hbuf); break;
      default: m_chunk<FMT, 8, EPI>(a, e, off + done, hbuf); break;
    }
  }
  pdl_launch();
}

// Expert-parallel combine (K4) for GGUF-format experts: one warp per hidden row sums, per token,
// the route-weighted down projections of this rank's experts (experts in order, pairs in token
// order; lane t holds token t) and pushes the sums to every rank's receive region as flagged
// words, which the next RMSNorm (tp_allreduce_rmsnorm_q8) adds into the residual. The hidden
// state is replicated by the attention all-reduce, so nothing is dispatched: each rank's experts
// read their pairs' gathered rows locally.
template <int FMT>
__global__ void __launch_bounds__(256) moe_combine_push_kernel(MoeGemvArgs a, int n_local) {
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + warp;
  const int n_units = a.K / 128;
  float acc = 0.f;
  for (int le = 0; le < n_local; ++le) {
    const int e = a.e_lo + le;
    const int c = a.counts[e], off = a.offsets[e];
    for (int p = 0; p < c; ++p) {
      const int sp = off + p;
      float v[1];
      m_row_dot<FMT, 1>(a.w0, (int64_t)le * a.N + n, n_units, a.xq + (int64_t)sp * a.K, a.xd + (int64_t)sp * (a.K / 32),
                        a.xs + (int64_t)sp * (a.K / 32), a.K, v);
      const int pair = a.sorted[sp];
      if (lane == pair / a.k) acc += a.route_w[pair] * v[0];
    }
  }
  pdl_launch();
  if (lane < a.T) {
    if (a.base) acc += a.base[(int64_t)lane * a.base_stride + n];
    const uint32_t flag = (uint32_t)*a.push_epoch;
    for (int p = 0; p < a.push_n; ++p) ll_store(a.push_recv[p] + (int64_t)lane * a.N + n, __float_as_uint(acc), flag);
  }
}

template <int EPI>
static void moe_gemv_fmt(int fmt, const MoeGemvArgs& a, cudaStream_t s, bool pdl) {
  const int rows_per_cta = EPI == 0 ? 32 : 8;
  dim3 grid(a.N / rows_per_cta, a.E);
  switch (fmt) {
    case WF_Q4_K: launch(moe_gemv_kernel<WF_Q4_K, EPI>, grid, dim3(256), 0, s, pdl, a); break;
    case WF_Q4_0: launch(moe_gemv_kernel<WF_Q4_0, EPI>, grid, dim3(256), 0, s, pdl, a); break;
    case WF_Q8_0: launch(moe_gemv_kernel<WF_Q8_0, EPI>, grid, dim3(256), 0, s, pdl, a); break;
    case WF_Q6_K: launch(moe_gemv_kernel<WF_Q6_K, EPI>, grid, dim3(256), 0, s, pdl, a); break;
    default: throw std::runtime_error("moe_gemv: unsupported weight format");
  }
}

void moe_gemv_launch(int fmt, int epi, const MoeGemvArgs& a, cudaStream_t s, bool pdl) {
  if (a.K % 128) throw std::runtime_error("moe_gemv: K must be a multiple of 128");
  if (epi == 2) {
    if (a.N % 8) throw std::runtime_error("moe combine push: hidden must be a multiple of 8");
    if (!a.push_recv || !a.push_epoch || a.push_n <= 0 || a.T < 1 || a.T > 8)
      throw std::runtime_error("moe combine push: peer tables and 1..8 tokens required");
    const dim3 grid(a.N / 8);
    switch (fmt) {
      case WF_Q4_K: launch(moe_combine_push_kernel<WF_Q4_K>, grid, dim3(256), 0, s, pdl, a, a.E); break;
      case WF_Q4_0: launch(moe_combine_push_kernel<WF_Q4_0>, grid, dim3(256), 0, s, pdl, a, a.E); break;
      case WF_Q8_0: launch(moe_combine_push_kernel<WF_Q8_0>, grid, dim3(256), 0, s, pdl, a, a.E); break;
      case WF_Q6_K: launch(moe_combine_push_kernel<WF_Q6_K>, grid, dim3(256), 0, s, pdl, a, a.E); break;
      default: throw std::runtime_error("moe combine push: unsupported weight format");
    }
    return;
  }
  if (epi == 0) {
    if (a.N % 32) throw std::runtime_error("moe_gemv: expert FFN width must be a multiple of 32");
    moe_gemv_fmt<0>(fmt, a, s, pdl);
  } else {
    if (a.N % 8) throw std::runtime_error("moe_gemv: hidden must be a multiple of 8");
    moe_gemv_fmt<1>(fmt, a, s, pdl);
  }
}

}  // namespace hk
