// Paged GQA decode attention (K5), split-KV with a log-sum-exp merge.
//
// Work decomposition: grid (num_splits, n_kv_heads, rows). One CTA owns one KV head, the G query
// heads that share it, and a contiguous token range of one query row; its 4 warps interleave over
// tiles of T = 32/G tokens. Each lane holds hd/32 contiguous dims of the G query vectors, so a
// tile's G*T partial dot products are reduced with one 31-shuffle transpose-butterfly (lane L ends
// with score L) instead of G*T separate warp reductions. Online softmax per head, then the partial
// (o, lse) of every split goes to scratch and a combine kernel merges the splits, writes the fp32
// output and re-quantises it into q8 blocks for the output projection.
//
// KV layout: [num_blocks, n_kv_heads, block_size, head_dim] bf16, so one head's tokens in a block
// are contiguous (a warp reads whole 256-byte K/V rows).
//
// Parity: crates/hawking-core/shaders/mha.metal (mha_decode_f32, flash split-K
// mha_decode_llama_b9430_fattn_{main,reduce}, multiseq variant with per-sequence regions);
// CPU oracle crates/hawking-core/src/attn.rs:23 (mha_decode_step).
#include "decode_ops.cuh"

namespace hk {

template <int HPL>
__device__ __forceinline__ void load_bf16(const __nv_bfloat16* p, float (&v)[HPL]) {
  if constexpr (HPL == 2) {
    uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(p));
    v[0] = __uint_as_float(w << 16);
    v[1] = __uint_as_float(w & 0xFFFF0000u);
  } else if constexpr (HPL == 4) {
    uint2 w = __ldg(reinterpret_cast<const uint2*>(p));
    v[0] = __uint_as_float(w.x << 16);
    v[1] = __uint_as_float(w.x & 0xFFFF0000u);
    v[2] = __uint_as_float(w.y << 16);
    v[3] = __uint_as_float(w.y & 0xFFFF0000u);
  } else {
    uint4 w = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(ws[i] << 16);
      v[2 * i + 1] = __uint_as_float(ws[i] & 0xFFFF0000u);
    }
  }
}

// G query heads per KV head, HPL = head_dim / 32 dims per lane.
template <int G, int HPL>
__global__ void __launch_bounds__(128) attn_decode_kernel(AttnDecodeArgs a) {
  constexpr int T = 32 / G;  // tokens per tile
  constexpr int HD = HPL * 32;
  const int split = blockIdx.x, kvh = blockIdx.y, r = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float s_m[4][G], s_l[4][G];
  __shared__ float s_o[4][G][HD];

  pdl_wait();
  const int ctx = a.row_ctx[r];
  const int* btab = a.block_tables + (int64_t)a.row_seq[r] * a.max_blocks;
  const int chunk = ((ctx + a.num_splits - 1) / a.num_splits + T - 1) / T * T;
  const int t0 = split * chunk, t1 = min(ctx, t0 + chunk);

  float q[G][HPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float* qp = a.q + ((int64_t)r * a.nh + kvh * G + g) * HD + lane * HPL;
#pragma unroll
    for (int i = 0; i < HPL; ++i) q[g][i] = qp[i] * a.scale;
  }
  float m[G], l[G], acc[G][HPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < HPL; ++i) acc[g][i] = 0.f;
  }
  const int bs = a.block_size;
  const int64_t head_stride = (int64_t)bs * HD;  // one head's slab inside a block
  for (int tt = t0 + warp * T; tt < t1; tt += 4 * T) {
    // ---- scores for T tokens x G heads ----
    float part[32];
#pragma unroll
    for (int j = 0; j < T; ++j) {
      const int t = tt + j;
      float k[HPL];
      if (t < t1) {
        const int blk = btab[t / bs];
        const __nv_bfloat16* kp = a.k_cache + ((int64_t)blk * a.nkv + kvh) * head_stride + (int64_t)(t % bs) * HD + lane * HPL;
        load_bf16<HPL>(kp, k);
      } else {
#pragma unroll
        for (int i = 0; i < HPL; ++i) k[i] = 0.f;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < HPL; ++i) s = fmaf(q[g][i], k[i], s);
        part[g * T + j] = s;
      }
    }
    // Transpose-butterfly: afterwards lane L holds the full sum of value L = (g = L / T, j = L % T).
#pragma unroll
    for (int o = 16, n = 32; o > 0; o >>= 1, n >>= 1) {
      const bool up = lane & o;
#pragma unroll
      for (int i = 0; i < n / 2; ++i) {
        const float send = up ? part[i] : part[i + n / 2];
        const float keep = up ? part[i + n / 2] : part[i];
        part[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    const int my_g = lane / T, my_j = lane % T;
    const float score = (tt + my_j < t1) ? part[0] : -INFINITY;
    // Per-head tile max over the T lanes of the group.
    float tmax = score;
#pragma unroll
    for (int o = T / 2; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
    float p_new_m[G], alpha[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float tm = __shfl_sync(0xffffffffu, tmax, g * T);
      p_new_m[g] = fmaxf(m[g], tm);
      alpha[g] = __expf(m[g] - p_new_m[g]);  // m = -inf at start gives 0
    }
    const float p = (score == -INFINITY) ? 0.f : __expf(score - p_new_m[my_g]);
    float psum = p;
#pragma unroll
    for (int o = T / 2; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float ps = __shfl_sync(0xffffffffu, psum, g * T);
      l[g] = l[g] * alpha[g] + ps;
      m[g] = p_new_m[g];
#pragma unroll
      for (int i = 0; i < HPL; ++i) acc[g][i] *= alpha[g];
    }
    // ---- P.V ----
#pragma unroll
    for (int j = 0; j < T; ++j) {
      const int t = tt + j;
      if (t < t1) {
        const int blk = btab[t / bs];
        float v[HPL];
        const __nv_bfloat16* vp = a.v_cache + ((int64_t)blk * a.nkv + kvh) * head_stride + (int64_t)(t % bs) * HD + lane * HPL;
        load_bf16<HPL>(vp, v);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float pg = __shfl_sync(0xffffffffu, p, g * T + j);
#pragma unroll
          for (int i = 0; i < HPL; ++i) acc[g][i] = fmaf(pg, v[i], acc[g][i]);
        }
      }
    }
  }
  // ---- merge the 4 warps ----
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) { s_m[warp][g] = m[g]; s_l[warp][g] = l[g]; }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < HPL; ++i) s_o[warp][g][lane * HPL + i] = acc[g][i];
  __syncthreads();
  pdl_launch();
  for (int idx = threadIdx.x; idx < G * HD; idx += blockDim.x) {
    const int g = idx / HD, d = idx % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w][g]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = (s_m[w][g] == -INFINITY) ? 0.f : __expf(s_m[w][g] - M);
      L += s_l[w][g] * f;
      O += s_o[w][g][d] * f;
    }
    const int h = kvh * G + g;
    const int64_t base = ((int64_t)r * a.nh + h) * a.num_splits + split;
    a.part_o[base * HD + d] = L > 0.f ? O / L : 0.f;
    if (d == 0) a.part_lse[base] = L > 0.f ? M + __logf(L) : -INFINITY;
  }
}

// Merge splits: one warp per (row, head). Writes fp32 output and/or q8 blocks.
template <int HPL>
__global__ void __launch_bounds__(128) attn_combine_kernel(AttnDecodeArgs a) {
  constexpr int HD = HPL * 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t pair = (int64_t)blockIdx.x * 4 + warp;
  if (pair >= (int64_t)a.R * a.nh) return;
  pdl_wait();
  const int r = (int)(pair / a.nh), h = (int)(pair % a.nh);
  const int64_t base = pair * a.num_splits;
  float M = -INFINITY;
  for (int s = 0; s < a.num_splits; ++s) M = fmaxf(M, a.part_lse[base + s]);
  if (a.sinks) M = fmaxf(M, a.sinks[h]);
  float o[HPL] = {};
  float L = 0.f;
  for (int s = 0; s < a.num_splits; ++s) {
    const float lse = a.part_lse[base + s];
    if (lse == -INFINITY) continue;
    const float f = __expf(lse - M);
    L += f;
    const float* po = a.part_o + (base + s) * HD + lane * HPL;
#pragma unroll
    for (int i = 0; i < HPL; ++i) o[i] = fmaf(f, po[i], o[i]);
  }
  if (a.sinks) L += __expf(a.sinks[h] - M);
  const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
  for (int i = 0; i < HPL; ++i) o[i] *= inv;
  const int64_t col0 = (int64_t)h * HD + lane * HPL;
  const int64_t width = (int64_t)a.nh * HD;
  if (a.out) {
#pragma unroll
    for (int i = 0; i < HPL; ++i) a.out[(int64_t)r * width + col0 + i] = o[i];
  }
  if (a.out_bf16) {
#pragma unroll
    for (int i = 0; i < HPL; ++i) a.out_bf16[(int64_t)r * width + col0 + i] = __float2bfloat16(o[i]);
  }
  if (a.oq) {
    // A q8 block of 32 dims spans 32/HPL lanes.
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < HPL; ++i) amax = fmaxf(amax, fabsf(o[i]));
    constexpr int LPB = 32 / HPL;
#pragma unroll
    for (int off = LPB / 2; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float d = amax / 127.f;
    int qs = 0;
#pragma unroll
    for (int i = 0; i < HPL; ++i) {
      const int qv = amax > 0.f ? __float2int_rn(o[i] / d) : 0;
      qs += qv;
      a.oq[(int64_t)r * width + col0 + i] = (int8_t)qv;
    }
#pragma unroll
    for (int off = LPB / 2; off > 0; off >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, off);
    if ((lane % LPB) == 0) {
      const int64_t blk = (col0 >> 5);
      a.od[(int64_t)r * (width / 32) + blk] = d;
      a.os[(int64_t)r * (width / 32) + blk] = d * (float)qs;
    }
  }
  pdl_launch();
}

template <int G, int HPL>
static void launch_g(const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  launch(attn_decode_kernel<G, HPL>, dim3(a.num_splits, a.nkv, a.R), dim3(128), 0, s, pdl, a);
  launch(attn_combine_kernel<HPL>, dim3((a.R * a.nh + 3) / 4), dim3(128), 0, s, pdl, a);
}

template <int HPL>
static void launch_hpl(const AttnDecodeArgs& a, int G, cudaStream_t s, bool pdl) {
  switch (G) {
    case 1: launch_g<1, HPL>(a, s, pdl); break;
    case 2: launch_g<2, HPL>(a, s, pdl); break;
    case 4: launch_g<4, HPL>(a, s, pdl); break;
    case 8: launch_g<8, HPL>(a, s, pdl); break;
    case 16:
      if constexpr (HPL <= 4) { launch_g<16, HPL>(a, s, pdl); break; }
      [[fallthrough]];
    default: throw std::runtime_error("attention: GQA group must be 1, 2, 4, 8 or 16");
  }
}

void attention_decode_launch(const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  if (a.nh % a.nkv) throw std::runtime_error("attention: n_heads must be a multiple of n_kv_heads");
  const int G = a.nh / a.nkv;
  switch (a.hd) {
    case 64: launch_hpl<2>(a, G, s, pdl); break;
    case 128: launch_hpl<4>(a, G, s, pdl); break;
    case 256: launch_hpl<8>(a, G, s, pdl); break;
    default: throw std::runtime_error("attention: head_dim must be 64, 128 or 256");
  }
}

}  // namespace hk
