// Paged GQA decode attention (K5), split-KV with a log-sum-exp merge.
//
// Work decomposition: grid (num_splits, n_kv_heads, rows). One CTA owns one KV head, the G query
// heads that share it, and a contiguous token range of one query row; its 4 warps interleave over
// tiles of T = 32/G tokens. Each lane holds hd/32 contiguous dims of the G query vectors, so a
// tile's G*T partial dot products are reduced with one 31-shuffle transpose-butterfly (lane L ends
// with score L) instead of G*T separate warp reductions. Online softmax per head; with several
// splits each CTA writes its partial (o, lse) to scratch and bumps a per-(row, kv head) counter,
// and the last CTA to finish merges all splits (independent loads in flight) and writes the
// output as fp32, bf16 and/or q8 blocks for the output projection — no separate combine launch.
//
// KV layout: [num_blocks, n_kv_heads, block_size, head_dim] bf16, so one head's tokens in a block
// are contiguous (a warp reads whole 256-byte K/V rows).
//
// Parity: crates/hawking-core/shaders/mha.metal (mha_decode_f32, flash split-K
// mha_decode_llama_b9430_fattn_{main,reduce}, multiseq variant with per-sequence regions);
// CPU oracle crates/hawking-core/src/attn.rs:23 (mha_decode_step).
#include "decode_ops.cuh"
#include "sm100.cuh"

#include <algorithm>
#include <cooperative_groups.h>

namespace cg = cooperative_groups;

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
  // Tokens per tile: G*T <= 32 partial scores per butterfly; capped to bound the K/V registers.
  constexpr int T = (32 / G) > (HPL >= 8 ? 4 : 8) ? (HPL >= 8 ? 4 : 8) : (32 / G);
  constexpr int NV = G * T;
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
    // ---- issue the K and V loads of the whole tile up front (one round trip) ----
    const int blk_a = btab[tt / bs];
    const int blk_b = btab[min(tt + T - 1, t1 - 1) / bs];
    float kreg[T][HPL], vreg[T][HPL];
#pragma unroll
    for (int j = 0; j < T; ++j) {
      const int t = tt + j;
      if (t < t1) {
        const int blk = (t / bs == tt / bs) ? blk_a : blk_b;
        const int64_t off = ((int64_t)blk * a.nkv + kvh) * head_stride + (int64_t)(t % bs) * HD + lane * HPL;
        load_bf16<HPL>(a.k_cache + off, kreg[j]);
        load_bf16<HPL>(a.v_cache + off, vreg[j]);
      } else {
#pragma unroll
        for (int i = 0; i < HPL; ++i) { kreg[j][i] = 0.f; vreg[j][i] = 0.f; }
      }
    }
    // ---- scores for T tokens x G heads ----
    float part[32];
#pragma unroll
    for (int v = NV; v < 32; ++v) part[v] = 0.f;
#pragma unroll
    for (int j = 0; j < T; ++j) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float sdot = 0.f;
#pragma unroll
        for (int i = 0; i < HPL; ++i) sdot = fmaf(q[g][i], kreg[j][i], sdot);
        part[g * T + j] = sdot;
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
    const int my_g = min(lane / T, G - 1), my_j = lane % T;
    const float score = (lane < NV && tt + my_j < t1) ? part[0] : -INFINITY;
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
    float mg = p_new_m[0];
#pragma unroll
    for (int g = 1; g < G; ++g)
      if (my_g == g) mg = p_new_m[g];
    const float p = (score == -INFINITY) ? 0.f : __expf(score - mg);
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
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pg = __shfl_sync(0xffffffffu, p, g * T + j);
#pragma unroll
        for (int i = 0; i < HPL; ++i) acc[g][i] = fmaf(pg, vreg[j][i], acc[g][i]);
      }
    }
  }
  // ---- merge the 4 warps ----
  __shared__ float s_fin[G][HD];
  __shared__ float s_lse[G][64];
  __shared__ int s_last;
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
  const bool single = a.num_splits == 1;
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
    if (single) {
      if (a.sinks) L += __expf(a.sinks[kvh * G + g] - M);
      s_fin[g][d] = L > 0.f ? O / L : 0.f;
    } else {
      const int h = kvh * G + g;
      const int64_t base = ((int64_t)r * a.nh + h) * a.num_splits + split;
      a.part_o[base * HD + d] = L > 0.f ? O / L : 0.f;
      if (d == 0) a.part_lse[base] = L > 0.f ? M + __logf(L) : -INFINITY;
    }
  }
  if (!single) {
    // The last split CTA of this (row, kv head) merges every split (threadfence reduction).
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const int prev = atomicAdd(&a.counters[r * a.nkv + kvh], 1);
      s_last = prev == a.num_splits - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int S = a.num_splits;
    for (int idx = threadIdx.x; idx < G * S; idx += blockDim.x) {
      const int g = idx / S, sp = idx % S;
      s_lse[g][sp] = __ldcg(a.part_lse + ((int64_t)r * a.nh + kvh * G + g) * S + sp);
    }
    __syncthreads();
    if (threadIdx.x < G) {  // per-head max and normaliser; weights stored back in s_lse
      const int g = threadIdx.x;
      float M = -INFINITY;
      for (int sp = 0; sp < S; ++sp) M = fmaxf(M, s_lse[g][sp]);
      if (a.sinks) M = fmaxf(M, a.sinks[kvh * G + g]);
      float L = 0.f;
      for (int sp = 0; sp < S; ++sp) {
        const float f = s_lse[g][sp] == -INFINITY ? 0.f : __expf(s_lse[g][sp] - M);
        s_lse[g][sp] = f;
        L += f;
      }
      if (a.sinks) L += __expf(a.sinks[kvh * G + g] - M);
      s_m[0][g] = L > 0.f ? 1.f / L : 0.f;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * HD; idx += blockDim.x) {
      const int g = idx / HD, d = idx % HD;
      const float* po = a.part_o + (((int64_t)r * a.nh + kvh * G + g) * S) * HD + d;
      float O0 = 0.f, O1 = 0.f, O2 = 0.f, O3 = 0.f;
      int sp = 0;
      for (; sp + 4 <= S; sp += 4) {  // independent loads in flight
        O0 = fmaf(s_lse[g][sp], __ldcg(po + (int64_t)sp * HD), O0);
        O1 = fmaf(s_lse[g][sp + 1], __ldcg(po + (int64_t)(sp + 1) * HD), O1);
        O2 = fmaf(s_lse[g][sp + 2], __ldcg(po + (int64_t)(sp + 2) * HD), O2);
        O3 = fmaf(s_lse[g][sp + 3], __ldcg(po + (int64_t)(sp + 3) * HD), O3);
      }
      for (; sp < S; ++sp) O0 = fmaf(s_lse[g][sp], __ldcg(po + (int64_t)sp * HD), O0);
      s_fin[g][d] = (O0 + O1 + O2 + O3) * s_m[0][g];
    }
    if (threadIdx.x == 0) a.counters[r * a.nkv + kvh] = 0;  // ready for the next launch
    __syncthreads();
  } else {
    __syncthreads();
  }
  // ---- final outputs of the G heads: fp32 / bf16 / q8 blocks of 32 dims ----
  const int64_t width = (int64_t)a.nh * HD;
  const int64_t col0 = (int64_t)kvh * G * HD;
  for (int idx = threadIdx.x; idx < G * HD; idx += blockDim.x) {
    const float v = s_fin[idx / HD][idx % HD];
    if (a.out) a.out[(int64_t)r * width + col0 + idx] = v;
    if (a.out_bf16) a.out_bf16[(int64_t)r * width + col0 + idx] = __float2bfloat16(v);
  }
  if (a.oq) {
    for (int blk = warp; blk < G * HD / 32; blk += 4) {
      const int idx = blk * 32 + lane;
      const float v = s_fin[idx / HD][idx % HD];
      const float amax = warp_max(fabsf(v));
      const float dq = amax / 127.f;
      const int qv = amax > 0.f ? __float2int_rn(v / dq) : 0;
      const float qsum = warp_sum((float)qv);
      a.oq[(int64_t)r * width + col0 + idx] = (int8_t)qv;
      if (lane == 0) {
        a.od[(int64_t)r * (width / 32) + (col0 >> 5) + blk] = dq;
        a.os[(int64_t)r * (width / 32) + (col0 >> 5) + blk] = dq * qsum;
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Cluster variant: the S = num_splits (1..16) CTAs of one (row, kv head) form a thread-block cluster; CTA s
// owns the s-th contiguous token range (a whole number of KV blocks). One thread streams the
// range's K and V block slabs (block_size x head_dim bf16, contiguous per head) into shared
// memory with untiled bulk async copies completing on an mbarrier: every byte of the window is in
// flight at once (one memory round trip), and when the range exceeds the shared ring it is
// processed in two alternating windows (the next window loads while this one is computed). The
// WARPS warps then take tiles of T tokens from shared memory (lane = HPL dims of every head of the
// group; transpose-butterfly score reduction; online softmax). The warps' partials are folded into
// one (max, sum, o) per CTA; after a cluster barrier each CTA merges whole 32-dim output blocks
// across the S CTAs by reading their shared memory directly (distributed shared memory). No
// global scratch, no split counters, no second pass over memory.
template <int HPL>
__device__ __forceinline__ void lds_bf16(const __nv_bfloat16* p, float (&v)[HPL]) {
  if constexpr (HPL == 2) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
    v[0] = __uint_as_float(w << 16);
    v[1] = __uint_as_float(w & 0xFFFF0000u);
  } else if constexpr (HPL == 4) {
    const uint2 w = *reinterpret_cast<const uint2*>(p);
    v[0] = __uint_as_float(w.x << 16);
    v[1] = __uint_as_float(w.x & 0xFFFF0000u);
    v[2] = __uint_as_float(w.y << 16);
    v[3] = __uint_as_float(w.y & 0xFFFF0000u);
  } else {
    const uint4 w = *reinterpret_cast<const uint4*>(p);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(ws[i] << 16);
      v[2 * i + 1] = __uint_as_float(ws[i] & 0xFFFF0000u);
    }
  }
}

template <int G, int HPL, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) attn_decode_cluster_kernel(AttnDecodeArgs a) {
  constexpr int T = (32 / G) > 8 ? 8 : (32 / G);
  constexpr int NV = G * T;
  constexpr int HD = HPL * 32;
  cg::cluster_group cluster = cg::this_cluster();
  const int S = (int)cluster.num_blocks();
  const int split = (int)cluster.block_rank();
  const int kvh = blockIdx.y, r = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  extern __shared__ __align__(128) uint8_t att_smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(att_smem);  // [2] window barriers
  __nv_bfloat16* ring = reinterpret_cast<__nv_bfloat16*>(att_smem + 128);
  __shared__ float s_wm[WARPS][G];
  __shared__ float s_m[G], s_l[G];
  __shared__ __align__(16) float s_o[G][HD];
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) (&s_o[0][0])[i] = 0.f;
  if (threadIdx.x < G) s_l[threadIdx.x] = 0.f;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&full[0], 1);
    sm100::mbar_init(&full[1], 1);
    sm100::fence_barrier_init();
  }
  __syncthreads();

  pdl_wait();
  const int bs = a.block_size;
  const int slab = bs * HD;  // elements of one head's K (or V) in one block
  const int ctx = a.row_ctx[r];
  const int* btab = a.block_tables + (int64_t)a.row_seq[r] * a.max_blocks;
  const int nblk_ctx = (ctx + bs - 1) / bs;
  const int bpc = (nblk_ctx + S - 1) / S;  // blocks per CTA
  const int b0 = split * bpc, b1 = min(nblk_ctx, b0 + bpc);
  const int t0 = b0 * bs, t1 = min(ctx, b1 * bs);
  const int nb = max(0, b1 - b0);
  const int NS = a.stage_blocks;
  const bool dbl = nb > NS;
  const int WB = dbl ? NS / 2 : NS;
  const int nwin = nb > 0 ? (nb + WB - 1) / WB : 0;

  auto issue = [&](int w) {  // thread 0: bulk-copy window w's K/V slabs into its ring half
    const int buf = dbl ? (w & 1) : 0;
    const int wb0 = b0 + w * WB, wb1 = min(b1, wb0 + WB);
    sm100::mbar_arrive_expect_tx(&full[buf], (uint32_t)((wb1 - wb0) * 2 * slab * 2));
    for (int b = wb0; b < wb1; ++b) {
      const int64_t src = ((int64_t)btab[b] * a.nkv + kvh) * slab;
      __nv_bfloat16* dst = ring + (int64_t)(buf * WB + (b - wb0)) * 2 * slab;
      sm100::bulk_g2s(dst, a.k_cache + src, (uint32_t)slab * 2, &full[buf]);
      sm100::bulk_g2s(dst + slab, a.v_cache + src, (uint32_t)slab * 2, &full[buf]);
    }
  };
  if (threadIdx.x == 0 && nwin > 0) {
    issue(0);
    if (dbl && nwin > 1) issue(1);
  }

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
  bool ok = true;
  for (int w = 0; w < nwin; ++w) {
    const int buf = dbl ? (w & 1) : 0;
    const uint32_t parity = (uint32_t)((dbl ? (w >> 1) : w) & 1);
    if (ok) {
      ok = sm100::mbar_wait(&full[buf], parity, a.status);
      if (!ok && threadIdx.x == 0) {  // timed out: give this window's copies one more bounded wait
        for (uint32_t i = 0; i < (1u << 20) && !sm100::mbar_try_wait(&full[buf], parity); ++i) {
        }
      }
    }
    const int wb0 = b0 + w * WB;
    const int tw0 = max(t0, wb0 * bs), tw1 = min(t1, min(b1, wb0 + WB) * bs);
    const __nv_bfloat16* base = ring + (int64_t)buf * WB * 2 * slab;
    for (int tt = tw0 + warp * T; ok && tt < tw1; tt += WARPS * T) {
      float part[32];
#pragma unroll
      for (int v = NV; v < 32; ++v) part[v] = 0.f;
#pragma unroll
      for (int j = 0; j < T; ++j) {
        const int t = min(tt + j, tw1 - 1);
        const int lb = t / bs - wb0;
        float kr[HPL];
        lds_bf16<HPL>(base + (int64_t)lb * 2 * slab + (t % bs) * HD + lane * HPL, kr);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float sdot = 0.f;
#pragma unroll
          for (int i = 0; i < HPL; ++i) sdot = fmaf(q[g][i], kr[i], sdot);
          part[g * T + j] = sdot;
        }
      }
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
      const int my_g = min(lane / T, G - 1), my_j = lane % T;
      const float score = (lane < NV && tt + my_j < tw1) ? part[0] : -INFINITY;
      float tmax = score;
#pragma unroll
      for (int o = T / 2; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      float p_new_m[G], alpha[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float tm = __shfl_sync(0xffffffffu, tmax, g * T);
        p_new_m[g] = fmaxf(m[g], tm);
        alpha[g] = __expf(m[g] - p_new_m[g]);
      }
      float mg = p_new_m[0];
#pragma unroll
      for (int g = 1; g < G; ++g)
        if (my_g == g) mg = p_new_m[g];
      const float p = (score == -INFINITY) ? 0.f : __expf(score - mg);
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
#pragma unroll
      for (int j = 0; j < T; ++j) {
        const int t = min(tt + j, tw1 - 1);
        const int lb = t / bs - wb0;
        float vr[HPL];
        lds_bf16<HPL>(base + (int64_t)lb * 2 * slab + slab + (t % bs) * HD + lane * HPL, vr);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float pg = __shfl_sync(0xffffffffu, p, g * T + j);
#pragma unroll
          for (int i = 0; i < HPL; ++i) acc[g][i] = fmaf(pg, vr[i], acc[g][i]);
        }
      }
    }
    __syncthreads();  // every warp is done with this ring half
    if (threadIdx.x == 0 && dbl && w + 2 < nwin && ok) issue(w + 2);
  }
  // ---- fold the warps into one (m, l, o) per CTA ----
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) s_wm[warp][g] = m[g];
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, s_wm[w][g]);
    const float f = (m[g] == -INFINITY) ? 0.f : __expf(m[g] - M);
    if (f != 0.f) {
#pragma unroll
      for (int i = 0; i < HPL; ++i) atomicAdd(&s_o[g][lane * HPL + i], acc[g][i] * f);
      if (lane == 0) atomicAdd(&s_l[g], l[g] * f);
    }
    if (warp == 0 && lane == 0) s_m[g] = M;
  }
  pdl_launch();
  cluster.sync();  // every CTA's (m, l, o) is complete and visible to the cluster

  // ---- merge whole 32-dim blocks across the cluster; CTA s takes blocks s, s + S, ... ----
  const int64_t width = (int64_t)a.nh * HD;
  const int64_t col0 = (int64_t)kvh * G * HD;
  constexpr int NBLK = G * HD / 32;
  for (int blk = split + S * warp; blk < NBLK; blk += S * WARPS) {
    const int idx = blk * 32 + lane;
    const int g = idx / HD, d = idx % HD;
    float mk[16], lk[16], okv[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      if (k < S) {
        mk[k] = *cluster.map_shared_rank(&s_m[g], k);
        lk[k] = *cluster.map_shared_rank(&s_l[g], k);
        okv[k] = *cluster.map_shared_rank(&s_o[g][d], k);
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < 16; ++k)
      if (k < S) M = fmaxf(M, mk[k]);
    const float sink = a.sinks ? a.sinks[kvh * G + g] : -INFINITY;
    M = fmaxf(M, sink);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      if (k < S && mk[k] != -INFINITY) {
        const float f = __expf(mk[k] - M);
        L += lk[k] * f;
        O += okv[k] * f;
      }
    }
    if (a.sinks) L += __expf(sink - M);
    const float v = L > 0.f ? O / L : 0.f;
    if (a.out) a.out[(int64_t)r * width + col0 + idx] = v;
    if (a.out_bf16) a.out_bf16[(int64_t)r * width + col0 + idx] = __float2bfloat16(v);
    if (a.oq) {
      const float amax = warp_max(fabsf(v));
      const float dq = amax / 127.f;
      const int qv = amax > 0.f ? __float2int_rn(v / dq) : 0;
      const float qsum = warp_sum((float)qv);
      a.oq[(int64_t)r * width + col0 + idx] = (int8_t)qv;
      if (lane == 0) {
        a.od[(int64_t)r * (width / 32) + (col0 >> 5) + blk] = dq;
        a.os[(int64_t)r * (width / 32) + (col0 >> 5) + blk] = dq * qsum;
      }
    }
  }
  cluster.sync();  // keep this CTA's shared memory alive until every CTA has read it
}

// Shared-memory ring: at most kAttnRingBytes of K/V slabs per CTA (enough blocks for the CTA's
// largest possible token range, bounded by the block-table width).
constexpr int kAttnRingBytes = 192 * 1024;

template <int G, int HPL>
static void launch_cluster_g(AttnDecodeArgs a, cudaStream_t s, bool pdl) {
  constexpr int WARPS = G * HPL <= 16 ? 16 : 8;
  constexpr int HD = HPL * 32;
  const int pair = 2 * a.block_size * HD * 2;  // K + V slab bytes of one block
  const int most = (a.max_blocks + a.num_splits - 1) / a.num_splits;
  int ns = std::min(most, kAttnRingBytes / pair);
  if (ns < most && ns >= 2) ns &= ~1;  // two equal windows when the range does not fit at once
  if (ns < 1 || (ns < most && ns < 2))
    throw std::runtime_error("attention: KV block too large for the shared-memory ring");
  a.stage_blocks = ns;
  const size_t smem = 128 + (size_t)ns * pair;
  auto kern = attn_decode_cluster_kernel<G, HPL, WARPS>;
  HK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  // 16-CTA clusters (splits of one (row, kv head)) need the non-portable size (sm_90+)
  if (a.num_splits > 8) HK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  launch_cluster(kern, dim3(a.num_splits, a.nkv, a.R), dim3(WARPS * 32), smem, s, pdl, a.num_splits, a);
}

template <int HPL>
static void launch_cluster_hpl(const AttnDecodeArgs& a, int G, cudaStream_t s, bool pdl) {
  switch (G) {
    case 1: launch_cluster_g<1, HPL>(a, s, pdl); break;
    case 2: launch_cluster_g<2, HPL>(a, s, pdl); break;
    case 4: launch_cluster_g<4, HPL>(a, s, pdl); break;
    case 8: launch_cluster_g<8, HPL>(a, s, pdl); break;
    case 16:
      if constexpr (HPL <= 4) { launch_cluster_g<16, HPL>(a, s, pdl); break; }
      [[fallthrough]];
    default: throw std::runtime_error("attention: GQA group must be 1, 2, 4, 8 or 16");
  }
}

void attention_decode_cluster_launch(const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  if (a.nh % a.nkv) throw std::runtime_error("attention: n_heads must be a multiple of n_kv_heads");
  if ((reinterpret_cast<uintptr_t>(a.k_cache) | reinterpret_cast<uintptr_t>(a.v_cache)) & 15)
    throw std::runtime_error("attention (cluster): K/V caches must be 16-byte aligned");
  if (a.num_splits != 1 && a.num_splits != 2 && a.num_splits != 4 && a.num_splits != 8 && a.num_splits != 16)
    throw std::runtime_error("attention (cluster): num_splits must be 1, 2, 4, 8 or 16");
  const int G = a.nh / a.nkv;
  switch (a.hd) {
    case 64: launch_cluster_hpl<2>(a, G, s, pdl); break;
    case 128: launch_cluster_hpl<4>(a, G, s, pdl); break;
    case 256: launch_cluster_hpl<8>(a, G, s, pdl); break;
    default: throw std::runtime_error("attention: head_dim must be 64, 128 or 256");
  }
}

template <int G, int HPL>
static void launch_g(const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  launch(attn_decode_kernel<G, HPL>, dim3(a.num_splits, a.nkv, a.R), dim3(128), 0, s, pdl, a);
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
  if (a.num_splits > 64) throw std::runtime_error("attention: at most 64 splits");
  if (a.num_splits > 1 && !a.counters) throw std::runtime_error("attention: split-KV needs the counter scratch");
  if (a.block_size < 8) throw std::runtime_error("attention: block_size must be at least 8");
  const int G = a.nh / a.nkv;
  switch (a.hd) {
    case 64: launch_hpl<2>(a, G, s, pdl); break;
    case 128: launch_hpl<4>(a, G, s, pdl); break;
    case 256: launch_hpl<8>(a, G, s, pdl); break;
    default: throw std::runtime_error("attention: head_dim must be 64, 128 or 256");
  }
}

}  // namespace hk

// =================================================================================================
// Allocation-free entry point: hk_attention_decode_noalloc (declared, with its limits and the
// rules for callers, in noalloc.h). No counterpart in the reference.
//
// Callers that cannot call cudaMalloc (an engine embedded in a host whose allocator owns the
// device memory, or a decode loop where allocation and its possible device synchronisation are
// not allowed) get the same split-KV decode attention with its scratch in fixed file-scope device
// arrays. Their device addresses are looked up once per device (cudaGetSymbolAddress with that
// device current) on the first call, which should come before any stream capture.
// =================================================================================================
#include <mutex>

#include "noalloc.h"

namespace {
constexpr int64_t kNoAllocPartElems = int64_t(1) << 20;  // 4 MiB of fp32 partial outputs
constexpr int64_t kNoAllocLseElems = int64_t(1) << 14;   // 64 KiB of fp32 log-sum-exps
constexpr int64_t kNoAllocCounters = 4096;                // 16 KiB of split counters

static __device__ __align__(256) float g_noalloc_part_o[kNoAllocPartElems];
static __device__ __align__(256) float g_noalloc_lse[kNoAllocLseElems];
static __device__ __align__(256) int g_noalloc_counters[kNoAllocCounters];

struct NoAllocScratch {
  float* part_o = nullptr;
  float* lse = nullptr;
  int* counters = nullptr;
  bool ready = false;
};
constexpr int kMaxDevices = 64;
NoAllocScratch g_noalloc[kMaxDevices];
std::mutex g_noalloc_mu;
thread_local std::string g_noalloc_error;

int noalloc_fail(int code, const std::string& msg) {
  g_noalloc_error = msg;
  return code;
}
}  // namespace

// Message of the last failing call on this host thread ("" after a success).
extern "C" __attribute__((visibility("default"))) const char* hk_attention_decode_noalloc_error(void) {
  return g_noalloc_error.c_str();
}

// Paged GQA decode attention without any allocation (see the block comment above).
//   q            [rows, n_heads, head_dim] fp32 (already RoPE'd)
//   k_cache      [num_blocks, n_kv_heads, block_size, head_dim] bf16 (v_cache alike)
//   block_tables [*, max_blocks] int32; row_seq / row_ctx [rows] int32
//   out          [rows, n_heads * head_dim] fp32
//   stream       cudaStream_t to launch on (nullptr = legacy default stream)
// Returns HK_NOALLOC_OK or an error code; hk_attention_decode_noalloc_error() explains it.
extern "C" __attribute__((visibility("default"))) int hk_attention_decode_noalloc(
    const float* q, const void* k_cache, const void* v_cache, const int* block_tables, int max_blocks,
    const int* row_seq, const int* row_ctx, float scale, int rows, int n_heads, int n_kv_heads, int head_dim,
    int block_size, int num_splits, float* out, void* stream) {
  using namespace hk;
  g_noalloc_error.clear();
  if (!q || !k_cache || !v_cache || !block_tables || !row_seq || !row_ctx || !out)
    return noalloc_fail(HK_NOALLOC_BAD_ARG, "null pointer argument");
  if (rows <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || num_splits <= 0 || num_splits > 64 ||
      block_size <= 0 || max_blocks <= 0)
    return noalloc_fail(HK_NOALLOC_BAD_ARG, "invalid geometry");
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return noalloc_fail(HK_NOALLOC_BAD_ARG, "head_dim must be 64, 128 or 256");
  // a tile of up to 8 consecutive tokens may span at most two KV blocks
  if (block_size < 8) return noalloc_fail(HK_NOALLOC_BAD_ARG, "block_size must be at least 8");
  // vector loads of K/V (up to 16 bytes per lane) and q / out rows
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(q) |
       reinterpret_cast<uintptr_t>(out)) & 15)
    return noalloc_fail(HK_NOALLOC_BAD_ARG, "q, k_cache, v_cache and out must be 16-byte aligned");
  const int64_t part = (int64_t)rows * n_heads * num_splits * head_dim;
  const int64_t lse = (int64_t)rows * n_heads * num_splits;
  const int64_t cnt = (int64_t)rows * n_kv_heads;
  if (part > kNoAllocPartElems || lse > kNoAllocLseElems || cnt > kNoAllocCounters)
    return noalloc_fail(HK_NOALLOC_TOO_LARGE,
                        "request needs " + std::to_string(part) + " partial floats, " + std::to_string(lse) +
                            " log-sum-exps and " + std::to_string(cnt) + " counters; the fixed scratch holds " +
                            std::to_string(kNoAllocPartElems) + ", " + std::to_string(kNoAllocLseElems) + " and " +
                            std::to_string(kNoAllocCounters));
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return noalloc_fail(HK_NOALLOC_CUDA_ERROR, "no current CUDA device");
  NoAllocScratch sc;
  {
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    NoAllocScratch& s = g_noalloc[dev];
    if (!s.ready) {  // once per device, with that device current
      cudaError_t e1 = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.part_o), g_noalloc_part_o);
      cudaError_t e2 = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.lse), g_noalloc_lse);
      cudaError_t e3 = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.counters), g_noalloc_counters);
      if (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess)
        return noalloc_fail(HK_NOALLOC_CUDA_ERROR, std::string("cudaGetSymbolAddress failed: ") +
                                                       cudaGetErrorString(e1 != cudaSuccess ? e1 : (e2 != cudaSuccess ? e2 : e3)));
      s.ready = true;
    }
    sc = s;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (st) {  // the scratch looked up above is the current device's: the stream must be on it too
    int sdev = -1;
    if (cudaStreamGetDevice(st, &sdev) != cudaSuccess)
      return noalloc_fail(HK_NOALLOC_BAD_ARG, "stream is not a valid CUDA stream");
    if (sdev != dev) return noalloc_fail(HK_NOALLOC_BAD_ARG, "stream belongs to another device than the current one");
  }
  // The split counters must start at zero (a previous call may have been interrupted).
  cudaError_t e = cudaMemsetAsync(sc.counters, 0, sizeof(int) * cnt, st);
  if (e != cudaSuccess) return noalloc_fail(HK_NOALLOC_CUDA_ERROR, std::string("clearing counters: ") + cudaGetErrorString(e));
  AttnDecodeArgs a{};
  a.q = q;
  a.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache);
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache);
  a.block_tables = block_tables;
  a.max_blocks = max_blocks;
  a.row_seq = row_seq;
  a.row_ctx = row_ctx;
  a.scale = scale;
  a.R = rows;
  a.nh = n_heads;
  a.nkv = n_kv_heads;
  a.hd = head_dim;
  a.block_size = block_size;
  a.num_splits = num_splits;
  a.part_o = sc.part_o;
  a.part_lse = sc.lse;
  a.counters = sc.counters;
  a.out = out;
  try {
    attention_decode_launch(a, st, false);
  } catch (const std::exception& ex) {
    return noalloc_fail(HK_NOALLOC_CUDA_ERROR, ex.what());
  }
  return HK_NOALLOC_OK;
}
