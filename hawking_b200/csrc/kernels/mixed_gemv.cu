// `.gravity` sub-2-bit / low-bit GEMV (K8): binary sign + group scale (HGRAVB01) and uniform
// 2/4/8-bit group codes (HGRAVU01; 2-bit with bound 1 is the ternary point), dequantised in
// registers against q8 activation blocks with dp4a; block-scaled fp8 e4m3 and fp4 e2m1 (e8m0
// exponents per 32 columns) decoded to fp32 against the same blocks.
//
// Storage on the GPU is the codec's own payload bytes, split into two planes per tensor: the
// LSB-first code stream of every row ([rows, K * bits / 8] bytes, exactly the body bits) and the
// fp16 group scales ([rows, K / group]). A per-tensor descriptor carries the codec, so one launch
// can mix codecs across experts (the per-tensor bit assignment of a mixed artifact).
//
// Per 32-element activation block (d_x, s_x = d_x * sum q):
//   binary   w_i = s_g * (2 b_i - 1):        s_g * (2 d_x sum_{b_i=1} q_i - s_x)
//   uniform  w_i = s_g * (c_i - bound):      s_g * (d_x sum c_i q_i - bound * s_x)
// Bits are widened to bytes with shift-multiply (1 bit) or shift-OR (2 bits) spreads, or nibble masks with a
// byte permute of the activations (4 bits, LSB-first pairs), then one dp4a per 4 elements.
//
// Dense kernel: one warp per output row, lane = 32-element blocks lane, lane + 32, ...;
// epilogues STORE (fp32), RESID (+=) and SWIGLU_Q8 (gate/up descriptor pair -> q8, 32 rows per
// CTA). Expert kernel: the routed (token, expert) pairs in expert order (moe_align), one grid row
// per active expert, chunks of <= 8 pairs; SwiGLU -> q8 in pair order, or the route-weighted
// atomic add into each token's residual.
//
// Parity: crates/hawking-core/src/model/qwen_complete_binary/q80_mixed_decode.rs:135-1070
// (binary / uniform matvec oracles), crates/hawking-core/shaders/q80_mixed_decode.metal and
// qwen_uniform_q4.metal / qwen_binary*.metal (packed matvec families),
// qwen80_all_ten_routed_expert_wave.metal (10 routed experts through a 512-way expert table).
#include <cuda_fp8.h>

#include "api.h"
#include "qformats.cuh"
#include "tp.cuh"

namespace hk {

// 4 bits -> 4 bytes of 0/1 (bit k to byte k).
__device__ __forceinline__ uint32_t spread1(uint32_t nib) { return (nib * 0x00204081u) & 0x01010101u; }
// 4 two-bit codes (one byte) -> 4 bytes (shifted copies overlap, so OR them: no carries).
__device__ __forceinline__ uint32_t spread2(uint32_t byte) {
  return (byte | (byte << 6) | (byte << 12) | (byte << 18)) & 0x03030303u;
}

// Dot of one 32-element block of row `row` of tensor `t` with activation block `blk`.
__device__ __forceinline__ float mixed_block_dot(const MixedDesc& t, int64_t row, int blk, const int8_t* xq,
                                                  float dx, float sx) {
  const uint8_t* codes = t.codes + row * t.code_row_bytes;
  const int4 qa = *reinterpret_cast<const int4*>(xq + blk * 32);
  const int4 qb = *reinterpret_cast<const int4*>(xq + blk * 32 + 16);
  const int q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  int dot = 0;
  if (t.kind == MIXED_FP8) {  // fp8 e4m3 codes, fp32 scale per 128-column block of the row
    const float sw = t.scales_f32[row * t.scale_row_elems + (blk * 32) / t.group];
    const uint4 w0 = __ldg(reinterpret_cast<const uint4*>(codes) + 2 * blk);
    const uint4 w1 = __ldg(reinterpret_cast<const uint4*>(codes) + 2 * blk + 1);
    const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(ws[j] & 0xFFFFu), __NV_E4M3);
      const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(ws[j] >> 16), __NV_E4M3);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
      const uint32_t qw = (uint32_t)q[j];
      acc += a.x * (float)(int8_t)(qw & 0xFF) + a.y * (float)(int8_t)((qw >> 8) & 0xFF) +
             b.x * (float)(int8_t)((qw >> 16) & 0xFF) + b.y * (float)(int8_t)(qw >> 24);
    }
    (void)sx;
    return sw * dx * acc;
  }
  if (t.kind == MIXED_FP4) {  // e2m1 codes, element k of a word in nibble k; fp32 scale per block
    const float sw = t.scales_f32[row * t.scale_row_elems + blk];
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(codes) + blk);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const uint32_t c = (ws[e >> 3] >> (4 * (e & 7))) & 0xFu;
      acc += e2m1_value(c) * (float)(int8_t)(((uint32_t)q[e >> 2] >> (8 * (e & 3))) & 0xFFu);
    }
    (void)sx;
    return sw * dx * acc;
  }
  if (t.kind == MIXED_Q4K) {
    // GGUF Q4_K sub-block j of super-block sb: w = d * sc_j * q - dmin * m_j, q the low (even j) or
    // high (odd j) nibbles of the 32 quant bytes the sub-block pair shares
    const int sb = blk >> 3, j = blk & 7;
    const uint4 h = __ldg(reinterpret_cast<const uint4*>(t.scales + row * t.scale_row_elems) + sb);
    int sc, mn;
    q4k_scale_min(j, h.y, h.z, h.w, sc, mn);
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    const uint4* qp = reinterpret_cast<const uint4*>(codes + sb * 128 + (j >> 1) * 32);
    const uint4 w0 = __ldg(qp), w1 = __ldg(qp + 1);
    const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    const int sh = (j & 1) * 4;
#pragma unroll
    for (int k = 0; k < 8; ++k) dot = dp4a((int)((ws[k] >> sh) & 0x0F0F0F0Fu), q[k], dot);
    return d * (float)sc * dx * (float)dot - dmin * (float)mn * sx;
  }
  const float sg = __half2float(t.scales[row * t.scale_row_elems + (blk * 32) / t.group]);
  if (t.kind == MIXED_BINARY) {
    const uint32_t b = __ldg(reinterpret_cast<const uint32_t*>(codes) + blk);
#pragma unroll
    for (int j = 0; j < 8; ++j) dot = dp4a((int)spread1((b >> (4 * j)) & 0xFu), q[j], dot);
    return sg * (2.f * dx * (float)dot - sx);
  }
  if (t.bits == 2) {
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(codes) + blk);
#pragma unroll
    for (int j = 0; j < 4; ++j) dot = dp4a((int)spread2((w.x >> (8 * j)) & 0xFFu), q[j], dot);
#pragma unroll
    for (int j = 0; j < 4; ++j) dot = dp4a((int)spread2((w.y >> (8 * j)) & 0xFFu), q[4 + j], dot);
  } else if (t.bits == 4) {
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(codes) + blk);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // word j: elements 8j..8j+7, element 8j+2i in the low nibble of byte i
      const int even = (int)__byte_perm((uint32_t)q[2 * j], (uint32_t)q[2 * j + 1], 0x6420);
      const int odd = (int)__byte_perm((uint32_t)q[2 * j], (uint32_t)q[2 * j + 1], 0x7531);
      dot = dp4a((int)(ws[j] & 0x0F0F0F0Fu), even, dot);
      dot = dp4a((int)((ws[j] >> 4) & 0x0F0F0F0Fu), odd, dot);
    }
  } else {  // 8 bits: codes c as signed (c - 128), so sum (c - bound) q = dot + (128 - bound) sum q
    const uint4 w0 = __ldg(reinterpret_cast<const uint4*>(codes) + 2 * blk);
    const uint4 w1 = __ldg(reinterpret_cast<const uint4*>(codes) + 2 * blk + 1);
    const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) dot = dp4a((int)(ws[j] ^ 0x80808080u), q[j], dot);
    return sg * (dx * (float)dot + (float)(128 - t.bound) * sx);
  }
  return sg * (dx * (float)dot - (float)t.bound * sx);
}

__device__ __forceinline__ float mixed_row_dot(const MixedDesc& t, int64_t row, int K, const int8_t* xq,
                                               const float* xd, const float* xs) {
  const int lane = threadIdx.x & 31;
  float acc = 0.f;
  for (int blk = lane; blk < K / 32; blk += 32) acc += mixed_block_dot(t, row, blk, xq, xd[blk], xs[blk]);
  return warp_sum(acc);
}

// ---- dense ------------------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(256) mixed_gemv_kernel(MixedGemvArgs a) {
  __shared__ float hbuf[8][32];
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const MixedDesc t0 = a.desc[a.d0];
  for (int b = 0; b < a.nb; ++b) {
    const int8_t* xq = a.xq + (int64_t)b * a.x_stride_q;
    const float* xd = a.xd + (int64_t)b * a.x_stride_s;
    const float* xs = a.xs + (int64_t)b * a.x_stride_s;
    if constexpr (EPI == EPI_SWIGLU_Q8) {
      const MixedDesc t1 = a.desc[a.d1];
#pragma unroll 1
      for (int r = 0; r < 4; ++r) {
        const int n = blockIdx.x * 32 + warp * 4 + r;
        float h = 0.f;
        if (n < a.N) {
          const float g = mixed_row_dot(t0, n, a.K, xq, xd, xs);
          const float u = mixed_row_dot(t1, n, a.K, xq, xd, xs);
          h = g / (1.f + __expf(-g)) * u;
        }
        if (lane == 0) hbuf[warp][r] = h;
      }
      __syncthreads();
      if (warp == 0) {
        const int n = blockIdx.x * 32 + lane;
        const float v = hbuf[lane >> 2][lane & 3];
        const float amax = warp_max(fabsf(v));
        const float d = amax / 127.f;
        const int q = amax > 0.f ? __float2int_rn(v / d) : 0;
        const float qs = warp_sum((float)q);
        if (n < a.N) a.oq[(int64_t)b * a.o_stride_q + n] = (int8_t)q;
        if (lane == 0 && n < a.N) {
          a.od[(int64_t)b * a.o_stride_s + (n >> 5)] = d;
          a.os[(int64_t)b * a.o_stride_s + (n >> 5)] = d * qs;
        }
      }
      __syncthreads();
    } else {
      const int n = blockIdx.x * 8 + warp;
      if (n < a.N) {
        float v = mixed_row_dot(t0, n, a.K, xq, xd, xs) * a.alpha;
        if (a.gate_logit) v *= 1.f / (1.f + __expf(-a.gate_logit[(int64_t)b * a.gate_stride]));
        if constexpr (EPI == EPI_PUSH) {
          // row-parallel projection: this rank's partial to every rank (lanes spread the peers)
          const uint32_t flag = (uint32_t)*a.push_epoch;
          for (int p = lane; p < a.push_n; p += 32) ll_store(a.push_recv[p] + (int64_t)b * a.N + n, __float_as_uint(v), flag);
        } else if (lane == 0) {
          float* y = a.y + (int64_t)b * a.y_stride + n;
          if constexpr (EPI == EPI_RESID) *y += v;
          else *y = v;
          if constexpr (EPI == EPI_STORE) {
            if (a.argmax_slots)
              atomicMax(a.argmax_slots + (int64_t)b * kArgmaxSlots + (n % kArgmaxSlots),
                        argmax_key(v, (int)(n + a.argmax_offset)));
          }
        }
      }
    }
  }
  pdl_launch();
}

void mixed_gemv_launch(int epi, const MixedGemvArgs& a, cudaStream_t s, bool pdl) {
  if (a.K % 32) throw std::runtime_error("mixed gemv: K must be a multiple of 32");
  if (epi == EPI_SWIGLU_Q8) {
    if (a.N % 32) throw std::runtime_error("mixed gemv swiglu: N must be a multiple of 32");
    launch(mixed_gemv_kernel<EPI_SWIGLU_Q8>, dim3(a.N / 32), dim3(256), 0, s, pdl, a);
  } else if (epi == EPI_RESID) {
    launch(mixed_gemv_kernel<EPI_RESID>, dim3((a.N + 7) / 8), dim3(256), 0, s, pdl, a);
  } else if (epi == EPI_PUSH) {
    if (!a.push_recv || !a.push_epoch || a.push_n <= 0 || a.nb > 8) throw std::runtime_error("mixed gemv push: peer tables, <= 8 rows");
    launch(mixed_gemv_kernel<EPI_PUSH>, dim3((a.N + 7) / 8), dim3(256), 0, s, pdl, a);
  } else {
    launch(mixed_gemv_kernel<EPI_STORE>, dim3((a.N + 7) / 8), dim3(256), 0, s, pdl, a);
  }
}

// ---- routed experts ----------------------------------------------------------------------------
// Table slot of global expert e: e itself, or under expert parallelism its local index (the
// shared expert, global id E, follows the local experts).
__device__ __forceinline__ int moe_desc_index(const MoeMixedArgs& a, int e) {
  if (a.e_count == 0) return e;
  const int l = e - a.e_lo;
  return (l >= 0 && l < a.e_count) ? l : a.e_count;
}

// Weight of sorted pair `pair` of token `tok`: its route weight, or the shared expert's gate.
__device__ __forceinline__ float moe_pair_weight(const MoeMixedArgs& a, int pair, int tok) {
  if (pair < a.routed_pairs) return a.route_w[pair];
  return a.shared_gate ? 1.f / (1.f + __expf(-a.shared_gate[(int64_t)tok * a.shared_gate_stride])) : 1.f;
}

// Grid (row blocks, active experts): blockIdx.y indexes a.active (experts with >= 1 pair).
template <int EPI>
__global__ void __launch_bounds__(256) moe_mixed_gemv_kernel(MoeMixedArgs a) {
  __shared__ float hbuf[8][8][4];
  pdl_wait();
  const int na = *a.n_active;
  if ((int)blockIdx.y >= na) { pdl_launch(); return; }
  const int e = a.active[blockIdx.y];
  const int c = a.counts[e], off = a.offsets[e];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int di = moe_desc_index(a, e);
  const MixedDesc tg = a.desc[a.desc_base0 + di];
  const MixedDesc tu = EPI == 0 ? a.desc[a.desc_base1 + di] : tg;
  for (int p = 0; p < c; ++p) {
    const int sp = off + p;  // sorted pair index
    const int8_t* xq = a.xq + (int64_t)sp * a.K;
    const float* xd = a.xd + (int64_t)sp * (a.K / 32);
    const float* xs = a.xs + (int64_t)sp * (a.K / 32);
    if (EPI == 0 && a.direct) {  // the pair's token row, no gathered copy
      const int pair = a.sorted[sp];
      const int tok = pair < a.routed_pairs ? pair / a.k : pair - a.routed_pairs;
      xq = a.xq + (int64_t)tok * a.x_stride_q;
      xd = a.xd + (int64_t)tok * a.x_stride_s;
      xs = a.xs + (int64_t)tok * a.x_stride_s;
    }
    if constexpr (EPI == 0) {
#pragma unroll 1
      for (int r = 0; r < 4; ++r) {
        const int n = blockIdx.x * 32 + warp * 4 + r;
        const float g = mixed_row_dot(tg, n, a.K, xq, xd, xs);
        const float u = mixed_row_dot(tu, n, a.K, xq, xd, xs);
        if (lane == 0) hbuf[warp][r][0] = g / (1.f + __expf(-g)) * u;
      }
      __syncthreads();
      if (warp == 0) {
        const int n = blockIdx.x * 32 + lane;
        const float v = hbuf[lane >> 2][lane & 3][0];
        const float amax = warp_max(fabsf(v));
        const float d = amax / 127.f;
        const int q = amax > 0.f ? __float2int_rn(v / d) : 0;
        const float qs = warp_sum((float)q);
        a.oq[(int64_t)sp * a.N + n] = (int8_t)q;
        if (lane == 0) {
          a.od[(int64_t)sp * (a.N / 32) + (n >> 5)] = d;
          a.os[(int64_t)sp * (a.N / 32) + (n >> 5)] = d * qs;
        }
      }
      __syncthreads();
    } else {
      const int n = blockIdx.x * 8 + warp;
      const float v = mixed_row_dot(tg, n, a.K, xq, xd, xs);
      if (lane == 0) {
        const int pair = a.sorted[sp];
        const bool routed = pair < a.routed_pairs;
        const int tok = routed ? pair / a.k : pair - a.routed_pairs;
        atomicAdd(a.y + (int64_t)tok * a.y_stride + n, moe_pair_weight(a, pair, tok) * v);
      }
    }
  }
  pdl_launch();
}

// Expert-parallel combine (K4): the down projection of this rank's active experts for every
// token, summed per token in registers (lane t of a warp holds token t) over the experts in
// active-list order and their pairs in token order, then pushed to every rank's receive region as
// flagged words: the combine IS this rank's contribution to the layer's all-reduce, and the next
// RMSNorm (tp_allreduce_rmsnorm_q8) adds the ranks' contributions into the residual. One warp per
// hidden row, no atomics, no partial buffer. Tokens were never dispatched: the hidden state is
// replicated on every rank by the attention all-reduce, so each rank reads its pairs' rows locally.
__global__ void __launch_bounds__(256) moe_mixed_combine_push_kernel(MoeMixedArgs a) {
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + warp;
  const int na = *a.n_active;
  float acc = 0.f;
  for (int i = 0; i < na; ++i) {
    const int e = a.active[i];
    const int c = a.counts[e], off = a.offsets[e];
    const MixedDesc t = a.desc[a.desc_base0 + moe_desc_index(a, e)];
    for (int p = 0; p < c; ++p) {
      const int sp = off + p;
      const float v = mixed_row_dot(t, n, a.K, a.xq + (int64_t)sp * a.K, a.xd + (int64_t)sp * (a.K / 32),
                                    a.xs + (int64_t)sp * (a.K / 32));
      const int pair = a.sorted[sp];
      const bool routed = pair < a.routed_pairs;
      const int tok = routed ? pair / a.k : pair - a.routed_pairs;
      if (lane == tok) acc += moe_pair_weight(a, pair, tok) * v;
    }
  }
  pdl_launch();
  if (lane < a.T) {
    const uint32_t flag = (uint32_t)*a.push_epoch;
    for (int p = 0; p < a.push_n; ++p) ll_store(a.push_recv[p] + (int64_t)lane * a.N + n, __float_as_uint(acc), flag);
  }
}

void moe_mixed_gemv_launch(int epi, const MoeMixedArgs& a, int max_active, cudaStream_t s, bool pdl) {
  if (a.K % 32) throw std::runtime_error("moe mixed gemv: K must be a multiple of 32");
  if (epi == 2) {
    if (a.N % 8) throw std::runtime_error("moe combine push: hidden must be a multiple of 8");
    if (!a.push_recv || !a.push_epoch || a.push_n <= 0 || a.T < 1 || a.T > 8)
      throw std::runtime_error("moe combine push: peer tables and 1..8 tokens required");
    launch(moe_mixed_combine_push_kernel, dim3(a.N / 8), dim3(256), 0, s, pdl, a);
    return;
  }
  if (epi == 0) {
    if (a.N % 32) throw std::runtime_error("moe mixed gemv: expert FFN width must be a multiple of 32");
    launch(moe_mixed_gemv_kernel<0>, dim3(a.N / 32, max_active), dim3(256), 0, s, pdl, a);
  } else {
    if (a.N % 8) throw std::runtime_error("moe mixed gemv: hidden must be a multiple of 8");
    launch(moe_mixed_gemv_kernel<1>, dim3(a.N / 8, max_active), dim3(256), 0, s, pdl, a);
  }
}

// Compact list of experts with at least one routed pair (for the expert grid's y dimension).
__global__ void moe_active_kernel(const int* counts, int E, int* active, int* n_active) {
  pdl_wait();
  __shared__ int n;
  if (threadIdx.x == 0) n = 0;
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    if (counts[e] > 0) {
      const int slot = atomicAdd(&n, 1);
      active[slot] = e;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *n_active = n;
  pdl_launch();
}

// ---- HGRAVR02 outlier residual (the binary base runs on the mixed GEMV) -----------------------
// y[b, n] += s * sum_j sign_j * x[b, col_j] over the outliers j of row n (CSR built at load from the
// Rice-coded flat indices). One warp per output row, lanes over the row's outliers in a fixed
// order, a fixed warp reduction: deterministic. x is the q8 activation blocks of the GEMV.
__global__ void __launch_bounds__(256) sparse_residual_kernel(const int* row_ptr, const int* cols,
                                                              const int8_t* signs, float s, int N, const int8_t* xq,
                                                              const float* xd, int K, int nb, float* y,
                                                              int64_t y_stride) {
  pdl_wait();
  const int n = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (n < N) {
    const int j0 = row_ptr[n], j1 = row_ptr[n + 1];
    float acc[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) acc[b] = 0.f;
    for (int j = j0 + lane; j < j1; j += 32) {
      const int c = cols[j];
      const float sg = (float)signs[j];
#pragma unroll
      for (int b = 0; b < 8; ++b)
        if (b < nb) acc[b] += sg * (float)xq[(int64_t)b * K + c] * xd[(int64_t)b * (K / 32) + c / 32];
    }
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      if (b >= nb) break;
      const float v = warp_sum(acc[b]);
      if (lane == 0) y[(int64_t)b * y_stride + n] += s * v;
    }
  }
  pdl_launch();
}

void sparse_residual_launch(const int* row_ptr, const int* cols, const int8_t* signs, float scale, int N,
                            const int8_t* xq, const float* xd, int K, int nb, float* y, int64_t y_stride,
                            cudaStream_t s, bool pdl) {
  if (nb < 1 || nb > 8 || K % 32) throw std::runtime_error("sparse_residual: 1..8 rows, K % 32 == 0");
  launch(sparse_residual_kernel, dim3((unsigned)((N + 7) / 8)), dim3(256), 0, s, pdl, row_ptr, cols, signs, scale, N,
         xq, xd, K, nb, y, y_stride);
}

void moe_active_launch(const int* counts, int E, int* active, int* n_active, cudaStream_t s, bool pdl) {
  launch(moe_active_kernel, dim3(1), dim3(512), 0, s, pdl, counts, E, active, n_active);
}

}  // namespace hk
