// Prefill of the mixed-codec MoE models on the tensor cores (many rows per forward).
//
// A prefill forward of T tokens routes T * k (token, expert) pairs. Instead of one GEMV pass per
// pair, every expert's weights are decoded once per forward into a bf16 copy (the table kinds:
// binary / uniform group codes, fp8 with block scales, Q4_K planes) and the experts run as one
// grouped tcgen05 GEMM over the pairs sorted by expert (gemm_tc.cu, bf16-weight mode):
//   1. mixed_dequant_bf16: descriptor list -> bf16 rows (experts stacked, [gate | up] per expert);
//   2. moe_tiles: the (expert, first row, end row) tiles of BN pairs from the counting sort;
//   3. moe_gather_bf16: token rows -> pair rows in sorted order;
//   4. grouped GEMM gate | up with the SwiGLU epilogue -> h (bf16), grouped GEMM down -> fp32;
//   5. moe_combine: per token, in pair order, x += sum_j w_j y[pos(t, j)] (+ the gated shared
//      expert), deterministic (no atomics).
// Also q8_to_bf16 (int8 activation blocks back to bf16 rows for the dense projections' GEMMs).
//
// Parity: crates/hawking-core/shaders/moe.metal moe_batched_gemm_*_indexed (batched experts over
// the routed token lists), crates/hawking-core/src/model/deepseek_v2.rs:2276
// (forward_tokens_batched_tcb).
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "api.h"
#include "qformats.cuh"

namespace hk {

// Value i (0..31) of 32-element block `blk` of row `row` of tensor `t`.
__device__ __forceinline__ void mixed_block_values(const MixedDesc& t, int64_t row, int blk, float (&v)[32]) {
  const uint8_t* codes = t.codes + row * t.code_row_bytes;
  if (t.kind == MIXED_FP8) {
    const float sw = t.scales_f32[row * t.scale_row_elems + (blk * 32) / t.group];
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const uint16_t pr = *reinterpret_cast<const uint16_t*>(codes + blk * 32 + i);
      const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)pr, __NV_E4M3);
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
      v[i] = f.x * sw;
      v[i + 1] = f.y * sw;
    }
    return;
  }
  if (t.kind == MIXED_FP4) {
    const float sw = t.scales_f32[row * t.scale_row_elems + blk];
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const uint32_t b = codes[blk * 16 + i / 2];
      v[i] = e2m1_value(b & 0xFu) * sw;
      v[i + 1] = e2m1_value(b >> 4) * sw;
    }
    return;
  }
  if (t.kind == MIXED_Q4K) {
    const int sb = blk >> 3, j = blk & 7;
    const uint4 h = *(reinterpret_cast<const uint4*>(t.scales + row * t.scale_row_elems) + sb);
    int sc, mn;
    q4k_scale_min(j, h.y, h.z, h.w, sc, mn);
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    const uint8_t* q = codes + sb * 128 + (j >> 1) * 32;
    const int sh = (j & 1) * 4;
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = d * (float)sc * (float)((q[i] >> sh) & 0xF) - dmin * (float)mn;
    return;
  }
  const float sg = __half2float(t.scales[row * t.scale_row_elems + (blk * 32) / t.group]);
  if (t.kind == MIXED_BINARY) {
    const uint32_t b = *reinterpret_cast<const uint32_t*>(codes + blk * 4);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = ((b >> i) & 1u) ? sg : -sg;
    return;
  }
  const int bits = t.bits;
  const uint8_t* c = codes + (int64_t)blk * 32 * bits / 8;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int bit = i * bits;
    const uint32_t code = (c[bit >> 3] >> (bit & 7)) & ((1u << bits) - 1u);
    v[i] = ((float)code - (float)t.bound) * sg;
  }
}

// grid (rows, count): descriptor didx[g], row r -> out row drow[g] + r.
__global__ void __launch_bounds__(128) mixed_dequant_bf16_kernel(const MixedDesc* desc, const int* didx,
                                                                 const int* drow, int K, __nv_bfloat16* out,
                                                                 int64_t out_stride) {
  pdl_wait();
  const int r = blockIdx.x, g = blockIdx.y;
  const MixedDesc t = desc[didx[g]];
  __nv_bfloat16* o = out + (int64_t)(drow[g] + r) * out_stride;
  for (int blk = threadIdx.x; blk < K / 32; blk += blockDim.x) {
    float v[32];
    mixed_block_values(t, r, blk, v);
    uint4* dst = reinterpret_cast<uint4*>(o + blk * 32);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      __nv_bfloat162 p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) p[e] = __floats2bfloat162_rn(v[8 * c + 2 * e], v[8 * c + 2 * e + 1]);
      dst[c] = *reinterpret_cast<uint4*>(p);
    }
  }
  pdl_launch();
}

void mixed_dequant_bf16_launch(const MixedDesc* desc, const int* didx, const int* drow, int count, int rows, int K,
                               __nv_bfloat16* out, int64_t out_stride, cudaStream_t s, bool pdl) {
  if (K % 32 || out_stride % 8) throw std::runtime_error("mixed dequant: K must be a multiple of 32, rows 16-byte aligned");
  if (count <= 0 || rows <= 0) return;
  if (count > 65535) throw std::runtime_error("mixed dequant: at most 65535 tensors per launch");
  launch(mixed_dequant_bf16_kernel, dim3(rows, count), dim3(128), 0, s, pdl, desc, didx, drow, K, out, out_stride);
}

// ---- GGUF block formats -> bf16 (the stacked expert matrices of the GGUF MoE models) -----------
// Value i (0..31) of 32-element block b of row r, from the planes of a re-laid GGUF tensor (each
// plane holds one byte range of every block; api.h WPlanes). The formulas are the GGUF formats'.
__device__ __forceinline__ void gguf_block_values(int fmt, const WPlanes& w, int64_t r, int b, float (&v)[32]) {
  if (fmt == WF_Q8_0) {
    const int8_t* q = reinterpret_cast<const int8_t*>(w.p0 + r * w.rb0 + (int64_t)b * 32);
    const float d = __half2float(*reinterpret_cast<const __half*>(w.p1 + r * w.rb1 + (int64_t)b * 2));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = d * (float)q[i];
  } else if (fmt == WF_Q4_0 || fmt == WF_Q5_0) {
    const uint8_t* q = w.p0 + r * w.rb0 + (int64_t)b * 16;
    const float d = __half2float(*reinterpret_cast<const __half*>(w.p1 + r * w.rb1 + (int64_t)b * 2));
    uint32_t qh = 0;
    if (fmt == WF_Q5_0) {
      const uint8_t* h = w.p2 + r * w.rb2 + (int64_t)b * 4;
      qh = (uint32_t)h[0] | ((uint32_t)h[1] << 8) | ((uint32_t)h[2] << 16) | ((uint32_t)h[3] << 24);
    }
    const int off = fmt == WF_Q5_0 ? 16 : 8;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      int n = i < 16 ? (q[i] & 0xF) : (q[i - 16] >> 4);
      if (fmt == WF_Q5_0) n |= ((qh >> i) & 1u) << 4;
      v[i] = d * (float)(n - off);
    }
  } else if (fmt == WF_Q4_K) {
    const int sb = b >> 3, j = b & 7;
    const uint4 h = *reinterpret_cast<const uint4*>(w.p1 + r * w.rb1 + (int64_t)sb * 16);
    int sc, mn;
    q4k_scale_min(j, h.y, h.z, h.w, sc, mn);
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    const uint8_t* q = w.p0 + r * w.rb0 + (int64_t)sb * 128 + (j >> 1) * 32;
    const int sh = (j & 1) * 4;
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = d * (float)sc * (float)((q[i] >> sh) & 0xF) - dmin * (float)mn;
  } else {  // Q6_K: 32-element quarter qd of half n of super-block sb
    const int sb = b >> 3, j = b & 7, n = j >> 2, qd = j & 3;
    const uint8_t* ql = w.p0 + r * w.rb0 + (int64_t)sb * 128 + 64 * n + (qd & 1) * 32;
    const uint8_t* qh = w.p1 + r * w.rb1 + (int64_t)sb * 64 + 32 * n;
    const int8_t* sc = reinterpret_cast<const int8_t*>(w.p2 + r * w.rb2 + (int64_t)sb * 16 + 8 * n);
    const float d = __half2float(*reinterpret_cast<const __half*>(w.p3 + r * w.rb3 + (int64_t)sb * 2));
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const int nib = qd < 2 ? (ql[l] & 0xF) : (ql[l] >> 4);
      const int q = (nib | (((qh[l] >> (2 * qd)) & 3) << 4)) - 32;
      v[l] = d * (float)sc[l / 16 + 2 * qd] * (float)q;
    }
  }
}

// grid (rows): source row r of a stacked [groups * group_rows, K] tensor -> out row
// (r / group_rows) * dst_group_rows + dst_off + r % group_rows.
__global__ void __launch_bounds__(128) qweight_dequant_bf16_kernel(int fmt, WPlanes w, int K, int group_rows,
                                                                   int dst_group_rows, int dst_off,
                                                                   __nv_bfloat16* out, int64_t out_stride) {
  pdl_wait();
  const int r = blockIdx.x;
  const int64_t dr = (int64_t)(r / group_rows) * dst_group_rows + dst_off + r % group_rows;
  __nv_bfloat16* o = out + dr * out_stride;
  for (int b = threadIdx.x; b < K / 32; b += blockDim.x) {
    float v[32];
    gguf_block_values(fmt, w, r, b, v);
    uint4* dst = reinterpret_cast<uint4*>(o + b * 32);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      __nv_bfloat162 p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) p[e] = __floats2bfloat162_rn(v[8 * c + 2 * e], v[8 * c + 2 * e + 1]);
      dst[c] = *reinterpret_cast<uint4*>(p);
    }
  }
  pdl_launch();
}

void qweight_dequant_bf16_launch(int fmt, const WPlanes& w, int rows, int K, int group_rows, int dst_group_rows,
                                 int dst_off, __nv_bfloat16* out, int64_t out_stride, cudaStream_t s, bool pdl) {
  if (fmt != WF_Q8_0 && fmt != WF_Q4_0 && fmt != WF_Q5_0 && fmt != WF_Q4_K && fmt != WF_Q6_K)
    throw std::runtime_error("qweight dequant: Q8_0, Q4_0, Q5_0, Q4_K or Q6_K");
  if (K % ((fmt == WF_Q4_K || fmt == WF_Q6_K) ? 256 : 32) || out_stride % 8)
    throw std::runtime_error("qweight dequant: K must be whole blocks, rows 16-byte aligned");
  if (rows <= 0) return;
  launch(qweight_dequant_bf16_kernel, dim3(rows), dim3(128), 0, s, pdl, fmt, w, K, group_rows, dst_group_rows,
         dst_off, out, out_stride);
}

// Tiles of bn pairs per expert from the counting sort (one CTA; E1 <= 1024).
// Under expert parallelism only this rank's experts [e_lo, e_hi) (e_hi = 0: all) and the folded
// shared expert (shared_e, -1: none) get tiles.
__global__ void __launch_bounds__(1024) moe_tiles_kernel(const int* counts, const int* offsets, int E1, int bn,
                                                         int* tiles, int* n_tiles, int e_lo, int e_hi,
                                                         int shared_e) {
  __shared__ int pre[1025];
  pdl_wait();
  const int e = threadIdx.x;
  const bool mine = e_hi == 0 || (e >= e_lo && e < e_hi) || e == shared_e;
  const int c = (e < E1 && mine) ? counts[e] : 0;
  const int nt = (c + bn - 1) / bn;
  pre[e + 1] = nt;
  if (e == 0) pre[0] = 0;
  __syncthreads();
  for (int st = 1; st < 1024; st <<= 1) {  // inclusive scan of the tile counts
    const int add = e + 1 > st ? pre[e + 1 - st] : 0;
    __syncthreads();
    pre[e + 1] += add;
    __syncthreads();
  }
  if (e < E1) {
    const int off = offsets[e];
    for (int j = 0; j < nt; ++j) {
      int* t = tiles + 3 * (pre[e] + j);
      t[0] = e;
      t[1] = off + j * bn;
      t[2] = min(off + c, off + (j + 1) * bn);
    }
  }
  if (e == 0) *n_tiles = pre[1024];
  pdl_launch();
}

void moe_tiles_launch(const int* counts, const int* offsets, int E1, int bn, int* tiles, int* n_tiles, int e_lo,
                      int e_hi, int shared_e, cudaStream_t s, bool pdl) {
  if (E1 > 1024) throw std::runtime_error("moe tiles: at most 1024 experts");
  launch(moe_tiles_kernel, dim3(1), dim3(1024), 0, s, pdl, counts, offsets, E1, bn, tiles, n_tiles, e_lo, e_hi,
         shared_e);
}

// Pair rows in sorted order (pairs below P are routed: token pair / k; the rest shared: pair - P),
// plus pos[pair] = sorted position.
__global__ void __launch_bounds__(256) moe_gather_bf16_kernel(const int* sorted, int PS, int P, int k,
                                                              const __nv_bfloat16* x, int64_t x_stride, int K,
                                                              __nv_bfloat16* xg, int64_t xg_stride, int* pos) {
  pdl_wait();
  const int sp = blockIdx.x;
  const int pr = sorted[sp];
  const int tok = pr < P ? pr / k : pr - P;
  if (threadIdx.x == 0) pos[pr] = sp;
  const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)tok * x_stride);
  uint4* dst = reinterpret_cast<uint4*>(xg + (int64_t)sp * xg_stride);
  for (int i = threadIdx.x; i < K / 8; i += blockDim.x) dst[i] = src[i];
  pdl_launch();
}

void moe_gather_bf16_launch(const int* sorted, int PS, int P, int k, const __nv_bfloat16* x, int64_t x_stride, int K,
                            __nv_bfloat16* xg, int64_t xg_stride, int* pos, cudaStream_t s, bool pdl) {
  if (K % 8 || x_stride % 8 || xg_stride % 8) throw std::runtime_error("moe gather: 16-byte aligned rows");
  if (PS <= 0) return;
  launch(moe_gather_bf16_kernel, dim3(PS), dim3(256), 0, s, pdl, sorted, PS, P, k, x, x_stride, K, xg, xg_stride, pos);
}

// x[t] += sum_j w[t k + j] y[pos[t k + j]] (+ g(t) y[pos[P + t]] with a shared expert: g = 1, or
// sigmoid of the shared-gate logit).
// Under expert parallelism (ids given, e_hi > 0) only the pairs of this rank's experts [e_lo, e_hi)
// were computed; the others are skipped.
__global__ void __launch_bounds__(256) moe_combine_kernel(const float* y, int64_t y_stride, const int* pos,
                                                          const float* w, int T, int k, int shared,
                                                          const float* shared_gate, int64_t gate_stride, float* x,
                                                          int64_t x_stride, int H, const int* ids, int e_lo,
                                                          int e_hi) {
  pdl_wait();
  const int t = blockIdx.y;
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n < H) {
    float acc = 0.f;
    for (int j = 0; j < k; ++j) {
      if (ids && e_hi > 0) {
        const int e = ids[t * k + j];
        if (e < e_lo || e >= e_hi) continue;
      }
      acc += w[t * k + j] * y[(int64_t)pos[t * k + j] * y_stride + n];
    }
    if (shared) {
      const float g = shared_gate ? 1.f / (1.f + __expf(-shared_gate[(int64_t)t * gate_stride])) : 1.f;
      acc += g * y[(int64_t)pos[T * k + t] * y_stride + n];
    }
    x[(int64_t)t * x_stride + n] += acc;
  }
  pdl_launch();
}

void moe_combine_launch(const float* y, int64_t y_stride, const int* pos, const float* w, int T, int k, bool shared,
                        const float* shared_gate, int64_t gate_stride, float* x, int64_t x_stride, int H,
                        const int* ids, int e_lo, int e_hi, cudaStream_t s, bool pdl) {
  if (T <= 0) return;
  launch(moe_combine_kernel, dim3((H + 255) / 256, T), dim3(256), 0, s, pdl, y, y_stride, pos, w, T, k,
         shared ? 1 : 0, shared_gate, gate_stride, x, x_stride, H, ids, e_lo, e_hi);
}

// int8 activation blocks (q, d per 32) -> bf16 rows.
__global__ void __launch_bounds__(256) q8_to_bf16_kernel(const int8_t* q, const float* d, int64_t q_stride,
                                                         int64_t d_stride, int K, __nv_bfloat16* out,
                                                         int64_t out_stride) {
  pdl_wait();
  const int r = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // pair of elements
  if (2 * i < K) {
    const float s = d[(int64_t)r * d_stride + (2 * i) / 32];
    const int8_t* qr = q + (int64_t)r * q_stride;
    reinterpret_cast<__nv_bfloat162*>(out + (int64_t)r * out_stride)[i] =
        __floats2bfloat162_rn((float)qr[2 * i] * s, (float)qr[2 * i + 1] * s);
  }
  pdl_launch();
}

void q8_to_bf16_launch(const int8_t* q, const float* d, int64_t q_stride, int64_t d_stride, int rows, int K,
                       __nv_bfloat16* out, int64_t out_stride, cudaStream_t s, bool pdl) {
  if (K % 32 || out_stride % 2) throw std::runtime_error("q8_to_bf16: K must be a multiple of 32");
  if (rows <= 0) return;
  launch(q8_to_bf16_kernel, dim3((K / 2 + 255) / 256, rows), dim3(256), 0, s, pdl, q, d, q_stride, d_stride, K, out,
         out_stride);
}

}  // namespace hk
