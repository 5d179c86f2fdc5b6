// Device-side GGML block decoders for the W4A8/W8A8 dp4a GEMV.
//
// Weight storage on the GPU (lossless re-layouts of the GGUF bytes, done once at load):
//   Q4_K : raw 144-byte super-blocks (16-byte aligned already) — [N, K/256, 144]
//   Q6_K : raw 210-byte super-blocks re-packed as planes: ql [N,K/2], qh [N,K/4], sc i8 [N,K/16],
//          d f16 [N,K/256]
//   Q4_0 : planes qs [N, K/2] (the 16 block bytes, unchanged order) + d f16 [N, K/32]
//   Q5_0 : planes qs [N, K/2], qh u32 [N, K/32], d f16 [N, K/32]
//   Q8_0 : planes qs i8 [N, K] + d f16 [N, K/32]
// The math of each decode is the GGUF formula (oracle: crates/hawking-core/src/quant.rs:34-160
// and gemv_q4_k_q8k :722, which is exactly this W4A8 dot with an int8 activation block).
//
// Activations are int8 blocks of 32 ("q8 activations"): q [K] i8, d [K/32] f32 (scale) and
// s [K/32] f32 (= d * sum(q)), so a block dot is d_w * (d_x * sum(qw*qx)) with offsets folded
// through s.
#pragma once
#include "common.cuh"
#include "api.h"

namespace hk {

// fp4 e2m1 code (sign | 2 exponent bits | 1 mantissa bit, exponent bias 1) as fp32, built from its
// bits: exponent 0 is the subnormal m * 0.5, otherwise 2^(e - 1) * (1 + m / 2); the magnitudes
// are 0, 0.5, 1, 1.5, 2, 3, 4, 6.
__device__ __forceinline__ float e2m1_value(uint32_t c) {
  const uint32_t e = (c >> 1) & 3u, m = c & 1u;
  const uint32_t mag = e ? (((e + 126u) << 23) | (m << 22)) : (m ? (126u << 23) : 0u);
  return __uint_as_float(mag | ((c & 8u) << 28));
}



// Activation loads use generic addressing: the q8 input may live in global or shared memory.
__device__ __forceinline__ int4 ldx16(const int8_t* p) { return *reinterpret_cast<const int4*>(p); }
__device__ __forceinline__ float ldxf(const float* p) { return *p; }

// Shared-memory swizzle of the q8 activation bytes, in 16-byte granules. With the chunk mapping,
// lane L reads granule g of chunk c = L + 32 i, so 8 consecutive lanes (one phase of a 16-byte
// shared load) read granules 4 (or 2) apart and hit the same banks. Permuting the granules of a
// chunk by bits of the chunk index spreads those 8 reads over all 32 banks:
//   GPC = 4 (64-byte chunks, Q4_K): granule g of chunk c is stored at g ^ ((c >> 1) & 3)
//   GPC = 2 (32-byte chunks, Q8_0 / Q4_0): granule g of chunk c is stored at g ^ ((c >> 2) & 1)
// The permutation stays inside each aligned group of 4 (or 2) granules, so it is a bijection on
// any K that is a multiple of 64. GPC = 0 is the identity (global activations, unit formats).
template <int GPC>
__device__ __forceinline__ int swz_granule(int G) {
  if constexpr (GPC == 4) return G ^ ((G >> 3) & 3);
  else if constexpr (GPC == 2) return G ^ ((G >> 3) & 1);
  else return G;
}
template <int GPC>
__device__ __forceinline__ int4 ldx_granule(const int8_t* xq, int G) {
  return ldx16(xq + 16 * swz_granule<GPC>(G));
}

// Q4_K/Q5_K six-bit scale & min of sub-block j (0..7) from the 12 scale bytes packed in 3 words.
__device__ __forceinline__ void q4k_scale_min(int j, uint32_t s0, uint32_t s1, uint32_t s2, int& sc, int& mn) {
  auto B = [&](int i) -> int {
    uint32_t w = i < 4 ? s0 : (i < 8 ? s1 : s2);
    return (w >> (8 * (i & 3))) & 0xFF;
  };
  if (j < 4) {
    sc = B(j) & 63;
    mn = B(j + 4) & 63;
  } else {
    sc = (B(j + 4) & 0xF) | ((B(j - 4) >> 6) << 4);
    mn = (B(j + 4) >> 4) | ((B(j) >> 6) << 4);
  }
}

// ---- Q4_K planes ------------------------------------------------------------------------------
// p0 = quants [N, K/2] (the 128 quant bytes of every super-block, in order), p1 = headers
// [N, K/256 * 16] (d, dmin, 12 packed scale bytes). Together exactly the GGUF block bytes.
//
// Unit (legacy per-lane mapping, used by the grouped MoE GEMV): half a super-block, 128 elements.
struct UnitQ4K {
  uint4 hdr;   // d, dmin, scales[12]
  uint4 q[4];  // 64 bytes of qs for this half
};
__device__ __forceinline__ void load_unit_q4k(const WPlanes& w, int64_t row, int u, UnitQ4K& r) {
  r.hdr = __ldg(reinterpret_cast<const uint4*>(w.p1 + row * w.rb1 + (int64_t)(u >> 1) * 16));
  const uint8_t* qs = w.p0 + row * w.rb0 + (int64_t)u * 64;
#pragma unroll
  for (int i = 0; i < 4; ++i) r.q[i] = ldg_stream(qs + 16 * i);
}
__device__ __forceinline__ float dot_unit_q4k(const UnitQ4K& r, int u, const int8_t* xq, const float* xd,
                                              const float* xs) {
  const float d = __half2float(__ushort_as_half((uint16_t)(r.hdr.x & 0xFFFF)));
  const float dmin = __half2float(__ushort_as_half((uint16_t)(r.hdr.x >> 16)));
  const int h = u & 1;
  const int k0 = u * 128;
  float acc = 0.f;
#pragma unroll
  for (int t = 0; t < 4; ++t) {  // sub-block 4h+t
    int sc, mn;
    q4k_scale_min(4 * h + t, r.hdr.y, r.hdr.z, r.hdr.w, sc, mn);
    const uint4 qa = r.q[(t >> 1) * 2], qb = r.q[(t >> 1) * 2 + 1];
    const int shift = (t & 1) * 4;
    const int4 x0 = ldx16(xq + k0 + 32 * t), x1 = ldx16(xq + k0 + 32 * t + 16);
    int dot = 0;
    dot = dp4a((qa.x >> shift) & 0x0F0F0F0F, x0.x, dot);
    dot = dp4a((qa.y >> shift) & 0x0F0F0F0F, x0.y, dot);
    dot = dp4a((qa.z >> shift) & 0x0F0F0F0F, x0.z, dot);
    dot = dp4a((qa.w >> shift) & 0x0F0F0F0F, x0.w, dot);
    dot = dp4a((qb.x >> shift) & 0x0F0F0F0F, x1.x, dot);
    dot = dp4a((qb.y >> shift) & 0x0F0F0F0F, x1.y, dot);
    dot = dp4a((qb.z >> shift) & 0x0F0F0F0F, x1.z, dot);
    dot = dp4a((qb.w >> shift) & 0x0F0F0F0F, x1.w, dot);
    const int blk = (k0 >> 5) + t;
    acc += d * (float)sc * ldxf(xd + blk) * (float)dot - dmin * (float)mn * ldxf(xs + blk);
  }
  return acc;
}

// Chunk (coalesced mapping used by the decode GEMV): 64 elements = sub-blocks 2q, 2q+1 of
// super-block c/4 (q = c % 4), i.e. 32 contiguous quant bytes; lane L owns chunks L + 32 i so a
// warp's loads cover contiguous 1 KB spans of the quant plane.
struct ChunkQ4K {
  uint4 q0, q1;
  uint4 hdr;
};
__device__ __forceinline__ void load_chunk_q4k(const WPlanes& w, int64_t row, int c, ChunkQ4K& r) {
  const uint8_t* qs = w.p0 + row * w.rb0 + (int64_t)c * 32;
  r.q0 = ldg_stream(qs);
  r.q1 = ldg_stream(qs + 16);
  r.hdr = __ldg(reinterpret_cast<const uint4*>(w.p1 + row * w.rb1 + (int64_t)(c >> 2) * 16));
}
template <int GPC = 0>
__device__ __forceinline__ float dot_chunk_q4k(const ChunkQ4K& r, int c, const int8_t* xq, const float* xd,
                                               const float* xs) {
  const float d = __half2float(__ushort_as_half((uint16_t)(r.hdr.x & 0xFFFF)));
  const float dmin = __half2float(__ushort_as_half((uint16_t)(r.hdr.x >> 16)));
  const int q = c & 3, sh = 8 * ((2 * q) & 3);  // byte lane of sub-block j0 = 2q inside its word
  // scales of j0 = 2q and j1 = 2q+1 (both < 4 or both >= 4)
  const uint32_t lo_sc = r.hdr.y, lo_mn = r.hdr.z, hi = r.hdr.w;
  int sc0, mn0, sc1, mn1;
  {
    const int b0 = (lo_sc >> sh) & 0xFF, b1 = (lo_sc >> (sh + 8)) & 0xFF;
    const int m0 = (lo_mn >> sh) & 0xFF, m1 = (lo_mn >> (sh + 8)) & 0xFF;
    const int h0 = (hi >> sh) & 0xFF, h1 = (hi >> (sh + 8)) & 0xFF;
    if (q < 2) {
      sc0 = b0 & 63; mn0 = m0 & 63; sc1 = b1 & 63; mn1 = m1 & 63;
    } else {
      sc0 = (h0 & 0xF) | ((b0 >> 6) << 4); mn0 = (h0 >> 4) | ((m0 >> 6) << 4);
      sc1 = (h1 & 0xF) | ((b1 >> 6) << 4); mn1 = (h1 >> 4) | ((m1 >> 6) << 4);
    }
  }
  const int k0 = c * 64;
  const int4 xa = ldx_granule<GPC>(xq, 4 * c), xb = ldx_granule<GPC>(xq, 4 * c + 1);
  const int4 xc = ldx_granule<GPC>(xq, 4 * c + 2), xe = ldx_granule<GPC>(xq, 4 * c + 3);
  int d0 = 0, d1 = 0;
  d0 = dp4a(r.q0.x & 0x0F0F0F0F, xa.x, d0); d1 = dp4a((r.q0.x >> 4) & 0x0F0F0F0F, xc.x, d1);
  d0 = dp4a(r.q0.y & 0x0F0F0F0F, xa.y, d0); d1 = dp4a((r.q0.y >> 4) & 0x0F0F0F0F, xc.y, d1);
  d0 = dp4a(r.q0.z & 0x0F0F0F0F, xa.z, d0); d1 = dp4a((r.q0.z >> 4) & 0x0F0F0F0F, xc.z, d1);
  d0 = dp4a(r.q0.w & 0x0F0F0F0F, xa.w, d0); d1 = dp4a((r.q0.w >> 4) & 0x0F0F0F0F, xc.w, d1);
  d0 = dp4a(r.q1.x & 0x0F0F0F0F, xb.x, d0); d1 = dp4a((r.q1.x >> 4) & 0x0F0F0F0F, xe.x, d1);
  d0 = dp4a(r.q1.y & 0x0F0F0F0F, xb.y, d0); d1 = dp4a((r.q1.y >> 4) & 0x0F0F0F0F, xe.y, d1);
  d0 = dp4a(r.q1.z & 0x0F0F0F0F, xb.z, d0); d1 = dp4a((r.q1.z >> 4) & 0x0F0F0F0F, xe.z, d1);
  d0 = dp4a(r.q1.w & 0x0F0F0F0F, xb.w, d0); d1 = dp4a((r.q1.w >> 4) & 0x0F0F0F0F, xe.w, d1);
  const int blk = k0 >> 5;
  const float2 dx = *reinterpret_cast<const float2*>(xd + blk);
  const float2 sx = *reinterpret_cast<const float2*>(xs + blk);
  return d * ((float)sc0 * dx.x * (float)d0 + (float)sc1 * dx.y * (float)d1) -
         dmin * ((float)mn0 * sx.x + (float)mn1 * sx.y);
}

// ---- Q8_0 chunk: one 32-element block (32 quant bytes + one fp16 scale) -------------------------
struct ChunkQ8_0 {
  uint4 q0, q1;
  float d;
};
__device__ __forceinline__ void load_chunk_q8_0(const WPlanes& w, int64_t row, int c, ChunkQ8_0& r) {
  const uint8_t* qs = w.p0 + row * w.rb0 + (int64_t)c * 32;
  r.q0 = ldg_stream(qs);
  r.q1 = ldg_stream(qs + 16);
  r.d = __half2float(__ldg(reinterpret_cast<const __half*>(w.p1 + row * w.rb1) + c));
}
template <int GPC = 0>
__device__ __forceinline__ float dot_chunk_q8_0(const ChunkQ8_0& r, int c, const int8_t* xq, const float* xd,
                                                const float* xs) {
  const int4 xa = ldx_granule<GPC>(xq, 2 * c), xb = ldx_granule<GPC>(xq, 2 * c + 1);
  int dot = 0;
  dot = dp4a(r.q0.x, xa.x, dot); dot = dp4a(r.q0.y, xa.y, dot);
  dot = dp4a(r.q0.z, xa.z, dot); dot = dp4a(r.q0.w, xa.w, dot);
  dot = dp4a(r.q1.x, xb.x, dot); dot = dp4a(r.q1.y, xb.y, dot);
  dot = dp4a(r.q1.z, xb.z, dot); dot = dp4a(r.q1.w, xb.w, dot);
  (void)xs;
  return r.d * ldxf(xd + c) * (float)dot;
}

// ---- Q4_0 chunk: one 32-element block (16 quant bytes + one fp16 scale) -------------------------
struct ChunkQ4_0 {
  uint4 q;
  float d;
};
__device__ __forceinline__ void load_chunk_q4_0(const WPlanes& w, int64_t row, int c, ChunkQ4_0& r) {
  r.q = ldg_stream(w.p0 + row * w.rb0 + (int64_t)c * 16);
  r.d = __half2float(__ldg(reinterpret_cast<const __half*>(w.p1 + row * w.rb1) + c));
}
template <int GPC = 0>
__device__ __forceinline__ float dot_chunk_q4_0(const ChunkQ4_0& r, int c, const int8_t* xq, const float* xd,
                                                const float* xs) {
  const int4 xa = ldx_granule<GPC>(xq, 2 * c), xb = ldx_granule<GPC>(xq, 2 * c + 1);
  int dot = 0;
  dot = dp4a(r.q.x & 0x0F0F0F0F, xa.x, dot); dot = dp4a((r.q.x >> 4) & 0x0F0F0F0F, xb.x, dot);
  dot = dp4a(r.q.y & 0x0F0F0F0F, xa.y, dot); dot = dp4a((r.q.y >> 4) & 0x0F0F0F0F, xb.y, dot);
  dot = dp4a(r.q.z & 0x0F0F0F0F, xa.z, dot); dot = dp4a((r.q.z >> 4) & 0x0F0F0F0F, xb.z, dot);
  dot = dp4a(r.q.w & 0x0F0F0F0F, xa.w, dot); dot = dp4a((r.q.w >> 4) & 0x0F0F0F0F, xb.w, dot);
  return r.d * (ldxf(xd + c) * (float)dot - 8.f * ldxf(xs + c));
}

// ---- Q4_0 planes: unit = 4 blocks (128 elements) -------------------------------------------
struct UnitQ4_0 {
  uint4 q[4];
  uint2 d;  // 4 x f16
};
__device__ __forceinline__ void load_unit_q4_0(const WPlanes& w, int64_t row, int u, UnitQ4_0& r) {
  const uint8_t* qs = w.p0 + row * w.rb0 + (int64_t)u * 64;
#pragma unroll
  for (int i = 0; i < 4; ++i) r.q[i] = ldg_stream(qs + 16 * i);
  r.d = __ldg(reinterpret_cast<const uint2*>(w.p1 + row * w.rb1 + (int64_t)u * 8));
}
__device__ __forceinline__ float dot_unit_q4_0(const UnitQ4_0& r, int u, const int8_t* xq, const float* xd,
                                               const float* xs) {
  const int k0 = u * 128;
  float acc = 0.f;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint4 q = r.q[b];
    const int4 x0 = ldx16(xq + k0 + 32 * b), x1 = ldx16(xq + k0 + 32 * b + 16);
    int dot = 0;
    dot = dp4a(q.x & 0x0F0F0F0F, x0.x, dot);
    dot = dp4a(q.y & 0x0F0F0F0F, x0.y, dot);
    dot = dp4a(q.z & 0x0F0F0F0F, x0.z, dot);
    dot = dp4a(q.w & 0x0F0F0F0F, x0.w, dot);
    dot = dp4a((q.x >> 4) & 0x0F0F0F0F, x1.x, dot);
    dot = dp4a((q.y >> 4) & 0x0F0F0F0F, x1.y, dot);
    dot = dp4a((q.z >> 4) & 0x0F0F0F0F, x1.z, dot);
    dot = dp4a((q.w >> 4) & 0x0F0F0F0F, x1.w, dot);
    const uint32_t dw = b < 2 ? r.d.x : r.d.y;
    const float dwf = __half2float(__ushort_as_half((uint16_t)(dw >> (16 * (b & 1)))));
    const int blk = (k0 >> 5) + b;
    acc += dwf * (ldxf(xd + blk) * (float)dot - 8.f * ldxf(xs + blk));
  }
  return acc;
}

// ---- Q8_0 planes: unit = 4 blocks --------------------------------------------------------------
struct UnitQ8_0 {
  uint4 q[8];
  uint2 d;
};
__device__ __forceinline__ void load_unit_q8_0(const WPlanes& w, int64_t row, int u, UnitQ8_0& r) {
  const uint8_t* qs = w.p0 + row * w.rb0 + (int64_t)u * 128;
#pragma unroll
  for (int i = 0; i < 8; ++i) r.q[i] = ldg_stream(qs + 16 * i);
  r.d = __ldg(reinterpret_cast<const uint2*>(w.p1 + row * w.rb1 + (int64_t)u * 8));
}
__device__ __forceinline__ float dot_unit_q8_0(const UnitQ8_0& r, int u, const int8_t* xq, const float* xd,
                                               const float* xs) {
  const int k0 = u * 128;
  float acc = 0.f;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint4 qa = r.q[2 * b], qb = r.q[2 * b + 1];
    const int4 x0 = ldx16(xq + k0 + 32 * b), x1 = ldx16(xq + k0 + 32 * b + 16);
    int dot = 0;
    dot = dp4a(qa.x, x0.x, dot);
    dot = dp4a(qa.y, x0.y, dot);
    dot = dp4a(qa.z, x0.z, dot);
    dot = dp4a(qa.w, x0.w, dot);
    dot = dp4a(qb.x, x1.x, dot);
    dot = dp4a(qb.y, x1.y, dot);
    dot = dp4a(qb.z, x1.z, dot);
    dot = dp4a(qb.w, x1.w, dot);
    const uint32_t dw = b < 2 ? r.d.x : r.d.y;
    const float dwf = __half2float(__ushort_as_half((uint16_t)(dw >> (16 * (b & 1)))));
    acc += dwf * ldxf(xd + (k0 >> 5) + b) * (float)dot;
  }
  (void)xs;
  return acc;
}

// ---- Q5_0 planes: unit = 4 blocks --------------------------------------------------------------
struct UnitQ5_0 {
  uint4 q[4];
  uint4 qh;   // 4 x u32 high-bit masks
  uint2 d;
};
__device__ __forceinline__ void load_unit_q5_0(const WPlanes& w, int64_t row, int u, UnitQ5_0& r) {
  const uint8_t* qs = w.p0 + row * w.rb0 + (int64_t)u * 64;
#pragma unroll
  for (int i = 0; i < 4; ++i) r.q[i] = ldg_stream(qs + 16 * i);
  r.qh = __ldg(reinterpret_cast<const uint4*>(w.p2 + row * w.rb2 + (int64_t)u * 16));
  r.d = __ldg(reinterpret_cast<const uint2*>(w.p1 + row * w.rb1 + (int64_t)u * 8));
}
// Spread 4 bits (bit i of nib4) into bit 4 of byte i.
__device__ __forceinline__ uint32_t spread4_bit4(uint32_t nib4) {
  return ((nib4 & 1u) << 4) | ((nib4 & 2u) << 11) | ((nib4 & 4u) << 18) | ((nib4 & 8u) << 25);
}
__device__ __forceinline__ float dot_unit_q5_0(const UnitQ5_0& r, int u, const int8_t* xq, const float* xd,
                                               const float* xs) {
  const int k0 = u * 128;
  float acc = 0.f;
  const uint32_t qhs[4] = {r.qh.x, r.qh.y, r.qh.z, r.qh.w};
  const uint32_t words[4][4] = {{r.q[0].x, r.q[0].y, r.q[0].z, r.q[0].w}, {r.q[1].x, r.q[1].y, r.q[1].z, r.q[1].w},
                                {r.q[2].x, r.q[2].y, r.q[2].z, r.q[2].w}, {r.q[3].x, r.q[3].y, r.q[3].z, r.q[3].w}};
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const int4 x0 = ldx16(xq + k0 + 32 * b), x1 = ldx16(xq + k0 + 32 * b + 16);
    const int xa[4] = {x0.x, x0.y, x0.z, x0.w}, xb[4] = {x1.x, x1.y, x1.z, x1.w};
    int dot = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t lo = (words[b][i] & 0x0F0F0F0F) | spread4_bit4((qhs[b] >> (4 * i)) & 0xF);
      uint32_t hi = ((words[b][i] >> 4) & 0x0F0F0F0F) | spread4_bit4((qhs[b] >> (16 + 4 * i)) & 0xF);
      dot = dp4a((int)lo, xa[i], dot);
      dot = dp4a((int)hi, xb[i], dot);
    }
    const uint32_t dw = b < 2 ? r.d.x : r.d.y;
    const float dwf = __half2float(__ushort_as_half((uint16_t)(dw >> (16 * (b & 1)))));
    const int blk = (k0 >> 5) + b;
    acc += dwf * (ldxf(xd + blk) * (float)dot - 16.f * ldxf(xs + blk));
  }
  return acc;
}

// ---- Q6_K planes: unit = half super-block (128 elements) ---------------------------------------
// ql: 64 bytes per half, qh: 32 bytes per half, sc: 8 int8 per half, d: one f16 per super-block.
struct UnitQ6K {
  uint4 ql[4];
  uint4 qh[2];
  uint2 sc;
  float d;
};
__device__ __forceinline__ void load_unit_q6k(const WPlanes& w, int64_t row, int u, UnitQ6K& r) {
  const uint8_t* ql = w.p0 + row * w.rb0 + (int64_t)u * 64;
#pragma unroll
  for (int i = 0; i < 4; ++i) r.ql[i] = ldg_stream(ql + 16 * i);
  const uint8_t* qh = w.p1 + row * w.rb1 + (int64_t)u * 32;
  r.qh[0] = ldg_stream(qh);
  r.qh[1] = ldg_stream(qh + 16);
  r.sc = __ldg(reinterpret_cast<const uint2*>(w.p2 + row * w.rb2 + (int64_t)u * 8));
  r.d = __half2float(__ldg(reinterpret_cast<const __half*>(w.p3 + row * w.rb3) + (u >> 1)));
}
__device__ __forceinline__ float dot_unit_q6k(const UnitQ6K& r, int u, const int8_t* xq, const float* xd,
                                              const float* xs) {
  // Element e (0..127) of the half: group g = e/32 (0..3), l = e%32.
  //   g0: ql[l] lo | qh[l]>>0 ; g1: ql[l+32] lo | qh[l]>>2 ; g2: ql[l] hi | qh[l]>>4 ; g3: ql[l+32] hi | qh[l]>>6
  const int k0 = u * 128;
  const uint32_t ql[16] = {r.ql[0].x, r.ql[0].y, r.ql[0].z, r.ql[0].w, r.ql[1].x, r.ql[1].y, r.ql[1].z, r.ql[1].w,
                           r.ql[2].x, r.ql[2].y, r.ql[2].z, r.ql[2].w, r.ql[3].x, r.ql[3].y, r.ql[3].z, r.ql[3].w};
  const uint32_t qh[8] = {r.qh[0].x, r.qh[0].y, r.qh[0].z, r.qh[0].w, r.qh[1].x, r.qh[1].y, r.qh[1].z, r.qh[1].w};
  const int8_t* sc = reinterpret_cast<const int8_t*>(&r.sc);
  float acc = 0.f;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int qlo = (g & 1) ? 8 : 0;       // word offset into ql (bytes l or l+32)
    const int nshift = (g & 2) ? 4 : 0;    // low or high nibble
    const int hshift = 2 * g;              // qh bit pair
    int dot16[2] = {0, 0}, xs16[2] = {0, 0};
    const int4 xa = ldx16(xq + k0 + 32 * g), xb = ldx16(xq + k0 + 32 * g + 16);
    const int xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {          // 8 words = 32 elements of group g
      // 6-bit codes 0..63; the -32 offset is applied through the activation sum below.
      uint32_t v = ((ql[qlo + i] >> nshift) & 0x0F0F0F0F) | (((qh[i] >> hshift) & 0x03030303) << 4);
      dot16[i >> 2] = dp4a((int)v, xw[i], dot16[i >> 2]);
      xs16[i >> 2] = dp4a(xw[i], 0x01010101, xs16[i >> 2]);
    }
    // Two 16-element sub-blocks per group: scale index 2g + h.
    const float dx = ldxf(xd + (k0 >> 5) + g);
    acc += r.d * dx * ((float)sc[2 * g] * (float)(dot16[0] - 32 * xs16[0]) +
                       (float)sc[2 * g + 1] * (float)(dot16[1] - 32 * xs16[1]));
  }
  (void)xs;
  return acc;
}

}  // namespace hk
