// Device building blocks of the W4A16 GEMV shared by the stand-alone kernel (mma_gemv.cu) and the
// persistent decode-step kernel (decode_step.cu): the Q4_K tile format, the integer-math tile
// consumer, the two-limb activation quantiser and the split-K ownership arithmetic.
#pragma once
#include "common.cuh"

namespace hk {
namespace mg {

template <int FMT> struct Tile;
template <> struct Tile<WF_Q4_K> {
  static constexpr int BYTES = 2304;  // 16 headers x 16 B + 16 rows x 128 quant bytes
};

__device__ __forceinline__ uint32_t pick(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// 32-bit word index of the pair x[n][k], x[n][k + 1] (k even) in the B-fragment order. Column n
// starts at n * cstride uint4s.
__device__ __forceinline__ int64_t frag_u32(int n, int k, int64_t cstride) {
  const int ks = k >> 4, kk = k & 15, q = (kk & 7) >> 1, reg = kk >> 3;
  return ((int64_t)n * cstride + (((ks >> 2) * 4 + q) * 2 + ((ks & 3) >> 1))) * 4 + (ks & 1) * 2 + reg;
}

// ---- integer math ------------------------------------------------------------------------------
// Activations: per 32-element block b of column n, x_k ~= d2 * (254 * hi_k + lo_k) with
// d1 = amax_b / 127, hi = round(x / d1), lo = round((x - hi d1) / d2), d2 = d1 / 254 (both limbs in
// [-127, 127]): 16-bit fixed point per block, rounding error at most d2 / 2 = amax_b / 64516. The
// block's (d2, sum of its represented values) goes with it.
// Weight tiles (integer layout): per lane and sub-block two words; byte i of the first holds row
// g's nibble of column 32 sb + 4q + i in its low half and row g + 8's in its high half (second
// word: columns + 16). Masking yields the u8 A fragment of mma.m16n8k32 directly: rows g take
// w & 0x0F0F0F0F (n), rows g + 8 take w & 0xF0F0F0F0 (16 n, their weight scale carries the 1/16).
// One sub-block is one k32 MMA per limb; the integer dot 254 * dot_hi + dot_lo is exact.

__device__ __forceinline__ void imma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// (S, M) per (row, sub-block): S = d * sc (rows 8..15: d * sc / 16), M = dmin * mn. Lane t handles
// row t/2, sub-blocks 4*(t&1) .. +3.
__device__ __forceinline__ void decode_scales_q4k_int(const uint8_t* tile, float2* scs, int lane) {
  const int row = lane >> 1, half = lane & 1;
  const uint4 h = *reinterpret_cast<const uint4*>(tile + row * 16);
  float d = __half2float(__ushort_as_half((uint16_t)(h.x & 0xFFFF)));
  const float dmin = __half2float(__ushort_as_half((uint16_t)(h.x >> 16)));
  if (row >= 8) d *= 0.0625f;  // these rows enter the MMA as 16 n (exact)
  const uint32_t scb = half ? ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u)) : (h.y & 0x3F3F3F3Fu);
  const uint32_t mnb = half ? (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u)) : (h.z & 0x3F3F3F3Fu);
  const float c_sc = -d * 8388608.f, c_mn = -dmin * 8388608.f;
  float v[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = fmaf(d, __uint_as_float(__byte_perm(scb, 0x4B000000u, 0x7650 + i)), c_sc);
    v[2 * i + 1] = fmaf(dmin, __uint_as_float(__byte_perm(mnb, 0x4B000000u, 0x7650 + i)), c_mn);
  }
  float4* dst = reinterpret_cast<float4*>(scs + row * 8 + half * 4);
  dst[0] = make_float4(v[0], v[1], v[2], v[3]);
  dst[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// Activation source of the integer math: limbs in B-fragment order (uint4 (hi.b0, hi.b1, lo.b0,
// lo.b1) of lane quad q, block b, column n at n * cstride + b * 4 + q) and per (column, block)
// float2 (d2, block sum) at n * istride + b.
struct XInt {
  const uint4* p;
  int64_t cstride;
  const float2* info;
  int64_t istride;
};

template <int NB>
__device__ __forceinline__ void consume_q4k_int(const uint8_t* tile, int s, const XInt& x, int nb, float2* scs,
                                                int lane, float (&sum)[4]) {
  const int q = lane & 3, r0 = lane >> 2;
  const int n = (lane >> 2) < nb ? (lane >> 2) : 0;  // lanes beyond the batch read column 0
  const uint4* qp = reinterpret_cast<const uint4*>(tile + 256) + lane;
  uint4 qv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) qv[j] = qp[j * 32];
  decode_scales_q4k_int(tile, scs, lane);
  __syncwarp();
  const uint4* xp = x.p + (n * (int)x.cstride + s * 32 + q);
  // columns 2q and 2q + 1 of the C fragment (clamped into the batch)
  const int c0 = 2 * q < nb ? 2 * q : 0, c1 = 2 * q + 1 < nb ? 2 * q + 1 : 0;
  const float4* ip0 = reinterpret_cast<const float4*>(x.info + (c0 * (int)x.istride + s * 8));
  const float4* ip1 = reinterpret_cast<const float4*>(x.info + (c1 * (int)x.istride + s * 8));
  const float4* sp0 = reinterpret_cast<const float4*>(scs + r0 * 8);
  const float4* sp1 = reinterpret_cast<const float4*>(scs + (r0 + 8) * 8);
  constexpr uint32_t LO = 0x0F0F0F0Fu, HI = 0xF0F0F0F0u;
  // shared-memory operands of a pair of sub-blocks (2j, 2j+1): activation fragments, the rows'
  // (S, M) and the columns' (d2, block sum), fetched together one pair ahead of their use
  struct Ops {
    uint4 x0, x1;
    float4 s0, s1, i0, i1;
  };
  auto fetch = [&](int j, Ops& o) {
    o.x0 = xp[(2 * j) * 4];
    o.x1 = xp[(2 * j + 1) * 4];
    o.s0 = sp0[j];
    o.s1 = sp1[j];
    o.i0 = ip0[j];
    if (NB > 1) o.i1 = ip1[j];
  };
  Ops cur, nxt;
  fetch(0, cur);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (j < 3) fetch(j + 1, nxt);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t w0 = pick(qv[j], 2 * h), w1 = pick(qv[j], 2 * h + 1);
      const uint4 xb = h ? cur.x1 : cur.x0;
      int dh[4], dl[4];
      imma_u8s8(dh, w0 & LO, w0 & HI, w1 & LO, w1 & HI, xb.x, xb.y);
      imma_u8s8(dl, w0 & LO, w0 & HI, w1 & LO, w1 & HI, xb.z, xb.w);
      const float s0x = h ? cur.s0.z : cur.s0.x, s0y = h ? cur.s0.w : cur.s0.y;
      const float s1x = h ? cur.s1.z : cur.s1.x, s1y = h ? cur.s1.w : cur.s1.y;
      const float d20 = h ? cur.i0.z : cur.i0.x, x0 = h ? cur.i0.w : cur.i0.y;
      sum[0] = fmaf(s0x, d20 * __int2float_rn(254 * dh[0] + dl[0]), fmaf(-s0y, x0, sum[0]));
      sum[2] = fmaf(s1x, d20 * __int2float_rn(254 * dh[2] + dl[2]), fmaf(-s1y, x0, sum[2]));
      if (NB > 1) {
        const float d21 = h ? cur.i1.z : cur.i1.x, x1 = h ? cur.i1.w : cur.i1.y;
        sum[1] = fmaf(s0x, d21 * __int2float_rn(254 * dh[1] + dl[1]), fmaf(-s0y, x1, sum[1]));
        sum[3] = fmaf(s1x, d21 * __int2float_rn(254 * dh[3] + dl[3]), fmaf(-s1y, x1, sum[3]));
      }
    }
    if (j < 3) cur = nxt;
  }
  __syncwarp();  // every lane is done with the tile and the scales before they are overwritten
}

// Quantise one 32-element block held by a pair of adjacent lanes into the two limbs. Lane half h
// holds v[0..7] = elements 8h .. 8h+7 and v[8..15] = elements 16+8h .. 16+8h+7, and writes lane quads
// q = 2h, 2h+1 of the block's 64 bytes (uint4 q = (hi k=4q.., hi k=16+4q.., lo k=4q.., lo k=16+4q..)).
// Rounding to the nearest integer is one fma against 1.5 * 2^23 (the integer lands in the low
// mantissa bits, so its low byte is the int8 limb). Returns (d2, sum of the represented values).
__device__ __forceinline__ uint32_t pack_low_bytes(float a, float b, float c, float d) {
  const uint32_t ab = __byte_perm(__float_as_uint(a), __float_as_uint(b), 0x0040);
  const uint32_t cd = __byte_perm(__float_as_uint(c), __float_as_uint(d), 0x0040);
  return __byte_perm(ab, cd, 0x5410);
}
__device__ __forceinline__ float2 quant_half_block(const float (&v)[16], int h, uint4* dst) {
  constexpr float MAGIC = 12582912.f;  // 1.5 * 2^23
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  const float d1 = amax * (1.f / 127.f), d2 = d1 * (1.f / 254.f);
  const float inv1 = amax > 0.f ? 127.f / amax : 0.f, inv2 = 254.f * inv1;
  float th[16], tl[16], sh = 0.f, sl = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    th[i] = fmaf(v[i], inv1, MAGIC);
    const float hf = th[i] - MAGIC;
    tl[i] = fmaf(fmaf(-hf, d1, v[i]), inv2, MAGIC);
    sh += hf;
    sl += tl[i] - MAGIC;
  }
#pragma unroll
  for (int qq = 0; qq < 2; ++qq)
    dst[2 * h + qq] = make_uint4(pack_low_bytes(th[4 * qq], th[4 * qq + 1], th[4 * qq + 2], th[4 * qq + 3]),
                                 pack_low_bytes(th[8 + 4 * qq], th[9 + 4 * qq], th[10 + 4 * qq], th[11 + 4 * qq]),
                                 pack_low_bytes(tl[4 * qq], tl[4 * qq + 1], tl[4 * qq + 2], tl[4 * qq + 3]),
                                 pack_low_bytes(tl[8 + 4 * qq], tl[9 + 4 * qq], tl[10 + 4 * qq], tl[11 + 4 * qq]));
  float ms = fmaf(254.f, sh, sl);  // exact: integers below 2^24
  ms += __shfl_xor_sync(0xffffffffu, ms, 1);
  return make_float2(d2, d2 * ms);
}

// The 16 values of lane half h of block b of a bf16 row (elements 32b + 8h .., 32b + 16 + 8h ..).
__device__ __forceinline__ void load_half_block_bf16(const __nv_bfloat16* row, int b, int h, float (&v)[16]) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + 32 * b + 16 * c + 8 * h);
    const uint32_t ws[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[8 * c + 2 * j] = __uint_as_float(ws[j] << 16);
      v[8 * c + 2 * j + 1] = __uint_as_float(ws[j] & 0xFFFF0000u);
    }
  }
}

// Last piece (warp range) holding tile t: pieces p own [p*T/P, (p+1)*T/P). When T < P some
// pieces are empty; owner() always names the non-empty one.
// 32-bit arithmetic: the launcher checks T * P < 2^32.
__device__ __forceinline__ uint32_t owner(uint32_t t, uint32_t T, uint32_t P) { return ((t + 1) * P - 1) / T; }
__device__ __forceinline__ uint32_t start_of(uint32_t p, uint32_t T, uint32_t P) { return p * T / P; }
// The non-empty piece after `p` whose range continues past p's end.
__device__ __forceinline__ uint32_t next_owner(uint32_t p, uint32_t T, uint32_t P) {
  return owner(start_of(p + 1, T, P), T, P);
}
// Number of distinct pieces holding tiles of row group g (tiles [g*KT, (g+1)*KT)).
__device__ __forceinline__ int pieces_of_group(uint32_t g, uint32_t KT, uint32_t T, uint32_t P) {
  const uint32_t last = g * KT + KT - 1;
  int n = 1;
  for (uint32_t pp = owner(g * KT, T, P); start_of(pp + 1, T, P) <= last; pp = next_owner(pp, T, P)) ++n;
  return n;
}

// Head dims of packed tile rows r (0..7) and r + 8 of 16-row group j of a q / k head. The QKV
// matrix is packed so that the two members of every RoPE pair share a lane: adjacent pairs
// (2i, 2i + 1) for style 0, halves (i, i + rot/2) for style 1; dims past rot_dim keep their order.
// p: the pair's frequency index (-1: not rotated).
__device__ __forceinline__ void rope_pair(int j, int r, int rot, int style, int& da, int& db, int& p) {
  if (16 * j < rot) {
    if (style == 0) {
      da = 16 * j + 2 * r;
      db = da + 1;
      p = da >> 1;
    } else {
      da = 8 * j + r;
      db = da + rot / 2;
      p = da;
    }
    return;
  }
  da = 16 * j + r;
  db = da + 8;
  p = -1;
}

// Logical row of packed row R of a QKV matrix packed in RoPE-pair order (`heads` q and k heads
// of hd rows each come first; later rows keep their order).
__device__ __forceinline__ int64_t rope_unpermute(int64_t R, int hd, int rot, int style, int heads) {
  const int64_t head = R / hd;
  if (head >= heads) return R;
  const int w = (int)(R - head * hd), j = w >> 4, rr = w & 15;
  int da, db, p;
  rope_pair(j, rr & 7, rot, style, da, db, p);
  return head * hd + (rr < 8 ? da : db);
}

// QKV epilogue in RoPE-pair order (one row group of 16 packed rows; the lane holds rows r0, r0 + 8
// x columns 2q, 2q + 1): bias, rotation of q / k pairs in registers, q to fp32 rows, k / v to the
// paged bf16 cache of one layer at each column's position.
struct RopeEpi {
  const float* rope;         // [max_pos, rot / 2, 2] (cos, sin)
  const int* positions;      // [nb]
  const int* row_seq;        // [nb]
  const int* block_tables;   // [seqs, max_blocks]
  int max_blocks, block_size;
  __nv_bfloat16* k_cache;    // this layer's [blocks, nkv, block_size, hd]
  __nv_bfloat16* v_cache;
  float* q;                  // [nb, nh, hd]
  const float* bias;         // logical row order; may be null
  int nh, nkv, hd, rot, style;
  int64_t cache_blocks;      // blocks in the caches (out-of-range appends are skipped)
};

template <int NB>
__device__ __forceinline__ void rope_epilogue(const RopeEpi& r, int nb, uint32_t g, const float (&v)[4], int lane) {
  const int r0 = lane >> 2, q = lane & 3;
  const int R = (int)g * 16, head = R / r.hd, j = (R % r.hd) / 16;
  const int kind = head < r.nh ? 0 : (head < r.nh + r.nkv ? 1 : 2);
  int da, db, p = -1;
  if (kind < 2) {
    rope_pair(j, r0, r.rot, r.style, da, db, p);
  } else {
    da = 16 * j + r0;
    db = da + 8;
  }
#pragma unroll
  for (int i = 0; i < (NB > 1 ? 2 : 1); ++i) {
    const int col = 2 * q + i;
    if (col >= nb) continue;
    float x0 = v[i], x1 = v[2 + i];
    if (r.bias) {
      x0 += r.bias[head * r.hd + da];
      x1 += r.bias[head * r.hd + db];
    }
    const int pos = r.positions[col];
    if (p >= 0) {
      const float2 cs = *reinterpret_cast<const float2*>(r.rope + ((int64_t)pos * (r.rot / 2) + p) * 2);
      const float ya = x0 * cs.x - x1 * cs.y, yb = x0 * cs.y + x1 * cs.x;
      x0 = ya;
      x1 = yb;
    }
    if (kind == 0) {
      float* dst = r.q + ((int64_t)col * r.nh + head) * r.hd;
      __stcg(dst + da, x0);
      __stcg(dst + db, x1);
    } else {
      const int kh = head - r.nh - (kind == 2 ? r.nkv : 0);
      if (pos < 0 || pos / r.block_size >= r.max_blocks) continue;  // past the row's table: skip
      const int blk = r.block_tables[(int64_t)r.row_seq[col] * r.max_blocks + pos / r.block_size];
      if (blk < 0 || blk >= r.cache_blocks) continue;
      const int64_t row = ((int64_t)blk * r.nkv + kh) * r.block_size + pos % r.block_size;
      __nv_bfloat16* dst = (kind == 1 ? r.k_cache : r.v_cache) + row * r.hd;
      dst[da] = __float2bfloat16_rn(x0);
      dst[db] = __float2bfloat16_rn(x1);
    }
  }
}

}  // namespace mg
}  // namespace hk
