// CPU dequant/quant for GGML block formats. See ggml_quant.h for provenance.
#include "ggml_quant.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <thread>
#include <vector>

namespace hk {

namespace {
const TypeTraits kUnknown{"unknown", 1, 0, false};

const TypeTraits& lookup(uint32_t t, bool* known) {
  static const TypeTraits F32{"F32", 1, 4, true}, F16{"F16", 1, 2, true}, BF16{"BF16", 1, 2, true},
      Q4_0{"Q4_0", 32, 18, true}, Q4_1{"Q4_1", 32, 20, true}, Q5_0{"Q5_0", 32, 22, true},
      Q5_1{"Q5_1", 32, 24, true}, Q8_0{"Q8_0", 32, 34, true}, Q8_1{"Q8_1", 32, 36, false},
      Q2_K{"Q2_K", 256, 84, true}, Q3_K{"Q3_K", 256, 110, true}, Q4_K{"Q4_K", 256, 144, true},
      Q5_K{"Q5_K", 256, 176, true}, Q6_K{"Q6_K", 256, 210, true}, Q8_K{"Q8_K", 256, 292, true},
      I8{"I8", 1, 1, false}, I16{"I16", 1, 2, false}, I32{"I32", 1, 4, false},
      I64{"I64", 1, 8, false}, F64{"F64", 1, 8, true};
  *known = true;
  switch (static_cast<GgmlType>(t)) {
    case GgmlType::F32: return F32;
    case GgmlType::F16: return F16;
    case GgmlType::BF16: return BF16;
    case GgmlType::Q4_0: return Q4_0;
    case GgmlType::Q4_1: return Q4_1;
    case GgmlType::Q5_0: return Q5_0;
    case GgmlType::Q5_1: return Q5_1;
    case GgmlType::Q8_0: return Q8_0;
    case GgmlType::Q8_1: return Q8_1;
    case GgmlType::Q2_K: return Q2_K;
    case GgmlType::Q3_K: return Q3_K;
    case GgmlType::Q4_K: return Q4_K;
    case GgmlType::Q5_K: return Q5_K;
    case GgmlType::Q6_K: return Q6_K;
    case GgmlType::Q8_K: return Q8_K;
    case GgmlType::I8: return I8;
    case GgmlType::I16: return I16;
    case GgmlType::I32: return I32;
    case GgmlType::I64: return I64;
    case GgmlType::F64: return F64;
  }
  *known = false;
  return kUnknown;
}

inline uint16_t rd16(const uint8_t* p) { uint16_t v; std::memcpy(&v, p, 2); return v; }
inline void wr16(uint8_t* p, uint16_t v) { std::memcpy(p, &v, 2); }
inline float half_at(const uint8_t* p) { return fp16_to_f32(rd16(p)); }
inline int nearest(float x) { return static_cast<int>(std::nearbyint(x)); }

void check_blocks(uint32_t t, size_t n) {
  const auto& tt = type_traits(t);
  if (!tt.supported) throw std::runtime_error(std::string("ggml type not supported: ") + tt.name);
  if (n % tt.block_elems)
    throw std::runtime_error(std::string("element count not a multiple of the block for ") + tt.name);
}

// ---- block dequantisers (one block each) ---------------------------------------------------
void dq_q4_0(const uint8_t* b, float* y) {
  float d = half_at(b);
  const uint8_t* qs = b + 2;
  for (int j = 0; j < 16; ++j) {
    y[j] = d * (float)((qs[j] & 0xF) - 8);
    y[j + 16] = d * (float)((qs[j] >> 4) - 8);
  }
}
void dq_q4_1(const uint8_t* b, float* y) {
  float d = half_at(b), m = half_at(b + 2);
  const uint8_t* qs = b + 4;
  for (int j = 0; j < 16; ++j) {
    y[j] = d * (float)(qs[j] & 0xF) + m;
    y[j + 16] = d * (float)(qs[j] >> 4) + m;
  }
}
void dq_q5_0(const uint8_t* b, float* y) {
  float d = half_at(b);
  uint32_t qh; std::memcpy(&qh, b + 2, 4);
  const uint8_t* qs = b + 6;
  for (int j = 0; j < 16; ++j) {
    int h0 = ((qh >> j) << 4) & 0x10;
    int h1 = (qh >> (j + 12)) & 0x10;
    y[j] = d * (float)(((qs[j] & 0xF) | h0) - 16);
    y[j + 16] = d * (float)(((qs[j] >> 4) | h1) - 16);
  }
}
void dq_q5_1(const uint8_t* b, float* y) {
  float d = half_at(b), m = half_at(b + 2);
  uint32_t qh; std::memcpy(&qh, b + 4, 4);
  const uint8_t* qs = b + 8;
  for (int j = 0; j < 16; ++j) {
    int h0 = ((qh >> j) << 4) & 0x10;
    int h1 = (qh >> (j + 12)) & 0x10;
    y[j] = d * (float)((qs[j] & 0xF) | h0) + m;
    y[j + 16] = d * (float)((qs[j] >> 4) | h1) + m;
  }
}
void dq_q8_0(const uint8_t* b, float* y) {
  float d = half_at(b);
  const int8_t* qs = reinterpret_cast<const int8_t*>(b + 2);
  for (int j = 0; j < 32; ++j) y[j] = d * (float)qs[j];
}
void dq_q2_k(const uint8_t* b, float* y) {
  const uint8_t* sc = b;
  const uint8_t* q = b + 16;
  float d = half_at(b + 80), mn = half_at(b + 82);
  int is = 0;
  for (int n = 0; n < 256; n += 128) {
    int shift = 0;
    for (int j = 0; j < 4; ++j) {
      uint8_t s = sc[is++];
      float dl = d * (s & 0xF), ml = mn * (s >> 4);
      for (int l = 0; l < 16; ++l) *y++ = dl * ((q[l] >> shift) & 3) - ml;
      s = sc[is++];
      dl = d * (s & 0xF); ml = mn * (s >> 4);
      for (int l = 0; l < 16; ++l) *y++ = dl * ((q[l + 16] >> shift) & 3) - ml;
      shift += 2;
    }
    q += 32;
  }
}
void q3k_scales(const uint8_t* s12, int8_t* out16) {
  // 16 six-bit scales: low 4 bits in bytes 0..7 (two nibbles each), high 2 bits in bytes 8..11.
  for (int i = 0; i < 16; ++i) {
    int lo = (i < 8) ? (s12[i] & 0xF) : (s12[i - 8] >> 4);
    int hi = (s12[8 + (i % 4)] >> (2 * (i / 4))) & 3;
    out16[i] = (int8_t)((lo | (hi << 4)) - 32);
  }
}
void dq_q3_k(const uint8_t* b, float* y) {
  const uint8_t* hm = b;
  const uint8_t* q = b + 32;
  int8_t sc[16];
  q3k_scales(b + 96, sc);
  float d = half_at(b + 108);
  int is = 0;
  uint8_t m = 1;
  for (int n = 0; n < 256; n += 128) {
    int shift = 0;
    for (int j = 0; j < 4; ++j) {
      float dl = d * sc[is++];
      for (int l = 0; l < 16; ++l) *y++ = dl * (float)(((q[l] >> shift) & 3) - ((hm[l] & m) ? 0 : 4));
      dl = d * sc[is++];
      for (int l = 0; l < 16; ++l)
        *y++ = dl * (float)(((q[l + 16] >> shift) & 3) - ((hm[l + 16] & m) ? 0 : 4));
      shift += 2;
      m <<= 1;
    }
    q += 32;
  }
}
void dq_q4_k(const uint8_t* b, float* y) {
  float d = half_at(b), dmin = half_at(b + 2);
  const uint8_t* scales = b + 4;
  const uint8_t* q = b + 16;
  for (int j = 0; j < 4; ++j) {
    uint8_t sc, m;
    kquant_scale_min(2 * j, scales, &sc, &m);
    float d1 = d * sc, m1 = dmin * m;
    kquant_scale_min(2 * j + 1, scales, &sc, &m);
    float d2 = d * sc, m2 = dmin * m;
    for (int l = 0; l < 32; ++l) y[l] = d1 * (q[l] & 0xF) - m1;
    for (int l = 0; l < 32; ++l) y[l + 32] = d2 * (q[l] >> 4) - m2;
    y += 64;
    q += 32;
  }
}
void dq_q5_k(const uint8_t* b, float* y) {
  float d = half_at(b), dmin = half_at(b + 2);
  const uint8_t* scales = b + 4;
  const uint8_t* qh = b + 16;
  const uint8_t* ql = b + 48;
  uint8_t u1 = 1, u2 = 2;
  for (int j = 0; j < 4; ++j) {
    uint8_t sc, m;
    kquant_scale_min(2 * j, scales, &sc, &m);
    float d1 = d * sc, m1 = dmin * m;
    kquant_scale_min(2 * j + 1, scales, &sc, &m);
    float d2 = d * sc, m2 = dmin * m;
    for (int l = 0; l < 32; ++l) y[l] = d1 * ((ql[l] & 0xF) + ((qh[l] & u1) ? 16 : 0)) - m1;
    for (int l = 0; l < 32; ++l) y[l + 32] = d2 * ((ql[l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - m2;
    y += 64;
    ql += 32;
    u1 <<= 2;
    u2 <<= 2;
  }
}
void dq_q6_k(const uint8_t* b, float* y) {
  const uint8_t* ql = b;
  const uint8_t* qh = b + 128;
  const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
  float d = half_at(b + 208);
  for (int n = 0; n < 256; n += 128) {
    for (int l = 0; l < 32; ++l) {
      int is = l / 16;
      int q1 = (int)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
      int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
      int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
      int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
      y[l] = d * sc[is] * q1;
      y[l + 32] = d * sc[is + 2] * q2;
      y[l + 64] = d * sc[is + 4] * q3;
      y[l + 96] = d * sc[is + 6] * q4;
    }
    y += 128;
    ql += 64;
    qh += 32;
    sc += 8;
  }
}
void dq_q8_k(const uint8_t* b, float* y) {
  float d; std::memcpy(&d, b, 4);
  const int8_t* qs = reinterpret_cast<const int8_t*>(b + 4);
  for (int j = 0; j < 256; ++j) y[j] = d * qs[j];
}

// ---- block quantisers ----------------------------------------------------------------------
void q_q8_0(const float* x, uint8_t* b) {
  float amax = 0;
  for (int j = 0; j < 32; ++j) amax = std::max(amax, std::fabs(x[j]));
  float d = amax / 127.f, id = d ? 1.f / d : 0.f;
  wr16(b, f32_to_fp16(d));
  int8_t* qs = reinterpret_cast<int8_t*>(b + 2);
  for (int j = 0; j < 32; ++j) qs[j] = (int8_t)std::clamp(nearest(x[j] * id), -127, 127);
}
// Signed symmetric: the element of largest magnitude maps to -2^(bits-1).
float signed_extreme(const float* x, int n) {
  float amax = 0, mx = 0;
  for (int j = 0; j < n; ++j)
    if (std::fabs(x[j]) > amax) { amax = std::fabs(x[j]); mx = x[j]; }
  return mx;
}
void q_q4_0(const float* x, uint8_t* b) {
  float mx = signed_extreme(x, 32);
  float d = mx / -8.f, id = d ? 1.f / d : 0.f;
  wr16(b, f32_to_fp16(d));
  uint8_t* qs = b + 2;
  for (int j = 0; j < 16; ++j) {
    int a = std::clamp(nearest(x[j] * id) + 8, 0, 15);
    int c = std::clamp(nearest(x[j + 16] * id) + 8, 0, 15);
    qs[j] = (uint8_t)(a | (c << 4));
  }
}
void q_q5_0(const float* x, uint8_t* b) {
  float mx = signed_extreme(x, 32);
  float d = mx / -16.f, id = d ? 1.f / d : 0.f;
  wr16(b, f32_to_fp16(d));
  uint32_t qh = 0;
  uint8_t* qs = b + 6;
  for (int j = 0; j < 16; ++j) {
    int a = std::clamp(nearest(x[j] * id) + 16, 0, 31);
    int c = std::clamp(nearest(x[j + 16] * id) + 16, 0, 31);
    qs[j] = (uint8_t)((a & 0xF) | ((c & 0xF) << 4));
    qh |= ((uint32_t)(a >> 4) & 1u) << j;
    qh |= ((uint32_t)(c >> 4) & 1u) << (j + 16);
  }
  std::memcpy(b + 2, &qh, 4);
}
void minmax(const float* x, int n, float* lo, float* hi) {
  *lo = x[0]; *hi = x[0];
  for (int j = 1; j < n; ++j) { *lo = std::min(*lo, x[j]); *hi = std::max(*hi, x[j]); }
}
void q_q4_1(const float* x, uint8_t* b) {
  float lo, hi; minmax(x, 32, &lo, &hi);
  float d = (hi - lo) / 15.f, id = d ? 1.f / d : 0.f;
  wr16(b, f32_to_fp16(d)); wr16(b + 2, f32_to_fp16(lo));
  uint8_t* qs = b + 4;
  for (int j = 0; j < 16; ++j) {
    int a = std::clamp(nearest((x[j] - lo) * id), 0, 15);
    int c = std::clamp(nearest((x[j + 16] - lo) * id), 0, 15);
    qs[j] = (uint8_t)(a | (c << 4));
  }
}
void q_q5_1(const float* x, uint8_t* b) {
  float lo, hi; minmax(x, 32, &lo, &hi);
  float d = (hi - lo) / 31.f, id = d ? 1.f / d : 0.f;
  wr16(b, f32_to_fp16(d)); wr16(b + 2, f32_to_fp16(lo));
  uint32_t qh = 0;
  uint8_t* qs = b + 8;
  for (int j = 0; j < 16; ++j) {
    int a = std::clamp(nearest((x[j] - lo) * id), 0, 31);
    int c = std::clamp(nearest((x[j + 16] - lo) * id), 0, 31);
    qs[j] = (uint8_t)((a & 0xF) | ((c & 0xF) << 4));
    qh |= ((uint32_t)(a >> 4) & 1u) << j;
    qh |= ((uint32_t)(c >> 4) & 1u) << (j + 16);
  }
  std::memcpy(b + 4, &qh, 4);
}
// Pack eight 6-bit scales and mins into the 12-byte K-quant scale field (inverse of
// kquant_scale_min).
void pack_scale_min(const uint8_t* sc, const uint8_t* mn, uint8_t* s12) {
  for (int j = 0; j < 4; ++j) {
    s12[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    s12[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
    s12[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4));
  }
}
// Shared search for Q4_K (nmax=15) and Q5_K (nmax=31): per 32-element sub-block an affine
// min/max fit, then 6-bit quantisation of the sub-block scales and mins.
void kquant_affine(const float* x, int nmax, uint8_t* d_out, uint8_t* dmin_out, uint8_t* s12,
                   uint8_t* L) {
  float scale[8], mins[8];
  for (int j = 0; j < 8; ++j) {
    float lo, hi; minmax(x + 32 * j, 32, &lo, &hi);
    lo = std::min(lo, 0.f);
    scale[j] = (hi - lo) / nmax;
    mins[j] = -lo;
  }
  float max_s = *std::max_element(scale, scale + 8), max_m = *std::max_element(mins, mins + 8);
  float d = max_s / 63.f, dmin = max_m / 63.f;
  uint8_t sc[8], mn[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = (uint8_t)std::clamp(d ? nearest(scale[j] / d) : 0, 0, 63);
    mn[j] = (uint8_t)std::clamp(dmin ? nearest(mins[j] / dmin) : 0, 0, 63);
  }
  uint16_t dh = f32_to_fp16(d), mh = f32_to_fp16(dmin);
  std::memcpy(d_out, &dh, 2); std::memcpy(dmin_out, &mh, 2);
  pack_scale_min(sc, mn, s12);
  float dq = fp16_to_f32(dh), mq = fp16_to_f32(mh);
  for (int j = 0; j < 8; ++j) {
    float ds = dq * sc[j], dm = mq * mn[j];
    for (int l = 0; l < 32; ++l) {
      int q = ds ? nearest((x[32 * j + l] + dm) / ds) : 0;
      L[32 * j + l] = (uint8_t)std::clamp(q, 0, nmax);
    }
  }
}
void q_q4_k(const float* x, uint8_t* b) {
  uint8_t L[256];
  kquant_affine(x, 15, b, b + 2, b + 4, L);
  uint8_t* q = b + 16;
  for (int j = 0; j < 4; ++j)
    for (int l = 0; l < 32; ++l) q[32 * j + l] = (uint8_t)(L[64 * j + l] | (L[64 * j + 32 + l] << 4));
}
void q_q5_k(const float* x, uint8_t* b) {
  uint8_t L[256];
  kquant_affine(x, 31, b, b + 2, b + 4, L);
  uint8_t* qh = b + 16;
  uint8_t* ql = b + 48;
  std::memset(qh, 0, 32);
  for (int j = 0; j < 4; ++j)
    for (int l = 0; l < 32; ++l) {
      int a = L[64 * j + l], c = L[64 * j + 32 + l];
      ql[32 * j + l] = (uint8_t)((a & 0xF) | ((c & 0xF) << 4));
      if (a & 16) qh[l] |= (uint8_t)(1u << (2 * j));
      if (c & 16) qh[l] |= (uint8_t)(1u << (2 * j + 1));
    }
}
void q_q6_k(const float* x, uint8_t* b) {
  float sub[16];
  for (int j = 0; j < 16; ++j) sub[j] = signed_extreme(x + 16 * j, 16) / -32.f;
  float amax = 0, mx = 0;
  for (int j = 0; j < 16; ++j)
    if (std::fabs(sub[j]) > amax) { amax = std::fabs(sub[j]); mx = sub[j]; }
  float d = mx / -128.f;
  int8_t* sc = reinterpret_cast<int8_t*>(b + 192);
  uint16_t dh = f32_to_fp16(d);
  std::memcpy(b + 208, &dh, 2);
  float dq = fp16_to_f32(dh);
  uint8_t L[256];
  for (int j = 0; j < 16; ++j) {
    sc[j] = (int8_t)std::clamp(dq ? nearest(sub[j] / dq) : 0, -128, 127);
    float ds = dq * sc[j];
    for (int l = 0; l < 16; ++l) {
      int q = ds ? nearest(x[16 * j + l] / ds) : 0;
      L[16 * j + l] = (uint8_t)(std::clamp(q, -32, 31) + 32);
    }
  }
  uint8_t* ql = b;
  uint8_t* qh = b + 128;
  for (int n = 0; n < 2; ++n) {
    const uint8_t* Ln = L + 128 * n;
    uint8_t* qln = ql + 64 * n;
    uint8_t* qhn = qh + 32 * n;
    for (int l = 0; l < 32; ++l) {
      uint8_t q1 = Ln[l], q2 = Ln[l + 32], q3 = Ln[l + 64], q4 = Ln[l + 96];
      qln[l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
      qln[l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
      qhn[l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  }
}

template <typename F>
void parallel_rows(size_t rows, int threads, F fn) {
  if (threads <= 1 || rows < 64) { fn(0, rows); return; }
  threads = std::min<int>(threads, (int)std::max<size_t>(1, rows / 16));
  std::vector<std::thread> ts;
  size_t per = (rows + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    size_t a = t * per, e = std::min(rows, a + per);
    if (a >= e) break;
    ts.emplace_back([=] { fn(a, e); });
  }
  for (auto& th : ts) th.join();
}
}  // namespace

const TypeTraits& type_traits(uint32_t t) { bool k; return lookup(t, &k); }
bool type_known(uint32_t t) { bool k; lookup(t, &k); return k; }

size_t type_nbytes(uint32_t t, size_t n) {
  const auto& tt = type_traits(t);
  if (!tt.block_bytes) throw std::runtime_error("unknown ggml type " + std::to_string(t));
  if (n % tt.block_elems) throw std::runtime_error(std::string("count not a multiple of block for ") + tt.name);
  return n / tt.block_elems * (size_t)tt.block_bytes;
}

float fp16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF, bits;
  if (exp == 0) {
    if (man == 0) bits = sign;
    else {  // subnormal: renormalise
      int e = -1;
      do { man <<= 1; ++e; } while (!(man & 0x400));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
    }
  } else if (exp == 31) bits = sign | 0x7F800000u | (man << 13);
  else bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  float f; std::memcpy(&f, &bits, 4);
  return f;
}

uint16_t f32_to_fp16(float f) {
  uint32_t x; std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000;
  int32_t exp = (int32_t)((x >> 23) & 0xFF);
  uint32_t man = x & 0x7FFFFF;
  if (exp == 255) return (uint16_t)(sign | 0x7C00 | (man ? 0x200 : 0));
  int32_t e = exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7C00);
  if (e <= 0) {  // subnormal or zero, round to nearest even
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000;
    int shift = 14 - e;
    uint32_t half = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1), mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1))) ++half;
    return (uint16_t)(sign | half);
  }
  uint32_t half = ((uint32_t)e << 10) | (man >> 13);
  uint32_t rem = man & 0x1FFF;
  if (rem > 0x1000 || (rem == 0x1000 && (half & 1))) ++half;  // may carry into exponent: correct
  return (uint16_t)(sign | half);
}

float bf16_to_f32(uint16_t h) {
  uint32_t bits = (uint32_t)h << 16;
  float f; std::memcpy(&f, &bits, 4);
  return f;
}

uint16_t f32_to_bf16(float f) {
  uint32_t x; std::memcpy(&x, &f, 4);
  if ((x & 0x7FFFFFFF) > 0x7F800000) return (uint16_t)((x >> 16) | 0x40);
  uint32_t r = 0x7FFF + ((x >> 16) & 1);
  return (uint16_t)((x + r) >> 16);
}

void kquant_scale_min(int j, const uint8_t* q, uint8_t* sc, uint8_t* mn) {
  if (j < 4) {
    *sc = q[j] & 63;
    *mn = q[j + 4] & 63;
  } else {
    *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
    *mn = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

void dequantize(uint32_t t, const void* src, float* out, size_t n) {
  check_blocks(t, n);
  const uint8_t* p = static_cast<const uint8_t*>(src);
  const auto& tt = type_traits(t);
  size_t nb = n / tt.block_elems;
  void (*fn)(const uint8_t*, float*) = nullptr;
  switch (static_cast<GgmlType>(t)) {
    case GgmlType::F32: std::memcpy(out, src, n * 4); return;
    case GgmlType::F64:
      for (size_t i = 0; i < n; ++i) { double v; std::memcpy(&v, p + 8 * i, 8); out[i] = (float)v; }
      return;
    case GgmlType::F16: for (size_t i = 0; i < n; ++i) out[i] = fp16_to_f32(rd16(p + 2 * i)); return;
    case GgmlType::BF16: for (size_t i = 0; i < n; ++i) out[i] = bf16_to_f32(rd16(p + 2 * i)); return;
    case GgmlType::Q4_0: fn = dq_q4_0; break;
    case GgmlType::Q4_1: fn = dq_q4_1; break;
    case GgmlType::Q5_0: fn = dq_q5_0; break;
    case GgmlType::Q5_1: fn = dq_q5_1; break;
    case GgmlType::Q8_0: fn = dq_q8_0; break;
    case GgmlType::Q2_K: fn = dq_q2_k; break;
    case GgmlType::Q3_K: fn = dq_q3_k; break;
    case GgmlType::Q4_K: fn = dq_q4_k; break;
    case GgmlType::Q5_K: fn = dq_q5_k; break;
    case GgmlType::Q6_K: fn = dq_q6_k; break;
    case GgmlType::Q8_K: fn = dq_q8_k; break;
    default: throw std::runtime_error(std::string("dequant: unsupported ") + tt.name);
  }
  for (size_t i = 0; i < nb; ++i) fn(p + i * tt.block_bytes, out + i * tt.block_elems);
}

void quantize(uint32_t t, const float* src, void* dst, size_t n) {
  check_blocks(t, n);
  uint8_t* p = static_cast<uint8_t*>(dst);
  const auto& tt = type_traits(t);
  size_t nb = n / tt.block_elems;
  void (*fn)(const float*, uint8_t*) = nullptr;
  switch (static_cast<GgmlType>(t)) {
    case GgmlType::F32: std::memcpy(dst, src, n * 4); return;
    case GgmlType::F16: for (size_t i = 0; i < n; ++i) wr16(p + 2 * i, f32_to_fp16(src[i])); return;
    case GgmlType::BF16: for (size_t i = 0; i < n; ++i) wr16(p + 2 * i, f32_to_bf16(src[i])); return;
    case GgmlType::Q4_0: fn = q_q4_0; break;
    case GgmlType::Q4_1: fn = q_q4_1; break;
    case GgmlType::Q5_0: fn = q_q5_0; break;
    case GgmlType::Q5_1: fn = q_q5_1; break;
    case GgmlType::Q8_0: fn = q_q8_0; break;
    case GgmlType::Q4_K: fn = q_q4_k; break;
    case GgmlType::Q5_K: fn = q_q5_k; break;
    case GgmlType::Q6_K: fn = q_q6_k; break;
    default: throw std::runtime_error(std::string("quantize: unsupported ") + tt.name);
  }
  for (size_t i = 0; i < nb; ++i) fn(src + i * tt.block_elems, p + i * tt.block_bytes);
}

void dequantize_rows(uint32_t t, const void* src, float* out, size_t rows, size_t cols, int threads) {
  size_t rb = type_nbytes(t, cols);
  const uint8_t* p = static_cast<const uint8_t*>(src);
  parallel_rows(rows, threads, [&](size_t a, size_t e) {
    for (size_t r = a; r < e; ++r) dequantize(t, p + r * rb, out + r * cols, cols);
  });
}

void quantize_rows(uint32_t t, const float* src, void* dst, size_t rows, size_t cols, int threads) {
  size_t rb = type_nbytes(t, cols);
  uint8_t* p = static_cast<uint8_t*>(dst);
  parallel_rows(rows, threads, [&](size_t a, size_t e) {
    for (size_t r = a; r < e; ++r) quantize(t, src + r * cols, p + r * rb, cols);
  });
}

}  // namespace hk
