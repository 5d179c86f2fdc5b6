// SHA-256 per FIPS 180-4 (round constants are the first 32 bits of the fractional parts of the
// cube roots of the first 64 primes; initial hash values from the square roots of the first 8).
#include "sha256.h"

#include <algorithm>
#include <cstring>
#if defined(__x86_64__)
#include <immintrin.h>
#endif

namespace hk {

namespace {
const uint32_t K[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};
inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
}  // namespace

Sha256::Sha256() {
  const uint32_t init[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                            0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  std::memcpy(h_, init, sizeof h_);
}

void Sha256::block(const uint8_t* p) {
  uint32_t w[64];
  for (int i = 0; i < 16; ++i)
    w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
  for (int i = 16; i < 64; ++i) {
    uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
    uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
    w[i] = w[i - 16] + s0 + w[i - 7] + s1;
  }
  uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
  for (int i = 0; i < 64; ++i) {
    uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
    uint32_t ch = (e & f) ^ (~e & g);
    uint32_t t1 = h + S1 + ch + K[i] + w[i];
    uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
    uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
    uint32_t t2 = S0 + mj;
    h = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
  }
  h_[0] += a; h_[1] += b; h_[2] += c; h_[3] += d; h_[4] += e; h_[5] += f; h_[6] += g; h_[7] += h;
}

#if defined(__x86_64__)
namespace {
// The compression function on the x86 SHA extensions. State held as (A B E F) and (C D G H);
// sha256rnds2 runs two rounds on the low two dwords of W + K; sha256msg1 / msg2 extend the message
// schedule (sigma0 and sigma1 terms), four words at a time.
__attribute__((target("sha,sse4.1,ssse3"))) void blocks_shani(uint32_t h[8], const uint8_t* p, size_t nblocks) {
  const __m128i bswap = _mm_set_epi64x(0x0c0d0e0f08090a0bULL, 0x0405060700010203ULL);
  __m128i t = _mm_shuffle_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(h)), 0xB1);
  __m128i s1 = _mm_shuffle_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(h + 4)), 0x1B);
  __m128i s0 = _mm_alignr_epi8(t, s1, 8);  // A B E F
  s1 = _mm_blend_epi16(s1, t, 0xF0);       // C D G H
  for (; nblocks; --nblocks, p += 64) {
    const __m128i save0 = s0, save1 = s1;
    __m128i w[4];
    for (int i = 0; i < 4; ++i)
      w[i] = _mm_shuffle_epi8(_mm_loadu_si128(reinterpret_cast<const __m128i*>(p + 16 * i)), bswap);
    for (int i = 0; i < 16; ++i) {
      if (i >= 4) {  // W[4i .. 4i + 3] from the four previous groups
        __m128i x = _mm_sha256msg1_epu32(w[(i - 4) & 3], w[(i - 3) & 3]);
        x = _mm_add_epi32(x, _mm_alignr_epi8(w[(i - 1) & 3], w[(i - 2) & 3], 4));
        w[i & 3] = _mm_sha256msg2_epu32(x, w[(i - 1) & 3]);
      }
      __m128i m = _mm_add_epi32(w[i & 3], _mm_loadu_si128(reinterpret_cast<const __m128i*>(K + 4 * i)));
      s1 = _mm_sha256rnds2_epu32(s1, s0, m);
      m = _mm_shuffle_epi32(m, 0x0E);
      s0 = _mm_sha256rnds2_epu32(s0, s1, m);
    }
    s0 = _mm_add_epi32(s0, save0);
    s1 = _mm_add_epi32(s1, save1);
  }
  t = _mm_shuffle_epi32(s0, 0x1B);    // F E B A
  s1 = _mm_shuffle_epi32(s1, 0xB1);   // D C H G
  s0 = _mm_blend_epi16(t, s1, 0xF0);  // D C B A
  s1 = _mm_alignr_epi8(s1, t, 8);     // H G F E
  _mm_storeu_si128(reinterpret_cast<__m128i*>(h), s0);
  _mm_storeu_si128(reinterpret_cast<__m128i*>(h + 4), s1);
}
bool have_shani() {
  static const bool ok = __builtin_cpu_supports("sha") && __builtin_cpu_supports("sse4.1") &&
                         __builtin_cpu_supports("ssse3");
  return ok;
}
}  // namespace
#endif

void Sha256::blocks(const uint8_t* p, size_t n) {
#if defined(__x86_64__)
  if (!portable_ && have_shani()) {
    blocks_shani(h_, p, n);
    return;
  }
#endif
  for (size_t i = 0; i < n; ++i) block(p + 64 * i);
}

void Sha256::update(const void* data, size_t n) {
  const uint8_t* p = static_cast<const uint8_t*>(data);
  total_ += n;
  if (blen_) {
    size_t take = std::min(n, 64 - blen_);
    std::memcpy(buf_ + blen_, p, take);
    blen_ += take; p += take; n -= take;
    if (blen_ == 64) { blocks(buf_, 1); blen_ = 0; }
  }
  if (n >= 64) {
    blocks(p, n / 64);
    p += n / 64 * 64;
    n %= 64;
  }
  if (n) { std::memcpy(buf_, p, n); blen_ = n; }
}

void Sha256::final(uint8_t out[32]) {
  uint64_t bits = total_ * 8;
  uint8_t pad = 0x80;
  update(&pad, 1);
  uint8_t z = 0;
  while (blen_ != 56) update(&z, 1);
  uint8_t len[8];
  for (int i = 0; i < 8; ++i) len[i] = (uint8_t)(bits >> (56 - 8 * i));
  update(len, 8);
  for (int i = 0; i < 8; ++i) {
    out[4 * i] = (uint8_t)(h_[i] >> 24);
    out[4 * i + 1] = (uint8_t)(h_[i] >> 16);
    out[4 * i + 2] = (uint8_t)(h_[i] >> 8);
    out[4 * i + 3] = (uint8_t)h_[i];
  }
}

std::string Sha256::hex() {
  uint8_t d[32];
  final(d);
  static const char* H = "0123456789abcdef";
  std::string s(64, '0');
  for (int i = 0; i < 32; ++i) { s[2 * i] = H[d[i] >> 4]; s[2 * i + 1] = H[d[i] & 15]; }
  return s;
}

std::string Sha256::hex_of(const void* data, size_t n) {
  Sha256 h;
  h.update(data, n);
  return h.hex();
}

}  // namespace hk
