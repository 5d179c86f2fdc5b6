// Fixed-header tensor codecs (PQ, residual PQ, activation-aware low rank, HQ30 complete binary /
// uniform Q4 / sparse residual) and the `.hawking` sidecar. Layouts: codecs.h.
#include "codecs.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <stdexcept>

#include "ggml_quant.h"

namespace hk {
namespace {

uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24); }
uint64_t rd64(const uint8_t* p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }
void wr16(std::vector<uint8_t>& o, uint16_t v) { o.push_back(v & 0xFF); o.push_back(v >> 8); }
void wr32(std::vector<uint8_t>& o, uint32_t v) { for (int i = 0; i < 4; ++i) o.push_back((v >> (8 * i)) & 0xFF); }
void wr64(std::vector<uint8_t>& o, uint64_t v) { for (int i = 0; i < 8; ++i) o.push_back((v >> (8 * i)) & 0xFF); }

[[noreturn]] void fail(const std::string& what) { throw std::runtime_error(what); }

void need_magic(const uint8_t* p, size_t n, const char* magic, const char* what) {
  if (n < 8 || std::memcmp(p, magic, 8) != 0) fail(std::string(what) + ": bad magic");
}

// checked a * b * elem_bytes + base
size_t section_end(size_t base, uint64_t count, uint64_t elem_bytes, const char* what) {
  const unsigned __int128 e = (unsigned __int128)count * elem_bytes + base;
  if (e > (unsigned __int128)SIZE_MAX) fail(std::string(what) + ": size overflow");
  return (size_t)e;
}

std::vector<float> f16_array(const uint8_t* p, size_t count) {
  std::vector<float> v(count);
  for (size_t i = 0; i < count; ++i) v[i] = fp16_to_f32(rd16(p + 2 * i));
  return v;
}

constexpr size_t kPqHeader = 64;
constexpr size_t kHq30Header = 32;

}  // namespace

// ---- MSB-first bit packing ----
std::vector<uint32_t> unpack_msb(const uint8_t* p, size_t n, size_t count, int bits) {
  if (bits < 1 || bits > 32) fail("unpack: bits must be 1..32");
  const size_t need = (size_t)(((unsigned __int128)count * bits + 7) / 8);
  if (n < need) fail("unpack: index stream too short");
  const uint64_t mask = bits >= 32 ? 0xFFFFFFFFull : ((1ull << bits) - 1);
  std::vector<uint32_t> out(count);
  uint64_t acc = 0;
  int have = 0;
  size_t pos = 0;
  for (size_t i = 0; i < count; ++i) {
    while (have < bits) {
      acc = (acc << 8) | p[pos++];
      have += 8;
    }
    out[i] = (uint32_t)((acc >> (have - bits)) & mask);
    have -= bits;
  }
  return out;
}

std::vector<uint8_t> pack_msb(const std::vector<uint32_t>& v, int bits) {
  if (bits < 1 || bits > 32) fail("pack: bits must be 1..32");
  const uint64_t lim = bits >= 32 ? 0xFFFFFFFFull : ((1ull << bits) - 1);
  std::vector<uint8_t> out;
  out.reserve((v.size() * bits + 7) / 8);
  uint64_t acc = 0;
  int have = 0;
  for (uint32_t x : v) {
    if (x > lim) fail("pack: value does not fit the bit width");
    acc = (acc << bits) | x;
    have += bits;
    while (have >= 8) {
      out.push_back((uint8_t)((acc >> (have - 8)) & 0xFF));
      have -= 8;
    }
  }
  if (have > 0) out.push_back((uint8_t)((acc << (8 - have)) & 0xFF));
  return out;
}

// ---- GLM52CPK ----
PqHeader pq_parse(const uint8_t* p, size_t n) {
  if (n < kPqHeader) fail("pq: header needs 64 bytes");
  need_magic(p, n, "GLM52CPK", "pq");
  const uint8_t* f = p + 8;
  PqHeader h;
  h.d = rd16(f);
  h.s = rd16(f + 2);
  h.sub = rd16(f + 4);
  h.card = rd16(f + 6);
  h.rows = rd32(f + 8);
  h.cols = rd32(f + 12);
  h.nchunk = rd32(f + 16);
  h.seed = rd32(f + 20);
  h.bits = rd16(f + 24);
  h.rotate = f[26];
  h.n_codebooks = f[27];
  if (h.rotate > 1) fail("pq: rotate must be 0 or 1");
  if (h.d != (uint32_t)h.s * h.sub) fail("pq: D != S * sub");
  if ((uint64_t)h.cols != (uint64_t)h.nchunk * h.d) fail("pq: cols != nchunk * D");
  if (h.n_codebooks != h.s) fail("pq: codebook count != S");
  return h;
}

void pq_sections(const uint8_t* p, size_t n, PqHeader& h, std::vector<float>& cb, std::vector<uint16_t>& idx) {
  h = pq_parse(p, n);
  if (h.rotate) fail("pq: rotated payloads are not supported");
  if (h.bits < 1 || h.bits > 16) fail("pq: bits must be 1..16");
  const size_t cb_end = section_end(kPqHeader, (uint64_t)h.n_codebooks * h.card * h.sub, 2, "pq codebooks");
  const uint64_t count = (uint64_t)h.rows * h.nchunk * h.s;
  const size_t idx_end = section_end(cb_end, (count * h.bits + 7) / 8, 1, "pq indices");
  if (n < idx_end) fail("pq: payload truncated");
  cb = f16_array(p + kPqHeader, (size_t)h.n_codebooks * h.card * h.sub);
  const auto u = unpack_msb(p + cb_end, n - cb_end, (size_t)count, h.bits);
  idx.resize(u.size());
  for (size_t i = 0; i < u.size(); ++i) {
    if (u[i] >= h.card) fail("pq: index beyond the codebook");
    idx[i] = (uint16_t)u[i];
  }
}

std::vector<float> pq_decode(const uint8_t* p, size_t n) {
  PqHeader h;
  std::vector<float> cb;
  std::vector<uint16_t> idx;
  pq_sections(p, n, h, cb, idx);
  std::vector<float> w((size_t)h.rows * h.cols);
  for (uint32_t r = 0; r < h.rows; ++r)
    for (uint32_t c = 0; c < h.nchunk; ++c)
      for (uint32_t j = 0; j < h.s; ++j) {
        const uint16_t code = idx[((size_t)r * h.nchunk + c) * h.s + j];
        const float* src = &cb[((size_t)j * h.card + code) * h.sub];
        std::copy(src, src + h.sub, &w[(size_t)r * h.cols + (size_t)c * h.d + (size_t)j * h.sub]);
      }
  return w;
}

std::vector<double> pq_matvec_f64(const uint8_t* p, size_t n, const float* x) {
  const auto w = pq_decode(p, n);
  const PqHeader h = pq_parse(p, n);
  std::vector<double> y(h.rows, 0.0);
  for (uint32_t r = 0; r < h.rows; ++r)
    for (uint32_t c = 0; c < h.cols; ++c) y[r] += (double)w[(size_t)r * h.cols + c] * (double)x[c];
  return y;
}

std::vector<uint8_t> pq_encode(const PqHeader& h, const std::vector<uint16_t>& cb_f16, const std::vector<uint32_t>& idx) {
  if (cb_f16.size() != (size_t)h.s * h.card * h.sub) fail("pq encode: codebook size");
  if (idx.size() != (size_t)h.rows * h.nchunk * h.s) fail("pq encode: index count");
  std::vector<uint8_t> o(8);
  std::memcpy(o.data(), "GLM52CPK", 8);
  wr16(o, h.d); wr16(o, h.s); wr16(o, h.sub); wr16(o, h.card);
  wr32(o, h.rows); wr32(o, h.cols); wr32(o, h.nchunk); wr32(o, h.seed);
  wr16(o, h.bits); o.push_back(h.rotate); o.push_back(h.n_codebooks);
  o.resize(kPqHeader, 0);
  for (uint16_t v : cb_f16) wr16(o, v);
  const auto packed = pack_msb(idx, h.bits);
  o.insert(o.end(), packed.begin(), packed.end());
  pq_parse(o.data(), o.size());
  return o;
}

// ---- LLM52RPK ----
RpqHeader rpq_parse(const uint8_t* p, size_t n) {
  if (n < kPqHeader) fail("residual pq: header needs 64 bytes");
  need_magic(p, n, "LLM52RPK", "residual pq");
  const uint8_t* f = p + 8;
  RpqHeader h;
  h.d = rd16(f);
  h.stages = rd16(f + 2);
  h.card = rd16(f + 4);
  h.rows = rd32(f + 8);
  h.cols = rd32(f + 12);
  h.nchunk = rd32(f + 16);
  h.seed = rd32(f + 20);
  h.bits = rd16(f + 24);
  if (h.d == 0 || h.stages == 0 || h.card < 2 || h.bits == 0 || h.bits > 16) fail("residual pq: invalid geometry");
  if (h.card > (1u << h.bits) || (uint64_t)h.cols != (uint64_t)h.nchunk * h.d) fail("residual pq: invalid card / shape");
  if (f[26] != 0 || f[27] != (uint8_t)h.stages) fail("residual pq: flags / codebook count not canonical");
  return h;
}

void rpq_sections(const uint8_t* p, size_t n, RpqHeader& h, std::vector<float>& cb, std::vector<uint16_t>& idx) {
  h = rpq_parse(p, n);
  const size_t cb_end = section_end(kPqHeader, (uint64_t)h.stages * h.card * h.d, 2, "residual pq codebooks");
  const uint64_t count = (uint64_t)h.rows * h.nchunk * h.stages;
  const size_t idx_end = section_end(cb_end, (count * h.bits + 7) / 8, 1, "residual pq indices");
  if (n < idx_end) fail("residual pq: payload truncated");
  cb = f16_array(p + kPqHeader, (size_t)h.stages * h.card * h.d);
  const auto u = unpack_msb(p + cb_end, n - cb_end, (size_t)count, h.bits);
  idx.resize(u.size());
  for (size_t i = 0; i < u.size(); ++i) {
    if (u[i] >= h.card) fail("residual pq: index beyond the codebook");
    idx[i] = (uint16_t)u[i];
  }
}

std::vector<float> rpq_decode(const uint8_t* p, size_t n) {
  RpqHeader h;
  std::vector<float> cb;
  std::vector<uint16_t> idx;
  rpq_sections(p, n, h, cb, idx);
  std::vector<float> w((size_t)h.rows * h.cols, 0.f);
  for (uint32_t r = 0; r < h.rows; ++r)
    for (uint32_t c = 0; c < h.nchunk; ++c)
      for (uint32_t s = 0; s < h.stages; ++s) {
        const uint16_t code = idx[((size_t)r * h.nchunk + c) * h.stages + s];
        const float* src = &cb[((size_t)s * h.card + code) * h.d];
        float* dst = &w[(size_t)r * h.cols + (size_t)c * h.d];
        for (uint32_t j = 0; j < h.d; ++j) dst[j] += src[j];
      }
  return w;
}

std::vector<double> rpq_matvec_f64(const uint8_t* p, size_t n, const float* x) {
  RpqHeader h;
  std::vector<float> cb;
  std::vector<uint16_t> idx;
  rpq_sections(p, n, h, cb, idx);
  std::vector<double> y(h.rows, 0.0);
  for (uint32_t r = 0; r < h.rows; ++r)
    for (uint32_t c = 0; c < h.nchunk; ++c)
      for (uint32_t s = 0; s < h.stages; ++s) {
        const uint16_t code = idx[((size_t)r * h.nchunk + c) * h.stages + s];
        const float* src = &cb[((size_t)s * h.card + code) * h.d];
        for (uint32_t j = 0; j < h.d; ++j) y[r] += (double)src[j] * (double)x[(size_t)c * h.d + j];
      }
  return y;
}

std::vector<uint8_t> rpq_encode(const RpqHeader& h, const std::vector<uint16_t>& cb_f16, const std::vector<uint32_t>& idx) {
  if (cb_f16.size() != (size_t)h.stages * h.card * h.d) fail("residual pq encode: codebook size");
  if (idx.size() != (size_t)h.rows * h.nchunk * h.stages) fail("residual pq encode: index count");
  std::vector<uint8_t> o;
  o.insert(o.end(), {'L', 'L', 'M', '5', '2', 'R', 'P', 'K'});
  wr16(o, h.d); wr16(o, h.stages); wr16(o, h.card); wr16(o, 0);
  wr32(o, h.rows); wr32(o, h.cols); wr32(o, h.nchunk); wr32(o, h.seed);
  wr16(o, h.bits); o.push_back(0); o.push_back((uint8_t)h.stages);
  o.resize(kPqHeader, 0);
  for (uint16_t v : cb_f16) wr16(o, v);
  const auto packed = pack_msb(idx, h.bits);
  o.insert(o.end(), packed.begin(), packed.end());
  rpq_parse(o.data(), o.size());
  return o;
}

// ---- GLM52AAP ----
AapHeader aap_parse(const uint8_t* p, size_t n) {
  if (n < kPqHeader) fail("aap: header needs 64 bytes");
  need_magic(p, n, "GLM52AAP", "aap");
  AapHeader h;
  h.rows = rd32(p + 8);
  h.cols = rd32(p + 12);
  h.rank = rd32(p + 16);
  h.basis_layer = rd16(p + 20);
  const uint16_t side = rd16(p + 22);
  if (side != 1 && side != 2) fail("aap: side must be 1 (input) or 2 (output)");
  h.side = side;
  if (p[24] > 1) fail("aap: has_basis must be 0 or 1");
  h.has_basis = p[24] == 1;
  if (!h.rows || !h.cols || !h.rank) fail("aap: zero geometry");
  if (h.rank > (h.side == 1 ? h.cols : h.rows)) fail("aap: rank exceeds the basis width");
  return h;
}

namespace {
void aap_parts(const uint8_t* p, size_t n, AapHeader& h, std::vector<float>& coeff, std::vector<float>& basis) {
  h = aap_parse(p, n);
  if (!h.has_basis) fail("aap: payload without a basis");
  const uint64_t nc = h.side == 1 ? (uint64_t)h.rows * h.rank : (uint64_t)h.rank * h.cols;
  const uint64_t nb = h.side == 1 ? (uint64_t)h.cols * h.rank : (uint64_t)h.rows * h.rank;
  const size_t c_end = section_end(kPqHeader, nc, 2, "aap coefficients");
  const size_t end = section_end(c_end, nb, 2, "aap basis");
  if (n != end) fail("aap: payload size does not match the header");
  coeff = f16_array(p + kPqHeader, (size_t)nc);
  basis = f16_array(p + c_end, (size_t)nb);
}
}  // namespace

std::vector<float> aap_decode(const uint8_t* p, size_t n) {
  AapHeader h;
  std::vector<float> C, B;
  aap_parts(p, n, h, C, B);
  std::vector<float> w((size_t)h.rows * h.cols, 0.f);
  for (uint32_t r = 0; r < h.rows; ++r)
    for (uint32_t c = 0; c < h.cols; ++c) {
      float s = 0.f;
      for (uint32_t k = 0; k < h.rank; ++k)
        s += h.side == 1 ? C[(size_t)r * h.rank + k] * B[(size_t)c * h.rank + k]
                         : B[(size_t)r * h.rank + k] * C[(size_t)k * h.cols + c];
      w[(size_t)r * h.cols + c] = s;
    }
  return w;
}

std::vector<double> aap_matvec_f64(const uint8_t* p, size_t n, const float* x) {
  AapHeader h;
  std::vector<float> C, B;
  aap_parts(p, n, h, C, B);
  std::vector<double> lat(h.rank, 0.0), y(h.rows, 0.0);
  if (h.side == 1) {
    for (uint32_t c = 0; c < h.cols; ++c)
      for (uint32_t k = 0; k < h.rank; ++k) lat[k] += (double)B[(size_t)c * h.rank + k] * x[c];
    for (uint32_t r = 0; r < h.rows; ++r)
      for (uint32_t k = 0; k < h.rank; ++k) y[r] += (double)C[(size_t)r * h.rank + k] * lat[k];
  } else {
    for (uint32_t k = 0; k < h.rank; ++k)
      for (uint32_t c = 0; c < h.cols; ++c) lat[k] += (double)C[(size_t)k * h.cols + c] * x[c];
    for (uint32_t r = 0; r < h.rows; ++r)
      for (uint32_t k = 0; k < h.rank; ++k) y[r] += (double)B[(size_t)r * h.rank + k] * lat[k];
  }
  return y;
}

std::vector<uint8_t> aap_encode(const AapHeader& h, const std::vector<uint16_t>& coeff_f16,
                                const std::vector<uint16_t>& basis_f16) {
  std::vector<uint8_t> o;
  o.insert(o.end(), {'G', 'L', 'M', '5', '2', 'A', 'A', 'P'});
  wr32(o, h.rows); wr32(o, h.cols); wr32(o, h.rank);
  wr16(o, h.basis_layer); wr16(o, (uint16_t)h.side);
  o.push_back(h.has_basis ? 1 : 0);
  o.resize(kPqHeader, 0);
  for (uint16_t v : coeff_f16) wr16(o, v);
  for (uint16_t v : basis_f16) wr16(o, v);
  AapHeader chk;
  std::vector<float> c, b;
  aap_parts(o.data(), o.size(), chk, c, b);
  return o;
}

// ---- HQ30 family ----
namespace {
Hq30Header hq30_common(const uint8_t* p, size_t n, const char* magic, const char* what, bool uq4) {
  if (n < kHq30Header) fail(std::string(what) + ": header needs 32 bytes");
  need_magic(p, n, magic, what);
  Hq30Header h;
  h.version = rd32(p + 8);
  if (h.version != 1) fail(std::string(what) + ": unsupported version");
  h.group_size = rd32(p + 12);
  const uint32_t rank = rd16(p + 16);
  if (rd16(p + 18) != 0 || rd32(p + 28) != 0) fail(std::string(what) + ": reserved fields must be zero");
  if (uq4 ? (h.group_size != 64 && h.group_size != 128) : (h.group_size == 0 || h.group_size % 8))
    fail(std::string(what) + ": bad group size");
  if (rank == 0) fail(std::string(what) + ": rank must be positive");
  h.elements = rd64(p + 20);
  const size_t dims_end = section_end(kHq30Header, rank, 4, what);
  if (dims_end > n) fail(std::string(what) + ": truncated dimensions");
  uint64_t prod = 1;
  for (uint32_t i = 0; i < rank; ++i) {
    const uint32_t v = rd32(p + kHq30Header + 4 * i);
    if (!v) fail(std::string(what) + ": zero dimension");
    prod *= v;
    h.shape.push_back(v);
  }
  if (prod != h.elements) fail(std::string(what) + ": element count disagrees with the shape");
  h.groups = (h.elements + h.group_size - 1) / h.group_size;
  h.scale_offset = dims_end;
  h.code_offset = section_end(h.scale_offset, h.groups, 2, what);
  h.payload_bytes = section_end(h.code_offset, h.groups, uq4 ? h.group_size / 2 : h.group_size / 8, what);
  if (h.payload_bytes != n) fail(std::string(what) + ": payload size does not match the fixed layout");
  for (uint64_t g = 0; g < h.groups; ++g)
    if (!std::isfinite(fp16_to_f32(rd16(p + h.scale_offset + 2 * g)))) fail(std::string(what) + ": non-finite scale");
  return h;
}
}  // namespace

Hq30Header hq30_binary_parse(const uint8_t* p, size_t n) { return hq30_common(p, n, "HQ30G1B1", "complete binary", false); }
Hq30Header hq30_uq4_parse(const uint8_t* p, size_t n) { return hq30_common(p, n, "HQ30UQ4\0", "uniform q4", true); }

std::vector<float> hq30_binary_decode(const uint8_t* p, size_t n) {
  const Hq30Header h = hq30_binary_parse(p, n);
  std::vector<float> v((size_t)h.elements);
  const size_t gb = h.group_size / 8;
  for (uint64_t e = 0; e < h.elements; ++e) {
    const uint64_t g = e / h.group_size, b = e % h.group_size;
    const float s = fp16_to_f32(rd16(p + h.scale_offset + 2 * g));
    const uint8_t byte = p[h.code_offset + g * gb + b / 8];
    v[e] = ((byte >> (b % 8)) & 1) ? s : -s;
  }
  return v;
}

std::vector<float> hq30_uq4_decode(const uint8_t* p, size_t n) {
  const Hq30Header h = hq30_uq4_parse(p, n);
  std::vector<float> v((size_t)h.elements);
  const size_t gb = h.group_size / 2;
  for (uint64_t e = 0; e < h.elements; ++e) {
    const uint64_t g = e / h.group_size, i = e % h.group_size;
    const float s = fp16_to_f32(rd16(p + h.scale_offset + 2 * g));
    const uint8_t byte = p[h.code_offset + g * gb + i / 2];
    const int q = (int)((i & 1) ? (byte >> 4) : (byte & 0xF)) - 8;
    v[e] = (float)q * s;
  }
  return v;
}

Hq30Residual hq30_residual_parse(const uint8_t* p, size_t n) {
  if (n < kHq30Header) fail("quality residual: header needs 32 bytes");
  need_magic(p, n, "HQ30GR2\0", "quality residual");
  if (rd32(p + 8) != 1 || rd32(p + 12) != 1 || rd32(p + 16) != 128 || rd32(p + 20) == 0)
    fail("quality residual: unsupported version / group / rank");
  const uint32_t group = rd32(p + 16), rank = rd32(p + 20), base_bytes = rd32(p + 24), count = rd32(p + 28);
  Hq30Residual r;
  r.base_offset = section_end(kHq30Header, rank, 4, "quality residual");
  const size_t base_end = section_end(r.base_offset, base_bytes, 1, "quality residual");
  const size_t idx_end = section_end(base_end, count, 4, "quality residual");
  const size_t val_end = section_end(idx_end, count, 2, "quality residual");
  if (val_end != n) fail("quality residual: payload size does not match the header");
  std::vector<uint32_t> shape;
  for (uint32_t i = 0; i < rank; ++i) {
    const uint32_t v = rd32(p + kHq30Header + 4 * i);
    if (!v) fail("quality residual: zero dimension");
    shape.push_back(v);
  }
  r.base_bytes = base_bytes;
  r.base = hq30_binary_parse(p + r.base_offset, base_bytes);
  if (r.base.group_size != group || r.base.shape != shape) fail("quality residual: embedded payload geometry differs");
  r.indices.resize(count);
  r.values.resize(count);
  for (uint32_t i = 0; i < count; ++i) {
    r.indices[i] = rd32(p + base_end + 4 * i);
    r.values[i] = rd16(p + idx_end + 2 * i);
    if (r.indices[i] >= r.base.elements || (i && r.indices[i] <= r.indices[i - 1]))
      fail("quality residual: indices must be sorted, unique and in bounds");
    if (!std::isfinite(fp16_to_f32(r.values[i]))) fail("quality residual: non-finite correction");
  }
  return r;
}

std::vector<float> hq30_residual_decode(const uint8_t* p, size_t n) {
  const Hq30Residual r = hq30_residual_parse(p, n);
  std::vector<float> v = hq30_binary_decode(p + r.base_offset, r.base_bytes);
  for (size_t i = 0; i < r.indices.size(); ++i) v[r.indices[i]] += fp16_to_f32(r.values[i]);
  return v;
}

namespace {
std::vector<uint8_t> hq30_head(const char* magic, const std::vector<uint32_t>& shape, uint64_t elements, int group) {
  std::vector<uint8_t> o(magic, magic + 8);
  wr32(o, 1);
  wr32(o, (uint32_t)group);
  wr16(o, (uint16_t)shape.size());
  wr16(o, 0);
  wr64(o, elements);
  wr32(o, 0);
  for (uint32_t d : shape) wr32(o, d);
  return o;
}
uint64_t prod_of(const std::vector<uint32_t>& s) {
  uint64_t p = 1;
  for (uint32_t d : s) p *= d;
  return p;
}
}  // namespace

std::vector<uint8_t> hq30_binary_encode(const std::vector<uint32_t>& shape, const float* w, int group) {
  const uint64_t n = prod_of(shape), groups = (n + group - 1) / group;
  auto o = hq30_head("HQ30G1B1", shape, n, group);
  std::vector<uint8_t> signs(groups * (group / 8), 0);
  for (uint64_t g = 0; g < groups; ++g) {
    double s = 0.0;
    uint64_t cnt = 0;
    for (uint64_t e = g * group; e < std::min(n, (g + 1) * group); ++e, ++cnt) s += std::fabs(w[e]);
    wr16(o, f32_to_fp16((float)(cnt ? s / cnt : 0.0)));
    for (uint64_t e = g * group; e < std::min(n, (g + 1) * group); ++e)
      if (w[e] >= 0.f) signs[g * (group / 8) + (e - g * group) / 8] |= (uint8_t)(1u << ((e - g * group) % 8));
  }
  o.insert(o.end(), signs.begin(), signs.end());
  hq30_binary_parse(o.data(), o.size());
  return o;
}

std::vector<uint8_t> hq30_uq4_encode(const std::vector<uint32_t>& shape, const float* w, int group) {
  const uint64_t n = prod_of(shape), groups = (n + group - 1) / group;
  auto o = hq30_head("HQ30UQ4\0", shape, n, group);
  std::vector<uint8_t> codes(groups * (group / 2), 0x88);  // nibble 8 = 0
  for (uint64_t g = 0; g < groups; ++g) {
    float amax = 0.f;
    for (uint64_t e = g * group; e < std::min(n, (g + 1) * group); ++e) amax = std::max(amax, std::fabs(w[e]));
    const uint16_t s16 = f32_to_fp16(amax / 7.f);
    wr16(o, s16);
    const float s = fp16_to_f32(s16);
    for (uint64_t e = g * group; e < std::min(n, (g + 1) * group); ++e) {
      const int q = s > 0.f ? std::max(-8, std::min(7, (int)std::lrintf(w[e] / s))) : 0;
      const uint64_t i = e - g * group;
      uint8_t& b = codes[g * (group / 2) + i / 2];
      b = (i & 1) ? (uint8_t)((b & 0x0F) | ((q + 8) << 4)) : (uint8_t)((b & 0xF0) | (q + 8));
    }
  }
  o.insert(o.end(), codes.begin(), codes.end());
  hq30_uq4_parse(o.data(), o.size());
  return o;
}

std::vector<uint8_t> hq30_residual_encode(const std::vector<uint32_t>& shape, const float* w, int group, size_t keep) {
  const auto base = hq30_binary_encode(shape, w, group);
  const auto dec = hq30_binary_decode(base.data(), base.size());
  const uint64_t n = prod_of(shape);
  std::vector<uint32_t> order(n);
  for (uint64_t i = 0; i < n; ++i) order[i] = (uint32_t)i;
  keep = std::min<size_t>(keep, n);
  std::partial_sort(order.begin(), order.begin() + keep, order.end(), [&](uint32_t a, uint32_t b) {
    const float da = std::fabs(w[a] - dec[a]), db = std::fabs(w[b] - dec[b]);
    return da != db ? da > db : a < b;
  });
  order.resize(keep);
  std::sort(order.begin(), order.end());
  std::vector<uint8_t> o(8);
  std::memcpy(o.data(), "HQ30GR2\0", 8);
  wr32(o, 1); wr32(o, 1); wr32(o, (uint32_t)group); wr32(o, (uint32_t)shape.size());
  wr32(o, (uint32_t)base.size()); wr32(o, (uint32_t)keep);
  for (uint32_t d : shape) wr32(o, d);
  o.insert(o.end(), base.begin(), base.end());
  for (uint32_t i : order) wr32(o, i);
  for (uint32_t i : order) wr16(o, f32_to_fp16(w[i] - dec[i]));
  hq30_residual_parse(o.data(), o.size());
  return o;
}

// ---- sidecar ----
std::vector<float> predecode_q4k_scales(const uint8_t* q, size_t n) {
  if (n % 144) fail("predecode: Q4_K bytes must be a multiple of 144");
  const size_t nb = n / 144;
  std::vector<float> out(nb * 16);
  for (size_t b = 0; b < nb; ++b) {
    const uint8_t* blk = q + b * 144;
    const float d = fp16_to_f32(rd16(blk)), dmin = fp16_to_f32(rd16(blk + 2));
    const uint8_t* sc = blk + 4;
    for (int j = 0; j < 8; ++j) {
      int s, m;
      if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
      } else {
        s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
      }
      out[b * 16 + 2 * j] = d * (float)s;
      out[b * 16 + 2 * j + 1] = dmin * (float)m;
    }
  }
  return out;
}

static const char kSidecarMagic[8] = {'D', 'S', 'M', 'T', 'L', 1, 0, 0};

void sidecar_write(const std::string& path, const std::string& header_json, const std::vector<SidecarEntry>& entries) {
  std::vector<uint8_t> o(kSidecarMagic, kSidecarMagic + 8);
  wr32(o, (uint32_t)header_json.size());
  o.insert(o.end(), header_json.begin(), header_json.end());
  for (const auto& e : entries) {
    wr64(o, e.offset);
    wr32(o, (uint32_t)e.scales.size());
    const uint8_t* b = reinterpret_cast<const uint8_t*>(e.scales.data());
    o.insert(o.end(), b, b + 4 * e.scales.size());
  }
  const std::string tmp = path + ".tmp";
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (!f) fail("sidecar: cannot create " + tmp);
  const bool ok = std::fwrite(o.data(), 1, o.size(), f) == o.size();
  std::fclose(f);
  if (!ok || std::rename(tmp.c_str(), path.c_str()) != 0) fail("sidecar: write failed for " + path);
}

void sidecar_read(const std::string& path, std::string& header_json, std::vector<SidecarEntry>& entries) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) fail("sidecar: cannot open " + path);
  std::vector<uint8_t> d;
  uint8_t buf[1 << 16];
  size_t k;
  while ((k = std::fread(buf, 1, sizeof buf, f)) > 0) d.insert(d.end(), buf, buf + k);
  std::fclose(f);
  if (d.size() < 12 || std::memcmp(d.data(), kSidecarMagic, 8) != 0) fail("sidecar: bad magic in " + path);
  const uint32_t hl = rd32(d.data() + 8);
  if (12 + (size_t)hl > d.size()) fail("sidecar: header runs past the end");
  header_json.assign(reinterpret_cast<const char*>(d.data() + 12), hl);
  entries.clear();
  size_t pos = 12 + hl;
  while (pos < d.size()) {
    if (pos + 12 > d.size()) fail("sidecar: truncated entry header");
    SidecarEntry e;
    e.offset = rd64(d.data() + pos);
    const uint32_t cnt = rd32(d.data() + pos + 8);
    pos += 12;
    if (pos + 4 * (size_t)cnt > d.size()) fail("sidecar: truncated entry scales");
    e.scales.resize(cnt);
    std::memcpy(e.scales.data(), d.data() + pos, 4 * (size_t)cnt);
    pos += 4 * (size_t)cnt;
    entries.push_back(std::move(e));
  }
}

}  // namespace hk
