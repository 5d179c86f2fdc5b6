// HGRAV* mixed codecs and the HQ80M15 catalog; see mixed.h.
#include "mixed.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <numeric>
#include <stdexcept>

#include "ggml_quant.h"

namespace hk {

namespace {
const char* kSchemaBinary = "hawking.gravity.binary_sign_scale.v1";
const char* kSchemaResidual = "hawking.gravity.binary_outlier_residual.v2";
const char* kSchemaLowRank = "hawking.gravity.activation_weighted_svd_low_rank.v1";
const char* kSchemaUniform = "hawking.gravity.uniform_group.v1";
const char* kLowRankRepr = "activation_weighted_svd_low_rank_q";

[[noreturn]] void fail(const std::string& m) { throw std::runtime_error(m); }
uint64_t U(const Json& h, const char* k, const char* who) {
  if (!h[k].is_number()) fail(std::string(who) + ": header missing " + k);
  return h[k].as_uint();
}
void need_str(const Json& h, const char* k, const char* v, const char* who) {
  if (!h[k].is_string() || h[k].as_string() != v) fail(std::string(who) + ": header " + k + " must be " + v);
}
void rows_cols(const Json& h, const char* key, uint64_t elements, int* r, int* c, const char* who) {
  const Json& s = h[key];
  if (!s.is_array() || s.size() == 0) fail(std::string(who) + ": bad shape");
  uint64_t cols = s.at(s.size() - 1).as_uint(), prod = 1;
  for (const auto& d : s.items()) prod *= d.as_uint();
  if (prod != elements || cols == 0) fail(std::string(who) + ": shape disagrees with elements");
  *r = (int)(elements / cols);
  *c = (int)cols;
}
std::vector<uint16_t> f16s(const uint8_t* p, size_t n) {
  std::vector<uint16_t> v(n);
  std::memcpy(v.data(), p, n * 2);
  return v;
}
void put_bit(std::vector<uint8_t>& b, size_t i, bool v) {
  if (b.size() <= i / 8) b.resize(i / 8 + 1, 0);
  if (v) b[i / 8] |= (uint8_t)(1u << (i & 7));
}
std::vector<uint8_t> envelope(const char* magic, const Json& header, const std::vector<uint8_t>& body) {
  const std::string h = header.canonical();
  std::vector<uint8_t> out(8 + 4 + h.size() + body.size());
  std::memcpy(out.data(), magic, 8);
  const uint32_t hl = (uint32_t)h.size();
  std::memcpy(out.data() + 8, &hl, 4);
  std::memcpy(out.data() + 12, h.data(), h.size());
  std::memcpy(out.data() + 12 + h.size(), body.data(), body.size());
  return out;
}
Json shape2(int r, int c) {
  Json s = Json::array();
  s.push(Json::uinteger(r));
  s.push(Json::uinteger(c));
  return s;
}
UniformGroup uniform_body(int rows, int cols, int bits, int group, const uint8_t* body, size_t n, const char* who) {
  if (bits < 1 || bits > 8 || group <= 0) fail(std::string(who) + ": bad uniform geometry");
  UniformGroup u;
  u.rows = rows; u.cols = cols; u.bits = bits; u.group = group;
  u.bound = bits == 1 ? 1 : (1 << (bits - 1)) - 1;
  const size_t el = (size_t)rows * cols, groups = (el + group - 1) / group;
  const size_t code_bytes = (groups * group * bits + 7) / 8;
  if (n != groups * 2 + code_bytes) fail(std::string(who) + ": body length disagrees with geometry");
  u.scales = f16s(body, groups);
  u.codes.assign(body + groups * 2, body + n);
  return u;
}
std::vector<uint8_t> uniform_encode_body(const float* w, size_t el, int group, int bits, int* bound_out) {
  const int bound = (1 << (bits - 1)) - 1;
  const size_t groups = (el + group - 1) / group;
  std::vector<uint8_t> scales(groups * 2), codes((groups * group * bits + 7) / 8, 0);
  for (size_t g = 0; g < groups; ++g) {
    float amax = 0;
    for (int i = 0; i < group; ++i) {
      size_t e = g * group + i;
      if (e < el) amax = std::max(amax, std::fabs(w[e]));
    }
    const uint16_t sh = f32_to_fp16(amax / (float)std::max(bound, 1));
    std::memcpy(&scales[g * 2], &sh, 2);
    const float s = fp16_to_f32(sh);
    for (int i = 0; i < group; ++i) {
      size_t e = g * group + i;
      int q = 0;
      if (e < el && s > 0) q = std::clamp((int)std::nearbyint(w[e] / s), -bound, bound);
      const uint32_t code = (uint32_t)(q + bound);
      for (int b = 0; b < bits; ++b) put_bit(codes, e * bits + b, (code >> b) & 1);
    }
  }
  codes.resize((groups * group * bits + 7) / 8, 0);
  if (bound_out) *bound_out = bound;
  scales.insert(scales.end(), codes.begin(), codes.end());
  return scales;
}
Json uniform_header(int rows, int cols, int group, int bits) {
  Json h = Json::object();
  const size_t el = (size_t)rows * cols, groups = (el + group - 1) / group;
  h.set("schema", Json::string(kSchemaUniform));
  h.set("shape", shape2(rows, cols));
  h.set("elements", Json::uinteger(el));
  h.set("bits", Json::uinteger(bits));
  h.set("group_size", Json::uinteger(group));
  h.set("groups", Json::uinteger(groups));
  h.set("bound", Json::uinteger((1 << (bits - 1)) - 1));
  h.set("scale_bytes", Json::uinteger(groups * 2));
  h.set("code_bytes", Json::uinteger((groups * group * bits + 7) / 8));
  return h;
}
}  // namespace

MixedEnvelope mixed_split(const uint8_t* d, size_t n) {
  if (n < 12) fail("mixed: payload shorter than the envelope prefix");
  MixedEnvelope e;
  e.magic.assign(reinterpret_cast<const char*>(d), 8);
  uint32_t hl;
  std::memcpy(&hl, d + 8, 4);
  if (12 + (size_t)hl > n) fail("mixed: header exceeds payload");
  e.header = Json::parse(reinterpret_cast<const char*>(d + 12), hl);
  e.body = d + 12 + hl;
  e.body_bytes = n - 12 - hl;
  return e;
}

uint32_t extract_bits_lsb(const uint8_t* codes, size_t element, int bits) {
  uint32_t v = 0;
  const size_t b0 = element * bits;
  for (int b = 0; b < bits; ++b) v |= (uint32_t)((codes[(b0 + b) >> 3] >> ((b0 + b) & 7)) & 1) << b;
  return v;
}

std::vector<uint32_t> unpack_rice(const uint8_t* p, size_t n, size_t count, uint32_t k) {
  std::vector<uint32_t> out;
  out.reserve(count);
  size_t bit = 0;
  auto rd = [&]() -> uint32_t {
    if (bit / 8 >= n) fail("rice: stream overran its payload");
    uint32_t v = (p[bit / 8] >> (bit & 7)) & 1;
    ++bit;
    return v;
  };
  for (size_t i = 0; i < count; ++i) {
    uint32_t q = 0;
    while (rd() == 1) ++q;
    uint32_t r = 0;
    for (uint32_t b = 0; b < k; ++b) r |= rd() << b;
    out.push_back((q << k) | r);
  }
  return out;
}

BinaryGroup parse_hgravb01(const uint8_t* d, size_t n) {
  auto e = mixed_split(d, n);
  if (e.magic != std::string("HGRAVB01", 8)) fail("HGRAVB01: magic mismatch");
  need_str(e.header, "schema", kSchemaBinary, "HGRAVB01");
  const uint64_t el = U(e.header, "elements", "HGRAVB01"), gs = U(e.header, "group_size", "HGRAVB01");
  const uint64_t groups = U(e.header, "groups", "HGRAVB01");
  const uint64_t sb = U(e.header, "scale_bytes", "HGRAVB01"), gb = U(e.header, "sign_bytes", "HGRAVB01");
  if (!gs || groups != (el + gs - 1) / gs) fail("HGRAVB01: group ledger disagrees with elements");
  if (sb != groups * 2 || gb != (groups * gs + 7) / 8) fail("HGRAVB01: scale/sign ledger is invalid");
  if (e.body_bytes != sb + gb) fail("HGRAVB01: body length disagrees with ledger");
  BinaryGroup b;
  rows_cols(e.header, "shape", el, &b.rows, &b.cols, "HGRAVB01");
  if (b.cols % gs) fail("HGRAVB01: cols must be a multiple of group_size");
  b.group = (int)gs;
  b.scales = f16s(e.body, groups);
  b.signs.assign(e.body + sb, e.body + sb + gb);
  return b;
}

RiceResidual parse_hgravr02(const uint8_t* d, size_t n) {
  auto e = mixed_split(d, n);
  const Json& h = e.header;
  if (e.magic != std::string("HGRAVR02", 8)) fail("HGRAVR02: magic mismatch");
  need_str(h, "schema", kSchemaResidual, "HGRAVR02");
  need_str(h, "index_mode", "rice", "HGRAVR02");
  need_str(h, "value_scale", "rms", "HGRAVR02");
  if (U(h, "value_bits", "HGRAVR02") != 1) fail("HGRAVR02: value_bits must be 1");
  const uint64_t el = U(h, "elements", "HGRAVR02"), gs = U(h, "group_size", "HGRAVR02");
  const uint64_t groups = U(h, "groups", "HGRAVR02"), sb = U(h, "scale_bytes", "HGRAVR02");
  const uint64_t gb = U(h, "sign_bytes", "HGRAVR02"), ib = U(h, "index_bytes", "HGRAVR02");
  const uint64_t rsb = U(h, "residual_scale_bytes", "HGRAVR02"), rb = U(h, "residual_bytes", "HGRAVR02");
  const uint64_t cnt = U(h, "outlier_count", "HGRAVR02"), k = U(h, "rice_k", "HGRAVR02");
  const uint64_t rice_b = U(h, "rice_bytes", "HGRAVR02"), fib = U(h, "first_index_bytes", "HGRAVR02");
  if (fib != 4 || ib != fib + rice_b || rsb != 2) fail("HGRAVR02: index ledger is invalid");
  if (e.body_bytes != sb + gb + ib + rsb + rb) fail("HGRAVR02: body length disagrees with ledger");
  RiceResidual r;
  rows_cols(h, "shape", el, &r.base.rows, &r.base.cols, "HGRAVR02");
  if (r.base.cols % gs || groups != (uint64_t)r.base.rows * (r.base.cols / gs)) fail("HGRAVR02: groups not row-aligned");
  r.base.group = (int)gs;
  size_t c = 0;
  r.base.scales = f16s(e.body, groups);
  c += sb;
  r.base.signs.assign(e.body + c, e.body + c + gb);
  c += gb;
  uint32_t first;
  std::memcpy(&first, e.body + c, 4);
  c += 4;
  r.rice_k = (uint32_t)k;
  if (cnt == 0) fail("HGRAVR02: rice residual requires at least one outlier");
  r.indices.push_back(first);
  if (cnt > 1) {
    auto diffs = unpack_rice(e.body + c, rice_b, cnt - 1, (uint32_t)k);
    uint64_t acc = first;
    for (auto df : diffs) {
      acc += df;
      if (acc > 0xFFFFFFFFull) fail("HGRAVR02: rice index exceeds u32");
      r.indices.push_back((uint32_t)acc);
    }
  }
  c += rice_b;
  std::memcpy(&r.residual_scale, e.body + c, 2);
  c += 2;
  r.residual_signs.assign(e.body + c, e.body + c + rb);
  for (auto i : r.indices)
    if (i >= el) fail("HGRAVR02: residual index out of range");
  return r;
}

UniformGroup parse_hgravu01(const uint8_t* d, size_t n) {
  auto e = mixed_split(d, n);
  if (e.magic != std::string("HGRAVU01", 8)) fail("HGRAVU01: magic mismatch");
  need_str(e.header, "schema", kSchemaUniform, "HGRAVU01");
  const uint64_t el = U(e.header, "elements", "HGRAVU01");
  int r, c;
  rows_cols(e.header, "shape", el, &r, &c, "HGRAVU01");
  return uniform_body(r, c, (int)U(e.header, "bits", "HGRAVU01"), (int)U(e.header, "group_size", "HGRAVU01"), e.body,
                      e.body_bytes, "HGRAVU01");
}

LowRank parse_hgravs01(const uint8_t* d, size_t n) {
  auto e = mixed_split(d, n);
  const Json& h = e.header;
  if (e.magic != std::string("HGRAVS01", 8)) fail("HGRAVS01: magic mismatch");
  need_str(h, "schema", kSchemaLowRank, "HGRAVS01");
  need_str(h, "representation", kLowRankRepr, "HGRAVS01");
  const Json& ms = h["matrix_shape"];
  if (!ms.is_array() || ms.size() != 2) fail("HGRAVS01: matrix_shape must be rank-2");
  const int out = (int)ms.at(0).as_uint(), in = (int)ms.at(1).as_uint();
  const int rank = (int)U(h, "rank", "HGRAVS01"), bits = (int)U(h, "factor_bits", "HGRAVS01");
  const int gs = (int)U(h, "factor_group_size", "HGRAVS01");
  const uint64_t lb = U(h, "left_body_bytes", "HGRAVS01"), rbb = U(h, "right_body_bytes", "HGRAVS01");
  if (lb + rbb != e.body_bytes) fail("HGRAVS01: physical body disagrees with factor ledgers");
  LowRank lr;
  lr.rank = rank;
  lr.left = uniform_body(out, rank, bits, gs, e.body, lb, "HGRAVS01 left");
  lr.right = uniform_body(rank, in, bits, gs, e.body + lb, rbb, "HGRAVS01 right");
  return lr;
}

namespace {
std::vector<float> dense_uniform(const UniformGroup& u) {
  std::vector<float> w((size_t)u.rows * u.cols);
  for (size_t e = 0; e < w.size(); ++e) {
    const float s = fp16_to_f32(u.scales[e / u.group]);
    w[e] = ((int)extract_bits_lsb(u.codes.data(), e, u.bits) - u.bound) * s;
  }
  return w;
}
std::vector<float> dense_binary(const BinaryGroup& b) {
  std::vector<float> w((size_t)b.rows * b.cols);
  for (size_t e = 0; e < w.size(); ++e) {
    const float s = fp16_to_f32(b.scales[e / b.group]);
    w[e] = ((b.signs[e >> 3] >> (e & 7)) & 1) ? s : -s;
  }
  return w;
}
}  // namespace

std::vector<float> decode_mixed(const uint8_t* d, size_t n, int* rows, int* cols) {
  auto e = mixed_split(d, n);
  if (e.magic == std::string("HGRAVB01", 8)) {
    auto b = parse_hgravb01(d, n);
    *rows = b.rows; *cols = b.cols;
    return dense_binary(b);
  }
  if (e.magic == std::string("HGRAVU01", 8)) {
    auto u = parse_hgravu01(d, n);
    *rows = u.rows; *cols = u.cols;
    return dense_uniform(u);
  }
  if (e.magic == std::string("HGRAVR02", 8)) {
    auto r = parse_hgravr02(d, n);
    *rows = r.base.rows; *cols = r.base.cols;
    auto w = dense_binary(r.base);
    const float s = fp16_to_f32(r.residual_scale);
    for (size_t i = 0; i < r.indices.size(); ++i) w[r.indices[i]] += ((r.residual_signs[i >> 3] >> (i & 7)) & 1) ? s : -s;
    return w;
  }
  if (e.magic == std::string("HGRAVS01", 8)) {
    auto lr = parse_hgravs01(d, n);
    auto L = dense_uniform(lr.left), R = dense_uniform(lr.right);
    const int out = lr.left.rows, rank = lr.rank, in = lr.right.cols;
    *rows = out; *cols = in;
    std::vector<float> w((size_t)out * in, 0.f);
    for (int o = 0; o < out; ++o)
      for (int k = 0; k < rank; ++k) {
        const float l = L[(size_t)o * rank + k];
        for (int i = 0; i < in; ++i) w[(size_t)o * in + i] += l * R[(size_t)k * in + i];
      }
    return w;
  }
  fail("mixed: unknown payload magic " + e.magic);
}

namespace {
Json binary_header(int rows, int cols, int group, size_t sign_bytes) {
  const size_t el = (size_t)rows * cols, groups = el / group;
  Json h = Json::object();
  h.set("schema", Json::string(kSchemaBinary));
  h.set("shape", shape2(rows, cols));
  h.set("elements", Json::uinteger(el));
  h.set("group_size", Json::uinteger(group));
  h.set("groups", Json::uinteger(groups));
  h.set("scale_bytes", Json::uinteger(groups * 2));
  h.set("sign_bytes", Json::uinteger(sign_bytes));
  return h;
}
}  // namespace

std::vector<uint8_t> wrap_hgravb01(int rows, int cols, int group, const uint8_t* scales, size_t scale_bytes,
                                   const uint8_t* signs, size_t sign_bytes) {
  if (group <= 0 || cols % group) fail("HGRAVB01 wrap: cols must be a multiple of group");
  const size_t el = (size_t)rows * cols, groups = el / group;
  if (scale_bytes != groups * 2 || sign_bytes != (el + 7) / 8) fail("HGRAVB01 wrap: plane sizes do not match the shape");
  std::vector<uint8_t> body(scales, scales + scale_bytes);
  body.insert(body.end(), signs, signs + sign_bytes);
  return envelope("HGRAVB01", binary_header(rows, cols, group, sign_bytes), body);
}

std::vector<uint8_t> wrap_hgravu01(int rows, int cols, int group, int bits, const uint8_t* scales,
                                   size_t scale_bytes, const uint8_t* codes, size_t code_bytes) {
  if (bits < 2 || bits > 8 || group <= 0 || cols % group) fail("HGRAVU01 wrap: bad geometry");
  const size_t el = (size_t)rows * cols, groups = el / group;
  if (scale_bytes != groups * 2 || code_bytes != (groups * group * bits + 7) / 8)
    fail("HGRAVU01 wrap: plane sizes do not match the shape");
  std::vector<uint8_t> body(scales, scales + scale_bytes);
  body.insert(body.end(), codes, codes + code_bytes);
  return envelope("HGRAVU01", uniform_header(rows, cols, group, bits), body);
}

std::vector<uint8_t> encode_hgravb01(const float* w, int rows, int cols, int group) {
  if (cols % group) fail("HGRAVB01 encode: cols must be a multiple of group");
  const size_t el = (size_t)rows * cols, groups = el / group;
  std::vector<uint8_t> body(groups * 2), signs((el + 7) / 8, 0);
  for (size_t g = 0; g < groups; ++g) {
    double s = 0;
    for (int i = 0; i < group; ++i) s += std::fabs(w[g * group + i]);
    const uint16_t sh = f32_to_fp16((float)(s / group));
    std::memcpy(&body[g * 2], &sh, 2);
  }
  for (size_t e = 0; e < el; ++e)
    if (w[e] >= 0) signs[e >> 3] |= (uint8_t)(1u << (e & 7));
  body.insert(body.end(), signs.begin(), signs.end());
  return envelope("HGRAVB01", binary_header(rows, cols, group, signs.size()), body);
}

std::vector<uint8_t> encode_hgravu01(const float* w, int rows, int cols, int group, int bits) {
  if (bits < 2 || bits > 8) fail("HGRAVU01 encode: bits must be 2..8");
  auto body = uniform_encode_body(w, (size_t)rows * cols, group, bits, nullptr);
  return envelope("HGRAVU01", uniform_header(rows, cols, group, bits), body);
}

std::vector<uint8_t> encode_hgravr02(const float* w, int rows, int cols, int group, double ratio, uint32_t k) {
  const size_t el = (size_t)rows * cols;
  auto bin = encode_hgravb01(w, rows, cols, group);
  auto b = parse_hgravb01(bin.data(), bin.size());
  auto base = dense_binary(b);
  const size_t cnt = std::max<size_t>(1, (size_t)std::ceil(el * ratio));
  std::vector<uint32_t> idx(el);
  std::iota(idx.begin(), idx.end(), 0);
  std::partial_sort(idx.begin(), idx.begin() + cnt, idx.end(), [&](uint32_t a, uint32_t c) {
    const float ra = std::fabs(w[a] - base[a]), rc = std::fabs(w[c] - base[c]);
    return ra != rc ? ra > rc : a < c;
  });
  idx.resize(cnt);
  std::sort(idx.begin(), idx.end());
  double ss = 0;
  for (auto i : idx) ss += (double)(w[i] - base[i]) * (w[i] - base[i]);
  const uint16_t rs = f32_to_fp16((float)std::sqrt(ss / cnt));
  std::vector<uint8_t> rice, rsign;
  size_t bit = 0;
  for (size_t i = 1; i < cnt; ++i) {
    const uint32_t v = idx[i] - idx[i - 1];
    for (uint32_t q = v >> k; q > 0; --q) put_bit(rice, bit++, true);
    put_bit(rice, bit++, false);
    for (uint32_t bb = 0; bb < k; ++bb) put_bit(rice, bit++, (v >> bb) & 1);
  }
  rice.resize((bit + 7) / 8, 0);
  for (size_t i = 0; i < cnt; ++i) put_bit(rsign, i, w[idx[i]] - base[idx[i]] > 0);
  rsign.resize((cnt + 7) / 8, 0);
  // body: binary body | u32 first | rice | f16 scale | signs
  auto benv = mixed_split(bin.data(), bin.size());
  std::vector<uint8_t> body(benv.body, benv.body + benv.body_bytes);
  const uint32_t first = idx[0];
  body.insert(body.end(), reinterpret_cast<const uint8_t*>(&first), reinterpret_cast<const uint8_t*>(&first) + 4);
  body.insert(body.end(), rice.begin(), rice.end());
  body.push_back((uint8_t)(rs & 0xFF));
  body.push_back((uint8_t)(rs >> 8));
  body.insert(body.end(), rsign.begin(), rsign.end());
  Json h = benv.header;
  h.set("schema", Json::string(kSchemaResidual));
  h.set("index_mode", Json::string("rice"));
  h.set("value_bits", Json::uinteger(1));
  h.set("value_scale", Json::string("rms"));
  h.set("outlier_count", Json::uinteger(cnt));
  h.set("rice_k", Json::uinteger(k));
  h.set("rice_bytes", Json::uinteger(rice.size()));
  h.set("first_index_bytes", Json::uinteger(4));
  h.set("index_bytes", Json::uinteger(4 + rice.size()));
  h.set("residual_scale_bytes", Json::uinteger(2));
  h.set("residual_bytes", Json::uinteger(rsign.size()));
  return envelope("HGRAVR02", h, body);
}

std::vector<uint8_t> encode_hgravs01(const float* left, const float* right, int out, int rank, int in, int group,
                                     int bits) {
  auto lb = uniform_encode_body(left, (size_t)out * rank, group, bits, nullptr);
  auto rb = uniform_encode_body(right, (size_t)rank * in, group, bits, nullptr);
  Json h = Json::object();
  h.set("schema", Json::string(kSchemaLowRank));
  h.set("representation", Json::string(kLowRankRepr));
  h.set("shape", shape2(out, in));
  h.set("matrix_shape", shape2(out, in));
  h.set("elements", Json::uinteger((uint64_t)out * in));
  h.set("rank", Json::uinteger(rank));
  h.set("factor_bits", Json::uinteger(bits));
  h.set("factor_group_size", Json::uinteger(group));
  h.set("left", uniform_header(out, rank, group, bits));
  h.set("right", uniform_header(rank, in, group, bits));
  h.set("left_body_bytes", Json::uinteger(lb.size()));
  h.set("right_body_bytes", Json::uinteger(rb.size()));
  Json cap = Json::object();
  cap.set("fit_kind", Json::string("real_routed_activation_capture"));
  cap.set("sha256", Json::string(std::string(64, '0')));
  h.set("activation_capture", cap);
  lb.insert(lb.end(), rb.begin(), rb.end());
  return envelope("HGRAVS01", h, lb);
}

// ---- HQ80M15 catalog ----------------------------------------------------------------------------
namespace {
const char kCatMagic[8] = {'H', 'Q', '8', '0', 'M', '1', '5', '\0'};
std::string hex32(const uint8_t* p) {
  static const char* H = "0123456789abcdef";
  std::string s(64, '0');
  for (int i = 0; i < 32; ++i) { s[2 * i] = H[p[i] >> 4]; s[2 * i + 1] = H[p[i] & 15]; }
  return s;
}
void unhex32(const std::string& s, uint8_t* out) {
  std::memset(out, 0, 32);
  for (size_t i = 0; i + 1 < s.size() && i / 2 < 32; i += 2)
    out[i / 2] = (uint8_t)std::stoi(s.substr(i, 2), nullptr, 16);
}
}  // namespace

Catalog read_catalog(const std::string& path) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) fail("catalog: cannot open " + path);
  std::vector<uint8_t> b;
  uint8_t buf[65536];
  size_t k;
  while ((k = std::fread(buf, 1, sizeof buf, f)) > 0) b.insert(b.end(), buf, buf + k);
  std::fclose(f);
  if (b.size() < 32 || std::memcmp(b.data(), kCatMagic, 8) != 0) fail("catalog: bad magic");
  auto u32 = [&](size_t o) { uint32_t v; std::memcpy(&v, &b[o], 4); return v; };
  auto u16 = [&](size_t o) { uint16_t v; std::memcpy(&v, &b[o], 2); return v; };
  auto u64 = [&](size_t o) { uint64_t v; std::memcpy(&v, &b[o], 8); return v; };
  Catalog c;
  c.version = u32(8);
  const uint32_t nt = u32(12), ns = u32(16);
  c.flags = u32(20);
  const uint32_t name_blob = u32(24);
  size_t o = 32;
  for (uint32_t i = 0; i < ns; ++i) {
    if (o + 44 > b.size()) fail("catalog: truncated segment table");
    CatalogSegment s;
    s.id = u16(o);
    const uint16_t nl = u16(o + 2);
    s.bytes = u64(o + 4);
    s.sha256 = hex32(&b[o + 12]);
    if (o + 44 + nl > b.size()) fail("catalog: truncated segment name");
    s.name.assign(reinterpret_cast<const char*>(&b[o + 44]), nl);
    o += 44 + nl;
    c.segments.push_back(s);
  }
  const size_t names = o + (size_t)nt * 128;
  if (names + name_blob > b.size()) fail("catalog: truncated tensor table");
  for (uint32_t i = 0; i < nt; ++i, o += 128) {
    CatalogTensor t;
    const uint32_t no = u32(o);
    const uint16_t nl = u16(o + 4);
    if (no + nl > name_blob) fail("catalog: name out of range");
    t.name.assign(reinterpret_cast<const char*>(&b[names + no]), nl);
    t.codec = b[o + 6]; t.organ = b[o + 7]; t.ndim = b[o + 8];
    for (int d = 0; d < 4; ++d) t.dims[d] = u32(o + 12 + 4 * d);
    t.elements = u64(o + 28);
    t.segment = u16(o + 36);
    t.rank = u16(o + 38);
    t.offset = u64(o + 40);
    t.nbytes = u64(o + 48);
    t.sha256 = hex32(&b[o + 56]);
    t.flags = u32(o + 88);
    t.n_fit_rows = u32(o + 92);
    std::memcpy(&t.codec_bpw, &b[o + 96], 4);
    c.tensors.push_back(t);
  }
  return c;
}

void write_catalog(const std::string& path, const Catalog& c) {
  std::vector<uint8_t> b(32, 0), names;
  auto p32 = [&](size_t o, uint32_t v) { std::memcpy(&b[o], &v, 4); };
  std::memcpy(b.data(), kCatMagic, 8);
  p32(8, c.version);
  p32(12, (uint32_t)c.tensors.size());
  p32(16, (uint32_t)c.segments.size());
  p32(20, c.flags);
  for (const auto& t : c.tensors) names.insert(names.end(), t.name.begin(), t.name.end());
  p32(24, (uint32_t)names.size());
  for (const auto& s : c.segments) {
    const size_t o = b.size();
    b.resize(o + 44 + s.name.size(), 0);
    const uint16_t nl = (uint16_t)s.name.size();
    std::memcpy(&b[o], &s.id, 2);
    std::memcpy(&b[o + 2], &nl, 2);
    std::memcpy(&b[o + 4], &s.bytes, 8);
    unhex32(s.sha256, &b[o + 12]);
    std::memcpy(&b[o + 44], s.name.data(), s.name.size());
  }
  uint32_t noff = 0;
  for (const auto& t : c.tensors) {
    const size_t o = b.size();
    b.resize(o + 128, 0);
    const uint16_t nl = (uint16_t)t.name.size();
    std::memcpy(&b[o], &noff, 4);
    std::memcpy(&b[o + 4], &nl, 2);
    b[o + 6] = t.codec; b[o + 7] = t.organ; b[o + 8] = t.ndim;
    std::memcpy(&b[o + 12], t.dims, 16);
    std::memcpy(&b[o + 28], &t.elements, 8);
    std::memcpy(&b[o + 36], &t.segment, 2);
    std::memcpy(&b[o + 38], &t.rank, 2);
    std::memcpy(&b[o + 40], &t.offset, 8);
    std::memcpy(&b[o + 48], &t.nbytes, 8);
    unhex32(t.sha256, &b[o + 56]);
    std::memcpy(&b[o + 88], &t.flags, 4);
    std::memcpy(&b[o + 92], &t.n_fit_rows, 4);
    std::memcpy(&b[o + 96], &t.codec_bpw, 4);
    noff += nl;
  }
  b.insert(b.end(), names.begin(), names.end());
  const std::string tmp = path + ".tmp";
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (!f) fail("catalog: cannot create " + tmp);
  const bool ok = std::fwrite(b.data(), 1, b.size(), f) == b.size();
  if (std::fclose(f) != 0 || !ok || std::rename(tmp.c_str(), path.c_str()) != 0) fail("catalog: write failed");
}

}  // namespace hk
