// Sub-2-bit mixed codecs of the `.gravity` family (HGRAV*) and the HQ80M15 compact catalog.
//
// Envelope of every payload: 8-byte magic | u32 LE header_len | canonical JSON header | body.
//   HGRAVB01  binary sign x fp16 group scale (mean |w|); body = groups * f16 scales + sign bits
//             (LSB-first, 1 = non-negative). Reconstruction sign * scale.
//   HGRAVR02  HGRAVB01 + a Rice-coded outlier residual: u32 first_index, Rice(k) deltas (unary
//             quotient LSB-first, then k remainder bits), one f16 rms scale, 1-bit signs.
//   HGRAVS01  low-rank W ~= L @ R with L [out, rank] and R [rank, in] stored as HGRAVU01-style
//             uniform groups (left body then right body); decode as y = L @ (R @ x).
//   HGRAVU01  uniform group codes: groups * f16 scale (absmax / bound) + packed unsigned codes
//             (code = signed + bound, bound = 2^(bits-1) - 1, LSB-first).
// The benchmark's ternary codec point is HGRAVU01 with bits = 2 (bound 1) and Q4 is HGRAVU01
// with bits = 4 (bound 7), both in 64-element groups.
//
// Parity: docs/QWEN80_MIXED_1P5_PACKED_FORMAT.md:84-231 and
// crates/hawking-core/src/model/qwen_complete_binary/q80_mixed_decode.rs:135-1070 (split_gravity_container,
// extract_unsigned, unpack_rice, expand_rice_indices, parse_*_container, *_matvec_f32 oracles),
// crates/hawking-core/src/model/qwen80_mixed_catalog.rs:20-33 (catalog magic "HQ80M15\0").
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "json.h"

namespace hk {

struct MixedEnvelope {
  std::string magic;
  Json header;
  const uint8_t* body = nullptr;
  size_t body_bytes = 0;
};
MixedEnvelope mixed_split(const uint8_t* data, size_t n);

struct BinaryGroup {       // HGRAVB01 (also the base of HGRAVR02)
  int rows = 0, cols = 0, group = 0;
  std::vector<uint16_t> scales;  // f16 bits, [rows * cols / group]
  std::vector<uint8_t> signs;    // LSB-first bits, 1 = non-negative
};
struct UniformGroup {      // HGRAVU01 / HGRAVS01 factors
  int rows = 0, cols = 0, group = 0, bits = 0, bound = 0;
  std::vector<uint16_t> scales;
  std::vector<uint8_t> codes;    // packed LSB-first
};
struct RiceResidual {      // HGRAVR02
  BinaryGroup base;
  uint32_t rice_k = 0;
  std::vector<uint32_t> indices; // flat element indices, ascending
  uint16_t residual_scale = 0;   // f16 bits
  std::vector<uint8_t> residual_signs;
};
struct LowRank {           // HGRAVS01
  UniformGroup left, right;
  int rank = 0;
};

uint32_t extract_bits_lsb(const uint8_t* codes, size_t element, int bits);
std::vector<uint32_t> unpack_rice(const uint8_t* p, size_t n, size_t count, uint32_t k);

BinaryGroup parse_hgravb01(const uint8_t* data, size_t n);
RiceResidual parse_hgravr02(const uint8_t* data, size_t n);
UniformGroup parse_hgravu01(const uint8_t* data, size_t n);
LowRank parse_hgravs01(const uint8_t* data, size_t n);

// Dense fp32 reconstruction (row-major [rows, cols]) — the CPU oracle.
std::vector<float> decode_mixed(const uint8_t* data, size_t n, int* rows, int* cols);

// Encoders (synthetic artifacts). Inputs are row-major fp32 [rows, cols].
std::vector<uint8_t> encode_hgravb01(const float* w, int rows, int cols, int group);
std::vector<uint8_t> encode_hgravu01(const float* w, int rows, int cols, int group, int bits);
// Envelopes around planes that are already quantised (fp16 group scales, then the LSB-first sign or
// code stream), with no re-quantisation: the artifact writer of models quantised on the device.
std::vector<uint8_t> wrap_hgravb01(int rows, int cols, int group, const uint8_t* scales, size_t scale_bytes,
                                   const uint8_t* signs, size_t sign_bytes);
std::vector<uint8_t> wrap_hgravu01(int rows, int cols, int group, int bits, const uint8_t* scales,
                                   size_t scale_bytes, const uint8_t* codes, size_t code_bytes);
std::vector<uint8_t> encode_hgravr02(const float* w, int rows, int cols, int group, double outlier_ratio,
                                     uint32_t rice_k);
std::vector<uint8_t> encode_hgravs01(const float* left, const float* right, int out, int rank, int in, int group,
                                     int bits);

// HQ80M15 compact catalog (little endian, 128-byte tensor records).
struct CatalogSegment { uint16_t id; std::string name; uint64_t bytes; std::string sha256; };
struct CatalogTensor {
  std::string name;
  uint8_t codec = 0, organ = 0, ndim = 0;
  uint32_t dims[4] = {0, 0, 0, 0};
  uint64_t elements = 0;
  uint16_t segment = 0, rank = 0;
  uint64_t offset = 0, nbytes = 0;
  std::string sha256;
  uint32_t flags = 0, n_fit_rows = 0;
  float codec_bpw = 0;
};
struct Catalog {
  uint32_t version = 1, flags = 0;
  std::vector<CatalogSegment> segments;
  std::vector<CatalogTensor> tensors;
};
Catalog read_catalog(const std::string& path);
void write_catalog(const std::string& path, const Catalog& c);

}  // namespace hk
