// Fixed-header tensor codecs of the `.gravity` family beyond the HGRAV* envelopes, and the
// `.hawking` sidecar.
//
//   GLM52CPK  product quantisation: a 64-byte header {d, s, sub, card, rows, cols, nchunk, seed,
//             bits, rotate, n_codebooks}; s codebooks [s][card][sub] fp16; indices
//             [row][chunk][sub-space] packed MSB-first at `bits` each. Row chunk c, sub-space j
//             is codeword code(r, c, j) of codebook j; d = s * sub, cols = nchunk * d.
//   LLM52RPK  additive residual PQ: a 64-byte header {d, stages, card, rows, cols, nchunk, seed,
//             bits, 0, stages}; codebooks [stage][card][d] fp16; indices [row][chunk][stage]
//             MSB-first. Row chunk c is the sum over stages of codeword code(r, c, stage).
//   GLM52AAP  activation-aware low rank: a 64-byte header {rows, cols, rank, basis_layer, side
//             (1 input, 2 output), has_basis}; fp16 coefficients then fp16 basis.
//             Input side:  W = C [rows, rank] . B [cols, rank]^T.
//             Output side: W = B [rows, rank] . C [rank, cols].
//   HQ30G1B1  complete binary: a 32-byte header {magic, version 1, group_size, rank, 0,
//             elements, 0}, u32 dims, fp16 group scales, sign bits (LSB-first, 1 = +scale) over
//             the flattened tensor.
//   HQ30UQ4   uniform 4-bit: the same header, fp16 group scales (group 64 or 128), then
//             group/2 code bytes per group (even element low nibble, odd high; q = nibble - 8).
//   HQ30GR2   an HQ30G1B1 payload plus sorted unique flat indices (u32) and fp16 corrections.
//   .hawking  sidecar: magic "DSMTL\x01\0\0" | u32 JSON header length | JSON header | entries
//             {u64 tensor offset | u32 n | n f32} of predecoded Q4_K scale tables (per 144-byte
//             block, (d * sc_j, dmin * m_j) for the 8 sub-blocks).
//
// Parity: crates/hawking-core/src/artifact_pq.rs:1-420 (headers, MSB-first index unpack,
// PqTensor / ResidualPqTensor row and matvec), crates/hawking-core/src/artifact_aap.rs:4-164,
// crates/hawking-core/src/model/qwen_complete_binary/mod.rs:39-80, :137-272, :279-430 and
// uniform_q4.rs:1-60, crates/hawking-core/src/sidecar.rs:1-330 and
// crates/hawking-core/src/kernels/mod.rs:1849-1888 (predecode_q4_k_scale_table).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace hk {

// ---- product quantisation ----
struct PqHeader {
  uint16_t d = 0, s = 0, sub = 0, card = 0;
  uint32_t rows = 0, cols = 0, nchunk = 0, seed = 0;
  uint16_t bits = 0;
  uint8_t rotate = 0, n_codebooks = 0;
};
struct RpqHeader {
  uint16_t d = 0, stages = 0, card = 0;
  uint32_t rows = 0, cols = 0, nchunk = 0, seed = 0;
  uint16_t bits = 0;
};
PqHeader pq_parse(const uint8_t* p, size_t n);
RpqHeader rpq_parse(const uint8_t* p, size_t n);
// codebooks as f32 and the unpacked indices
void pq_sections(const uint8_t* p, size_t n, PqHeader& h, std::vector<float>& cb, std::vector<uint16_t>& idx);
void rpq_sections(const uint8_t* p, size_t n, RpqHeader& h, std::vector<float>& cb, std::vector<uint16_t>& idx);
std::vector<float> pq_decode(const uint8_t* p, size_t n);    // [rows * cols]
std::vector<float> rpq_decode(const uint8_t* p, size_t n);
std::vector<double> pq_matvec_f64(const uint8_t* p, size_t n, const float* x);
std::vector<double> rpq_matvec_f64(const uint8_t* p, size_t n, const float* x);
std::vector<uint8_t> pack_msb(const std::vector<uint32_t>& v, int bits);
std::vector<uint32_t> unpack_msb(const uint8_t* p, size_t n, size_t count, int bits);
std::vector<uint8_t> pq_encode(const PqHeader& h, const std::vector<uint16_t>& cb_f16, const std::vector<uint32_t>& idx);
std::vector<uint8_t> rpq_encode(const RpqHeader& h, const std::vector<uint16_t>& cb_f16, const std::vector<uint32_t>& idx);

// ---- activation-aware low rank ----
struct AapHeader {
  uint32_t rows = 0, cols = 0, rank = 0;
  uint16_t basis_layer = 0;
  int side = 1;  // 1 input, 2 output
  bool has_basis = true;
};
AapHeader aap_parse(const uint8_t* p, size_t n);
std::vector<float> aap_decode(const uint8_t* p, size_t n);
std::vector<double> aap_matvec_f64(const uint8_t* p, size_t n, const float* x);
std::vector<uint8_t> aap_encode(const AapHeader& h, const std::vector<uint16_t>& coeff_f16,
                                const std::vector<uint16_t>& basis_f16);

// ---- HQ30 complete-binary family ----
struct Hq30Header {
  uint32_t version = 1, group_size = 0;
  std::vector<uint32_t> shape;
  uint64_t elements = 0, groups = 0;
  size_t scale_offset = 0, code_offset = 0, payload_bytes = 0;
};
Hq30Header hq30_binary_parse(const uint8_t* p, size_t n);
Hq30Header hq30_uq4_parse(const uint8_t* p, size_t n);
std::vector<float> hq30_binary_decode(const uint8_t* p, size_t n);
std::vector<float> hq30_uq4_decode(const uint8_t* p, size_t n);
struct Hq30Residual {
  Hq30Header base;
  size_t base_offset = 0, base_bytes = 0;
  std::vector<uint32_t> indices;
  std::vector<uint16_t> values;  // f16 bits
};
Hq30Residual hq30_residual_parse(const uint8_t* p, size_t n);
std::vector<float> hq30_residual_decode(const uint8_t* p, size_t n);
std::vector<uint8_t> hq30_binary_encode(const std::vector<uint32_t>& shape, const float* w, int group);
std::vector<uint8_t> hq30_uq4_encode(const std::vector<uint32_t>& shape, const float* w, int group);
std::vector<uint8_t> hq30_residual_encode(const std::vector<uint32_t>& shape, const float* w, int group, size_t keep);

// ---- sidecar ----
std::vector<float> predecode_q4k_scales(const uint8_t* q4k, size_t n);
struct SidecarEntry {
  uint64_t offset = 0;
  std::vector<float> scales;
};
void sidecar_write(const std::string& path, const std::string& header_json, const std::vector<SidecarEntry>& entries);
void sidecar_read(const std::string& path, std::string& header_json, std::vector<SidecarEntry>& entries);

}  // namespace hk
