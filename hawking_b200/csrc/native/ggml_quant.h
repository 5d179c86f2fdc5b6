// GGML block-quant formats: type table, CPU dequantisers (the bit-exact oracle for every GPU
// dequant kernel) and CPU quantisers used by the synthetic-model writers.
//
// Byte layouts follow the public GGUF/ggml specification; the reference reads the same blocks in
// crates/hawking-core/src/gguf.rs:87-111 (block table) and crates/hawking-core/src/quant.rs:34-160
// (dequant oracle). The quantisers are our own (simple min/max searches, not ggml's iterative
// refinement): any encoder is valid as long as the bytes decode with the standard formula.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>

namespace hk {

enum class GgmlType : uint32_t {
  F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q8_1 = 9,
  Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14, Q8_K = 15,
  I8 = 24, I16 = 25, I32 = 26, I64 = 27, F64 = 28, BF16 = 30,
};

struct TypeTraits {
  const char* name;
  int block_elems;   // elements per block (1 for plain types)
  int block_bytes;   // bytes per block
  bool supported;    // dequant implemented
};

const TypeTraits& type_traits(uint32_t t);
bool type_known(uint32_t t);
// Bytes needed to store n elements of type t (n must be a multiple of the block size).
size_t type_nbytes(uint32_t t, size_t n);

float fp16_to_f32(uint16_t h);
uint16_t f32_to_fp16(float f);
float bf16_to_f32(uint16_t h);
uint16_t f32_to_bf16(float f);

// Dequantise n elements stored as type t into out (fp32). Throws std::runtime_error on an
// unsupported type or a size that is not a multiple of the block.
void dequantize(uint32_t t, const void* src, float* out, size_t n);
// Quantise n fp32 elements into type t. Supported: F32 F16 BF16 Q4_0 Q4_1 Q5_0 Q5_1 Q8_0 Q4_K Q5_K Q6_K.
void quantize(uint32_t t, const float* src, void* dst, size_t n);

// Multithreaded helpers over rows (each row an independent run of blocks).
void dequantize_rows(uint32_t t, const void* src, float* out, size_t rows, size_t cols, int threads);
void quantize_rows(uint32_t t, const float* src, void* dst, size_t rows, size_t cols, int threads);

// Q4_K / Q5_K packed 6-bit sub-block scale and min for sub-block j (0..7).
void kquant_scale_min(int j, const uint8_t* scales12, uint8_t* sc, uint8_t* mn);

}  // namespace hk
