// Register-fragment helpers of mma.sync m16n8k16 (bf16) shared by the tensor-core attention kernels
// (attention_tc.cu, decode_step.cu): ldmatrix loads from 128-byte-swizzled TMA boxes, the MMA, and
// bf16 packing.
#pragma once
#include "common.cuh"

namespace hk {
namespace frag {

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Shared-memory byte address of the 16-byte chunk `chunk` (8 dims) of token row `row` in a stage's
// K (or V) boxes: boxes of [rows x 64 dims] (128 bytes per row) with the 128-byte swizzle.
__device__ __forceinline__ uint32_t sw_addr(uint32_t box_base, int rows, int row, int chunk) {
  const int box = chunk >> 3, c = chunk & 7;
  return box_base + (uint32_t)(box * rows * 128 + row * 128 + ((c ^ (row & 7)) << 4));
}

}  // namespace frag
}  // namespace hk
