// Host-side TMA tensor-map encoding (cuTensorMapEncodeTiled through the runtime's driver entry
// point, so no libcuda link-time dependency beyond what torch already loads).
#pragma once
#include <cudaTypedefs.h>

#include "common.cuh"

namespace hk {

inline PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    HK_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (!p || q != cudaDriverEntryPointSuccess) throw std::runtime_error("cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D map over [outer, inner] elements with the given row stride (bytes) and box.
inline CUtensorMap tma_map_2d(CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                              CUtensorMapSwizzle swz) {
  if (reinterpret_cast<uintptr_t>(base) % 16) throw std::runtime_error("tma: base not 16-byte aligned");
  if (row_stride_bytes % 16) throw std::runtime_error("tma: row stride not a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = tma_encode_fn()(&m, dt, 2, const_cast<void*>(base), dims, strides, box, es,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

}  // namespace hk
