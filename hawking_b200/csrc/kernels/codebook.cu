// Codebook and low-rank GEMVs of the `.gravity` family (K8): product quantisation (GLM52CPK),
// additive residual PQ (LLM52RPK), activation-aware low rank (GLM52AAP) and the sparse fp16
// corrections of HQ30GR2, at decode batch sizes (nb <= 8 activation columns, q8 blocks).
//
// Codebook GEMV = table lookups: every codeword of every (chunk, sub-space) is dotted with the
// activation slice it multiplies once per step (the LUT, nb x nchunk x nsub x card floats, built
// by one thread per entry), then every output row is a sum of LUT entries picked by its codes:
// one warp per row, lanes over the row's (chunk, sub-space) slots, codes read straight from the
// MSB-first packed stream (a 5-byte window per code). PQ and residual PQ differ only in where a
// sub-space's slice starts (j * sub for PQ, 0 for residual stages spanning the whole chunk).
//
// Parity: crates/hawking-core/src/artifact_pq.rs:300-420 (PqTensor / ResidualPqTensor matvec),
// crates/hawking-core/shaders/gravity_pq.metal (gravity_pq_matvec*), artifact_aap.rs:120-164,
// qwen_complete_binary/mod.rs:380-430 (residual corrections).
#include "api.h"
#include "common.cuh"

namespace hk {
namespace {

__device__ __forceinline__ float xval(const CodebookArgs& a, int b, int c) {
  return (float)a.xq[(int64_t)b * a.x_stride_q + c] * a.xd[(int64_t)b * a.x_stride_s + (c >> 5)];
}

// lut[b][(chunk * nsub + j) * card + k] = <codebook[j][k][:width], x_b[chunk * d + j * sub_stride : +width]>
__global__ void __launch_bounds__(256) codebook_lut_kernel(CodebookArgs a) {
  pdl_wait();
  const int64_t per_col = (int64_t)a.nchunk * a.nsub * a.card;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < per_col * a.nb) {
    const int b = (int)(i / per_col);
    const int64_t e = i % per_col;
    const int k = (int)(e % a.card);
    const int j = (int)((e / a.card) % a.nsub);
    const int chunk = (int)(e / ((int64_t)a.card * a.nsub));
    const __half* cw = a.codebooks + ((int64_t)j * a.card + k) * a.width;
    const int x0 = chunk * a.d + j * a.sub_stride;
    float s = 0.f;
    for (int t = 0; t < a.width; ++t) s += __half2float(cw[t]) * xval(a, b, x0 + t);
    a.lut[i] = s;
  }
  pdl_launch();
}

__device__ __forceinline__ uint32_t code_at(const uint8_t* stream, int64_t index, int bits) {
  const int64_t bit = index * bits;
  const uint8_t* p = stream + (bit >> 3);
  const int skip = (int)(bit & 7);
  // up to 16 + 7 bits: a 4-byte big-endian window always covers them (the stream is padded)
  const uint32_t w = ((uint32_t)p[0] << 24) | ((uint32_t)p[1] << 16) | ((uint32_t)p[2] << 8) | (uint32_t)p[3];
  return (w << skip) >> (32 - bits);
}

// y[b][r] (+)= sum over the row's (chunk, sub-space) slots of the LUT entry its code picks
__global__ void __launch_bounds__(256) codebook_gather_kernel(CodebookArgs a) {
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  if (r < a.rows) {
    const int slots = a.nchunk * a.nsub;
    const int64_t per_col = (int64_t)slots * a.card;
    float acc[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) acc[b] = 0.f;
    for (int s = lane; s < slots; s += 32) {
      const uint32_t code = code_at(a.codes, (int64_t)r * slots + s, a.bits);
      const int64_t li = (int64_t)s * a.card + code;
#pragma unroll
      for (int b = 0; b < 8; ++b)
        if (b < a.nb) acc[b] += a.lut[b * per_col + li];
    }
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      if (b >= a.nb) break;
      const float v = warp_sum(acc[b]) * a.alpha;
      if (lane == 0) {
        float* dst = a.y + (int64_t)b * a.y_stride + r;
        *dst = a.accumulate ? *dst + v : v;
      }
    }
  }
  pdl_launch();
}

// ---- activation-aware low rank ----
// latent[b][k] = sum_c P[c][k] x_b[c]   (input side: P = basis [cols, rank]; stride rank)
//             or sum_c P[k][c] x_b[c]   (output side: P = coefficients [rank, cols])
// One warp per (b, k); lanes over columns.
__global__ void __launch_bounds__(256) aap_latent_kernel(AapArgs a) {
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp < a.nb * a.rank) {
    const int b = warp / a.rank, k = warp % a.rank;
    float s = 0.f;
    for (int c = lane; c < a.cols; c += 32) {
      const float p = a.side == 1 ? __half2float(a.in_proj[(int64_t)c * a.rank + k])
                                  : __half2float(a.in_proj[(int64_t)k * a.cols + c]);
      s += p * (float)a.xq[(int64_t)b * a.x_stride_q + c] * a.xd[(int64_t)b * a.x_stride_s + (c >> 5)];
    }
    s = warp_sum(s);
    if (lane == 0) a.latent[(int64_t)b * a.rank + k] = s;
  }
  pdl_launch();
}

// y[b][r] (+)= sum_k Q[r][k] latent[b][k]   (Q = coefficients [rows, rank] or basis [rows, rank])
__global__ void __launch_bounds__(256) aap_out_kernel(AapArgs a) {
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp < a.rows) {
    const int r = warp;
    for (int b = 0; b < a.nb; ++b) {
      float s = 0.f;
      for (int k = lane; k < a.rank; k += 32) s += __half2float(a.out_proj[(int64_t)r * a.rank + k]) * a.latent[(int64_t)b * a.rank + k];
      s = warp_sum(s) * a.alpha;
      if (lane == 0) {
        float* dst = a.y + (int64_t)b * a.y_stride + r;
        *dst = a.accumulate ? *dst + s : s;
      }
    }
  }
  pdl_launch();
}

// ---- sparse corrections (CSR by output row) ----
__global__ void __launch_bounds__(256) sparse_rows_kernel(SparseArgs a) {
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp < a.rows) {
    const int r = warp;
    const int e0 = a.row_ptr[r], e1 = a.row_ptr[r + 1];
    for (int b = 0; b < a.nb; ++b) {
      float s = 0.f;
      for (int e = e0 + lane; e < e1; e += 32) {
        const int c = a.col[e];
        s += __half2float(a.val[e]) * (float)a.xq[(int64_t)b * a.x_stride_q + c] * a.xd[(int64_t)b * a.x_stride_s + (c >> 5)];
      }
      s = warp_sum(s) * a.alpha;
      if (lane == 0 && e1 > e0) a.y[(int64_t)b * a.y_stride + r] += s;
    }
  }
  pdl_launch();
}

}  // namespace

void codebook_gemv_launch(const CodebookArgs& a, cudaStream_t s, bool pdl) {
  if (a.nb < 1 || a.nb > 8) throw std::runtime_error("codebook gemv: 1..8 activation columns");
  if (a.bits < 1 || a.bits > 16) throw std::runtime_error("codebook gemv: index bits 1..16");
  const int64_t lut_n = (int64_t)a.nb * a.nchunk * a.nsub * a.card;
  launch(codebook_lut_kernel, dim3((unsigned)((lut_n + 255) / 256)), dim3(256), 0, s, pdl, a);
  launch(codebook_gather_kernel, dim3((a.rows + 7) / 8), dim3(256), 0, s, pdl, a);
}

void aap_gemv_launch(const AapArgs& a, cudaStream_t s, bool pdl) {
  if (a.nb < 1 || a.nb > 8) throw std::runtime_error("aap gemv: 1..8 activation columns");
  launch(aap_latent_kernel, dim3((a.nb * a.rank * 32 + 255) / 256), dim3(256), 0, s, pdl, a);
  launch(aap_out_kernel, dim3((a.rows * 32 + 255) / 256), dim3(256), 0, s, pdl, a);
}

void sparse_rows_launch(const SparseArgs& a, cudaStream_t s, bool pdl) {
  launch(sparse_rows_kernel, dim3((a.rows * 32 + 255) / 256), dim3(256), 0, s, pdl, a);
}

}  // namespace hk
