// Small-batch dequant GEMV (K1, bs 1..8): y[b, n] = sum_k W[n, k] * x[b, k] with W in a GGUF
// block format dequantised in registers and x as q8 activation blocks, int8 dot products (dp4a).
//
// Design: one warp per output row (RPW rows per warp), lanes stride over 128-element units of
// the row so a warp streams each weight row exactly once with 16-byte loads that bypass L1.
// Rows are independent, so the grid is N / (8 * RPW) CTAs of 8 warps — many resident CTAs per
// SM keep enough bytes in flight to saturate HBM. The activation columns (a few KB) are read
// through the read-only path and stay in L1/L2. Programmatic dependent launch: the first weight
// unit of every row is fetched before waiting on the producer kernel.
//
// Epilogues: STORE (y), RESID (x += y, fp32 residual stream), SWIGLU_Q8 (pair mode: gate and up
// rows, h = silu(g) * u, re-quantised to q8 blocks for the down projection).
//
// Parity: replaces the reference's Q4_K/Q6_K/Q8_0 GEMV family (crates/hawking-core/shaders/quant.metal,
// gemm_q4_k_m_fused*, _pair* gate+up with SwiGLU, _add residual-fused variants); numerics oracle
// crates/hawking-core/src/quant.rs:722 (gemv_q4_k_q8k).
#include "gemv.cuh"

namespace hk {

template <int FMT> struct UnitOf;
template <> struct UnitOf<WF_Q4_K> { using T = UnitQ4K; };
template <> struct UnitOf<WF_Q4_0> { using T = UnitQ4_0; };
template <> struct UnitOf<WF_Q8_0> { using T = UnitQ8_0; };
template <> struct UnitOf<WF_Q5_0> { using T = UnitQ5_0; };
template <> struct UnitOf<WF_Q6_K> { using T = UnitQ6K; };

template <int FMT>
__device__ __forceinline__ void load_unit(const WPlanes& w, int64_t row, int u, typename UnitOf<FMT>::T& r) {
  if constexpr (FMT == WF_Q4_K) load_unit_q4k(w, row, u, r);
  else if constexpr (FMT == WF_Q4_0) load_unit_q4_0(w, row, u, r);
  else if constexpr (FMT == WF_Q8_0) load_unit_q8_0(w, row, u, r);
  else if constexpr (FMT == WF_Q5_0) load_unit_q5_0(w, row, u, r);
  else load_unit_q6k(w, row, u, r);
}
template <int FMT>
__device__ __forceinline__ float dot_unit(const typename UnitOf<FMT>::T& r, int u, const int8_t* xq,
                                          const float* xd, const float* xs) {
  if constexpr (FMT == WF_Q4_K) return dot_unit_q4k(r, u, xq, xd, xs);
  else if constexpr (FMT == WF_Q4_0) return dot_unit_q4_0(r, u, xq, xd, xs);
  else if constexpr (FMT == WF_Q8_0) return dot_unit_q8_0(r, u, xq, xd, xs);
  else if constexpr (FMT == WF_Q5_0) return dot_unit_q5_0(r, u, xq, xd, xs);
  else return dot_unit_q6k(r, u, xq, xd, xs);
}

// Sum over the row for NB activation columns; the result is complete on every lane.
template <int FMT, int NB>
__device__ __forceinline__ void row_dot(const WPlanes& w, int64_t row, int n_units, const XQ& x, float (&acc)[NB],
                                        bool prefetched, const typename UnitOf<FMT>::T& first) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = 0.f;
  int u = lane;
  if (prefetched && u < n_units) {
#pragma unroll
    for (int b = 0; b < NB; ++b)
      acc[b] += dot_unit<FMT>(first, u, x.q + b * x.stride_q, x.d + b * x.stride_s, x.s + b * x.stride_s);
    u += 32;
  }
#pragma unroll 2
  for (; u < n_units; u += 32) {
    typename UnitOf<FMT>::T r;
    load_unit<FMT>(w, row, u, r);
#pragma unroll
    for (int b = 0; b < NB; ++b)
      acc[b] += dot_unit<FMT>(r, u, x.q + b * x.stride_q, x.d + b * x.stride_s, x.s + b * x.stride_s);
  }
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = warp_sum(acc[b]);
}

template <int FMT, int NB, int EPI>
__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs a) {
  constexpr int RPW = (EPI == EPI_SWIGLU_Q8) ? 4 : 1;  // swiglu needs 32 rows per CTA for q8 blocks
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_units = a.K / 128;
  const int64_t row0 = ((int64_t)blockIdx.x * 8 + warp) * RPW;

  // Prefetch the first unit of the first row before the producer finishes.
  typename UnitOf<FMT>::T first;
  const bool pf = row0 < a.N && lane < n_units;
  if (pf) load_unit<FMT>(a.w0, row0, lane, first);
  pdl_wait();

  XQ x{a.xq, a.xd, a.xs, a.x_stride_q, a.x_stride_s};
  if constexpr (EPI == EPI_SWIGLU_Q8) {
    __shared__ float hbuf[NB][32];
    typename UnitOf<FMT>::T dummy;
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int64_t row = row0 + r;
      float g[NB], u[NB];
      if (row < a.N) {
        row_dot<FMT, NB>(a.w0, row, n_units, x, g, r == 0 && pf, first);
        row_dot<FMT, NB>(a.w1, row, n_units, x, u, false, dummy);
      }
      if (lane == 0) {
#pragma unroll
        for (int b = 0; b < NB; ++b)
          hbuf[b][warp * RPW + r] = row < a.N ? g[b] / (1.f + __expf(-g[b])) * u[b] : 0.f;
      }
    }
    __syncthreads();
    pdl_launch();
    // Warp b quantises column b's 32 values (one q8 block).
    for (int b = warp; b < NB; b += 8) {
      const int64_t n = (int64_t)blockIdx.x * 32 + lane;
      const float v = hbuf[b][lane];
      const float amax = warp_max(fabsf(v));
      const float d = amax / 127.f;
      const int q = amax > 0.f ? __float2int_rn(v / d) : 0;
      const float qs = warp_sum((float)q);
      if (n < a.N) a.oq[b * a.o_stride_q + n] = (int8_t)q;
      if (lane == 0 && n < a.N) {
        a.od[b * a.o_stride_s + (n >> 5)] = d;
        a.os[b * a.o_stride_s + (n >> 5)] = d * qs;
      }
    }
  } else {
    if (row0 >= a.N) { pdl_launch(); return; }
    float acc[NB];
    row_dot<FMT, NB>(a.w0, row0, n_units, x, acc, pf, first);
    pdl_launch();
    if (lane < NB) {
      float v = acc[0];
#pragma unroll
      for (int b = 1; b < NB; ++b)
        if (lane == b) v = acc[b];
      float* y = a.y + (int64_t)lane * a.y_stride + row0;
      if (a.bias) v += a.bias[row0];
      if constexpr (EPI == EPI_RESID) *y += v;
      else *y = v;
    }
  }
}

template <int FMT, int EPI>
static void dispatch_nb(const GemvArgs& a, int nb, cudaStream_t s, bool pdl) {
  const int rows_per_cta = (EPI == EPI_SWIGLU_Q8) ? 32 : 8;
  dim3 grid((a.N + rows_per_cta - 1) / rows_per_cta), block(256);
#define HK_NB(n) \
  case n: launch(gemv_kernel<FMT, n, EPI>, grid, block, 0, s, pdl, a); break;
  switch (nb) {
    HK_NB(1) HK_NB(2) HK_NB(3) HK_NB(4) HK_NB(5) HK_NB(6) HK_NB(7) HK_NB(8)
    default: throw std::runtime_error("gemv: batch columns must be 1..8");
  }
#undef HK_NB
}

template <int EPI>
static void dispatch_fmt(int fmt, const GemvArgs& a, int nb, cudaStream_t s, bool pdl) {
  switch (fmt) {
    case WF_Q4_K: dispatch_nb<WF_Q4_K, EPI>(a, nb, s, pdl); break;
    case WF_Q4_0: dispatch_nb<WF_Q4_0, EPI>(a, nb, s, pdl); break;
    case WF_Q8_0: dispatch_nb<WF_Q8_0, EPI>(a, nb, s, pdl); break;
    case WF_Q5_0: dispatch_nb<WF_Q5_0, EPI>(a, nb, s, pdl); break;
    case WF_Q6_K: dispatch_nb<WF_Q6_K, EPI>(a, nb, s, pdl); break;
    default: throw std::runtime_error("gemv: unsupported weight format " + std::to_string(fmt));
  }
}

void gemv_launch(int fmt, int epi, const GemvArgs& a, int nb, cudaStream_t s, bool pdl) {
  if (a.K % 128) throw std::runtime_error("gemv: K must be a multiple of 128");
  if (fmt == WF_Q4_K || fmt == WF_Q6_K) {
    if (a.K % 256) throw std::runtime_error("gemv: K-quant rows must be a multiple of 256");
  }
  switch (epi) {
    case EPI_STORE: dispatch_fmt<EPI_STORE>(fmt, a, nb, s, pdl); break;
    case EPI_RESID: dispatch_fmt<EPI_RESID>(fmt, a, nb, s, pdl); break;
    case EPI_SWIGLU_Q8:
      if (a.N % 32) throw std::runtime_error("gemv swiglu: N must be a multiple of 32");
      dispatch_fmt<EPI_SWIGLU_Q8>(fmt, a, nb, s, pdl);
      break;
    default: throw std::runtime_error("gemv: bad epilogue");
  }
}

}  // namespace hk
