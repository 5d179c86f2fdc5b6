// Small-batch dequant GEMV (K1, bs 1..8): y[b, n] = sum_k W[n, k] * x[b, k] with W in a GGUF
// block format dequantised in registers and x as q8 activation blocks, int8 dot products (dp4a).
//
// Decode at batch 1 is a chain of dependent kernels, so each kernel's critical path is kept to
// one round trip to memory:
//  * one warp per output row (a gate/up row pair for SwiGLU); every lane issues all of its weight
//    loads (16-byte, L1-bypassing) before anything else, and the first loads are issued before
//    the programmatic-dependent-launch wait, overlapping the previous kernel's tail;
//  * the input can be the fp32 residual stream: the CTA then computes RMSNorm and the q8 blocks
//    itself into shared memory (XIN_NORM), removing the separate normalisation kernel;
//  * the SwiGLU variant runs clusters of 4 CTAs whose 32 rows form one q8 block of the output.
// Epilogues: STORE (y), RESID (y += acc, fp32 residual stream), SWIGLU_Q8 (h = silu(g) * u -> q8).
//
// Parity: replaces the reference's Q4_K/Q6_K/Q8_0 GEMV family (crates/hawking-core/shaders/quant.metal,
// gemm_q4_k_m_fused*, _pair* gate+up with SwiGLU, _add residual-fused variants, add_rmsnorm_fused_q8
// feeding them); numerics oracle crates/hawking-core/src/quant.rs:722 (gemv_q4_k_q8k).
#include "gemv.cuh"
#include "tp.cuh"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace hk {

// Format traits: the per-lane work item ("unit") and how many a lane loads per round. Q4_K /
// Q8_0 / Q4_0 use the coalesced chunk mapping (lane L owns units L + 32 i, adjacent lanes read
// adjacent bytes); Q6_K / Q5_0 use 128-element units.
template <int FMT> struct Fmt;
template <> struct Fmt<WF_Q4_K> {
  using T = ChunkQ4K;
  static constexpr int ELEMS = 64, UPL = 2, GPC = 4;
  static __device__ __forceinline__ void load(const WPlanes& w, int64_t r, int c, T& u) { load_chunk_q4k(w, r, c, u); }
  static __device__ __forceinline__ float dot(const T& u, int c, const int8_t* q, const float* d, const float* s) {
    return dot_chunk_q4k<GPC>(u, c, q, d, s);
  }
};
template <> struct Fmt<WF_Q8_0> {
  using T = ChunkQ8_0;
  static constexpr int ELEMS = 32, UPL = 4, GPC = 2;
  static __device__ __forceinline__ void load(const WPlanes& w, int64_t r, int c, T& u) { load_chunk_q8_0(w, r, c, u); }
  static __device__ __forceinline__ float dot(const T& u, int c, const int8_t* q, const float* d, const float* s) {
    return dot_chunk_q8_0<GPC>(u, c, q, d, s);
  }
};
template <> struct Fmt<WF_Q4_0> {
  using T = ChunkQ4_0;
  static constexpr int ELEMS = 32, UPL = 4, GPC = 2;
  static __device__ __forceinline__ void load(const WPlanes& w, int64_t r, int c, T& u) { load_chunk_q4_0(w, r, c, u); }
  static __device__ __forceinline__ float dot(const T& u, int c, const int8_t* q, const float* d, const float* s) {
    return dot_chunk_q4_0<GPC>(u, c, q, d, s);
  }
};
template <> struct Fmt<WF_Q6_K> {
  using T = UnitQ6K;
  static constexpr int ELEMS = 128, UPL = 1, GPC = 0;
  static __device__ __forceinline__ void load(const WPlanes& w, int64_t r, int c, T& u) { load_unit_q6k(w, r, c, u); }
  static __device__ __forceinline__ float dot(const T& u, int c, const int8_t* q, const float* d, const float* s) {
    return dot_unit_q6k(u, c, q, d, s);
  }
};
template <> struct Fmt<WF_Q5_0> {
  using T = UnitQ5_0;
  static constexpr int ELEMS = 128, UPL = 1, GPC = 0;
  static __device__ __forceinline__ void load(const WPlanes& w, int64_t r, int c, T& u) { load_unit_q5_0(w, r, c, u); }
  static __device__ __forceinline__ float dot(const T& u, int c, const int8_t* q, const float* d, const float* s) {
    return dot_unit_q5_0(u, c, q, d, s);
  }
};

// The activation source of one launch, resolved to plain pointers (global or shared memory).
struct XSrc {
  const int8_t* q;
  const float* d;
  const float* s;
  int64_t sq, ss;  // per-column strides
};

// One round: up to UPL units per lane (u = base + lane + 32 j).
template <int FMT>
__device__ __forceinline__ void load_round(const WPlanes& w, int64_t row, int base, int n_units,
                                           typename Fmt<FMT>::T (&r)[Fmt<FMT>::UPL]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < Fmt<FMT>::UPL; ++j) {
    const int u = base + lane + 32 * j;
    if (u < n_units) Fmt<FMT>::load(w, row, u, r[j]);
  }
}
template <int FMT, int NB>
__device__ __forceinline__ void dot_round(const typename Fmt<FMT>::T (&r)[Fmt<FMT>::UPL], int base, int n_units,
                                          const XSrc& x, int nb, float (&acc)[NB]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < Fmt<FMT>::UPL; ++j) {
    const int u = base + lane + 32 * j;
    if (u < n_units) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const int bb = b < nb ? b : 0;  // padded columns recompute column 0 and are discarded
        acc[b] += Fmt<FMT>::dot(r[j], u, x.q + bb * x.sq, x.d + bb * x.ss, x.s + bb * x.ss);
      }
    }
  }
}
// Full row dot: the first round was loaded by the caller (before the PDL wait), the rest stream.
template <int FMT, int NB>
__device__ __forceinline__ void row_dot(const WPlanes& w, int64_t row, int n_units,
                                        typename Fmt<FMT>::T (&first)[Fmt<FMT>::UPL], const XSrc& x, int nb,
                                        float (&acc)[NB]) {
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = 0.f;
  constexpr int STEP = 32 * Fmt<FMT>::UPL;
  dot_round<FMT, NB>(first, 0, n_units, x, nb, acc);
  for (int base = STEP; base < n_units; base += STEP) {
    typename Fmt<FMT>::T r[Fmt<FMT>::UPL];
    load_round<FMT>(w, row, base, n_units, r);
    dot_round<FMT, NB>(r, base, n_units, x, nb, acc);
  }
}

// CTA-cooperative RMSNorm + q8 of nb fp32 rows into shared memory. Thread t handles elements
// t + e * blockDim.x (EPT of them, all loaded before any reduction), so each warp owns whole
// 32-element blocks. Columns are processed one after another.
template <int EPT, int GPC>
__device__ __forceinline__ void norm_q8_to_smem(const GemvArgs& a, int nb, int8_t* sq, float* sd, float* ss,
                                                float* red) {
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31;
  const int K = a.K;
  float w[EPT];
#pragma unroll
  for (int e = 0; e < EPT; ++e) {
    const int i = tid + e * nt;
    w[e] = (i < K && a.norm_w) ? a.norm_w[i] : 1.f;
  }
  for (int b = 0; b < nb; ++b) {
    float v[EPT];
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const int i = tid + e * nt;
      v[e] = i < K ? a.x_f32[(int64_t)b * a.x_f32_stride + i] : 0.f;
    }
    float scale = 1.f;
    if (a.norm) {
      float s2 = 0.f;
#pragma unroll
      for (int e = 0; e < EPT; ++e) s2 += v[e] * v[e];
      s2 = warp_sum(s2);
      if (lane == 0) red[b * 32 + (tid >> 5)] = s2;
      __syncthreads();
      s2 = lane < (nt >> 5) ? red[b * 32 + lane] : 0.f;
      s2 = warp_sum(s2);
      scale = rsqrtf(s2 / K + a.eps);
    }
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const int i = tid + e * nt;
      if (i < K) {  // K % 32 == 0 and nt % 32 == 0: whole warps are in or out
        const float x = v[e] * scale * w[e];
        const float amax = warp_max(fabsf(x));
        const float d = amax / 127.f;
        const int q = amax > 0.f ? __float2int_rn(x / d) : 0;
        const float qs = warp_sum((float)q);
        sq[b * K + 16 * swz_granule<GPC>(i >> 4) + (i & 15)] = (int8_t)q;
        if (lane == 0) {
          sd[b * (K / 32) + (i >> 5)] = d;
          ss[b * (K / 32) + (i >> 5)] = d * qs;
        }
      }
    }
  }
  __syncthreads();
}

// Kernel: one warp per row (STORE / RESID) or per gate/up row pair (SWIGLU_Q8), 8 warps per CTA.
// SWIGLU_Q8 launches clusters of 4 CTAs: their 4 x 8 rows form one 32-element q8 block of the
// output, which the cluster's first CTA quantises after reading the other CTAs' values through
// distributed shared memory.
// This CTA's share of the next kernel's weights, prefetched into L2 by warp 0 in pieces of <= 4 KB
// (cp.async.bulk.prefetch: 16-byte aligned starts and sizes; nothing is written, no completion).
__device__ __forceinline__ void prefetch_next_weights(const GemvArgs& a) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  for (int r = 0; r < a.pf_n; ++r) {
    const int64_t total = a.pf_bytes[r];
    const int64_t per = (((total + gridDim.x - 1) / gridDim.x) + 15) & ~int64_t(15);
    const int64_t s0 = (int64_t)blockIdx.x * per, s1 = min(total, s0 + per);
    for (int64_t off = s0 + (int64_t)lane * 4096; off < s1; off += 32 * 4096) {
      const uint32_t len = (uint32_t)min((int64_t)4096, s1 - off) & ~15u;
      if (len) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.pf_ptr[r] + off), "r"(len) : "memory");
    }
  }
}

template <int FMT, int NB, int EPI, int XIN>
__global__ void __launch_bounds__(256, (NB == 1 && XIN == XIN_Q8) ? (EPI == EPI_SWIGLU_Q8 ? 3 : 4) : 1) gemv_kernel(GemvArgs a, int nb) {
  extern __shared__ __align__(16) uint8_t gsm[];
  __shared__ float red[8 * 32];
  __shared__ float hbuf[NB][8];
  constexpr int WARPS = 8;
  constexpr int UPL = Fmt<FMT>::UPL;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_units = a.K / Fmt<FMT>::ELEMS;
  const int64_t row = (int64_t)blockIdx.x * WARPS + warp;
  const bool live = row < a.N;

  // 1) first round of weights (independent of the producer kernel)
  typename Fmt<FMT>::T wg[UPL];
  typename Fmt<FMT>::T wu[EPI == EPI_SWIGLU_Q8 ? UPL : 1];
  if (live) {
    load_round<FMT>(a.w0, row, 0, n_units, wg);
    if constexpr (EPI == EPI_SWIGLU_Q8) load_round<FMT>(a.w1, row, 0, n_units, wu);
  }
  if (a.pf_n) prefetch_next_weights(a);
  pdl_wait();

  // 2) activations into shared memory (granule-swizzled, see swz_granule)
  XSrc x;
  {
    int8_t* sq = reinterpret_cast<int8_t*>(gsm);
    float* sd = reinterpret_cast<float*>(gsm + nb * a.K);
    float* ss = sd + nb * (a.K / 32);
    if constexpr (XIN == XIN_NORM) {
      constexpr int NT = WARPS * 32;
      constexpr int EPT = (4096 + NT - 1) / NT;
      norm_q8_to_smem<EPT, Fmt<FMT>::GPC>(a, nb, sq, sd, ss, red);
    } else {
      const int nt = blockDim.x, tid = threadIdx.x;
      const int kq16 = a.K / 16, ks = a.K / 32;
      for (int i = tid; i < nb * kq16; i += nt) {
        const int b = i / kq16, c = i - b * kq16;
        reinterpret_cast<int4*>(sq)[b * kq16 + swz_granule<Fmt<FMT>::GPC>(c)] =
            __ldg(reinterpret_cast<const int4*>(a.xq + (int64_t)b * a.x_stride_q) + c);
      }
      for (int i = tid; i < nb * ks; i += nt) {
        const int b = i / ks, c = i - b * ks;
        sd[i] = __ldg(a.xd + (int64_t)b * a.x_stride_s + c);
        ss[i] = __ldg(a.xs + (int64_t)b * a.x_stride_s + c);
      }
      __syncthreads();
    }
    x = XSrc{sq, sd, ss, a.K, a.K / 32};
  }

  // 3) dot products + epilogue
  if constexpr (EPI == EPI_SWIGLU_Q8) {
    float g[NB], u[NB];
    if (live) {
      row_dot<FMT, NB>(a.w0, row, n_units, wg, x, nb, g);
      row_dot<FMT, NB>(a.w1, row, n_units, wu, x, nb, u);
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      g[b] = live ? warp_sum(g[b]) : 0.f;
      u[b] = live ? warp_sum(u[b]) : 0.f;
    }
    if (lane == 0) {
#pragma unroll
      for (int b = 0; b < NB; ++b) hbuf[b][warp] = live ? g[b] / (1.f + __expf(-g[b])) * u[b] : 0.f;
    }
    pdl_launch();
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // every CTA's hbuf is written and visible to the cluster
    if (cluster.block_rank() == 0) {
      const int64_t n = (int64_t)(blockIdx.x / 4) * 32 + lane;  // this cluster's q8 block
      const float* src = cluster.map_shared_rank(&hbuf[0][0], lane >> 3);
      for (int b = warp; b < nb; b += WARPS) {
        const float v = src[b * 8 + (lane & 7)];
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
    }
    cluster.sync();  // the other CTAs' shared memory stays alive until the first CTA has read it
  } else if constexpr (EPI == EPI_PUSH) {
    // tensor parallel: partial rows to every rank's receive region, then one arrival per CTA
    float acc[NB];
    if (live) {
      row_dot<FMT, NB>(a.w0, row, n_units, wg, x, nb, acc);
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[b] = warp_sum(acc[b]);
    }
    pdl_launch();
    if (live && lane < nb) {
      float v = acc[0];
#pragma unroll
      for (int c = 1; c < NB; ++c)
        if (lane == c) v = acc[c];
      if (a.bias) v += a.bias[row];
      const uint32_t flag = (uint32_t)*a.push_epoch;
      for (int p = 0; p < a.push_n; ++p) ll_store(a.push_recv[p] + (int64_t)lane * a.N + row, __float_as_uint(v), flag);
    }
  } else {
    if (!live) { pdl_launch(); return; }
    float acc[NB];
    row_dot<FMT, NB>(a.w0, row, n_units, wg, x, nb, acc);
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = warp_sum(acc[b]);
    pdl_launch();
    if (lane < nb) {
      float v = acc[0];
#pragma unroll
      for (int c = 1; c < NB; ++c)
        if (lane == c) v = acc[c];
      float* y = a.y + (int64_t)lane * a.y_stride + row;
      if (a.bias) v += a.bias[row];
      if constexpr (EPI == EPI_RESID) *y += v;
      else *y = v;
      if constexpr (EPI == EPI_STORE) {
        if (a.argmax_slots)
          atomicMax(a.argmax_slots + (int64_t)lane * kArgmaxSlots + (row % kArgmaxSlots),
                    argmax_key(v, (int)(row + a.argmax_offset)));
      }
    }
  }
}

template <int FMT, int EPI, int XIN>
static void dispatch_nb(const GemvArgs& a, int nb, cudaStream_t s, bool pdl) {
  const int rows_per_cta = 8;
  const int threads = 256;
  dim3 grid((a.N + rows_per_cta - 1) / rows_per_cta), block(threads);
  const size_t smem = (size_t)nb * a.K + 2 * (size_t)nb * (a.K / 32) * 4;  // q8 activations staged in smem
  auto go = [&](auto kern) {
    if (smem > 48 * 1024) HK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (EPI == EPI_SWIGLU_Q8) launch_cluster(kern, grid, block, smem, s, pdl, 4, a, nb);
    else launch(kern, grid, block, smem, s, pdl, a, nb);
  };
  if (nb == 1) go(gemv_kernel<FMT, 1, EPI, XIN>);
  else if (nb == 2) go(gemv_kernel<FMT, 2, EPI, XIN>);
  else if (nb <= 4) go(gemv_kernel<FMT, 4, EPI, XIN>);
  else if (nb <= 8) go(gemv_kernel<FMT, 8, EPI, XIN>);
  else throw std::runtime_error("gemv: batch columns must be 1..8");
}

template <int EPI, int XIN>
static void dispatch_fmt(int fmt, const GemvArgs& a, int nb, cudaStream_t s, bool pdl) {
  switch (fmt) {
    case WF_Q4_K: dispatch_nb<WF_Q4_K, EPI, XIN>(a, nb, s, pdl); break;
    case WF_Q4_0: dispatch_nb<WF_Q4_0, EPI, XIN>(a, nb, s, pdl); break;
    case WF_Q8_0: dispatch_nb<WF_Q8_0, EPI, XIN>(a, nb, s, pdl); break;
    case WF_Q5_0: dispatch_nb<WF_Q5_0, EPI, XIN>(a, nb, s, pdl); break;
    case WF_Q6_K: dispatch_nb<WF_Q6_K, EPI, XIN>(a, nb, s, pdl); break;
    default: throw std::runtime_error("gemv: unsupported weight format " + std::to_string(fmt));
  }
}

void gemv_launch(int fmt, int epi, const GemvArgs& a, int nb, cudaStream_t s, bool pdl) {
  // whole weight units: 32-element chunks (Q4_0 / Q8_0), 128-element units (Q5_0), 256 (K-quants)
  if (a.K % 32 || ((fmt == WF_Q5_0) && a.K % 128)) throw std::runtime_error("gemv: K must be a multiple of the weight unit");
  if ((fmt == WF_Q4_K || fmt == WF_Q6_K) && a.K % 256) throw std::runtime_error("gemv: K-quant rows need K % 256 == 0");
  if (a.K > 65536) throw std::runtime_error("gemv: K too large for the shared activation buffer");
  if (epi == EPI_SWIGLU_Q8 && a.N % 32) throw std::runtime_error("gemv swiglu: N must be a multiple of 32");
  if (a.x_f32) {  // fused RMSNorm -> q8 prologue (K <= 4096)
    if (a.K > 4096) throw std::runtime_error("gemv: the fused-norm input path needs K <= 4096");
    if (epi == EPI_STORE) dispatch_fmt<EPI_STORE, XIN_NORM>(fmt, a, nb, s, pdl);
    else if (epi == EPI_SWIGLU_Q8) dispatch_fmt<EPI_SWIGLU_Q8, XIN_NORM>(fmt, a, nb, s, pdl);
    else throw std::runtime_error("gemv: fused-norm input supports STORE and SWIGLU_Q8");
    return;
  }
  switch (epi) {
    case EPI_STORE: dispatch_fmt<EPI_STORE, XIN_Q8>(fmt, a, nb, s, pdl); break;
    case EPI_RESID: dispatch_fmt<EPI_RESID, XIN_Q8>(fmt, a, nb, s, pdl); break;
    case EPI_PUSH:
      if (!a.push_recv || !a.push_epoch || a.push_n <= 0) throw std::runtime_error("gemv push: peer tables required");
      dispatch_fmt<EPI_PUSH, XIN_Q8>(fmt, a, nb, s, pdl);
      break;
    case EPI_SWIGLU_Q8: dispatch_fmt<EPI_SWIGLU_Q8, XIN_Q8>(fmt, a, nb, s, pdl); break;
    default: throw std::runtime_error("gemv: bad epilogue");
  }
}

}  // namespace hk
