// Full-precision small-batch dequant GEMV (K1, batch 1..8): y[b, n] = sum_k W[n, k] * x[b, k] with
// W in GGUF Q4_K and x in bf16 (W4A16), fp32 accumulation. Default decode path for batches <= 8.
//
// Design (sm_100a, batch <= 8 is a bandwidth problem with a small matrix multiply inside it):
//  * Weight layout. At load time every [N, K] Q4_K matrix is re-laid (losslessly) into tiles of
//    16 rows x 256 columns: the 16 rows' 16-byte super-block headers, then the 2048 quant bytes
//    in the register-fragment order of mma.sync m16n8k16 (lane t of a warp finds the 8 nibbles of
//    its A fragment for one k-step in one 32-bit word, four k-steps per 16-byte load). Tiles are
//    stored row-group major, so any contiguous range of tiles is one contiguous byte range.
//  * Streaming. The tiles are split into gridDim.x * 8 contiguous, equal ranges, one per warp (two
//    or three CTAs of 8 warps per SM). Each
//    warp owns a ring of 2 stages of 2 tiles in shared memory, each stage filled by one cp.async.bulk
//    (the TMA copy engine, completing on an mbarrier); lane 0 issues the first copies before the
//    programmatic-dependent-launch wait, so a kernel's weights stream in while the kernel before it
//    finishes. No multicast (the kernel may run in multi-GPU processes).
//  * Math. A nibble n becomes the bf16 value 1 + n/16 with one shift and one lop3 (the nibble lands
//    in the top four mantissa bits of 1.0). acc1 = sum_k (1 + n_k/16) x_k comes from mma.sync with
//    fp32 accumulation, acc2 = sum_k x_k from a second mma against an all-ones fragment, and the
//    sub-block's contribution d*sc*sum(n x) - dmin*mn*sum(x) = S16 * acc1 - (S16 + dmin*mn) * acc2
//    with S16 = 16 * d * sc is applied in fp32 per 32-element sub-block. The weight enters the
//    tensor core as exact small integers, so the only rounding of operands is x to bf16.
//    Why mma.sync and not tcgen05 here: at batch <= 8 the dequantised A operand would have to be
//    written to shared memory for tcgen05 (2 bytes per weight, then read again by the tensor core),
//    which at the HBM weight rate exceeds the SM's shared-memory bandwidth; mma.sync takes A from
//    registers, where the dequantisation leaves it.
//  * Split-K fix-up, deterministic. A row group (16 rows) split over several warps: each writes its
//    partial fragment to scratch (two slots per warp: the first and last row group of its range),
//    bumps the row group's counter, and the warp that completes the count sums the partials in
//    warp order (fixed, independent of arrival order), runs the epilogue and clears the counter.
//  * Activations. x is staged in shared memory in the B-fragment order (from fp32 rows with a fused
//    RMSNorm, or from bf16 rows), or read in that order from global memory (the SwiGLU epilogue of
//    the gate/up GEMV writes h that way for the down projection, whose K is too wide to stage).
//  * Epilogues: STORE (y = v + bias, optional fused greedy keys), RESID (y += v), SWIGLU (gate and
//    up rows of the fused [gate | up] matrix are interleaved 8 + 8 in each tile, so one lane holds a
//    gate value and its up value: h = silu(g) * u in registers), PUSH (tensor parallel: flagged
//    words into every rank's receive region, as the dp4a GEMV's push epilogue).
//
// Every mbarrier wait is bounded (HK_ERR_MBAR_TIMEOUT in the status word); a warp that gives up
// waits (bounded) for its own copies still in flight before it exits.
//
// Parity: crates/hawking-core/shaders/quant.metal gemm_q4_k_m_fused* (f32 activations, the
// reference's default; its W4A8 GEMV is held off as quality-blocked in
// workspace/docs/reference/env_flags.md:38); Q4_K formula crates/hawking-core/src/quant.rs:34-160.
#include <cstdlib>

#include "mma_gemv.cuh"
#include "mg_device.cuh"
#include "sm100.cuh"
#include "tp.cuh"

namespace hk {
namespace mg {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
#ifndef HK_MG_STAGES
#define HK_MG_STAGES 2
#endif
#ifndef HK_MG_TPC
#define HK_MG_TPC 2
#endif
constexpr int kStages = HK_MG_STAGES;  // ring stages per warp
constexpr int kTpc = HK_MG_TPC;        // tiles per stage (one bulk copy each)
constexpr int kScaleBytes = 16 * 8 * 8;  // per warp: [16 rows][8 sub-blocks] float2 (S16, M'')
constexpr int kMaxCtasPerSm = 3;         // resident CTAs per SM (the partial scratch is sized for this)

__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t mask, uint32_t magic) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(magic));  // (a & mask) | magic
  return d;
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A * B (zero accumulator input): no zeroed registers to materialise per sub-block.
__device__ __forceinline__ void mma_bf16_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// Decode the 16 rows' Q4_K scales of one tile into per-warp shared memory. For sub-block k of a row
// the contribution is S_k * c_k - M_k * e_k with S = 16 * d * sc, M = S + dmin * mn, c_k / e_k the
// sub-block's sums of (1 + n/16) x and of x. The MMA accumulators run on across the tile's 8
// sub-blocks (cumulative C_k, E_k: no zeroing per sub-block), so by Abel summation the tile adds
// sum_k C_k (S_k - S_{k+1}) - E_k (M_k - M_{k+1}) with S_8 = M_8 = 0: the table holds those
// differences. Lane t handles row t/2, sub-blocks 4*(t&1) .. +3; the first sub-block of the upper
// half comes from the neighbouring lane.
__device__ __forceinline__ void decode_scales_q4k(const uint8_t* tile, float2* scs, int lane) {
  const int row = lane >> 1, half = lane & 1;
  const uint4 h = *reinterpret_cast<const uint4*>(tile + row * 16);
  const float d = __half2float(__ushort_as_half((uint16_t)(h.x & 0xFFFF)));
  const float dmin = __half2float(__ushort_as_half((uint16_t)(h.x >> 16)));
  // 6-bit scales / mins of the four sub-blocks as bytes (GGUF get_scale_min_k4, four at a time)
  const uint32_t scb = half ? ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u)) : (h.y & 0x3F3F3F3Fu);
  const uint32_t mnb = half ? (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u)) : (h.z & 0x3F3F3F3Fu);
  const float d16 = 16.f * d;
  const float c_sc = -d16 * 8388608.f, c_mn = -dmin * 8388608.f;
  float S[5], M[5];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // byte i placed in the mantissa of 2^23: the float 2^23 + byte, exact; one fma removes 2^23
    // and applies the scale with a single rounding
    const float scf = __uint_as_float(__byte_perm(scb, 0x4B000000u, 0x7650 + i));
    const float mnf = __uint_as_float(__byte_perm(mnb, 0x4B000000u, 0x7650 + i));
    S[i] = fmaf(d16, scf, c_sc);
    M[i] = S[i] + fmaf(dmin, mnf, c_mn);
  }
  const float s_up = __shfl_down_sync(0xffffffffu, S[0], 1), m_up = __shfl_down_sync(0xffffffffu, M[0], 1);
  S[4] = half ? 0.f : s_up;
  M[4] = half ? 0.f : m_up;
  float4* dst = reinterpret_cast<float4*>(scs + row * 8 + half * 4);
  dst[0] = make_float4(S[0] - S[1], M[0] - M[1], S[1] - S[2], M[1] - M[2]);
  dst[1] = make_float4(S[2] - S[3], M[2] - M[3], S[3] - S[4], M[3] - M[4]);
}

struct XFrag {
  const uint4* p;   // shared or global (generic address)
  int64_t cstride;  // uint4s between columns
};

// One tile: 16 rows x 256 columns (super-block s) accumulated into sum[4] (the lane's C fragment:
// rows r0, r0 + 8 x columns 2q, 2q + 1).
template <int NB, bool XGLOBAL>
__device__ __forceinline__ void consume_q4k(const uint8_t* tile, int s, const XFrag& x, int nb, float2* scs,
                                            int lane, float (&sum)[4]) {
  const int q = lane & 3, r0 = lane >> 2;
  // lanes of batch columns beyond nb read column 0 (valid data; their outputs are discarded)
  const int n = (lane >> 2) < nb ? (lane >> 2) : 0;
  // every load of the tile first (quants, activation fragments), so they are in flight together
  const uint4* qp = reinterpret_cast<const uint4*>(tile + 256) + lane;
  uint4 qv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) qv[j] = qp[j * 32];
  const uint4* xp = x.p + (n * (int)x.cstride + s * 32 + q * 2);
  // activations from global memory (long latency) are all requested up front; from shared memory
  // they are loaded per k-step group, right before use (fewer live registers, more resident warps)
  uint4 xv[XGLOBAL ? 8 : 2];
  if constexpr (XGLOBAL) {
#pragma unroll
    for (int j = 0; j < 8; ++j) xv[j] = __ldg(xp + (j >> 1) * 8 + (j & 1));
  }
  decode_scales_q4k(tile, scs, lane);
  __syncwarp();  // scales visible to every lane
  constexpr uint32_t ONES = 0x3F803F80u;
  constexpr uint32_t M = 0x00780078u;
  float c[4] = {0.f, 0.f, 0.f, 0.f}, e[4] = {0.f, 0.f, 0.f, 0.f};  // cumulative over the tile
#pragma unroll
  for (int j = 0; j < 4; ++j) {  // k-step groups of 4 (two sub-blocks)
    if constexpr (!XGLOBAL) {
      xv[0] = xp[j * 8];
      xv[1] = xp[j * 8 + 1];
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // sub-block 2j + h = k-steps 4j + 2h, 4j + 2h + 1
      const uint4 b = XGLOBAL ? xv[(2 * j + h) % (XGLOBAL ? 8 : 2)] : xv[h];
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const uint32_t w = pick(qv[j], 2 * h + kk);
        const uint32_t bx = kk ? b.z : b.x, by = kk ? b.w : b.y;
        mma_bf16(c, and_or(w << 3, M, ONES), and_or(w >> 1, M, ONES), and_or(w >> 5, M, ONES),
                 and_or(w >> 9, M, ONES), bx, by);
        mma_bf16(e, ONES, ONES, ONES, ONES, bx, by);
      }
      const int sb = 2 * j + h;
      const float2 s0 = scs[r0 * 8 + sb], s1 = scs[(r0 + 8) * 8 + sb];
      sum[0] = fmaf(s0.x, c[0], fmaf(-s0.y, e[0], sum[0]));
      sum[2] = fmaf(s1.x, c[2], fmaf(-s1.y, e[2], sum[2]));
      if (NB > 1) {
        sum[1] = fmaf(s0.x, c[1], fmaf(-s0.y, e[1], sum[1]));
        sum[3] = fmaf(s1.x, c[3], fmaf(-s1.y, e[3], sum[3]));
      }
    }
  }
  __syncwarp();  // every lane is done with the tile and the scales before they are overwritten
}

// Stage the activations of `nb` columns into shared memory as limbs + block info (integer math):
// each pair of threads quantises one 32-element block from registers.
template <int XIN>
__device__ __forceinline__ void stage_x_int(const MgArgs& a, uint8_t* xs, int64_t cstride, float2* info,
                                            int64_t istride, float* red) {
  const int tid = threadIdx.x, K = a.K, nblk = K / 32, h = tid & 1;
  uint4* xq = reinterpret_cast<uint4*>(xs);
  for (int n = 0; n < a.nb; ++n) {
    float scale = 1.f;
    if constexpr (XIN == MG_X_NORM) {
      const float4* xr = reinterpret_cast<const float4*>(a.x_f32 + (int64_t)n * a.x_f32_stride);
      float ss = 0.f;
      for (int i = tid; i < K / 4; i += kThreads) {
        const float4 v = xr[i];
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
      scale = rsqrtf(block_sum(ss, red) / (float)K + a.eps);
    }
    // every lane of a warp runs the same number of iterations (the pair shuffles need both lanes)
    for (int b0 = 0; b0 < nblk; b0 += kThreads / 2) {
      const int b = b0 + (tid >> 1);
      const bool on = b < nblk;
      float v[16];
      if (on) {
        if constexpr (XIN == MG_X_NORM) {
          const float* xr = a.x_f32 + (int64_t)n * a.x_f32_stride + 32 * b + 8 * h;
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const float4 x4 = *reinterpret_cast<const float4*>(xr + 16 * c + 4 * j);
              const float4 w4 = a.norm_w ? *reinterpret_cast<const float4*>(a.norm_w + 32 * b + 8 * h + 16 * c + 4 * j)
                                         : make_float4(1.f, 1.f, 1.f, 1.f);
              v[8 * c + 4 * j] = x4.x * scale * w4.x;
              v[8 * c + 4 * j + 1] = x4.y * scale * w4.y;
              v[8 * c + 4 * j + 2] = x4.z * scale * w4.z;
              v[8 * c + 4 * j + 3] = x4.w * scale * w4.w;
            }
        } else {
          load_half_block_bf16(a.xb + (int64_t)n * a.xb_stride, b, h, v);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
      }
      uint4 scratch[4];
      const float2 inf = quant_half_block(v, h, on ? xq + n * cstride + b * 4 : scratch);
      if (on && h == 0) info[(int64_t)n * istride + b] = inf;
    }
  }
  __syncthreads();
}

// Global two-limb quantiser (integer math, inputs too wide to stage): a lane pair per 32-block.
__global__ void __launch_bounds__(256) quant_limbs_kernel(const __nv_bfloat16* x, int64_t x_stride, int nb, int K,
                                                          uint4* out, int64_t cstride, float2* info) {
  pdl_wait();
  const int nblk = K / 32;
  const int t = blockIdx.x * blockDim.x + threadIdx.x, h = t & 1, pb = t >> 1;
  const bool on = pb < nb * nblk;
  const int n = on ? pb / nblk : 0, b = on ? pb - n * nblk : 0;
  float v[16];
  load_half_block_bf16(x + (int64_t)n * x_stride, b, h, v);
  uint4 scratch[4];
  const float2 inf = quant_half_block(v, h, on ? out + n * cstride + b * 4 : scratch);
  if (on && h == 0) info[(int64_t)n * nblk + b] = inf;
  pdl_launch();
}

// Store the bf16 value of x[n][k] into a B-fragment-order buffer.
__device__ __forceinline__ void frag_store_bf16(__nv_bfloat16* base, int64_t cstride, int n, int k, float v) {
  base[frag_u32(n, k & ~1, cstride) * 2 + (k & 1)] = __float2bfloat16_rn(v);
}

template <int EPI>
__device__ __forceinline__ void epilogue(const MgArgs& a, uint32_t g_, const float (&v)[4], int lane) {
  const int64_t g = g_;
  const int r0 = lane >> 2, q = lane & 3;
  if constexpr (EPI == MG_ROPE) {
    const RopeEpi r{a.rope, a.positions, a.row_seq, a.block_tables, a.max_blocks, a.block_size, a.k_cache,
                    a.v_cache, a.q_out, a.bias, a.nh, a.nkv, a.rp_hd, a.rp_rot, a.rp_style, a.cache_blocks};
    rope_epilogue<2>(r, a.nb, g_, v, lane);
  } else if constexpr (EPI == MG_SWIGLU) {
    const int64_t o = g * 8 + r0;  // output row: gate in tile row r0, up in r0 + 8
    if (o >= a.F) return;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int col = 2 * q + i;
      if (col < a.nb) {
        const float gt = v[i], up = v[2 + i];
        const float hv = gt / (1.f + __expf(-gt)) * up;
        if (a.hfrag) frag_store_bf16(a.hfrag, a.hfrag_cstride, col, (int)o, hv);
        if (a.hb) a.hb[(int64_t)col * a.hb_stride + o] = __float2bfloat16_rn(hv);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int64_t row = g * 16 + (i >> 1) * 8 + r0;
      const int col = 2 * q + (i & 1);
      if (row >= a.N || col >= a.nb) continue;
      if (EPI == MG_STORE && a.rp_heads) row = rope_unpermute(row, a.rp_hd, a.rp_rot, a.rp_style, a.rp_heads);
      float val = v[i];
      if (a.bias) val += a.bias[row];
      if constexpr (EPI == MG_PUSH) {
        const uint32_t flag = (uint32_t)*a.push_epoch;
        for (int p = 0; p < a.push_n; ++p)
          ll_store(a.push_recv[p] + (int64_t)col * a.N + row, __float_as_uint(val), flag);
      } else {
        float* yp = a.y + (int64_t)col * a.y_stride + row;
        if constexpr (EPI == MG_RESID) *yp += val;
        else *yp = val;
        if (EPI == MG_STORE && a.argmax_slots)
          atomicMax(a.argmax_slots + (int64_t)col * kArgmaxSlots + (row % kArgmaxSlots),
                    argmax_key(val, (int)(row + a.argmax_offset)));
      }
    }
  }
}

// Stage the activations of `nb` columns into shared memory in B-fragment order.
template <int XIN>
__device__ __forceinline__ void stage_x(const MgArgs& a, uint4* xs, int64_t cstride, float* red) {
  const int tid = threadIdx.x, K = a.K;
  uint32_t* xw = reinterpret_cast<uint32_t*>(xs);
  if constexpr (XIN == MG_X_BF16) {
    const int kp = K / 2;
    for (int i = tid; i < a.nb * kp; i += kThreads) {
      const int n = i / kp, k = 2 * (i - n * kp);
      xw[frag_u32(n, k, cstride)] = *reinterpret_cast<const uint32_t*>(a.xb + (int64_t)n * a.xb_stride + k);
    }
  } else {  // MG_X_NORM: RMSNorm of fp32 rows (K <= 8192: at most 8 float4 per thread)
    constexpr int MAXV = 8;
    const int nv = K / 4;
    for (int n = 0; n < a.nb; ++n) {
      const float4* xr = reinterpret_cast<const float4*>(a.x_f32 + (int64_t)n * a.x_f32_stride);
      float4 v[MAXV];
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < MAXV; ++e) {
        const int i = tid + e * kThreads;
        v[e] = i < nv ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        ss += v[e].x * v[e].x + v[e].y * v[e].y + v[e].z * v[e].z + v[e].w * v[e].w;
      }
      const float tot = block_sum(ss, red);
      const float scale = rsqrtf(tot / (float)K + a.eps);
#pragma unroll
      for (int e = 0; e < MAXV; ++e) {
        const int i = tid + e * kThreads;
        if (i < nv) {
          const float4 w = a.norm_w ? reinterpret_cast<const float4*>(a.norm_w)[i] : make_float4(1.f, 1.f, 1.f, 1.f);
          const __nv_bfloat162 p0 = __floats2bfloat162_rn(v[e].x * scale * w.x, v[e].y * scale * w.y);
          const __nv_bfloat162 p1 = __floats2bfloat162_rn(v[e].z * scale * w.z, v[e].w * scale * w.w);
          xw[frag_u32(n, 4 * i, cstride)] = *reinterpret_cast<const uint32_t*>(&p0);
          xw[frag_u32(n, 4 * i + 2, cstride)] = *reinterpret_cast<const uint32_t*>(&p1);
        }
      }
    }
  }
  __syncthreads();
}

template <int FMT, int MATH, int NB, int XIN, int EPI>
__global__ void __launch_bounds__(kThreads, MATH == MG_MATH_INT ? 2 : kMaxCtasPerSm) mg_gemv_kernel(MgArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int TB = Tile<FMT>::BYTES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem + warp * kStages * kTpc * TB;
  float2* scs = reinterpret_cast<float2*>(smem + kWarps * kStages * kTpc * TB + warp * kScaleBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * (kStages * kTpc * TB + kScaleBytes)) + warp * kStages;
  float* red = reinterpret_cast<float*>(smem + kWarps * (kStages * kTpc * TB + kScaleBytes) + kWarps * kStages * 8);
  uint4* xs = reinterpret_cast<uint4*>(smem + kWarps * (kStages * kTpc * TB + kScaleBytes) + kWarps * kStages * 8 + 128);

  const uint32_t T = (uint32_t)a.G * (uint32_t)a.KT;
  const uint32_t P = gridDim.x * kWarps;
  const uint32_t p = blockIdx.x * kWarps + warp;
  const uint32_t t0 = start_of(p, T, P), t1 = start_of(p + 1, T, P);
  const int n_tiles = (int)(t1 - t0);
  const uint32_t KT = (uint32_t)a.KT;

  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) sm100::mbar_init(&bars[s], 1);
    sm100::fence_barrier_init();
  }
  __syncwarp();
  // the warp's tiles stream in chunks of kTpc tiles, one bulk copy per chunk, kStages chunks ahead
  const int n_chunks = (n_tiles + kTpc - 1) / kTpc;
  auto issue = [&](int c) {
    const int st = c % kStages;
    const int cnt = min(kTpc, n_tiles - c * kTpc);
    sm100::mbar_arrive_expect_tx(&bars[st], (uint32_t)(cnt * TB));
    sm100::bulk_g2s(ring + st * kTpc * TB, a.tiles + (int64_t)(t0 + c * kTpc) * TB, (uint32_t)(cnt * TB), &bars[st]);
  };
  // weights first: they do not depend on the previous kernel
  int issued = n_chunks < kStages ? n_chunks : kStages;  // chunks issued; same value on every lane
  if (lane == 0)
    for (int k = 0; k < issued; ++k) issue(k);
  pdl_launch();
  pdl_wait();

  XFrag x;
  XInt xi;
  bool x_ok = true;
  if constexpr (MATH == MG_MATH_INT) {
    const int64_t cs = (int64_t)a.K / 8 + 1;  // limbs: 2K bytes per column, one spare uint4 (bank spread)
    const int64_t is = a.K / 32;
    float2* info = reinterpret_cast<float2*>(reinterpret_cast<uint8_t*>(xs) + (int64_t)a.nb * cs * 16);
    if constexpr (XIN == MG_X_FRAG_SMEM) {
      uint64_t* xbar = reinterpret_cast<uint64_t*>(red);
      if (threadIdx.x == 0) {
        sm100::mbar_init(xbar, 1);
        sm100::fence_barrier_init();
        const uint32_t colb = (uint32_t)a.K * 2, infb = (uint32_t)is * 8;
        sm100::mbar_arrive_expect_tx(xbar, (colb + infb) * (uint32_t)a.nb);
        for (int n = 0; n < a.nb; ++n) {
          sm100::bulk_g2s(xs + n * cs, a.xfrag + (int64_t)n * a.xfrag_cstride, colb, xbar);
          sm100::bulk_g2s(info + n * is, a.xinfo + (int64_t)n * is, infb, xbar);
        }
      }
      __syncthreads();
      x_ok = sm100::mbar_wait(xbar, 0, a.status);
      xi = XInt{xs, cs, info, is};
    } else if constexpr (XIN == MG_X_FRAG) {
      xi = XInt{a.xfrag, a.xfrag_cstride, a.xinfo, is};
    } else {
      stage_x_int<XIN>(a, reinterpret_cast<uint8_t*>(xs), cs, info, is, red);
      xi = XInt{xs, cs, info, is};
    }
  } else if constexpr (XIN == MG_X_FRAG_SMEM) {
    // fragment-order activations copied into shared memory, one bulk copy per column (2K bytes)
    const int64_t cs = (int64_t)a.K / 64 * 8 + 1;
    uint64_t* xbar = reinterpret_cast<uint64_t*>(red);  // the reduction scratch is unused in this mode
    if (threadIdx.x == 0) {
      sm100::mbar_init(xbar, 1);
      sm100::fence_barrier_init();
      const uint32_t colb = (uint32_t)a.K * 2;
      sm100::mbar_arrive_expect_tx(xbar, colb * (uint32_t)a.nb);
      for (int n = 0; n < a.nb; ++n)
        sm100::bulk_g2s(xs + n * cs, a.xfrag + (int64_t)n * a.xfrag_cstride, colb, xbar);
    }
    __syncthreads();
    x_ok = sm100::mbar_wait(xbar, 0, a.status);
    x.p = xs;
    x.cstride = cs;
  } else if constexpr (XIN == MG_X_FRAG) {
    x.p = a.xfrag;
    x.cstride = a.xfrag_cstride;
  } else {
    const int64_t cs = (int64_t)a.K / 64 * 8 + 1;  // one spare uint4 per column: bank spread
    stage_x<XIN>(a, xs, cs, red);
    x.p = xs;
    x.cstride = cs;
  }

  float sum[4] = {0.f, 0.f, 0.f, 0.f};
  int i = 0;
  bool ok = x_ok;  // a failed activation copy skips the tiles (the ring is drained below)
  uint32_t g = t0 / KT, s = t0 - g * KT;  // row group and column tile, advanced incrementally
  const uint32_t first_g = g;
  int st = 0, u = 0, c = 0;  // stage, tile within the chunk, chunk
  uint32_t phase = 0;
  for (; ok && i < n_tiles; ++i) {
    if (u == 0 && !sm100::mbar_wait(&bars[st], phase, a.status)) {
      ok = false;
      break;
    }
    const uint8_t* tile = ring + (st * kTpc + u) * TB;
    if constexpr (MATH == MG_MATH_INT) consume_q4k_int<NB>(tile, (int)s, xi, a.nb, scs, lane, sum);
    else consume_q4k<NB, XIN == MG_X_FRAG>(tile, (int)s, x, a.nb, scs, lane, sum);  // both end with __syncwarp
    if (++u == kTpc || i == n_tiles - 1) {  // chunk consumed: refill its stage
      if (c + kStages < n_chunks) {
        if (lane == 0) {
          sm100::fence_proxy_async_smem();  // this stage's generic reads before the async overwrite
          issue(c + kStages);
        }
        issued = c + kStages + 1;
      }
      u = 0;
      ++c;
      if (++st == kStages) {
        st = 0;
        phase ^= 1u;
      }
    }
    const bool last = (i == n_tiles - 1) || (s == KT - 1);
    if (++s == KT) s = 0;
    if (!last) continue;
    // row group g done for this warp: direct epilogue, or partial + deterministic fix-up
    const uint32_t pf = owner(g * KT, T, P), pl = owner(g * KT + KT - 1, T, P);
    if (pf == pl) {
      epilogue<EPI>(a, g, sum, lane);
    } else {
      const int slot = (g == first_g) ? 0 : 1;
      __stcg(a.part + ((int64_t)p * 2 + slot) * 32 + lane, make_float4(sum[0], sum[1], sum[2], sum[3]));
      __threadfence();
      int old = 0;
      if (lane == 0) old = atomicAdd(a.counters + g, 1);
      old = __shfl_sync(0xffffffffu, old, 0);
      // with T >= P no piece is empty: the contributors are exactly pf..pl
      const bool dense = T >= P;
      if (old == (dense ? (int)(pl - pf) : pieces_of_group(g, KT, T, P) - 1)) {
        __threadfence();
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        const int sl0 = (start_of(pf, T, P) / KT == g) ? 0 : 1;  // later pieces start inside g: slot 0
        // the contributing pieces in piece order (a fixed summation order); empty pieces skipped
        for (uint32_t pp = pf;; pp = dense ? pp + 1 : next_owner(pp, T, P)) {
          const int sl = pp == pf ? sl0 : 0;
          const float4 pv = __ldcg(a.part + ((int64_t)pp * 2 + sl) * 32 + lane);
          v[0] += pv.x;
          v[1] += pv.y;
          v[2] += pv.z;
          v[3] += pv.w;
          if (pp == pl) break;
        }
        if (lane == 0) a.counters[g] = 0;
        epilogue<EPI>(a, g, v, lane);
      }
    }
    sum[0] = sum[1] = sum[2] = sum[3] = 0.f;
    ++g;
  }
  if (!ok && lane == 0) {
    // wait (bounded) for this warp's copies still in flight before the CTA may exit
    for (int k = c; k < issued; ++k) sm100::mbar_wait(&bars[k % kStages], (uint32_t)((k / kStages) & 1), nullptr, 1u << 22);
  }
}

size_t smem_bytes(int fmt, int math, int xin, int nb, int K) {
  const size_t tb = (size_t)mg_tile_bytes(fmt);
  size_t s = kWarps * (kStages * kTpc * tb + kScaleBytes) + kWarps * kStages * 8 + 128;
  if (xin != MG_X_FRAG) {
    s += (size_t)nb * ((size_t)K / 8 + 1) * 16;                  // bf16 elements or the two int8 limbs
    if (math == MG_MATH_INT) s += (size_t)nb * ((size_t)K / 32) * 8;  // per-block (d2, sum)
  }
  return s;
}

// CTAs per SM a launch may use (HK_MG_PER_SM, default: as many as fit, at most kMaxCtasPerSm).
// Fewer leave shared memory free on every SM for the next kernel of the chain, whose CTAs then
// become resident at the programmatic launch and stream their first weight tiles while this
// kernel finishes.
inline int per_sm_cap() {
  static const int cap = [] {
    const char* e = getenv("HK_MG_PER_SM");
    const int v = e ? atoi(e) : 0;
    return v >= 1 && v <= kMaxCtasPerSm ? v : kMaxCtasPerSm;
  }();
  return cap;
}

template <int FMT, int MATH, int XIN, int EPI>
void dispatch_nb(const MgArgs& a, int sms, cudaStream_t st, bool pdl) {
  const size_t smem = smem_bytes(FMT, MATH, XIN, a.nb, a.K);
  auto go = [&](auto kern) {
    HK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 1;
    HK_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem));
    const int cap = per_sm_cap();
    per_sm = per_sm < 1 ? 1 : (per_sm > cap ? cap : per_sm);
    launch(kern, dim3(sms * per_sm), dim3(kThreads), smem, st, pdl, a);
  };
  if (a.nb == 1) go(mg_gemv_kernel<FMT, MATH, 1, XIN, EPI>);
  else if (a.nb == 2) go(mg_gemv_kernel<FMT, MATH, 2, XIN, EPI>);
  else if (a.nb <= 4) go(mg_gemv_kernel<FMT, MATH, 4, XIN, EPI>);
  else go(mg_gemv_kernel<FMT, MATH, 8, XIN, EPI>);
}

template <int FMT, int MATH, int XIN>
void dispatch_epi(int epi, const MgArgs& a, int grid, cudaStream_t st, bool pdl) {
  switch (epi) {
    case MG_STORE: dispatch_nb<FMT, MATH, XIN, MG_STORE>(a, grid, st, pdl); break;
    case MG_RESID: dispatch_nb<FMT, MATH, XIN, MG_RESID>(a, grid, st, pdl); break;
    case MG_SWIGLU: dispatch_nb<FMT, MATH, XIN, MG_SWIGLU>(a, grid, st, pdl); break;
    case MG_PUSH: dispatch_nb<FMT, MATH, XIN, MG_PUSH>(a, grid, st, pdl); break;
    case MG_ROPE:
      if constexpr (XIN == MG_X_NORM || XIN == MG_X_BF16) {
        dispatch_nb<FMT, MATH, XIN, MG_ROPE>(a, grid, st, pdl);
        break;
      }
      throw std::runtime_error("mg_gemv: the RoPE epilogue takes fp32 (normalised) or bf16 input");
    default: throw std::runtime_error("mg_gemv: bad epilogue");
  }
}

// ---- packing: GGUF Q4_K planes -> fragment-ordered tiles ------------------------------------
__global__ void pack_q4k_kernel(const uint8_t* qs, int64_t rb0, const uint8_t* hdr, int64_t rb1, const int* rowmap,
                                int G, int KT, uint32_t* out, int int_layout) {
  const int64_t total = (int64_t)G * KT * 576;  // 32-bit words per tile: 64 header + 512 quant
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tile = idx / 576;
    const int w = (int)(idx - tile * 576);
    const int64_t g = tile / KT;
    const int s = (int)(tile - g * KT);
    if (w < 64) {
      const int src = rowmap[g * 16 + (w >> 2)];
      out[idx] = src < 0 ? 0u
                         : *reinterpret_cast<const uint32_t*>(hdr + (int64_t)src * rb1 + (int64_t)s * 16 + (w & 3) * 4);
      continue;
    }
    const int qw = w - 64;  // ((j * 32 + t) * 4 + e
    const int t = (qw >> 2) & 31;
    auto nib = [&](int src, int e) -> uint32_t {
      if (src < 0) return 0u;
      const uint8_t b = qs[(int64_t)src * rb0 + (int64_t)s * 128 + 32 * (e >> 6) + (e & 31)];
      return (e & 32) ? (uint32_t)(b >> 4) : (uint32_t)(b & 15);
    };
    if (int_layout) {  // integer math: sub-block 2j + e/2, word e&1; byte i = row g | row g+8 << 4
      const int sb = (qw >> 7) * 2 + ((qw & 3) >> 1), word = qw & 1;
      const int g8 = t >> 2, q = t & 3, k0 = 32 * sb + 16 * word + 4 * q;
      const int s0 = rowmap[g * 16 + g8], s1 = rowmap[g * 16 + g8 + 8];
      uint32_t v = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) v |= (nib(s0, k0 + i) | (nib(s1, k0 + i) << 4)) << (8 * i);
      out[idx] = v;
      continue;
    }
    const int ks = (qw >> 7) * 4 + (qw & 3);
    const int r0 = t >> 2, q = t & 3, e0 = 16 * ks + 2 * q;
    const int s0 = rowmap[g * 16 + r0], s1 = rowmap[g * 16 + r0 + 8];
    out[idx] = nib(s0, e0) | nib(s0, e0 + 1) << 16 | nib(s1, e0) << 4 | nib(s1, e0 + 1) << 20 | nib(s0, e0 + 8) << 8 |
               nib(s0, e0 + 9) << 24 | nib(s1, e0 + 8) << 12 | nib(s1, e0 + 9) << 28;
  }
}

}  // namespace mg

// Largest fragment-order activation block copied into shared memory (two CTAs per SM still fit).
constexpr int64_t kFragSmemMax = 34 * 1024;

int mg_tile_bytes(int fmt) {
  switch (fmt) {
    case WF_Q4_K: return mg::Tile<WF_Q4_K>::BYTES;
    default: return 0;
  }
}

size_t mg_smem_bytes(int fmt, int math, int xin, int nb, int K) { return mg::smem_bytes(fmt, math, xin, nb, K); }

void mg_pack_launch(int fmt, int math, const WPlanes& w, const int* rowmap, int G, int KT, uint8_t* out,
                    cudaStream_t s) {
  if (fmt != WF_Q4_K) throw std::runtime_error("mg_pack: format not supported by the W4A16 GEMV");
  const int64_t total = (int64_t)G * KT * 576;
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>((total + threads - 1) / threads, 65536);
  mg::pack_q4k_kernel<<<blocks, threads, 0, s>>>(w.p0, w.rb0, w.p1, w.rb1, rowmap, G, KT,
                                                 reinterpret_cast<uint32_t*>(out), math == MG_MATH_INT ? 1 : 0);
  HK_CUDA_CHECK(cudaGetLastError());
}

void mg_quant_launch(const __nv_bfloat16* x, int64_t x_stride, int nb, int K, uint4* xfrag, int64_t cstride,
                     float2* xinfo, cudaStream_t s, bool pdl) {
  if (K % 256 || nb < 1 || nb > 8 || cstride < K / 8) throw std::runtime_error("mg_quant: bad shape");
  const int threads = 2 * nb * (K / 32);  // a lane pair per block
  launch(mg::quant_limbs_kernel, dim3((threads + 255) / 256), dim3(256), 0, s, pdl, x, x_stride, nb, K, xfrag,
         cstride, xinfo);
}

template <int MATH>
static void dispatch_xin(int xin, int epi, const MgArgs& a, int sms, cudaStream_t s, bool pdl) {
  switch (xin) {
    case MG_X_NORM: mg::dispatch_epi<WF_Q4_K, MATH, MG_X_NORM>(epi, a, sms, s, pdl); break;
    case MG_X_BF16: mg::dispatch_epi<WF_Q4_K, MATH, MG_X_BF16>(epi, a, sms, s, pdl); break;
    case MG_X_FRAG: {
      // stage the fragment-order activations in shared memory when they fit beside the rings
      int64_t bytes = (int64_t)a.nb * (a.K / 8 + 1) * 16;
      if (MATH == MG_MATH_INT) bytes += (int64_t)a.nb * (a.K / 32) * 8;
      if (bytes <= kFragSmemMax) mg::dispatch_epi<WF_Q4_K, MATH, MG_X_FRAG_SMEM>(epi, a, sms, s, pdl);
      else mg::dispatch_epi<WF_Q4_K, MATH, MG_X_FRAG>(epi, a, sms, s, pdl);
      break;
    }
    default: throw std::runtime_error("mg_gemv: bad input mode");
  }
}

void mg_gemv_launch(int fmt, int xin, int epi, const MgArgs& a, int sms, cudaStream_t s, bool pdl) {
  if (fmt != WF_Q4_K) throw std::runtime_error("mg_gemv: format not supported");
  if (a.nb < 1 || a.nb > 8) throw std::runtime_error("mg_gemv: batch columns must be 1..8");
  if (a.K % 256) throw std::runtime_error("mg_gemv: K must be a multiple of 256");
  if (xin == MG_X_NORM && a.K > 8192) throw std::runtime_error("mg_gemv: fused RMSNorm input needs K <= 8192");
  if (a.math != MG_MATH_BF16 && a.math != MG_MATH_INT) throw std::runtime_error("mg_gemv: bad math");
  if (a.math == MG_MATH_INT && xin == MG_X_FRAG && !a.xinfo) throw std::runtime_error("mg_gemv: block info required");
  if (xin != MG_X_FRAG && mg::smem_bytes(fmt, a.math, xin, a.nb, a.K) > 220 * 1024)
    throw std::runtime_error("mg_gemv: activations too wide to stage in shared memory (use the fragment input)");
  if (epi == MG_SWIGLU && !a.hfrag && !a.hb) throw std::runtime_error("mg_gemv swiglu: output buffer required");
  if ((epi == MG_STORE || epi == MG_RESID) && !a.y) throw std::runtime_error("mg_gemv: output y required");
  if (epi == MG_PUSH && (!a.push_recv || !a.push_epoch || a.push_n <= 0))
    throw std::runtime_error("mg_gemv push: peer tables required");
  if (!a.part || !a.counters) throw std::runtime_error("mg_gemv: scratch required");
  if ((uint64_t)a.G * a.KT * ((uint64_t)sms * mg::kMaxCtasPerSm * mg::kWarps + 1) >= (1ull << 32))
    throw std::runtime_error("mg_gemv: matrix too large for 32-bit tile arithmetic");
  if ((int64_t)a.nb * (a.K / 64 * 8 + 1) >= (1ll << 31)) throw std::runtime_error("mg_gemv: activation index overflow");
  if (a.math == MG_MATH_INT) dispatch_xin<MG_MATH_INT>(xin, epi, a, sms, s, pdl);
  else dispatch_xin<MG_MATH_BF16>(xin, epi, a, sms, s, pdl);
}

}  // namespace hk
