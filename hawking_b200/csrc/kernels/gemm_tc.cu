// Tensor-core dequant GEMM (K1, batch >= 16 and prefill): Y[M, N] (+)= X[M, K] . W[N, K]^T with W
// in GGUF Q4_K, X bf16, fp32 accumulation in TMEM via tcgen05.mma (kind::f16, M=128, N=BN, K=16),
// BN in {32, 64, 128, 256} (256 for prefill-sized M: the dequantised tile serves twice the tokens).
//
// One CTA owns a 128-row weight tile and a BN-token tile over a K range (split-K across
// blockIdx.z, reduced with fp32 atomics). Warp roles:
//   warp 0      TMA producer of the Q4_K bytes (16-byte header + 64 quant bytes per row per stage,
//               from the header and quants planes)
//   warp 1      TMA producer of the bf16 activation tile (128-byte swizzle, two 64-wide atoms)
//   warp 2      TMEM allocation and the single-thread UMMA issuer
//   warps 4-11  dequantisers: raw smem -> bf16 A tile in the canonical K-major SW128 layout
//               (bf16x2 FMAs of 128+q nibbles against the sub-block scale/min); warps 4-7 then run
//               the epilogue (tcgen05.ld 32x32b -> coalesced fp32 stores or atomics)
// Pipelines: raw (depth 4, TMA -> dequant warps), A (depth 2-3, dequant warps -> UMMA) and X
// (depth 2-4, TMA -> UMMA), A and X released by tcgen05.commit. All waits are bounded and report
// through the status word.
//
// SwiGLU variant (SW): the weight is the fused [gate | up] matrix of an FFN; tile i's 128 rows are
// gate rows [64 i, 64 i + 64) and the matching up rows [F + 64 i, ...) (two 64-row TMA boxes per
// plane), so one TMEM accumulator holds both halves of 64 FFN columns. The epilogue warps holding
// the up half park it in the (now idle) A stage buffers, and the gate half's warps write
// h = silu(g) * u as bf16: the fp32 gate/up activations never reach global memory.
// No TMA multicast is used (the kernel may run in multi-GPU processes).
//
// Numerics: the sub-block scale and min products are rounded to bf16 before the dequant FMA and
// the dequantised weight is bf16, i.e. W4A16 with bf16 weights, fp32 accumulate.
//
// Parity: crates/hawking-core/shaders/quant.metal gemm_q4_k_m_batched_v3w(_mma) (simdgroup-MMA batched
// Q4_K GEMM used by forward_tokens_batch_tcb / multiseq decode, crates/hawking-core/src/model/qwen_dense.rs:7569).
#include <cudaTypedefs.h>

#include <cstdlib>

#include "api.h"
#include "qformats.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace hk {
namespace {

using namespace sm100;

constexpr int BM = 128;        // weight rows per tile (UMMA M)
constexpr int BK = 128;        // K per stage (half a Q4_K super-block)
constexpr int DA = 2;          // A/X stages
constexpr int DR_MAX = 4;      // raw weight stages (2 at BN = 256, where shared memory is short)
constexpr int kDequantWarp0 = 4;
constexpr int kDequantWarps = 8;
constexpr uint32_t A_ATOM = BM * 128;       // 16 KB: 128 rows x 64 bf16
constexpr uint32_t A_STAGE = 2 * A_ATOM;    // 32 KB
constexpr uint32_t RAW_HDR = BM * 16;       // 2 KB
constexpr uint32_t RAW_QS = BM * 64;        // 8 KB

template <int BN>
struct Layout {
  static constexpr int DR = BN >= 256 ? 2 : DR_MAX;
  static constexpr uint32_t X_ATOM = BN * 128;
  static constexpr uint32_t X_STAGE = 2 * X_ATOM;
  static constexpr uint32_t off_a = 0;
  static constexpr uint32_t off_x = off_a + DA * A_STAGE;
  static constexpr uint32_t off_hdr = off_x + DA * X_STAGE;
  static constexpr uint32_t off_qs = off_hdr + DR * RAW_HDR;
  static constexpr uint32_t off_bar = off_qs + DR * RAW_QS;
  static constexpr uint32_t n_bars = 2 * DR + 2 * DA + 1;
  static constexpr uint32_t total = off_bar + n_bars * 8 + 16 + 1024;  // + alignment slack
  static_assert(total <= 232448, "tc_gemm: shared memory over the 227 KB per-CTA limit");
};

struct TcArgs {
  int N, K, M;
  int stages_total, stages_per_split;
  float* y;
  int64_t y_stride;
  int atomic;
  int serialize;
  int* status;
  __nv_bfloat16* h;   // SwiGLU output
  int64_t h_stride;
  int F;              // SwiGLU: FFN width (up rows start at F)
  // grouped (ABF only): CTA row blockIdx.y takes tile tiles[3 y .. 3 y + 2] = (group g, first
  // row, end row) of the gathered activations while y < *n_tiles; its weight rows are those of
  // group g (g * group_rows + the local row), its output columns the local rows
  const int* tiles;
  const int* n_tiles;
  int group_rows;
  // persistent kernel, stream-K: CTA b takes the units [b U / G, (b + 1) U / G) of the
  // U = tiles x K-stages units (tile major), accumulating partial tiles into y with atomics
  int stream_k;
};

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __nv_bfloat162 bits_bf2(uint32_t u) { return *reinterpret_cast<__nv_bfloat162*>(&u); }

// 4 consecutive nibbles (bytes b0..b3 of v, low or high nibble) -> two bf16x2 = q * s + o.
// (128 + q) is built exactly as a bf16 bit pattern, 128 is subtracted exactly, then one FMA.
__device__ __forceinline__ uint2 dq4(uint32_t v, int hi, __nv_bfloat162 s2, __nv_bfloat162 o2) {
  uint32_t t0 = __byte_perm(v, 0, 0x4140);  // [b0, 0, b1, 0]
  uint32_t t1 = __byte_perm(v, 0, 0x4342);  // [b2, 0, b3, 0]
  if (hi) { t0 >>= 4; t1 >>= 4; }
  const uint32_t p0 = (t0 & 0x000F000Fu) | 0x43004300u;  // bf16 (128 + q)
  const uint32_t p1 = (t1 & 0x000F000Fu) | 0x43004300u;
  const __nv_bfloat162 c128 = bits_bf2(0x43004300u);
  uint2 r;
  r.x = bf2_bits(__hfma2(__hsub2(bits_bf2(p0), c128), s2, o2));
  r.y = bf2_bits(__hfma2(__hsub2(bits_bf2(p1), c128), s2, o2));
  return r;
}

// Shared memory of the one-tile kernel: the activation tile has a ring of its own (DX stages,
// released by the MMA's commit), so its TMA loads run DX stages ahead instead of waiting for the
// A stage they used to share: at 64 tokens per tile every launch spent about 1.2 us per K stage
// with the activation load (L2 latency) on the critical path of each stage. Rings are deeper
// where shared memory allows (tiles of <= 64 tokens: 3 A stages, 4 activation stages).
template <int BN>
struct OLayout {
  static constexpr int DR = BN >= 256 ? 2 : DR_MAX;
  static constexpr int DA = BN <= 64 ? 3 : 2;
  static constexpr int DX = BN <= 64 ? 4 : (BN == 128 ? 3 : 2);
  // dequantising warps (half a weight row each); 16 warps with a quarter row each measured slower
  // at 64 tokens per tile (gate/up 66.8 -> 71.1 us)
  static constexpr int DQW = 8;
  static constexpr int THREADS = (kDequantWarp0 + DQW) * 32;
  static constexpr uint32_t X_ATOM = BN * 128;
  static constexpr uint32_t X_STAGE = 2 * X_ATOM;
  static constexpr uint32_t off_a = 0;
  static constexpr uint32_t off_x = off_a + DA * A_STAGE;
  static constexpr uint32_t off_hdr = off_x + DX * X_STAGE;
  static constexpr uint32_t off_qs = off_hdr + DR * RAW_HDR;
  static constexpr uint32_t off_bar = off_qs + DR * RAW_QS;
  static constexpr uint32_t n_bars = 2 * DR + 2 * DA + 2 * DX + 1;
  static constexpr uint32_t total = off_bar + n_bars * 8 + 16 + 1024;  // + alignment slack
  static_assert(total <= 232448, "tc_gemm: shared memory over the 227 KB per-CTA limit");
};

// ABF: the weights are bf16 [rows, K] already (a dequantised copy): warp 0 loads them with TMA
// straight into the A stages (tm_hdr is their map, tm_qs unused) and the dequantisers only run
// the epilogue.
template <int BN, bool SW, bool ABF>
__global__ void __launch_bounds__(OLayout<BN>::THREADS, 1)
    tc_gemm_q4k_kernel(const __grid_constant__ CUtensorMap tm_hdr, const __grid_constant__ CUtensorMap tm_qs,
                       const __grid_constant__ CUtensorMap tm_x, TcArgs a) {
  using L = OLayout<BN>;
  constexpr int DA = L::DA, DX = L::DX, DQW = L::DQW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::off_bar);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = bars + L::DR;
  uint64_t* a_full = bars + 2 * L::DR;
  uint64_t* a_empty = bars + 2 * L::DR + DA;
  uint64_t* x_full = bars + 2 * L::DR + 2 * DA;
  uint64_t* x_empty = x_full + DX;
  uint64_t* acc_full = x_empty + DX;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::n_bars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // SW: n0 is the tile's first gate row (64 per tile); otherwise its first weight row
  const int n0 = SW ? blockIdx.x * (BM / 2) : blockIdx.x * BM;
  int m0 = blockIdx.y * BN, m_end = a.M, nw0 = n0;  // nw0: first weight row in the (stacked) matrix
  if (ABF && a.tiles) {
    pdl_wait();  // the tile list comes from the previous kernel
    if ((int)blockIdx.y >= *a.n_tiles) return;  // the whole CTA, before any barrier or TMEM use
    const int* tl = a.tiles + 3 * blockIdx.y;
    nw0 = n0 + tl[0] * a.group_rows;
    m0 = tl[1];
    m_end = tl[2];
  }
  const int s0 = blockIdx.z * a.stages_per_split;
  const int s1 = min(a.stages_total, s0 + a.stages_per_split);
  const int nst = max(0, s1 - s0);
  constexpr uint32_t tmem_cols = BN < 32 ? 32 : BN;

  if (threadIdx.x == 0) {
    for (int i = 0; i < L::DR; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], DQW); }
    for (int i = 0; i < DA; ++i) { mbar_init(&a_full[i], ABF ? 1 : DQW); mbar_init(&a_empty[i], 1); }
    for (int i = 0; i < DX; ++i) { mbar_init(&x_full[i], 1); mbar_init(&x_empty[i], 1); }
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) { prefetch_tmap(&tm_hdr); prefetch_tmap(&tm_qs); prefetch_tmap(&tm_x); }
  if (warp == 2) tmem_alloc(tmem_slot, tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Weights do not depend on the previous kernel: only the raw producer skips the PDL wait
  // (a dequantised bf16 copy does: every warp waits).
  if (ABF || warp != 0) pdl_wait();

  if (nst > 0) {
    if (ABF && warp == 0 && lane == 0) {
      // ---- bf16 weight producer: TMA straight into the A stages ----
      int issued = 0;
      for (int i = 0; i < nst; ++i) {
        const int slot = i % DA;
        if (!mbar_wait(&a_empty[slot], ((i / DA) & 1) ^ 1, a.status)) break;
        const int gs = s0 + i;
        mbar_arrive_expect_tx(&a_full[slot], A_STAGE);
        uint8_t* as = smem + L::off_a + slot * A_STAGE;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          if constexpr (SW) {  // 64 gate rows, then the 64 matching up rows
            tma_load_2d(as + c * A_ATOM, &tm_hdr, gs * BK + c * 64, nw0, &a_full[slot]);
            tma_load_2d(as + c * A_ATOM + A_ATOM / 2, &tm_hdr, gs * BK + c * 64, a.F + nw0, &a_full[slot]);
          } else {
            tma_load_2d(as + c * A_ATOM, &tm_hdr, gs * BK + c * 64, nw0, &a_full[slot]);
          }
        }
        ++issued;
      }
      for (int i = max(0, issued - DA); i < issued; ++i) mbar_wait(&a_full[i % DA], (i / DA) & 1, nullptr, 1u << 22);
    } else if (!ABF && warp == 0 && lane == 0) {
      // ---- raw Q4_K producer ----
      int issued = 0;
      for (int i = 0; i < nst; ++i) {
        const int slot = i % L::DR;
        if (!mbar_wait(&raw_empty[slot], ((i / L::DR) & 1) ^ 1, a.status)) break;
        const int gs = s0 + i, sb = gs >> 1, h = gs & 1;
        mbar_arrive_expect_tx(&raw_full[slot], RAW_HDR + RAW_QS);
        if constexpr (SW) {  // 64 gate rows, then the 64 matching up rows (boxes of 64 rows)
          tma_load_2d(smem + L::off_hdr + slot * RAW_HDR, &tm_hdr, sb * 16, n0, &raw_full[slot]);
          tma_load_2d(smem + L::off_hdr + slot * RAW_HDR + RAW_HDR / 2, &tm_hdr, sb * 16, a.F + n0, &raw_full[slot]);
          tma_load_2d(smem + L::off_qs + slot * RAW_QS, &tm_qs, (2 * sb + h) * 64, n0, &raw_full[slot]);
          tma_load_2d(smem + L::off_qs + slot * RAW_QS + RAW_QS / 2, &tm_qs, (2 * sb + h) * 64, a.F + n0,
                      &raw_full[slot]);
        } else {
          tma_load_2d(smem + L::off_hdr + slot * RAW_HDR, &tm_hdr, sb * 16, n0, &raw_full[slot]);
          tma_load_2d(smem + L::off_qs + slot * RAW_QS, &tm_qs, (2 * sb + h) * 64, n0, &raw_full[slot]);
        }
        ++issued;
      }
      // Drain: every issued copy has landed before the CTA may exit.
      for (int i = max(0, issued - L::DR); i < issued; ++i) mbar_wait(&raw_full[i % L::DR], (i / L::DR) & 1, nullptr, 1u << 22);
    } else if (warp == 1 && lane == 0) {
      // ---- activation producer ----
      int issued = 0;
      for (int i = 0; i < nst; ++i) {
        const int slot = i % DX;
        if (!mbar_wait(&x_empty[slot], ((i / DX) & 1) ^ 1, a.status)) break;
        const int gs = s0 + i;
        mbar_arrive_expect_tx(&x_full[slot], L::X_STAGE);
        uint8_t* xs = smem + L::off_x + slot * L::X_STAGE;
        tma_load_2d(xs, &tm_x, gs * BK, m0, &x_full[slot]);
        tma_load_2d(xs + L::X_ATOM, &tm_x, gs * BK + 64, m0, &x_full[slot]);
        ++issued;
      }
      if (issued < nst) {  // error path: give copies in flight time to land before exiting
        for (int k = 0; k < 2000; ++k) __nanosleep(100);
      }
    } else if (warp == 2 && lane == 0) {
      // ---- UMMA issuer ----
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      bool ok = true;
      for (int i = 0; i < nst && ok; ++i) {
        const int slot = i % DA, xslot = i % DX;
        ok = mbar_wait(&a_full[slot], (i / DA) & 1, a.status) && mbar_wait(&x_full[xslot], (i / DX) & 1, a.status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + L::off_a + slot * A_STAGE);
        const uint32_t x_base = smem_u32(smem + L::off_x + xslot * L::X_STAGE);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = sdesc_k_sw128(a_base + c * A_ATOM + kk * 32);
            const uint64_t bd = sdesc_k_sw128(x_base + c * L::X_ATOM + kk * 32);
            umma_f16(tmem, ad, bd, idesc, (i | c | kk) != 0);
          }
        umma_commit(&a_empty[slot]);
        umma_commit(&x_empty[xslot]);
        if (a.serialize) ok = mbar_wait(&a_empty[slot], (i / DA) & 1, a.status);  // debug: no MMA/dequant overlap
      }
      umma_commit(acc_full);
    } else if (!ABF && warp >= kDequantWarp0 && warp < kDequantWarp0 + DQW) {
      // ---- dequantisers ----
      // TPR threads per weight row: thread (r, c, p) expands quant bytes [32 c + 16 p, + 16 NQ) of
      // the row's 64-byte chunk, i.e. the low nibbles into sub-block 2 c and the high nibbles into
      // sub-block 2 c + 1 of the stage's half super-block
      constexpr int TPR = DQW * 32 / BM;   // 2 or 4
      constexpr int NQ = 4 / TPR;          // 16-byte quant pieces per thread: 2 or 1
      const int t = (warp - kDequantWarp0) * 32 + lane;
      const int r = t / TPR, c = (t % TPR) / (TPR / 2), p = t % (TPR / 2);
      for (int i = 0; i < nst; ++i) {
        const int rs = i % L::DR, as = i % DA;
        const bool ok_raw = __shfl_sync(0xffffffffu, mbar_wait(&raw_full[rs], (i / L::DR) & 1, a.status), 0);
        if (!ok_raw) break;
        const uint4 hdr = *reinterpret_cast<const uint4*>(smem + L::off_hdr + rs * RAW_HDR + r * 16);
        uint32_t w[4 * NQ];
#pragma unroll
        for (int e = 0; e < NQ; ++e) {
          const uint4 qv = *reinterpret_cast<const uint4*>(smem + L::off_qs + rs * RAW_QS + r * 64 + c * 32 +
                                                           (p * NQ + e) * 16);
          w[4 * e] = qv.x;
          w[4 * e + 1] = qv.y;
          w[4 * e + 2] = qv.z;
          w[4 * e + 3] = qv.w;
        }
        const int gs = s0 + i, h = gs & 1;
        const int j0 = 4 * h + 2 * c;
        int sc0, mn0, sc1, mn1;
        q4k_scale_min(j0, hdr.y, hdr.z, hdr.w, sc0, mn0);
        q4k_scale_min(j0 + 1, hdr.y, hdr.z, hdr.w, sc1, mn1);
        const float d = __half2float(__ushort_as_half((uint16_t)(hdr.x & 0xFFFF)));
        const float dm = __half2float(__ushort_as_half((uint16_t)(hdr.x >> 16)));
        // w = q * (d * sc) - dmin * m, with the two products rounded to bf16
        const __nv_bfloat162 s2A = __float2bfloat162_rn(d * sc0), s2B = __float2bfloat162_rn(d * sc1);
        const __nv_bfloat162 o2A = __float2bfloat162_rn(-dm * mn0), o2B = __float2bfloat162_rn(-dm * mn1);
        const bool ok_a = __shfl_sync(0xffffffffu, mbar_wait(&a_empty[as], ((i / DA) & 1) ^ 1, a.status), 0);
        if (!ok_a) break;
        uint8_t* atom = smem + L::off_a + as * A_STAGE + c * A_ATOM;
#pragma unroll
        for (int cc = 0; cc < 2 * NQ; ++cc) {  // 16-byte chunk = 8 elements = 2 words
          const int ch = p * 2 * NQ + cc;
          const uint2 lo0 = dq4(w[2 * cc], 0, s2A, o2A), lo1 = dq4(w[2 * cc + 1], 0, s2A, o2A);
          const uint2 hi0 = dq4(w[2 * cc], 1, s2B, o2B), hi1 = dq4(w[2 * cc + 1], 1, s2B, o2B);
          *reinterpret_cast<uint4*>(atom + sw128_offset(r, ch)) = make_uint4(lo0.x, lo0.y, lo1.x, lo1.y);
          *reinterpret_cast<uint4*>(atom + sw128_offset(r, ch + 4)) = make_uint4(hi0.x, hi0.y, hi1.x, hi1.y);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&a_full[as]);
          mbar_arrive(&raw_empty[rs]);  // raw values were consumed above
        }
      }
    }

    // ---- epilogue: warps 4..7 (TMEM lane quarter = warp % 4) ----
    if (SW && warp >= kDequantWarp0 && warp < kDequantWarp0 + 4) {
      // lanes 0-63 hold gate rows, 64-127 the matching up rows: warps 6-7 park the up half in
      // the idle A stages ([64 rows][BN] fp32 = BN * 256 bytes <= 64 KB), warps 4-5 combine
      const bool ok = __shfl_sync(0xffffffffu, mbar_wait(acc_full, 0, a.status), 0);
      tc_fence_after();
      const int q = warp & 3;
      float* park = reinterpret_cast<float*>(smem + L::off_a);  // [BN / 8][64 rows][8]
      if (ok && q >= 2) {
#pragma unroll 1
        for (int j = 0; j < BN / 8; ++j) {
          float v[8];
          tmem_ld_x8(tmem + ((uint32_t)(q * 32) << 16) + j * 8, v);
          tmem_wait_ld();
          float4* dst = reinterpret_cast<float4*>(park + ((j * 64) + (q - 2) * 32 + lane) * 8);
          dst[0] = make_float4(v[0], v[1], v[2], v[3]);
          dst[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
      if (ok && q < 2) {
        const int f = n0 + q * 32 + lane;
#pragma unroll 1
        for (int j = 0; j < BN / 8; ++j) {
          float v[8];
          tmem_ld_x8(tmem + ((uint32_t)(q * 32) << 16) + j * 8, v);
          tmem_wait_ld();
          const float4* src = reinterpret_cast<const float4*>(park + ((j * 64) + q * 32 + lane) * 8);
          const float4 u0 = src[0], u1 = src[1];
          const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int m = m0 + j * 8 + e;
            if (m < m_end) a.h[(int64_t)m * a.h_stride + f] = __float2bfloat16(v[e] / (1.f + __expf(-v[e])) * u[e]);
          }
        }
      }
    } else if (!SW && warp >= kDequantWarp0 && warp < kDequantWarp0 + 4) {
      const bool ok = __shfl_sync(0xffffffffu, mbar_wait(acc_full, 0, a.status), 0);
      tc_fence_after();
      if (ok) {
        const int q = warp & 3;
        const int n = n0 + q * 32 + lane;
#pragma unroll 1
        for (int j = 0; j < BN / 8; ++j) {
          float v[8];
          tmem_ld_x8(tmem + ((uint32_t)(q * 32) << 16) + j * 8, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int m = m0 + j * 8 + e;
            if (m < m_end && n < a.N) {
              float* dst = a.y + (int64_t)m * a.y_stride + n;
              if (a.atomic) atomicAdd(dst, v[e]);
              else *dst = v[e];
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  pdl_launch();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
    tmem_relinquish();
  }
}

// ---- persistent variant (prefill-sized M, no split-K; stream-K for decode batches) --------------
// One CTA per SM walks the tiles t = blockIdx.x, + gridDim.x, ... (weight tile major, token tile
// minor, so the CTAs in flight share weight tiles in L2). Stream-K mode (TcArgs.stream_k, decode
// batches whose launch has more weight tiles than SMs): CTA b instead walks the units
// [b U / G, (b + 1) U / G) of the U = tiles x K-stages (tile major), i.e. a partial tile, whole
// tiles, a partial tile; every segment gets its own accumulator buffer and the epilogue adds it
// into y with atomics (zeroed or residual y), so no launch ends in a partial wave of whole tiles.
// The activation tile has a ring of its own (released by the MMA's commit, as in the one-tile
// kernel). Every role runs its own loop over the
// same tile sequence with stage counters that continue across tiles, and the accumulator is
// double-buffered in TMEM (2 x BN columns): the four dedicated epilogue warps drain tile j while
// the issuer and the dequantisers already fill tile j + 1, so neither the epilogue nor a partial
// last wave stalls the tensor cores. Stages are those of the one-tile kernel (K = 128: half a
// Q4_K super-block, two 128-byte swizzle atoms of A and of X); 64-wide stages with twice the
// depth measured slower (the per-stage hand-offs dominate).
//   warp 0 raw Q4_K TMA producer, warp 1 activation TMA producer, warp 2 TMEM owner + UMMA issuer,
//   warps 4-11 dequantisers, warps 12-15 epilogue (TMEM lane quarter = warp % 4). (Sixteen
//   dequantising warps with half the work each measured no faster.)
constexpr int kPThreads = 512;
constexpr int kPDequantWarps = kDequantWarps;
constexpr int kPEpi0 = kDequantWarp0 + kPDequantWarps;

template <int BN>
struct PLayout {
  // rings as in the one-tile kernel: A (dequantisers -> UMMA), X (TMA -> UMMA) and raw (TMA ->
  // dequantisers), deeper where shared memory allows (tiles of 64 tokens: 3 A, 4 X stages)
  static constexpr int DR = BN >= 256 ? 2 : DR_MAX;
  static constexpr int DA = BN <= 64 ? 3 : 2;
  static constexpr int DX = BN <= 64 ? 4 : 2;
  static constexpr uint32_t X_ATOM = BN * 128;
  static constexpr uint32_t X_STAGE = 2 * X_ATOM;
  static constexpr uint32_t off_a = 0;
  static constexpr uint32_t off_x = off_a + DA * A_STAGE;
  static constexpr uint32_t off_hdr = off_x + DX * X_STAGE;
  static constexpr uint32_t off_qs = off_hdr + DR * RAW_HDR;
  static constexpr uint32_t off_park = off_qs + DR * RAW_QS;       // SwiGLU exchange [2][64][8] fp32
  static constexpr uint32_t off_bar = off_park + 2 * 64 * 8 * 4;
  static constexpr uint32_t n_bars = 2 * DR + 2 * DA + 2 * DX + 4;
  static constexpr uint32_t total = off_bar + n_bars * 8 + 16 + 1024;
  static_assert(total <= 232448, "tc_gemm persistent: shared memory over the 227 KB per-CTA limit");
};

template <int BN, bool SW>
__global__ void __launch_bounds__(kPThreads, 1)
    tc_gemm_q4k_persistent(const __grid_constant__ CUtensorMap tm_hdr, const __grid_constant__ CUtensorMap tm_qs,
                           const __grid_constant__ CUtensorMap tm_x, TcArgs a) {
  using P = PLayout<BN>;
  using L = P;  // ring offsets
  constexpr int PDR = P::DR, PDA = P::DA, PDX = P::DX;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P::off_bar);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = bars + PDR;
  uint64_t* a_full = bars + 2 * PDR;
  uint64_t* a_empty = bars + 2 * PDR + PDA;
  uint64_t* x_full = bars + 2 * PDR + 2 * PDA;
  uint64_t* x_empty = x_full + PDX;
  uint64_t* acc_full = x_empty + PDX;              // [2]
  uint64_t* acc_empty = acc_full + 2;              // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + P::n_bars);
  float* park = reinterpret_cast<float*>(smem + P::off_park);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int RB = SW ? BM / 2 : BM;  // weight rows (gate rows under SW) a tile advances by
  const int m_tiles = (a.M + BN - 1) / BN;
  const int n_tiles = SW ? a.F / RB : a.N / BM;
  const int tiles = m_tiles * n_tiles;
  const int nst = a.K / BK;
  constexpr uint32_t tmem_cols = 2 * BN;
  // work list: tiles blockIdx.x, + gridDim.x, ... (whole K each), or under stream-K one balanced
  // range of (tile, stage) units; segment j is a run of stages [ka, kb) of one tile t
  const int64_t units = (int64_t)tiles * nst;
  const int64_t u_lo = a.stream_k ? units * blockIdx.x / gridDim.x : 0;
  const int64_t u_hi = a.stream_k ? units * (blockIdx.x + 1) / gridDim.x : 0;
  auto first_seg = [&](int& t, int& ka, int& kb) {
    if (a.stream_k) {
      t = (int)(u_lo / nst);
      ka = (int)(u_lo - (int64_t)t * nst);
      kb = (int)(ka + (u_hi - u_lo) < nst ? ka + (u_hi - u_lo) : nst);
      if (u_hi <= u_lo) t = tiles;
    } else {
      t = blockIdx.x;
      ka = 0;
      kb = nst;
    }
  };
  auto next_seg = [&](int& t, int& ka, int& kb) {
    if (a.stream_k) {
      const int64_t u = (int64_t)t * nst + kb;  // first unit after this segment
      if (u >= u_hi) {
        t = tiles;
        return;
      }
      t += 1;
      ka = 0;
      kb = (int)(u_hi - u < nst ? u_hi - u : nst);
    } else {
      t += gridDim.x;
    }
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < PDR; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], kPDequantWarps); }
    for (int i = 0; i < PDA; ++i) { mbar_init(&a_full[i], kPDequantWarps); mbar_init(&a_empty[i], 1); }
    for (int i = 0; i < PDX; ++i) { mbar_init(&x_full[i], 1); mbar_init(&x_empty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 4); }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) { prefetch_tmap(&tm_hdr); prefetch_tmap(&tm_qs); prefetch_tmap(&tm_x); }
  if (warp == 2) tmem_alloc(tmem_slot, tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp != 0) pdl_wait();  // weights do not depend on the previous kernel

  if (warp == 0 && lane == 0) {
    // ---- raw Q4_K producer: stage s = half (s & 1) of super-block (s >> 1) ----
    int it = 0;
    bool ok = true;
    int t, ka, kb;
    for (first_seg(t, ka, kb); t < tiles && ok; next_seg(t, ka, kb)) {
      const int n0 = (t / m_tiles) * RB;
      for (int s = ka; s < kb; ++s, ++it) {
        const int slot = it % PDR;
        if (!(ok = mbar_wait(&raw_empty[slot], ((it / PDR) & 1) ^ 1, a.status))) break;
        const int sbk = s >> 1, h = s & 1;
        mbar_arrive_expect_tx(&raw_full[slot], RAW_HDR + RAW_QS);
        uint8_t* hd = smem + L::off_hdr + slot * RAW_HDR;
        uint8_t* qd = smem + L::off_qs + slot * RAW_QS;
        if constexpr (SW) {
          tma_load_2d(hd, &tm_hdr, sbk * 16, n0, &raw_full[slot]);
          tma_load_2d(hd + RAW_HDR / 2, &tm_hdr, sbk * 16, a.F + n0, &raw_full[slot]);
          tma_load_2d(qd, &tm_qs, (2 * sbk + h) * 64, n0, &raw_full[slot]);
          tma_load_2d(qd + RAW_QS / 2, &tm_qs, (2 * sbk + h) * 64, a.F + n0, &raw_full[slot]);
        } else {
          tma_load_2d(hd, &tm_hdr, sbk * 16, n0, &raw_full[slot]);
          tma_load_2d(qd, &tm_qs, (2 * sbk + h) * 64, n0, &raw_full[slot]);
        }
      }
    }
    // drain: every issued copy has landed before the CTA may exit
    for (int i = max(0, it - PDR); i < it; ++i) mbar_wait(&raw_full[i % PDR], (i / PDR) & 1, nullptr, 1u << 22);
  } else if (warp == 1 && lane == 0) {
    // ---- activation producer ----
    int it = 0;
    bool ok = true;
    int t, ka, kb;
    for (first_seg(t, ka, kb); t < tiles && ok; next_seg(t, ka, kb)) {
      const int m0 = (t % m_tiles) * BN;
      for (int s = ka; s < kb; ++s, ++it) {
        const int slot = it % PDX;
        if (!(ok = mbar_wait(&x_empty[slot], ((it / PDX) & 1) ^ 1, a.status))) break;
        mbar_arrive_expect_tx(&x_full[slot], P::X_STAGE);
        uint8_t* xs = smem + P::off_x + slot * P::X_STAGE;
        tma_load_2d(xs, &tm_x, s * BK, m0, &x_full[slot]);
        tma_load_2d(xs + P::X_ATOM, &tm_x, s * BK + 64, m0, &x_full[slot]);
      }
    }
    if (!ok) for (int k = 0; k < 2000; ++k) __nanosleep(100);  // error path: let copies in flight land
  } else if (warp == 2 && lane == 0) {
    // ---- UMMA issuer ----
    constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
    int it = 0, j = 0;
    bool ok = true;
    int t, ka, kb;
    for (first_seg(t, ka, kb); t < tiles && ok; next_seg(t, ka, kb), ++j) {
      const int ab = j & 1;
      if (!(ok = mbar_wait(&acc_empty[ab], ((j >> 1) & 1) ^ 1, a.status))) break;
      tc_fence_after();
      const uint32_t acc = tmem + (uint32_t)(ab * BN);
      for (int s = ka; s < kb; ++s, ++it) {
        const int slot = it % PDA, xslot = it % PDX;
        if (!(ok = mbar_wait(&a_full[slot], (it / PDA) & 1, a.status) &&
                   mbar_wait(&x_full[xslot], (it / PDX) & 1, a.status)))
          break;
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + P::off_a + slot * A_STAGE);
        const uint32_t x_base = smem_u32(smem + P::off_x + xslot * P::X_STAGE);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(acc, sdesc_k_sw128(a_base + c * A_ATOM + kk * 32), sdesc_k_sw128(x_base + c * P::X_ATOM + kk * 32),
                     idesc, ((s - ka) | c | kk) != 0);
        umma_commit(&a_empty[slot]);
        umma_commit(&x_empty[xslot]);
      }
      if (ok) umma_commit(&acc_full[ab]);
    }
  } else if (warp >= kDequantWarp0 && warp < kPEpi0) {
    // ---- dequantisers: thread (row r, chunk c) expands the 32 quant bytes of chunk c of the
    // stage's half super-block (low nibbles: sub-block 4h + 2c, high: 4h + 2c + 1)
    const int tt = (warp - kDequantWarp0) * 32 + lane;
    const int r = tt >> 1, c = tt & 1;
    int it = 0;
    bool ok = true;
    int t, ka, kb;
    for (first_seg(t, ka, kb); t < tiles && ok; next_seg(t, ka, kb)) {
      for (int s = ka; s < kb; ++s, ++it) {
        const int rs = it % PDR, as = it % PDA;
        ok = __shfl_sync(0xffffffffu, mbar_wait(&raw_full[rs], (it / PDR) & 1, a.status), 0);
        if (!ok) break;
        const uint4 hdr = *reinterpret_cast<const uint4*>(smem + L::off_hdr + rs * RAW_HDR + r * 16);
        const uint4 q0 = *reinterpret_cast<const uint4*>(smem + L::off_qs + rs * RAW_QS + r * 64 + c * 32);
        const uint4 q1 = *reinterpret_cast<const uint4*>(smem + L::off_qs + rs * RAW_QS + r * 64 + c * 32 + 16);
        const int j0 = 4 * (s & 1) + 2 * c;
        int sc0, mn0, sc1, mn1;
        q4k_scale_min(j0, hdr.y, hdr.z, hdr.w, sc0, mn0);
        q4k_scale_min(j0 + 1, hdr.y, hdr.z, hdr.w, sc1, mn1);
        const float d = __half2float(__ushort_as_half((uint16_t)(hdr.x & 0xFFFF)));
        const float dm = __half2float(__ushort_as_half((uint16_t)(hdr.x >> 16)));
        const __nv_bfloat162 s2A = __float2bfloat162_rn(d * sc0), s2B = __float2bfloat162_rn(d * sc1);
        const __nv_bfloat162 o2A = __float2bfloat162_rn(-dm * mn0), o2B = __float2bfloat162_rn(-dm * mn1);
        ok = __shfl_sync(0xffffffffu, mbar_wait(&a_empty[as], ((it / PDA) & 1) ^ 1, a.status), 0);
        if (!ok) break;
        uint8_t* atom = smem + L::off_a + as * A_STAGE + c * A_ATOM;
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {  // 16-byte chunk = 8 elements = 2 words
          const uint2 lo0 = dq4(w[2 * ch], 0, s2A, o2A), lo1 = dq4(w[2 * ch + 1], 0, s2A, o2A);
          const uint2 hi0 = dq4(w[2 * ch], 1, s2B, o2B), hi1 = dq4(w[2 * ch + 1], 1, s2B, o2B);
          *reinterpret_cast<uint4*>(atom + sw128_offset(r, ch)) = make_uint4(lo0.x, lo0.y, lo1.x, lo1.y);
          *reinterpret_cast<uint4*>(atom + sw128_offset(r, ch + 4)) = make_uint4(hi0.x, hi0.y, hi1.x, hi1.y);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&a_full[as]);
          // the raw slot is released only after its values were consumed: releasing it right
          // after the shared-memory loads let the next TMA write overtake a load (rows of the
          // tile came out wrong in about one run in four)
          mbar_arrive(&raw_empty[rs]);
        }
      }
    }
  } else if (warp >= kPEpi0) {
    // ---- epilogue ----
    const int q = warp & 3;
    int j = 0;
    int t, ka, kb;
    for (first_seg(t, ka, kb); t < tiles; next_seg(t, ka, kb), ++j) {
      const int ab = j & 1;
      const bool ok = __shfl_sync(0xffffffffu, mbar_wait(&acc_full[ab], (j >> 1) & 1, a.status), 0);
      if (!ok) break;
      tc_fence_after();
      const int n0 = (t / m_tiles) * RB, m0 = (t % m_tiles) * BN;
      const uint32_t acc = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BN);
      if constexpr (SW) {
        // lanes 0-63: gate rows n0.., lanes 64-127: the matching up rows; warps q = 2, 3 hand their
        // up values to warps q = 0, 1 through a two-slot park, 8 tokens at a time
        const int f = n0 + (q & 1) * 32 + lane;
#pragma unroll 1
        for (int cj = 0; cj < BN / 8; ++cj) {
          float v[8];
          tmem_ld_x8(acc + cj * 8, v);
          tmem_wait_ld();
          float* slot = park + ((cj & 1) * 64 + (q & 1) * 32 + lane) * 8;
          if (q >= 2) {
            reinterpret_cast<float4*>(slot)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4*>(slot)[1] = make_float4(v[4], v[5], v[6], v[7]);
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (q < 2) {
            const float4 u0 = reinterpret_cast<const float4*>(slot)[0], u1 = reinterpret_cast<const float4*>(slot)[1];
            const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int m = m0 + cj * 8 + e;
              if (m < a.M) a.h[(int64_t)m * a.h_stride + f] = __float2bfloat16(v[e] / (1.f + __expf(-v[e])) * u[e]);
            }
          }
          // slot cj & 1 is rewritten at cj + 2, after the next chunk's barrier: no second barrier
        }
      } else {
        const int n = n0 + q * 32 + lane;
#pragma unroll 1
        for (int cj = 0; cj < BN / 8; ++cj) {
          float v[8];
          tmem_ld_x8(acc + cj * 8, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int m = m0 + cj * 8 + e;
            if (m < a.M && n < a.N) {
              // accumulate with fire-and-forget reductions: a load-add-store would put a load
              // round trip per element on the epilogue (measured: prefill 43 -> 53 ms)
              float* dst = a.y + (int64_t)m * a.y_stride + n;
              if (a.atomic) atomicAdd(dst, v[e]);
              else *dst = v[e];
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  pdl_launch();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
    tmem_relinquish();
  }
}

// ---- CTA-pair persistent variant (cta_group::2) ------------------------------------------------
// A 2-CTA cluster owns a 256-weight-row x 256-token tile: each CTA dequantises its own 128 weight
// rows (A) and loads its own 128 tokens of the activation tile (B); rank 0 issues one
// M = 256, N = 256 pair MMA per K = 16 slice that reads both CTAs' shared memory, and each CTA's
// TMEM receives its 128 rows of the result. Per CTA this halves the activation bytes per FLOP
// (the operand the one-CTA kernel waits on: a 64 KB activation stage per 1.1k-cycle MMA stage),
// which leaves room for three operand stages. The peer's readiness reaches rank 0 through
// cluster-scope mbarrier arrivals (its dequantisers directly; its activation copies through a
// relay thread that waits for them locally); rank 0's commits arrive on both CTAs' barriers.
// No TMA multicast: every load goes from global memory into the loading CTA's own shared memory.
constexpr int kQDA = 3;  // operand stages
constexpr uint32_t Q_X_ATOM = 128 * 128;  // 128 tokens x 64 bf16
constexpr uint32_t Q_X_STAGE = 2 * Q_X_ATOM;
struct QLayout {
  static constexpr int DR = 2;
  static constexpr uint32_t off_a = 0;
  static constexpr uint32_t off_x = off_a + kQDA * A_STAGE;
  static constexpr uint32_t off_hdr = off_x + kQDA * Q_X_STAGE;
  static constexpr uint32_t off_qs = off_hdr + DR * RAW_HDR;
  static constexpr uint32_t off_park = off_qs + DR * RAW_QS;
  static constexpr uint32_t off_bar = off_park + 2 * 64 * 8 * 4;
  static constexpr uint32_t n_bars = 2 * DR + 2 * kQDA + 4;
  static constexpr uint32_t total = off_bar + n_bars * 8 + 16 + 1024;
  static_assert(total <= 232448, "tc_gemm pair: shared memory over the 227 KB per-CTA limit");
};

template <bool SW>
__global__ void __launch_bounds__(kPThreads, 1)
    tc_gemm_q4k_pair(const __grid_constant__ CUtensorMap tm_hdr, const __grid_constant__ CUtensorMap tm_qs,
                     const __grid_constant__ CUtensorMap tm_x, TcArgs a) {
  using L = QLayout;
  constexpr int PDR = L::DR, PDA = kQDA, BNP = 256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::off_bar);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = bars + PDR;
  uint64_t* a_full = bars + 2 * PDR;          // rank 0: the pair's stage is ready; rank 1: own copies landed
  uint64_t* a_empty = bars + 2 * PDR + PDA;   // both: rank 0's MMAs on the stage completed
  uint64_t* acc_full = bars + 2 * PDR + 2 * PDA;
  uint64_t* acc_empty = acc_full + 2;         // rank 0: both CTAs drained the accumulator
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::n_bars);
  float* park = reinterpret_cast<float*>(smem + L::off_park);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool lead = rank == 0;
  constexpr int RB = SW ? BM / 2 : BM;
  const int m_tiles = (a.M + BNP - 1) / BNP;
  const int n_tiles = SW ? a.F / (2 * RB) : a.N / (2 * BM);
  const int tiles = m_tiles * n_tiles;
  const int nst = a.K / BK;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  constexpr uint32_t tmem_cols = 2 * BNP;

  if (threadIdx.x == 0) {
    for (int i = 0; i < PDR; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], kPDequantWarps); }
    for (int i = 0; i < PDA; ++i) {
      mbar_init(&a_full[i], lead ? 2 * kPDequantWarps + 2 : 1);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 8); }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) { prefetch_tmap(&tm_hdr); prefetch_tmap(&tm_qs); prefetch_tmap(&tm_x); }
  if (warp == 2) tmem_alloc_pair(tmem_slot, tmem_cols);
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp != 0) pdl_wait();

  if (warp == 0 && lane == 0) {
    // ---- raw Q4_K producer (this CTA's 128 weight rows) ----
    int it = 0;
    bool ok = true;
    for (int t = pair; t < tiles && ok; t += pairs) {
      const int n0 = (t / m_tiles) * 2 * RB + (int)rank * RB;
      for (int s = 0; s < nst; ++s, ++it) {
        const int slot = it % PDR;
        if (!(ok = mbar_wait(&raw_empty[slot], ((it / PDR) & 1) ^ 1, a.status))) break;
        const int sb = s >> 1, h = s & 1;
        mbar_arrive_expect_tx(&raw_full[slot], RAW_HDR + RAW_QS);
        uint8_t* hd = smem + L::off_hdr + slot * RAW_HDR;
        uint8_t* qd = smem + L::off_qs + slot * RAW_QS;
        if constexpr (SW) {
          tma_load_2d(hd, &tm_hdr, sb * 16, n0, &raw_full[slot]);
          tma_load_2d(hd + RAW_HDR / 2, &tm_hdr, sb * 16, a.F + n0, &raw_full[slot]);
          tma_load_2d(qd, &tm_qs, (2 * sb + h) * 64, n0, &raw_full[slot]);
          tma_load_2d(qd + RAW_QS / 2, &tm_qs, (2 * sb + h) * 64, a.F + n0, &raw_full[slot]);
        } else {
          tma_load_2d(hd, &tm_hdr, sb * 16, n0, &raw_full[slot]);
          tma_load_2d(qd, &tm_qs, (2 * sb + h) * 64, n0, &raw_full[slot]);
        }
      }
    }
    for (int i = max(0, it - PDR); i < it; ++i) mbar_wait(&raw_full[i % PDR], (i / PDR) & 1, nullptr, 1u << 22);
  } else if (warp == 1 && lane == 0) {
    // ---- activation producer (this CTA's 128 tokens of the tile) ----
    int it = 0;
    bool ok = true;
    for (int t = pair; t < tiles && ok; t += pairs) {
      const int m0 = (t % m_tiles) * BNP + (int)rank * 128;
      for (int s = 0; s < nst; ++s, ++it) {
        const int slot = it % PDA;
        if (!(ok = mbar_wait(&a_empty[slot], ((it / PDA) & 1) ^ 1, a.status))) break;
        mbar_arrive_expect_tx(&a_full[slot], Q_X_STAGE);
        uint8_t* xs = smem + L::off_x + slot * Q_X_STAGE;
        tma_load_2d(xs, &tm_x, s * BK, m0, &a_full[slot]);
        tma_load_2d(xs + Q_X_ATOM, &tm_x, s * BK + 64, m0, &a_full[slot]);
      }
    }
    if (!ok) for (int k = 0; k < 2000; ++k) __nanosleep(100);
  } else if (warp == 3 && lane == 0 && !lead) {
    // ---- relay (rank 1): this CTA's activation stage landed -> count it on rank 0's barrier ----
    int it = 0;
    bool ok = true;
    for (int t = pair; t < tiles && ok; t += pairs) {
      for (int s = 0; s < nst; ++s, ++it) {
        const int slot = it % PDA;
        if (!(ok = mbar_wait(&a_full[slot], (it / PDA) & 1, a.status))) break;
        mbar_arrive_cluster(&a_full[slot], 0);
      }
    }
  } else if (warp == 2 && lane == 0 && lead) {
    // ---- pair UMMA issuer ----
    constexpr uint32_t idesc = idesc_bf16_f32(2 * BM, BNP);
    int it = 0, j = 0;
    bool ok = true;
    for (int t = pair; t < tiles && ok; t += pairs, ++j) {
      const int ab = j & 1;
      if (!(ok = mbar_wait_cluster(&acc_empty[ab], ((j >> 1) & 1) ^ 1, a.status))) break;
      tc_fence_after();
      const uint32_t acc = tmem + (uint32_t)(ab * BNP);
      for (int s = 0; s < nst; ++s, ++it) {
        const int slot = it % PDA;
        if (!(ok = mbar_wait_cluster(&a_full[slot], (it / PDA) & 1, a.status))) break;
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + L::off_a + slot * A_STAGE);
        const uint32_t x_base = smem_u32(smem + L::off_x + slot * Q_X_STAGE);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_pair(acc, sdesc_k_sw128(a_base + c * A_ATOM + kk * 32), sdesc_k_sw128(x_base + c * Q_X_ATOM + kk * 32),
                          idesc, (s | c | kk) != 0);
        umma_commit_pair(&a_empty[slot], 0);
        umma_commit_pair(&a_empty[slot], 1);
      }
      if (ok) {
        umma_commit_pair(&acc_full[ab], 0);
        umma_commit_pair(&acc_full[ab], 1);
      }
    }
  } else if (warp >= kDequantWarp0 && warp < kPEpi0) {
    // ---- dequantisers (this CTA's 128 rows; same mapping as the one-CTA persistent kernel) ----
    const int tt = (warp - kDequantWarp0) * 32 + lane;
    const int r = tt >> 1, c = tt & 1;
    int it = 0;
    bool ok = true;
    for (int t = pair; t < tiles && ok; t += pairs) {
      for (int s = 0; s < nst; ++s, ++it) {
        const int rs = it % PDR, as = it % PDA;
        ok = __shfl_sync(0xffffffffu, mbar_wait(&raw_full[rs], (it / PDR) & 1, a.status), 0);
        if (!ok) break;
        const uint4 hdr = *reinterpret_cast<const uint4*>(smem + L::off_hdr + rs * RAW_HDR + r * 16);
        const uint4 q0 = *reinterpret_cast<const uint4*>(smem + L::off_qs + rs * RAW_QS + r * 64 + c * 32);
        const uint4 q1 = *reinterpret_cast<const uint4*>(smem + L::off_qs + rs * RAW_QS + r * 64 + c * 32 + 16);
        const int j0 = 4 * (s & 1) + 2 * c;
        int sc0, mn0, sc1, mn1;
        q4k_scale_min(j0, hdr.y, hdr.z, hdr.w, sc0, mn0);
        q4k_scale_min(j0 + 1, hdr.y, hdr.z, hdr.w, sc1, mn1);
        const float d = __half2float(__ushort_as_half((uint16_t)(hdr.x & 0xFFFF)));
        const float dm = __half2float(__ushort_as_half((uint16_t)(hdr.x >> 16)));
        const __nv_bfloat162 s2A = __float2bfloat162_rn(d * sc0), s2B = __float2bfloat162_rn(d * sc1);
        const __nv_bfloat162 o2A = __float2bfloat162_rn(-dm * mn0), o2B = __float2bfloat162_rn(-dm * mn1);
        ok = __shfl_sync(0xffffffffu, mbar_wait(&a_empty[as], ((it / PDA) & 1) ^ 1, a.status), 0);
        if (!ok) break;
        uint8_t* atom = smem + L::off_a + as * A_STAGE + c * A_ATOM;
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {  // 16-byte chunk = 8 elements = 2 words
          const uint2 lo0 = dq4(w[2 * ch], 0, s2A, o2A), lo1 = dq4(w[2 * ch + 1], 0, s2A, o2A);
          const uint2 hi0 = dq4(w[2 * ch], 1, s2B, o2B), hi1 = dq4(w[2 * ch + 1], 1, s2B, o2B);
          *reinterpret_cast<uint4*>(atom + sw128_offset(r, ch)) = make_uint4(lo0.x, lo0.y, lo1.x, lo1.y);
          *reinterpret_cast<uint4*>(atom + sw128_offset(r, ch + 4)) = make_uint4(hi0.x, hi0.y, hi1.x, hi1.y);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (lead) mbar_arrive(&a_full[as]);
          else mbar_arrive_cluster(&a_full[as], 0);
          mbar_arrive(&raw_empty[rs]);  // after the raw values were consumed
        }
      }
    }
  } else if (warp >= kPEpi0) {
    // ---- epilogue: this CTA's 128 weight rows x the tile's 256 tokens ----
    const int q = warp & 3;
    int j = 0;
    for (int t = pair; t < tiles; t += pairs, ++j) {
      const int ab = j & 1;
      const bool ok = __shfl_sync(0xffffffffu, mbar_wait(&acc_full[ab], (j >> 1) & 1, a.status), 0);
      if (!ok) break;
      tc_fence_after();
      const int n0 = (t / m_tiles) * 2 * RB + (int)rank * RB, m0 = (t % m_tiles) * BNP;
      const uint32_t acc = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BNP);
      if constexpr (SW) {
        const int f = n0 + (q & 1) * 32 + lane;
#pragma unroll 1
        for (int cj = 0; cj < BNP / 8; ++cj) {
          float v[8];
          tmem_ld_x8(acc + cj * 8, v);
          tmem_wait_ld();
          float* slot = park + ((cj & 1) * 64 + (q & 1) * 32 + lane) * 8;
          if (q >= 2) {
            reinterpret_cast<float4*>(slot)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4*>(slot)[1] = make_float4(v[4], v[5], v[6], v[7]);
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (q < 2) {
            const float4 u0 = reinterpret_cast<const float4*>(slot)[0], u1 = reinterpret_cast<const float4*>(slot)[1];
            const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int m = m0 + cj * 8 + e;
              if (m < a.M) a.h[(int64_t)m * a.h_stride + f] = __float2bfloat16(v[e] / (1.f + __expf(-v[e])) * u[e]);
            }
          }
        }
      } else {
        const int n = n0 + q * 32 + lane;
#pragma unroll 1
        for (int cj = 0; cj < BNP / 8; ++cj) {
          float v[8];
          tmem_ld_x8(acc + cj * 8, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int m = m0 + cj * 8 + e;
            if (m < a.M && n < a.N) {
              float* dst = a.y + (int64_t)m * a.y_stride + n;
              if (a.atomic) atomicAdd(dst, v[e]);
              else *dst = v[e];
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (lead) mbar_arrive(&acc_empty[ab]);
        else mbar_arrive_cluster(&acc_empty[ab], 0);
      }
    }
  }
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still signal it or read the pair's TMEM
  pdl_launch();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, tmem_cols);
    tmem_relinquish_pair();
  }
}

CUtensorMap make_map_2d(CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                        uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swz) {
  return tma_map_2d(dt, base, inner, outer, row_stride_bytes, box_inner, box_outer, swz);
}

template <int BN, bool SW>
void launch_bn(const TcGemmArgs& g, cudaStream_t s) {
  using L = OLayout<BN>;
  const uint64_t rb = (uint64_t)g.w_row_bytes, hb = (uint64_t)g.w_hdr_row_bytes;
  const uint32_t box_rows = SW ? BM / 2 : BM;
  CUtensorMap tm_hdr = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_UINT8, g.w_hdr, hb, g.N, hb, 16, box_rows,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
  CUtensorMap tm_qs = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_UINT8, g.w, rb, g.N, rb, 64, box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
  CUtensorMap tm_x = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, g.x, g.K, g.M, (uint64_t)g.x_stride * 2, 64, BN,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  TcArgs a;
  a.N = g.N;
  a.K = g.K;
  a.M = g.M;
  a.stages_total = g.K / BK;
  int splits = std::max(1, std::min(g.k_splits, a.stages_total));
  a.stages_per_split = (a.stages_total + splits - 1) / splits;
  splits = (a.stages_total + a.stages_per_split - 1) / a.stages_per_split;
  a.y = g.y;
  a.y_stride = g.y_stride;
  a.atomic = (g.atomic || splits > 1) ? 1 : 0;
  a.status = g.status;
  a.serialize = getenv("HK_GEMM_SERIALIZE") != nullptr;
  a.h = g.h;
  a.h_stride = g.h_stride;
  a.F = g.N / 2;
  if (SW && splits != 1) throw std::runtime_error("tc_gemm swiglu: no split-K");
  static bool attr_set = false;
  if (!attr_set) {
    HK_CUDA_CHECK(cudaFuncSetAttribute(tc_gemm_q4k_kernel<BN, SW, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::total));
    attr_set = true;
  }
  dim3 grid(g.N / BM, (g.M + BN - 1) / BN, splits);
  launch(tc_gemm_q4k_kernel<BN, SW, false>, grid, dim3(L::THREADS), L::total, s, g.pdl, tm_hdr, tm_qs, tm_x, a);
}

template <int BN, bool SW>
void launch_persistent(const TcGemmArgs& g, cudaStream_t s, bool stream_k = false) {
  using P = PLayout<BN>;
  const uint64_t rb = (uint64_t)g.w_row_bytes, hb = (uint64_t)g.w_hdr_row_bytes;
  const uint32_t box_rows = SW ? BM / 2 : BM;
  CUtensorMap tm_hdr = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_UINT8, g.w_hdr, hb, g.N, hb, 16, box_rows,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
  CUtensorMap tm_qs = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_UINT8, g.w, rb, g.N, rb, 64, box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
  CUtensorMap tm_x = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, g.x, g.K, g.M, (uint64_t)g.x_stride * 2, 64, BN,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  TcArgs a{};
  a.N = g.N;
  a.K = g.K;
  a.M = g.M;
  a.stages_total = g.K / BK;
  a.stages_per_split = a.stages_total;
  a.y = g.y;
  a.y_stride = g.y_stride;
  a.atomic = (g.atomic || stream_k) ? 1 : 0;
  a.stream_k = stream_k ? 1 : 0;
  a.status = g.status;
  a.h = g.h;
  a.h_stride = g.h_stride;
  a.F = g.N / 2;
  static bool attr_set = false;
  static int sms = 0;
  if (!attr_set) {
    HK_CUDA_CHECK(cudaFuncSetAttribute(tc_gemm_q4k_persistent<BN, SW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       P::total));
    int dev = 0;
    HK_CUDA_CHECK(cudaGetDevice(&dev));
    HK_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    attr_set = true;
  }
  const int tiles = ((g.M + BN - 1) / BN) * (g.N / BM);
  // stream-K: one CTA per SM (at least 4 K stages each), every CTA the same number of stages
  // within one; otherwise one CTA per tile up to one per SM
  const int64_t units = (int64_t)tiles * a.stages_total;
  const int grid = stream_k ? (int)std::max<int64_t>(1, std::min<int64_t>(sms, units / 4)) : std::min(tiles, sms);
  launch(tc_gemm_q4k_persistent<BN, SW>, dim3(grid), dim3(kPThreads), P::total, s, g.pdl, tm_hdr, tm_qs, tm_x, a);
}

// True when the CTA-pair kernel covers the shape (whole 256-row weight pair tiles).
bool pair_ok(const TcGemmArgs& g) {
  const char* e = getenv("HK_GEMM_PAIR");
  if (!e || e[0] != '1') return false;
  return g.bn == 256 && (g.h ? (g.N / 2) % 128 == 0 : g.N % 256 == 0);
}

template <bool SW>
void launch_pair(const TcGemmArgs& g, cudaStream_t s) {
  using L = QLayout;
  const uint64_t rb = (uint64_t)g.w_row_bytes, hb = (uint64_t)g.w_hdr_row_bytes;
  const uint32_t box_rows = SW ? BM / 2 : BM;
  CUtensorMap tm_hdr = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_UINT8, g.w_hdr, hb, g.N, hb, 16, box_rows,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
  CUtensorMap tm_qs = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_UINT8, g.w, rb, g.N, rb, 64, box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
  CUtensorMap tm_x = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, g.x, g.K, g.M, (uint64_t)g.x_stride * 2, 64, 128,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  TcArgs a{};
  a.N = g.N;
  a.K = g.K;
  a.M = g.M;
  a.stages_total = g.K / BK;
  a.stages_per_split = a.stages_total;
  a.y = g.y;
  a.y_stride = g.y_stride;
  a.atomic = g.atomic ? 1 : 0;
  a.status = g.status;
  a.h = g.h;
  a.h_stride = g.h_stride;
  a.F = g.N / 2;
  static bool attr_set = false;
  static int max_pairs = 0;
  if (!attr_set) {
    HK_CUDA_CHECK(cudaFuncSetAttribute(tc_gemm_q4k_pair<SW>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::total));
    // pairs that can be resident at once (a pair needs two SMs of one TPC)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = L::total;
    cudaLaunchAttribute at;
    at.id = cudaLaunchAttributeClusterDimension;
    at.val.clusterDim.x = 2;
    at.val.clusterDim.y = 1;
    at.val.clusterDim.z = 1;
    cfg.attrs = &at;
    cfg.numAttrs = 1;
    HK_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&max_pairs, tc_gemm_q4k_pair<SW>, &cfg));
    if (max_pairs < 1) throw std::runtime_error("tc_gemm pair: no CTA pair fits on this device");
    attr_set = true;
  }
  const int pair_tiles = ((g.M + 255) / 256) * (SW ? (g.N / 2) / 128 : g.N / 256);
  const int pairs = std::max(1, std::min(pair_tiles, max_pairs));
  launch_cluster(tc_gemm_q4k_pair<SW>, dim3(2 * pairs), dim3(kPThreads), L::total, s, g.pdl, 2, tm_hdr, tm_qs,
                 tm_x, a);
}

template <int BN, bool SW>
void launch_abf(const TcBf16Args& g, cudaStream_t s) {
  using L = OLayout<BN>;
  const uint32_t box_rows = SW ? BM / 2 : BM;
  CUtensorMap tm_a = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, g.w, g.K, g.w_rows, (uint64_t)g.w_stride * 2, 64,
                                 box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tm_x = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, g.x, g.K, g.x_rows, (uint64_t)g.x_stride * 2, 64, BN,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  TcArgs a{};
  a.N = g.N;
  a.K = g.K;
  a.M = g.M;
  a.stages_total = g.K / BK;
  int splits = g.tiles ? 1 : std::max(1, std::min(g.k_splits, a.stages_total));
  a.stages_per_split = (a.stages_total + splits - 1) / splits;
  splits = (a.stages_total + a.stages_per_split - 1) / a.stages_per_split;
  a.y = g.y;
  a.y_stride = g.y_stride;
  a.atomic = (g.atomic || splits > 1) ? 1 : 0;
  a.status = g.status;
  a.h = g.h;
  a.h_stride = g.h_stride;
  a.F = SW ? g.N / 2 : 0;
  a.tiles = g.tiles;
  a.n_tiles = g.n_tiles;
  a.group_rows = g.group_rows;
  if (SW && splits != 1) throw std::runtime_error("tc_gemm bf16 swiglu: no split-K");
  static bool attr_set = false;
  if (!attr_set) {
    HK_CUDA_CHECK(cudaFuncSetAttribute(tc_gemm_q4k_kernel<BN, SW, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       L::total));
    attr_set = true;
  }
  const int ty = g.tiles ? g.max_tiles : (g.M + BN - 1) / BN;
  if (ty <= 0) return;
  dim3 grid((g.N + BM - 1) / BM, ty, splits);
  launch(tc_gemm_q4k_kernel<BN, SW, true>, grid, dim3(L::THREADS), L::total, s, g.pdl, tm_a, tm_a, tm_x, a);
}

}  // namespace

void tc_gemm_bf16_launch(const TcBf16Args& g, cudaStream_t s) {
  // plain products may end in a partial 128-row weight tile (the TMA box reads zeros past the last
  // row, the epilogue stores rows < N only); SwiGLU pairs and expert groups are whole tiles
  if ((g.h || g.tiles) && g.N % BM) throw std::runtime_error("tc_gemm bf16: output rows must be a multiple of 128");
  if (g.K % BK) throw std::runtime_error("tc_gemm bf16: K must be a multiple of 128");
  if ((reinterpret_cast<uintptr_t>(g.w) | reinterpret_cast<uintptr_t>(g.x)) & 15 || (g.w_stride * 2) % 16 ||
      (g.x_stride * 2) % 16)
    throw std::runtime_error("tc_gemm bf16: operands must be 16-byte aligned rows");
  if (g.tiles && (g.group_rows % BM || g.group_rows != g.N)) throw std::runtime_error("tc_gemm bf16 grouped: group rows");
  if (g.k_splits > 1 && !g.atomic && !g.y_zeroed && !g.h) throw std::runtime_error("tc_gemm bf16: split-K needs a zeroed output");
  if (g.h) {
    switch (g.bn) {
      case 64: launch_abf<64, true>(g, s); break;
      case 128: launch_abf<128, true>(g, s); break;
      default: throw std::runtime_error("tc_gemm bf16 swiglu: bn must be 64 or 128");
    }
    return;
  }
  switch (g.bn) {
    case 32: launch_abf<32, false>(g, s); break;
    case 64: launch_abf<64, false>(g, s); break;
    case 128: launch_abf<128, false>(g, s); break;
    default: throw std::runtime_error("tc_gemm bf16: bn must be 32, 64 or 128");
  }
}

int tc_gemm_splits(int N, int M, int K, int bn, int sms) {
  const int tiles = (N / BM) * ((M + bn - 1) / bn);
  const int stages = K / BK;
  // one CTA fills an SM (shared memory): as many splits as keep the launch within one wave, since
  // a partial second wave costs a whole K slice (48 tiles: 3 splits / 144 CTAs, not 4 / 192)
  int splits = tiles >= sms ? 1 : sms / tiles;
  splits = std::min(splits, std::max(1, stages / 4));  // keep >= 4 stages per split
  return std::max(1, splits);
}

void tc_gemm_launch(const TcGemmArgs& g, cudaStream_t s) {
  if (g.fmt != WF_Q4_K) throw std::runtime_error("tc_gemm: only Q4_K weights are supported");
  if (g.N % BM) throw std::runtime_error("tc_gemm: N must be a multiple of 128");
  if (g.K % 256) throw std::runtime_error("tc_gemm: K must be a multiple of 256");
  if (g.k_splits > 1 && !g.atomic && !g.y_zeroed) throw std::runtime_error("tc_gemm: split-K needs a zeroed output");
  if (g.persistent == 2) {  // stream-K: balanced (tile, stage) ranges, partial tiles by atomics
    if (g.h) throw std::runtime_error("tc_gemm stream-K: no SwiGLU epilogue");
    if (!g.atomic && !g.y_zeroed) throw std::runtime_error("tc_gemm stream-K: needs a zeroed or accumulated output");
    switch (g.bn) {
      case 64: launch_persistent<64, false>(g, s, true); break;
      case 128: launch_persistent<128, false>(g, s, true); break;
      default: throw std::runtime_error("tc_gemm stream-K: bn must be 64 or 128");
    }
    return;
  }
  if (g.persistent) {  // prefill-sized M: persistent CTAs, double-buffered TMEM accumulators
    if (g.bn != 256 && g.bn != 128) throw std::runtime_error("tc_gemm persistent: bn must be 128 or 256");
    if (g.h && g.N % 128) throw std::runtime_error("tc_gemm swiglu: F must be a multiple of 64");
    if (pair_ok(g)) {  // CTA pairs: half the activation traffic per CTA, three operand stages
      if (g.h) launch_pair<true>(g, s);
      else launch_pair<false>(g, s);
      return;
    }
    if (g.h) {
      if (g.bn == 256) launch_persistent<256, true>(g, s);
      else launch_persistent<128, true>(g, s);
    } else {
      if (g.bn == 256) launch_persistent<256, false>(g, s);
      else launch_persistent<128, false>(g, s);
    }
    return;
  }
  if (g.h) {  // fused SwiGLU epilogue
    if (g.N % 128) throw std::runtime_error("tc_gemm swiglu: F must be a multiple of 64");
    switch (g.bn) {
      case 64: launch_bn<64, true>(g, s); break;
      case 128: launch_bn<128, true>(g, s); break;
      case 256: launch_bn<256, true>(g, s); break;
      default: throw std::runtime_error("tc_gemm swiglu: bn must be 64, 128 or 256");
    }
    return;
  }
  switch (g.bn) {
    case 32: launch_bn<32, false>(g, s); break;
    case 64: launch_bn<64, false>(g, s); break;
    case 128: launch_bn<128, false>(g, s); break;
    case 256: launch_bn<256, false>(g, s); break;
    default: throw std::runtime_error("tc_gemm: bn must be 32, 64, 128 or 256");
  }
}

}  // namespace hk
