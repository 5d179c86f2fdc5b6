// Persistent decode step (K1 + K5 + K6 of a dense decode layer, all layers, LM head): one launch
// per decode step for up to kDsMaxRows batch rows of a Llama-family model with Q4_K weights.
//
// Why: at batch 1 a decode step is ~4.5 GB of weights streamed through ~200 small kernels; each
// kernel pays launch, ramp-up (first DRAM bytes), staging of its activations and a drain tail,
// which together cost more than the bytes themselves for the small matrices (QKV, O). Here one CTA
// per SM (16 warps) runs every phase of every layer back to back:
//   A  RMSNorm(x) -> QKV GEMV; epilogue: bias, RoPE, q -> global, k / v -> the paged cache
//   B  split-KV attention on the tensor cores (TMA tensor loads of 16-token K/V units, 128-byte
//      swizzle, the query heads of a KV head as MMA rows); the last split of a (row, KV head)
//      merges and writes the output as two-limb integer activations
//   C  O GEMV (activations copied into shared memory by one bulk copy) + residual
//   D  RMSNorm(x) -> gate/up GEMV; epilogue: SwiGLU, and the fourth row group of each 32-row block
//      quantises that block of h
//   E  down GEMV + residual
// and finally RMSNorm -> LM head GEMV (logits, fused greedy keys). Phases are separated by a
// grid-wide barrier (all CTAs resident: the grid is one CTA per SM and the launch is cooperative).
//
// Weight streaming: each warp owns a contiguous range of 16x256 tiles of every matrix (the
// partition of mma_gemv.cu) and a ring of 2 stages x 2 tiles. Its copies follow one sequence over
// all phases: after consuming a chunk the warp issues the next chunk of the sequence, whichever
// phase it belongs to, so the next matrix's first tiles are in flight while the CTA waits at the
// barrier, runs attention, or stages activations. The GEMV math is the integer math of
// mma_gemv.cu (u8 x s8 mma.sync, activations as 16-bit fixed point per 32-element block).
//
// Every wait is bounded: mbarrier waits as in sm100.cuh, grid-barrier waits by `wait_ns` of
// globaltimer. A failure records a status code; every CTA then leaves at its next wait, after
// waiting (bounded) for its own copies in flight.
//
// Parity: crates/hawking-core/src/engine.rs decode step (embed -> per-layer attention / MLP ->
// final norm -> LM head -> sample), with the layer kernels of crates/hawking-core/shaders
// (quant.metal gemm_q4_k_m_fused*, mha.metal mha_decode_llama_b9430_fattn_*); the fusion into one
// persistent launch has no counterpart in the reference.
#include <cooperative_groups.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "api.h"
#include "mg_device.cuh"
#include "mma_frag.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace hk {
namespace ds {

using namespace mg;
using namespace frag;

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 2;           // weight ring stages per warp
constexpr int kTpc = 2;              // tiles per stage
constexpr int TB = Tile<WF_Q4_K>::BYTES;
constexpr int kScaleBytes = 16 * 8 * 8;
constexpr int kAttnStages = 4;       // KV ring: one 16-token unit (K and V) per stage
constexpr int kAttnConsumers = 8;    // warps 0..7 compute attention (a pair per stage), warp 8 lane 0 loads
static_assert(kAttnConsumers == 2 * kAttnStages, "one warp pair per KV ring stage");
constexpr int kProducerWarp = 8;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kRingBytes = kWarps * kStages * kTpc * TB;
constexpr int kBarOff = kRingBytes + kWarps * kScaleBytes;   // mbarriers, reduction scratch, cursors
constexpr int kXsOff = kBarOff + 2048;                        // activations / attention region
constexpr int kSmemMax = 232448;                              // 227 KB per CTA
constexpr int kXsBytes = kSmemMax - kXsOff - 1024;            // (1024 of alignment slack)
static_assert(kXsOff % 1024 == 0, "attention stages need 1024-byte alignment");

enum Phase { PH_QKV = 0, PH_ATTN = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4 };

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ long long gtimer() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Generic-proxy global writes (the K/V append) before async-proxy reads (TMA) in a later phase.
__device__ __forceinline__ void fence_proxy_async_all() { asm volatile("fence.proxy.async;" ::: "memory"); }

// First failed wait of this CTA (site, phase, warp) into the optional trace.
__device__ __forceinline__ void trace_fail(const DsArgs& a, int site, int phase) {
  if (!a.trace) return;
  int* t = a.trace + blockIdx.x * 4;
  if (atomicCAS(t + 1, 0, site) == 0) {
    t[2] = phase;
    t[3] = threadIdx.x >> 5;
  }
}

// Grid-wide barrier of `n` CTAs: arrival counter bar[0], generation bar[1]. The last arrival resets
// the counter and publishes the next generation (release); the others poll it (acquire) for at
// most wait_ns, and leave early once the status word is set. Returns false on failure.
// `proxy`: the phase before wrote memory (global K/V, or shared memory) that the async proxy (TMA,
// bulk copies) reads after the barrier; every thread fences its own generic writes.
__device__ __forceinline__ bool grid_sync(const DsArgs& a, int phase, int* s_flag, bool proxy) {
  unsigned* bar = a.bar;
  const unsigned n = gridDim.x;
  int* status = a.status;
  const long long wait_ns = a.wait_ns;
  if (proxy) fence_proxy_async_all();
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    if (a.tstamp) {  // earliest and latest arrival over the CTAs
      const unsigned long long t = (unsigned long long)gtimer();
      atomicMin(reinterpret_cast<unsigned long long*>(a.tstamp) + (phase + 1) * 4 + 1, t);
      atomicMax(reinterpret_cast<unsigned long long*>(a.tstamp) + (phase + 1) * 4 + 2, t);
    }
    const unsigned gen = ld_acquire(bar + 1);
    __threadfence();
    if (atomicAdd(bar, 1u) == n - 1) {
      atomicExch(bar, 0u);
      __threadfence();
      st_release(bar + 1, gen + 1);
    } else {
      const long long t0 = gtimer();
      for (int i = 0;; ++i) {
        if (ld_acquire(bar + 1) != gen) break;
        if ((i & 63) == 63) {
          if (*((volatile int*)status) != 0) { ok = 0; break; }
          if (gtimer() - t0 > wait_ns) {
            set_error(status, HK_ERR_PEER_TIMEOUT);
            trace_fail(a, 5, phase);
            ok = 0;
            break;
          }
        }
      }
    }
    if (ok && *((volatile int*)status) != 0) ok = 0;
    if (ok && a.trace) a.trace[blockIdx.x * 4] += 1;
    if (ok && a.tstamp && blockIdx.x == 0) a.tstamp[(phase + 1) * 4] = gtimer();
    *s_flag = ok;
  }
  __syncthreads();
  const bool ok = *(volatile int*)s_flag != 0;
  if (proxy && threadIdx.x == 0) fence_proxy_async_all();
  return ok;
}

// ---- activation staging (whole CTA) -------------------------------------------------------------
// x rows (fp32, written earlier in this launch: read through L2) -> RMSNorm * w -> two limbs per
// element in B-fragment order at xs (column n at n * cs uint4s) + per-block info.
__device__ void stage_norm(const float* x, int H, int nb, const float* w, float eps, uint4* xs, int64_t cs,
                           float2* info, int64_t is, float* red) {
  const int tid = threadIdx.x, h = tid & 1, nblk = H / 32;
  for (int n = 0; n < nb; ++n) {
    const float4* xr = reinterpret_cast<const float4*>(x + (int64_t)n * H);
    float ss = 0.f;
    for (int i = tid; i < H / 4; i += kThreads) {
      const float4 v = __ldcg(xr + i);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    const float scale = rsqrtf(block_sum(ss, red) / (float)H + eps);
    for (int b0 = 0; b0 < nblk; b0 += kThreads / 2) {
      const int b = b0 + (tid >> 1);
      const bool on = b < nblk;
      float v[16];
      if (on) {
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int k = 32 * b + 16 * c + 8 * h + 4 * j;
            const float4 x4 = __ldcg(reinterpret_cast<const float4*>(x + (int64_t)n * H + k));
            const float4 w4 = w ? *reinterpret_cast<const float4*>(w + k) : make_float4(1.f, 1.f, 1.f, 1.f);
            v[8 * c + 4 * j] = x4.x * scale * w4.x;
            v[8 * c + 4 * j + 1] = x4.y * scale * w4.y;
            v[8 * c + 4 * j + 2] = x4.z * scale * w4.z;
            v[8 * c + 4 * j + 3] = x4.w * scale * w4.w;
          }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
      }
      uint4 scratch[4];
      const float2 inf = quant_half_block(v, h, on ? xs + n * cs + b * 4 : scratch);
      if (on && h == 0) info[n * is + b] = inf;
    }
  }
  __syncthreads();
}

// Limbs + info already in global memory (written earlier in this launch) -> shared memory, one
// bulk copy per column and one for its info, on `bar` (single use per phase: parity tracked by the
// caller).
__device__ bool stage_copy(const DsArgs& a, int phase, const uint4* limbs, const float2* ginfo, int K, int nb,
                           uint4* xs, int64_t cs, float2* info, int64_t is, uint64_t* bar, uint32_t parity) {
  int* status = a.status;
  if (threadIdx.x == 0) {
    const uint32_t colb = (uint32_t)K * 2, infb = (uint32_t)(K / 32) * 8;
    sm100::mbar_arrive_expect_tx(bar, (colb + infb) * (uint32_t)nb);
    for (int n = 0; n < nb; ++n) {
      sm100::bulk_g2s(xs + n * cs, limbs + (int64_t)n * (K / 8), colb, bar);
      sm100::bulk_g2s(info + n * is, ginfo + (int64_t)n * (K / 32), infb, bar);
    }
  }
  const bool ok = sm100::mbar_wait(bar, parity, status);
  // a wait that left early (status set elsewhere) still lets the copies land before the region
  // is reused or the CTA exits
  if (!ok && threadIdx.x == 0) {
    trace_fail(a, 4, phase);
    sm100::mbar_wait(bar, parity, nullptr, 1u << 22);
  }
  return ok;
}

// Quantise one 32-element block of fp32 values (a lane pair; every lane of the warp takes part)
// from `src` (read through L2) into the global two-limb layout.
__device__ __forceinline__ void quant_block_to_global(const float* src, bool on, int h, uint4* dst, float2* dinfo) {
  float v[16];
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float4 x4 = on ? __ldcg(reinterpret_cast<const float4*>(src + 16 * c + 8 * h + 4 * j))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      v[8 * c + 4 * j] = x4.x;
      v[8 * c + 4 * j + 1] = x4.y;
      v[8 * c + 4 * j + 2] = x4.z;
      v[8 * c + 4 * j + 3] = x4.w;
    }
  uint4 scratch[4];
  const float2 inf = quant_half_block(v, h, on ? dst : scratch);
  if (on && h == 0) *dinfo = inf;
}

// ---- epilogues (one row group of 16 tile rows; lane holds rows r0, r0 + 8 x columns 2q, 2q + 1) --
enum Epi { EPI_QKV = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_HEAD = 3 };

struct EpiCtx {
  int l;
  const float* qkv_bias;
};

template <int NB, int EPI>
__device__ __forceinline__ void epilogue(const DsArgs& a, const EpiCtx& e, uint32_t g, const float (&v)[4],
                                         int lane) {
  const int r0 = lane >> 2, q = lane & 3;
  if constexpr (EPI == EPI_QKV) {
    const int64_t layer = (int64_t)e.l * a.num_cache_blocks * a.nkv * a.block_size * a.hd;
    const RopeEpi r{a.rope, a.positions, a.row_seq, a.block_tables, a.max_blocks, a.block_size,
                    a.k_cache + layer, a.v_cache + layer, a.q, e.qkv_bias, a.nh, a.nkv, a.hd, a.rot, a.rope_style,
                    (int64_t)a.num_cache_blocks};
    rope_epilogue<NB>(r, a.nb, g, v, lane);
  } else if constexpr (EPI == EPI_RESID) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int col = 2 * q + (i & 1);
      if ((NB == 1 && (i & 1)) || col >= a.nb) continue;
      float* yp = a.x + (int64_t)col * a.H + g * 16 + (i >> 1) * 8 + r0;
      __stcg(yp, __ldcg(yp) + v[i]);
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    const int o = (int)g * 8 + r0;  // h row: gate in tile row r0, up in r0 + 8
#pragma unroll
    for (int i = 0; i < (NB > 1 ? 2 : 1); ++i) {
      const int col = 2 * q + i;
      if (col >= a.nb) continue;
      const float gt = v[i], up = v[2 + i];
      __stcg(a.hf + (int64_t)col * a.F + o, gt / (1.f + __expf(-gt)) * up);
    }
    // the fourth row group of a 32-row block quantises the block (all columns)
    __threadfence();
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(a.h_cnt + (g >> 2), 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old == 3) {
      __threadfence();
      const int b = (int)(g >> 2), col = lane >> 1, h = lane & 1;
      const bool on = col < a.nb;
      const int cc = on ? col : 0;
      quant_block_to_global(a.hf + (int64_t)cc * a.F + 32 * b, on, h, a.h_limbs + (int64_t)cc * (a.F / 8) + b * 4,
                            a.h_info + (int64_t)cc * (a.F / 32) + b);
      if (lane == 0) a.h_cnt[b] = 0;
    }
  } else {  // EPI_HEAD
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = (int)g * 16 + (i >> 1) * 8 + r0, col = 2 * q + (i & 1);
      if ((NB == 1 && (i & 1)) || row >= a.V || col >= a.nb) continue;
      if (a.logits) a.logits[(int64_t)col * a.V + row] = v[i];
      if (a.argmax_slots)
        atomicMax(a.argmax_slots + (int64_t)col * kArgmaxSlots + (row % kArgmaxSlots), argmax_key(v[i], row));
    }
  }
}

// ---- the per-warp weight stream --------------------------------------------------------------
// Weight phases in launch order: for each layer QKV (5l), O (5l + 2), gate/up (5l + 3), down
// (5l + 4); the LM head is phase 5L. Phase 5l + 1 (attention) has no weights.
struct Mat {
  const uint8_t* tiles;
  uint32_t G, KT;
};
__device__ __forceinline__ Mat matrix_of(const DsArgs& a, int ph) {
  const int Ka = a.nh * a.hd;
  if (ph >= 5 * a.L) return Mat{a.head, (uint32_t)((a.V + 15) / 16), (uint32_t)(a.H / 256)};
  const DsLayer* ly = a.layers + ph / 5;
  switch (ph % 5) {
    case PH_QKV: return Mat{ly->qkv, (uint32_t)((a.nh + 2 * a.nkv) * a.hd / 16), (uint32_t)(a.H / 256)};
    case PH_O: return Mat{ly->o, (uint32_t)(a.H / 16), (uint32_t)(Ka / 256)};
    case PH_GU: return Mat{ly->gu, (uint32_t)(a.F / 8), (uint32_t)(a.H / 256)};
    default: return Mat{ly->down, (uint32_t)(a.H / 16), (uint32_t)(a.F / 256)};
  }
}
__device__ __forceinline__ int next_weight_phase(int ph) { return ph % 5 == PH_QKV ? ph + 2 : ph + 1; }

// Issue cursor of a warp's stream: lane 0 only, in shared memory (keeps the registers of the
// consuming loop free).
struct IssueCursor {
  const uint8_t* itiles;
  uint32_t issued, ichunk, inchunks, it0, intiles;
  int iph;
};
static_assert(sizeof(IssueCursor) <= 64, "one 64-byte slot per warp");

struct WarpStream {
  uint8_t* ring;
  uint64_t* bars;
  IssueCursor* ic;
  uint32_t cons;  // chunks consumed so far (one sequence over all phases; every lane)

  __device__ static void open(const DsArgs& a, IssueCursor& c, int ph, uint32_t p, uint32_t P) {
    c.iph = ph;
    c.ichunk = 0;
    if (ph > 5 * a.L) {
      c.inchunks = 0;
      return;
    }
    const Mat m = matrix_of(a, ph);
    const uint32_t T = m.G * m.KT;
    c.it0 = start_of(p, T, P);
    c.intiles = start_of(p + 1, T, P) - c.it0;
    c.inchunks = (c.intiles + kTpc - 1) / kTpc;
    c.itiles = m.tiles;
  }
  // Lane 0: issue the next chunk of the sequence, whichever phase it belongs to.
  __device__ void issue_next(const DsArgs& a, uint32_t p, uint32_t P, int lane) {
    if (lane != 0) return;
    IssueCursor& c = *ic;
    while (c.ichunk >= c.inchunks) {
      if (c.iph >= 5 * a.L) return;
      open(a, c, next_weight_phase(c.iph), p, P);
    }
    const uint32_t st = c.issued % kStages;
    const uint32_t cnt = min((uint32_t)kTpc, c.intiles - c.ichunk * kTpc);
    sm100::mbar_arrive_expect_tx(&bars[st], cnt * TB);
    sm100::bulk_g2s(ring + st * kTpc * TB, c.itiles + (int64_t)(c.it0 + c.ichunk * kTpc) * TB, cnt * TB, &bars[st]);
    ++c.ichunk;
    ++c.issued;
  }
  // Wait (bounded, no early exit) for every chunk still in flight: before the CTA may exit.
  __device__ void drain(int lane) {
    if (lane == 0)
      for (uint32_t k = cons; k < ic->issued; ++k)
        sm100::mbar_wait(&bars[k % kStages], (k / kStages) & 1, nullptr, 1u << 22);
  }
};

// One GEMV phase for this warp: consume its tile range of matrix `m` (the chunks at the head of its
// stream), with the deterministic split-K fix-up of mma_gemv.cu, then the epilogue.
template <int NB, int EPI>
__device__ __forceinline__ bool gemv_phase(const DsArgs& a, const EpiCtx& e, int ph, const XInt& xi, WarpStream& ws, float2* scs,
                           uint32_t p, uint32_t P, int lane) {
  const Mat m = matrix_of(a, ph);
  const uint32_t KT = m.KT, T = m.G * KT;
  const uint32_t t0 = start_of(p, T, P), t1 = start_of(p + 1, T, P);
  const int n_tiles = (int)(t1 - t0);
  float sum[4] = {0.f, 0.f, 0.f, 0.f};
  uint32_t g = t0 / KT, s = t0 - g * KT;
  const uint32_t first_g = g;
  int u = 0;
  for (int i = 0; i < n_tiles; ++i) {
    const uint32_t st = ws.cons % kStages;
    if (u == 0 && !sm100::mbar_wait(&ws.bars[st], (ws.cons / kStages) & 1, a.status)) {
      if (lane == 0) trace_fail(a, 1, ph);
      return false;
    }
    consume_q4k_int<NB>(ws.ring + (st * kTpc + u) * TB, (int)s, xi, a.nb, scs, lane, sum);
    if (++u == kTpc || i == n_tiles - 1) {  // chunk consumed: the next one of the stream takes its stage
      u = 0;
      ++ws.cons;
      if (lane == 0) sm100::fence_proxy_async_smem();
      ws.issue_next(a, p, P, lane);
    }
    const bool last = (i == n_tiles - 1) || (s == KT - 1);
    if (++s == KT) s = 0;
    if (!last) continue;
    const uint32_t pf = owner(g * KT, T, P), pl = owner(g * KT + KT - 1, T, P);
    if (pf == pl) {
      epilogue<NB, EPI>(a, e, g, sum, lane);
    } else {
      const int slot = (g == first_g) ? 0 : 1;
      __stcg(a.part + ((int64_t)p * 2 + slot) * 32 + lane, make_float4(sum[0], sum[1], sum[2], sum[3]));
      __threadfence();
      int old = 0;
      if (lane == 0) old = atomicAdd(a.counters + g, 1);
      old = __shfl_sync(0xffffffffu, old, 0);
      const bool dense = T >= P;
      if (old == (dense ? (int)(pl - pf) : pieces_of_group(g, KT, T, P) - 1)) {
        __threadfence();
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        const int sl0 = (start_of(pf, T, P) / KT == g) ? 0 : 1;
        for (uint32_t pp = pf;; pp = dense ? pp + 1 : next_owner(pp, T, P)) {
          const float4 pv = __ldcg(a.part + ((int64_t)pp * 2 + (pp == pf ? sl0 : 0)) * 32 + lane);
          v[0] += pv.x;
          v[1] += pv.y;
          v[2] += pv.z;
          v[3] += pv.w;
          if (pp == pl) break;
        }
        if (lane == 0) a.counters[g] = 0;
        epilogue<NB, EPI>(a, e, g, v, lane);
      }
    }
    sum[0] = sum[1] = sum[2] = sum[3] = 0.f;
    ++g;
  }
  return true;
}

// ---- attention phase ----------------------------------------------------------------------------
// Items (row c, KV head, split) over the CTAs. Per item: warp 8 lane 0 streams the split's 16-token
// units of K and V (TMA tensor loads from the maps over every layer's cache, 128-byte swizzle) into
// a ring of kAttnStages stages; warps 0..7 take units round robin (mma.sync with the query heads of
// the KV head as M rows, online softmax in the log2 domain, as attention_tc.cu), fold into shared
// memory, and either finish (one split) or publish a partial and let the last split merge. The
// result goes out as two-limb activations for the O projection.
struct AttnSmem {
  uint8_t* ring;   // kAttnStages x (K, V) of 16 tokens, 1024-aligned
  float* s_o;      // [16][HD]
  float* s_wm;     // [kAttnConsumers][16]
  float* s_m;      // [16]
  float* s_l;      // [16]
  int* s_flag;
};

template <int HD>
__device__ __forceinline__ bool attn_phase(const DsArgs& a, int l, const CUtensorMap* tk, const CUtensorMap* tv, const AttnSmem& sm,
                           uint64_t* afull, uint64_t* aempty, uint32_t& useq) {
  constexpr int NKS = HD / 16, NDT = HD / 8;
  constexpr uint32_t kUnitBytes = 2 * 16 * HD * 2;  // K and V of 16 tokens
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int G = a.nh / a.nkv, S = a.splits, bs = a.block_size;
  const int Ka = a.nh * HD;
  const int n_items = a.nb * a.nkv * S;
  const int g = lane >> 2, q4 = lane & 3;
  const uint32_t ring_s = sm100::smem_u32(sm.ring);
  bool ok = true;
  for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
    const int s = it % S, kvh = (it / S) % a.nkv, c = it / (S * a.nkv);
    const int ctx = a.row_ctx[c];
    const int* btab = a.block_tables + (int64_t)a.row_seq[c] * a.max_blocks;
    const int nblk_ctx = (ctx + bs - 1) / bs;
    const int bpc = (nblk_ctx + S - 1) / S;
    const int b0 = s * bpc, b1 = min(nblk_ctx, b0 + bpc);
    const int tok0 = b0 * bs, tok1 = min(ctx, b1 * bs);
    const int n_units = tok1 > tok0 ? (tok1 - tok0 + 15) / 16 : 0;
    for (int i = tid; i < 16 * HD; i += kThreads) sm.s_o[i] = 0.f;
    if (tid < 16) sm.s_l[tid] = 0.f;
    __syncthreads();
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
    float o[NDT / 2][4];  // this warp's half of the head dims
#pragma unroll
    for (int d = 0; d < NDT / 2; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
    if (warp == kProducerWarp) {
      if (lane == 0) {
        int issued = 0;
        for (int u = 0; u < n_units && ok; ++u) {
          const uint32_t sq = useq + u, st = sq % kAttnStages;
          if (sq >= kAttnStages && !sm100::mbar_wait(&aempty[st], ((sq / kAttnStages) - 1) & 1, a.status)) {
            trace_fail(a, 3, 5 * l + PH_ATTN);
            ok = false;
            break;
          }
          const int tok = tok0 + 16 * u;
          const int blk = btab[tok / bs];
          const int row0 = (int)((((int64_t)l * a.num_cache_blocks + blk) * a.nkv + kvh) * bs + tok % bs);
          uint8_t* dst = sm.ring + st * kUnitBytes;
          sm100::mbar_arrive_expect_tx(&afull[st], kUnitBytes);
#pragma unroll
          for (int bx = 0; bx < HD / 64; ++bx) {
            sm100::tma_load_2d(dst + bx * 16 * 128, tk, bx * 64, row0, &afull[st]);
            sm100::tma_load_2d(dst + 16 * HD * 2 + bx * 16 * 128, tv, bx * 64, row0, &afull[st]);
          }
          issued = u + 1;
        }
        // every issued copy lands before the region is reused or the CTA exits (in the normal
        // course the consumers have waited for them already)
        for (int u = max(0, issued - kAttnStages); u < issued; ++u)
            sm100::mbar_wait(&afull[(useq + u) % kAttnStages], ((useq + u) / kAttnStages) & 1, nullptr, 1u << 22);
      }
    } else if (warp < kAttnConsumers) {
      uint32_t qa[NKS][4];
      {
        const float* qb = a.q + ((int64_t)c * a.nh + (int64_t)kvh * G) * HD;
        const bool v0 = g < G, v1 = g + 8 < G;
#pragma unroll
        for (int ks = 0; ks < NKS; ++ks) {
          const int d0 = 16 * ks + 2 * q4, d1 = d0 + 8;
          const float2 z = make_float2(0.f, 0.f);
          const float2 a0 = v0 ? __ldcg(reinterpret_cast<const float2*>(qb + g * HD + d0)) : z;
          const float2 a1 = v1 ? __ldcg(reinterpret_cast<const float2*>(qb + (g + 8) * HD + d0)) : z;
          const float2 a2 = v0 ? __ldcg(reinterpret_cast<const float2*>(qb + g * HD + d1)) : z;
          const float2 a3 = v1 ? __ldcg(reinterpret_cast<const float2*>(qb + (g + 8) * HD + d1)) : z;
          qa[ks][0] = pack_bf16(a0.x, a0.y);
          qa[ks][1] = pack_bf16(a1.x, a1.y);
          qa[ks][2] = pack_bf16(a2.x, a2.y);
          qa[ks][3] = pack_bf16(a3.x, a3.y);
        }
      }
      const float qs = a.scale * kLog2e;
      // stage st belongs to the warp pair (st, st + 4): both wait every phase of it in order (a
      // parity wait is sound only for a waiter that saw the stage's previous phase), both form
      // the scores, and each takes half of the head dims in P V
      const int pair = warp & (kAttnStages - 1), half = warp / kAttnStages;
      const int u0 = (int)((pair + kAttnStages - useq % kAttnStages) % kAttnStages);
      for (int u = u0; u < n_units && ok; u += kAttnStages) {
        const uint32_t sq = useq + u, st = sq % kAttnStages;
        if (!sm100::mbar_wait(&afull[st], (sq / kAttnStages) & 1, a.status)) {
          if (lane == 0) trace_fail(a, 2, 5 * l + PH_ATTN);
          ok = false;
          break;
        }
        const uint32_t kb = ring_s + st * kUnitBytes, vb = kb + 16 * HD * 2;
        float sc[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
          const int row = 8 * j + (lane & 7);
#pragma unroll
          for (int pq = 0; pq < HD / 32; ++pq) {
            uint32_t kr[4];
            ldsm_x4(sw_addr(kb, 16, row, 4 * pq + (lane >> 3)), kr);
            mma16816(sc[j], qa[2 * pq], kr[0], kr[1]);
            mma16816(sc[j], qa[2 * pq + 1], kr[2], kr[3]);
          }
        }
        const int tk0 = tok0 + 16 * u + 2 * q4;
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[j][e] = tk0 + 8 * j + (e & 1) < ctx ? sc[j][e] * qs : -INFINITY;
        float mx[2] = {fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1])),
                       fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]))};
        float alpha[2], mref[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
          mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
          const float mn = fmaxf(m_r[h], mx[h]);
          mref[h] = mn == -INFINITY ? 0.f : mn;
          alpha[h] = exp2f(m_r[h] - mref[h]);
          m_r[h] = mn;
        }
        float pv[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) pv[j][e] = exp2f(sc[j][e] - mref[e >> 1]);
        l_r[0] = l_r[0] * alpha[0] + (pv[0][0] + pv[0][1] + pv[1][0] + pv[1][1]);
        l_r[1] = l_r[1] * alpha[1] + (pv[0][2] + pv[0][3] + pv[1][2] + pv[1][3]);
        const uint32_t pa[4] = {pack_bf16(pv[0][0], pv[0][1]), pack_bf16(pv[0][2], pv[0][3]),
                                pack_bf16(pv[1][0], pv[1][1]), pack_bf16(pv[1][2], pv[1][3])};
        const int vrow = ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
        for (int dd = 0; dd < NDT / 4; ++dd) {
          uint32_t vr[4];
          ldsm_x4_t(sw_addr(vb, 16, vrow, 2 * (half * (NDT / 4) + dd) + (lane >> 4)), vr);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float* od = o[2 * dd + h];
            od[0] *= alpha[0];
            od[1] *= alpha[0];
            od[2] *= alpha[1];
            od[3] *= alpha[1];
            mma16816(o[2 * dd + h], pa, vr[2 * h], vr[2 * h + 1]);
          }
        }
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&aempty[st]);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 1);
        l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 2);
      }
      if (q4 == 0) {
        sm.s_wm[warp * 16 + g] = m_r[0];
        sm.s_wm[warp * 16 + g + 8] = m_r[1];
      }
    }
    __syncthreads();
    if (warp < kAttnConsumers) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = g + 8 * h;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnConsumers; ++w) M = fmaxf(M, sm.s_wm[w * 16 + row]);
        const float f = m_r[h] == -INFINITY ? 0.f : exp2f(m_r[h] - M);
        const int half = warp / kAttnStages;
        if (f != 0.f && row < G) {
#pragma unroll
          for (int d = 0; d < NDT / 2; ++d) {
            const int col = half * (HD / 2) + 8 * d + 2 * q4;
            atomicAdd(&sm.s_o[row * HD + col], o[d][2 * h] * f);
            atomicAdd(&sm.s_o[row * HD + col + 1], o[d][2 * h + 1] * f);
          }
          if (q4 == 0 && half == 0) atomicAdd(&sm.s_l[row], l_r[h] * f);  // both halves hold the same sums
        }
        if (warp == 0 && q4 == 0) sm.s_m[row] = M;
      }
    }
    const bool fail = __syncthreads_or(!ok || *((volatile int*)a.status) != 0);
    useq += (uint32_t)n_units;
    if (fail) return false;
    const int nout = G * HD;
    const int64_t pair = (int64_t)c * a.nkv + kvh;
    if (S == 1) {
      for (int i = tid; i < nout; i += kThreads) {
        const float L = sm.s_l[i / HD];
        sm.s_o[i] = L > 0.f ? sm.s_o[i] / L : 0.f;
      }
    } else {
      float* po = a.att_o + (int64_t)it * nout;
      for (int i = tid; i < nout; i += kThreads) __stcg(po + i, sm.s_o[i]);
      if (tid < G) __stcg(a.att_ml + (int64_t)it * G + tid, make_float2(sm.s_m[tid], sm.s_l[tid]));
      __threadfence();
      __syncthreads();
      if (tid == 0) *sm.s_flag = atomicAdd(a.att_cnt + pair, 1) == S - 1;
      __syncthreads();
      if (!*(volatile int*)sm.s_flag) continue;
      __threadfence();
      const int64_t base = pair * S;
      for (int i = tid; i < nout; i += kThreads) {
        const int row = i / HD;
        float M = -INFINITY;
        for (int k = 0; k < S; ++k) M = fmaxf(M, __ldcg(a.att_ml + (base + k) * G + row).x);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY)
          for (int k = 0; k < S; ++k) {
            const float2 ml = __ldcg(a.att_ml + (base + k) * G + row);
            if (ml.x == -INFINITY) continue;
            const float f = exp2f(ml.x - M);
            L += ml.y * f;
            O += __ldcg(a.att_o + (base + k) * nout + i) * f;
          }
        sm.s_o[i] = L > 0.f ? O / L : 0.f;
      }
      if (tid == 0) a.att_cnt[pair] = 0;
    }
    __syncthreads();
    // the KV head's G * HD outputs -> two-limb blocks of the O projection's input
    const int nblk = nout / 32, b0g = kvh * nout / 32;
    for (int bb = 0; bb < nblk; bb += kThreads / 2) {
      const int b = bb + (tid >> 1), h = tid & 1;
      const bool on = b < nblk;
      float v[16];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc)
#pragma unroll
        for (int j = 0; j < 8; ++j) v[8 * cc + j] = on ? sm.s_o[32 * b + 16 * cc + 8 * h + j] : 0.f;
      uint4 scratch[4];
      const float2 inf = quant_half_block(v, h, on ? a.a_limbs + (int64_t)c * (Ka / 8) + (b0g + b) * 4 : scratch);
      if (on && h == 0) a.a_info[(int64_t)c * (Ka / 32) + b0g + b] = inf;
    }
    __syncthreads();
  }
  return ok;
}

// ---- the kernel ----------------------------------------------------------------------------------
// Shared memory (dynamic, 1024-aligned): per-warp weight rings | per-warp scale tables | mbarriers
// and reduction scratch | activation region (staged limbs, or the attention ring + merge scratch).
template <int NB, int HD>
__global__ void __launch_bounds__(kThreads, 1)
    ds_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
              const __grid_constant__ DsArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float2* scs = reinterpret_cast<float2*>(smem + kRingBytes + warp * kScaleBytes);
  uint64_t* wbars = reinterpret_cast<uint64_t*>(smem + kBarOff);          // [kWarps][kStages]
  uint64_t* afull = wbars + kWarps * kStages;                              // [kAttnStages]
  uint64_t* aempty = afull + kAttnStages;                                  // [kAttnStages]
  uint64_t* xbar = aempty + kAttnStages;                                   // activation copies
  float* red = reinterpret_cast<float*>(smem + kBarOff + 512);             // [32]
  int* s_flag = reinterpret_cast<int*>(smem + kBarOff + 640);
  uint8_t* xsr = smem + kXsOff;

  if (lane == 0)
    for (int s = 0; s < kStages; ++s) sm100::mbar_init(&wbars[warp * kStages + s], 1);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kAttnStages; ++s) {
      sm100::mbar_init(&afull[s], 1);
      sm100::mbar_init(&aempty[s], kAttnConsumers / kAttnStages);  // both warps of the stage's pair
    }
    sm100::mbar_init(xbar, 1);
    sm100::prefetch_tmap(&tk);
    sm100::prefetch_tmap(&tv);
  }
  if (threadIdx.x == 0 || lane == 0) sm100::fence_barrier_init();
  if (threadIdx.x == 0 && blockIdx.x == 0 && a.tstamp) a.tstamp[0] = gtimer();
  if (threadIdx.x == 0 && a.tstamp) a.tstamp[2] = 0;  // (slot 2 of row 0 unused)
  __syncthreads();

  const uint32_t P = gridDim.x * kWarps, p = blockIdx.x * kWarps + warp;
  WarpStream ws;
  ws.ring = smem + warp * kStages * kTpc * TB;
  ws.bars = wbars + warp * kStages;
  ws.ic = reinterpret_cast<IssueCursor*>(smem + kBarOff + 1024 + warp * 64);
  ws.cons = 0;
  if (lane == 0) {
    ws.ic->issued = 0;
    WarpStream::open(a, *ws.ic, 0, p, P);
  }
  for (int k = 0; k < kStages; ++k) ws.issue_next(a, p, P, lane);

  const int H = a.H, F = a.F, Ka = a.nh * HD;
  AttnSmem as;
  as.ring = xsr;
  as.s_o = reinterpret_cast<float*>(xsr + kAttnStages * 2 * 16 * HD * 2);
  as.s_wm = as.s_o + 16 * HD;
  as.s_m = as.s_wm + kAttnConsumers * 16;
  as.s_l = as.s_m + 16;
  as.s_flag = s_flag;
  uint4* xs = reinterpret_cast<uint4*>(xsr);
  const int64_t csH = H / 8 + 1, isH = H / 32;  // staged column stride (uint4, one spare), info stride
  auto info_at = [&](int64_t cs) { return reinterpret_cast<float2*>(xs + (int64_t)a.nb * cs); };
  const bool down_smem = (int64_t)a.nb * ((F / 8 + 1) * 16 + (F / 32) * 8) <= kXsBytes;
  uint32_t useq = 0, xph = 0;
  bool ok = true;

  for (int l = 0; l < a.L && ok; ++l) {
    const DsLayer ly = a.layers[l];
    const EpiCtx e{l, ly.qkv_bias};
    // A: RMSNorm -> QKV, RoPE + K/V append
    stage_norm(a.x, H, a.nb, ly.attn_norm, a.eps, xs, csH, info_at(csH), isH, red);
    if (a.tstamp && blockIdx.x == 0 && threadIdx.x == 0) a.tstamp[(5 * l + PH_QKV + 1) * 4 + 3] = gtimer();
    gemv_phase<NB, EPI_QKV>(a, e, 5 * l + PH_QKV, XInt{xs, csH, info_at(csH), isH}, ws, scs, p, P, lane);
    if (!(ok = grid_sync(a, 5 * l + PH_QKV, s_flag, true))) break;
    // B: attention -> limbs of the O projection's input
    attn_phase<HD>(a, l, &tk, &tv, as, afull, aempty, useq);
    if (!(ok = grid_sync(a, 5 * l + PH_ATTN, s_flag, true))) break;
    // C: O projection + residual
    {
      const int64_t cs = Ka / 8 + 1, is = Ka / 32;
      stage_copy(a, 5 * l + PH_O, a.a_limbs, a.a_info, Ka, a.nb, xs, cs, info_at(cs), is, xbar, xph++ & 1);
      gemv_phase<NB, EPI_RESID>(a, e, 5 * l + PH_O, XInt{xs, cs, info_at(cs), is}, ws, scs, p, P, lane);
    }
    if (!(ok = grid_sync(a, 5 * l + PH_O, s_flag, false))) break;
    // D: RMSNorm -> gate/up, SwiGLU (+ block quantisation of h)
    stage_norm(a.x, H, a.nb, ly.ffn_norm, a.eps, xs, csH, info_at(csH), isH, red);
    if (a.tstamp && blockIdx.x == 0 && threadIdx.x == 0) a.tstamp[(5 * l + PH_GU + 1) * 4 + 3] = gtimer();
    gemv_phase<NB, EPI_SWIGLU>(a, e, 5 * l + PH_GU, XInt{xs, csH, info_at(csH), isH}, ws, scs, p, P,
                               lane);
    if (!(ok = grid_sync(a, 5 * l + PH_GU, s_flag, true))) break;
    // E: down projection + residual
    if (down_smem) {
      const int64_t cs = F / 8 + 1, is = F / 32;
      stage_copy(a, 5 * l + PH_DOWN, a.h_limbs, a.h_info, F, a.nb, xs, cs, info_at(cs), is, xbar, xph++ & 1);
      gemv_phase<NB, EPI_RESID>(a, e, 5 * l + PH_DOWN, XInt{xs, cs, info_at(cs), is}, ws, scs, p, P,
                                lane);
    } else {
      gemv_phase<NB, EPI_RESID>(a, e, 5 * l + PH_DOWN, XInt{a.h_limbs, F / 8, a.h_info, F / 32}, ws,
                                scs, p, P, lane);
    }
    if (!(ok = grid_sync(a, 5 * l + PH_DOWN, s_flag, false))) break;
  }
  if (ok) {
    // final RMSNorm -> LM head (logits, greedy keys)
    stage_norm(a.x, H, a.nb, a.out_norm, a.eps, xs, csH, info_at(csH), isH, red);
    gemv_phase<NB, EPI_HEAD>(a, EpiCtx{a.L, nullptr}, 5 * a.L, XInt{xs, csH, info_at(csH), isH}, ws,
                             scs, p, P, lane);
  }
  if (ok && a.tstamp && blockIdx.x == 0 && threadIdx.x == 0) a.tstamp[(5 * a.L + 1) * 4] = gtimer();
  ws.drain(lane);  // nothing in flight on the normal path; after a failure, the prefetched chunks
}

// ---- host ----------------------------------------------------------------------------------------
struct MapKey {
  const void* base;
  int64_t rows;
  int hd;
  bool operator==(const MapKey& o) const { return base == o.base && rows == o.rows && hd == o.hd; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.base) ^ (std::hash<int64_t>()(k.rows) * 31) ^ ((size_t)k.hd << 20);
  }
};
// [rows, hd] bf16 map of a whole cache (every layer), boxes of [64 dims x 16 tokens], 128-byte swizzle.
const CUtensorMap& unit_map(const void* base, int64_t rows, int hd) {
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  const MapKey k{base, rows, hd};
  auto it = cache.find(k);
  if (it != cache.end()) return it->second;
  CUtensorMap m = tma_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, (uint64_t)hd, (uint64_t)rows, (uint64_t)hd * 2, 64,
                             16, CU_TENSOR_MAP_SWIZZLE_128B);
  return cache.emplace(k, m).first->second;
}

size_t staging_bytes(int K, int nb) { return (size_t)nb * (((size_t)K / 8 + 1) * 16 + (size_t)K / 32 * 8); }

}  // namespace ds

bool ds_supported(const DsArgs& a) {
  const int Ka = a.nh * a.hd;
  const int G = a.nkv > 0 ? a.nh / a.nkv : 0;
  if (!(a.hd == 64 || a.hd == 128) || a.nkv <= 0 || a.nh % a.nkv || G > 16) return false;
  if (!(a.block_size == 16 || a.block_size == 32 || a.block_size == 64)) return false;
  if (a.rot % 16 || a.rot > a.hd || a.rot <= 0 || (a.rope_style != 0 && a.rope_style != 1)) return false;
  if (a.H % 256 || a.F % 256 || Ka % 256 || a.nb < 1 || a.nb > kDsMaxRows || a.splits < 1) return false;
  const size_t attn = (size_t)ds::kAttnStages * 2 * 16 * a.hd * 2 + 16 * a.hd * 4 + (ds::kAttnConsumers + 2) * 16 * 4;
  const size_t need = std::max(std::max(ds::staging_bytes(a.H, a.nb), ds::staging_bytes(Ka, a.nb)), attn);
  return need <= (size_t)ds::kXsBytes;
}

int ds_grid(int device) {
  int sms = 0;
  HK_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  return sms;
}

template <int NB, int HD>
static void ds_launch_t(const DsArgs& a, int grid, cudaStream_t s) {
  const int64_t rows = (int64_t)a.L * a.num_cache_blocks * a.nkv * a.block_size;
  const CUtensorMap tk = ds::unit_map(a.k_cache, rows, a.hd);
  const CUtensorMap tv = ds::unit_map(a.v_cache, rows, a.hd);
  auto kern = ds::ds_kernel<NB, HD>;
  static bool attr_set = false;
  if (!attr_set) {
    HK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, ds::kSmemMax));
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(ds::kThreads);
  cfg.dynamicSmemBytes = ds::kSmemMax;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident (the phases wait on one another)
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  HK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, tk, tv, a));
}

void ds_launch(const DsArgs& a, cudaStream_t s) {
  if (!ds_supported(a)) throw std::runtime_error("decode step: unsupported shape");
  if ((reinterpret_cast<uintptr_t>(a.k_cache) | reinterpret_cast<uintptr_t>(a.v_cache)) & 15)
    throw std::runtime_error("decode step: K/V caches must be 16-byte aligned");
  int dev = 0;
  HK_CUDA_CHECK(cudaGetDevice(&dev));
  const int grid = ds_grid(dev);
  if ((int64_t)grid * ds::kWarps * ((int64_t)((a.V + 15) / 16) * (a.H / 256)) >= (1ll << 32))
    throw std::runtime_error("decode step: tile count overflows the 32-bit partition arithmetic");
  if (a.nb == 1) {
    if (a.hd == 64) ds_launch_t<1, 64>(a, grid, s);
    else ds_launch_t<1, 128>(a, grid, s);
  } else {
    if (a.hd == 64) ds_launch_t<kDsMaxRows, 64>(a, grid, s);
    else ds_launch_t<kDsMaxRows, 128>(a, grid, s);
  }
}

}  // namespace hk
