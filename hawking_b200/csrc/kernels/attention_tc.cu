// Paged GQA decode attention on the tensor cores (K5, decode): flash decoding with the query heads of
// one KV head as the M rows of mma.sync m16n8k16 (up to 16 heads per KV head; fewer are zero rows).
//
// Per CTA: one (row, KV head, split); the S splits of a (row, KV head) form a thread-block cluster
// and merge through distributed shared memory (as the CUDA-core cluster kernel in attention.cu).
//  * Data movement. One producer warp streams the split's KV blocks through a ring of shared-memory
//    stages with TMA tensor loads (cp.async.bulk.tensor, 128-byte swizzle, no multicast): each
//    stage holds one block's K and V as boxes of [block_size tokens x 64 dims]. The swizzle makes
//    the ldmatrix reads below bank-conflict free.
//  * Math. Consumer warps take 16-token units. S = Q K^T: the bf16 query fragments stay in
//    registers, K fragments come from ldmatrix (HD / 16 k-steps x 2 token tiles). The query is
//    rounded unscaled and the scale applied to the fp32 scores, as the prefill kernel does, so a
//    row gets the same scores whichever of the two kernels runs it. Online softmax in the log2
//    domain on the accumulator fragments (row statistics over the four lanes of a quad).
//    O += P V: the score accumulators are repacked as the bf16 A fragment (the FA2 register reuse),
//    V fragments come from ldmatrix.trans. fp32 accumulation throughout.
//  * Merge. The warps fold (max, sum, O) into shared memory; after a cluster barrier every CTA merges
//    whole 32-dim output blocks across the S CTAs by reading their shared memory.
// Every wait is bounded (status word, then the CTA unwinds: the producer waits for its own copies).
//
// Parity: crates/hawking-core/shaders/mha.metal mha_decode_llama_b9430_fattn_{main,reduce} (split-K
// flash decode), oracle crates/hawking-core/src/attn.rs:23 (mha_decode_step).
#include <cooperative_groups.h>

#include <cstdlib>

#include <mutex>
#include <unordered_map>

#include "api.h"
#include "sm100.cuh"
#include "tma_host.cuh"
#include "mma_frag.cuh"

namespace cg = cooperative_groups;

namespace hk {
namespace atc {
using namespace frag;

// Consumer warps: 8 for blocks of 32 / 64 tokens, 4 for blocks of 16. Warp w takes units
// w, w + NC, ... of the split; a parity wait is sound only for a warp that saw the stage's previous
// phase, which holds when NC units span a whole number of stage rounds or stay within one stage:
// block size 64 (4 units per block, a warp visits every other block, and stage s holds blocks
// s, s + 4, ... of which it sees each), 32 (2 units per block, a warp's blocks step by 4) and
// 16 with 4 consumers (one warp per stage).
template <int NC> struct Cfg {
  static constexpr int kConsumers = NC;
  static constexpr int kThreads = (NC + 1) * 32;  // + one producer warp
};
constexpr int kStages = 4;                    // ring stages at most (one KV block each)
// Stages a launch uses (TcArgs.stages): 4, or 2 with HK_ATTN_STAGES=2 for blocks of 32 / 64 tokens
// (a smaller ring leaves shared memory for the neighbouring kernels of the decode chain to be
// resident at their programmatic launch); launches of more than one wave take 3 for blocks of 64
// and 2 for blocks of 32. Parity soundness with 2 or 3 stages: at 64 tokens per block every
// consumer visits every block; at 32 (2 stages only) a consumer's blocks step by 2, all in one
// stage.
// Blocks of 16 keep 4 stages (a consumer's blocks step by 4).
constexpr float kLog2e = 1.4426950408889634f;

struct TcArgs {
  const float* q;          // [R, nh, HD] fp32 (roped)
  const __nv_bfloat16* k_base;  // caches as raw pointers (speculative L2 prefetch)
  const __nv_bfloat16* v_base;
  int stages;              // ring stages used (2, 3 or 4)
  int64_t pf_bytes;        // L2 prefetch cap per CTA (the launch's share of an L2 budget)
  int64_t cache_rows;
  int table_rows;
  const int* block_tables;
  int max_blocks;
  const int* row_seq;
  const int* row_ctx;
  float scale;
  int nh, nkv, G, block_size;
  float* out;
  __nv_bfloat16* out_bf16;
  int8_t* oq;
  float* od;
  float* os;
  const float* sinks;
  int* status;
};

template <int HD, int NC>
__global__ void __launch_bounds__(Cfg<NC>::kThreads, 2)
    attn_decode_tc_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, TcArgs a) {
  constexpr int kConsumers = Cfg<NC>::kConsumers, kThreads = Cfg<NC>::kThreads;
  constexpr int NKS = HD / 16;   // k-steps of S = Q K^T
  constexpr int NDT = HD / 8;    // n8 dim tiles of O
  cg::cluster_group cluster = cg::this_cluster();
  const int S = (int)cluster.num_blocks();
  const int split = (int)cluster.block_rank();
  const int kvh = blockIdx.y, r = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bs = a.block_size;
  const int ns = a.stages;  // ring stages
  const int stage_bytes = 2 * bs * HD * 2;  // K and V of one block
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned stage area (the 128-byte swizzle repeats every 8 rows of 128 bytes)
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[kStages], empty[kStages];
  __shared__ float s_wm[kConsumers][16];
  __shared__ float s_m[16], s_l[16];
  __shared__ __align__(16) float s_o[16][HD];
  for (int i = threadIdx.x; i < 16 * HD; i += kThreads) (&s_o[0][0])[i] = 0.f;
  if (threadIdx.x < 16) s_l[threadIdx.x] = 0.f;
  if (threadIdx.x == 0) {
    for (int i = 0; i < ns; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], (uint32_t)(a.block_size / 16));  // one arrival per 16-token unit
    }
    sm100::fence_barrier_init();
  }
  if (warp == kConsumers && lane == 0 && a.table_rows > 0) {
    // Before the dependency wait: L2 prefetch of this split's K/V blocks. The context length and
    // block table may still be changing (read speculatively, clamped to valid indices); only the
    // block the kernel before this one appends to is certain to be new, and a wrong guess costs
    // a prefetch, never a result. Each CTA prefetches at most its share of an L2 budget: a wide
    // batch (64 rows x 8 KV heads x 2048 tokens = 512 MB per layer) would otherwise evict its own
    // prefetched lines before the ring reads them and fetch every byte twice.
    const int seq = a.row_seq[r], cx = a.row_ctx[r];
    if (seq >= 0 && seq < a.table_rows && cx > 0) {
      const int* bt = a.block_tables + (int64_t)seq * a.max_blocks;
      const int nbc = min((cx + bs - 1) / bs, a.max_blocks);
      const int per = (nbc + S - 1) / S;
      const uint32_t bytes = (uint32_t)bs * HD * 2;
      const int64_t pfb = a.pf_bytes / (2 * (int64_t)bytes);
      const int cap = pfb < per ? (int)pfb : per;
      const int e = min(nbc, split * per + cap);
      for (int i = split * per; i < e; ++i) {
        const int blk = bt[i];
        if (blk < 0 || (int64_t)(blk + 1) * a.nkv * bs > a.cache_rows) continue;
        const int64_t off = ((int64_t)blk * a.nkv + kvh) * bs * HD;
        sm100::prefetch_l2(a.k_base + off, bytes);
        sm100::prefetch_l2(a.v_base + off, bytes);
      }
    }
  }
  __syncthreads();
  pdl_wait();

  const int ctx = a.row_ctx[r];
  const int* btab = a.block_tables + (int64_t)a.row_seq[r] * a.max_blocks;
  const int nblk_ctx = min((ctx + bs - 1) / bs, a.max_blocks);  // never past the row's table
  const int bpc = (nblk_ctx + S - 1) / S;
  const int b0 = split * bpc, b1 = min(nblk_ctx, b0 + bpc);
  const int nb = max(0, b1 - b0);
  const int upb = bs / 16;  // 16-token units per block
  bool ok = true;

  float m_r[2] = {-INFINITY, -INFINITY};  // rows g, g + 8 (log2 domain)
  float l_r[2] = {0.f, 0.f};              // this lane's partial row sums
  float o[NDT][4];
#pragma unroll
  for (int d = 0; d < NDT; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  const int g = lane >> 2, q4 = lane & 3;

  if (warp == kConsumers) {
    // ---- producer: one lane streams the split's blocks through the ring ----
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nb && ok; ++i) {
        const int st = i % ns;
        if (i >= ns && !sm100::mbar_wait(&empty[st], (uint32_t)(((i / ns) - 1) & 1), a.status)) {
          ok = false;
          break;
        }
        issued = i + 1;
        const int row0 = (btab[b0 + i] * a.nkv + kvh) * bs;  // first token row of the block in the map
        uint8_t* dst = ring + st * stage_bytes;
        sm100::mbar_arrive_expect_tx(&full[st], (uint32_t)stage_bytes);
#pragma unroll
        for (int bx = 0; bx < HD / 64; ++bx) {
          sm100::tma_load_2d(dst + bx * bs * 128, &tk, bx * 64, row0, &full[st]);
          sm100::tma_load_2d(dst + bs * HD * 2 + bx * bs * 128, &tv, bx * 64, row0, &full[st]);
        }
      }
      // unwinding or done: every issued copy must land before the CTA may exit
      for (int i = max(0, issued - ns); i < issued; ++i)
        sm100::mbar_wait(&full[i % ns], (uint32_t)((i / ns) & 1), nullptr, 1u << 22);
    }
  } else {
    // ---- consumers: 16-token units, unit u of block u / upb taken by warp u % kConsumers ----
    const float qs = a.scale * kLog2e;
    uint32_t qa[NKS][4];
    {
      const float* qb = a.q + ((int64_t)r * a.nh + (int64_t)kvh * a.G) * HD;
      const bool v0 = g < a.G, v1 = g + 8 < a.G;
#pragma unroll
      for (int ks = 0; ks < NKS; ++ks) {
        const int d0 = 16 * ks + 2 * q4, d1 = d0 + 8;
        const float* r0 = qb + (int64_t)g * HD;
        const float* r1 = qb + (int64_t)(g + 8) * HD;
        qa[ks][0] = v0 ? pack_bf16(r0[d0], r0[d0 + 1]) : 0u;
        qa[ks][1] = v1 ? pack_bf16(r1[d0], r1[d0 + 1]) : 0u;
        qa[ks][2] = v0 ? pack_bf16(r0[d1], r0[d1 + 1]) : 0u;
        qa[ks][3] = v1 ? pack_bf16(r1[d1], r1[d1 + 1]) : 0u;
      }
    }
    const uint32_t ring_s = sm100::smem_u32(ring);
    for (int u = warp; u < nb * upb && ok; u += kConsumers) {
      const int i = u / upb, t = u - i * upb, st = i % ns;
      if (!sm100::mbar_wait(&full[st], (uint32_t)((i / ns) & 1), a.status)) {
        ok = false;
        break;
      }
      const uint32_t kb = ring_s + st * stage_bytes, vb = kb + bs * HD * 2;
      // S = Q K^T for tokens 16t .. 16t + 15 of the block (two n8 tiles)
      float sc[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
        const int row = 16 * t + 8 * j + (lane & 7);
#pragma unroll
        for (int pq = 0; pq < HD / 32; ++pq) {
          uint32_t kr[4];
          ldsm_x4(sw_addr(kb, bs, row, 4 * pq + (lane >> 3)), kr);
          mma16816(sc[j], qa[2 * pq], kr[0], kr[1]);
          mma16816(sc[j], qa[2 * pq + 1], kr[2], kr[3]);
        }
      }
      // scale into the log2 domain, mask tokens past the context, online softmax per head row
      const int tok0 = (b0 + i) * bs + 16 * t + 2 * q4;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          sc[j][e] = tok0 + 8 * j + (e & 1) < ctx ? sc[j][e] * qs : -INFINITY;
      float mx[2] = {fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1])),
                     fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]))};
      float alpha[2], mref[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
        const float mn = fmaxf(m_r[h], mx[h]);
        mref[h] = mn == -INFINITY ? 0.f : mn;  // all masked so far: p = 0 and nothing to rescale
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
      // O = O * alpha + P V
      const int vrow = 16 * t + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
      for (int dd = 0; dd < NDT / 2; ++dd) {
        uint32_t vr[4];
        ldsm_x4_t(sw_addr(vb, bs, vrow, 2 * dd + (lane >> 4)), vr);
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
      if (lane == 0) sm100::mbar_arrive(&empty[st]);
    }
  }

  // ---- fold the consumer warps into one (max, sum, O) per CTA ----
  if (warp < kConsumers) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 1);
      l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 2);
    }
    if (q4 == 0) {
      s_wm[warp][g] = m_r[0];
      s_wm[warp][g + 8] = m_r[1];
    }
  }
  __syncthreads();
  if (warp < kConsumers) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = g + 8 * h;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) M = fmaxf(M, s_wm[w][row]);
      const float f = m_r[h] == -INFINITY ? 0.f : exp2f(m_r[h] - M);
      if (f != 0.f) {
#pragma unroll
        for (int d = 0; d < NDT; ++d) {
          atomicAdd(&s_o[row][8 * d + 2 * q4], o[d][2 * h] * f);
          atomicAdd(&s_o[row][8 * d + 2 * q4 + 1], o[d][2 * h + 1] * f);
        }
        if (q4 == 0) atomicAdd(&s_l[row], l_r[h] * f);
      }
      if (warp == 0 && q4 == 0) s_m[row] = M;
    }
  }
  pdl_launch();
  cluster.sync();  // every CTA's (m, l, o) is complete and visible to the cluster

  // ---- merge whole 32-dim blocks across the cluster; CTA s takes blocks s, s + S, ... ----
  const int64_t width = (int64_t)a.nh * HD;
  const int64_t col0 = (int64_t)kvh * a.G * HD;
  const int nblk_out = a.G * HD / 32;
  constexpr int W = kThreads / 32;
  for (int blk = split + S * warp; blk < nblk_out; blk += S * W) {
    const int idx = blk * 32 + lane;
    const int hr = idx / HD, d = idx % HD;
    float mk[8], lk[8], okv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k < S) {
        mk[k] = *cluster.map_shared_rank(&s_m[hr], k);
        lk[k] = *cluster.map_shared_rank(&s_l[hr], k);
        okv[k] = *cluster.map_shared_rank(&s_o[hr][d], k);
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (k < S) M = fmaxf(M, mk[k]);
    const float sink = a.sinks ? a.sinks[kvh * a.G + hr] * kLog2e : -INFINITY;
    M = fmaxf(M, sink);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k < S && mk[k] != -INFINITY) {
        const float f = exp2f(mk[k] - M);
        L += lk[k] * f;
        O += okv[k] * f;
      }
    }
    if (a.sinks) L += exp2f(sink - M);
    const float v = L > 0.f ? O / L : 0.f;
    if (a.out) a.out[(int64_t)r * width + col0 + idx] = v;
    if (a.out_bf16) a.out_bf16[(int64_t)r * width + col0 + idx] = __float2bfloat16(v);
    if (a.oq) {
      const float amax = warp_max(fabsf(v));
      const float dq = amax / 127.f;
      const int qv = amax > 0.f ? __float2int_rn(v / dq) : 0;
      const float qsum = warp_sum((float)qv);
      a.oq[(int64_t)r * width + col0 + idx] = (int8_t)qv;
      if (lane == 0) {
        a.od[(int64_t)r * (width / 32) + (col0 >> 5) + blk] = dq;
        a.os[(int64_t)r * (width / 32) + (col0 >> 5) + blk] = dq * qsum;
      }
    }
  }
  cluster.sync();  // keep this CTA's shared memory alive until every CTA has read it
}

// Tensor maps of the K and V caches ([num_blocks * nkv * block_size rows, HD cols] bf16, boxes of
// [64 dims x block_size rows], 128-byte swizzle), encoded once per cache tensor on the host.
struct MapKey {
  const void* base;
  int64_t rows;
  int hd, bs;
  bool operator==(const MapKey& o) const { return base == o.base && rows == o.rows && hd == o.hd && bs == o.bs; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.base) ^ (std::hash<int64_t>()(k.rows) * 31) ^ ((size_t)k.hd << 20) ^ k.bs;
  }
};

const CUtensorMap& kv_map(const void* base, int64_t rows, int hd, int bs) {
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  const MapKey k{base, rows, hd, bs};
  auto it = cache.find(k);
  if (it != cache.end()) return it->second;
  CUtensorMap m = tma_map_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, (uint64_t)hd, (uint64_t)rows, (uint64_t)hd * 2,
                             64, (uint32_t)bs, CU_TENSOR_MAP_SWIZZLE_128B);
  return cache.emplace(k, m).first->second;
}

template <int HD, int NC>
void launch_hd_nc(const AttnDecodeArgs& a, int64_t cache_rows, cudaStream_t s, bool pdl) {
  TcArgs t{};
  t.q = a.q;
  t.k_base = a.k_cache;
  t.v_base = a.v_cache;
  t.cache_rows = cache_rows;
  t.table_rows = a.table_rows;
  t.block_tables = a.block_tables;
  t.max_blocks = a.max_blocks;
  t.row_seq = a.row_seq;
  t.row_ctx = a.row_ctx;
  t.scale = a.scale;
  t.nh = a.nh;
  t.nkv = a.nkv;
  t.G = a.nh / a.nkv;
  t.block_size = a.block_size;
  t.out = a.out;
  t.out_bf16 = a.out_bf16;
  t.oq = a.oq;
  t.od = a.od;
  t.os = a.os;
  t.sinks = a.sinks;
  t.status = a.status;
  const CUtensorMap tk = kv_map(a.k_cache, cache_rows, HD, a.block_size);
  const CUtensorMap tv = kv_map(a.v_cache, cache_rows, HD, a.block_size);
  static const int env_stages = [] {
    const char* e = getenv("HK_ATTN_STAGES");
    return e && atoi(e) == 2 ? 2 : kStages;
  }();
  // Many CTAs (wide decode batches): the launch has more than one wave and 2 CTAs share an SM
  // (162 registers per thread), so ring depth sets the bytes in flight per SM. Blocks of 64 tokens
  // take 3 stages (2 x 105 KB fits an SM; every consumer visits every block, so a 3-stage parity
  // wait stays sound), blocks of 32 keep 2. Measured at Llama-3-8B bs64 (64 rows x 8 KV heads x
  // 2048 tokens): 3 stages 98.9 us, 2 stages 100.6 us; 128 registers for 3 CTAs per SM with 2
  // stages measured 126.9 us.
  const bool many = (int64_t)a.num_splits * a.nkv * a.R > 148;
  if (a.block_size == 16) t.stages = kStages;
  else if (!many) t.stages = env_stages;
  else t.stages = a.block_size == 64 ? 3 : 2;
  // L2 prefetch budget of the whole launch (default 48 MB of the 126 MB L2), split evenly per CTA
  static const int64_t pf_budget = [] {
    const char* e = getenv("HK_ATTN_PREFETCH_MB");
    return (int64_t)(e ? atoi(e) : 48) << 20;
  }();
  t.pf_bytes = pf_budget / ((int64_t)a.num_splits * a.nkv * a.R);
  const size_t smem = 1024 + (size_t)t.stages * 2 * a.block_size * HD * 2;
  auto kern = attn_decode_tc_kernel<HD, NC>;
  HK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  launch_cluster(kern, dim3(a.num_splits, a.nkv, a.R), dim3(Cfg<NC>::kThreads), smem, s, pdl, a.num_splits, tk, tv, t);
}

template <int HD>
void launch_hd(const AttnDecodeArgs& a, int64_t cache_rows, cudaStream_t s, bool pdl) {
  // 4 consumers: 8 (sound for blocks of 32 / 64) measured slower both at Llama-3-8B bs1 decode
  // shapes (12.4 vs 10.6 us per layer; the fold into shared memory doubles) and at bs64
  // (187 vs 135 us per layer); 2 splits at bs64 measured slower too (153 us)
  launch_hd_nc<HD, 4>(a, cache_rows, s, pdl);
}

}  // namespace atc

bool attention_decode_tc_supported(const AttnDecodeArgs& a) {
  const int G = a.nkv > 0 ? a.nh / a.nkv : 0;
  return (a.hd == 64 || a.hd == 128) && G >= 1 && G <= 16 && a.nh % a.nkv == 0 &&
         (a.block_size == 16 || a.block_size == 32 || a.block_size == 64) &&
         (a.num_splits == 1 || a.num_splits == 2 || a.num_splits == 4 || a.num_splits == 8);
}

void attention_decode_tc_launch(const AttnDecodeArgs& a, int64_t cache_rows, cudaStream_t s, bool pdl) {
  if (a.R <= 0) return;  // no rows: nothing to launch (and no per-CTA prefetch share to compute)
  if (!attention_decode_tc_supported(a)) throw std::runtime_error("attention (tensor cores): unsupported shape");
  if ((reinterpret_cast<uintptr_t>(a.k_cache) | reinterpret_cast<uintptr_t>(a.v_cache)) & 15)
    throw std::runtime_error("attention (tensor cores): K/V caches must be 16-byte aligned");
  if (a.hd == 64) atc::launch_hd<64>(a, cache_rows, s, pdl);
  else atc::launch_hd<128>(a, cache_rows, s, pdl);
}

}  // namespace hk
