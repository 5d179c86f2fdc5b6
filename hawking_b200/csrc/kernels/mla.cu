// Multi-head latent attention (MLA, K6): decode over the compressed latent cache, with the key and
// value up-projections absorbed into the query and the output.
//
// Cache: one 576-wide bf16 vector per token, [num_blocks, block_size, 576] = RMSNorm'd latent c
// (512) followed by the RoPE'd shared key k_pe (64). Per head h of the token being decoded:
//   q_lat[h] = W_UK[h]^T q_nope[h]        (mla_absorb_q: [128] -> [512]; q_pe[h] RoPE'd)
//   s_t      = (q_lat[h] . c_t + q_pe[h] . k_pe_t) * scale
//   o_lat[h] = sum_t softmax(s)_t c_t      (mla_decode: every head reads the same latent tokens)
//   o[h]     = W_UV[h] o_lat[h]            (mla_out: [512] -> [128], emitted as q8 for W_o)
// mla_kv_append normalises the new token's latent (kv_a RMSNorm), RoPEs its k_pe and writes the
// cache slot; RoPE is the neox (halves) rotation over the 64 rope dims.
//
// mla_decode follows the cluster split-KV design of attention.cu: the splits of one (row, head
// group) are a thread-block cluster; each CTA streams its token range's latent block slabs into
// shared memory with bulk async copies (double-buffered windows when the range does not fit),
// warps take tiles of 8 tokens (lane = latent dims lane + 32 i, so both the 576-dim score and the
// 512-dim value read the same shared row), and the partial (max, sum, o_lat) are merged across the
// cluster through distributed shared memory.
//
// Parity: crates/hawking-core/src/attn.rs:185 (mla_decode_step: scores over uk @ c plus the shared
// rope key, values uv @ c), crates/hawking-core/shaders/attn.metal:18-47 (absorbed W_UK into q,
// W_UV after the weighted sum), crates/hawking-core/src/model/deepseek_v2.rs:98-158 (kv_lora 512,
// rope 64, nope 128, v 128).
#include "decode_ops.cuh"
#include "sm100.cuh"

#include <algorithm>
#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace hk {

constexpr int kMlaLat = 512, kMlaRope = 64, kMlaRow = 576;

__device__ __forceinline__ void rope_neox_pair(float& a, float& b, float c, float s) {
  const float x = a, y = b;
  a = x * c - y * s;
  b = y * c + x * s;
}

// ---- new token: latent RMSNorm + k_pe RoPE -> cache slot -----------------------------------------
__global__ void __launch_bounds__(256) mla_kv_append_kernel(MlaAppendArgs a) {
  __shared__ float red[32];
  pdl_wait();
  const int r = blockIdx.x, tid = threadIdx.x;
  const float* kv = a.kv_a + (int64_t)r * a.kv_a_stride;
  const int pos = a.positions[r];
  const int* btab = a.block_tables + (int64_t)a.row_seq[r] * a.max_blocks;
  const int64_t slot = (int64_t)btab[pos / a.block_size] * a.block_size + pos % a.block_size;
  __nv_bfloat16* dst = a.cache + slot * kMlaRow;
  float v0 = kv[tid], v1 = kv[tid + 256];
  const float ss = block_sum(v0 * v0 + v1 * v1, red);
  const float inv = rsqrtf(ss / kMlaLat + a.eps);
  dst[tid] = __float2bfloat16(v0 * inv * a.norm_w[tid]);
  dst[tid + 256] = __float2bfloat16(v1 * inv * a.norm_w[tid + 256]);
  if (tid < kMlaRope / 2) {
    float x = kv[kMlaLat + tid], y = kv[kMlaLat + tid + kMlaRope / 2];
    const float* cs = a.rope + (int64_t)pos * kMlaRope + 2 * tid;
    rope_neox_pair(x, y, cs[0], cs[1]);
    dst[kMlaLat + tid] = __float2bfloat16(x);
    dst[kMlaLat + tid + kMlaRope / 2] = __float2bfloat16(y);
  }
  pdl_launch();
}

void mla_kv_append_launch(const MlaAppendArgs& a, int rows, cudaStream_t s, bool pdl) {
  launch(mla_kv_append_kernel, dim3(rows), dim3(256), 0, s, pdl, a);
}

// ---- q absorption: q_lat[h] = W_UK[h]^T q_nope[h]; q_pe RoPE ------------------------------------
// Grid (heads, rows), 256 threads; W_UK is [heads, nope, 512] bf16 (row i = key dim i of head h).
__global__ void __launch_bounds__(256) mla_absorb_q_kernel(MlaAbsorbArgs a) {
  __shared__ float qn[256];
  pdl_wait();
  const int h = blockIdx.x, r = blockIdx.y, tid = threadIdx.x;
  const float* q = a.q + ((int64_t)r * a.nh + h) * (a.nope + kMlaRope);
  if (tid < a.nope) qn[tid] = q[tid];
  __syncthreads();
  const __nv_bfloat16* w = a.w_uk + (int64_t)h * a.nope * kMlaLat;
  float acc0 = 0.f, acc1 = 0.f;
  for (int i = 0; i < a.nope; ++i) {
    acc0 += qn[i] * __bfloat162float(w[(int64_t)i * kMlaLat + tid]);
    acc1 += qn[i] * __bfloat162float(w[(int64_t)i * kMlaLat + tid + 256]);
  }
  float* ql = a.q_lat + ((int64_t)r * a.nh + h) * kMlaLat;
  ql[tid] = acc0;
  ql[tid + 256] = acc1;
  if (tid < kMlaRope / 2) {
    const int pos = a.positions[r];
    float x = q[a.nope + tid], y = q[a.nope + tid + kMlaRope / 2];
    const float* cs = a.rope + (int64_t)pos * kMlaRope + 2 * tid;
    rope_neox_pair(x, y, cs[0], cs[1]);
    float* qp = a.q_pe + ((int64_t)r * a.nh + h) * kMlaRope;
    qp[tid] = x;
    qp[tid + kMlaRope / 2] = y;
  }
  pdl_launch();
}

void mla_absorb_q_launch(const MlaAbsorbArgs& a, int rows, cudaStream_t s, bool pdl) {
  if (a.nope > 256) throw std::runtime_error("mla: nope dim must be <= 256");
  launch(mla_absorb_q_kernel, dim3(a.nh, rows), dim3(256), 0, s, pdl, a);
}

// ---- output: o[h] = W_UV[h] o_lat[h] -> q8 ------------------------------------------------------
// Grid (heads, rows), 128 threads (4 warps); W_UV is [heads, v_dim, 512] bf16; warp-per-row.
__global__ void __launch_bounds__(128) mla_out_kernel(MlaOutArgs a) {
  __shared__ float ol[kMlaLat];
  __shared__ float ov[256];
  pdl_wait();
  const int h = blockIdx.x, r = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* src = a.o_lat + ((int64_t)r * a.nh + h) * kMlaLat;
  for (int i = tid; i < kMlaLat; i += blockDim.x) ol[i] = src[i];
  __syncthreads();
  const __nv_bfloat16* w = a.w_uv + (int64_t)h * a.vdim * kMlaLat;
  for (int j = warp; j < a.vdim; j += 4) {
    const __nv_bfloat16* wr = w + (int64_t)j * kMlaLat;
    float acc = 0.f;
#pragma unroll 4
    for (int k = lane; k < kMlaLat; k += 32) acc += __bfloat162float(wr[k]) * ol[k];
    acc = warp_sum(acc);
    if (lane == 0) ov[j] = acc;
  }
  __syncthreads();
  pdl_launch();
  const int64_t width = (int64_t)a.nh * a.vdim;
  for (int j = tid; j < a.vdim; j += blockDim.x) {  // whole warps: vdim % 32 == 0
    const float v = ov[j];
    const int64_t col = (int64_t)h * a.vdim + j;
    const float amax = warp_max(fabsf(v));
    const float d = amax / 127.f;
    const int q = amax > 0.f ? __float2int_rn(v / d) : 0;
    const float qs = warp_sum((float)q);
    a.oq[(int64_t)r * width + col] = (int8_t)q;
    if (lane == 0) {
      a.od[(int64_t)r * (width / 32) + (col >> 5)] = d;
      a.os[(int64_t)r * (width / 32) + (col >> 5)] = d * qs;
    }
  }
}

void mla_out_launch(const MlaOutArgs& a, int rows, cudaStream_t s, bool pdl) {
  if (a.vdim % 32 || a.vdim > 256) throw std::runtime_error("mla: v dim must be a multiple of 32, <= 256");
  launch(mla_out_kernel, dim3(a.nh, rows), dim3(128), 0, s, pdl, a);
}

// ---- attention over the latent cache --------------------------------------------------------
template <int G, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) mla_decode_kernel(MlaDecodeArgs a) {
  constexpr int T = 16 / G > 4 ? 4 : 16 / G;  // tokens per warp tile (register budget: 18 dims per token)
  constexpr int NV = G * T;
  constexpr int NQ = kMlaRow / 32;   // 18 score dims per lane
  constexpr int NO = kMlaLat / 32;   // 16 value dims per lane
  cg::cluster_group cluster = cg::this_cluster();
  const int S = (int)cluster.num_blocks();
  const int split = (int)cluster.block_rank();
  const int hg = blockIdx.y, r = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  extern __shared__ __align__(128) uint8_t mla_smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(mla_smem);
  __nv_bfloat16* ring = reinterpret_cast<__nv_bfloat16*>(mla_smem + 128);
  __shared__ float s_wm[WARPS][G];
  __shared__ float s_m[G], s_l[G];
  __shared__ __align__(16) float s_o[G][kMlaLat];
  for (int i = threadIdx.x; i < G * kMlaLat; i += blockDim.x) (&s_o[0][0])[i] = 0.f;
  if (threadIdx.x < G) s_l[threadIdx.x] = 0.f;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&full[0], 1);
    sm100::mbar_init(&full[1], 1);
    sm100::fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();
  const int bs = a.block_size;
  const int slab = bs * kMlaRow;
  const int ctx = a.row_ctx[r];
  const int* btab = a.block_tables + (int64_t)a.row_seq[r] * a.max_blocks;
  const int nblk_ctx = (ctx + bs - 1) / bs;
  const int bpc = (nblk_ctx + S - 1) / S;
  const int b0 = split * bpc, b1 = min(nblk_ctx, b0 + bpc);
  const int t0 = b0 * bs, t1 = min(ctx, b1 * bs);
  const int nb = max(0, b1 - b0);
  const int NS = a.stage_blocks;
  const bool dbl = nb > NS;
  const int WB = dbl ? NS / 2 : NS;
  const int nwin = nb > 0 ? (nb + WB - 1) / WB : 0;
  auto issue = [&](int w) {
    const int buf = dbl ? (w & 1) : 0;
    const int wb0 = b0 + w * WB, wb1 = min(b1, wb0 + WB);
    sm100::mbar_arrive_expect_tx(&full[buf], (uint32_t)((wb1 - wb0) * slab * 2));
    for (int b = wb0; b < wb1; ++b)
      sm100::bulk_g2s(ring + (int64_t)(buf * WB + (b - wb0)) * slab, a.cache + (int64_t)btab[b] * slab,
                      (uint32_t)slab * 2, &full[buf]);
  };
  if (threadIdx.x == 0 && nwin > 0) {
    issue(0);
    if (dbl && nwin > 1) issue(1);
  }
  // queries of the head group in shared memory (lane-strided like the cache rows), scaled
  __shared__ float s_q[G][kMlaRow];
  for (int i = threadIdx.x; i < G * kMlaRow; i += blockDim.x) {
    const int g = i / kMlaRow, d = i % kMlaRow, h = hg * G + g;
    s_q[g][d] = (d < kMlaLat ? a.q_lat[((int64_t)r * a.nh + h) * kMlaLat + d]
                             : a.q_pe[((int64_t)r * a.nh + h) * kMlaRope + d - kMlaLat]) * a.scale;
  }
  __syncthreads();
  float m[G], l[G], acc[G][NO];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < NO; ++i) acc[g][i] = 0.f;
  }
  bool ok = true;
  for (int w = 0; w < nwin; ++w) {
    const int buf = dbl ? (w & 1) : 0;
    const uint32_t parity = (uint32_t)((dbl ? (w >> 1) : w) & 1);
    if (ok) {
      ok = sm100::mbar_wait(&full[buf], parity, a.status);
      if (!ok && threadIdx.x == 0)
        for (uint32_t i = 0; i < (1u << 20) && !sm100::mbar_try_wait(&full[buf], parity); ++i) {
        }
    }
    const int wb0 = b0 + w * WB;
    const int tw0 = max(t0, wb0 * bs), tw1 = min(t1, min(b1, wb0 + WB) * bs);
    const __nv_bfloat16* base = ring + (int64_t)buf * WB * slab;
    for (int tt = tw0 + warp * T; ok && tt < tw1; tt += WARPS * T) {
      float part[32];
#pragma unroll
      for (int v = NV; v < 32; ++v) part[v] = 0.f;
#pragma unroll
      for (int j = 0; j < T; ++j) {
        const int t = min(tt + j, tw1 - 1);
        const __nv_bfloat16* row = base + (int64_t)(t - wb0 * bs) * kMlaRow;
        float kr[NQ];  // (loaded per token)
#pragma unroll
        for (int i = 0; i < NQ; ++i) kr[i] = __bfloat162float(row[lane + 32 * i]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float sdot = 0.f;
#pragma unroll
          for (int i = 0; i < NQ; ++i) sdot = fmaf(s_q[g][lane + 32 * i], kr[i], sdot);
          part[g * T + j] = sdot;
        }
      }
#pragma unroll
      for (int o = 16, n = 32; o > 0; o >>= 1, n >>= 1) {
        const bool up = lane & o;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
          const float send = up ? part[i] : part[i + n / 2];
          const float keep = up ? part[i + n / 2] : part[i];
          part[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      const int my_g = min(lane / T, G - 1), my_j = lane % T;
      const float score = (lane < NV && tt + my_j < tw1) ? part[0] : -INFINITY;
      float tmax = score;
#pragma unroll
      for (int o = T / 2; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      float p_new_m[G], alpha[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float tm = __shfl_sync(0xffffffffu, tmax, g * T);
        p_new_m[g] = fmaxf(m[g], tm);
        alpha[g] = __expf(m[g] - p_new_m[g]);
      }
      float mg = p_new_m[0];
#pragma unroll
      for (int g = 1; g < G; ++g)
        if (my_g == g) mg = p_new_m[g];
      const float p = (score == -INFINITY) ? 0.f : __expf(score - mg);
      float psum = p;
#pragma unroll
      for (int o = T / 2; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float ps = __shfl_sync(0xffffffffu, psum, g * T);
        l[g] = l[g] * alpha[g] + ps;
        m[g] = p_new_m[g];
#pragma unroll
        for (int i = 0; i < NO; ++i) acc[g][i] *= alpha[g];
      }
#pragma unroll
      for (int j = 0; j < T; ++j) {
        const int t = min(tt + j, tw1 - 1);
        const __nv_bfloat16* row = base + (int64_t)(t - wb0 * bs) * kMlaRow;
        float vr[NO];
#pragma unroll
        for (int i = 0; i < NO; ++i) vr[i] = __bfloat162float(row[lane + 32 * i]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float pg = __shfl_sync(0xffffffffu, p, g * T + j);
#pragma unroll
          for (int i = 0; i < NO; ++i) acc[g][i] = fmaf(pg, vr[i], acc[g][i]);
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && dbl && w + 2 < nwin && ok) issue(w + 2);
  }
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) s_wm[warp][g] = m[g];
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, s_wm[w][g]);
    const float f = (m[g] == -INFINITY) ? 0.f : __expf(m[g] - M);
    if (f != 0.f) {
#pragma unroll
      for (int i = 0; i < NO; ++i) atomicAdd(&s_o[g][lane + 32 * i], acc[g][i] * f);
      if (lane == 0) atomicAdd(&s_l[g], l[g] * f);
    }
    if (warp == 0 && lane == 0) s_m[g] = M;
  }
  pdl_launch();
  cluster.sync();
  // merge: CTA s handles dims [s * 512 / S, (s + 1) * 512 / S) of every head of the group
  const int per = kMlaLat / S;
  for (int idx = threadIdx.x; idx < G * per; idx += blockDim.x) {
    const int g = idx / per, d = split * per + idx % per;
    float M = -INFINITY;
    for (int k = 0; k < S; ++k) M = fmaxf(M, *cluster.map_shared_rank(&s_m[g], k));
    float L = 0.f, O = 0.f;
    for (int k = 0; k < S; ++k) {
      const float mk = *cluster.map_shared_rank(&s_m[g], k);
      if (mk == -INFINITY) continue;
      const float f = __expf(mk - M);
      L += *cluster.map_shared_rank(&s_l[g], k) * f;
      O += *cluster.map_shared_rank(&s_o[g][d], k) * f;
    }
    a.o_lat[((int64_t)r * a.nh + hg * G + g) * kMlaLat + d] = L > 0.f ? O / L : 0.f;
  }
  cluster.sync();
}

void mla_decode_launch(MlaDecodeArgs a, cudaStream_t s, bool pdl) {
  constexpr int G = 4, WARPS = 8;
  if (a.nh % G) throw std::runtime_error("mla: heads must be a multiple of 4");
  if (a.num_splits != 1 && a.num_splits != 2 && a.num_splits != 4 && a.num_splits != 8)
    throw std::runtime_error("mla: num_splits must be 1, 2, 4 or 8");
  const int slab_bytes = a.block_size * kMlaRow * 2;
  const int most = (a.max_blocks + a.num_splits - 1) / a.num_splits;
  int ns = std::min(most, (192 * 1024) / slab_bytes);
  if (ns < most && ns >= 2) ns &= ~1;
  if (ns < 1 || (ns < most && ns < 2)) throw std::runtime_error("mla: latent block too large for the ring");
  a.stage_blocks = ns;
  const size_t smem = 128 + (size_t)ns * slab_bytes;
  auto kern = mla_decode_kernel<G, WARPS>;
  HK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  launch_cluster(kern, dim3(a.num_splits, a.nh / G, a.R), dim3(WARPS * 32), smem, s, pdl, a.num_splits, a);
}

}  // namespace hk
