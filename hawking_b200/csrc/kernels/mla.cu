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
// Grid (heads, 4 latent quarters); 256 threads: thread t owns 8 consecutive latent dims of the
// quarter (t / 16) and one sixteenth of the nope rows (t % 16), with 16-byte weight loads (two
// neighbouring threads read one 32-byte sector); the 16 partial sums of each dim meet through
// shuffles inside the half-warp. All rows (<= 8) reuse the loaded weights.
constexpr int kAbsorbMaxRows = 8;
__global__ void __launch_bounds__(256) mla_absorb_q_kernel(MlaAbsorbArgs a, int rows) {
  __shared__ float qn[kAbsorbMaxRows][256];
  pdl_wait();
  const int h = blockIdx.x, quarter = blockIdx.y, tid = threadIdx.x;
  const int stride_q = a.nh * (a.nope + kMlaRope);
  for (int i = tid; i < rows * a.nope; i += blockDim.x) {
    const int r = i / a.nope, k = i % a.nope;
    qn[r][k] = a.q[(int64_t)r * stride_q + (int64_t)h * (a.nope + kMlaRope) + k];
  }
  __syncthreads();
  const int c8 = tid >> 4, ig = tid & 15;
  const int d0 = quarter * 128 + c8 * 8;
  const int per = a.nope / 16;
  const __nv_bfloat16* w = a.w_uk + (int64_t)h * a.nope * kMlaLat + d0;
  float acc[kAbsorbMaxRows][8];
#pragma unroll
  for (int r = 0; r < kAbsorbMaxRows; ++r)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[r][e] = 0.f;
#pragma unroll 4
  for (int ii = 0; ii < per; ++ii) {
    const int i = ii * 16 + ig;
    const uint4 u = *reinterpret_cast<const uint4*>(w + (int64_t)i * kMlaLat);
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&u);
    float wv[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(b2[e]);
      wv[2 * e] = f.x;
      wv[2 * e + 1] = f.y;
    }
#pragma unroll
    for (int r = 0; r < kAbsorbMaxRows; ++r) {
      if (r < rows) {
        const float qv = qn[r][i];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[r][e] += qv * wv[e];
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kAbsorbMaxRows; ++r) {
    if (r < rows) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float v = acc[r][e];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[r][e] = v;
      }
      if (ig == 0) {
        float* dst = a.q_lat + ((int64_t)r * a.nh + h) * kMlaLat + d0;
        *reinterpret_cast<float4*>(dst) = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(acc[r][4], acc[r][5], acc[r][6], acc[r][7]);
      }
    }
  }
  if (quarter == 0) {
    for (int o = tid; o < rows * (kMlaRope / 2); o += blockDim.x) {
      const int r = o / (kMlaRope / 2), t = o % (kMlaRope / 2);
      const float* q = a.q + (int64_t)r * stride_q + (int64_t)h * (a.nope + kMlaRope);
      const int pos = a.positions[r];
      float x = q[a.nope + t], y = q[a.nope + t + kMlaRope / 2];
      const float* cs = a.rope + (int64_t)pos * kMlaRope + 2 * t;
      rope_neox_pair(x, y, cs[0], cs[1]);
      float* qp = a.q_pe + ((int64_t)r * a.nh + h) * kMlaRope;
      qp[t] = x;
      qp[t + kMlaRope / 2] = y;
    }
  }
  pdl_launch();
}

void mla_absorb_q_launch(const MlaAbsorbArgs& a, int rows, cudaStream_t s, bool pdl) {
  if (a.nope > 256 || a.nope % 16) throw std::runtime_error("mla: nope dim must be a multiple of 16, <= 256");
  if (rows > kAbsorbMaxRows) throw std::runtime_error("mla absorb: at most 8 rows");
  launch(mla_absorb_q_kernel, dim3(a.nh, 4), dim3(256), 0, s, pdl, a, rows);
}

// ---- output: o[h] = W_UV[h] o_lat[h] -> q8 ------------------------------------------------------
// Grid (heads, vdim / 32): one CTA per 32 output dims of a head (one q8 block); 8 warps x 4
// output rows, lanes over the 512 latent dims with 16-byte weight loads; all rows (<= 8) reuse
// the loaded weights.
constexpr int kOutMaxRows = 8;
__global__ void __launch_bounds__(256) mla_out_kernel(MlaOutArgs a, int rows) {
  __shared__ __align__(16) float ol[kOutMaxRows][kMlaLat];
  __shared__ float ov[kOutMaxRows][32];
  pdl_wait();
  const int h = blockIdx.x, jb = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < rows * kMlaLat; i += blockDim.x) {
    const int r = i / kMlaLat, d = i % kMlaLat;
    ol[r][d] = a.o_lat[((int64_t)r * a.nh + h) * kMlaLat + d];
  }
  __syncthreads();
  const __nv_bfloat16* w = a.w_uv + ((int64_t)h * a.vdim + jb * 32) * kMlaLat;
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const int j = warp * 4 + jj;
    const __nv_bfloat16* wr = w + (int64_t)j * kMlaLat;
    float acc[kOutMaxRows];
#pragma unroll
    for (int r = 0; r < kOutMaxRows; ++r) acc[r] = 0.f;
#pragma unroll
    for (int c = 0; c < 2; ++c) {  // 2 x 8 dims per lane covers 512
      const int d0 = (c * 32 + lane) * 8;
      const uint4 u = *reinterpret_cast<const uint4*>(wr + d0);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(b2[e]);
#pragma unroll
        for (int r = 0; r < kOutMaxRows; ++r)
          if (r < rows) acc[r] += f.x * ol[r][d0 + 2 * e] + f.y * ol[r][d0 + 2 * e + 1];
      }
    }
#pragma unroll
    for (int r = 0; r < kOutMaxRows; ++r) {
      if (r < rows) {
        const float v = warp_sum(acc[r]);
        if (lane == 0) ov[r][j] = v;
      }
    }
  }
  __syncthreads();
  pdl_launch();
  const int64_t width = (int64_t)a.nh * a.vdim;
  if (warp < rows) {  // warp r quantises row r's 32-dim block
    const int r = warp;
    const float v = ov[r][lane];
    const int64_t col = (int64_t)h * a.vdim + jb * 32 + lane;
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
  if (rows > kOutMaxRows) throw std::runtime_error("mla out: at most 8 rows");
  launch(mla_out_kernel, dim3(a.nh, a.vdim / 32), dim3(256), 0, s, pdl, a, rows);
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

int mla_heads_per_cta(int nh, int rows) {
  // 4 heads share each latent row a CTA stages, unless that leaves too few CTAs (tensor-parallel
  // shards hold nh / N heads): then 2 or 1, trading latent re-reads (L2) for parallelism
  if (nh % 4 == 0 && rows * (nh / 4) >= 16) return 4;
  if (nh % 2 == 0 && rows * (nh / 2) >= 16) return 2;
  return 1;
}

template <int G>
static void mla_decode_go(const MlaDecodeArgs& a, size_t smem, cudaStream_t s, bool pdl) {
  constexpr int WARPS = 8;
  auto kern = mla_decode_kernel<G, WARPS>;
  HK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  launch_cluster(kern, dim3(a.num_splits, a.nh / G, a.R), dim3(WARPS * 32), smem, s, pdl, a.num_splits, a);
}

void mla_decode_launch(MlaDecodeArgs a, cudaStream_t s, bool pdl) {
  const int G = mla_heads_per_cta(a.nh, a.R);
  if (a.num_splits != 1 && a.num_splits != 2 && a.num_splits != 4 && a.num_splits != 8)
    throw std::runtime_error("mla: num_splits must be 1, 2, 4 or 8");
  const int slab_bytes = a.block_size * kMlaRow * 2;
  const int most = (a.max_blocks + a.num_splits - 1) / a.num_splits;
  int ns = std::min(most, (192 * 1024) / slab_bytes);
  if (ns < most && ns >= 2) ns &= ~1;
  if (ns < 1 || (ns < most && ns < 2)) throw std::runtime_error("mla: latent block too large for the ring");
  a.stage_blocks = ns;
  const size_t smem = 128 + (size_t)ns * slab_bytes;
  if (G == 4) mla_decode_go<4>(a, smem, s, pdl);
  else if (G == 2) mla_decode_go<2>(a, smem, s, pdl);
  else mla_decode_go<1>(a, smem, s, pdl);
}

}  // namespace hk
