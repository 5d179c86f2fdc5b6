// Absorbed MLA decode on the tensor cores (K6): flash-style attention of up to 16 query heads
// (the MMA M dimension) over the paged bf16 latent cache (576 per token: 512 latent + 64 RoPE
// key), bf16 mma.sync m16n8k16 with fp32 accumulation.
//
// Grid (KV splits, head groups x output slices, rows); the splits of one (row, head group, slice)
// form a thread-block cluster and merge their partial outputs through distributed shared memory.
// Per 64-token tile, staged with 16-byte cp.async copies by all threads into padded rows (1168
// bytes: the ldmatrix phases fall on distinct banks; rows past the context are zero-filled) and
// double-buffered (one bulk copy per token row measured 2-4x slower: the small-copy overhead):
//   S = Q L^T        each of the 4 warps 16 tokens x 576 dims (36 k-steps), Q re-read from shared
//   softmax          running max / sum per head in shared memory (4-warp exchange)
//   O += P L[:, :512] each warp its quarter of the CTA's output slice (P from shared memory,
//                    the latent rows as the B operand through ldmatrix.trans)
// A CTA owns 512 / DS output dims (DS = 1, 2 or 4 slices; S is recomputed per slice) so that
// tensor-parallel shards with few heads still cover the GPU.
//
// Parity: crates/hawking-core/src/attn.rs:185 (mla_decode_step), crates/hawking-core/shaders/
// attn.metal:18-47 (absorbed MLA decode); same math as mla_decode_kernel (mla.cu) up to the bf16
// rounding of the scaled query and of P.
#include <cooperative_groups.h>

#include "api.h"
#include "common.cuh"

namespace cg = cooperative_groups;

namespace hk {
namespace {

constexpr int kFH = 16;     // heads per CTA (MMA M)
constexpr int kFT = 64;     // tokens per tile
constexpr int kRowE = 584;  // padded latent / query row, elements (1168 bytes)
constexpr int kPE = 72;     // padded P row, elements (144 bytes)
constexpr int kLat = 512, kRow = 576;

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ uint32_t bf2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int DS>
struct FLayout {
  static constexpr int OD = kLat / DS;
  static constexpr uint32_t off_q = 0;
  static constexpr uint32_t off_l = off_q + kFH * kRowE * 2;
  static constexpr uint32_t off_p = off_l + 2 * kFT * kRowE * 2;
  static constexpr uint32_t off_red = off_p + kFH * kPE * 2;          // [4][16] fp32
  static constexpr uint32_t off_m = off_red + 64 * 4;                // running max [16]
  static constexpr uint32_t off_s = off_m + 16 * 4;                  // running sum [16]
  static constexpr uint32_t off_a = off_s + 16 * 4;                  // this tile's rescale [16]
  static constexpr uint32_t off_o = off_a + 16 * 4;                  // partial O [16][OD]
  static constexpr uint32_t off_rows = off_o + kFH * OD * 4;         // [2][64] cache row of each tile token
  static constexpr uint32_t total = off_rows + 2 * kFT * 8;
  static_assert(total <= 232448, "mla flash: shared memory over the per-CTA limit");
};

template <int DS>
__global__ void __launch_bounds__(128) mla_flash_kernel(MlaDecodeArgs a) {
  using L = FLayout<DS>;
  constexpr int OD = L::OD, WD = OD / 4, NT = WD / 8;
  extern __shared__ __align__(128) uint8_t sm[];
  __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(sm + L::off_q);
  __nv_bfloat16* lt = reinterpret_cast<__nv_bfloat16*>(sm + L::off_l);
  __nv_bfloat16* ps = reinterpret_cast<__nv_bfloat16*>(sm + L::off_p);
  float* red = reinterpret_cast<float*>(sm + L::off_red);
  float* ms = reinterpret_cast<float*>(sm + L::off_m);
  float* ls = reinterpret_cast<float*>(sm + L::off_s);
  float* al = reinterpret_cast<float*>(sm + L::off_a);
  float* os = reinterpret_cast<float*>(sm + L::off_o);
  int64_t* rows_s = reinterpret_cast<int64_t*>(sm + L::off_rows);

  cg::cluster_group cluster = cg::this_cluster();
  const int S = (int)cluster.num_blocks(), split = (int)cluster.block_rank();
  const int hg = blockIdx.y / DS, ds = blockIdx.y % DS, r = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid < 16) {
    ms[tid] = -INFINITY;
    ls[tid] = 0.f;
  }
  __syncthreads();
  pdl_wait();

  const int bs = a.block_size;
  const int ctx = a.row_ctx[r];
  const int* btab = a.block_tables + (int64_t)a.row_seq[r] * a.max_blocks;
  const int tiles_all = (ctx + kFT - 1) / kFT, tps = (tiles_all + S - 1) / S;
  const int t0 = split * tps * kFT, t1 = min(ctx, t0 + tps * kFT);
  const int ntile = t1 > t0 ? (t1 - t0 + kFT - 1) / kFT : 0;

  // the cache rows of tile i's tokens (-1 past the context), one thread per token
  auto rows_of = [&](int i, int b) {
    const int tb = t0 + i * kFT, nv = min(kFT, t1 - tb);
    if (tid < kFT) {
      const int t = tb + tid;
      rows_s[b * kFT + tid] = tid < nv ? (int64_t)btab[t / bs] * bs + t % bs : -1;
    }
  };
  // every thread stages 16-byte chunks of tile i into buffer b (one cp.async group per tile);
  // rows past the context are zero-filled
  auto issue = [&](int b) {
    const uint32_t base = su32(lt + (int64_t)b * kFT * kRowE);
#pragma unroll 4
    for (int idx = tid; idx < kFT * (kRow / 8); idx += blockDim.x) {
      const int j = idx / (kRow / 8), c = idx % (kRow / 8);
      const int64_t row = rows_s[b * kFT + j];
      cp16(base + (uint32_t)((j * kRowE + c * 8) * 2), row >= 0 ? a.cache + row * kRow + c * 8 : a.cache, row >= 0);
    }
    cp_commit();
  };
  if (ntile > 0) rows_of(0, 0);
  if (ntile > 1) rows_of(1, 1);
  __syncthreads();
  if (ntile > 0) issue(0);
  if (ntile > 1) issue(1);
  // scaled query of the head group, bf16 (padding heads are zero): float4 loads, all in flight
  {
    constexpr int C4 = kRow / 4;  // float4 chunks per head (128 latent + 16 rope)
#pragma unroll 6
    for (int idx = tid; idx < kFH * C4; idx += blockDim.x) {
      const int h = idx / C4, c = idx % C4, head = hg * kFH + h;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (head < a.nh)
        v = c < kLat / 4 ? reinterpret_cast<const float4*>(a.q_lat + ((int64_t)r * a.nh + head) * kLat)[c]
                         : reinterpret_cast<const float4*>(a.q_pe + ((int64_t)r * a.nh + head) * (kRow - kLat))[c - kLat / 4];
      uint2 pk;
      pk.x = bf2(v.x * a.scale, v.y * a.scale);
      pk.y = bf2(v.z * a.scale, v.w * a.scale);
      *reinterpret_cast<uint2*>(qs + h * kRowE + c * 4) = pk;
    }
  }
  __syncthreads();

  const int mi = lane >> 3;
  const int h0 = lane >> 2, h1 = h0 + 8;
  const uint32_t q_base = su32(qs), p_base = su32(ps);
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  for (int it = 0; it < ntile; ++it) {
    const int b = it & 1;
    if (it + 1 < ntile) cp_wait<1>();
    else cp_wait<0>();
    __syncthreads();  // tile `it` landed for every thread's copies
    const int tb = t0 + it * kFT, nv = min(kFT, t1 - tb);
    __nv_bfloat16* tile = lt + (int64_t)b * kFT * kRowE;
    const uint32_t l_base = su32(tile);
    // ---- S = Q L^T: this warp's 16 tokens ----
    float s[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
    {
#pragma unroll 4
      for (int kk = 0; kk < kRow / 16; ++kk) {
        uint32_t qa[4], b0, b1, b2, b3;
        ldsm4(q_base + (uint32_t)((((mi & 1) * 8 + (lane & 7)) * kRowE + kk * 16 + (mi >> 1) * 8) * 2), qa[0], qa[1],
              qa[2], qa[3]);
        ldsm4(l_base + (uint32_t)(((warp * 16 + (mi >> 1) * 8 + (lane & 7)) * kRowE + kk * 16 + (mi & 1) * 8) * 2),
              b0, b1, b2, b3);
        mma16816(s[0], qa, b0, b1);
        mma16816(s[1], qa, b2, b3);
      }
    }
    // ---- online softmax over the tile's 64 tokens ----
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = warp * 16 + n * 8 + (lane & 3) * 2 + e;
        if (c >= nv) s[n][e] = s[n][2 + e] = -INFINITY;
        mx0 = fmaxf(mx0, s[n][e]);
        mx1 = fmaxf(mx1, s[n][2 + e]);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    if ((lane & 3) == 0) {
      red[warp * 16 + h0] = mx0;
      red[warp * 16 + h1] = mx1;
    }
    __syncthreads();
    if (tid < 16) {
      const float m_t = fmaxf(fmaxf(red[tid], red[16 + tid]), fmaxf(red[32 + tid], red[48 + tid]));
      const float mo = ms[tid], mn = fmaxf(mo, m_t);
      al[tid] = mo == -INFINITY ? 0.f : __expf(mo - mn);
      ms[tid] = mn;
    }
    __syncthreads();
    const float mh0 = ms[h0], mh1 = ms[h1];
    float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const float p0 = s[n][0] == -INFINITY ? 0.f : __expf(s[n][0] - mh0);
      const float p1 = s[n][1] == -INFINITY ? 0.f : __expf(s[n][1] - mh0);
      const float p2 = s[n][2] == -INFINITY ? 0.f : __expf(s[n][2] - mh1);
      const float p3 = s[n][3] == -INFINITY ? 0.f : __expf(s[n][3] - mh1);
      sum0 += p0 + p1;
      sum1 += p2 + p3;
      const int c = warp * 16 + n * 8 + (lane & 3) * 2;
      *reinterpret_cast<uint32_t*>(ps + h0 * kPE + c) = bf2(p0, p1);
      *reinterpret_cast<uint32_t*>(ps + h1 * kPE + c) = bf2(p2, p3);
    }
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
    if ((lane & 3) == 0) {  // the maxima in red were consumed before the last barrier
      red[warp * 16 + h0] = sum0;
      red[warp * 16 + h1] = sum1;
    }
    __syncthreads();
    if (tid < 16) ls[tid] = ls[tid] * al[tid] + red[tid] + red[16 + tid] + red[32 + tid] + red[48 + tid];
    // ---- O = O * alpha + P L[:, slice] ----
    const float a0 = al[h0], a1 = al[h1];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= a0;
      o[n][1] *= a0;
      o[n][2] *= a1;
      o[n][3] *= a1;
    }
    {
      const int dbase = ds * OD + warp * WD;
#pragma unroll
      for (int t = 0; t < kFT / 16; ++t) {
        uint32_t pa[4];
        ldsm4(p_base + (uint32_t)((((mi & 1) * 8 + (lane & 7)) * kPE + t * 16 + (mi >> 1) * 8) * 2), pa[0], pa[1],
              pa[2], pa[3]);
        const int key = t * 16 + (mi & 1) * 8 + (lane & 7);
#pragma unroll
        for (int n2 = 0; n2 < NT / 2; ++n2) {
          uint32_t v0, v1, v2, v3;
          ldsm4t(l_base + (uint32_t)((key * kRowE + dbase + n2 * 16 + (mi >> 1) * 8) * 2), v0, v1, v2, v3);
          mma16816(o[2 * n2], pa, v0, v1);
          mma16816(o[2 * n2 + 1], pa, v2, v3);
        }
      }
    }
    __syncthreads();  // every read of this buffer and of P is done
    if (it + 2 < ntile) {
      rows_of(it + 2, b);
      __syncthreads();
      issue(b);
    }
  }
  // ---- partial O -> shared memory, merge across the cluster's splits ----
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int d = warp * WD + n * 8 + (lane & 3) * 2;
    os[h0 * OD + d] = o[n][0];
    os[h0 * OD + d + 1] = o[n][1];
    os[h1 * OD + d] = o[n][2];
    os[h1 * OD + d + 1] = o[n][3];
  }
  cluster.sync();
  for (int e = split * blockDim.x + tid; e < kFH * OD; e += S * blockDim.x) {
    const int h = e / OD, d = e % OD, head = hg * kFH + h;
    if (head >= a.nh) continue;
    float M = -INFINITY;
    for (int k = 0; k < S; ++k) M = fmaxf(M, *cluster.map_shared_rank(&ms[h], k));
    float Lsum = 0.f, O = 0.f;
    for (int k = 0; k < S; ++k) {
      const float mk = *cluster.map_shared_rank(&ms[h], k);
      if (mk == -INFINITY) continue;
      const float f = __expf(mk - M);
      Lsum += *cluster.map_shared_rank(&ls[h], k) * f;
      O += *cluster.map_shared_rank(&os[h * OD + d], k) * f;
    }
    a.o_lat[((int64_t)r * a.nh + head) * kLat + ds * OD + d] = Lsum > 0.f ? O / Lsum : 0.f;
  }
  cluster.sync();  // no CTA leaves while a peer still reads its shared memory
  pdl_launch();
}

template <int DS>
void flash_go(const MlaDecodeArgs& a, int S, cudaStream_t s, bool pdl) {
  using L = FLayout<DS>;
  auto kern = mla_flash_kernel<DS>;
  static bool configured = false;  // per instantiation; one device per process
  if (!configured) {
    HK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::total));
    configured = true;
  }
  const int ng = (a.nh + kFH - 1) / kFH;
  launch_cluster(kern, dim3(S, ng * DS, a.R), dim3(128), L::total, s, pdl, S, a);
}

}  // namespace

void mla_flash_decode_launch(const MlaDecodeArgs& a, cudaStream_t s, bool pdl) {
  // splits (cluster size <= 8) first, then output slices, until the launch covers the SMs
  const int ng = (a.nh + kFH - 1) / kFH;
  const int max_tiles = (a.max_blocks * a.block_size + kFT - 1) / kFT;
  int S = 1, DS = 1;
  while (S < 8 && S * 2 <= max_tiles && a.R * ng * S * DS < 128) S *= 2;
  while (DS < 4 && a.R * ng * S * DS < 128) DS *= 2;
  if (DS == 1) flash_go<1>(a, S, s, pdl);
  else if (DS == 2) flash_go<2>(a, S, s, pdl);
  else flash_go<4>(a, S, s, pdl);
}

}  // namespace hk
