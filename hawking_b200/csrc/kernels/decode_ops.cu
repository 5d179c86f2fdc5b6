// Decode-path elementwise kernels: RMSNorm(+q8), RoPE + paged-KV append, argmax, sampling and
// embedding lookup.
//
// Parity: crates/hawking-core/shaders/common.metal (rmsnorm, add_rmsnorm_fused_q8, rope variants,
// kv append, embed lookup), crates/hawking-core/shaders/sample.metal (argmax, temperature,
// repetition penalty, top-k, top-p, multinomial); CPU oracles crates/hawking-core/src/kernels/mod.rs:8-342
// and crates/hawking-core/src/sample.rs:39-98.
#include "decode_ops.cuh"

namespace hk {

// ---- RMSNorm + q8 --------------------------------------------------------------------------
// Grid (K / 256, rows): every CTA reads the whole row (16-byte loads, all issued before the
// reduction) to get the sum of squares, then quantises its own 256 elements (8 warps x one
// 32-element block). One round trip to memory instead of a serial loop in a single CTA.
constexpr int kNormSlice = 256;
__global__ void __launch_bounds__(256) rmsnorm_q8_kernel(const float* x, int64_t x_stride, const float* w, float eps,
                                                          int norm, int K, int8_t* xq, float* xd, float* xs,
                                                          float* y) {
  __shared__ float red[32];
  pdl_wait();
  const int r = blockIdx.y;
  const float* xr = x + (int64_t)r * x_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int i = blockIdx.x * kNormSlice + tid;
  const float xv = i < K ? xr[i] : 0.f;
  float scale = 1.f;
  if (norm) {
    float ss = 0.f;
    constexpr int kV = 8;  // float4 loads per thread in flight (K <= 8192 in one pass)
    float4 v[kV];
#pragma unroll
    for (int j = 0; j < kV; ++j) {
      const int e = (tid + j * 256) * 4;
      v[j] = e < K ? *reinterpret_cast<const float4*>(xr + e) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < kV; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    for (int e = (tid + kV * 256) * 4; e < K; e += 1024) {
      const float4 t = *reinterpret_cast<const float4*>(xr + e);
      ss += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
    }
    ss = block_sum(ss, red);
    scale = rsqrtf(ss / K + eps);
  }
  pdl_launch();
  if (i < K) {  // whole warps (K % 32 == 0)
    float v = xv * scale;
    if (w) v *= w[i];
    if (y) y[(int64_t)r * K + i] = v;
    const float amax = warp_max(fabsf(v));
    const float d = amax / 127.f;
    const int q = amax > 0.f ? __float2int_rn(v / d) : 0;
    const float qsum = warp_sum((float)q);
    xq[(int64_t)r * K + i] = (int8_t)q;
    if (lane == 0) {
      xd[(int64_t)r * (K / 32) + (i >> 5)] = d;
      xs[(int64_t)r * (K / 32) + (i >> 5)] = d * qsum;
    }
  }
  (void)warp;
}

void rmsnorm_q8_launch(const float* x, int64_t x_stride, const float* w, float eps, bool norm, int rows, int K,
                       int8_t* xq, float* xd, float* xs, float* y, cudaStream_t s, bool pdl) {
  if (K % 32) throw std::runtime_error("rmsnorm_q8: K must be a multiple of 32");
  if (norm && (K % 4 || x_stride % 4)) throw std::runtime_error("rmsnorm_q8: rows must be 16-byte aligned");
  launch(rmsnorm_q8_kernel, dim3((K + kNormSlice - 1) / kNormSlice, rows), dim3(256), 0, s, pdl, x, x_stride, w, eps,
         (int)norm, K, xq, xd, xs, y);
}

__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* x, int64_t x_stride, const float* w, float eps,
                                                       int K, float* yf, __nv_bfloat16* yb, int64_t y_stride) {
  __shared__ float red[32];
  pdl_wait();
  const int r = blockIdx.x;
  const float* xr = x + (int64_t)r * x_stride;
  float ss = 0.f;
  for (int i = threadIdx.x; i < K; i += blockDim.x) ss += xr[i] * xr[i];
  ss = block_sum(ss, red);
  const float scale = rsqrtf(ss / K + eps);
  pdl_launch();
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    float v = xr[i] * scale * (w ? w[i] : 1.f);
    if (yf) yf[(int64_t)r * y_stride + i] = v;
    if (yb) yb[(int64_t)r * y_stride + i] = __float2bfloat16(v);
  }
}

// Prefill-sized RMSNorm -> bf16: one CTA per row, every element loaded once as float4 into
// registers (EPT4 vectors per thread), one block reduction, 8-byte bf16x4 stores.
template <int EPT4>
__global__ void __launch_bounds__(256) rmsnorm_bf16_vec_kernel(const float* x, int64_t x_stride, const float* w,
                                                                float eps, int K, __nv_bfloat16* yb, int64_t y_stride) {
  __shared__ float red[32];
  pdl_wait();
  const int r = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + (int64_t)r * x_stride);
  float4 v[EPT4];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < EPT4; ++j) {
    v[j] = xr[threadIdx.x + j * 256];
    ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  }
  ss = block_sum(ss, red);
  const float scale = rsqrtf(ss / K + eps);
  pdl_launch();
#pragma unroll
  for (int j = 0; j < EPT4; ++j) {
    const int i4 = threadIdx.x + j * 256;
    float4 wv = make_float4(1.f, 1.f, 1.f, 1.f);
    if (w) wv = reinterpret_cast<const float4*>(w)[i4];
    const __nv_bfloat162 lo = __floats2bfloat162_rn(v[j].x * scale * wv.x, v[j].y * scale * wv.y);
    const __nv_bfloat162 hi = __floats2bfloat162_rn(v[j].z * scale * wv.z, v[j].w * scale * wv.w);
    uint2 pk;
    pk.x = *reinterpret_cast<const uint32_t*>(&lo);
    pk.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(yb + (int64_t)r * y_stride + 4 * i4) = pk;
  }
}

void rmsnorm_launch(const float* x, int64_t x_stride, const float* w, float eps, int rows, int K, float* y_f32,
                    __nv_bfloat16* y_bf16, int64_t y_stride, cudaStream_t s, bool pdl) {
  const bool vec = !y_f32 && y_bf16 && K % 1024 == 0 && K <= 8192 && x_stride % 4 == 0 && y_stride % 4 == 0 &&
                   reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y_bf16) % 8 == 0 &&
                   reinterpret_cast<uintptr_t>(w) % 16 == 0;
  if (vec) {
    switch (K / 1024) {
      case 1: launch(rmsnorm_bf16_vec_kernel<1>, dim3(rows), dim3(256), 0, s, pdl, x, x_stride, w, eps, K, y_bf16, y_stride); return;
      case 2: launch(rmsnorm_bf16_vec_kernel<2>, dim3(rows), dim3(256), 0, s, pdl, x, x_stride, w, eps, K, y_bf16, y_stride); return;
      case 4: launch(rmsnorm_bf16_vec_kernel<4>, dim3(rows), dim3(256), 0, s, pdl, x, x_stride, w, eps, K, y_bf16, y_stride); return;
      case 8: launch(rmsnorm_bf16_vec_kernel<8>, dim3(rows), dim3(256), 0, s, pdl, x, x_stride, w, eps, K, y_bf16, y_stride); return;
      default: break;
    }
  }
  launch(rmsnorm_kernel, dim3(rows), dim3(256), 0, s, pdl, x, x_stride, w, eps, K, y_f32, y_bf16, y_stride);
}

// ---- RoPE + paged KV append -----------------------------------------------------------------
// Cache slot of row r (-1: skip the append): the given slot, or block_tables[row_seq[r]] at the
// position's block; a position past the row's table or a block outside the caches is skipped
// rather than written out of bounds.
__device__ __forceinline__ int64_t append_slot(const RopeAppendArgs& a, int r, int pos) {
  const int64_t limit = a.cache_blocks * a.block_size;
  if (a.slots) {
    const int64_t s = a.slots[r];
    return s >= 0 && s < limit ? s : -1;
  }
  if (!a.block_tables || pos < 0 || pos / a.block_size >= a.max_blocks) return -1;
  const int blk = a.block_tables[(int64_t)a.row_seq[r] * a.max_blocks + pos / a.block_size];
  return blk >= 0 && blk < a.cache_blocks ? (int64_t)blk * a.block_size + pos % a.block_size : -1;
}

// Grid (head groups, rows); one warp per head (q heads, then k heads, then v heads), so every
// head is a single round trip.
__global__ void __launch_bounds__(256) rope_append_kernel(RopeAppendArgs a) {
  pdl_wait();
  const int r = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int pos = a.positions[r];
  const int64_t slot = append_slot(a, r, pos);
  const int hd = a.hd, half = a.rot_dim / 2;
  const float* rope = a.rope + (int64_t)pos * half * 2;
  const int nheads = a.nh + 2 * a.nkv;
  for (int h = blockIdx.x * nw + warp; h < nheads; h += gridDim.x * nw) {
    const int kind = h < a.nh ? 0 : (h < a.nh + a.nkv ? 1 : 2);  // q, k, v
    const float* src = a.qkv + (int64_t)r * a.qkv_stride + (int64_t)h * hd;
    const float* bias = a.bias ? a.bias + (int64_t)h * hd : nullptr;
    float vals[8];  // hd <= 256
    const int per = hd / 32;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < per) vals[i] = src[lane * per + i] + (bias ? bias[lane * per + i] : 0.f);
    const float* nw_ = kind == 0 ? a.q_norm : (kind == 1 ? a.k_norm : nullptr);
    if (nw_) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < per) ss += vals[i] * vals[i];
      ss = warp_sum(ss);
      const float sc = rsqrtf(ss / hd + a.eps);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < per) vals[i] *= sc * nw_[lane * per + i];
    }
    // Stage through shared memory so each lane can rotate any pair.
    __shared__ float buf[8][256];
    float* hb = buf[warp];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < per) hb[lane * per + i] = vals[i];
    __syncwarp();
    if (kind < 2) {
      for (int p = lane; p < half; p += 32) {
        const int ia = a.rope_style == 0 ? 2 * p : p;
        const int ib = a.rope_style == 0 ? 2 * p + 1 : p + half;
        const float c = rope[2 * p], sn = rope[2 * p + 1];
        const float x0 = hb[ia], x1 = hb[ib];
        hb[ia] = x0 * c - x1 * sn;
        hb[ib] = x0 * sn + x1 * c;
      }
    }
    __syncwarp();
    if (kind == 0) {
      float* dst = a.q_out + ((int64_t)r * a.nh + h) * hd;
      for (int i = lane; i < hd; i += 32) dst[i] = hb[i];
    } else if (slot >= 0) {
      const int kh = kind == 1 ? h - a.nh : h - a.nh - a.nkv;
      const int64_t blk = slot / a.block_size, off = slot % a.block_size;
      __nv_bfloat16* cache = kind == 1 ? a.k_cache : a.v_cache;
      __nv_bfloat16* dst = cache + ((blk * a.nkv + kh) * a.block_size + off) * hd;
      for (int i = lane; i < hd; i += 32) dst[i] = __float2bfloat16(hb[i]);
    }
    __syncwarp();
  }
  pdl_launch();
}

// Head dim 128 with full-width rotation: every lane holds 4 consecutive elements of its head as
// one float4 (loaded once, stored once), adjacent-pair rotation stays inside the lane and the neox
// halves swap with the lane 16 apart; no shared-memory staging.
__global__ void __launch_bounds__(256) rope_append_hd128_kernel(RopeAppendArgs a) {
  pdl_wait();
  const int r = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int pos = a.positions[r];
  const int64_t slot = append_slot(a, r, pos);
  const float* rope = a.rope + (int64_t)pos * 128;  // 64 (cos, sin) pairs
  const int nheads = a.nh + 2 * a.nkv;
  for (int h = blockIdx.x * nw + warp; h < nheads; h += gridDim.x * nw) {
    const int kind = h < a.nh ? 0 : (h < a.nh + a.nkv ? 1 : 2);  // q, k, v
    float4 v = reinterpret_cast<const float4*>(a.qkv + (int64_t)r * a.qkv_stride + (int64_t)h * 128)[lane];
    if (a.bias) {
      const float4 b = reinterpret_cast<const float4*>(a.bias + (int64_t)h * 128)[lane];
      v.x += b.x; v.y += b.y; v.z += b.z; v.w += b.w;
    }
    const float* nw_ = kind == 0 ? a.q_norm : (kind == 1 ? a.k_norm : nullptr);
    if (nw_) {
      const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
      const float sc = rsqrtf(ss / 128.f + a.eps);
      const float4 w = reinterpret_cast<const float4*>(nw_)[lane];
      v.x *= sc * w.x; v.y *= sc * w.y; v.z *= sc * w.z; v.w *= sc * w.w;
    }
    if (kind < 2) {
      if (a.rope_style == 0) {  // pairs (4l, 4l+1), (4l+2, 4l+3): rotation indices 2l, 2l+1
        const float4 cs = reinterpret_cast<const float4*>(rope)[lane];
        const float x0 = v.x, x1 = v.y, x2 = v.z, x3 = v.w;
        v.x = x0 * cs.x - x1 * cs.y;
        v.y = x0 * cs.y + x1 * cs.x;
        v.z = x2 * cs.z - x3 * cs.w;
        v.w = x2 * cs.w + x3 * cs.z;
      } else {  // neox: element e < 64 pairs with e + 64 (lane ^ 16); rotation index e mod 64
        float4 o;
        o.x = __shfl_xor_sync(0xffffffffu, v.x, 16);
        o.y = __shfl_xor_sync(0xffffffffu, v.y, 16);
        o.z = __shfl_xor_sync(0xffffffffu, v.z, 16);
        o.w = __shfl_xor_sync(0xffffffffu, v.w, 16);
        const int p0 = (lane & 15) * 4;
        const float4 c01 = reinterpret_cast<const float4*>(rope + 2 * p0)[0];  // c0 s0 c1 s1
        const float4 c23 = reinterpret_cast<const float4*>(rope + 2 * p0)[1];  // c2 s2 c3 s3
        if (lane < 16) {  // first half: x0 = mine, x1 = partner
          v.x = v.x * c01.x - o.x * c01.y;
          v.y = v.y * c01.z - o.y * c01.w;
          v.z = v.z * c23.x - o.z * c23.y;
          v.w = v.w * c23.z - o.w * c23.w;
        } else {          // second half: x0 = partner, x1 = mine
          v.x = o.x * c01.y + v.x * c01.x;
          v.y = o.y * c01.w + v.y * c01.z;
          v.z = o.z * c23.y + v.z * c23.x;
          v.w = o.w * c23.w + v.w * c23.z;
        }
      }
    }
    if (kind == 0) {
      reinterpret_cast<float4*>(a.q_out + ((int64_t)r * a.nh + h) * 128)[lane] = v;
    } else if (slot >= 0) {
      const int kh = kind == 1 ? h - a.nh : h - a.nh - a.nkv;
      const int64_t blk = slot / a.block_size, off = slot % a.block_size;
      __nv_bfloat16* cache = kind == 1 ? a.k_cache : a.v_cache;
      const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
      uint2 pk;
      pk.x = *reinterpret_cast<const uint32_t*>(&lo);
      pk.y = *reinterpret_cast<const uint32_t*>(&hi);
      reinterpret_cast<uint2*>(cache + ((blk * a.nkv + kh) * a.block_size + off) * 128)[lane] = pk;
    }
  }
  pdl_launch();
}

void rope_append_launch(const RopeAppendArgs& a, cudaStream_t s, bool pdl) {
  if (a.hd % 32 || a.hd > 256) throw std::runtime_error("rope_append: head_dim must be a multiple of 32, <= 256");
  const int heads = a.nh + 2 * a.nkv;
  const bool fast = a.hd == 128 && a.rot_dim == 128 && a.qkv_stride % 4 == 0 &&
                    reinterpret_cast<uintptr_t>(a.qkv) % 16 == 0 && reinterpret_cast<uintptr_t>(a.bias) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(a.q_norm) % 16 == 0 && reinterpret_cast<uintptr_t>(a.k_norm) % 16 == 0;
  if (fast) launch(rope_append_hd128_kernel, dim3((heads + 7) / 8, a.R), dim3(256), 0, s, pdl, a);
  else launch(rope_append_kernel, dim3((heads + 7) / 8, a.R), dim3(256), 0, s, pdl, a);
}

// ---- SwiGLU over a fused gate|up GEMM output ---------------------------------------------------
__global__ void __launch_bounds__(256) swiglu_bf16_kernel(float* gu, int64_t gs, int F, __nv_bfloat16* h,
                                                           int64_t hs, int clear) {
  pdl_wait();
  const int m = blockIdx.y;
  float* g = gu + (int64_t)m * gs;
  for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < F; f += gridDim.x * blockDim.x) {
    const float gv = g[f], uv = g[F + f];
    h[(int64_t)m * hs + f] = __float2bfloat16(gv / (1.f + __expf(-gv)) * uv);
    if (clear) { g[f] = 0.f; g[F + f] = 0.f; }
  }
  pdl_launch();
}

// Four columns per thread (16-byte loads of g and u, one 8-byte store of h): the prefill-sized
// SwiGLU (2048 rows x 14336) streams 294 MB, which the one-column kernel above moved at about a
// third of the HBM rate.
__global__ void __launch_bounds__(256) swiglu_bf16_v4_kernel(float* gu, int64_t gs, int F, __nv_bfloat16* h,
                                                              int64_t hs, int clear) {
  pdl_wait();
  const int m = blockIdx.y;
  float4* g = reinterpret_cast<float4*>(gu + (int64_t)m * gs);
  float4* u = reinterpret_cast<float4*>(gu + (int64_t)m * gs + F);
  uint2* out = reinterpret_cast<uint2*>(h + (int64_t)m * hs);
  for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < F / 4; f += gridDim.x * blockDim.x) {
    const float4 gv = g[f], uv = u[f];
    const float a0 = gv.x / (1.f + __expf(-gv.x)) * uv.x, a1 = gv.y / (1.f + __expf(-gv.y)) * uv.y;
    const float a2 = gv.z / (1.f + __expf(-gv.z)) * uv.z, a3 = gv.w / (1.f + __expf(-gv.w)) * uv.w;
    const __nv_bfloat162 p0 = __floats2bfloat162_rn(a0, a1), p1 = __floats2bfloat162_rn(a2, a3);
    out[f] = make_uint2(*reinterpret_cast<const uint32_t*>(&p0), *reinterpret_cast<const uint32_t*>(&p1));
    if (clear) {
      g[f] = make_float4(0.f, 0.f, 0.f, 0.f);
      u[f] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  pdl_launch();
}

void swiglu_bf16_launch(float* gu, int64_t gu_stride, int M, int F, __nv_bfloat16* h, int64_t h_stride, bool clear,
                        cudaStream_t s, bool pdl) {
  if (M <= 0) return;
  const bool v4 = F % 4 == 0 && gu_stride % 4 == 0 && h_stride % 4 == 0 &&
                  ((reinterpret_cast<uintptr_t>(gu) & 15) | (reinterpret_cast<uintptr_t>(h) & 7)) == 0;
  if (v4) {
    dim3 grid(std::min(64, (F / 4 + 255) / 256), M);
    launch(swiglu_bf16_v4_kernel, grid, dim3(256), 0, s, pdl, gu, gu_stride, F, h, h_stride, (int)clear);
    return;
  }
  dim3 grid(std::min(64, (F + 255) / 256), M);
  launch(swiglu_bf16_kernel, grid, dim3(256), 0, s, pdl, gu, gu_stride, F, h, h_stride, (int)clear);
}

// ---- step advance ----------------------------------------------------------------------------
__global__ void advance_kernel(int* ids, const int* next_ids, int* positions, int* row_ctx, int R) {
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < R) {
    ids[r] = next_ids[r];
    positions[r] += 1;
    row_ctx[r] += 1;
  }
}

void advance_launch(int* ids, const int* next_ids, int* positions, int* row_ctx, int R, cudaStream_t s, bool pdl) {
  launch(advance_kernel, dim3((R + 127) / 128), dim3(128), 0, s, pdl, ids, next_ids, positions, row_ctx, R);
}

// ---- argmax -----------------------------------------------------------------------------------
__device__ __forceinline__ void argmax_merge(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}

__global__ void __launch_bounds__(1024) argmax_kernel(const float* logits, int64_t stride, int V, int* out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_wait();
  const float* l = logits + (int64_t)blockIdx.x * stride;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  const bool vec = ((reinterpret_cast<uintptr_t>(l) & 15) == 0);
  const int V4 = vec ? V / 4 : 0;
  // 4 independent 16-byte loads in flight per thread per iteration
  int i = threadIdx.x;
  for (; i + 3 * 1024 < V4; i += 4 * 1024) {
    float4 x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) x[u] = __ldg(reinterpret_cast<const float4*>(l) + i + u * 1024);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int b = 4 * (i + u * 1024);
      argmax_merge(bv, bi, x[u].x, b);
      argmax_merge(bv, bi, x[u].y, b + 1);
      argmax_merge(bv, bi, x[u].z, b + 2);
      argmax_merge(bv, bi, x[u].w, b + 3);
    }
  }
  for (; i < V4; i += 1024) {
    const float4 x = __ldg(reinterpret_cast<const float4*>(l) + i);
    argmax_merge(bv, bi, x.x, 4 * i);
    argmax_merge(bv, bi, x.y, 4 * i + 1);
    argmax_merge(bv, bi, x.z, 4 * i + 2);
    argmax_merge(bv, bi, x.w, 4 * i + 3);
  }
  for (int j = 4 * V4 + threadIdx.x; j < V; j += 1024) argmax_merge(bv, bi, l[j], j);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
    int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_merge(bv, bi, v2, i2);
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) { sv[w] = bv; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    bv = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
      int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      argmax_merge(bv, bi, v2, i2);
    }
    if (lane == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  }
  pdl_launch();
}


void argmax_launch(const float* logits, int64_t stride, int rows, int V, int* out, cudaStream_t s, bool pdl) {
  launch(argmax_kernel, dim3(rows), dim3(1024), 0, s, pdl, logits, stride, V, out);
}

// One CTA per batch column: max over the packed slots, decode the index, clear the slots.
__global__ void __launch_bounds__(256) argmax_finalize_kernel(unsigned long long* slots, int* out) {
  pdl_wait();
  unsigned long long* sl = slots + (int64_t)blockIdx.x * kArgmaxSlots;
  unsigned long long best = 0;
  for (int i = threadIdx.x; i < kArgmaxSlots; i += blockDim.x) {
    const unsigned long long k = sl[i];
    best = k > best ? k : best;
    sl[i] = 0ull;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
    best = k > best ? k : best;
  }
  __shared__ unsigned long long wbest[8];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) wbest[w] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int j = 1; j < (int)(blockDim.x >> 5); ++j) best = wbest[j] > best ? wbest[j] : best;
    best = wbest[0] > best ? wbest[0] : best;
    out[blockIdx.x] = best == 0ull ? 0 : (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
  }
  pdl_launch();
}

void argmax_finalize_launch(unsigned long long* slots, int rows, int* out, cudaStream_t s, bool pdl) {
  launch(argmax_finalize_kernel, dim3(rows), dim3(256), 0, s, pdl, slots, out);
}

// ---- sampling ---------------------------------------------------------------------------------
// Order (as the CPU sampler): repetition penalty -> temperature (<=0: argmax) -> softmax over the
// full vocabulary -> top-k -> top-p -> renormalise -> draw. Candidates are the top min(top_k,
// 1024) logits, selected by a threshold search, then sorted with a bitonic sort in shared memory.
constexpr int kCand = 1024;

__device__ __forceinline__ float penalised(const float* l, int i, const int* recent, int rn, float pen) {
  float v = l[i];
  if (pen != 1.f)
    for (int j = 0; j < rn; ++j)
      if (recent[j] == i) { v = v >= 0.f ? v / pen : v * pen; break; }
  return v;
}

__global__ void __launch_bounds__(1024) sample_kernel(SampleArgs a) {
  __shared__ float red[32];
  __shared__ float cv[kCand];
  __shared__ int ci[kCand];
  __shared__ int ccount;
  __shared__ int hist[256];
  pdl_wait();
  const int r = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  const float* l = a.logits + (int64_t)r * a.stride;
  const int* recent = a.recent ? a.recent + (int64_t)r * a.recent_n : nullptr;
  const int rn = a.recent ? a.recent_n : 0;
  const float pen = a.rep_penalty ? a.rep_penalty[r] : 1.f;
  const float temp = a.temperature[r];
  const int V = a.V;
  // Greedy lane.
  if (temp <= 0.f) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < V; i += nt) argmax_merge(bv, bi, penalised(l, i, recent, rn, pen), i);
    for (int o = 16; o > 0; o >>= 1) {
      float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
      int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      argmax_merge(bv, bi, v2, i2);
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    if ((tid & 31) == 0) { sv[tid >> 5] = bv; si[tid >> 5] = bi; }
    __syncthreads();
    if (tid < 32) {
      bv = tid < (nt >> 5) ? sv[tid] : -INFINITY;
      bi = tid < (nt >> 5) ? si[tid] : 0x7fffffff;
      for (int o = 16; o > 0; o >>= 1) {
        float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
        int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, v2, i2);
      }
      if (tid == 0) a.out[r] = bi;
    }
    return;
  }
  const float inv_t = 1.f / temp;
  // Softmax normaliser over the full vocabulary.
  float m = -INFINITY;
  for (int i = tid; i < V; i += nt) m = fmaxf(m, penalised(l, i, recent, rn, pen) * inv_t);
  m = block_max(m, red);
  float z = 0.f;
  for (int i = tid; i < V; i += nt) z += __expf(penalised(l, i, recent, rn, pen) * inv_t - m);
  z = block_sum(z, red);
  // Candidate threshold: find the 8-bit bucket (of the scaled logit distance from the max)
  // containing the kc-th largest, refined once; then gather everything above it.
  int kc = a.top_k && a.top_k[r] > 0 ? min(a.top_k[r], kCand) : kCand;
  kc = min(kc, V);
  // Threshold search on the distance from the max: a 256-bucket histogram over [0, 64), then one
  // refinement inside the bucket that crosses kc. Tokens with distance below the threshold are the
  // candidates (ties at the boundary beyond kCand are dropped).
  __shared__ int sel_bucket, sel_before;
  float lo = 0.f, hi = 64.f, thr_dist = 64.f;
  for (int pass = 0; pass < 2; ++pass) {
    for (int i = tid; i < 256; i += nt) hist[i] = 0;
    __syncthreads();
    const float bw = (hi - lo) / 256.f;
    for (int i = tid; i < V; i += nt) {
      const float dist = m - penalised(l, i, recent, rn, pen) * inv_t;
      if (dist >= lo && dist < hi) atomicAdd(&hist[min(255, (int)((dist - lo) / bw))], 1);
    }
    __syncthreads();
    if (tid == 0) {
      int acc = 0, b = 0;
      for (; b < 256; ++b) {
        if (acc + hist[b] >= kc) break;
        acc += hist[b];
      }
      sel_bucket = b;
      sel_before = acc;
    }
    __syncthreads();
    const int b = sel_bucket, before = sel_before;
    const int inb = b < 256 ? hist[b] : 0;
    __syncthreads();
    if (b >= 256) { thr_dist = hi; break; }
    thr_dist = lo + (b + 1) * bw;
    if (before + inb == kc) break;
    kc -= before;
    hi = thr_dist;
    lo = lo + b * bw;
  }
  __syncthreads();
  if (tid == 0) ccount = 0;
  __syncthreads();
  for (int i = tid; i < V; i += nt) {
    float x = penalised(l, i, recent, rn, pen) * inv_t;
    if (m - x < thr_dist) {
      int slot = atomicAdd(&ccount, 1);
      if (slot < kCand) { cv[slot] = x; ci[slot] = i; }
    }
  }
  __syncthreads();
  const int nc = min(ccount, kCand);
  for (int i = tid + nc; i < kCand; i += nt) { cv[i] = -INFINITY; ci[i] = 0x7fffffff; }
  __syncthreads();
  // Bitonic sort, descending by value then ascending index.
  for (int k = 2; k <= kCand; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < kCand; i += nt) {
        int p = i ^ j;
        if (p > i) {
          bool desc = (i & k) == 0;
          float vi = cv[i], vp = cv[p];
          int ii = ci[i], ip = ci[p];
          bool i_before_p = (vi > vp) || (vi == vp && ii < ip);
          if (desc != i_before_p) { cv[i] = vp; cv[p] = vi; ci[i] = ip; ci[p] = ii; }
        }
      }
      __syncthreads();
    }
  }
  if (tid == 0) {
    int keep = nc;
    if (a.top_k && a.top_k[r] > 0) keep = min(keep, a.top_k[r]);
    const float tp = a.top_p ? a.top_p[r] : 1.f;
    const float invz = 1.f / z;
    if (tp > 0.f && tp < 1.f) {
      float cum = 0.f;
      for (int k = 0; k < keep; ++k) {
        cum += __expf(cv[k] - m) * invz;
        if (cum >= tp) { keep = k + 1; break; }
      }
    }
    float total = 0.f;
    for (int k = 0; k < keep; ++k) total += __expf(cv[k] - m) * invz;
    const float u = a.uniforms[r] * total;
    float acc = 0.f;
    int pick = keep > 0 ? ci[keep - 1] : 0;
    for (int k = 0; k < keep; ++k) {
      acc += __expf(cv[k] - m) * invz;
      if (u <= acc) { pick = ci[k]; break; }
    }
    a.out[r] = pick;
  }
  pdl_launch();
}

void sample_launch(const SampleArgs& a, cudaStream_t s, bool pdl) {
  launch(sample_kernel, dim3(a.R), dim3(1024), 0, s, pdl, a);
}

// ---- embedding --------------------------------------------------------------------------------
__device__ __forceinline__ float dequant_elem(int fmt, const WPlanes& t, int64_t row, int k) {
  switch (fmt) {
    case 0: return reinterpret_cast<const float*>(t.p0 + row * t.rb0)[k];
    case 1: return __half2float(reinterpret_cast<const __half*>(t.p0 + row * t.rb0)[k]);
    case 30: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(t.p0 + row * t.rb0)[k]);
    case WF_Q8_0: {
      const int8_t q = reinterpret_cast<const int8_t*>(t.p0 + row * t.rb0)[k];
      return __half2float(reinterpret_cast<const __half*>(t.p1 + row * t.rb1)[k >> 5]) * q;
    }
    case WF_Q4_0: {
      const uint8_t b = (t.p0 + row * t.rb0)[(k >> 5) * 16 + (k & 15)];
      const int q = (k & 16) ? (b >> 4) : (b & 0xF);
      return __half2float(reinterpret_cast<const __half*>(t.p1 + row * t.rb1)[k >> 5]) * (q - 8);
    }
    case WF_Q5_0: {
      const uint8_t b = (t.p0 + row * t.rb0)[(k >> 5) * 16 + (k & 15)];
      const uint32_t qh = reinterpret_cast<const uint32_t*>(t.p2 + row * t.rb2)[k >> 5];
      const int j = k & 31;
      const int q = ((j & 16) ? (b >> 4) : (b & 0xF)) | (((qh >> j) & 1) << 4);
      return __half2float(reinterpret_cast<const __half*>(t.p1 + row * t.rb1)[k >> 5]) * (q - 16);
    }
    case WF_Q4_K: {  // planes: quants [N, K/2], headers [N, K/256 * 16]
      const uint8_t* hdr = t.p1 + row * t.rb1 + (int64_t)(k >> 8) * 16;
      const int e = k & 255, j = e >> 5;  // sub-block
      const uint32_t* s = reinterpret_cast<const uint32_t*>(hdr + 4);
      int sc, mn;
      q4k_scale_min(j, s[0], s[1], s[2], sc, mn);
      const uint8_t qb = (t.p0 + row * t.rb0 + (int64_t)(k >> 8) * 128)[(j >> 1) * 32 + (e & 31)];
      const int q = (j & 1) ? (qb >> 4) : (qb & 0xF);
      const float d = __half2float(reinterpret_cast<const __half*>(hdr)[0]);
      const float dmin = __half2float(reinterpret_cast<const __half*>(hdr)[1]);
      return d * sc * q - dmin * mn;
    }
    case WF_Q6_K: {
      const int hb = k >> 7, e = k & 127, g = e >> 5, l = e & 31;
      const uint8_t* ql = t.p0 + row * t.rb0 + (int64_t)hb * 64;
      const uint8_t* qh = t.p1 + row * t.rb1 + (int64_t)hb * 32;
      const int8_t* sc = reinterpret_cast<const int8_t*>(t.p2 + row * t.rb2) + hb * 8;
      const float d = __half2float(reinterpret_cast<const __half*>(t.p3 + row * t.rb3)[k >> 8]);
      const uint8_t lb = ql[l + ((g & 1) ? 32 : 0)];
      const int lo = (g & 2) ? (lb >> 4) : (lb & 0xF);
      const int q = (lo | (((qh[l] >> (2 * g)) & 3) << 4)) - 32;
      return d * sc[2 * g + (l >> 4)] * q;
    }
  }
  return 0.f;
}

__global__ void __launch_bounds__(256) embed_kernel(int fmt, WPlanes t, const int* ids, int H, float* out,
                                                     int64_t out_stride) {
  pdl_wait();
  const int r = blockIdx.x;
  const int64_t row = ids[r];
  for (int k = threadIdx.x; k < H; k += blockDim.x) out[(int64_t)r * out_stride + k] = dequant_elem(fmt, t, row, k);
  pdl_launch();
}

void embed_launch(int fmt, const WPlanes& table, const int* ids, int R, int H, float* out, int64_t out_stride,
                  cudaStream_t s, bool pdl) {
  launch(embed_kernel, dim3(R), dim3(256), 0, s, pdl, fmt, table, ids, H, out, out_stride);
}

}  // namespace hk
