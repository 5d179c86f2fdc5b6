// GPU quantisers: fp32 rows -> GGUF block formats in the engine's device layout (K-quants as raw
// super-blocks, 32-element formats as planes). Used to materialise random-init weights of the
// benchmark architectures directly on the device; the encoding decisions mirror the CPU
// quantisers in csrc/native/ggml_quant.cpp (same min/max fits, IEEE division, round-to-nearest-
// even), so a row quantised on either side gives the same bytes.
#include "common.cuh"
#include "quantize.cuh"

namespace hk {

__device__ __forceinline__ uint16_t f2h_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ float signed_extreme(const float* x, int n) {
  float amax = 0.f, mx = 0.f;
  for (int j = 0; j < n; ++j)
    if (fabsf(x[j]) > amax) { amax = fabsf(x[j]); mx = x[j]; }
  return mx;
}

// One thread per 256-element super-block.
__global__ void quantize_q4k_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ out) {
  int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* xb = x + b * 256;
  uint8_t* o = out + b * 144;
  float scale[8], mins[8];
  for (int j = 0; j < 8; ++j) {
    float lo = xb[32 * j], hi = lo;
    for (int l = 1; l < 32; ++l) { lo = fminf(lo, xb[32 * j + l]); hi = fmaxf(hi, xb[32 * j + l]); }
    lo = fminf(lo, 0.f);
    scale[j] = (hi - lo) / 15.f;
    mins[j] = -lo;
  }
  float max_s = 0.f, max_m = 0.f;
  for (int j = 0; j < 8; ++j) { max_s = fmaxf(max_s, scale[j]); max_m = fmaxf(max_m, mins[j]); }
  const float d = max_s / 63.f, dmin = max_m / 63.f;
  uint8_t sc[8], mn[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = (uint8_t)min(max(d != 0.f ? __float2int_rn(scale[j] / d) : 0, 0), 63);
    mn[j] = (uint8_t)min(max(dmin != 0.f ? __float2int_rn(mins[j] / dmin) : 0, 0), 63);
  }
  const uint16_t dh = f2h_bits(d), mh = f2h_bits(dmin);
  reinterpret_cast<uint16_t*>(o)[0] = dh;  // 16-bit stores (o is 4-byte aligned: 144-byte blocks)
  reinterpret_cast<uint16_t*>(o)[1] = mh;
  for (int j = 0; j < 4; ++j) {
    o[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    o[8 + j] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
    o[12 + j] = (uint8_t)((sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4));
  }
  const float dq = h2f_bits(dh), mq = h2f_bits(mh);
  for (int c = 0; c < 4; ++c) {
    const float ds0 = dq * sc[2 * c], dm0 = mq * mn[2 * c];
    const float ds1 = dq * sc[2 * c + 1], dm1 = mq * mn[2 * c + 1];
    for (int l = 0; l < 32; ++l) {
      int q0 = ds0 != 0.f ? __float2int_rn((xb[64 * c + l] + dm0) / ds0) : 0;
      int q1 = ds1 != 0.f ? __float2int_rn((xb[64 * c + 32 + l] + dm1) / ds1) : 0;
      q0 = min(max(q0, 0), 15);
      q1 = min(max(q1, 0), 15);
      o[16 + 32 * c + l] = (uint8_t)(q0 | (q1 << 4));
    }
  }
}

// One thread per 32-element block; planes qs [rows, cols] / d [rows, cols/32].
__global__ void quantize_q8_0_kernel(const float* __restrict__ x, int64_t nblocks, int8_t* __restrict__ qs,
                                     __half* __restrict__ dout) {
  int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* xb = x + b * 32;
  float amax = 0.f;
  for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(xb[j]));
  const float d = amax / 127.f, id = d != 0.f ? 1.f / d : 0.f;
  dout[b] = __float2half_rn(d);
  for (int j = 0; j < 32; ++j) qs[b * 32 + j] = (int8_t)min(max(__float2int_rn(xb[j] * id), -127), 127);
}

__global__ void quantize_q4_0_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ qs,
                                     __half* __restrict__ dout) {
  int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* xb = x + b * 32;
  const float mx = signed_extreme(xb, 32);
  const float d = mx / -8.f, id = d != 0.f ? 1.f / d : 0.f;
  dout[b] = __float2half_rn(d);
  for (int j = 0; j < 16; ++j) {
    int a = min(max(__float2int_rn(xb[j] * id) + 8, 0), 15);
    int c = min(max(__float2int_rn(xb[j + 16] * id) + 8, 0), 15);
    qs[b * 16 + j] = (uint8_t)(a | (c << 4));
  }
}

// Q5_0 planes: qs [rows, cols/2], d [rows, cols/32], qh u32 [rows, cols/32].
__global__ void quantize_q5_0_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ qs,
                                     __half* __restrict__ dout, uint32_t* __restrict__ qhp) {
  int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* xb = x + b * 32;
  const float mx = signed_extreme(xb, 32);
  const float d = mx / -16.f, id = d != 0.f ? 1.f / d : 0.f;
  dout[b] = __float2half_rn(d);
  uint32_t qh = 0;
  for (int j = 0; j < 16; ++j) {
    int a = min(max(__float2int_rn(xb[j] * id) + 16, 0), 31);
    int c = min(max(__float2int_rn(xb[j + 16] * id) + 16, 0), 31);
    qs[b * 16 + j] = (uint8_t)((a & 0xF) | ((c & 0xF) << 4));
    qh |= ((uint32_t)(a >> 4) & 1u) << j;
    qh |= ((uint32_t)(c >> 4) & 1u) << (j + 16);
  }
  qhp[b] = qh;
}

// Q6_K planes: ql [rows, cols/2], qh [rows, cols/4], sc [rows, cols/16], d [rows, cols/256].
__global__ void quantize_q6k_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ ql,
                                    uint8_t* __restrict__ qh, int8_t* __restrict__ scp, __half* __restrict__ dp) {
  int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* xb = x + b * 256;
  float sub[16];
  for (int j = 0; j < 16; ++j) sub[j] = signed_extreme(xb + 16 * j, 16) / -32.f;
  float amax = 0.f, mx = 0.f;
  for (int j = 0; j < 16; ++j)
    if (fabsf(sub[j]) > amax) { amax = fabsf(sub[j]); mx = sub[j]; }
  const float d = mx / -128.f;
  const __half dh = __float2half_rn(d);
  dp[b] = dh;
  const float dq = __half2float(dh);
  int8_t* sc = scp + b * 16;
  uint8_t* qlb = ql + b * 128;
  uint8_t* qhb = qh + b * 64;
  for (int n = 0; n < 2; ++n)
    for (int l = 0; l < 32; ++l) {
      int q[4];
      for (int g = 0; g < 4; ++g) {
        const int e = 128 * n + 32 * g + l, j = e / 16;
        const int scj = min(max(dq != 0.f ? __float2int_rn(sub[j] / dq) : 0, -128), 127);
        if (l % 16 == 0) sc[j] = (int8_t)scj;
        const float ds = dq * scj;
        const int v = ds != 0.f ? __float2int_rn(xb[e] / ds) : 0;
        q[g] = min(max(v, -32), 31) + 32;
      }
      qlb[64 * n + l] = (uint8_t)((q[0] & 0xF) | ((q[2] & 0xF) << 4));
      qlb[64 * n + l + 32] = (uint8_t)((q[1] & 0xF) | ((q[3] & 0xF) << 4));
      qhb[32 * n + l] = (uint8_t)((q[0] >> 4) | ((q[1] >> 4) << 2) | ((q[2] >> 4) << 4) | ((q[3] >> 4) << 6));
    }
}

void quantize_launch(int fmt, const float* x, int64_t n, void* p0, void* p1, void* p2, void* p3, cudaStream_t s) {
  const int bs = 128;
  switch (fmt) {
    case WF_Q4_K: {
      int64_t nb = n / 256;
      quantize_q4k_kernel<<<(unsigned)((nb + bs - 1) / bs), bs, 0, s>>>(x, nb, (uint8_t*)p0);
      break;
    }
    case WF_Q8_0: {
      int64_t nb = n / 32;
      quantize_q8_0_kernel<<<(unsigned)((nb + bs - 1) / bs), bs, 0, s>>>(x, nb, (int8_t*)p0, (__half*)p1);
      break;
    }
    case WF_Q4_0: {
      int64_t nb = n / 32;
      quantize_q4_0_kernel<<<(unsigned)((nb + bs - 1) / bs), bs, 0, s>>>(x, nb, (uint8_t*)p0, (__half*)p1);
      break;
    }
    case WF_Q5_0: {
      int64_t nb = n / 32;
      quantize_q5_0_kernel<<<(unsigned)((nb + bs - 1) / bs), bs, 0, s>>>(x, nb, (uint8_t*)p0, (__half*)p1,
                                                                          (uint32_t*)p2);
      break;
    }
    case WF_Q6_K: {
      int64_t nb = n / 256;
      quantize_q6k_kernel<<<(unsigned)((nb + bs - 1) / bs), bs, 0, s>>>(x, nb, (uint8_t*)p0, (uint8_t*)p1,
                                                                         (int8_t*)p2, (__half*)p3);
      break;
    }
    default: throw std::runtime_error("quantize: unsupported format " + std::to_string(fmt));
  }
  HK_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hk
