// Gated DeltaNet linear attention, decode (K7), and the gated full-attention output gate.
//
// Per token and DeltaNet layer (key heads kh, value heads vh = kh * r, key dim dk, value dim dv):
//   1. causal depthwise conv (kernel kc, per-sequence state of the last kc - 1 inputs) + SiLU over
//      the q, k, v channels of the fused qkvz projection (per key head: q[dk] k[dk] v[r*dv] z[r*dv]);
//   2. L2-normalise q and k per key head (q also scaled by dk^-1/2) and share them with the key
//      head's r value heads;
//   3. decay = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b) from the ba projection;
//   4. per value head, with state S [dk, dv]: S *= decay; kv = S^T k; delta = (v - kv) * beta;
//      S += k (x) delta; o = S^T q;
//   5. gated RMSNorm: o * rsqrt(mean(o^2) + eps) * w * silu(z), emitted as q8 blocks (32 dims) for
//      the output projection.
// Kernel deltanet_conv: grid (key heads, rows). Kernel deltanet_recurrent: grid (value heads, rows),
// 4 x dv threads; thread (quarter, column j) keeps rows [quarter * dk / 4, ...) of column j of S in
// registers. Rows of one sequence may follow one another in a forward (a prompt chunk, in position
// order): the CTA of a run's first row walks the whole run token by token, with the conv state and
// the recurrent state S carried across tokens (S read once and written once per run); the CTAs of
// the run's other rows return at once.
//
// Parity: crates/hawking-core/shaders/qwen80_device_activations.metal (causal conv update, q/k L2
// + repeat :120-185, ba_to_decay_beta :187-206, gated rmsnorm :208-277, gated_delta_decode
// :281-393), qwen_next.metal; CPU oracle = the token-serial recurrence (models/qwen_next.py).
#include "decode_ops.cuh"

namespace hk {

// ---- 1 + 2: conv + SiLU + L2 ------------------------------------------------------------------
// The run of rows [r0, r1] that shares row r0's state slot, or r1 < r0 when row r0 continues a run.
__device__ __forceinline__ int2 deltanet_run(const int* state_slot, int r0, int rows) {
  if (!state_slot) return make_int2(r0, r0);
  const int slot = state_slot[r0];
  if (r0 > 0 && state_slot[r0 - 1] == slot) return make_int2(r0, r0 - 1);
  int r1 = r0;
  while (r1 + 1 < rows && state_slot[r1 + 1] == slot) ++r1;
  return make_int2(r0, r1);
}

__global__ void __launch_bounds__(256) deltanet_conv_kernel(DeltaConvArgs a) {
  __shared__ float red[2][8];
  pdl_wait();
  const int kh = blockIdx.x, tid = threadIdx.x;
  const int2 run = deltanet_run(a.state_slot, blockIdx.y, gridDim.y);
  const int dk = a.dk, rv = a.r * a.dv;  // value rows per key head
  const int key_elems = a.kh * dk;
  const int ch_total = 2 * key_elems + a.kh * rv;
  const int slot = a.state_slot ? a.state_slot[run.x] : run.x;
  float* cst = a.conv_state + (int64_t)slot * ch_total * (a.kc - 1);
  for (int r = run.x; r <= run.y; ++r) {
  __syncthreads();  // the previous token's reduction scratch is free
  const float* in = a.qkvz + (int64_t)r * a.qkvz_stride + (int64_t)kh * (2 * dk + 2 * rv);
  auto conv = [&](int ch, float cur) {
    float* st = cst + (int64_t)ch * (a.kc - 1);
    const float* w = a.conv_w + (int64_t)ch * a.kc;
    float s = 0.f;
    for (int t = 0; t < a.kc - 1; ++t) s += st[t] * w[t];
    for (int t = 0; t + 1 < a.kc - 1; ++t) st[t] = st[t + 1];
    st[a.kc - 2] = cur;
    s += cur * w[a.kc - 1];
    return s / (1.f + __expf(-s));
  };
  float qv = 0.f, kv = 0.f;
  if (tid < dk) {
    qv = conv(kh * dk + tid, in[tid]);
    kv = conv(key_elems + kh * dk + tid, in[dk + tid]);
  }
  for (int i = tid; i < rv; i += blockDim.x) {
    const int vh = kh * a.r + i / a.dv, d = i % a.dv;
    a.v[(int64_t)r * a.kh * rv + (int64_t)vh * a.dv + d] = conv(2 * key_elems + kh * rv + i, in[2 * dk + i]);
    a.z[(int64_t)r * a.kh * rv + (int64_t)vh * a.dv + d] = in[2 * dk + rv + i];
  }
  float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv);
  if ((tid & 31) == 0) { red[0][tid >> 5] = sq; red[1][tid >> 5] = sk; }
  __syncthreads();
  if (tid < dk) {
    float tq = 0.f, tk = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { tq += red[0][w]; tk += red[1][w]; }
    const float qs = rsqrtf(tq + a.eps) * rsqrtf((float)dk), ks = rsqrtf(tk + a.eps);
    for (int j = 0; j < a.r; ++j) {
      const int vh = kh * a.r + j;
      a.q[((int64_t)r * a.kh * a.r + vh) * dk + tid] = qv * qs;
      a.k[((int64_t)r * a.kh * a.r + vh) * dk + tid] = kv * ks;
    }
  }
  }  // rows of the run
  pdl_launch();
}

// ---- wide forwards (prefill): every row's convolution in parallel ----------------------------
// Input j steps back from row r (j = 0: row r itself): a row of the same run while j <= back (the
// run's rows before r, at most kc - 1 looked at), else the (j - back)-th newest entry of the
// sequence's conv state (entries oldest first). The state is only read here; the rows that end a
// run write their sequence's new state in deltanet_conv_state_kernel afterwards.
struct ConvIn {
  const DeltaConvArgs& a;
  int r, kh, back, ch_total;
  const float* cst;
  __device__ __forceinline__ float at(int ch, int col, int j) const {
    if (j <= back) return a.qkvz[(int64_t)(r - j) * a.qkvz_stride + (int64_t)kh * (2 * a.dk + 2 * a.r * a.dv) + col];
    return cst[(int64_t)ch * (a.kc - 1) + (a.kc - 1) - (j - back)];
  }
};

__device__ __forceinline__ int conv_back(const DeltaConvArgs& a, int r, int slot) {
  int back = 0;
  if (a.state_slot)
    while (back < a.kc - 1 && r - back - 1 >= 0 && a.state_slot[r - back - 1] == slot) ++back;
  return back;
}

__global__ void __launch_bounds__(256) deltanet_conv_wide_kernel(DeltaConvArgs a) {
  __shared__ float red[2][8];
  pdl_wait();
  const int kh = blockIdx.x, r = blockIdx.y, tid = threadIdx.x;
  const int dk = a.dk, rv = a.r * a.dv;
  const int key_elems = a.kh * dk;
  const int ch_total = 2 * key_elems + a.kh * rv;
  const int slot = a.state_slot ? a.state_slot[r] : r;
  const ConvIn in{a, r, kh, conv_back(a, r, slot), ch_total,
                  a.conv_state + (int64_t)slot * ch_total * (a.kc - 1)};
  auto conv = [&](int ch, int col) {
    const float* w = a.conv_w + (int64_t)ch * a.kc;
    float s = 0.f;
    for (int j = 0; j < a.kc; ++j) s += w[a.kc - 1 - j] * in.at(ch, col, j);
    return s / (1.f + __expf(-s));
  };
  const float* row = a.qkvz + (int64_t)r * a.qkvz_stride + (int64_t)kh * (2 * dk + 2 * rv);
  float qv = 0.f, kv = 0.f;
  if (tid < dk) {
    qv = conv(kh * dk + tid, tid);
    kv = conv(key_elems + kh * dk + tid, dk + tid);
  }
  for (int i = tid; i < rv; i += blockDim.x) {
    const int vh = kh * a.r + i / a.dv, d = i % a.dv;
    a.v[(int64_t)r * a.kh * rv + (int64_t)vh * a.dv + d] = conv(2 * key_elems + kh * rv + i, 2 * dk + i);
    a.z[(int64_t)r * a.kh * rv + (int64_t)vh * a.dv + d] = row[2 * dk + rv + i];
  }
  float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv);
  if ((tid & 31) == 0) { red[0][tid >> 5] = sq; red[1][tid >> 5] = sk; }
  __syncthreads();
  if (tid < dk) {
    float tq = 0.f, tk = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { tq += red[0][w]; tk += red[1][w]; }
    const float qs = rsqrtf(tq + a.eps) * rsqrtf((float)dk), ks = rsqrtf(tk + a.eps);
    for (int j = 0; j < a.r; ++j) {
      const int vh = kh * a.r + j;
      a.q[((int64_t)r * a.kh * a.r + vh) * dk + tid] = qv * qs;
      a.k[((int64_t)r * a.kh * a.r + vh) * dk + tid] = kv * ks;
    }
  }
  pdl_launch();
}

// The rows that end a run: the sequence's conv state becomes the run's last kc - 1 inputs (older
// state entries where the run is shorter). Each thread reads its channels' values, then writes.
__global__ void __launch_bounds__(256) deltanet_conv_state_kernel(DeltaConvArgs a, int rows) {
  pdl_wait();
  const int kh = blockIdx.x, r = blockIdx.y, tid = threadIdx.x;
  const int slot = a.state_slot ? a.state_slot[r] : r;
  const bool last = r == rows - 1 || !a.state_slot || a.state_slot[r + 1] != slot;
  if (last) {
    const int dk = a.dk, rv = a.r * a.dv;
    const int key_elems = a.kh * dk;
    const int ch_total = 2 * key_elems + a.kh * rv;
    float* cst = a.conv_state + (int64_t)slot * ch_total * (a.kc - 1);
    const ConvIn in{a, r, kh, conv_back(a, r, slot), ch_total, cst};
    auto update = [&](int ch, int col) {
      float v[8];
      for (int t = 0; t < a.kc - 1; ++t) v[t] = in.at(ch, col, a.kc - 2 - t);
      for (int t = 0; t < a.kc - 1; ++t) cst[(int64_t)ch * (a.kc - 1) + t] = v[t];
    };
    if (tid < dk) {
      update(kh * dk + tid, tid);
      update(key_elems + kh * dk + tid, dk + tid);
    }
    for (int i = tid; i < rv; i += blockDim.x) update(2 * key_elems + kh * rv + i, 2 * dk + i);
  }
  pdl_launch();
}

void deltanet_conv_launch(const DeltaConvArgs& a, int rows, cudaStream_t s, bool pdl) {
  if (a.dk > 256 || a.dk % 32) throw std::runtime_error("deltanet: key head dim must be a multiple of 32, <= 256");
  if (rows > 8 && a.kc <= 9) {  // prefill-sized forwards: every row in parallel, then the states
    launch(deltanet_conv_wide_kernel, dim3(a.kh, rows), dim3(256), 0, s, pdl, a);
    launch(deltanet_conv_state_kernel, dim3(a.kh, rows), dim3(256), 0, s, pdl, a, rows);
    return;
  }
  launch(deltanet_conv_kernel, dim3(a.kh, rows), dim3(256), 0, s, pdl, a);
}

// ---- 3 + 4 + 5: decay/beta, recurrence, gated RMSNorm -> q8 ----------------------------------
template <int DK, int DV>
__global__ void __launch_bounds__(4 * DV) deltanet_recurrent_kernel(DeltaRecArgs a) {
  constexpr int QR = DK / 4;  // rows of S per thread
  __shared__ float sk[DK], sq[DK];
  __shared__ float part[4][DV];
  __shared__ float red[32];
  __shared__ float s_decay, s_beta;
  pdl_wait();
  const int vh = blockIdx.x, tid = threadIdx.x;
  const int2 run = deltanet_run(a.state_slot, blockIdx.y, gridDim.y);
  if (run.y < run.x) { pdl_launch(); return; }  // another CTA walks this row's run
  const int j = tid % DV, qr = tid / DV;
  const int nvh = gridDim.x, kh = vh / a.r;
  const int slot = a.state_slot ? a.state_slot[run.x] : run.x;
  float* S = a.state + ((int64_t)slot * nvh + vh) * DK * DV;
  float s[QR];
#pragma unroll
  for (int i = 0; i < QR; ++i) s[i] = S[(int64_t)(qr * QR + i) * DV + j];
  for (int r = run.x; r <= run.y; ++r) {
  __syncthreads();  // the previous token's shared values are consumed
  for (int i = tid; i < DK; i += blockDim.x) {
    sk[i] = a.k[((int64_t)r * nvh + vh) * DK + i];
    sq[i] = a.q[((int64_t)r * nvh + vh) * DK + i];
  }
  if (tid == 0) {
    const float* ba = a.ba + (int64_t)r * a.ba_stride + (int64_t)kh * 2 * a.r;
    const float b = ba[vh % a.r], av = ba[a.r + vh % a.r];
    const float x = av + a.dt_bias[vh];
    const float sp = fmaxf(x, 0.f) + log1pf(__expf(-fabsf(x)));
    s_decay = __expf(-__expf(a.a_log[vh]) * sp);
    s_beta = 1.f / (1.f + __expf(-b));
  }
  __syncthreads();
  const float decay = s_decay, beta = s_beta;
  float kvp = 0.f;
#pragma unroll
  for (int i = 0; i < QR; ++i) {
    s[i] *= decay;
    kvp += s[i] * sk[qr * QR + i];
  }
  part[qr][j] = kvp;
  __syncthreads();
  const float kv = part[0][j] + part[1][j] + part[2][j] + part[3][j];
  const float delta = (a.v[((int64_t)r * nvh + vh) * DV + j] - kv) * beta;
  float op = 0.f;
#pragma unroll
  for (int i = 0; i < QR; ++i) {
    s[i] += sk[qr * QR + i] * delta;
    op += s[i] * sq[qr * QR + i];
  }
  __syncthreads();
  part[qr][j] = op;
  __syncthreads();
  if (qr == 0) {
    const float o = part[0][j] + part[1][j] + part[2][j] + part[3][j];
    // gated RMSNorm over the head's DV outputs (threads 0..DV-1 = whole warps)
    float ss = warp_sum(o * o);
    if ((j & 31) == 0) red[j >> 5] = ss;
    asm volatile("bar.sync 1, %0;" ::"r"(DV));
    float tot = 0.f;
    for (int w = 0; w < DV / 32; ++w) tot += red[w];
    const float inv = rsqrtf(tot / DV + a.eps);
    const float zv = a.z[((int64_t)r * nvh + vh) * DV + j];
    const float y = o * inv * a.norm_w[j] * (zv / (1.f + __expf(-zv)));
    const int64_t col = (int64_t)vh * DV + j, width = (int64_t)nvh * DV;
    if (a.out) a.out[(int64_t)r * width + col] = y;
    const float amax = warp_max(fabsf(y));
    const float d = amax / 127.f;
    const int qv = amax > 0.f ? __float2int_rn(y / d) : 0;
    const float qsum = warp_sum((float)qv);
    a.oq[(int64_t)r * width + col] = (int8_t)qv;
    if ((j & 31) == 0) {
      a.od[(int64_t)r * (width / 32) + (col >> 5)] = d;
      a.os[(int64_t)r * (width / 32) + (col >> 5)] = d * qsum;
    }
  }
  }  // rows of the run
#pragma unroll
  for (int i = 0; i < QR; ++i) S[(int64_t)(qr * QR + i) * DV + j] = s[i];
  pdl_launch();
}

void deltanet_recurrent_launch(const DeltaRecArgs& a, int n_value_heads, int rows, cudaStream_t s, bool pdl) {
  if (a.dk == 128 && a.dv == 128)
    launch(deltanet_recurrent_kernel<128, 128>, dim3(n_value_heads, rows), dim3(512), 0, s, pdl, a);
  else if (a.dk == 64 && a.dv == 64)
    launch(deltanet_recurrent_kernel<64, 64>, dim3(n_value_heads, rows), dim3(256), 0, s, pdl, a);
  else
    throw std::runtime_error("deltanet: head dims (dk, dv) must be (128, 128) or (64, 64)");
}

// ---- gated attention output: o *= sigmoid(gate), emitted as q8 ---------------------------------
__global__ void __launch_bounds__(256) sigmoid_gate_q8_kernel(const float* o, const float* gate, int64_t gate_stride,
                                                             int W, int8_t* oq, float* od, float* os) {
  pdl_wait();
  const int r = blockIdx.y, i = blockIdx.x * 256 + threadIdx.x, lane = threadIdx.x & 31;
  if (i < W) {
    const float g = gate[(int64_t)r * gate_stride + i];
    const float v = o[(int64_t)r * W + i] / (1.f + __expf(-g));
    const float amax = warp_max(fabsf(v));
    const float d = amax / 127.f;
    const int q = amax > 0.f ? __float2int_rn(v / d) : 0;
    const float qs = warp_sum((float)q);
    oq[(int64_t)r * W + i] = (int8_t)q;
    if (lane == 0) {
      od[(int64_t)r * (W / 32) + (i >> 5)] = d;
      os[(int64_t)r * (W / 32) + (i >> 5)] = d * qs;
    }
  }
  pdl_launch();
}

void sigmoid_gate_q8_launch(const float* o, const float* gate, int64_t gate_stride, int rows, int W, int8_t* oq,
                            float* od, float* os, cudaStream_t s, bool pdl) {
  if (W % 32) throw std::runtime_error("sigmoid gate: width must be a multiple of 32");
  launch(sigmoid_gate_q8_kernel, dim3((W + 255) / 256, rows), dim3(256), 0, s, pdl, o, gate, gate_stride, W, oq, od,
         os);
}

}  // namespace hk
