// Tensor-parallel collectives fused into the decode kernels (K2), over NVLink peer memory.
//
// All-reduce of a row-parallel projection (attention output, FFN down) at decode batch sizes is
// a one-shot push: the projection GEMV's epilogue stores each of its output rows straight into
// every rank's receive region (peer pointers from CUDA IPC) as flagged words (tp.cuh). The next
// kernel on every rank, the RMSNorm that feeds the following projection, polls the words of the
// elements it owns until their flag is this step's epoch (bounded), sums the N partials into the
// new residual (a second buffer, so no CTA reads what another CTA writes), normalises and
// quantises. The CTAs of one row form a cluster that adds up the row's sum of squares through
// distributed shared memory. No separate all-reduce launch, no fence, no counter, no host round
// trip: the partials cross NVLink once, from the producing SMs.
//
// Every rank bumps the epoch at the start of each forward that uses the push sites (the
// tensor-core prefill path all-reduces with NCCL and does not). A rank cannot overwrite a
// receive region that a slower rank has not consumed yet, because its own next write into that
// region needs the slower rank's contribution to an earlier site of the next step.
//
// The sum x_in + p_0 + ... + p_{N-1} runs in the same order on every rank from the same words,
// so the residual stream stays bitwise identical across ranks.
//
// The vocabulary-parallel LM head pushes each rank's packed (logit, global index) maximum the
// same way (two flagged words per key); every rank then reduces the N keys to the token id.
//
// Every wait is bounded (status word HK_ERR_PEER_TIMEOUT, then the kernel carries on with what
// it has; the engine reads the status after the step and discards the step's tokens): a rank that
// stopped cannot hang the others' GPUs. The bound is a kernel argument (default one second).
#include <cooperative_groups.h>

#include "decode_ops.cuh"
#include "tp.cuh"

namespace cg = cooperative_groups;

namespace hk {

__global__ void tp_begin_kernel(int* epoch) {
  pdl_wait();
  if (threadIdx.x == 0) epoch[0] += 1;
  pdl_launch();
}

void tp_begin_launch(int* epoch, cudaStream_t s, bool pdl) { launch(tp_begin_kernel, dim3(1), dim3(32), 0, s, pdl, epoch); }

constexpr int kTpCluster = 8;   // CTAs per row (one cluster)
constexpr int kTpMaxE = 4;      // elements per thread: K <= kTpCluster * 256 * kTpMaxE
constexpr int kTpMaxRanks = 8;

// Consumer: x_out = x_in + sum over ranks of the partials, then RMSNorm (weight w) -> q8 blocks
// (or bf16 rows when xq is null).
// Grid (kTpCluster, rows), clusters of kTpCluster CTAs along x; CTA c owns elements
// [c * K / C, (c + 1) * K / C) of its row, 256 threads striding over them (a warp owns whole
// 32-element q8 blocks).
__global__ void __cluster_dims__(kTpCluster, 1, 1) __launch_bounds__(256)
    tp_allreduce_rmsnorm_q8_kernel(TpReduceArgs a) {
  __shared__ float red[8];
  __shared__ float part_ss;
  pdl_wait();
  cg::cluster_group cluster = cg::this_cluster();
  const int c = (int)cluster.block_rank();
  const int r = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = a.K, chunk = K / kTpCluster, base = c * chunk, n = a.n;
  const uint32_t flag = (uint32_t)*a.epoch;
  const unsigned long long deadline = global_ns() + (a.wait_ns ? a.wait_ns : kTpWaitNs);
  const unsigned long long* rr = a.recv + (int64_t)r * K;
  const float* xr = a.x_in + (int64_t)r * a.x_stride;

  // issue every load first (independent loads in flight), then settle the stragglers
  uint2 w[kTpMaxE][kTpMaxRanks];
  float v[kTpMaxE];
#pragma unroll
  for (int j = 0; j < kTpMaxE; ++j) {
    const bool on = j * 256 + warp * 32 < chunk;
    const int e = base + j * 256 + tid;
    v[j] = on ? xr[e] : 0.f;
#pragma unroll
    for (int p = 0; p < kTpMaxRanks; ++p)
      if (on && p < n) w[j][p] = ll_load(rr + (int64_t)p * a.rank_stride + e);
  }
  bool ok = true;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kTpMaxE; ++j) {
    const bool on = j * 256 + warp * 32 < chunk;
    const int e = base + j * 256 + tid;
#pragma unroll
    for (int p = 0; p < kTpMaxRanks; ++p) {
      if (on && p < n) {
        ll_settle(w[j][p], rr + (int64_t)p * a.rank_stride + e, flag, deadline, ok);
        v[j] += __uint_as_float(w[j][p].x);
      }
    }
    ss += v[j] * v[j];
  }
  if (!ok) set_error(a.status, HK_ERR_PEER_TIMEOUT);
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i];
    part_ss = t;
  }
  cluster.sync();
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < kTpCluster; ++i) total += *cluster.map_shared_rank(&part_ss, i);
  cluster.sync();  // no CTA leaves while another still reads its partial
  const float scale = rsqrtf(total / K + a.eps);
  pdl_launch();
#pragma unroll
  for (int j = 0; j < kTpMaxE; ++j) {
    if (j * 256 + warp * 32 >= chunk) continue;  // warp-uniform
    const int e = base + j * 256 + tid;
    a.x_out[(int64_t)r * a.x_stride + e] = v[j];
    float y = v[j] * scale;
    if (a.w) y *= a.w[e];
    if (!a.xq) {  // bf16 output (uniform across the grid)
      if (a.yb) a.yb[(int64_t)r * a.yb_stride + e] = __float2bfloat16_rn(y);
      continue;
    }
    const float amax = warp_max(fabsf(y));
    const float d = amax / 127.f;
    const int q = amax > 0.f ? __float2int_rn(y / d) : 0;
    const float qsum = warp_sum((float)q);
    a.xq[(int64_t)r * K + e] = (int8_t)q;
    if (lane == 0) {
      a.xd[(int64_t)r * (K / 32) + (e >> 5)] = d;
      a.xs[(int64_t)r * (K / 32) + (e >> 5)] = d * qsum;
    }
  }
}

void tp_allreduce_rmsnorm_q8_launch(const TpReduceArgs& a, int rows, cudaStream_t s, bool pdl) {
  if (a.K % (32 * kTpCluster) || a.K > kTpCluster * 256 * kTpMaxE || a.x_stride % 4)
    throw std::runtime_error("tp all-reduce norm: K must be a multiple of 256 and at most 8192");
  if (a.n < 1 || a.n > kTpMaxRanks) throw std::runtime_error("tp all-reduce norm: 1..8 ranks");
  // the cluster shape is static (__cluster_dims__), so this is a plain launch
  launch(tp_allreduce_rmsnorm_q8_kernel, dim3(kTpCluster, rows), dim3(256), 0, s, pdl, a);
}

// ---- tensor-core path: P2P-read all-reduce + RMSNorm ----------------------------------------------
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid (kTpCluster, rows) as the push consumer. Every CTA's thread 0 raises this rank's flag of the
// site on every rank (the GEMM that wrote the partial completed before this kernel: the dependency
// wait), threads 0..n-1 wait for the n flags, then the CTA reads its elements of the n partials
// (remote ones over NVLink, uncached loads) in rank order.
__global__ void __cluster_dims__(kTpCluster, 1, 1) __launch_bounds__(256)
    tp_p2p_allreduce_rmsnorm_kernel(TpP2PArgs a) {
  __shared__ float red[8];
  __shared__ float part_ss;
  pdl_wait();
  cg::cluster_group cluster = cg::this_cluster();
  const int c = (int)cluster.block_rank();
  const int r = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = a.K, chunk = K / kTpCluster, base = c * chunk, n = a.n;
  const unsigned flag = (unsigned)*a.epoch;
  if (tid == 0) {
    __threadfence_system();
    for (int p = 0; p < n; ++p) st_release_sys(reinterpret_cast<unsigned*>(a.flag_ptrs[p]) + a.me, flag);
  }
  bool ok = true;
  if (tid < n) {
    const unsigned long long deadline = global_ns() + (a.wait_ns ? a.wait_ns : kTpWaitNs);
    while (ld_acquire_sys(a.flags_local + tid) != flag) {
      if (global_ns() > deadline) {
        ok = false;
        break;
      }
    }
  }
  ok = __syncthreads_and(ok);
  if (!ok && tid == 0) set_error(a.status, HK_ERR_PEER_TIMEOUT);
  const float* xr = a.x_in + (int64_t)r * a.x_stride;
  float v[kTpMaxE];
#pragma unroll
  for (int j = 0; j < kTpMaxE; ++j) {
    const bool on = j * 256 + warp * 32 < chunk;
    v[j] = on ? xr[base + j * 256 + tid] : 0.f;
  }
  for (int p = 0; p < n; ++p) {  // fixed rank order: the same sum on every rank
    const float* pr = reinterpret_cast<const float*>(a.parts[p]) + (int64_t)r * K;
    float t[kTpMaxE];
#pragma unroll
    for (int j = 0; j < kTpMaxE; ++j) {
      const bool on = j * 256 + warp * 32 < chunk;
      t[j] = on ? __ldcv(pr + base + j * 256 + tid) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kTpMaxE; ++j) v[j] += t[j];
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kTpMaxE; ++j) ss += v[j] * v[j];
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (tid == 0) {
    float tt = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tt += red[i];
    part_ss = tt;
  }
  cluster.sync();
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < kTpCluster; ++i) total += *cluster.map_shared_rank(&part_ss, i);
  cluster.sync();
  const float scale = rsqrtf(total / K + a.eps);
  pdl_launch();
#pragma unroll
  for (int j = 0; j < kTpMaxE; ++j) {
    if (j * 256 + warp * 32 >= chunk) continue;  // warp-uniform
    const int e = base + j * 256 + tid;
    a.x_out[(int64_t)r * a.x_stride + e] = v[j];
    float y = v[j] * scale;
    if (a.w) y *= a.w[e];
    if (!a.xq) {
      if (a.yb) a.yb[(int64_t)r * a.yb_stride + e] = __float2bfloat16_rn(y);
      continue;
    }
    const float amax = warp_max(fabsf(y));
    const float d = amax / 127.f;
    const int q = amax > 0.f ? __float2int_rn(y / d) : 0;
    const float qsum = warp_sum((float)q);
    a.xq[(int64_t)r * K + e] = (int8_t)q;
    if (lane == 0) {
      a.xd[(int64_t)r * (K / 32) + (e >> 5)] = d;
      a.xs[(int64_t)r * (K / 32) + (e >> 5)] = d * qsum;
    }
  }
}

void tp_p2p_allreduce_rmsnorm_launch(const TpP2PArgs& a, int rows, cudaStream_t s, bool pdl) {
  if (a.K % (32 * kTpCluster) || a.K > kTpCluster * 256 * kTpMaxE || a.x_stride % 4)
    throw std::runtime_error("tp p2p all-reduce norm: K must be a multiple of 256 and at most 8192");
  if (a.n < 1 || a.n > kTpMaxRanks || a.me < 0 || a.me >= a.n) throw std::runtime_error("tp p2p all-reduce norm: 1..8 ranks");
  launch(tp_p2p_allreduce_rmsnorm_kernel, dim3(kTpCluster, rows), dim3(256), 0, s, pdl, a);
}

// Vocabulary-parallel greedy: local best packed key per row (from the fused LM-head slots,
// already holding global indices) -> pushed to every rank -> max of the N keys -> token id.
__global__ void __launch_bounds__(256) tp_argmax_kernel(TpArgmaxArgs a) {
  __shared__ unsigned long long best_s[8];
  __shared__ uint32_t flag_s;
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) flag_s = (uint32_t)(++a.uses[0]);  // this site's own round count (greedy steps only)
  __syncthreads();
  const uint32_t flag = flag_s;
  for (int r = 0; r < a.rows; ++r) {
    unsigned long long* sl = a.slots + (int64_t)r * kArgmaxSlots;
    unsigned long long best = 0;
    for (int i = tid; i < kArgmaxSlots; i += blockDim.x) {
      const unsigned long long k = sl[i];
      best = k > best ? k : best;
      sl[i] = 0ull;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
      best = k > best ? k : best;
    }
    if (lane == 0) best_s[warp] = best;
    __syncthreads();
    if (tid < a.n) {
      unsigned long long b = 0;
      for (int wi = 0; wi < (int)(blockDim.x >> 5); ++wi) b = best_s[wi] > b ? best_s[wi] : b;
      // this rank's key for row r -> rank tid's key region, words [me][r][0..1]
      unsigned long long* dst = a.keys[tid] + ((int64_t)a.me * a.max_rows + r) * 2;
      ll_store(dst, (uint32_t)(b >> 32), flag);
      ll_store(dst + 1, (uint32_t)(b & 0xFFFFFFFFull), flag);
    }
    __syncthreads();
  }
  const unsigned long long deadline = global_ns() + (a.wait_ns ? a.wait_ns : kTpWaitNs);
  bool ok = true;
  for (int r = tid; r < a.rows; r += blockDim.x) {
    unsigned long long b = 0;
    for (int p = 0; p < a.n; ++p) {
      const unsigned long long* src = a.keys_local + ((int64_t)p * a.max_rows + r) * 2;
      uint2 hi = ll_load(src), lo = ll_load(src + 1);
      ll_settle(hi, src, flag, deadline, ok);
      ll_settle(lo, src + 1, flag, deadline, ok);
      const unsigned long long k = ((unsigned long long)hi.x << 32) | lo.x;
      b = k > b ? k : b;
    }
    a.out[r] = b == 0ull ? 0 : (int)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
  }
  if (!ok) set_error(a.status, HK_ERR_PEER_TIMEOUT);
  pdl_launch();
}

void tp_argmax_launch(const TpArgmaxArgs& a, cudaStream_t s, bool pdl) {
  if (a.n > 256) throw std::runtime_error("tp argmax: at most 256 ranks");
  launch(tp_argmax_kernel, dim3(1), dim3(256), 0, s, pdl, a);
}

}  // namespace hk
