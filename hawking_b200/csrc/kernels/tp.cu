// Tensor-parallel collectives fused into the decode kernels (K2), over NVLink peer memory.
//
// All-reduce of a row-parallel projection (attention output, FFN down) at decode batch sizes is
// a one-shot push: the projection GEMV's epilogue stores each of its output rows straight into
// every rank's receive region (peer pointers from CUDA IPC), then each CTA bumps every rank's
// arrival counter once with a system-scope release. The next kernel on every rank, the RMSNorm
// that feeds the following projection, waits (bounded) until all producer CTAs of all ranks have
// arrived, sums the N partial vectors into the new residual (a second buffer, so no CTA reads
// what another CTA writes), normalises and quantises. No separate all-reduce launch, no host
// round trip, no staging copy: the partials cross NVLink once, from the producing SMs.
//
// Arrival counters never reset: every rank bumps an epoch at the start of each forward that uses
// the push sites (the tensor-core prefill path all-reduces with NCCL and does not),
// and a consumer waits for epoch * (producer CTAs) * N arrivals. A rank cannot overwrite a
// receive region that a slower rank has not consumed yet, because its own next write into that
// region needs the slower rank's contribution to an earlier site of the next step.
//
// The vocabulary-parallel LM head pushes each rank's packed (logit, global index) maximum the
// same way; every rank then reduces the N keys to the token id.
//
// Every wait is bounded (status word HK_ERR_PEER_TIMEOUT, then the kernel carries on with what
// it has): a rank that stopped cannot hang the others' GPUs.
#include "decode_ops.cuh"
#include "tp.cuh"

namespace hk {

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait by one thread for counter >= target.
__device__ __forceinline__ bool wait_arrivals(const unsigned long long* counter, unsigned long long target, int* status) {
  for (uint32_t i = 0; i < (1u << 24); ++i) {
    if (ld_acquire_sys_u64(counter) >= target) return true;
    if (i > 64) __nanosleep(64);
  }
  set_error(status, HK_ERR_PEER_TIMEOUT);
  return false;
}

__global__ void tp_begin_kernel(int* epoch) {
  pdl_wait();
  if (threadIdx.x == 0) epoch[0] += 1;
  pdl_launch();
}

void tp_begin_launch(int* epoch, cudaStream_t s, bool pdl) { launch(tp_begin_kernel, dim3(1), dim3(32), 0, s, pdl, epoch); }

// Consumer: x_out = x_in + sum over ranks of the partials, then RMSNorm (weight w) -> q8 blocks.
// Grid (ceil(K / 256), rows); every CTA sums the whole row (for the norm) and writes its slice.
__global__ void __launch_bounds__(256) tp_allreduce_rmsnorm_q8_kernel(TpReduceArgs a) {
  __shared__ float red[32];
  __shared__ int ok_s;
  pdl_wait();
  const int r = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
  if (tid == 0) {
    const unsigned long long target = (unsigned long long)(*a.epoch) * (unsigned long long)a.producer_ctas * a.n;
    ok_s = wait_arrivals(a.counter, target, a.status);
  }
  __syncthreads();
  const int K = a.K;
  const float* xr = a.x_in + (int64_t)r * a.x_stride;
  float ss = 0.f, mine = 0.f;
  const int i_mine = blockIdx.x * 256 + tid;
  for (int e = tid * 4; e < K; e += 1024) {
    float4 v = *reinterpret_cast<const float4*>(xr + e);
    for (int p = 0; p < a.n; ++p) {
      const float4 q = __ldcg(reinterpret_cast<const float4*>(a.recv + (int64_t)p * a.rank_stride + (int64_t)r * K + e));
      v.x += q.x;
      v.y += q.y;
      v.z += q.z;
      v.w += q.w;
    }
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  // this thread's own element of the CTA's slice (same sum, same order)
  if (i_mine < K) {
    float v = xr[i_mine];
    for (int p = 0; p < a.n; ++p) v += __ldcg(a.recv + (int64_t)p * a.rank_stride + (int64_t)r * K + i_mine);
    mine = v;
  }
  ss = block_sum(ss, red);
  const float scale = rsqrtf(ss / K + a.eps);
  pdl_launch();
  if (i_mine < K) {
    a.x_out[(int64_t)r * a.x_stride + i_mine] = mine;
    float v = mine * scale;
    if (a.w) v *= a.w[i_mine];
    const float amax = warp_max(fabsf(v));
    const float d = amax / 127.f;
    const int q = amax > 0.f ? __float2int_rn(v / d) : 0;
    const float qsum = warp_sum((float)q);
    a.xq[(int64_t)r * K + i_mine] = (int8_t)q;
    if (lane == 0) {
      a.xd[(int64_t)r * (K / 32) + (i_mine >> 5)] = d;
      a.xs[(int64_t)r * (K / 32) + (i_mine >> 5)] = d * qsum;
    }
  }
  (void)ok_s;
}

void tp_allreduce_rmsnorm_q8_launch(const TpReduceArgs& a, int rows, cudaStream_t s, bool pdl) {
  if (a.K % 256 || a.x_stride % 4) throw std::runtime_error("tp all-reduce norm: K must be a multiple of 256");
  launch(tp_allreduce_rmsnorm_q8_kernel, dim3(a.K / 256, rows), dim3(256), 0, s, pdl, a);
}

// Vocabulary-parallel greedy: local best packed key per row (from the fused LM-head slots,
// already holding global indices) -> pushed to every rank -> max of the N keys -> token id.
__global__ void __launch_bounds__(256) tp_argmax_kernel(TpArgmaxArgs a) {
  __shared__ unsigned long long best_s[8];
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
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
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b = best_s[w] > b ? best_s[w] : b;
      // push this rank's key for row r into rank tid's key region, slot [me][r]
      a.keys[tid][(int64_t)a.me * a.max_rows + r] = b;
    }
    __syncthreads();
  }
  TpSite site{a.counters, a.me, a.n};
  tp_signal(site);
  if (tid == 0) {
    // this site has its own use count (greedy steps only), kept by this single-CTA kernel
    const int uses = ++a.uses[0];
    const unsigned long long target = (unsigned long long)uses * (unsigned long long)a.n;
    wait_arrivals(a.counter_local, target, a.status);
  }
  __syncthreads();
  for (int r = tid; r < a.rows; r += blockDim.x) {
    unsigned long long b = 0;
    for (int p = 0; p < a.n; ++p) {
      const unsigned long long k = __ldcg(a.keys_local + (int64_t)p * a.max_rows + r);
      b = k > b ? k : b;
    }
    a.out[r] = b == 0ull ? 0 : (int)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
  }
  pdl_launch();
}

void tp_argmax_launch(const TpArgmaxArgs& a, cudaStream_t s, bool pdl) {
  if (a.n > 256) throw std::runtime_error("tp argmax: at most 256 ranks");
  launch(tp_argmax_kernel, dim3(1), dim3(256), 0, s, pdl, a);
}

}  // namespace hk
