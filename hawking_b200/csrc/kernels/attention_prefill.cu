// Paged causal prefill attention on the tensor cores (K5 prefill): flash-style, one CTA per
// (64-query-row tile, HPC query heads of one KV group), bf16 mma.sync m16n8k16 with fp32
// accumulation. The HPC heads (4 warps each) share every K/V tile the CTA stages, so grouped-
// query attention moves each key and value through shared memory once per group, not per head.
//
// Rows are the forward's rows (row_seq picks the sequence's block-table row, row_ctx the number
// of keys the row sees, so causality is per row and a tile may hold the tail of one sequence and
// the head of the next: the tile is split into runs of rows of one sequence, each run streaming
// only its own sequence's keys). K/V tiles of 64 keys are gathered from the paged cache with
// cp.async into an XOR-swizzled double buffer (conflict-free ldmatrix), S = Q K^T and O += P V
// run on the tensor cores, and the online softmax (base-2, running max and sum per row) stays in
// registers; P never leaves the registers (the S accumulator fragment is the A fragment of P V).
// Tiles are taken last-first so the long causal rows start early.
//
// Parity: crates/hawking-core/src/kernels/attn.rs:23 (attention over the cached keys, causal),
// crates/hawking-core/src/kernels/mha.metal (prefill variants), same results as the decode
// kernel (attention.cu) up to bf16 rounding of q and P.
#include "common.cuh"
#include "api.h"

namespace hk {
namespace {

constexpr int kPfBM = 64;  // query rows per CTA: 4 warps x 16
constexpr int kPfBN = 64;  // keys per K/V tile

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // 0: zero-fill, nothing read
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// byte offset of 16-byte chunk c of row `row` in a swizzled [rows][HD] bf16 tile
template <int HD>
__device__ __forceinline__ uint32_t swz(int row, int c) {
  return (uint32_t)(row * HD * 2 + ((c ^ (row & 7)) << 4));
}

// Two CTAs per SM (HPC = 2: 16 warps; at most 128 registers per thread): the query fragments are
// re-read from shared memory per k-step instead of living in registers for the whole kernel
// (210 registers had left one CTA, 8 warps, per SM).
template <int HD, int HPC>
__global__ void __launch_bounds__(128 * HPC, HPC == 2 ? 2 : 4) attn_prefill_kernel(AttnDecodeArgs a) {
  constexpr int CH = HD / 8;           // 16-byte chunks per row
  constexpr int TILE = kPfBN * HD * 2;  // bytes of one K or V tile
  constexpr int NT = 128 * HPC;         // threads
  constexpr float kLog2e = 1.4426950408889634f;
  constexpr float NEG = -INFINITY;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* qs_all = smem;                      // [HPC][64][HD]
  uint8_t* ks = smem + HPC * kPfBM * HD * 2;   // [2][64][HD]
  uint8_t* vs = ks + 2 * TILE;                 // [2][64][HD]
  __shared__ int seq_s[kPfBM], ctx_s[kPfBM];

  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = (tid >> 5) & 3, hl = tid >> 7;
  const int ntiles = (a.R + kPfBM - 1) / kPfBM;
  // blockIdx.x (the fastest-launched index) is the head group, so every head group's longest
  // row tile is dispatched before any shorter tile (longest-first over the whole grid: the last
  // wave holds only short causal tiles)
  const int hg = (int)blockIdx.x;
  const int tile = ntiles - 1 - (int)blockIdx.y;
  const int h = hg * HPC + hl, g = (hg * HPC) / (a.nh / a.nkv);
  uint8_t* qs = qs_all + hl * kPfBM * HD * 2;  // this warp's head
  const int r0 = tile * kPfBM, nvalid = min(a.R - r0, kPfBM);
  if (tid < kPfBM) {
    seq_s[tid] = tid < nvalid ? a.row_seq[r0 + tid] : -1;
    ctx_s[tid] = tid < nvalid ? a.row_ctx[r0 + tid] : 0;
  }
  for (int i = tid; i < HPC * kPfBM * CH; i += NT) {  // q (fp32, roped) -> bf16 tiles, one per head
    const int hh = i / (kPfBM * CH), row = (i / CH) % kPfBM, c = i % CH;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < nvalid) {
      const float* src = a.q + ((int64_t)(r0 + row) * a.nh + hg * HPC + hh) * HD + c * 8;
      const float4 f0 = *reinterpret_cast<const float4*>(src), f1 = *reinterpret_cast<const float4*>(src + 4);
      v = make_uint4(pack_bf16(f0.x, f0.y), pack_bf16(f0.z, f0.w), pack_bf16(f1.x, f1.y), pack_bf16(f1.z, f1.w));
    }
    *reinterpret_cast<uint4*>(qs_all + hh * kPfBM * HD * 2 + swz<HD>(row, c)) = v;
  }
  __syncthreads();
  // this lane's ldmatrix row of the warp's 16 query rows (A fragments re-read per k-step)
  const uint32_t q_u = smem_u32(qs);
  const int q_row = warp * 16 + ((lane >> 3) & 1) * 8 + (lane & 7), q_hi = (lane >> 3) >> 1;
  const float sl2 = a.scale * kLog2e;
  const int lr0 = warp * 16 + (lane >> 2), lr1 = lr0 + 8;  // this thread's two accumulator rows
  const uint32_t ks_u = smem_u32(ks), vs_u = smem_u32(vs);
  const int64_t ostride = (int64_t)a.nh * HD;

  int s0 = 0;
  while (s0 < nvalid) {  // runs of rows of one sequence (uniform across the CTA)
    const int seq = seq_s[s0];
    int s1 = s0 + 1;
    while (s1 < nvalid && seq_s[s1] == seq) ++s1;
    int kv_len = 0;
    for (int i = s0; i < s1; ++i) kv_len = max(kv_len, ctx_s[i]);
    kv_len = min(kv_len, a.max_blocks * a.block_size);  // never past the row's table
    const bool in0 = lr0 >= s0 && lr0 < s1, in1 = lr1 >= s0 && lr1 < s1;
    const int c0 = in0 ? ctx_s[lr0] : 0, c1 = in1 ? ctx_s[lr1] : 0;
    float m0 = NEG, m1 = NEG, l0 = 0.f, l1 = 0.f;
    float o[HD / 8][4];
#pragma unroll
    for (int nd = 0; nd < HD / 8; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
    const int* bt = a.block_tables + (int64_t)seq * a.max_blocks;
    const int nkt = (kv_len + kPfBN - 1) / kPfBN;

    auto load_kv = [&](int kt, int buf) {
      for (int i = tid; i < kPfBN * CH; i += NT) {
        const int key = i / CH, c = i % CH;
        const int t = kt * kPfBN + key;
        const bool valid = t < kv_len;
        int64_t off = 0;
        if (valid) {
          const int blk = bt[t / a.block_size];
          off = (((int64_t)blk * a.nkv + g) * a.block_size + t % a.block_size) * HD + c * 8;
        }
        const uint32_t so = (uint32_t)(buf * TILE) + swz<HD>(key, c);
        cp_async16(ks_u + so, a.k_cache + off, valid);
        cp_async16(vs_u + so, a.v_cache + off, valid);
      }
      cp_async_commit();
    };

    if (nkt > 0) load_kv(0, 0);
    for (int kt = 0; kt < nkt; ++kt) {
      const int buf = kt & 1;
      if (kt + 1 < nkt) {
        load_kv(kt + 1, buf ^ 1);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      const uint32_t kb = ks_u + buf * TILE, vb = vs_u + buf * TILE;
      // S = Q K^T: 16 rows x 64 keys per warp
      float s[kPfBN / 8][4];
#pragma unroll
      for (int nb = 0; nb < kPfBN / 8; ++nb) s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
      {
        const int mi = lane >> 3;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          uint32_t qf[4];
          ldsm_x4(q_u + swz<HD>(q_row, kk * 2 + q_hi), qf[0], qf[1], qf[2], qf[3]);
#pragma unroll
          for (int nb2 = 0; nb2 < kPfBN / 16; ++nb2) {
            uint32_t b0, b1, b2, b3;
            const int key = nb2 * 16 + (mi >> 1) * 8 + (lane & 7);
            ldsm_x4(kb + swz<HD>(key, kk * 2 + (mi & 1)), b0, b1, b2, b3);
            mma_bf16(s[2 * nb2], qf, b0, b1);
            mma_bf16(s[2 * nb2 + 1], qf, b2, b3);
          }
        }
      }
      // causal mask + online softmax (base 2)
      const int kbase = kt * kPfBN + (lane & 3) * 2;
      float mx0 = NEG, mx1 = NEG;
#pragma unroll
      for (int nb = 0; nb < kPfBN / 8; ++nb) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = kbase + nb * 8 + e;
          s[nb][e] = key < c0 ? s[nb][e] * sl2 : NEG;
          s[nb][2 + e] = key < c1 ? s[nb][2 + e] * sl2 : NEG;
          mx0 = fmaxf(mx0, s[nb][e]);
          mx1 = fmaxf(mx1, s[nb][2 + e]);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float b0 = mn0 == NEG ? 0.f : mn0, b1 = mn1 == NEG ? 0.f : mn1;
      const float corr0 = exp2f(m0 - b0), corr1 = exp2f(m1 - b1);
      m0 = mn0;
      m1 = mn1;
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int nb = 0; nb < kPfBN / 8; ++nb) {
        s[nb][0] = exp2f(s[nb][0] - b0);
        s[nb][1] = exp2f(s[nb][1] - b0);
        s[nb][2] = exp2f(s[nb][2] - b1);
        s[nb][3] = exp2f(s[nb][3] - b1);
        rs0 += s[nb][0] + s[nb][1];
        rs1 += s[nb][2] + s[nb][3];
      }
      l0 = l0 * corr0 + rs0;
      l1 = l1 * corr1 + rs1;
#pragma unroll
      for (int nd = 0; nd < HD / 8; ++nd) {
        o[nd][0] *= corr0;
        o[nd][1] *= corr0;
        o[nd][2] *= corr1;
        o[nd][3] *= corr1;
      }
      // O += P V (P straight from the S fragments)
      {
        const int mi = lane >> 3;
#pragma unroll
        for (int t = 0; t < kPfBN / 16; ++t) {
          const uint32_t pa[4] = {pack_bf16(s[2 * t][0], s[2 * t][1]), pack_bf16(s[2 * t][2], s[2 * t][3]),
                                  pack_bf16(s[2 * t + 1][0], s[2 * t + 1][1]),
                                  pack_bf16(s[2 * t + 1][2], s[2 * t + 1][3])};
          const int key = t * 16 + (mi & 1) * 8 + (lane & 7);
#pragma unroll
          for (int nd2 = 0; nd2 < HD / 16; ++nd2) {
            uint32_t v0, v1, v2, v3;
            ldsm_x4_t(vb + swz<HD>(key, nd2 * 2 + (mi >> 1)), v0, v1, v2, v3);
            mma_bf16(o[2 * nd2], pa, v0, v1);
            mma_bf16(o[2 * nd2 + 1], pa, v2, v3);
          }
        }
      }
      __syncthreads();  // this buffer is refilled two tiles later
    }
    // finish the run: row sums across the quad, sinks, normalise, store
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    if (a.sinks) {
      const float sk = a.sinks[h] * kLog2e;
      l0 += exp2f(sk - (m0 == NEG ? 0.f : m0));
      l1 += exp2f(sk - (m1 == NEG ? 0.f : m1));
    }
    const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
    const int64_t row0 = r0 + lr0, row1 = r0 + lr1;
    const int col = h * HD + (lane & 3) * 2;
#pragma unroll
    for (int nd = 0; nd < HD / 8; ++nd) {
      o[nd][0] *= inv0;
      o[nd][1] *= inv0;
      o[nd][2] *= inv1;
      o[nd][3] *= inv1;
    }
    if (a.out_bf16) {
#pragma unroll
      for (int nd = 0; nd < HD / 8; ++nd) {
        if (in0) *reinterpret_cast<uint32_t*>(a.out_bf16 + row0 * ostride + col + nd * 8) = pack_bf16(o[nd][0], o[nd][1]);
        if (in1) *reinterpret_cast<uint32_t*>(a.out_bf16 + row1 * ostride + col + nd * 8) = pack_bf16(o[nd][2], o[nd][3]);
      }
    }
    if (a.out) {
#pragma unroll
      for (int nd = 0; nd < HD / 8; ++nd) {
        if (in0) *reinterpret_cast<float2*>(a.out + row0 * ostride + col + nd * 8) = make_float2(o[nd][0], o[nd][1]);
        if (in1) *reinterpret_cast<float2*>(a.out + row1 * ostride + col + nd * 8) = make_float2(o[nd][2], o[nd][3]);
      }
    }
    if (a.oq) {
      // q8 blocks of 32 dims = 4 n-blocks; the quad holds one row's whole block
#pragma unroll
      for (int b = 0; b < HD / 32; ++b) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          float am = 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) am = fmaxf(am, fmaxf(fabsf(o[4 * b + j][2 * half]), fabsf(o[4 * b + j][2 * half + 1])));
          am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
          am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
          const float d = am / 127.f, id = am > 0.f ? 127.f / am : 0.f;
          int qs_ = 0;
          const bool in = half ? in1 : in0;
          const int64_t row = half ? row1 : row0;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int qa = __float2int_rn(o[4 * b + j][2 * half] * id), qb = __float2int_rn(o[4 * b + j][2 * half + 1] * id);
            qs_ += qa + qb;
            if (in) {
              const uint16_t pk = (uint16_t)(uint8_t)(int8_t)qa | ((uint16_t)(uint8_t)(int8_t)qb << 8);
              *reinterpret_cast<uint16_t*>(a.oq + row * ostride + col + (4 * b + j) * 8) = pk;
            }
          }
          qs_ += __shfl_xor_sync(0xffffffffu, qs_, 1);
          qs_ += __shfl_xor_sync(0xffffffffu, qs_, 2);
          if (in && (lane & 3) == 0) {
            const int64_t blk = row * (ostride / 32) + (h * HD) / 32 + b;
            a.od[blk] = d;
            a.os[blk] = d * (float)qs_;
          }
        }
      }
    }
    s0 = s1;
  }
  pdl_launch();
}

template <int HD, int HPC>
void launch_prefill_hpc(const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  const int smem = HPC * kPfBM * HD * 2 + 4 * kPfBN * HD * 2;
  static bool configured = false;  // per instantiation; one device per process
  if (!configured) {
    HK_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_kernel<HD, HPC>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured = true;
  }
  const dim3 grid(a.nh / HPC, (a.R + kPfBM - 1) / kPfBM);
  launch(attn_prefill_kernel<HD, HPC>, grid, dim3(128 * HPC), smem, s, pdl, a);
}

template <int HD>
void launch_prefill(const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  if ((a.nh / a.nkv) % 2 == 0) launch_prefill_hpc<HD, 2>(a, s, pdl);  // two heads of one KV group per CTA
  else launch_prefill_hpc<HD, 1>(a, s, pdl);
}

}  // namespace

void attention_prefill_launch(const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  if (a.nh % a.nkv) throw std::runtime_error("attention prefill: heads must be a multiple of kv heads");
  if (a.R <= 0) return;
  switch (a.hd) {
    case 64: launch_prefill<64>(a, s, pdl); break;
    case 128: launch_prefill<128>(a, s, pdl); break;
    default: throw std::runtime_error("attention prefill: head_dim 64 or 128");
  }
}

}  // namespace hk
