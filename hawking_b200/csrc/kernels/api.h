// Host-visible kernel API: argument structs and launch entry points of every kernel group.
// Host-only code (the torch bindings) includes this header alone; device code is in the .cu/.cuh
// files.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hk {

enum WFmt : int { WF_Q4_K = 12, WF_Q6_K = 14, WF_Q4_0 = 2, WF_Q5_0 = 6, WF_Q8_0 = 8 };

struct WPlanes {
  const uint8_t* p0;   // main plane (raw blocks / qs / ql)
  const uint8_t* p1;   // scales plane (d), Q6_K: qh
  const uint8_t* p2;   // Q5_0: qh ; Q6_K: sc
  const uint8_t* p3;   // Q6_K: d
  int64_t rb0, rb1, rb2, rb3;  // per-row byte strides of each plane
};

struct XQ {
  const int8_t* q;  // [NB, K]
  const float* d;   // [NB, K/32]
  const float* s;   // [NB, K/32]
  int64_t stride_q, stride_s;  // per-column strides (elements)
};

// ---- small-batch dequant GEMV (gemv.cu) ----

enum GemvEpilogue : int { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU_Q8 = 2, EPI_PUSH = 3 };
enum GemvInput : int { XIN_Q8 = 0, XIN_NORM = 1 };

struct GemvArgs {
  WPlanes w0, w1;          // w1 used by the SwiGLU pair epilogue (up projection)
  int N, K;
  const int8_t* xq;        // q8 activations [nb, K]
  const float* xd;
  const float* xs;
  int64_t x_stride_q, x_stride_s;
  float* y;                // [nb, y_stride] (STORE / RESID)
  int64_t y_stride;
  const float* bias;       // optional [N]
  int8_t* oq;              // SWIGLU_Q8 output q8 [nb, N]
  float* od;
  float* os;
  int64_t o_stride_q, o_stride_s;
  // Fused-norm input (used instead of xq/xd/xs when x_f32 != nullptr): fp32 rows, optional
  // RMSNorm with weight norm_w, quantised to q8 blocks inside each CTA.
  const float* x_f32;
  int64_t x_f32_stride;
  const float* norm_w;
  float eps;
  int norm;
  // Greedy fusion (STORE epilogue): every row's value is folded into packed (value, index) keys
  // with atomicMax, kArgmaxSlots slots per batch column (spreads the contention);
  // argmax_finalize_launch turns them into token ids and clears them for the next launch.
  unsigned long long* argmax_slots;
  int64_t argmax_offset;   // added to row indices in the packed keys (vocabulary-parallel LM head)
  // EPI_PUSH (tensor-parallel row-parallel projection): every output (row, column b) is stored to
  // push_recv[p][b * N + row] on every rank p as one flagged word (value | step epoch << 32).
  unsigned long long* const* push_recv;
  const int* push_epoch;
  int push_n;
  // L2 prefetch of the NEXT kernel's weights (up to kPrefetchRanges byte ranges): every CTA issues
  // bulk L2 prefetches for its share before waiting on the previous kernel, so the chain of decode
  // GEMVs streams weights from HBM continuously and each kernel finds its own weights in L2.
  const uint8_t* pf_ptr[8];
  int64_t pf_bytes[8];
  int pf_n;
};
constexpr int kArgmaxSlots = 256;

// ---- tensor parallel (tp.cu) ----
struct TpReduceArgs {
  const float* x_in;            // residual before the projection [rows, x_stride]
  float* x_out;                 // residual after it (a different buffer)
  int64_t x_stride;
  const unsigned long long* recv;  // this rank's receive region of the site: [n][rows][K] flagged words
  int64_t rank_stride;          // words between source ranks in `recv`
  int n;
  const int* epoch;             // flag of this step's words
  const float* w;               // RMSNorm weight of the next projection
  float eps;
  int K;
  int8_t* xq;                   // q8 output of the normalised rows, or null:
  float* xd;
  float* xs;
  __nv_bfloat16* yb;            //   bf16 normalised rows [rows, yb_stride] (W4A16 consumers)
  int64_t yb_stride;
  int* status;
  unsigned long long wait_ns;   // bound of each peer wait (0: the default, one second)
};
// Tensor-core path (up to wide_rows rows): every rank's row-parallel GEMM accumulates its partial
// into its own IPC-shared buffer of the site; this consumer raises the rank's flag of the site on
// every peer, waits (bounded) for all N flags, reads the N partials over NVLink (P2P loads, fixed
// rank order), adds the residual and normalises, as tp_allreduce_rmsnorm does for pushed words.
struct TpP2PArgs {
  const float* x_in;
  float* x_out;
  int64_t x_stride;
  const unsigned long long* parts;      // [n] addresses of every rank's partial of the site [rows][K]
  unsigned int* flags_local;            // this rank's flags of the site [n] (peers write slot `src`)
  const unsigned long long* flag_ptrs;  // [n] addresses of every rank's flags of the site
  int n, me;
  const int* epoch;                     // flag value of this forward
  const float* w;
  float eps;
  int K;
  int8_t* xq;
  float* xd;
  float* xs;
  __nv_bfloat16* yb;
  int64_t yb_stride;
  int* status;
  unsigned long long wait_ns;
};
void tp_p2p_allreduce_rmsnorm_launch(const TpP2PArgs& a, int rows, cudaStream_t s, bool pdl);
struct TpArgmaxArgs {
  unsigned long long* slots;    // local fused-argmax slots [rows, kArgmaxSlots] (cleared here)
  int rows, max_rows;
  unsigned long long* const* keys;       // [n] every rank's key region [n][max_rows][2] flagged words
  const unsigned long long* keys_local;  // this rank's key region
  int* uses;                    // this rank's count of argmax rounds = the flag (device, updated here)
  int me, n;
  int* out;                     // token ids [rows]
  int* status;
  unsigned long long wait_ns;   // bound of each peer wait (0: the default, one second)
};
void tp_begin_launch(int* epoch, cudaStream_t s, bool pdl);
void tp_allreduce_rmsnorm_q8_launch(const TpReduceArgs& a, int rows, cudaStream_t s, bool pdl);
void tp_argmax_launch(const TpArgmaxArgs& a, cudaStream_t s, bool pdl);

void gemv_launch(int fmt, int epi, const GemvArgs& a, int nb, cudaStream_t s, bool pdl);

// ---- full-precision small-batch GEMV on the tensor cores (mma_gemv.cu) ----
// W4A16: weights in fragment-ordered tiles of 16 rows x 256 columns (mg_pack_launch), bf16
// activations, fp32 accumulation. See mma_gemv.cu for the design.
enum MgInput : int { MG_X_NORM = 0, MG_X_BF16 = 1, MG_X_FRAG = 2, MG_X_FRAG_SMEM = 3 };  // 3: internal (FRAG staged)
enum MgEpilogue : int { MG_STORE = 0, MG_RESID = 1, MG_SWIGLU = 2, MG_PUSH = 3, MG_ROPE = 4 };
// Math of the tiles: MG_MATH_BF16 (bf16 activations, bf16 MMA; tiles packed for it) or MG_MATH_INT
// (activations as 16-bit fixed point per 32-element block, held as two int8 limbs, u8 x s8 MMA;
// tiles packed for it). The input modes are the same; MG_X_FRAG of the integer math is the layout
// written by mg_quant_launch.
enum MgMath : int { MG_MATH_BF16 = 0, MG_MATH_INT = 1 };
struct MgArgs {
  const uint8_t* tiles;     // [G row groups][KT column tiles][tile bytes]
  int G, KT;                // row groups (16 rows each), 256-column tiles per row group
  int N, K;                 // logical rows (STORE / RESID / PUSH) and columns
  int nb;                   // batch columns 1..8
  // input (one of):
  const float* x_f32;       // MG_X_NORM: fp32 rows [nb, x_f32_stride], RMSNorm with norm_w (optional)
  int64_t x_f32_stride;
  const float* norm_w;
  float eps;
  const __nv_bfloat16* xb;  // MG_X_BF16: bf16 rows [nb, xb_stride]
  int64_t xb_stride;
  const uint4* xfrag;       // MG_X_FRAG: bf16 in B-fragment order, column n at n * xfrag_cstride uint4s
  int64_t xfrag_cstride;    //   (integer math: the two limbs in B-fragment order, see mg_quant_launch)
  const float2* xinfo;      // MG_X_FRAG, integer math: per (32-block b, column n) (d2, block sum) at
                            //   xinfo[b * 8 + n]
  int math;                 // MgMath of the tiles
  // outputs
  float* y;                 // STORE / RESID: fp32 [nb, y_stride]
  int64_t y_stride;
  const float* bias;        // optional [N]
  int F;                    // SWIGLU: output rows (tiles hold gate rows 8g..8g+7 then the matching up rows)
  __nv_bfloat16* hfrag;     // SWIGLU: h in B-fragment order (column stride hfrag_cstride uint4s), and/or
  int64_t hfrag_cstride;
  __nv_bfloat16* hb;        //   h as plain bf16 rows [nb, hb_stride]
  int64_t hb_stride;
  unsigned long long* argmax_slots;  // STORE: fused greedy keys (as GemvArgs)
  int64_t argmax_offset;
  unsigned long long* const* push_recv;  // PUSH: as GemvArgs
  const int* push_epoch;
  int push_n;
  // QKV packed in RoPE-pair order (rp_heads > 0): the store epilogue writes logical rows
  int rp_heads, rp_hd, rp_rot, rp_style;
  // MG_ROPE epilogue (QKV packed in RoPE-pair order): RoPE + paged K/V append, q to q_out
  const float* rope;
  const int* positions;
  const int* row_seq;
  const int* block_tables;
  int max_blocks, block_size;
  int64_t cache_blocks;        // blocks in the caches: a row whose block id or table column is out
                               // of range skips its K/V append
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  float* q_out;
  int nh, nkv;
  // scratch: partial fragments [SMs * 3 CTAs * 8 warps][2][32] float4, zeroed counters [G]
  float4* part;
  int* counters;
  int* status;
};
int mg_tile_bytes(int fmt);
size_t mg_smem_bytes(int fmt, int math, int xin, int nb, int K);
// rowmap[G * 16]: source row of each tile row (-1: zero row)
void mg_pack_launch(int fmt, int math, const WPlanes& w, const int* rowmap, int G, int KT, uint8_t* out,
                    cudaStream_t s);
// Integer math, wide inputs: quantise bf16 rows [nb, x_stride] (K % 256 == 0) into the two-limb
// B-fragment layout (column n at n * cstride uint4s) and the per-block info [K/32][8] float2.
void mg_quant_launch(const __nv_bfloat16* x, int64_t x_stride, int nb, int K, uint4* xfrag, int64_t cstride,
                     float2* xinfo, cudaStream_t s, bool pdl);
void mg_gemv_launch(int fmt, int xin, int epi, const MgArgs& a, int sms, cudaStream_t s, bool pdl);

// ---- persistent decode step (decode_step.cu) ----
// One launch runs every layer of a dense Llama-family model for up to kDsMaxRows batch rows, plus
// the final norm and the LM head: QKV GEMV with RoPE and the paged K/V append in its epilogue,
// split-KV attention on the tensor cores, O GEMV + residual, gate/up GEMV + SwiGLU, down GEMV +
// residual, all on the W4A16 integer-math tiles of mma_gemv.cu (Q4_K), separated by grid-wide
// barriers (one CTA per SM, all resident). Weights of the next phase stream into each warp's ring
// before the barrier that precedes it.
constexpr int kDsMaxRows = 4;
struct DsLayer {  // one per layer, in device memory
  const uint8_t* qkv;   // packed with RoPE pairs as tile rows r / r + 8 (mg pack, rope order)
  const uint8_t* o;
  const uint8_t* gu;    // SwiGLU-interleaved gate / up
  const uint8_t* down;
  const float* attn_norm;
  const float* ffn_norm;
  const float* qkv_bias;  // logical row order; may be null
};
struct DsArgs {
  const DsLayer* layers;
  int L;
  int H, F, nh, nkv, hd, rot, rope_style, block_size, max_blocks, num_cache_blocks;
  int nb;          // batch rows (<= kDsMaxRows)
  int splits;      // KV splits per (row, kv head)
  float eps, scale;
  const int* positions;
  const int* row_seq;
  const int* row_ctx;
  const int* block_tables;
  const float* rope;  // [max_pos, rot / 2, 2] (cos, sin)
  float* x;           // [nb, H] residual stream (in: embeddings; out: final hidden state)
  float* q;           // [nb, nh, hd] roped queries
  __nv_bfloat16* k_cache;  // [L, blocks, nkv, block_size, hd]
  __nv_bfloat16* v_cache;
  float* att_o;       // [nb * nkv * splits, G * hd] split partials
  float2* att_ml;     // [nb * nkv * splits, G] (max, sum)
  int* att_cnt;       // [nb * nkv] zeroed
  uint4* a_limbs;     // attention output, two-limb fragment order: [nb, H / 8] uint4
  float2* a_info;     // [nb, H / 32]
  float* hf;          // [nb, F] SwiGLU output
  uint4* h_limbs;     // [nb, F / 8]
  float2* h_info;     // [nb, F / 32]
  int* h_cnt;         // [F / 32] zeroed
  float4* part;       // split-K partials [grid * 16 warps][2][32]
  int* counters;      // [max row groups] zeroed
  const uint8_t* head;  // LM head tiles (plain row order)
  const float* out_norm;
  int V;
  float* logits;      // [nb, V] (may be null)
  unsigned long long* argmax_slots;  // [nb, kArgmaxSlots] (may be null)
  unsigned int* bar;  // [2] zeroed: arrivals, generation
  int* status;
  long long wait_ns;  // bound of every grid-barrier wait
  // optional [grid][4]: barriers passed, and the first failed wait of the CTA (site: 1 weight
  // ring, 2 attention K/V unit, 3 attention ring slot, 4 activation copy, 5 grid barrier; phase
  // 5l + k; warp)
  int* trace;
  // optional [5 * L + 2][4] globaltimer (ns): row 0 kernel start; row p + 1 for phase p: CTA 0's
  // exit from the barrier closing it, earliest and latest CTA arrival at that barrier, CTA 0's end
  // of activation staging (phases with staging); the caller presets columns 1 / 2 to max / 0
  long long* tstamp;
};
// Whether the shape is supported (head_dim 64 / 128, GQA group <= 16, block size 16 / 32 / 64,
// rot_dim % 16 == 0, H and F multiples of 256, rows <= kDsMaxRows, staging fits shared memory).
bool ds_supported(const DsArgs& a);
// CTAs of the persistent grid (one per SM).
int ds_grid(int device);
void ds_launch(const DsArgs& a, cudaStream_t s);

// ---- decode ops (decode_ops.cu, attention.cu) ----

// RMSNorm (optional weight) of rows of x, then q8 activation blocks. `norm=false` quantises x
// unchanged. Also writes the normalised row to y (fp32) when y != nullptr.
void rmsnorm_q8_launch(const float* x, int64_t x_stride, const float* w, float eps, bool norm, int rows, int K,
                       int8_t* xq, float* xd, float* xs, float* y, cudaStream_t s, bool pdl);

// Plain RMSNorm to bf16/fp32 (used ahead of tensor-core GEMMs).
void rmsnorm_launch(const float* x, int64_t x_stride, const float* w, float eps, int rows, int K, float* y_f32,
                    __nv_bfloat16* y_bf16, int64_t y_stride, cudaStream_t s, bool pdl);

struct RopeAppendArgs {
  const float* qkv;            // [R, (nh + 2*nkv) * hd] fp32 (projection output)
  int64_t qkv_stride;
  const float* bias;           // optional [(nh + 2*nkv) * hd]
  const float* q_norm;         // optional per-head RMSNorm weights [hd] (Qwen3 style)
  const float* k_norm;
  float eps;
  const int* positions;        // [R]
  const int* slots;            // [R] paged slot = block * block_size + offset (-1 = skip); or null:
  const int* block_tables;     //   slot from block_tables[row_seq[r], pos / bs] (when slots is null)
  const int* row_seq;
  int max_blocks;
  int64_t cache_blocks;        // blocks in the caches: a slot outside them (or a position past the
                               // row's table) skips the append
  const float* rope;           // [max_pos, rot/2, 2] (cos, sin)
  int rot_dim, rope_style;     // 0 adjacent pairs, 1 neox halves
  float* q_out;                // [R, nh, hd] fp32 (roped)
  __nv_bfloat16* k_cache;      // [num_blocks, nkv, bs, hd]
  __nv_bfloat16* v_cache;
  int R, nh, nkv, hd, block_size;
};
void rope_append_launch(const RopeAppendArgs& a, cudaStream_t s, bool pdl);

struct AttnDecodeArgs {
  const float* q;              // [R, nh, hd] fp32, roped
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  const int* block_tables;     // [S, max_blocks]
  int max_blocks;
  const int* row_seq;          // [R] block-table row of each query row
  const int* row_ctx;          // [R] number of keys visible to the row (causal length)
  float scale;
  int R, nh, nkv, hd, block_size, num_splits;
  float* part_o;               // [R, nh, num_splits, hd] scratch
  float* part_lse;             // [R, nh, num_splits] scratch
  float* out;                  // [R, nh*hd] fp32 (optional)
  int8_t* oq;                  // q8 output [R, nh*hd] (optional)
  float* od;
  float* os;
  const float* sinks;          // optional per-head attention sink logits [nh]
  __nv_bfloat16* out_bf16;     // optional [R, nh*hd] bf16 output (tensor-core GEMM path)
  int* counters;               // [R * nkv] zero-initialised split counters (scratch; reset after use)
  int* status;                 // optional device status word (bounded-wait timeouts)
  int stage_blocks;            // cluster path: KV blocks held in the shared ring (set by the launcher)
  int table_rows;              // rows of block_tables (0: unknown; bounds the speculative L2 prefetch)
};
void attention_decode_launch(const AttnDecodeArgs& a, cudaStream_t s, bool pdl);
// Cluster variant (num_splits in {1, 2, 4, 8}): the splits of one (row, kv head) merge through
// distributed shared memory; part_o / part_lse / counters are not used.
void attention_decode_cluster_launch(const AttnDecodeArgs& a, cudaStream_t s, bool pdl);
// Tensor-core decode (attention_tc.cu): TMA tensor loads of the K/V blocks, query heads of a KV head
// as MMA rows, splits in a cluster (num_splits 1, 2, 4 or 8). cache_rows = num_blocks * nkv *
// block_size (the rows of the caches viewed as [rows, hd]). head_dim 64 or 128, GQA group <= 16.
bool attention_decode_tc_supported(const AttnDecodeArgs& a);
void attention_decode_tc_launch(const AttnDecodeArgs& a, int64_t cache_rows, cudaStream_t s, bool pdl);
// Causal prefill on the tensor cores (attention_prefill.cu): any rows (runs of one sequence are
// found on the device), head_dim 64 or 128; outputs out / out_bf16 / q8 (split fields unused).
void attention_prefill_launch(const AttnDecodeArgs& a, cudaStream_t s, bool pdl);

// Reduce the packed argmax slots of `rows` batch columns to token ids and zero the slots.
void argmax_finalize_launch(unsigned long long* slots, int rows, int* out, cudaStream_t s, bool pdl);

// Greedy: index of the max logit per row (lowest index on ties).
void argmax_launch(const float* logits, int64_t stride, int rows, int V, int* out, cudaStream_t s, bool pdl);

struct SampleArgs {
  const float* logits;         // [R, V]
  int64_t stride;
  int R, V;
  const float* temperature;    // [R]; <= 0 means greedy
  const int* top_k;            // [R]; 0 = off (candidate pool capped at 1024)
  const float* top_p;          // [R]
  const float* rep_penalty;    // [R]
  const int* recent;           // [R, recent_n] recent token ids (-1 = empty) for repetition penalty
  int recent_n;
  const float* uniforms;       // [R] uniform draws in [0,1)
  int* out;                    // [R]
};
void sample_launch(const SampleArgs& a, cudaStream_t s, bool pdl);

// Device-side step advance for back-to-back decode: ids <- next_ids, positions += 1, ctx += 1.
void advance_launch(int* ids, const int* next_ids, int* positions, int* row_ctx, int R, cudaStream_t s, bool pdl);

// Embedding rows: out[r] = dequant(table[ids[r]]) (fp32).
void embed_launch(int fmt, const WPlanes& table, const int* ids, int R, int H, float* out, int64_t out_stride,
                  cudaStream_t s, bool pdl);

// ---- tensor-core dequant GEMM (gemm_tc.cu) ----
struct TcGemmArgs {
  int fmt;                      // weight format (Q4_K)
  const uint8_t* w;             // quants plane [N, w_row_bytes] (K/2 bytes per row)
  int64_t w_row_bytes;
  const uint8_t* w_hdr;         // header plane [N, w_hdr_row_bytes] (16 bytes per super-block)
  int64_t w_hdr_row_bytes;
  int N, K;
  const __nv_bfloat16* x;       // [M, x_stride] bf16
  int64_t x_stride;
  int M;
  float* y;                     // [M, y_stride] fp32
  int64_t y_stride;
  int atomic;                   // accumulate into y (residual / split-K)
  int y_zeroed;                 // caller zeroed y (allows split-K with a plain result)
  int k_splits;
  int bn;                       // token tile: 32, 64, 128 or 256
  int* status;                  // device status word (bounded-wait errors)
  bool pdl;
  // SwiGLU epilogue: W is a fused [gate (F rows) | up (F rows)] matrix (N = 2F); each CTA
  // dequantises 64 gate rows and the 64 matching up rows, and writes h = silu(g) * u as bf16
  // [M, h_stride] (no fp32 output, y unused)
  __nv_bfloat16* h;
  int64_t h_stride;
  // persistent launch (one CTA per SM looping over tiles, epilogue overlapped with the next
  // tile's main loop); no split-K. 2: stream-K, every CTA one balanced range of (tile, K stage)
  // units, partial tiles accumulated with atomics (atomic or zeroed y; no SwiGLU)
  int persistent;
};
int tc_gemm_splits(int N, int M, int K, int bn, int sms);
void tc_gemm_launch(const TcGemmArgs& g, cudaStream_t s);

// The same tcgen05 GEMM with bf16 weights loaded by TMA (a dequantised copy of any format):
// Y[M, N] (+)= X[M, K] W[N, K]^T, or h = silu(g) u (bf16) from a [gate | up] W of N = 2F rows.
// Grouped: CTA row y takes tile (group, first row, end row) = tiles[3 y ..] while y < *n_tiles
// (built on the device), reading weight rows group * group_rows + the tile's local rows; output
// columns are local (N = group_rows). One launch runs every expert of a MoE layer.
struct TcBf16Args {
  const __nv_bfloat16* w;       // [w_rows, w_stride] bf16
  int64_t w_stride;
  int w_rows;
  int N, K;
  const __nv_bfloat16* x;       // [x_rows, x_stride] bf16
  int64_t x_stride;
  int x_rows;
  int M;                        // rows of X the (ungrouped) product covers
  float* y;                     // [*, y_stride] fp32
  int64_t y_stride;
  int atomic, y_zeroed, k_splits, bn;
  __nv_bfloat16* h;             // SwiGLU output [*, h_stride] or null
  int64_t h_stride;
  const int* tiles;             // grouped tile list (device) or null
  const int* n_tiles;
  int max_tiles;                // grid rows launched (>= the number of tiles)
  int group_rows;
  int* status;
  bool pdl;
};
void tc_gemm_bf16_launch(const TcBf16Args& g, cudaStream_t s);

// SwiGLU over a fused [gate | up] fp32 GEMM output: h = silu(g) * u -> bf16, then zero the input
// (ready for the next split-K accumulation).
void swiglu_bf16_launch(float* gu, int64_t gu_stride, int M, int F, __nv_bfloat16* h, int64_t h_stride,
                        bool clear, cudaStream_t s, bool pdl);

// ---- mixture of experts (moe.cu) ----
void router_logits_launch(const float* w, int E, int K, const int8_t* xq, const float* xd, int64_t xs_q,
                          int64_t xs_d, float* logits, int T, cudaStream_t s, bool pdl);

struct MoeTopkArgs {
  const float* logits;   // [T, E]
  const float* bias;     // optional [E] selection bias (sigmoid scoring)
  int T, E, k;
  int scoring;           // 0 softmax, 1 sigmoid
  int n_groups, topk_groups;
  int renorm;
  float scale;           // routed scaling factor
  int* ids;              // [T, k]
  float* weights;        // [T, k]
};
void moe_topk_launch(const MoeTopkArgs& a, cudaStream_t s, bool pdl);

struct MoeRouteArgs {           // fused decode routing (moe.cu)
  const float* router;          // [E, K] fp32
  const int8_t* xq;             // q8 hidden [T, K]
  const float* xd;
  int64_t x_stride_q, x_stride_s;
  int T, E, K, k;
  const float* bias;
  int scoring, n_groups, topk_groups, renorm;
  float scale;
  float* logits;                // scratch [T, E]
  int* ids;                     // [T, k]
  float* weights;               // [T, k]
  int* counts;                  // [E + 1]
  int* offsets;                 // [E + 1]
  int* sorted;                  // [T * k + T]
  int* active;                  // [E + 1]
  int* n_active;
  int shared;                   // append the shared expert as expert E
  int* counter;                 // zero-initialised arrival counter (reset by the kernel)
  // expert parallelism: only experts in [e_lo, e_hi) (this rank's) enter the active list
  // (e_hi == 0: every expert); counts, offsets and sorted still cover all E experts
  int e_lo, e_hi;
};
void moe_route_launch(const MoeRouteArgs& a, cudaStream_t s, bool pdl);

struct MoeAlignArgs {
  const int* ids;        // [T, k]
  int T, k, E, K;
  const int8_t* xq;      // token activations (q8) [T, K]
  const float* xd;
  const float* xs;
  int64_t x_stride_q, x_stride_s;
  int* counts;           // [E] (+1 with `shared`)
  int* offsets;          // [E] (+1 with `shared`)
  int* sorted;           // [T*k] pair ids (t*k + j) grouped by expert (+T shared pairs)
  int8_t* gq;            // gathered activations [T*k, K] (sorted order)
  float* gd;
  float* gs;
  int shared;            // 1: append expert E (the shared expert) with pairs T*k + t, one per token
};
void moe_align_launch(const MoeAlignArgs& a, cudaStream_t s, bool pdl);

struct MoeGemvArgs {
  WPlanes w0, w1;        // stacked expert weights [E * N, K] (w1: up projection for epi 0)
  int N, K, E, k;
  const int* counts;
  const int* offsets;
  const int* sorted;
  const int8_t* xq;      // inputs in sorted order [T*k, K]
  const float* xd;
  const float* xs;
  int8_t* oq;            // epi 0: SwiGLU output q8 in sorted order [T*k, N]
  float* od;
  float* os;
  float* y;              // epi 1: residual [T, y_stride] (atomic add of route_w * y)
  int64_t y_stride;
  const float* route_w;  // [T*k]
  // expert parallelism: w0/w1 stack only experts [e_lo, e_lo + E) of the global numbering
  int e_lo;
  // epi 2 (expert-parallel combine): per token, the route-weighted sum over this rank's experts
  // is pushed to every rank's receive region as flagged words (see EpPush)
  int T;
  unsigned long long* const* push_recv;
  const int* push_epoch;
  int push_n;
  const float* base;     // epi 2: optional [T, base_stride] fp32 rows added to each token's sum
  int64_t base_stride;
};
void moe_gemv_launch(int fmt, int epi, const MoeGemvArgs& a, cudaStream_t s, bool pdl);

// ---- `.gravity` mixed low-bit codecs (mixed_gemv.cu) ----
// MIXED_Q4K: a GGUF Q4_K tensor as its two planes (quants [rows, K/2] as codes, the 16-byte
// super-block headers d | dmin | 12 scale bytes as `scales`, [rows, K/32] halves)
// MIXED_FP4: fp4 e2m1 codes two per byte (even column in the low nibble, [rows, K/2]) with one
// power-of-two scale per 32 columns (the e8m0 exponents, exact as fp32: scales_f32 [rows, K/32])
enum MixedKind : int { MIXED_BINARY = 0, MIXED_UNIFORM = 1, MIXED_FP8 = 2, MIXED_Q4K = 3, MIXED_FP4 = 4 };
struct MixedDesc {            // one weight tensor [rows, K] in device memory
  const uint8_t* codes;       // LSB-first code stream per row
  const __half* scales;       // fp16 group scales per row (binary / uniform)
  const float* scales_f32;    // fp8 / fp4: fp32 scale per (row, group of columns)
  int64_t code_row_bytes;     // K * bits / 8
  int64_t scale_row_elems;    // K / group
  int kind, bits, group, bound;
};
struct MixedGemvArgs {
  const MixedDesc* desc;      // device array of descriptors
  int d0, d1;                 // descriptor indices (d1: up projection of the SwiGLU pair)
  int N, K, nb;
  const int8_t* xq;
  const float* xd;
  const float* xs;
  int64_t x_stride_q, x_stride_s;
  float* y;                   // STORE / RESID output [nb, y_stride]
  int64_t y_stride;
  float alpha;                // output scale (STORE / RESID)
  const float* gate_logit;    // optional per-column logit g: outputs scaled by sigmoid(g) (shared-expert gate)
  int64_t gate_stride;
  int8_t* oq;                 // SWIGLU_Q8 output
  float* od;
  float* os;
  int64_t o_stride_q, o_stride_s;
  // EPI_PUSH: row-parallel projection pushed to every rank (same word layout as GemvArgs)
  unsigned long long* const* push_recv;
  const int* push_epoch;
  int push_n;
  // EPI_STORE greedy fusion (as GemvArgs): packed (value, row + argmax_offset) keys, atomicMax
  unsigned long long* argmax_slots;
  int64_t argmax_offset;
};
void mixed_gemv_launch(int epi, const MixedGemvArgs& a, cudaStream_t s, bool pdl);

// ---- prefill of the mixed-codec MoE models (moe_prefill.cu) ----
void mixed_dequant_bf16_launch(const MixedDesc* desc, const int* didx, const int* drow, int count, int rows, int K,
                               __nv_bfloat16* out, int64_t out_stride, cudaStream_t s, bool pdl);
void moe_tiles_launch(const int* counts, const int* offsets, int E1, int bn, int* tiles, int* n_tiles, int e_lo,
                      int e_hi, int shared_e, cudaStream_t s, bool pdl);
void moe_gather_bf16_launch(const int* sorted, int PS, int P, int k, const __nv_bfloat16* x, int64_t x_stride, int K,
                            __nv_bfloat16* xg, int64_t xg_stride, int* pos, cudaStream_t s, bool pdl);
void moe_combine_launch(const float* y, int64_t y_stride, const int* pos, const float* w, int T, int k, bool shared,
                        const float* shared_gate, int64_t gate_stride, float* x, int64_t x_stride, int H,
                        const int* ids, int e_lo, int e_hi, cudaStream_t s, bool pdl);
void qweight_dequant_bf16_launch(int fmt, const WPlanes& w, int rows, int K, int group_rows, int dst_group_rows,
                                 int dst_off, __nv_bfloat16* out, int64_t out_stride, cudaStream_t s, bool pdl);
void q8_to_bf16_launch(const int8_t* q, const float* d, int64_t q_stride, int64_t d_stride, int rows, int K,
                       __nv_bfloat16* out, int64_t out_stride, cudaStream_t s, bool pdl);
// HGRAVR02 outlier residual added into y [nb, >= N] (row_ptr [N + 1], cols / signs [nnz]).
void sparse_residual_launch(const int* row_ptr, const int* cols, const int8_t* signs, float scale, int N,
                            const int8_t* xq, const float* xd, int K, int nb, float* y, int64_t y_stride,
                            cudaStream_t s, bool pdl);
struct MoeMixedArgs {
  const MixedDesc* desc;      // expert e of matrix m at desc_base_m + e
  int desc_base0, desc_base1;
  int N, K, k;
  const int* counts;
  const int* offsets;
  const int* sorted;
  const int* active;          // experts with pairs (moe_active), first *n_active valid
  const int* n_active;
  const int8_t* xq;           // sorted-order activations [T*k, K]
  const float* xd;
  const float* xs;
  int8_t* oq;                 // epi 0 output (sorted order) [T*k, N]
  float* od;
  float* os;
  float* y;                   // epi 1: residual rows of the tokens
  int64_t y_stride;
  const float* route_w;
  int routed_pairs;           // pairs below this are routed (token pair / k, weight route_w[pair]);
                              // the rest are shared-expert pairs (token pair - routed_pairs, weight 1,
                              // or sigmoid(shared_gate[token]) for a gated shared expert)
  const float* shared_gate;   // per-token shared-expert gate logits (stride shared_gate_stride) or null
  int64_t shared_gate_stride;
  int direct;                 // epi 0: read each pair's token row of xq/xd/xs (strides below)
  int64_t x_stride_q, x_stride_s;
  // expert parallelism: the table holds this rank's experts e_lo .. e_lo + e_count - 1 at
  // desc_base + e - e_lo and the shared expert (global id E) right after them
  int e_lo, e_count;
  // epi 2 (expert-parallel combine into the tensor-parallel all-reduce): tokens T, receive tables
  int T;
  unsigned long long* const* push_recv;
  const int* push_epoch;
  int push_n;
};
void moe_mixed_gemv_launch(int epi, const MoeMixedArgs& a, int max_active, cudaStream_t s, bool pdl);
void moe_active_launch(const int* counts, int E, int* active, int* n_active, cudaStream_t s, bool pdl);

// ---- codebook / low-rank / sparse GEMVs (codebook.cu) ----
struct CodebookArgs {
  const __half* codebooks;    // [nsub][card][width]
  const uint8_t* codes;       // MSB-first packed indices [rows][nchunk][nsub] (+4 bytes padding)
  int rows, nchunk, nsub, card, width, d, sub_stride, bits;
  const int8_t* xq;           // q8 activations [nb, cols]
  const float* xd;
  int64_t x_stride_q, x_stride_s;
  int nb;
  float* lut;                 // scratch [nb][nchunk * nsub * card]
  float* y;                   // [nb, y_stride]
  int64_t y_stride;
  float alpha;
  int accumulate;
};
void codebook_gemv_launch(const CodebookArgs& a, cudaStream_t s, bool pdl);
struct AapArgs {
  const __half* in_proj;      // input side: basis [cols, rank]; output side: coefficients [rank, cols]
  const __half* out_proj;     // [rows, rank]: coefficients (input side) or basis (output side)
  int rows, cols, rank, side;
  const int8_t* xq;
  const float* xd;
  int64_t x_stride_q, x_stride_s;
  int nb;
  float* latent;              // scratch [nb, rank]
  float* y;
  int64_t y_stride;
  float alpha;
  int accumulate;
};
void aap_gemv_launch(const AapArgs& a, cudaStream_t s, bool pdl);
struct SparseArgs {           // y[b][r] += alpha * sum over row r's entries of val * x_b[col]
  const int* row_ptr;         // [rows + 1]
  const int* col;
  const __half* val;
  int rows;
  const int8_t* xq;
  const float* xd;
  int64_t x_stride_q, x_stride_s;
  int nb;
  float* y;
  int64_t y_stride;
  float alpha;
};
void sparse_rows_launch(const SparseArgs& a, cudaStream_t s, bool pdl);

// ---- gated DeltaNet (deltanet.cu) ----
struct DeltaConvArgs {
  const float* qkvz;          // [R, qkvz_stride] fused projection (per key head: q k v z)
  int64_t qkvz_stride;
  const float* conv_w;        // [2*kh*dk + kh*r*dv, kc]
  float* conv_state;          // [slots, channels, kc - 1]
  const int* state_slot;      // [R] recurrent-state slot of each row (null: slot = row)
  int kh, r, dk, dv, kc;
  float eps;
  float* q;                   // [R, kh*r, dk] (L2-normalised, scaled)
  float* k;                   // [R, kh*r, dk]
  float* v;                   // [R, kh*r*dv]
  float* z;                   // [R, kh*r*dv]
};
void deltanet_conv_launch(const DeltaConvArgs& a, int rows, cudaStream_t s, bool pdl);
struct DeltaRecArgs {
  float* state;               // [slots, kh*r, dk, dv]
  const int* state_slot;
  const float* q;
  const float* k;
  const float* v;
  const float* z;
  const float* ba;            // [R, ba_stride] (per key head: b[r] a[r])
  int64_t ba_stride;
  const float* a_log;         // [kh*r]
  const float* dt_bias;       // [kh*r]
  int r, dk, dv;
  const float* norm_w;        // [dv]
  float eps;
  float* out;                 // optional fp32 [R, kh*r*dv]
  int8_t* oq;                 // q8 [R, kh*r*dv]
  float* od;
  float* os;
};
void deltanet_recurrent_launch(const DeltaRecArgs& a, int n_value_heads, int rows, cudaStream_t s, bool pdl);
void sigmoid_gate_q8_launch(const float* o, const float* gate, int64_t gate_stride, int rows, int W, int8_t* oq,
                            float* od, float* os, cudaStream_t s, bool pdl);

// ---- MLA (mla.cu) ----
struct MlaAppendArgs {
  const float* kv_a;          // [R, kv_a_stride]: latent (512) then k_pe (64), pre-norm / pre-RoPE
  int64_t kv_a_stride;
  const float* norm_w;        // [512] kv_a RMSNorm weight
  float eps;
  const int* positions;
  const int* block_tables;
  const int* row_seq;
  int max_blocks, block_size;
  const float* rope;          // [max_pos, 32, 2] (cos, sin) over the 64 rope dims
  __nv_bfloat16* cache;       // [num_blocks, block_size, 576]
};
void mla_kv_append_launch(const MlaAppendArgs& a, int rows, cudaStream_t s, bool pdl);
struct MlaAbsorbArgs {
  const float* q;             // [R, nh, nope + 64]
  const __nv_bfloat16* w_uk;  // [nh, nope, 512]
  const int* positions;
  const float* rope;
  int nh, nope;
  float* q_lat;               // [R, nh, 512]
  float* q_pe;                // [R, nh, 64]
};
void mla_absorb_q_launch(const MlaAbsorbArgs& a, int rows, cudaStream_t s, bool pdl);
struct MlaDecodeArgs {
  const float* q_lat;
  const float* q_pe;
  const __nv_bfloat16* cache;
  const int* block_tables;
  int max_blocks;
  const int* row_seq;
  const int* row_ctx;
  float scale;
  int R, nh, block_size, num_splits, stage_blocks;
  float* o_lat;               // [R, nh, 512]
  int* status;
};
int mla_heads_per_cta(int nh, int rows);  // heads sharing one CTA in mla_decode
void mla_decode_launch(MlaDecodeArgs a, cudaStream_t s, bool pdl);
// Tensor-core variant (mla_flash.cu): 16 heads per CTA on mma.sync, splits and output slices chosen
// to cover the GPU (num_splits / stage_blocks ignored).
void mla_flash_decode_launch(const MlaDecodeArgs& a, cudaStream_t s, bool pdl);
struct MlaOutArgs {
  const float* o_lat;
  const __nv_bfloat16* w_uv;  // [nh, vdim, 512]
  int nh, vdim;
  int8_t* oq;                 // q8 [R, nh * vdim]
  float* od;
  float* os;
};
void mla_out_launch(const MlaOutArgs& a, int rows, cudaStream_t s, bool pdl);

// ---- quantisers (quantize.cu) ----
// n elements (rows * cols, cols a multiple of the block) -> planes p0..p3 of format fmt.
void quantize_launch(int fmt, const float* x, int64_t n, void* p0, void* p1, void* p2, void* p3, cudaStream_t s);
}  // namespace hk
