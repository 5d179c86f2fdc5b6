// Public C declaration of the allocation-free attention entry point (defined in attention.cu).
//
// No counterpart in the reference: its Metal engine exposes no C entry points of this kind.
//
// Callers that cannot allocate device memory use this entry point: an engine embedded in a host
// process whose own allocator already owns the GPU's memory, or a latency-critical decode loop
// where cudaMalloc / cudaFree (which may synchronise the device) are not allowed. It runs the same
// split-KV paged decode attention as the regular launcher, with its scratch (per-split partial
// outputs, their log-sum-exps, the split counters) in fixed-size arrays inside the library. The
// caller passes every input and output.
//
// Limits: rows * n_heads * num_splits * head_dim <= 2^20 partial floats, rows * n_heads *
// num_splits <= 2^14 log-sum-exps, rows * n_kv_heads <= 4096 counters (about 4.1 MiB held on every
// GPU that loads the library, until the process exits); larger requests return
// HK_NOALLOC_TOO_LARGE. block_size must be at least 8; q, k_cache, v_cache and out must be
// 16-byte aligned; `stream` must belong to the current device.
//
// The first call on a device looks up the arrays' device addresses with that device current; make
// it before any stream capture. All calls share the arrays: calls that may overlap on the GPU
// (different streams, or host threads with no ordering between their streams) race on the
// scratch. The split counters are cleared at the start of every call.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

enum HkNoAllocStatus {
  HK_NOALLOC_OK = 0,
  HK_NOALLOC_BAD_ARG = 1,
  HK_NOALLOC_TOO_LARGE = 2,
  HK_NOALLOC_CUDA_ERROR = 3
};

//   q            [rows, n_heads, head_dim] fp32 (already RoPE'd)
//   k_cache      [num_blocks, n_kv_heads, block_size, head_dim] bf16 (v_cache alike)
//   block_tables [*, max_blocks] int32; row_seq / row_ctx [rows] int32
//   out          [rows, n_heads * head_dim] fp32
//   stream       cudaStream_t to launch on (null = legacy default stream)
// Returns an HkNoAllocStatus; hk_attention_decode_noalloc_error() explains a failure.
int hk_attention_decode_noalloc(const float* q, const void* k_cache, const void* v_cache, const int* block_tables,
                                int max_blocks, const int* row_seq, const int* row_ctx, float scale, int rows,
                                int n_heads, int n_kv_heads, int head_dim, int block_size, int num_splits, float* out,
                                void* stream);

// Message of the last failing call on this host thread ("" after a success).
const char* hk_attention_decode_noalloc_error(void);

#ifdef __cplusplus
}
#endif
