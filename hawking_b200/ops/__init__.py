"""Python surface of the sm_100a kernels. Each function launches on the current CUDA stream.

The kernel module must be built (``python setup.py build_ext --inplace``); there is no eager
fallback on a GPU machine.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from .._ext import kernels
from .qweight import QWeight, cat_rows  # noqa: F401

PDL = os.environ.get("HK_PDL", "1") == "1"

EPI_STORE, EPI_RESID, EPI_SWIGLU_Q8 = 0, 1, 2


class _LaunchCounter:
    """Counts kernel launches issued through this module (per captured step)."""

    def __init__(self):
        self.n = 0

    def add(self, k: int = 1):
        self.n += k


launches = _LaunchCounter()


class Q8Act:
    """q8 activation blocks for ``rows`` rows of width ``K``: int8 quants + fp32 scale/sum."""

    def __init__(self, rows: int, K: int, device):
        self.K = K
        self.q = torch.zeros(rows, K, dtype=torch.int8, device=device)
        self.d = torch.zeros(rows, K // 32, dtype=torch.float32, device=device)
        self.s = torch.zeros(rows, K // 32, dtype=torch.float32, device=device)

    def view(self, n: int) -> "Q8Act":
        v = Q8Act.__new__(Q8Act)
        v.K, v.q, v.d, v.s = self.K, self.q[:n], self.d[:n], self.s[:n]
        return v

    def dequantize(self) -> torch.Tensor:
        return self.q.float() * self.d.repeat_interleave(32, dim=1)


def rmsnorm_q8(x: torch.Tensor, w: Optional[torch.Tensor], eps: float, out: Q8Act, norm: bool = True,
               y: Optional[torch.Tensor] = None):
    launches.add()
    kernels().rmsnorm_q8(x, w, eps, norm, out.q, out.d, out.s, y, PDL)


def rmsnorm(x, w, eps, yf=None, yb=None):
    launches.add()
    kernels().rmsnorm(x, w, eps, yf, yb, PDL)


def _prefetch_ranges(ws) -> list:
    """Weight planes of ``ws`` (QWeights) as byte ranges for the GEMV's next-kernel L2 prefetch."""
    if not ws or not PREFETCH_NEXT:
        return []
    out = []
    for w in ws:
        if w is None:
            continue
        for p in w.planes:
            if p.is_contiguous() and p.data_ptr() % 16 == 0 and len(out) < 8:
                out.append(p)
    return out


# Decode GEMVs can prefetch the next projection's weights into L2 (see GemvArgs.pf_ptr). Off by
# default: on Llama-3-8B Q4_K bs1 decode it measured 4% slower (410.7 vs 427.8 tok/s); HK_PREFETCH=1
# turns it on for A/B measurements.
PREFETCH_NEXT = os.environ.get("HK_PREFETCH", "0") == "1"


def gemv(w: QWeight, x: Q8Act, y: torch.Tensor, residual: bool = False, bias=None, argmax_slots=None,
         argmax_offset: int = 0, prefetch=None):
    """y[b] = W x[b] (or y += ... with ``residual``). ``argmax_slots`` (int64 [nb, 256], zeroed)
    additionally folds every output into packed greedy keys (row index + ``argmax_offset``);
    ``argmax_finalize`` reads them. ``prefetch``: the weights of the kernel that follows, pulled
    into L2 while this one runs."""
    launches.add()
    kernels().gemv(w.fmt, EPI_RESID if residual else EPI_STORE, w.planes, [], w.N, w.K, x.q, x.d, x.s, y, bias,
                   None, None, None, None, None, -1.0, PDL, argmax_slots, argmax_offset,
                   prefetch=_prefetch_ranges(prefetch))


ARGMAX_SLOTS = 256
EPI_PUSH = 3


def gemv_push(w: QWeight, x: Q8Act, tp, site: int, bias=None, prefetch=None):
    """Row-parallel projection: the partial outputs go to every rank's receive region of ``site``
    (tensor-parallel all-reduce push, see parallel/tp.py)."""
    launches.add()
    kernels().gemv(w.fmt, EPI_PUSH, w.planes, [], w.N, w.K, x.q, x.d, x.s, None, bias, None, None, None, None, None,
                   -1.0, PDL, None, 0, tp.push_recv[site], tp.epoch, prefetch=_prefetch_ranges(prefetch))


def tp_begin(tp):
    launches.add()
    kernels().tp_begin(tp.epoch, PDL)


def tp_allreduce_rmsnorm_q8(tp, site: int, x_in: torch.Tensor, x_out: torch.Tensor, w, eps: float,
                            out: Optional[Q8Act] = None, out_bf16: Optional[torch.Tensor] = None):
    """x_out = x_in + sum of every rank's partials at ``site``; then RMSNorm -> q8 (``out``) or
    bf16 rows (``out_bf16``)."""
    launches.add()
    kernels().tp_allreduce_rmsnorm_q8(x_in, x_out, tp.recv_local(site), tp.rank_stride, tp.world, tp.epoch, w, eps,
                                       out.q if out is not None else None, out.d if out is not None else None,
                                       out.s if out is not None else None, tp.status, PDL, yb=out_bf16,
                                       wait_ns=getattr(tp, "wait_ns", 0))


def tp_argmax(tp, slots: torch.Tensor, rows: int, out: torch.Tensor):
    """Global greedy ids from every rank's fused LM-head keys (vocabulary-parallel)."""
    launches.add()
    if rows > tp.key_rows:
        raise ValueError(f"tp_argmax: {rows} rows exceed the key region ({tp.key_rows})")
    kernels().tp_argmax(slots, rows, tp.key_rows, tp.keys_table, tp.base + tp.keys_off, tp.argmax_uses, tp.rank, out,
                        tp.status, PDL, wait_ns=getattr(tp, "wait_ns", 0))


def argmax_finalize(slots: torch.Tensor, rows: int, out: torch.Tensor):
    """Token ids from the packed greedy keys of a fused GEMV (lowest index on ties); clears them."""
    launches.add()
    kernels().argmax_finalize(slots, rows, out, PDL)


def gemv_swiglu(w_gate: QWeight, w_up: QWeight, x: Q8Act, out: Q8Act, prefetch=None):
    launches.add()
    kernels().gemv(w_gate.fmt, EPI_SWIGLU_Q8, w_gate.planes, w_up.planes, w_gate.N, w_gate.K, x.q, x.d, x.s, None,
                   None, out.q, out.d, out.s, None, None, -1.0, PDL, prefetch=_prefetch_ranges(prefetch))


def gemv_norm(w: QWeight, x: torch.Tensor, norm_w, eps: float, y: torch.Tensor, bias=None):
    """y = W @ q8(rmsnorm(x) * norm_w): the norm and activation quantisation run inside the GEMV
    (each CTA normalises the fp32 rows itself while its weight loads are in flight)."""
    launches.add()
    kernels().gemv(w.fmt, EPI_STORE, w.planes, [], w.N, w.K, None, None, None, y, bias, None, None, None, x, norm_w,
                   eps, PDL)


def gemv_norm_swiglu(w_gate: QWeight, w_up: QWeight, x: torch.Tensor, norm_w, eps: float, out: Q8Act):
    launches.add()
    kernels().gemv(w_gate.fmt, EPI_SWIGLU_Q8, w_gate.planes, w_up.planes, w_gate.N, w_gate.K, None, None, None,
                   None, None, out.q, out.d, out.s, x, norm_w, eps, PDL)


def rope_table(max_pos: int, rot_dim: int, theta: float, freq_factors: Optional[torch.Tensor] = None,
               device="cuda") -> torch.Tensor:
    """[max_pos, rot_dim/2, 2] (cos, sin), computed in float64."""
    half = rot_dim // 2
    i = torch.arange(half, dtype=torch.float64)
    freq = theta ** (-2.0 * i / rot_dim)
    if freq_factors is not None:
        freq = freq / freq_factors.double().cpu()
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * freq[None, :]
    return torch.stack([torch.cos(ang), torch.sin(ang)], -1).float().to(device)


def rope_append(qkv, positions, slots, rope, rot_dim, style, q_out, k_cache, v_cache, nh, nkv, hd, block_size,
                bias=None, q_norm=None, k_norm=None, eps=1e-6, block_tables=None, row_seq=None):
    """RoPE q/k (optional bias and per-head q/k RMSNorm) and append k/v to the paged cache at
    ``slots`` (or, when slots is None, at the slot the block table maps each row's position to)."""
    launches.add()
    kernels().rope_append(qkv, bias, q_norm, k_norm, eps, positions, slots, rope, rot_dim, style, q_out, k_cache,
                          v_cache, nh, nkv, hd, block_size, block_tables, row_seq, PDL)


def tp_p2p_allreduce_rmsnorm(tp, site: int, x_in, x_out, w, eps: float, out=None, out_bf16=None):
    """Tensor-core path all-reduce of a row-parallel site (the rank's GEMM accumulated into
    ``tp.wide_part(site)``): flags raised on every rank, the N partials read over NVLink in rank
    order, x_out = x_in + their sum, RMSNorm (weight ``w``) into q8 blocks or bf16 rows."""
    launches.add()
    kernels().tp_p2p_allreduce_rmsnorm(
        x_in, x_out, tp.wide_parts[site], tp.wide_flags_local(site), tp.wide_flag_ptrs[site], tp.world, tp.rank,
        tp.epoch, w, eps, xq=out.q if out is not None else None, xd=out.d if out is not None else None,
        xs=out.s if out is not None else None, yb=out_bf16, status=tp.status, pdl=PDL,
        wait_ns=getattr(tp, "wait_ns", 0))


def advance(ids, next_ids, positions, row_ctx, rows: int):
    launches.add()
    kernels().advance(ids, next_ids, positions, row_ctx, rows, PDL)


# Decode attention on the tensor cores (attention_tc.cu) where the shape allows it (head_dim 64 / 128,
# GQA group <= 16, block size 16 / 32 / 64, splits 1-8); HK_ATTN_TC=0 selects the CUDA-core kernels.
ATTN_TC = os.environ.get("HK_ATTN_TC", "1") == "1"


def attention_decode(q, k_cache, v_cache, block_tables, row_seq, row_ctx, scale, num_splits, part_o, part_lse,
                     out=None, out_q8: Optional[Q8Act] = None, sinks=None, out_bf16=None, counters=None,
                     cluster: Optional[bool] = None, tc: Optional[bool] = None, status=None):
    """Split-KV paged decode attention.

    Cluster path (default when num_splits is 1, 2, 4, 8 or 16): the splits of one (row, kv head) are a
    thread-block cluster and merge through distributed shared memory; no scratch is touched.
    Scratch path: the per-split partials go to part_o / part_lse with the zero-initialised int32
    ``counters`` [rows * n_kv_heads]; the last split CTA of each (row, kv head) merges them."""
    if cluster is None:
        cluster = num_splits in (1, 2, 4, 8, 16)
    launches.add(1)
    kernels().attention_decode(q, k_cache, v_cache, block_tables, row_seq, row_ctx, scale, num_splits, part_o,
                               part_lse, out, out_q8.q if out_q8 else None, out_q8.d if out_q8 else None,
                               out_q8.s if out_q8 else None, sinks, out_bf16, counters, PDL, cluster,
                               tc=(ATTN_TC if tc is None else tc) and cluster, status=status)


def attention_prefill(q, k_cache, v_cache, block_tables, row_seq, row_ctx, scale, out=None,
                      out_q8: Optional[Q8Act] = None, sinks=None, out_bf16=None):
    """Causal paged attention for many rows on the tensor cores (flash-style, 64-row tiles per
    query head); rows of different sequences may share a launch."""
    launches.add(1)
    kernels().attention_prefill(q, k_cache, v_cache, block_tables, row_seq, row_ctx, scale, out,
                                out_q8.q if out_q8 else None, out_q8.d if out_q8 else None,
                                out_q8.s if out_q8 else None, sinks, out_bf16, PDL)


def argmax(logits: torch.Tensor, out: torch.Tensor):
    launches.add()
    kernels().argmax(logits, out, PDL)


def sample(logits, temperature, top_k, top_p, rep_penalty, recent, uniforms, out):
    launches.add()
    kernels().sample(logits, temperature, top_k, top_p, rep_penalty, recent, uniforms, out, PDL)


def embed(table: QWeight, ids: torch.Tensor, out: torch.Tensor):
    launches.add()
    kernels().embed(table.fmt, table.planes, ids, out, PDL)


# Prefill-sized tensor-core GEMMs (256-token tiles) run as persistent kernels (one CTA per SM,
# epilogue overlapped with the next tile's main loop).
PERSISTENT_GEMM = True


# Decode-batch GEMMs (<= 64 rows, zeroed or accumulated output) with more weight tiles than SMs
# run stream-K: one CTA per SM, each a balanced range of (weight tile, K stage) units, so the
# launch does not end in a partial wave of whole tiles (Llama-3-8B gate/up at 64 rows: 224 tiles,
# 65.8 -> 52.5 us). Fewer tiles keep the one-tile split-K launch, which fills one wave already and
# measured faster there (QKV 15.1 vs 17.4 us). HK_STREAM_K=0 turns it off.
STREAM_K = os.environ.get("HK_STREAM_K", "1") != "0"
SMS = 148


def tc_gemm_stream_k(M: int, N: int) -> bool:
    """Whether a decode-batch tensor-core GEMM over M rows and N weight rows, with a zeroed or
    accumulated output, runs stream-K (then the FFN runs gate/up as a plain GEMM plus the SwiGLU
    kernel instead of the fused epilogue)."""
    return STREAM_K and M <= 64 and (N // 128) > SMS


# Below this many rows tensor-core GEMMs split K (or run stream-K) into a zeroed output.
SPLIT_K_MAX_ROWS = 191


def tc_gemm_bn(M: int) -> int:
    """The engine's token tile for a tensor-core GEMM over M rows (256 from SPLIT_K_MAX_ROWS + 1
    rows up: prefill-sized tiles halve the dequantisation per FLOP and run persistent)."""
    return 32 if M <= 32 else (64 if M <= 64 else (128 if M <= SPLIT_K_MAX_ROWS else 256))


def tc_gemm_overwrites(M: int) -> bool:
    """Whether a tensor-core GEMM over M rows (engine tile choice) writes every output element
    exactly once with a plain store (the persistent path: no split-K), so y needs no zeroing."""
    return PERSISTENT_GEMM and M > SPLIT_K_MAX_ROWS


def tc_gemm(w: QWeight, x: torch.Tensor, y: torch.Tensor, status: torch.Tensor, atomic: bool = False,
            y_zeroed: bool = False, k_splits: int = 0, bn: int = 0):
    """y[M, N] (+)= x[M, K] (bf16) @ w[N, K]^T on the tensor cores (Q4_K weights).

    ``k_splits`` 0 picks a split so the grid covers the GPU; split-K accumulates with fp32 atomics,
    so unless ``atomic`` (residual add) the caller passes a zeroed ``y`` and ``y_zeroed=True``."""
    M = x.shape[0]
    if bn == 0:
        bn = tc_gemm_bn(M)
    persistent = bn == 256 and k_splits in (0, None, 1) and PERSISTENT_GEMM
    stream_k = (not persistent and k_splits in (0, None) and (atomic or y_zeroed) and tc_gemm_stream_k(M, w.N)
                and w.K % 256 == 0)
    if stream_k:
        bn, k_splits = 64, 1
    elif persistent:
        k_splits = 1  # one CTA per SM walks the tiles: the grid is full without split-K
    elif k_splits == 0 or k_splits is None:
        k_splits = kernels().tc_gemm_splits(w.N, M, w.K, bn, 148) if (atomic or y_zeroed) else 1
    launches.add()
    kernels().tc_gemm(w.fmt, w.planes, w.N, w.K, x, y, atomic, y_zeroed, k_splits, bn, status, PDL,
                      persistent=persistent, stream_k=stream_k)


def tc_gemm_swiglu(w_gu: QWeight, x: torch.Tensor, h: torch.Tensor, status: torch.Tensor, bn: int = 0):
    """h[M, F] = silu(x @ gate^T) * (x @ up^T) as bf16, from the fused [gate | up] Q4_K weight
    (2F rows) in one tensor-core launch (the SwiGLU runs in the GEMM epilogue)."""
    M = x.shape[0]
    if bn == 0:
        bn = max(64, tc_gemm_bn(M))
    launches.add()
    kernels().tc_gemm(w_gu.fmt, w_gu.planes, w_gu.N, w_gu.K, x, h, False, False, 1, bn, status, PDL, h=h,
                      persistent=bn == 256 and PERSISTENT_GEMM)


def swiglu_bf16(gu: torch.Tensor, F: int, h: torch.Tensor, clear: bool = True):
    launches.add()
    kernels().swiglu_bf16(gu, F, h, clear, PDL)


# ---- mixture of experts ----
def router_logits(w: torch.Tensor, x: Q8Act, logits: torch.Tensor):
    launches.add()
    kernels().router_logits(w, x.q, x.d, logits, PDL)


def moe_topk(logits, bias, k: int, scoring: int, n_groups: int, topk_groups: int, renorm: bool, scale: float,
             ids, weights):
    launches.add()
    kernels().moe_topk(logits, bias, k, scoring, n_groups, topk_groups, renorm, scale, ids, weights, PDL)


def moe_route(router, x: Q8Act, k: int, scoring: int, bias, n_groups: int, topk_groups: int, renorm: bool,
              scale: float, logits, ids, weights, counts, offsets, sorted_pairs, active, n_active, shared: bool,
              counter, e_lo: int = 0, e_hi: int = 0):
    """Fused decode routing (one launch): router logits, top-k, the pairs sorted by expert (plus
    the shared expert as expert E when ``shared``) and the list of experts with pairs; under
    expert parallelism only experts in [e_lo, e_hi) enter the active list."""
    launches.add()
    kernels().moe_route(router, x.q, x.d, k, scoring, bias, n_groups, topk_groups, renorm, scale, logits, ids,
                        weights, counts, offsets, sorted_pairs, active, n_active, shared, counter, PDL,
                        e_lo=e_lo, e_hi=e_hi)


def moe_align(ids, E: int, x: Q8Act, counts, offsets, sorted_pairs, gathered: Optional[Q8Act], shared: bool = False):
    """Counting sort of the (token, expert) pairs by expert plus the gather of their q8 rows
    (``gathered`` None: the sort only); ``shared`` appends expert E (a shared expert) with one pair
    per token after the routed ones."""
    launches.add()
    if gathered is None:
        e8, ef = torch.empty(0, dtype=torch.int8, device=ids.device), torch.empty(0, device=ids.device)
        kernels().moe_align(ids, E, x.q, x.d, x.s, counts, offsets, sorted_pairs, e8, ef, ef, PDL, shared)
        return
    kernels().moe_align(ids, E, x.q, x.d, x.s, counts, offsets, sorted_pairs, gathered.q, gathered.d, gathered.s, PDL,
                        shared)


def moe_gemv_swiglu(w_gate: QWeight, w_up: QWeight, N: int, E: int, k: int, counts, offsets, sorted_pairs,
                    x: Q8Act, out: Q8Act):
    launches.add()
    kernels().moe_gemv(w_gate.fmt, 0, w_gate.planes, w_up.planes, N, w_gate.K, E, k, counts, offsets, sorted_pairs,
                       x.q, x.d, x.s, out.q, out.d, out.s, None, None, PDL)


def moe_gemv_down(w_down: QWeight, N: int, E: int, k: int, counts, offsets, sorted_pairs, h: Q8Act,
                  y: torch.Tensor, route_w: torch.Tensor):
    launches.add()
    kernels().moe_gemv(w_down.fmt, 1, w_down.planes, [], N, w_down.K, E, k, counts, offsets, sorted_pairs,
                       h.q, h.d, h.s, None, None, None, y, route_w, PDL)
