"""Tensor parallelism for the Llama family on the GPUs of one node.

Sharding (rank r of N): Q/K/V heads split by head (column-parallel; every rank keeps its own KV
heads in its own paged cache), gate/up split by FFN row, attention output and FFN down split along
K (row-parallel: each rank produces a partial hidden vector), LM head split by vocabulary row, the
embedding table replicated. Decode (GEMV path) all-reduces with the fused push kernels of
``csrc/kernels/tp.cu``: the row-parallel GEMV stores its partial rows into every rank's receive
region over NVLink and the next RMSNorm sums them; greedy sampling reduces per-rank (logit, index)
keys the same way. Prefill (tensor-core path) all-reduces its partials with NCCL.

``TPComm`` owns the shared buffers: one CUDA-IPC region per rank (receive regions of every
all-reduce site and the argmax key region, all as flagged 8-byte words), mapped into every other
rank's process. No NVLink multicast object is created.

Parity: the reference has no tensor parallelism (one Apple GPU); the sharding plan follows the
north-star requirement of column-parallel QKV/gate/up and row-parallel O/down with a vocabulary-
parallel LM head.
"""
from __future__ import annotations

from typing import List, Optional

import os

import torch
import torch.distributed as dist

from .._ext import kernels
from ..formats.ggml import type_id
from ..models.config import ModelConfig
from ..ops.qweight import QWeight


def local_config(cfg: ModelConfig, world: int) -> ModelConfig:
    """This rank's shard of the config: heads and dense FFN divided; MoE experts stay global (the
    router scores all of them; each rank holds E / world of them, see MoEFFN.shard), the shared
    expert's FFN divided."""
    if cfg.n_heads % world or cfg.n_kv_heads % world or cfg.ffn % (32 * world):
        raise ValueError(f"heads {cfg.n_heads}/{cfg.n_kv_heads} and ffn {cfg.ffn} must split over {world} ranks")
    if cfg.vocab % world:
        raise ValueError(f"vocab {cfg.vocab} must split over {world} ranks")
    if cfg.n_experts and cfg.n_experts % world:
        raise ValueError(f"{cfg.n_experts} experts must split over {world} ranks")
    return cfg.with_(n_heads=cfg.n_heads // world, n_kv_heads=cfg.n_kv_heads // world, ffn=cfg.ffn // world,
                     shared_ffn=cfg.shared_ffn // world)


def cols(w: QWeight, k0: int, k1: int) -> QWeight:
    """Columns [k0, k1) of an [N, K] block-format weight (whole blocks)."""
    from ..formats.ggml import LAYOUTS
    from ..ops.qweight import _PLANES
    be = LAYOUTS[w.fmt].block_elems
    if k0 % be or k1 % be:
        raise ValueError("column slice must align to the format's blocks")
    nb = w.K // be
    planes = []
    for p in w.planes:
        pb = p.shape[1] // nb
        planes.append(p.reshape(w.N, nb, pb)[:, k0 // be:k1 // be].reshape(w.N, -1).contiguous())
    return QWeight(w.fmt, w.N, k1 - k0, planes)


def shard_llama_weights(w, cfg: ModelConfig, rank: int, world: int):
    """Rank ``rank``'s shard of full LlamaWeights (dense FFN layers)."""
    from ..models.llama import LayerWeights, LlamaWeights
    from ..ops.qweight import cat_rows
    hd, nh, nkv, F = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.ffn
    lnh, lnkv, lF = nh // world, nkv // world, F // world
    layers = []
    for lw in w.layers:
        qkv = lw.wqkv[0] if len(lw.wqkv) == 1 else cat_rows(lw.wqkv)
        q = qkv.rows(rank * lnh * hd, lnh * hd)
        k = qkv.rows(nh * hd + rank * lnkv * hd, lnkv * hd)
        v = qkv.rows((nh + nkv) * hd + rank * lnkv * hd, lnkv * hd)
        nl = LayerWeights(attn_norm=lw.attn_norm, wqkv=[cat_rows([q, k, v])],
                          wo=cols(lw.wo, rank * lnh * hd, (rank + 1) * lnh * hd), ffn_norm=lw.ffn_norm)
        if lw.qkv_bias is not None:
            b = lw.qkv_bias
            nl.qkv_bias = torch.cat([b[rank * lnh * hd:(rank + 1) * lnh * hd],
                                     b[nh * hd + rank * lnkv * hd:nh * hd + (rank + 1) * lnkv * hd],
                                     b[(nh + nkv) * hd + rank * lnkv * hd:(nh + nkv) * hd + (rank + 1) * lnkv * hd]])
        nl.q_norm, nl.k_norm = lw.q_norm, lw.k_norm
        if lw.moe is not None:  # expert parallel: whole experts per rank, router replicated
            nl.moe = lw.moe.shard(rank, world)
            layers.append(nl)
            continue
        gate, up = lw.w_gate.rows(rank * lF, lF), lw.w_up.rows(rank * lF, lF)
        nl.w_gu = cat_rows([gate, up])
        nl.w_gate, nl.w_up = nl.w_gu.rows(0, lF), nl.w_gu.rows(lF, lF)
        nl.w_down = cols(lw.w_down, rank * lF, (rank + 1) * lF)
        layers.append(nl)
    V = w.lm_head.N
    head = w.lm_head.rows(rank * (V // world), V // world)
    head = QWeight(head.fmt, head.N, head.K, [p.contiguous() for p in head.planes])
    return LlamaWeights(embed=w.embed, out_norm=w.out_norm, lm_head=head, layers=layers, rope_freqs=w.rope_freqs)


def random_llama_weights_tp(cfg: ModelConfig, rank: int, world: int, device, seed: int = 0, std: float = 0.02):
    """Random-init weights generated directly in rank ``rank``'s shard shapes (benchmarks)."""
    from ..models.llama import LayerWeights, LlamaWeights
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1009 + rank)
    fmt = type_id(cfg.weight_type)
    efmt = type_id(cfg.embed_type or cfg.weight_type)
    H, hd = cfg.hidden, cfg.head_dim
    lnh, lnkv, lF = cfg.n_heads // world, cfg.n_kv_heads // world, cfg.ffn // world

    def W(N, K, f=fmt):
        return QWeight.random(f, N, K, std, g, device)

    g_rep = torch.Generator(device=device)
    g_rep.manual_seed(seed * 1009 + 5555)  # replicated MoE routers: identical on every rank
    layers = []
    for l in range(cfg.layers):
        lw = LayerWeights(attn_norm=torch.ones(H, device=device), wqkv=[W((lnh + 2 * lnkv) * hd, H)],
                          wo=W(H, lnh * hd), ffn_norm=torch.ones(H, device=device))
        if cfg.layer_is_moe(l):
            from ..models.moe import MoEFFN
            lw.moe = MoEFFN.random_shard(cfg, rank, world, device, g, g_rep, std)
            layers.append(lw)
            continue
        gu = W(2 * lF, H)
        lw.w_gu, lw.w_gate, lw.w_up = gu, gu.rows(0, lF), gu.rows(lF, lF)
        lw.w_down = W(H, lF)
        layers.append(lw)
    g2 = torch.Generator(device=device)
    g2.manual_seed(seed * 1009 + 7777)  # the replicated embedding is identical on every rank
    embed = QWeight.random(efmt, cfg.vocab, H, std, g2, device)
    head = W(cfg.vocab // world, H)
    torch.cuda.synchronize(device)
    return LlamaWeights(embed=embed, out_norm=torch.ones(H, device=device), lm_head=head, layers=layers)


class TPComm:
    """Shared buffers and pointer tables of the fused collectives for one rank."""

    def __init__(self, rank: int, world: int, n_sites: int, max_rows: int, width: int, device,
                 group: Optional[dist.ProcessGroup] = None, key_rows: int = 64, wide_rows: int = 64):
        """``max_rows``: rows of the push all-reduce (GEMV path); ``key_rows``: rows of the greedy
        key exchange (any decode batch)."""
        K = kernels()
        self.rank, self.world, self.n_sites = rank, world, n_sites
        self.max_rows, self.width, self.key_rows = max_rows, width, key_rows
        self.dev = torch.device(device)
        self.group = group
        # flagged 8-byte words: value | flag << 32 (see the kernels)
        self.rank_stride = max_rows * width                       # words per source rank
        self.site_words = world * self.rank_stride
        recv_bytes = n_sites * self.site_words * 8
        self.keys_off = recv_bytes
        keys_bytes = world * key_rows * 2 * 8                     # two flagged words per key
        total = (self.keys_off + keys_bytes + 255) // 256 * 256
        with torch.cuda.device(self.dev):
            self.base = K.ipc_malloc(total)
            handle = bytes(K.ipc_handle(self.base))
        handles: List[bytes] = [handle]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, handle, group=group)
        self.ptrs = []
        with torch.cuda.device(self.dev):
            for p, h in enumerate(handles):
                self.ptrs.append(self.base if p == rank else K.ipc_open(h))
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.dev)       # forwards on the push path
        self.argmax_uses = torch.zeros(1, dtype=torch.int32, device=self.dev)  # greedy rounds
        self.status = torch.zeros(1, dtype=torch.int32, device=self.dev)
        # bound of every peer wait in the fused collectives, in ns (0: the kernels' default, 1 s)
        self.wait_ns = int(os.environ.get("HK_TP_WAIT_NS", "0"))

        def table(vals):
            return torch.tensor(vals, dtype=torch.int64, device=self.dev)

        # per site: where MY partial goes in every rank's region
        self.push_recv = [table([self.ptrs[p] + 8 * (s * self.site_words + rank * self.rank_stride)
                                 for p in range(world)]) for s in range(n_sites)]
        self.keys_table = table([self.ptrs[p] + self.keys_off for p in range(world)])
        # tensor-core path sites (up to wide_rows rows): per site an fp32 partial [wide_rows, width]
        # that the rank's GEMM accumulates into, read by every rank over NVLink, and per site the
        # ranks' ready flags [world] (uint32, written by the peers)
        self.wide_rows = wide_rows if world > 1 else 0
        self.wide_base, self.wide_ptrs = 0, []
        if self.wide_rows:
            part_bytes = n_sites * wide_rows * width * 4
            self.wide_flags_off = part_bytes
            wtotal = (part_bytes + n_sites * world * 4 + 255) // 256 * 256
            with torch.cuda.device(self.dev):
                self.wide_base = K.ipc_malloc(wtotal)
                torch.cuda.synchronize(self.dev)
                K.wrap_f32(self.wide_base, wtotal // 4, self.dev.index or 0).zero_()
                torch.cuda.synchronize(self.dev)
                wh = bytes(K.ipc_handle(self.wide_base))
            whs = [None] * world
            dist.all_gather_object(whs, wh, group=group)
            with torch.cuda.device(self.dev):
                self.wide_ptrs = [self.wide_base if p == rank else K.ipc_open(h) for p, h in enumerate(whs)]
            site_floats = wide_rows * width
            self.wide_parts = [table([self.wide_ptrs[p] + 4 * s * site_floats for p in range(world)])
                               for s in range(n_sites)]
            self.wide_flag_ptrs = [table([self.wide_ptrs[p] + self.wide_flags_off + 4 * s * world
                                          for p in range(world)]) for s in range(n_sites)]
            self._wide_local = K.wrap_f32(self.wide_base, n_sites * site_floats, self.dev.index or 0).view(
                n_sites, wide_rows, width)
        self.closed = False

    def wide_part(self, site: int) -> torch.Tensor:
        """This rank's partial buffer of a tensor-core site, [wide_rows, width] fp32."""
        return self._wide_local[site]

    def wide_flags_local(self, site: int) -> int:
        return self.wide_base + self.wide_flags_off + 4 * site * self.world

    # local addresses
    def recv_local(self, site: int) -> int:
        return self.base + 8 * site * self.site_words

    @property
    def argmax_site(self) -> int:
        return self.n_sites

    def check(self):
        st = int(self.status.item())
        if st:
            raise RuntimeError(f"tensor-parallel collective reported device error {st} (peer timeout)")

    def close(self):
        if self.closed:
            return
        torch.cuda.synchronize(self.dev)
        if self.world > 1:
            dist.barrier(group=self.group)
        K = kernels()
        with torch.cuda.device(self.dev):
            for p, ptr in enumerate(self.ptrs):
                if p != self.rank:
                    K.ipc_close(ptr)
            for p, ptr in enumerate(self.wide_ptrs):
                if p != self.rank:
                    K.ipc_close(ptr)
        if self.world > 1:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.dev):
            K.ipc_free(self.base)
            if self.wide_base:
                self._wide_local = None
                K.ipc_free(self.wide_base)
        self.closed = True


def gather_vocab_logits(tp: "TPComm", local: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """Vocabulary-parallel logits [rows, V / world] of every rank -> the full logits [rows, V] on
    every rank (rank r's slice holds vocabulary ids r * V/world ...), so that each rank runs the same
    sampler on the same distribution with the same uniforms and draws the same token. One NCCL
    all-gather plus a transposing copy. Parity: crates/hawking-core/src/sample.rs:39-98 (the sampler
    runs once over the whole vocabulary)."""
    rows, vs = local.shape
    buf = torch.empty(tp.world * rows * vs, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, local.contiguous().view(-1), group=tp.group)
    out[:rows].view(rows, tp.world, vs).copy_(buf.view(tp.world, rows, vs).transpose(0, 1))
    return out[:rows]
