"""In-box library baseline: the Llama-3-8B decode/prefill step in plain PyTorch (cuBLAS GEMMs,
PyTorch SDPA attention, NCCL all-reduce for tensor parallelism), for comparing the framework's
own kernels against what the stock libraries give on the same box, model and workload.

The baseline cannot read GGUF Q4_K (no PyTorch kernel for it), so it holds the same architecture
with bf16 weights (random-init N(0, 0.02)), i.e. it streams about 3.6x the weight bytes of the
Q4_K model. Tensor parallelism is the Megatron split: QKV / gate-up column-parallel, O / down
row-parallel with an NCCL all-reduce each, vocabulary-parallel LM head (all-gather of the logits).
The KV cache is a contiguous bf16 [batch, kv_heads, capacity, head_dim] per layer; a decode step
attends over the whole capacity with an additive mask (static shapes, so the step is captured in
one CUDA graph, NCCL collectives included). Prefill runs eagerly with causal SDPA.

Used by ``bench.py --impl torch``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.nn.functional as F


@dataclass
class BaselineLayer:
    attn_norm: torch.Tensor
    wqkv: torch.Tensor   # [(lnh + 2 lnkv) hd, H]
    wo: torch.Tensor     # [H, lnh hd]
    ffn_norm: torch.Tensor
    wgu: torch.Tensor    # [2 lF, H]
    wdown: torch.Tensor  # [H, lF]


class TorchLlamaTP:
    """One rank's shard of a Llama-family decoder in plain PyTorch (bf16)."""

    def __init__(self, cfg, rank: int, world: int, device, batch: int, capacity: int, group=None, seed: int = 0):
        self.cfg, self.rank, self.world, self.dev, self.group = cfg, rank, world, torch.device(device), group
        H, hd = cfg.hidden, cfg.head_dim
        self.lnh, self.lnkv, self.lF = cfg.n_heads // world, cfg.n_kv_heads // world, cfg.ffn // world
        self.lV = cfg.vocab // world
        g = torch.Generator(device=self.dev).manual_seed(seed * 131 + rank)
        std = 0.02

        def W(n, k):
            return (torch.randn(n, k, generator=g, device=self.dev) * std).bfloat16()

        self.layers: List[BaselineLayer] = []
        for _ in range(cfg.layers):
            self.layers.append(BaselineLayer(torch.ones(H, device=self.dev, dtype=torch.bfloat16),
                                             W((self.lnh + 2 * self.lnkv) * hd, H), W(H, self.lnh * hd),
                                             torch.ones(H, device=self.dev, dtype=torch.bfloat16),
                                             W(2 * self.lF, H), W(H, self.lF)))
        g0 = torch.Generator(device=self.dev).manual_seed(seed * 131 + 99991)  # replicated embedding
        self.embed = (torch.randn(cfg.vocab, H, generator=g0, device=self.dev) * std).bfloat16()
        self.out_norm = torch.ones(H, device=self.dev, dtype=torch.bfloat16)
        self.lm_head = W(self.lV, H)
        self.batch, self.cap = batch, capacity
        self.k = [torch.zeros(batch, self.lnkv, capacity, hd, dtype=torch.bfloat16, device=self.dev)
                  for _ in range(cfg.layers)]
        self.v = [torch.zeros_like(t) for t in self.k]
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, device=self.dev).float() / hd))
        ang = torch.arange(capacity, device=self.dev).float()[:, None] * inv[None]
        self.cos, self.sin = ang.cos(), ang.sin()  # [cap, hd/2]
        # decode-step inputs (static for graph capture)
        self.ids = torch.zeros(batch, dtype=torch.long, device=self.dev)
        self.pos = torch.zeros(batch, dtype=torch.long, device=self.dev)
        self.next_ids = torch.zeros(batch, dtype=torch.long, device=self.dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    @property
    def nbytes(self) -> int:
        n = sum(t.numel() * 2 for L in self.layers for t in (L.wqkv, L.wo, L.wgu, L.wdown))
        return n + self.lm_head.numel() * 2

    def _rms(self, x, w):
        # fused RMSNorm where PyTorch has one (fp32 statistics inside)
        if hasattr(F, "rms_norm"):
            return F.rms_norm(x, (x.shape[-1],), w, self.cfg.eps)
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg.eps)).to(x.dtype) * w

    def _rope(self, t, pos):
        """neox-style rotation of t [..., T, hd] at positions pos [..., T]."""
        c, s = self.cos[pos].unsqueeze(-3), self.sin[pos].unsqueeze(-3)  # [B, 1, T, hd/2]
        h = t.shape[-1] // 2
        a, b = t[..., :h].float(), t[..., h:].float()
        return torch.cat([a * c - b * s, a * s + b * c], -1).to(t.dtype)

    def _allreduce(self, t):
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, group=self.group)
        return t

    def _layers(self, x, pos, mask, causal: bool, write):
        """x [B, T, H] bf16; pos [B, T]; write(l, k, v) stores the new keys/values; returns x."""
        cfg, hd = self.cfg, self.cfg.head_dim
        B, T, _ = x.shape
        for l, L in enumerate(self.layers):
            h = self._rms(x, L.attn_norm)
            qkv = h @ L.wqkv.t()
            q, k, v = qkv.split([self.lnh * hd, self.lnkv * hd, self.lnkv * hd], -1)
            q = self._rope(q.view(B, T, self.lnh, hd).transpose(1, 2), pos)
            k = self._rope(k.view(B, T, self.lnkv, hd).transpose(1, 2), pos)
            v = v.view(B, T, self.lnkv, hd).transpose(1, 2)
            kk, vv = write(l, k, v)
            if causal:  # prefill: fused SDPA (flash) with grouped heads
                o = F.scaled_dot_product_attention(q, kk, vv, is_causal=True, enable_gqa=True,
                                                   scale=1.0 / math.sqrt(hd))
            else:  # decode (T = 1): SDPA over the masked cache (grouped heads)
                o = F.scaled_dot_product_attention(q, kk, vv, attn_mask=mask, enable_gqa=True,
                                                   scale=1.0 / math.sqrt(hd))
            o = o.transpose(1, 2).reshape(B, T, self.lnh * hd)
            x = x + self._allreduce(o @ L.wo.t())
            h = self._rms(x, L.ffn_norm)
            gu = h @ L.wgu.t()
            a = F.silu(gu[..., :self.lF]) * gu[..., self.lF:]
            x = x + self._allreduce(a @ L.wdown.t())
        return x

    def _greedy(self, h):
        """Vocabulary-parallel argmax of h [B, H] -> global ids [B]."""
        logits = (self._rms(h, self.out_norm) @ self.lm_head.t()).float()
        if self.world == 1:
            return logits.argmax(-1)
        import torch.distributed as dist
        parts = [torch.empty_like(logits) for _ in range(self.world)]
        dist.all_gather(parts, logits, group=self.group)
        return torch.cat(parts, -1).argmax(-1)

    # ---- prefill (eager) ----
    def prefill(self, tokens: torch.Tensor) -> torch.Tensor:
        """tokens [B, T] (device, long) at positions 0..T-1; fills the cache; returns next ids [B]."""
        B, T = tokens.shape
        x = self.embed[tokens]
        pos = torch.arange(T, device=self.dev).expand(B, T)

        def write(l, k, v):
            self.k[l][:B, :, :T] = k
            self.v[l][:B, :, :T] = v
            return k, v

        x = self._layers(x, pos, None, True, write)
        return self._greedy(x[:, -1])

    # ---- decode (CUDA graph) ----
    def _decode_eager(self):
        B = self.batch
        x = self.embed[self.ids].unsqueeze(1)
        pos = self.pos.unsqueeze(1)
        ar = torch.arange(self.cap, device=self.dev)
        mask = torch.where(ar[None, :] <= self.pos[:, None], 0.0, float("-inf")).to(torch.bfloat16)
        mask = mask[:, None, None, :]  # [B, 1, 1, cap] additive
        bidx = torch.arange(B, device=self.dev)

        def write(l, k, v):
            self.k[l][bidx, :, self.pos] = k[:, :, 0]
            self.v[l][bidx, :, self.pos] = v[:, :, 0]
            return self.k[l], self.v[l]

        x = self._layers(x, pos, mask, False, write)
        self.next_ids.copy_(self._greedy(x[:, 0]))
        self.ids.copy_(self.next_ids)
        self.pos.add_(1)

    def decode_step(self):
        if self.graph is None:
            s = torch.cuda.Stream(self.dev)
            s.wait_stream(torch.cuda.current_stream(self.dev))
            saved = (self.ids.clone(), self.pos.clone())
            with torch.cuda.stream(s):
                for _ in range(2):
                    self._decode_eager()
            torch.cuda.current_stream(self.dev).wait_stream(s)
            self.ids.copy_(saved[0])
            self.pos.copy_(saved[1])
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._decode_eager()
        self.graph.replay()

    def release(self):
        self.graph = None
