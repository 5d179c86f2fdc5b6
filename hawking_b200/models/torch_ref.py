"""Plain-PyTorch fp32 reference forwards (no custom kernels).

Used as the numerics oracle for the GPU model path (and cross-checked against the C++ CPU
reference). Token-serial, contiguous KV, weights dequantised to fp32 once.
Parity: the same math as crates/hawking-core/src/model/llama.rs:2779 (forward_token) and
crates/hawking-core/src/moe.rs:24-117.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch

from ..formats.gguf import GgufModel
from .config import ModelConfig


def rope_ref(x: torch.Tensor, pos: torch.Tensor, theta: float, rot_dim: int, style: int,
             freq_factors: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x [..., T, H, D], pos [T]. style 0 = adjacent pairs, 1 = neox halves."""
    half = rot_dim // 2
    i = torch.arange(half, dtype=torch.float64, device=x.device)
    freq = theta ** (-2.0 * i / rot_dim)
    if freq_factors is not None:
        freq = freq / freq_factors.double()
    ang = pos.double()[:, None] * freq[None, :]                     # [T, half]
    c = torch.cos(ang).float()[:, None, :]
    s = torch.sin(ang).float()[:, None, :]
    out = x.clone()
    if style == 0:
        a, b = x[..., 0:rot_dim:2], x[..., 1:rot_dim:2]
        out[..., 0:rot_dim:2] = a * c - b * s
        out[..., 1:rot_dim:2] = a * s + b * c
    else:
        a, b = x[..., :half], x[..., half:rot_dim]
        out[..., :half] = a * c - b * s
        out[..., half:rot_dim] = a * s + b * c
    return out


def rmsnorm_ref(x: torch.Tensor, w: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    r = torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + eps)
    y = x.float() * r
    return y * w.float() if w is not None else y


# GGUF architectures of the reference's other families that this framework does not build: refused
# at load with the reason instead of failing on a missing attention key
NOT_BUILT_ARCHS = {
    "rwkv6": "RWKV-6 (state-space decoder) is not built in this framework",
    "rwkv7": "RWKV-7 (state-space decoder, WKV-7 recurrence) is not built in this framework",
    "mamba": "Mamba (state-space decoder) is not built in this framework",
}


def config_from_gguf(m: GgufModel) -> ModelConfig:
    a = m.architecture
    if a in NOT_BUILT_ARCHS:
        raise ValueError(f"GGUF architecture {a!r}: {NOT_BUILT_ARCHS[a]}")
    if a == "deepseek2":
        from .deepseek_gguf import deepseek_config_from_gguf
        return deepseek_config_from_gguf(m)
    g = lambda k, d=None: m.get(f"{a}.{k}", d)  # noqa: E731
    hidden = int(g("embedding_length"))
    nh = int(g("attention.head_count"))
    hd = int(g("attention.key_length", hidden // nh))
    E = int(g("expert_count", 0) or 0)
    cfg = ModelConfig(
        arch=("mixtral" if (a == "llama" and E) else a), vocab=int(g("vocab_size", m.tensors["token_embd.weight"].dims[1])),
        hidden=hidden, layers=int(g("block_count")), n_heads=nh,
        n_kv_heads=int(g("attention.head_count_kv", nh)), head_dim=hd, ffn=int(g("feed_forward_length", 0) or 0),
        eps=float(g("attention.layer_norm_rms_epsilon", 1e-5)), rope_theta=float(g("rope.freq_base", 10000.0)),
        rope_style=0 if a in ("llama", "mistral") else 1, rot_dim=int(g("rope.dimension_count", hd)),
        qkv_bias=m.has("blk.0.attn_q.bias"), qk_norm=m.has("blk.0.attn_q_norm.weight"),
        tie_embeddings=not m.has("output.weight"), n_experts=E, top_k=int(g("expert_used_count", 0) or 0),
        expert_ffn=int(g("expert_feed_forward_length", g("feed_forward_length", 0)) or 0),
        shared_ffn=int(g("expert_shared_feed_forward_length", 0) or 0),
        shared_gate=m.has("blk.0.ffn_gate_inp_shexp.weight"), norm_topk=(a != "qwen2moe"),
        weight_type=m.tensors["blk.0.attn_q.weight"].type_name,
        max_ctx=int(g("context_length", 4096)),
    )
    if cfg.shared_ffn:
        cfg.n_shared_experts = 1
    return cfg


class TorchRefLlama:
    """fp32 token-serial forward of the llama family from a GGUF file."""

    def __init__(self, path: str, device: str = "cpu", max_ctx: int = 2048):
        self.m = GgufModel(path)
        self.cfg = config_from_gguf(self.m)
        self.dev = device
        self.max_ctx = max_ctx
        self.w: Dict[str, torch.Tensor] = {}
        for name in self.m.tensors:
            self.w[name] = torch.from_numpy(self.m.dequantize(name)).to(device)
        self.ff = self.w.get("rope_freqs.weight")
        c = self.cfg
        self.k = torch.zeros(c.layers, max_ctx, c.n_kv_heads, c.head_dim, device=device)
        self.v = torch.zeros_like(self.k)
        self.n_past = 0

    def reset(self):
        self.n_past = 0

    def _ffn(self, l: int, x: torch.Tensor) -> torch.Tensor:
        p = f"blk.{l}."
        W = self.w
        c = self.cfg
        if not c.is_moe:
            return W[p + "ffn_down.weight"] @ (torch.nn.functional.silu(W[p + "ffn_gate.weight"] @ x) * (W[p + "ffn_up.weight"] @ x))
        logits = W[p + "ffn_gate_inp.weight"] @ x
        probs = torch.softmax(logits.double(), -1).float()
        order = sorted(range(c.n_experts), key=lambda e: (-probs[e].item(), e))[: c.top_k]
        ws = probs[order]
        if c.norm_topk:
            ws = ws / ws.sum()
        out = torch.zeros_like(x)
        for e, wgt in zip(order, ws):
            g = W[p + "ffn_gate_exps.weight"][e] @ x
            u = W[p + "ffn_up_exps.weight"][e] @ x
            out = out + wgt * (W[p + "ffn_down_exps.weight"][e] @ (torch.nn.functional.silu(g) * u))
        if p + "ffn_gate_shexp.weight" in W:
            h = torch.nn.functional.silu(W[p + "ffn_gate_shexp.weight"] @ x) * (W[p + "ffn_up_shexp.weight"] @ x)
            s = W[p + "ffn_down_shexp.weight"] @ h
            if p + "ffn_gate_inp_shexp.weight" in W:
                s = s * torch.sigmoid(W[p + "ffn_gate_inp_shexp.weight"] @ x)
            out = out + s
        return out

    @torch.no_grad()
    def forward(self, token: int, pos: int) -> torch.Tensor:
        c, W = self.cfg, self.w
        x = W["token_embd.weight"][token].clone()
        P = torch.tensor([pos], device=self.dev)
        for l in range(c.layers):
            p = f"blk.{l}."
            xn = rmsnorm_ref(x, W[p + "attn_norm.weight"], c.eps)
            q = W[p + "attn_q.weight"] @ xn
            k = W[p + "attn_k.weight"] @ xn
            v = W[p + "attn_v.weight"] @ xn
            if p + "attn_q.bias" in W:
                q, k, v = q + W[p + "attn_q.bias"], k + W[p + "attn_k.bias"], v + W[p + "attn_v.bias"]
            q = q.view(1, c.n_heads, c.head_dim)
            k = k.view(1, c.n_kv_heads, c.head_dim)
            if c.qk_norm:
                q = rmsnorm_ref(q, W[p + "attn_q_norm.weight"], c.eps)
                k = rmsnorm_ref(k, W[p + "attn_k_norm.weight"], c.eps)
            q = rope_ref(q, P, c.rope_theta, c.rope_dim, c.rope_style, self.ff)[0]
            k = rope_ref(k, P, c.rope_theta, c.rope_dim, c.rope_style, self.ff)[0]
            self.k[l, pos] = k
            self.v[l, pos] = v.view(c.n_kv_heads, c.head_dim)
            K = self.k[l, : pos + 1].repeat_interleave(c.n_heads // c.n_kv_heads, dim=1)  # [T, nh, hd]
            V = self.v[l, : pos + 1].repeat_interleave(c.n_heads // c.n_kv_heads, dim=1)
            s = torch.einsum("hd,thd->ht", q, K) / math.sqrt(c.head_dim)
            a = torch.einsum("ht,thd->hd", torch.softmax(s, -1), V).reshape(-1)
            x = x + W[p + "attn_output.weight"] @ a
            x = x + self._ffn(l, rmsnorm_ref(x, W[p + "ffn_norm.weight"], c.eps))
        xn = rmsnorm_ref(x, W["output_norm.weight"], c.eps)
        out = W["output.weight"] if "output.weight" in W else W["token_embd.weight"]
        self.n_past = pos + 1
        return out @ xn

    def generate_greedy(self, prompt: List[int], n_new: int) -> List[int]:
        self.reset()
        for i, t in enumerate(prompt):
            logits = self.forward(t, i)
        out, pos = [], len(prompt)
        for i in range(n_new):
            t = int(torch.argmax(logits).item())
            out.append(t)
            if i + 1 < n_new:
                logits = self.forward(t, pos)
                pos += 1
        return out
