"""Qwen3-Next-style weights as a `.gravity` artifact: writer, reader and architecture config.

An artifact directory holds shards (``model-NNNNN.gravity``, ``GRAVITY\\0`` container with a
canonical-JSON header and a sha256 per payload) and ``model.gravity.index.json`` (weight map,
shard sha256s, and the architecture: the model config as JSON). Tensors:

* mixed projections and experts: HGRAVB01 (binary) / HGRAVU01 (uniform 2 / 4 bits) envelopes,
  written straight from the device planes (fp16 group scales, LSB-first codes) with no
  re-quantisation, and mapped back onto the same planes on load, so a model loaded from the
  artifact computes bitwise what the in-memory model computes;
* norms, router, shared-expert gate, DeltaNet conv / decay / bias: ``native.f32``;
* token embedding: ``native.f16``.

Names: ``blk.{l}.{proj}`` (q, g, k, v, o / qkvz, ba, out / sg, su, sd), ``blk.{l}.{eg|eu|ed}.{e}``
for expert e, ``blk.{l}.{attn_norm|post_norm|q_norm|k_norm|conv_w|a_log|dt_bias|ssm_norm|router|
shared_gate}``, ``output_norm``, ``output``, ``token_embd``.

``load`` verifies every shard's sha256 (index) and, with ``verify=True``, every payload's sha256
once at admission; a mismatch is a hard error.

Parity: crates/hawking-core/src/model/gravity_engine.rs:251-450 (GravityEngine::load: container
sniff, architecture switch, shard / directory open), crates/hawking-core/src/model/
qwen80_mixed_catalog.rs:20-33 (mixed codecs per tensor), crates/hawking-core/src/artifact.rs
(container).
"""
from __future__ import annotations

import dataclasses
import json
import os
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from .._ext import native
from ..formats.gravity import GravityModel, write_index, write_shard
from ..ops.mixed import BINARY, UNIFORM, MixedTable, MixedWeight
from ..ops.qweight import QWeight
from .config import ModelConfig
from .qwen_next import QNLayer, QNWeights

ARCH = "qwen3next"
F32_FIELDS = ("attn_norm", "post_norm", "q_norm", "k_norm", "conv_w", "a_log", "dt_bias", "ssm_norm", "router",
              "shared_gate")
EXPERT_KEYS = ("eg", "eu", "ed")


def _payload(w: MixedWeight) -> Tuple[str, np.ndarray]:
    if w.zero >= 0 and w.kind == UNIFORM:
        raise ValueError("qwen-next artifact: uniform codes with a custom zero point have no HGRAVU01 form")
    scales = w.scales.detach().contiguous().view(torch.uint8).cpu().numpy().reshape(-1)
    codes = w.codes.detach().contiguous().cpu().numpy().reshape(-1)
    n = native()
    if w.kind == BINARY:
        return "hgrav.b01", n.wrap_hgravb01(w.N, w.K, w.group, scales, codes)
    if w.kind == UNIFORM:
        return "hgrav.u01", n.wrap_hgravu01(w.N, w.K, w.group, w.bits, scales, codes)
    raise ValueError(f"qwen-next artifact: codec kind {w.kind} not supported")


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().contiguous().cpu().numpy().view(np.uint8).reshape(-1)


def _config_json(cfg: ModelConfig) -> dict:
    return {k: v for k, v in dataclasses.asdict(cfg).items()}


def save(directory: str, cfg: ModelConfig, w: QNWeights, shard_bytes: int = 2 << 30) -> dict:
    """Write the artifact (shards of about ``shard_bytes``, then the index). Returns the index."""
    os.makedirs(directory, exist_ok=True)
    entries: List[dict] = []

    def mixed(name: str, i: int):
        codec, data = _payload(w.table.weights[i])
        mw = w.table.weights[i]
        entries.append({"name": name, "codec": codec, "shape": [mw.N, mw.K], "data": data})

    def f32(name: str, t: torch.Tensor):
        entries.append({"name": name, "codec": "native.f32", "shape": list(t.shape), "data": _f32(t)})

    for l, L in enumerate(w.layers):
        for key, i in L.idx.items():
            if key in EXPERT_KEYS:
                continue
            mixed(f"blk.{l}.{key}", i)
        for key in EXPERT_KEYS:
            for e in range(cfg.n_experts):
                mixed(f"blk.{l}.{key}.{e}", L.idx[key] + e)
        for key in F32_FIELDS:
            t = getattr(L, key)
            if t is not None:
                f32(f"blk.{l}.{key}", t)
    f32("output_norm", w.out_norm)
    mixed("output", w.lm_head)
    if w.embed.fmt != 1:
        raise ValueError("qwen-next artifact: the token embedding must be an F16 table")
    entries.append({"name": "token_embd", "codec": "native.f16", "shape": [w.embed.N, w.embed.K],
                    "data": w.embed.to_raw().cpu().numpy().reshape(-1)})
    weight_map: Dict[str, str] = {}
    dtypes: Dict[str, str] = {}
    shard: List[dict] = []
    size = 0
    n_shard = 0

    def flush():
        nonlocal shard, size, n_shard
        if not shard:
            return
        fn = f"model-{n_shard:05d}.gravity"
        write_shard(os.path.join(directory, fn), shard, {"architecture": {"name": ARCH}})
        for t in shard:
            weight_map[t["name"]] = fn
        n_shard += 1
        shard, size = [], 0

    for e in entries:
        dtypes[e["name"]] = e["codec"]
        shard.append(e)
        size += e["data"].size
        if size >= shard_bytes:
            flush()
    flush()
    return write_index(directory, weight_map, {"name": ARCH, "config": _config_json(cfg)}, dtypes)


def config_of(g: GravityModel) -> ModelConfig:
    a = g.index.get("architecture") or {}
    if not isinstance(a, dict) or a.get("name") != ARCH or "config" not in a:
        raise ValueError("not a qwen3next .gravity artifact (index architecture)")
    fields = {f.name for f in dataclasses.fields(ModelConfig)}
    return ModelConfig(**{k: v for k, v in a["config"].items() if k in fields})


def load(path: str, device, verify: bool = True, cfg: Optional[ModelConfig] = None) -> Tuple[ModelConfig, QNWeights]:
    """(config, weights) from an artifact directory; payload sha256s checked once when ``verify``."""
    g = GravityModel(path, verify_on_open=verify)
    cfg = cfg or config_of(g)
    ws: List[MixedWeight] = []

    def mixed(name: str) -> int:
        ws.append(MixedWeight.from_payload(np.ascontiguousarray(g.raw(name)), device))
        return len(ws) - 1

    def f32(name: str) -> Optional[torch.Tensor]:
        if not g.has(name):
            return None
        t = g.tensors[name]
        a = np.ascontiguousarray(g.raw(name)).view(np.float32).reshape(t.shape)
        return torch.from_numpy(a.copy()).to(device)

    layers = []
    for l in range(cfg.layers):
        full = cfg.layer_is_full_attention(l)
        L = QNLayer(full, attn_norm=f32(f"blk.{l}.attn_norm"), post_norm=f32(f"blk.{l}.post_norm"))
        keys = ("q", "g", "k", "v", "o") if full else ("qkvz", "ba", "out")
        for key in keys:
            L.idx[key] = mixed(f"blk.{l}.{key}")
        for key in EXPERT_KEYS:
            L.idx[key] = len(ws)
            for e in range(cfg.n_experts):
                mixed(f"blk.{l}.{key}.{e}")
        for key in ("sg", "su", "sd"):
            L.idx[key] = mixed(f"blk.{l}.{key}")
        for key in F32_FIELDS[2:]:
            setattr(L, key, f32(f"blk.{l}.{key}"))
        layers.append(L)
    out_norm = f32("output_norm")
    head = mixed("output")
    t = g.tensors["token_embd"]
    raw = torch.from_numpy(np.ascontiguousarray(g.raw("token_embd")).copy()).to(device)
    emb = QWeight.from_raw(raw, 1, t.shape[0], t.shape[1])
    return cfg, QNWeights(MixedTable(ws), emb, out_norm, layers, head)


def is_artifact(path: str) -> bool:
    p = os.path.join(path, "model.gravity.index.json")
    if not os.path.isfile(p):
        return False
    with open(p) as f:
        a = json.load(f).get("architecture", {})
    return isinstance(a, dict) and a.get("name") == ARCH
