"""Vocabulary pruning of the LM head, and the per-layer quantisation tier map.

``PrunedVocab``: the LM head keeps the rows of a whitelist of token ids (a corpus-supported subset,
or the first N ids); logits, the greedy argmax and the sampler run over the kept rows, and every
chosen row index is mapped back to its original token id on the device before it becomes the next
input or reaches the tokenizer. The input embedding keeps the whole vocabulary (a prompt may hold
any token). Whitelist file::

    {"vocab_size_original": V, "keep_token_ids": [ascending ids], "coverage": 0.995, ...}

``QuantTierMap``: the GGUF format each layer's FFN weights are materialised at (``gate_up`` /
``down`` per layer; layers or groups not listed keep their file format), applied once at load by
re-quantising on the device. File::

    {"schema_version": 1, "n_layers": L, "layers": [{"layer": 0, "gate_up": "q4_K", "down": "q6_K"}, ...]}

Parity: crates/hawking-core/src/vocab_prune.rs (whitelist, LM-head slice, pruned -> original id
translation after the argmax), crates/hawking-serve/src/lib.rs:562-568 (prune at serve start),
crates/hawking-core/src/quant_tier_map.rs (per-layer expert / FFN dtype map).
"""
from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

from ..formats.ggml import GgmlType
from ..ops.qweight import QWeight


@dataclass
class PrunedVocab:
    keep: List[int]          # ascending original token ids
    original_size: int

    @staticmethod
    def load(path: str) -> "PrunedVocab":
        with open(path) as f:
            d = json.load(f)
        keep = sorted(set(int(t) for t in d["keep_token_ids"]))
        return PrunedVocab(keep, int(d.get("vocab_size_original", (keep[-1] + 1) if keep else 0)))

    @staticmethod
    def first(n: int, vocab: int, always: Optional[List[int]] = None) -> "PrunedVocab":
        """The first ``n`` ids (BPE vocabularies are ordered by merge rank, so low ids are the
        frequent ones) plus ``always`` (end-of-generation and other control ids)."""
        keep = sorted(set(range(min(n, vocab))) | set(int(t) for t in (always or []) if 0 <= t < vocab))
        return PrunedVocab(keep, vocab)

    @staticmethod
    def from_counts(counts: Dict[int, int], vocab: int, coverage: float = 0.995,
                    always: Optional[List[int]] = None) -> Tuple["PrunedVocab", float]:
        """The most frequent ids of a tokenised corpus (``counts``: id -> occurrences) until they
        cover ``coverage`` of its tokens, plus ``always``. Returns (whitelist, coverage reached)."""
        total = sum(counts.values())
        keep, seen = set(), 0
        for t, c in sorted(counts.items(), key=lambda kv: (-kv[1], kv[0])):
            if total and seen / total >= coverage:
                break
            if 0 <= t < vocab:
                keep.add(int(t))
                seen += c
        keep |= {int(t) for t in (always or []) if 0 <= t < vocab}
        return PrunedVocab(sorted(keep), vocab), (seen / total if total else 1.0)

    def save(self, path: str, coverage: Optional[float] = None):
        d = {"vocab_size_original": self.original_size, "vocab_size_pruned": len(self.keep),
             "keep_token_ids": self.keep}
        if coverage is not None:
            d["coverage"] = coverage
        with open(path, "w") as f:
            json.dump(d, f)

    def __len__(self) -> int:
        return len(self.keep)

    def validate(self, vocab: int):
        if self.original_size != vocab or (self.keep and self.keep[-1] >= vocab):
            raise ValueError(f"vocab whitelist built for {self.original_size} tokens, model has {vocab}")
        if not self.keep:
            raise ValueError("vocab whitelist keeps no token")

    def slice_head(self, head: QWeight) -> QWeight:
        """The LM head rows of the kept ids (a new weight; a tied embedding is not touched)."""
        idx = torch.tensor(self.keep, dtype=torch.long, device=head.planes[0].device)
        return QWeight(head.fmt, len(self.keep), head.K, [p.index_select(0, idx).contiguous() for p in head.planes])

    def id_map(self, device) -> torch.Tensor:
        """int32 [len] original id of every kept row."""
        return torch.tensor(self.keep, dtype=torch.int32, device=device)


def apply_vocab_prune(model, pv: PrunedVocab):
    """Prune a LlamaModel's LM head in place (one GPU): the head (and its W4A16 re-lay) keep the
    whitelisted rows, the logits buffer shrinks, and the model maps chosen rows back to token ids."""
    from ..ops import mg
    if getattr(model, "tp", None) is not None:
        raise ValueError("vocabulary pruning under tensor parallelism is not supported")
    if getattr(model, "vocab_map", None) is not None:
        raise ValueError("the LM head is already pruned")
    w = model.w
    pv.validate(w.lm_head.N)
    head = pv.slice_head(w.lm_head)
    # a new weights record: the caller's (possibly shared) weights keep the whole head
    model.w = dataclasses.replace(w, lm_head=head,
                                  mg_head=mg.pack(head, math=w.mg_head.math) if w.mg_head is not None else None)
    model.logits = torch.zeros(model.max_logit_rows, len(pv), device=model.dev)
    model.vocab_map = pv.id_map(model.dev)
    if getattr(model, "dstep", None) is not None:
        model.dstep = None  # the persistent step writes full-vocabulary logits
    if hasattr(model, "release_graphs"):
        model.release_graphs()


_DTYPES = {"q4_k": GgmlType.Q4_K, "q6_k": GgmlType.Q6_K, "q8_0": GgmlType.Q8_0, "q4_0": GgmlType.Q4_0,
           "q5_0": GgmlType.Q5_0}


@dataclass
class QuantTierMap:
    layers: Dict[int, Dict[str, int]]   # layer -> {"gate_up": fmt, "down": fmt}
    n_layers: int = 0

    @staticmethod
    def load(path: str) -> "QuantTierMap":
        with open(path) as f:
            d = json.load(f)
        if int(d.get("schema_version", 1)) != 1:
            raise ValueError("quant tier map: schema_version 1 expected")
        out: Dict[int, Dict[str, int]] = {}
        for e in d.get("layers", []):
            l = int(e["layer"])
            if l in out:
                raise ValueError(f"quant tier map: layer {l} listed twice")
            ent = {}
            for g in ("gate_up", "down"):
                if e.get(g) is not None:
                    k = str(e[g]).lower()
                    if k not in _DTYPES:
                        raise ValueError(f"quant tier map: dtype {e[g]!r} (allowed: {sorted(_DTYPES)})")
                    ent[g] = int(_DTYPES[k])
            out[l] = ent
        return QuantTierMap(out, int(d.get("n_layers", 0)))

    def dtype_for(self, layer: int, group: str) -> Optional[int]:
        return self.layers.get(layer, {}).get(group)

    def apply(self, weights, cfg=None) -> int:
        """Re-quantise Llama-family FFN weights on the device to the mapped formats, before the model
        is built (dense gate / up / down, or a MoE layer's stacked expert gate / up / down). Returns
        the number of matrices changed."""
        if self.n_layers and cfg is not None and self.n_layers != cfg.layers:
            raise ValueError(f"quant tier map for {self.n_layers} layers, model has {cfg.layers}")
        n = 0
        for l, lw in enumerate(weights.layers):
            gu, dn = self.dtype_for(l, "gate_up"), self.dtype_for(l, "down")
            if lw.moe is not None:
                m = lw.moe
                if gu is not None and m.w_gate.fmt != gu:
                    m.w_gate, m.w_up = requantize(m.w_gate, gu), requantize(m.w_up, gu)
                    n += 2
                if dn is not None and m.w_down.fmt != dn:
                    m.w_down = requantize(m.w_down, dn)
                    n += 1
                continue
            if gu is not None and lw.w_gu is not None and lw.w_gu.fmt != gu:
                F = lw.w_gu.N // 2
                lw.w_gu = requantize(lw.w_gu, gu)
                lw.w_gate, lw.w_up = lw.w_gu.rows(0, F), lw.w_gu.rows(F, F)
                lw.mg_gu = None
                n += 1
            elif gu is not None and lw.w_gate is not None and lw.w_gate.fmt != gu:
                lw.w_gate, lw.w_up = requantize(lw.w_gate, gu), requantize(lw.w_up, gu)
                n += 2
            if dn is not None and lw.w_down is not None and lw.w_down.fmt != dn:
                lw.w_down = requantize(lw.w_down, dn)
                lw.mg_down = None
                n += 1
        return n


def requantize(w: QWeight, fmt: int, chunk_elems: int = 1 << 25) -> QWeight:
    """``w`` decoded and quantised again to ``fmt`` on its device, in row chunks of at most
    ``chunk_elems`` fp32 elements (a stacked expert tensor never materialises whole in fp32)."""
    out = QWeight.empty(fmt, w.N, w.K, w.planes[0].device)
    rows = max(1, chunk_elems // w.K)
    for r0 in range(0, w.N, rows):
        r1 = min(w.N, r0 + rows)
        part = QWeight.quantize(w.rows(r0, r1 - r0).dequantize().to(w.planes[0].device), fmt)
        for p, q in zip(out.planes, part.planes):
            p[r0:r1].copy_(q)
    return out
