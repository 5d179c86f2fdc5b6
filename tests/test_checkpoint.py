"""Checkpoint / resume of paged-KV sequences and recurrent state (CPU tensors; the same code runs on
the GPU cache). Parity: crates/hawking-core/src/cache/prefill_disk.rs (DSPRFKV2), engine.rs:423-445."""
import os

import pytest
import torch

from hawking_b200.engine.checkpoint import (PrefixDiskCache, load_recurrent, load_sequence, save_recurrent,
                                            save_sequence)
from hawking_b200.engine.kv_cache import PagedKVCache


def _cache():
    return PagedKVCache(3, 2, 8, 16, 4, 4, 8, "cpu", prefix_cache=False)


def test_kv_snapshot_roundtrip_and_integrity(tmp_path):
    kv = _cache()
    toks = list(range(100, 111))  # 11 tokens over 3 blocks
    assert kv.bm.reserve(1, len(toks))
    kv.k.normal_()
    kv.v.normal_()
    slots = kv.bm.slots(1, 0, len(toks))
    p = str(tmp_path / "s.hkkv")
    save_sequence(kv, 1, toks, p)
    kv2 = _cache()
    kv2.bm.reserve(9, 5)  # occupy other blocks so the restored sequence lands elsewhere
    assert load_sequence(kv2, 2, p) == toks
    slots2 = kv2.bm.slots(2, 0, len(toks))
    for a, b in zip(slots, slots2):
        assert torch.equal(kv.k[:, a // 4, :, a % 4], kv2.k[:, b // 4, :, b % 4])
        assert torch.equal(kv.v[:, a // 4, :, a % 4], kv2.v[:, b // 4, :, b % 4])
    data = bytearray(open(p, "rb").read())
    data[-3] ^= 0xFF
    bad = str(tmp_path / "bad.hkkv")
    open(bad, "wb").write(bytes(data))
    with pytest.raises(ValueError, match="digest"):
        load_sequence(_cache(), 3, bad)
    open(bad, "wb").write(bytes(data[:-10]))
    with pytest.raises(ValueError, match="truncated"):
        load_sequence(_cache(), 3, bad)


def test_prefix_disk_cache_longest_prefix_and_lru(tmp_path):
    kv = _cache()
    toks = list(range(7, 19))
    kv.bm.reserve(1, len(toks))
    kv.k.normal_()
    pc = PrefixDiskCache(str(tmp_path / "pc"), max_entries=2)
    pc.store(kv, 1, toks[:4])
    pc.store(kv, 1, toks[:8])
    n, path = pc.longest_prefix(toks + [99, 98])
    assert n == 8 and os.path.exists(path)
    assert pc.longest_prefix([1, 2, 3]) is None
    pc.store(kv, 1, toks[:12])  # evicts the least recently used entry (the 4-token prefix)
    assert len(os.listdir(tmp_path / "pc")) == 2
    assert pc.longest_prefix(toks[:6]) is None


def test_recurrent_state_roundtrip(tmp_path):
    state = torch.randn(3, 4, 2, 8, 8)
    conv = torch.randn(3, 4, 16, 3)
    p = str(tmp_path / "r.hkst")
    save_recurrent([state, conv], 2, p, meta={"pos": 17})
    s2, c2 = torch.zeros_like(state), torch.zeros_like(conv)
    assert load_recurrent([s2, c2], 1, p) == {"pos": 17}
    assert torch.equal(s2[:, 1], state[:, 2]) and torch.equal(c2[:, 1], conv[:, 2])
