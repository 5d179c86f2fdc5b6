"""Vocabulary whitelist and quantisation tier map files (host side)."""
import json

import pytest

from hawking_b200.engine.vocab_prune import PrunedVocab, QuantTierMap
from hawking_b200.formats.ggml import GgmlType


def test_whitelist_round_trip(tmp_path):
    pv = PrunedVocab([1, 5, 9], 16)
    p = tmp_path / "wl.json"
    pv.save(str(p), coverage=0.9)
    d = json.loads(p.read_text())
    assert d["vocab_size_original"] == 16 and d["keep_token_ids"] == [1, 5, 9] and d["vocab_size_pruned"] == 3
    back = PrunedVocab.load(str(p))
    assert back.keep == [1, 5, 9] and back.original_size == 16 and len(back) == 3


def test_whitelist_load_sorts_and_dedups(tmp_path):
    p = tmp_path / "wl.json"
    p.write_text(json.dumps({"vocab_size_original": 10, "keep_token_ids": [7, 2, 7, 3]}))
    assert PrunedVocab.load(str(p)).keep == [2, 3, 7]


def test_first_n_keeps_control_ids():
    pv = PrunedVocab.first(4, 100, always=[99, 2, 500])
    assert pv.keep == [0, 1, 2, 3, 99]


def test_validate_rejects_other_vocab_and_empty():
    with pytest.raises(ValueError):
        PrunedVocab([1, 2], 10).validate(12)
    with pytest.raises(ValueError):
        PrunedVocab([1, 20], 10).validate(10)
    with pytest.raises(ValueError):
        PrunedVocab([], 10).validate(10)
    PrunedVocab([0, 9], 10).validate(10)


def test_from_counts_reaches_coverage():
    counts = {3: 50, 7: 30, 1: 15, 4: 5}
    pv, cov = PrunedVocab.from_counts(counts, 10, coverage=0.8, always=[9])
    assert pv.keep == [3, 7, 9] and cov == pytest.approx(0.8)
    pv, cov = PrunedVocab.from_counts(counts, 10, coverage=0.96)
    assert pv.keep == [1, 3, 4, 7] and cov == pytest.approx(1.0)


def test_tier_map_parse(tmp_path):
    p = tmp_path / "tiers.json"
    p.write_text(json.dumps({"schema_version": 1, "n_layers": 3, "layers": [
        {"layer": 0, "gate_up": "q4_K", "down": "q6_K"}, {"layer": 2, "down": "Q8_0"}]}))
    m = QuantTierMap.load(str(p))
    assert m.n_layers == 3
    assert m.dtype_for(0, "gate_up") == int(GgmlType.Q4_K) and m.dtype_for(0, "down") == int(GgmlType.Q6_K)
    assert m.dtype_for(1, "down") is None and m.dtype_for(2, "gate_up") is None
    assert m.dtype_for(2, "down") == int(GgmlType.Q8_0)


@pytest.mark.parametrize("doc", [
    {"schema_version": 2, "layers": []},
    {"layers": [{"layer": 0, "down": "q3_K"}]},
    {"layers": [{"layer": 0, "down": "q6_K"}, {"layer": 0, "gate_up": "q4_K"}]},
])
def test_tier_map_rejects(tmp_path, doc):
    p = tmp_path / "tiers.json"
    p.write_text(json.dumps(doc))
    with pytest.raises(ValueError):
        QuantTierMap.load(str(p))


def test_tier_map_layer_count_checked():
    class Cfg:
        layers = 4

    class W:
        layers = []

    with pytest.raises(ValueError):
        QuantTierMap({}, n_layers=3).apply(W(), Cfg())
