"""GGUF container: write/read round trip, metadata kinds, alignment and failure modes."""
import numpy as np
import pytest

from hawking_b200.formats.ggml import GgmlType
from hawking_b200.formats.gguf import GgufBuilder, GgufModel


def test_round_trip(tmp_path, native):
    b = GgufBuilder("llama")
    b.set("general.name", "t").arch_set("block_count", 2).set_f32("llama.rope.freq_base", 500000.0)
    b.set("tokenizer.ggml.tokens", ["a", "b", "<s>"]).set("some.flag", True).set("neg", -5)
    x = np.arange(2 * 256, dtype=np.float32).reshape(2, 256) / 100
    b.add("w", x, GgmlType.F32).add("q", x, GgmlType.Q4_K).add("h", x[0], GgmlType.F16)
    p = b.write(str(tmp_path / "m.gguf"))
    m = GgufModel(p)
    assert m.version == 3 and m.alignment == 32
    assert m.architecture == "llama"
    assert m.get("llama.block_count") == 2
    assert m.get("llama.rope.freq_base") == 500000.0
    assert m.get("tokenizer.ggml.tokens") == ["a", "b", "<s>"]
    assert m.get("some.flag") is True and m.get("neg") == -5
    assert m.tensors["w"].shape == (2, 256) and m.tensors["w"].dims == [256, 2]
    np.testing.assert_array_equal(m.dequantize("w"), x)
    assert np.abs(m.dequantize("q") - x).max() < 0.05 * np.abs(x).max()
    for t in m.tensors.values():
        assert t.offset % 32 == 0
    assert m.raw("q").nbytes == 2 * 144


def test_rejects_corrupt(tmp_path, native):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUF\x03\x00\x00\x00" + b"\x01" * 7)
    with pytest.raises(RuntimeError, match="truncated"):
        GgufModel(str(p))
    p.write_bytes(b"GGML" + b"\x00" * 60)
    with pytest.raises(RuntimeError, match="bad magic"):
        GgufModel(str(p))


def test_tensor_past_end_rejected(tmp_path, native):
    b = GgufBuilder("llama")
    b.add("w", np.ones((4, 32), np.float32), GgmlType.Q8_0)
    p = tmp_path / "t.gguf"
    b.write(str(p))
    data = p.read_bytes()
    p.write_bytes(data[: len(data) - 64])
    with pytest.raises(RuntimeError, match="past end"):
        GgufModel(str(p))


def test_state_space_architectures_are_refused_with_a_reason(tmp_path):
    import numpy as np
    import pytest as _pytest

    from hawking_b200.formats.gguf import GgufBuilder, GgufModel
    from hawking_b200.models.torch_ref import config_from_gguf
    b = GgufBuilder("rwkv7")
    b.add("token_embd.weight", np.zeros((8, 16), np.float32))
    m = GgufModel(b.write(str(tmp_path / "r.gguf")))
    with _pytest.raises(ValueError, match="rwkv7.*not built"):
        config_from_gguf(m)
