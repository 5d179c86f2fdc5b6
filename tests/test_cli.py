"""The command-line front end on the CPU: version, doctor, tokenize, info, verify (and the exit
code of a failed verification).

Parity: crates/hawking/src/main.rs:401-814 (subcommands tokenize, stats, verify, doctor, version).
"""
import json

import numpy as np

from hawking_b200.__main__ import main


def test_version_and_doctor(capsys):
    assert main(["version"]) == 0
    v = json.loads(capsys.readouterr().out)
    assert "hawking_b200" in v
    assert main(["doctor"]) == 0
    d = json.loads(capsys.readouterr().out)
    assert "native_module" in d and "python" in d


def test_tokenize_and_info(tiny_gguf, capsys):
    assert main(["tokenize", "--gguf", tiny_gguf, "hello world"]) == 0
    ids = json.loads(capsys.readouterr().out)
    assert ids and all(isinstance(i, int) for i in ids)
    assert main(["tokenize", "--gguf", tiny_gguf, "--decode", " ".join(map(str, ids))]) == 0
    assert "hello world" in capsys.readouterr().out
    assert main(["info", tiny_gguf]) == 0
    info = json.loads(capsys.readouterr().out)
    assert info["architecture"] == "llama" and info["config"]["layers"] == 4 and "Q4_0" in info["tensor_types"]


def test_verify_gravity(tmp_path, capsys):
    from hawking_b200.formats.gravity import write_shard
    p = tmp_path / "m.gravity"
    write_shard(str(p), [{"name": "x", "codec": "native.f16", "shape": [8],
                          "data": np.arange(16, dtype=np.uint8)}])
    assert main(["verify", str(p)]) == 0
    assert json.loads(capsys.readouterr().out)["m.gravity"]["ok"]
    data = bytearray(p.read_bytes())
    data[-1] ^= 0xFF
    p.write_bytes(bytes(data))
    assert main(["verify", str(p)]) == 1


def test_info_on_a_safetensors_checkpoint(tmp_path, capsys):
    from hawking_b200.formats.safetensors import write_safetensors
    p = write_safetensors(str(tmp_path / "m.safetensors"), {
        "e.w1.weight": ("I8", (4, 16), bytes(64)), "e.w1.scale": ("F8_E8M0", (4, 1), bytes([127] * 4)),
        "norm.weight": ("F32", (4,), np.ones(4, np.float32).tobytes())})
    assert main(["info", p]) == 0
    info = json.loads(capsys.readouterr().out)
    assert info["format"] == "safetensors" and info["tensors"] == 3
    assert info["native_pairs"] == {"native.fp4_e2m1fn_x2_e8m0": 1}
