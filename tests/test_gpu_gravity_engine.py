"""The `.gravity` engine path: a Qwen3-Next-style model written as a multi-shard artifact with the
repo's own writer, opened by ``Engine.from_path`` (container sniff, architecture from the index,
payload sha256s verified at admission), decodes bitwise the greedy ids of the in-memory model; a
shard with one byte changed is refused."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

from hawking_b200.engine.engine import Engine  # noqa: E402
from hawking_b200.engine.sampling import SamplingParams  # noqa: E402
from hawking_b200.models import qwen_next_artifact as qa  # noqa: E402
from hawking_b200.models.config import preset  # noqa: E402
from hawking_b200.models.qwen_next import random_qwen_next_weights  # noqa: E402


@pytest.fixture(scope="module")
def model():
    cfg = preset("qwen3-next").with_(layers=4, n_experts=32, max_ctx=256)
    return cfg, random_qwen_next_weights(cfg, "cuda", seed=3)


def test_artifact_engine_matches_in_memory(model, tmp_path):
    cfg, w = model
    prompt = list(range(40, 60))
    sp = SamplingParams(max_tokens=12)
    ref = Engine.build_qwen_next(cfg, w, device="cuda", max_batch=2).generate([prompt], sp)[0]
    d = str(tmp_path / "qn")
    idx = qa.save(d, cfg, w, shard_bytes=32 << 20)
    assert len(set(idx["weight_map"].values())) > 1  # several shards
    eng = Engine.from_path(d, max_batch=2)
    assert eng.cfg.layers == cfg.layers and eng.cfg.n_experts == cfg.n_experts
    got = eng.generate([prompt], sp)[0]
    assert got == ref


def test_artifact_tamper_is_refused(model, tmp_path):
    cfg, w = model
    d = str(tmp_path / "qn")
    idx = qa.save(d, cfg, w, shard_bytes=32 << 20)
    fn = os.path.join(d, sorted(set(idx["weight_map"].values()))[0])
    with open(fn, "r+b") as f:
        f.seek(os.path.getsize(fn) - 5)
        b = f.read(1)
        f.seek(-1, os.SEEK_CUR)
        f.write(bytes([b[0] ^ 0x40]))
    with pytest.raises(RuntimeError):
        Engine.from_path(d, max_batch=2)
    torch.cuda.synchronize()
