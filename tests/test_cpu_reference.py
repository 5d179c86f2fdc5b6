"""C++ CPU reference forward (the oracle) vs the plain PyTorch fp32 forward, on benchmark
config 1 (tiny Llama-arch Q4_0), plus the pinned greedy golden hash."""
import hashlib

import numpy as np
import pytest
import torch

from hawking_b200.formats.synth import random_prompt
from hawking_b200.models.torch_ref import TorchRefLlama, rope_ref


def test_rope_cpp_matches_torch(native):
    x = np.random.default_rng(0).standard_normal((3, 64)).astype(np.float32)
    for style in (0, 1):
        a = native.ref_rope(x, 17, 64, 10000.0, style)
        b = rope_ref(torch.from_numpy(x)[None], torch.tensor([17]), 10000.0, 64, style)[0].numpy()
        np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-5)


def test_topk_gate_ties_lowest_index(native):
    ids, w = native.ref_topk_gate(np.array([1.0, 3.0, 3.0, 0.5], np.float32), 2, True)
    assert ids == [1, 2]
    assert abs(sum(w) - 1) < 1e-6


def test_sampler_greedy_and_topk(native):
    s = native.Sampler(42)
    p = native.SamplingParams()
    assert s.sample(np.array([1.0, 5.0, 2.0, 5.0], np.float32), p) == 1   # first max wins
    p.temperature, p.top_k = 1.0, 1
    assert s.sample(np.array([0.0, 0.1, 3.0], np.float32), p) == 2


def test_cpu_forward_matches_torch(tiny_gguf, native):
    cpu = native.CpuLlama(tiny_gguf, 256, 8)
    ref = TorchRefLlama(tiny_gguf, max_ctx=256)
    prompt = random_prompt(8, 32000, seed=1)
    for i, t in enumerate(prompt):
        a = cpu.forward(t, i)
        b = ref.forward(t, i).numpy()
        np.testing.assert_allclose(a, b, rtol=2e-3, atol=2e-3)


# sha256 (first 16 hex) of the greedy-32 ids from the 32-token seed-1 prompt, benchmark config 1.
GOLDEN_TINY_GREEDY = "05ec4c8530e402f3"


def test_cpu_greedy_golden(tiny_gguf, native):
    cpu = native.CpuLlama(tiny_gguf, 128, 8)
    prompt = random_prompt(32, 32000, seed=1)
    ids = cpu.generate_greedy(prompt, 32)
    assert len(ids) == 32
    ref = TorchRefLlama(tiny_gguf, max_ctx=128).generate_greedy(prompt, 32)
    assert ids == ref
    h = hashlib.sha256(np.asarray(ids, np.uint32).tobytes()).hexdigest()[:16]
    assert h == GOLDEN_TINY_GREEDY, h
