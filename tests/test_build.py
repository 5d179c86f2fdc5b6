"""Both native modules import (CPU box included) and expose the documented entry points."""
import importlib

import torch  # noqa: F401  (the kernel module links against libtorch)


def test_native_module_imports():
    m = importlib.import_module("hawking_b200._native")
    for name in ["GgufFile", "GgufWriter", "CpuLlama", "BlockManager", "Scheduler", "Sampler"]:
        assert hasattr(m, name), name


def test_kernel_module_imports():
    m = importlib.import_module("hawking_b200._kernels")
    for name in ["gemv", "rmsnorm_q8", "rope_append", "attention_decode", "argmax", "sample", "embed",
                 "quantize", "advance"]:
        assert hasattr(m, name), name
