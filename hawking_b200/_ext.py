"""Loads the in-tree native modules.

``native()`` returns the host C++ module; ``kernels()`` the CUDA kernel module. A missing
kernel module on a machine with a GPU is an error (never a silent fallback); on a CPU-only
machine ``kernels()`` raises ``KernelsUnavailable`` so callers can skip GPU-only work.
"""
import importlib
import os
import subprocess
import sys

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class KernelsUnavailable(RuntimeError):
    pass


def build(cuda: bool = True) -> None:
    """Compile both modules in place (``python setup.py build_ext --inplace``)."""
    env = dict(os.environ)
    env.setdefault("MAX_JOBS", str(os.cpu_count() or 8))
    if not cuda:
        env["HK_SKIP_CUDA"] = "1"
    subprocess.check_call([sys.executable, "setup.py", "build_ext", "--inplace"], cwd=_ROOT, env=env)


_native = None
_kernels = None


def native():
    global _native
    if _native is None:
        try:
            _native = importlib.import_module("hawking_b200._native")
        except ImportError:
            build(cuda=False)
            _native = importlib.import_module("hawking_b200._native")
    return _native


def kernels():
    """The sm_100a kernel module. Raises if it cannot be loaded."""
    global _kernels
    if _kernels is None:
        import torch  # noqa: F401  (the module links against libtorch)
        try:
            _kernels = importlib.import_module("hawking_b200._kernels")
        except ImportError as e:
            raise KernelsUnavailable(
                "hawking_b200._kernels is not built; run `python setup.py build_ext --inplace`"
            ) from e
    return _kernels
