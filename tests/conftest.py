import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "multigpu: needs 2 or more GPUs")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def native():
    from hawking_b200._ext import native as _n
    return _n()


@pytest.fixture(scope="session")
def tiny_gguf(tmp_path_factory):
    """The tiny Llama-arch Q4_0 model (benchmark config 1), written once per session."""
    from hawking_b200.formats.synth import write_llama_family_gguf
    from hawking_b200.models.config import preset
    p = tmp_path_factory.mktemp("models") / "tiny-llama-q4_0.gguf"
    write_llama_family_gguf(str(p), preset("tiny-llama"), seed=0)
    return str(p)
