"""Typed engine configuration, runtime profiles (lever plans), memory-budget refusal and the
serving loop's gather window, on the CPU.

Parity: crates/hawking-serve/src/lib.rs:34-200 (RuntimeProfile, LeverPlan, contract),
crates/hawking-core/src/model/mod.rs:96-115 (memory budget refusal).
"""
import pytest

from hawking_b200.config import (RUNTIME_PROFILES, EngineConfig, MemoryBudgetError, apply_profile,
                                 check_memory_budget, env_flag, runtime_profile)


def test_profiles_are_the_reference_set_with_contracts():
    assert set(RUNTIME_PROFILES) == {"default", "fast", "race", "efficient", "exact"}
    for name, plan in RUNTIME_PROFILES.items():
        assert plan.contract.startswith(f"profile={name}:")
    with pytest.raises(ValueError):
        runtime_profile("turbo")


def test_apply_profile_overrides_only_its_levers():
    base = EngineConfig(max_batch=4, block_size=16)
    race = apply_profile(base, "race")
    assert (race.max_batch, race.max_prefill_tokens, race.policy, race.block_size) == (64, 2048, 1, 16)
    assert apply_profile(base, "default") == base
    assert base.max_batch == 4  # not mutated
    assert runtime_profile("exact").model == {"tc_min_rows": 1}
    assert runtime_profile("efficient").serve["gather_ms"] > 0


def test_memory_budget_refusal():
    check_memory_budget(1 << 30, 4 << 30, "weights")
    with pytest.raises(MemoryBudgetError, match="weights of m.gguf: needs 8.00 GiB"):
        check_memory_budget(8 << 30, 6 << 30, "weights of m.gguf")
    with pytest.raises(MemoryError):  # a MemoryError subclass
        check_memory_budget(3 << 30, 3 << 30, "kv", reserve_bytes=1)


def test_startup_timing_flag_documented(monkeypatch):
    assert env_flag("HK_STARTUP_TIMING") == "0"
    monkeypatch.setenv("HK_STARTUP_TIMING", "1")
    assert env_flag("HK_STARTUP_TIMING") == "1"


def test_gather_window_waits_only_with_free_slots(native):
    from hawking_b200.serve import ServeLoop
    from test_tokenizer import bpe_spec

    class Busy:
        max_batch = 2

        def __init__(self):
            self.work = True

        def has_work(self):
            return self.work

        def step(self):
            return []

        def add_request(self, prompt, params):
            return 1

        def abort(self, rid):
            pass

    tok = native.Tokenizer.from_spec(bpe_spec(native))
    eng = Busy()
    loop = ServeLoop(eng, tok, port=0, model_id="m", gather_ms=40.0)
    waits = []

    class Recording:  # the native server, with poll() recording its wait
        def __init__(self, inner):
            self.inner = inner

        def poll(self, ms):
            waits.append(ms)
            return []

        def __getattr__(self, name):
            return getattr(self.inner, name)

    loop.server = Recording(loop.server)
    loop.iterate()
    assert waits[-1] == 40            # work in flight, free slots: gather
    loop._to_engine = {1: 1, 2: 2}    # batch full: no wait
    loop.iterate()
    assert waits[-1] == 0
    eng.work = False
    loop.iterate(idle_wait_ms=7)      # idle: the idle poll
    assert waits[-1] == 7


def test_every_runtime_env_flag_is_documented():
    """Every HK_* variable the package reads at run time (os.environ / getenv) has an entry in
    ENV_FLAGS with its default and meaning."""
    import pathlib
    import re

    from hawking_b200.config import ENV_FLAGS
    root = pathlib.Path(__file__).resolve().parent.parent / "hawking_b200"
    pat = re.compile(r'(?:environ\.get\(|getenv\()\s*"(HK_[A-Z0-9_]+)"')
    read = set()
    for f in list(root.rglob("*.py")) + list(root.rglob("*.cu")) + list(root.rglob("*.cpp")):
        read |= set(pat.findall(f.read_text(errors="ignore")))
    assert read, "no flags found: the pattern is stale"
    missing = sorted(read - set(ENV_FLAGS))
    assert not missing, missing


def test_tensor_core_gemm_row_regimes_agree():
    """Below SPLIT_K_MAX_ROWS + 1 rows the tensor-core GEMMs accumulate into a zeroed output
    (split-K or stream-K), from there on the persistent 256-token tiles overwrite it: the prefill
    SwiGLU re-zeroes exactly the gate/up rows the smaller forwards reuse, so the three rules must
    switch at the same row count."""
    from hawking_b200 import ops
    for M in range(1, 600):
        persistent = ops.tc_gemm_bn(M) == 256
        assert ops.tc_gemm_overwrites(M) == (persistent and ops.PERSISTENT_GEMM), M
        assert persistent == (M > ops.SPLIT_K_MAX_ROWS), M
        if ops.tc_gemm_stream_k(M, 28672):
            assert not persistent and M <= 64
