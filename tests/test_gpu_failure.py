"""Failure paths on one GPU, with no GPU fault: a bounded device wait that runs out, and the
engine refusing to commit a step whose device status word is set.

* The tensor-parallel all-reduce consumer polls a receive region that no peer ever writes, with a
  5 ms bound: it must give up, report HK_ERR_PEER_TIMEOUT (2) in its status word and return, and
  the CUDA context must stay usable.
* A status word set before a step (as a kernel would after a failed wait) makes Engine.step raise
  DeviceStatusError without appending that step's tokens.
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def test_peer_wait_times_out_and_reports():
    from hawking_b200._ext import kernels
    from hawking_b200.ops import Q8Act
    rows, K, n = 2, 2048, 2
    x_in = torch.randn(rows, K, device=DEV)
    x_out = torch.zeros(rows, K, device=DEV)
    recv = torch.zeros(n * rows * K, dtype=torch.int64, device=DEV)  # flags 0: never this step's
    epoch = torch.ones(1, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = Q8Act(rows, K, DEV)
    t0 = time.perf_counter()
    kernels().tp_allreduce_rmsnorm_q8(x_in, x_out, recv.data_ptr(), rows * K, n, epoch, None, 1e-5, out.q, out.d,
                                      out.s, status, False, wait_ns=5_000_000)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert status.item() == 2  # HK_ERR_PEER_TIMEOUT
    assert dt < 5.0
    # the context is still usable: the same kernel with the words flagged completes cleanly
    recv.view(n, rows * K).copy_((torch.ones(n, rows * K, dtype=torch.int64, device=DEV) << 32))
    status.zero_()
    kernels().tp_allreduce_rmsnorm_q8(x_in, x_out, recv.data_ptr(), rows * K, n, epoch, None, 1e-5, out.q, out.d,
                                      out.s, status, False, wait_ns=5_000_000)
    torch.cuda.synchronize()
    assert status.item() == 0
    torch.testing.assert_close(x_out, x_in)  # the pushed partials were 0.0


def test_engine_discards_step_with_status_set():
    from hawking_b200.engine.engine import DeviceStatusError, Engine
    from hawking_b200.engine.sampling import SamplingParams
    from hawking_b200.models.config import preset
    from hawking_b200.models.llama import random_llama_weights
    cfg = preset("llama3-8b", layers=2, hidden=512, n_heads=8, n_kv_heads=2, ffn=1024, vocab=2048, max_ctx=256)
    w = random_llama_weights(cfg, DEV, seed=0)
    eng = Engine.build(cfg, w, device=DEV, max_batch=2, max_ctx=256, block_size=64, num_blocks=16, max_rows=16)
    rid = eng.add_request([1, 2, 3, 4], SamplingParams(max_tokens=8))
    eng.step()  # prefill + first token
    n0 = len(eng.requests[rid].output)
    eng.model.status.fill_(3)  # as a kernel would after an mbarrier wait ran out
    with pytest.raises(DeviceStatusError):
        eng.step()
    assert len(eng.requests[rid].output) == n0
    eng.clear_device_status()
    assert eng.model.status.item() == 0
