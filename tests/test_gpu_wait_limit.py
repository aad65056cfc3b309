"""Failure detection on the GPU without a fault: every pipelined kernel's waits are bounded (common.cuh
``mbar_wait_for``), and a wait that runs out records KD_DEVICE_TIMEOUT in the launch's status word, makes the launch's
other waiters give up, and returns, leaving the context usable. ``kd_wait_selftest`` runs that same wait loop on a
shared-memory barrier nothing arrives on, with a short limit; the host then reads the status the way the forward does
(``ops.check_status`` raises) and keeps computing."""

import pytest
import torch

from karpo_decision_b200 import _lib, ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
LIMIT_NS = 20_000_000  # 20 ms


def test_a_wait_that_runs_out_records_a_timeout_and_the_launch_returns():
    status = ops.status_word(DEV)
    status.zero_()
    elapsed = torch.zeros(2, dtype=torch.int64, device=DEV)
    _lib.call("kd_wait_selftest", status.data_ptr(), LIMIT_NS, elapsed.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    first, second = elapsed.tolist()
    assert int(status.item()) == _lib.KD_DEVICE_TIMEOUT
    assert LIMIT_NS <= first < 50 * LIMIT_NS  # gave up at its limit, not later
    assert 0 < second < 32 * LIMIT_NS  # gave up on seeing the status, long before its own 64 x limit
    with pytest.raises(_lib.KernelError):
        ops.check_status(DEV)  # the host's read of the word, which also clears it
    assert int(status.item()) == 0
    # the context still computes: a GEMM after the timed-out launch is right
    a = torch.randn(300, 256, device=DEV).bfloat16()
    w = torch.randn(512, 256, device=DEV).bfloat16()
    got = ops.gemm(a, w).float()
    want = a.float() @ w.float().T
    assert (got - want).abs().max().item() <= 2 ** -8 * want.abs().max().item() + 1e-3
    ops.check_status(DEV)


def test_wait_selftest_rejects_limits_past_a_second():
    rc = _lib.load().kd_wait_selftest(None, 2_000_000_000, None, None)
    assert rc == -1
