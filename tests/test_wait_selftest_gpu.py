"""Failure detection of the bulk kernel's bounded waits, exercised without a GPU fault: a
self-test kernel waits on an mbarrier that nothing completes; the wait gives up after its
limit, counts itself, and the context stays usable for the next launch.  (Collected after
the parity tests, whose last check is that no real wait ever ran out.)"""
import time

import pytest
import torch

from physisserve_b200 import ops
from physisserve_b200.wan import rope

pytestmark = pytest.mark.gpu


def test_a_wait_that_runs_out_is_counted_and_the_context_survives():
    torch.cuda.synchronize()
    assert ops.device_timeouts(reset=True) == 0          # no real wait ran out before this test
    t0 = time.perf_counter()
    ops.wait_selftest(limit_us=20000)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert ops.device_timeouts(reset=True) == 1
    assert elapsed >= 0.02
    # the context is usable: a normal launch right after
    x = torch.randn(1, 8, 2, 64, device="cuda").bfloat16()
    t = torch.ones(1, 8, 1, 64, device="cuda")
    assert torch.equal(rope(x, t, torch.zeros_like(t)), x)
    assert ops.device_timeouts(reset=True) == 0


def test_selftest_limit_is_validated():
    with pytest.raises(ops.PrepError):
        ops.wait_selftest(limit_us=0)
    with pytest.raises(ops.PrepError):
        ops.wait_selftest(limit_us=2_000_000)
