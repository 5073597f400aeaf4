"""GPU: a device wait that can never complete gives up, reports, and leaves the GPU usable.

Every mbarrier and counter wait in this library's kernels is bounded (2 s);
on expiry the kernel raises GW_DEVICE_ERR_WAIT_TIMEOUT, unwinds and returns.
Here the self-test kernel waits on an mbarrier nothing arrives on and a
counter nothing increments, with a 1 ms limit: the launch must complete, the
error word must carry the timeout bit, and the next real gather-GEMM on the
same context must be correct with a clean error word. No fault, trap or hang
is involved: the wait ends by its own time limit.
"""

from __future__ import annotations

import time

import pytest
import torch

from ghostweight_triton_b200 import _native
from ghostweight_triton_b200.kernels.matmul import ghost_linear

pytestmark = pytest.mark.gpu


def test_wait_gives_up_reports_and_context_stays_usable():
    assert _native.device_error(reset=True) == 0
    t0 = time.perf_counter()
    _native.selftest_wait_timeout(1_000_000)          # 1 ms per wait
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert elapsed < 5.0, f"bounded waits took {elapsed:.2f} s"
    assert _native.device_error(reset=True) == _native.DEVICE_ERR_WAIT_TIMEOUT
    assert _native.device_error(reset=False) == 0     # the reset cleared it

    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(512, 1024, device="cuda", generator=g).half()
    w = (torch.randn(768, 1024, device="cuda", generator=g) / 32).half()
    idx = torch.arange(0, 1024, 2, device="cuda", dtype=torch.int64)
    wp = w[:, idx].contiguous()
    y = ghost_linear(x, wp, idx)
    ref = (x.float()[:, idx] @ wp.float().t()).half()
    torch.testing.assert_close(y, ref, atol=1e-2, rtol=1e-2)
    assert _native.device_error(reset=True) == 0


def test_limit_is_clamped_to_at_most_one_second():
    t0 = time.perf_counter()
    _native.selftest_wait_timeout(10 ** 12)            # asks for 1000 s, gets 1 s per wait
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 10.0
    assert _native.device_error(reset=True) == _native.DEVICE_ERR_WAIT_TIMEOUT
