"""GPU: the "runs" gather-GEMM strategy (alive columns in 64-column runs, x read in place).

When a mask kills whole 64- or 128-column blocks, each 64-wide k-block of the
compacted x' is one contiguous slice of x, so the GEMM loads it straight from
x and no gather runs. The result must be bit-identical to the pregather path
(same GEMM kernel, same operand values in the same order) and within the
reference's tolerances (tests/test_matmul.py:68-72) of the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from ghostweight_triton_b200 import GhostLinear, _native
from ghostweight_triton_b200.kernels.gather import pack_weight
from ghostweight_triton_b200.kernels.matmul import ghost_linear, index_runs
from oracle import gw_oracle as O
from tests.conftest import tols
from tests.golden.gw_inputs import alive_from_dead, dead_columns, rand_matrix
from tests.test_gpu_matmul import assert_close, to_dev, to_np

pytestmark = pytest.mark.gpu


def _lists(K):
    yield "block64", alive_from_dead(K, dead_columns(K, 0.5, 1, "block", 64))
    yield "block128", alive_from_dead(K, dead_columns(K, 0.7, 2, "block", 128))
    yield "random", alive_from_dead(K, dead_columns(K, 0.5, 3, "random"))
    yield "start8", np.arange(8, 8 + 128, dtype=np.int64)
    yield "start4", np.arange(4, 4 + 64, dtype=np.int64)
    yield "partial", np.arange(0, 96, dtype=np.int64)
    yield "past_end", np.arange(K - 32, K + 32, dtype=np.int64)
    yield "empty", np.zeros(0, dtype=np.int64)


@pytest.mark.parametrize("K", [1024, 4096])
def test_index_runs_matches_oracle(K):
    for name, idx in _lists(K):
        got = index_runs(torch.from_numpy(idx).cuda(), K)
        assert got == O.index_runs(idx, K), name


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("M,K,N,block,sp", [
    (4096, 4096, 4096, 64, 0.5),      # CTA-pair kernel
    (2048, 4096, 3072, 128, 0.75),
    (300, 4096, 1000, 128, 0.5),      # single-CTA kernel (ragged M and N)
    (16, 4096, 4096, 64, 0.5),        # cluster split-K (decode rows)
    (1, 2048, 768, 64, 0.25),
    (77, 1024, 136, 64, 0.0),         # dense: one run covers everything
])
@pytest.mark.parametrize("bias,act", [(False, None), (True, "gelu")])
def test_runs_equals_pregather_and_oracle(dt, M, K, N, block, sp, bias, act):
    seed = M + K + N + block
    x = rand_matrix((M, K), seed, dt, 0.5)
    w = rand_matrix((N, K), seed + 1, dt, 1.0 / np.sqrt(K))
    b = rand_matrix((N,), seed + 2, dt, 0.5) if bias else None
    idx = alive_from_dead(K, dead_columns(K, sp, seed, "block", block))
    assert O.index_runs(idx, K) == 0
    xd, wd, idd = to_dev(x), to_dev(w), torch.from_numpy(idx).cuda()
    wp = pack_weight(wd, idd)
    bd = to_dev(b) if bias else None
    _native.device_error(reset=True)
    y_runs = ghost_linear(xd, wp, idd, bias=bd, activation=act, strategy="runs")
    y_pre = ghost_linear(xd, wp, idd, bias=bd, activation=act, strategy="pregather")
    assert _native.device_error(reset=True) == 0
    assert torch.equal(y_runs, y_pre)
    if M * K * N <= 2 ** 33:
        ref = O.ghost_linear(x, w, idx, b, act, dtype=dt)
        assert_close(to_np(y_runs), ref, dt, f"runs {dt} {M}x{K}x{N}")
    else:
        rows = torch.arange(0, M, 61, device="cuda")
        dense = F.linear(xd[rows][:, idd].float(), wp.float()[:, : idx.size],
                         bd.float() if bias else None)
        if act:
            dense = F.gelu(dense)
        torch.testing.assert_close(y_runs[rows].float(), dense, **tols(xd.dtype))


def test_runs_never_reads_dead_columns():
    """NaN in every dead column of x leaves the runs result finite and unchanged."""
    M, K, N = 512, 2048, 1024
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(M, K, device="cuda", dtype=torch.float16, generator=g)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).half()
    idx = torch.from_numpy(alive_from_dead(K, dead_columns(K, 0.5, 5, "block", 128))).cuda()
    wp = pack_weight(w, idx)
    y0 = ghost_linear(x, wp, idx, strategy="runs")
    dead = torch.ones(K, dtype=torch.bool, device="cuda")
    dead[idx] = False
    x[:, dead] = float("nan")
    y1 = ghost_linear(x, wp, idx, strategy="runs")
    assert torch.isfinite(y1).all() and torch.equal(y0, y1)


def test_runs_flags_misaligned_start_without_fault():
    """A run starting at column 4 (not a 16-byte boundary) is not loaded from there:
    the kernel raises the bad-index bit and the call returns normally."""
    x = torch.randn(256, 512, device="cuda", dtype=torch.float16)
    w = torch.randn(256, 512, device="cuda", dtype=torch.float16) / 16
    idx = torch.arange(4, 4 + 64, device="cuda")
    _native.device_error(reset=True)
    y = ghost_linear(x, pack_weight(w, idx), idx, strategy="runs")
    torch.cuda.synchronize()
    assert y.shape == (256, 256)
    assert _native.device_error(reset=True) & _native.DEVICE_ERR_BAD_INDEX


def test_runs_requires_whole_runs():
    x = torch.randn(64, 512, device="cuda", dtype=torch.float16)
    w = torch.randn(128, 512, device="cuda", dtype=torch.float16)
    idx = torch.arange(0, 96, device="cuda")
    with pytest.raises(RuntimeError):
        _native.gather_gemm(x, pack_weight(w, idx), idx,
                            torch.empty(64, 128, device="cuda", dtype=torch.float16), strategy="runs")


def test_runs_falls_back_for_unaligned_x():
    """x whose rows are not 16-byte aligned goes through the gather path instead."""
    base = torch.randn(64 * 512 + 4, device="cuda", dtype=torch.float16)
    x = base[4:].view(64, 512)             # contiguous, first element 8 bytes past a 16-byte boundary
    w = torch.randn(128, 512, device="cuda", dtype=torch.float16) / 16
    idx = torch.arange(0, 128, device="cuda")
    y = ghost_linear(x, pack_weight(w, idx), idx, strategy="runs")
    ref = (x.float()[:, idx] @ w.float()[:, idx].t()).half()
    torch.testing.assert_close(y, ref, **tols(torch.float16))


@pytest.mark.parametrize("M", [384, 16])
@pytest.mark.parametrize("pattern,expect", [("block", True), ("random", False)])
def test_ghostlinear_frozen_picks_runs(pattern, expect, M):
    K, N = 2048, 1536
    layer = GhostLinear(K, N, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        layer.weight.normal_(0, K ** -0.5)
        layer.bias.normal_()
        dead = torch.from_numpy(dead_columns(K, 0.5, 9, pattern, 128)).cuda()
        layer.weight[:, dead] = 0
    layer.freeze_weight_mask()
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    y = layer(x)
    assert layer._runs is not None and layer._runs[-1] is expect
    torch.testing.assert_close(y.float(), F.linear(x.float(), layer.weight.float(), layer.bias.float()),
                               **tols(torch.bfloat16))
