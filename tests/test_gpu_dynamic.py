"""GPU: the dynamic activation mask without a host synchronisation.

The alive count written by the mask kernel stays on the device; the packing,
the gather and the GEMM read it there. Results must equal the oracle on the
same inputs (fp16/bf16 1e-2, fp32 1e-4 as in the reference's
tests/test_matmul.py:68-72), and a dynamic GhostLinear forward must be
capturable in a CUDA graph whose replays follow each new input's mask.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from ghostweight_triton_b200 import GhostLinear, _native
from ghostweight_triton_b200.kernels.gather import pack_weight_dev
from ghostweight_triton_b200.kernels.mask import dead_neuron_mask_compact
from ghostweight_triton_b200.kernels.matmul import ghost_linear_dev
from oracle import gw_oracle as O
from tests.conftest import tols
from tests.golden.gw_inputs import dead_columns, rand_matrix, zero_columns
from tests.test_gpu_matmul import TOL, assert_close, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("M,K,N,sp", [(4096, 4096, 4096, 0.5), (300, 1000, 520, 0.9), (7, 768, 3072, 0.25),
                                      (129, 640, 136, 1.0), (64, 256, 64, 0.0)])
def test_gather_gemm_device_count_vs_oracle(dt, M, K, N, sp):
    """mask -> device count -> pack -> gather -> GEMM, nothing read on the host."""
    seed = M + K + N
    dead = dead_columns(K, sp, seed, "random")
    x = zero_columns(rand_matrix((M, K), seed, dt, 0.5), dead)
    w = rand_matrix((N, K), seed + 1, dt, 1.0 / np.sqrt(K))
    b = rand_matrix((N,), seed + 2, dt, 0.5)
    xd, wd, bd = to_dev(x), to_dev(w), to_dev(b)
    _native.device_error(reset=True)
    _, buf, count = dead_neuron_mask_compact(xd, 0.0, want_mask=False)
    wp = pack_weight_dev(wd, buf, count)
    y = ghost_linear_dev(xd, wp, buf, count, bias=bd, activation="gelu")
    idx = np.setdiff1d(np.arange(K), dead)
    assert int(count.item()) == idx.size
    ref = O.ghost_linear(x, w, idx, b, "gelu", dtype=dt) if M * K * N <= 2 ** 31 else None
    if ref is not None:
        assert_close(to_np(y), ref, dt, f"device count {dt} {M}x{K}x{N} s={sp}")
    else:
        full = F.gelu(F.linear(xd.float(), wd.float(), bd.float()))
        torch.testing.assert_close(y.float(), full, atol=TOL[dt][0] * 3, rtol=TOL[dt][1])
    assert _native.device_error(reset=True) == 0


@pytest.mark.parametrize("transposed", [False, True])
def test_pack_device_count_zero_fill(transposed):
    """Columns [n, round_up(max(n, 1), 64)) are zero; the rest of the buffer is not written."""
    N, K, n = 96, 300, 70
    w = torch.randn(K, N, device="cuda").t() if transposed else torch.randn(N, K, device="cuda")
    idx = torch.randperm(K, device="cuda")
    cnt = torch.tensor([n], dtype=torch.int32, device="cuda")
    ld = 320
    buf = torch.full((N, ld), 7.0, device="cuda")
    if transposed:
        _native.gather_rows_t_dev(w.t(), idx, cnt, buf, pad_to=ld)
    else:
        _native.gather_columns_dev(w, idx, cnt, buf, pad_to=ld)
    torch.testing.assert_close(buf[:, :n], w[:, idx[:n]])
    assert torch.count_nonzero(buf[:, n:128]).item() == 0
    assert bool((buf[:, 128:] == 7.0).all())
    cnt.zero_()
    buf.fill_(7.0)
    _native.gather_columns_dev(w.contiguous(), idx, cnt, buf, pad_to=ld)
    assert torch.count_nonzero(buf[:, :64]).item() == 0 and bool((buf[:, 64:] == 7.0).all())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_dynamic_ghostlinear_in_cuda_graph(dtype):
    """A dynamic-mask forward is captured once; every replay follows its input's own mask."""
    torch.manual_seed(3)
    K, N, M = 1024, 768, 256
    lin = nn.Linear(K, N).to(device="cuda", dtype=dtype)
    gl = GhostLinear.from_linear(lin, threshold=0.0, min_sparsity_to_activate=0.0)
    x_static = torch.randn(M, K, device="cuda", dtype=dtype)
    x_static[:, ::3] = 0
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.no_grad():
        for _ in range(2):
            gl(x_static)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.no_grad(), torch.cuda.graph(g):
        y_static = gl(x_static)
    tol = tols(dtype)
    for trial, step in enumerate((2, 5, 7)):
        x = torch.randn(M, K, device="cuda", dtype=dtype)
        dead = torch.arange(0, K, step, device="cuda")
        x[:, dead] = 0
        x_static.copy_(x)
        g.replay()
        ref = F.linear(x.float(), lin.weight.float(), lin.bias.float()).to(dtype)
        torch.testing.assert_close(y_static, ref, **tol)
        assert gl.current_sparsity == pytest.approx(dead.numel() / K)
    del g


def test_sync_free_dense_fallback_follows_previous_forward():
    """With the count on the device, the dense-fallback choice uses the previous forward's
    sparsity once it has reached the host; both paths give the dense layer's result."""
    torch.manual_seed(4)
    lin = nn.Linear(512, 256).to("cuda")
    gl = GhostLinear.from_linear(lin, threshold=0.0, min_sparsity_to_activate=0.5)
    dense_x = torch.randn(8, 512, device="cuda")
    sparse_x = torch.randn(8, 512, device="cuda")
    sparse_x[:, ::4] = 0
    sparse_x[:, 1::4] = 0
    sparse_x[:, 2::4] = 0
    for x in (dense_x, dense_x, sparse_x, sparse_x):
        y = gl(x)
        torch.cuda.synchronize()
        torch.testing.assert_close(y, F.linear(x, lin.weight, lin.bias), atol=1e-4, rtol=1e-4)
    assert gl.current_sparsity == pytest.approx(0.75)
    gl.sync_free = False
    torch.testing.assert_close(gl(sparse_x), F.linear(sparse_x, lin.weight, lin.bias), atol=1e-4, rtol=1e-4)
    assert gl.current_sparsity == pytest.approx(0.75)


def test_device_count_edge_shapes():
    """M = 0 / N = 0 return at once; an upper bound of 0 gives act(bias); counts above the
    bound are clamped to it."""
    x = torch.randn(5, 64, device="cuda", dtype=torch.float16)
    w = torch.randn(24, 64, device="cuda", dtype=torch.float16) / 8
    b = torch.randn(24, device="cuda", dtype=torch.float16)
    cnt = torch.tensor([9], dtype=torch.int32, device="cuda")
    empty = torch.empty(0, dtype=torch.int64, device="cuda")
    wp = torch.zeros(24, 64, device="cuda", dtype=torch.float16)
    y = torch.empty(5, 24, device="cuda", dtype=torch.float16)
    _native.gather_gemm_dev(x, wp, empty, cnt, y, bias=b)
    torch.testing.assert_close(y, b.expand(5, 24))
    _native.gather_gemm_dev(x[:0], wp, empty, cnt, y[:0], bias=b)
    idx = torch.arange(0, 64, 2, device="cuda")                     # 32 entries, count says 40
    cnt.fill_(40)
    wp = pack_weight_dev(w, idx, cnt)
    _native.gather_gemm_dev(x, wp, idx, cnt, y, bias=b)
    ref = (x.float()[:, idx] @ w.float()[:, idx].t() + b.float()).half()
    torch.testing.assert_close(y, ref, **tols(torch.float16))


def test_frozen_layer_captured_without_warmup():
    """Freezing decides the runs strategy at once, so the first frozen forward can run
    inside CUDA-graph capture (no host read there)."""
    torch.manual_seed(6)
    lin = nn.Linear(1024, 512).half().cuda()
    with torch.no_grad():
        lin.weight[:, 128:384] = 0                # whole 64-column blocks: the runs strategy
    gl = GhostLinear.from_linear(lin, threshold=0.0)
    gl.freeze_weight_mask()
    assert gl._runs is not None and gl._runs[-1] is True
    x = torch.randn(256, 1024, device="cuda", dtype=torch.float16)
    g = torch.cuda.CUDAGraph()
    with torch.no_grad(), torch.cuda.graph(g):
        y = gl(x)
    x.copy_(torch.randn_like(x))
    g.replay()
    torch.testing.assert_close(y, F.linear(x, lin.weight, lin.bias), **tols(torch.float16))
    del g
