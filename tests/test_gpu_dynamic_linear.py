"""GPU: the dynamic-mask layer in one launch (gw_dynamic_linear) against the oracle.

The single launch computes the reference's activation mask (kernels/mask.py:
21-59 semantics: running max from 0, NaN ignored, strict fp32 greater-than),
the alive count, and act(x[:, alive] @ W[:, alive]^T + bias) for at most 32
rows. Its mask and count must equal the oracle's bit for bit and its output
must meet the 1e-2 contract (fp16/bf16). The cases cover cluster sizes 1 to 16
(K up to 8192), ragged N, rows 1..32, thresholds that keep or drop every
column, NaN columns, all-dead inputs and layouts the launch refuses.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ghostweight_triton_b200 import GhostLinear, _native
from oracle import gw_oracle as O
from tests.golden.gw_inputs import dead_columns, rand_matrix, zero_columns

pytestmark = pytest.mark.gpu

DT = {"f16": torch.float16, "bf16": torch.bfloat16}


def to_dev(a: np.ndarray) -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def to_np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.cpu().view(torch.int16).numpy().view(np.uint16)
    return t.cpu().numpy()


def run(x, w, thr, bias=None, act=None, with_mask=True):
    M, K = x.shape
    N = w.shape[0]
    y = torch.full((M, N), float("nan"), dtype=x.dtype, device="cuda")
    count = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    mask = torch.full((K,), -1, dtype=torch.int32, device="cuda") if with_mask else None
    st = _native.dynamic_linear(x, w, thr, y, bias=bias, activation=act, count=count, mask=mask)
    return st, y, count, mask


def check(dt, xn, wn, thr, bn=None, act=None):
    ref_mask = O.dead_neuron_mask(xn, thr, dtype=dt)
    idx = O.alive_indices(ref_mask)
    ref = O.ghost_linear(xn, wn, idx, bn, act, dtype=dt)
    st, y, count, mask = run(to_dev(xn), to_dev(wn), thr, None if bn is None else to_dev(bn), act)
    assert st == _native.GW_OK
    torch.cuda.synchronize()
    assert int(count.item()) == idx.size
    assert np.array_equal(mask.cpu().numpy(), ref_mask)
    to32 = lambda a: O.to_f32(a, dt).astype(np.float64)
    yr, rr = to32(to_np(y)), to32(ref)
    # A NaN in an alive column reaches its whole output row, here as in the
    # reference: NaN must sit in the same places, the rest meet the contract.
    assert np.array_equal(np.isnan(yr), np.isnan(rr))
    fin = ~np.isnan(rr)
    err = np.abs(yr[fin] - rr[fin]) - (1e-2 + 1e-2 * np.abs(rr[fin]))
    assert err.size == 0 or np.all(err <= 0), f"outside atol=rtol=1e-2 by {err.max()}"
    return idx.size


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("M,K,N,sp", [
    (1, 768, 3072, 0.5),      # two ranks of 384 columns
    (16, 4096, 4096, 0.5),    # eight ranks of 512
    (32, 3072, 768, 0.6),     # six ranks, 128 / 6 features per slice (uneven)
    (7, 512, 300, 0.3),       # one rank (cluster of one), ragged N
    (20, 8192, 520, 0.9),     # sixteen ranks (non-portable cluster size)
    (32, 4000, 1000, 0.75),   # last rank's range shorter (4000 = 7 x 512 + 416)
    (3, 64, 200, 0.0),        # everything alive, one k atom
])
def test_single_launch_vs_oracle(dt, M, K, N, sp):
    seed = M + 3 * K + 7 * N
    x = zero_columns(rand_matrix((M, K), seed, dt, 0.5), dead_columns(K, sp, seed, "random"))
    w = rand_matrix((N, K), seed + 1, dt, 1.0 / np.sqrt(K))
    b = rand_matrix((N,), seed + 2, dt, 0.5)
    kp = check(dt, x, w, 0.0, b, "gelu_tanh" if M % 2 else None)
    assert kp == K - int(K * sp)


@pytest.mark.parametrize("thr", [-1.0, 0.9, 5.0])
def test_thresholds_keep_or_drop_every_column(thr):
    # thr < 0: the running max starts at 0, so every column is alive; thr = 5:
    # nothing is alive and y = bias.
    x = rand_matrix((12, 1024), 5, "f16", 0.5)
    w = rand_matrix((640, 1024), 6, "f16", 1 / 32)
    b = rand_matrix((640,), 7, "f16", 0.5)
    kp = check("f16", x, w, thr, b, "gelu")
    assert (kp == 1024) if thr < 0 else (kp == 0 if thr >= 5 else 0 < kp < 1024)


def test_nan_column_semantics():
    # A NaN never wins the running max: a column with NaN and zeros is dead, one
    # with NaN and a value above the threshold is alive (kernels/mask.py:55).
    x = rand_matrix((8, 256), 11, "f16", 0.5)
    x[:, :32] = 0
    x[2, 0] = np.float16(np.nan)
    x[3, 1] = np.float16(np.nan)
    x[5, 1] = np.float16(0.75)
    w = rand_matrix((384, 256), 12, "f16", 1 / 16)
    ref_mask = O.dead_neuron_mask(x, 0.0, dtype="f16")
    assert ref_mask[0] == 0 and ref_mask[1] == 1
    check("f16", x, w, 0.0)
    x[3, 1] = np.float16(0.0)                  # the same without the NaN reaching any output
    check("f16", x, w, 0.0)


def test_refused_layouts_return_unsupported():
    x = torch.randn(40, 256, device="cuda", dtype=torch.float16)      # 40 rows > 32
    w = torch.randn(128, 256, device="cuda", dtype=torch.float16)
    st, *_ = run(x, w, 0.0)
    assert st == _native.GW_ERR_UNSUPPORTED
    x = torch.randn(4, 260, device="cuda", dtype=torch.float16)[:, :257]  # K % 8 != 0
    w = torch.randn(128, 257, device="cuda", dtype=torch.float16)
    st, *_ = run(x, w, 0.0)
    assert st == _native.GW_ERR_UNSUPPORTED
    assert _native.device_error(reset=True) == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_ghostlinear_dynamic_small_batch_uses_one_launch(dtype):
    torch.manual_seed(3)
    lin = torch.nn.Linear(2048, 1536).to(device="cuda", dtype=dtype)
    gl = GhostLinear.from_linear(lin, threshold=0.0)
    for step in range(3):
        x = torch.randn(2, 8, 2048, device="cuda", dtype=dtype)
        x[..., (step * 512):(step * 512 + 1024)] = 0            # half the columns dead
        y = gl(x)
        ref = torch.nn.functional.linear(x.float(), lin.weight.float(), lin.bias.float()).to(dtype)
        torch.testing.assert_close(y, ref, atol=1e-2, rtol=1e-2)
        assert gl.current_sparsity == pytest.approx(0.5)
    assert _native.device_error(reset=True) == 0
