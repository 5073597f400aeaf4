"""GPU parity of K1 (dead-column mask + compaction) through the C ABI.

Bit-exact against (a) the reference's own outputs (golden fixtures), (b) the
numpy oracle, and (c) the reference suite's known answers
(ghostweight_triton tests/test_mask.py:66-242). Large sizes are checked
through size-independent properties (constructed dead pattern, torch amax).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ghostweight_triton_b200 import _native
from ghostweight_triton_b200.kernels import dead_neuron_mask
from ghostweight_triton_b200.kernels.mask import dead_neuron_mask_compact, alive_indices
from oracle import gw_oracle as O
from tests.golden import gw_golden as G
from tests.golden.gw_inputs import rand_matrix, dead_columns, alive_from_dead, zero_columns

pytestmark = pytest.mark.gpu

NP2T = {"f16": torch.float16, "f32": torch.float32}


def to_dev(a: np.ndarray, dt: str) -> torch.Tensor:
    if dt == "bf16":
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def check_mask_and_compaction(x: torch.Tensor, a_np: np.ndarray, dt: str, thr: float):
    mask, buf, count = dead_neuron_mask_compact(x, thr)
    ref = O.dead_neuron_mask(a_np, thr, dt)
    got = mask.cpu().numpy()
    assert np.array_equal(got, ref), f"mask mismatch at {np.flatnonzero(got != ref)[:10]}"
    n = int(count.item())
    ref_idx = O.alive_indices(ref)
    assert n == len(ref_idx)
    assert np.array_equal(buf[:n].cpu().numpy(), ref_idx)


# ----------------------------------------------------------------- golden (reference outputs)
@pytest.mark.parametrize("name", G.names("mask"))
def test_golden_mask(name):
    meta, inp, exp = G.load(name)
    a = inp["a"]
    x = to_dev(a, meta["dtype"])
    got = dead_neuron_mask(x, threshold=meta["threshold"]).cpu().numpy()
    G.check_exact(got, exp, "mask")
    check_mask_and_compaction(x, a, meta["dtype"], meta["threshold"])


@pytest.mark.parametrize("name", G.names("chain"))
def test_golden_chain_mask_and_alive(name):
    meta, inp, exp = G.load(name)
    x = to_dev(inp["x"], meta["dtype"])
    G.check_exact(dead_neuron_mask(x, 1e-6).cpu().numpy(), exp, "mask")
    G.check_exact(alive_indices(x, 1e-6).cpu().numpy(), exp, "alive")


# ----------------------------------------------------------------- oracle sweep
@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("M,K,sp,pattern", [
    (1, 64, 0.5, "random"), (3, 200, 0.4, "random"), (5, 201, 0.3, "random"),
    (33, 1000, 0.7, "random"), (257, 768, 0.5, "random"), (1000, 4096, 0.9, "random"),
    (129, 4096, 0.5, "block"), (2, 40000, 0.25, "random"),
])
def test_oracle_sweep(dt, M, K, sp, pattern):
    seed = M * 31 + K
    a = zero_columns(rand_matrix((M, K), seed, dt), dead_columns(K, sp, seed, pattern, 64))
    x = to_dev(a, dt)
    check_mask_and_compaction(x, a, dt, 1e-6)


@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("M", [4096, 1000, 77, 9])
def test_single_row_columns_beside_dense_ones(dt, M):
    # Dense columns let their warps stop reading early; columns alive in one
    # row only (the last row, a row in a chunk's ragged last batch, the first
    # row) must still be found whatever batch that row falls in.
    K = 1024
    a = np.zeros((M, K), dtype=rand_matrix((1, 1), 0, dt).dtype)
    dense = rand_matrix((M, K), M + 7, dt)
    a[:, 0::4] = dense[:, 0::4]
    a[M - 1, 1::4] = dense[M - 1, 1::4]
    a[(M * 5) // 7, 2::8] = dense[(M * 5) // 7, 2::8]
    a[0, 3::8] = dense[0, 3::8]
    check_mask_and_compaction(to_dev(a, dt), a, dt, 1e-6)


@pytest.mark.parametrize("thr", [0.0, 0.5, 1.7, -1.0, float("inf")])
def test_thresholds_vs_oracle(thr):
    a = rand_matrix((64, 512), 3, "f16")
    check_mask_and_compaction(to_dev(a, "f16"), a, "f16", thr)


def test_nan_inf_semantics():
    a = rand_matrix((37, 96), 7, "f32")
    a[:, ::3] = 0.0
    a[5, 0] = np.nan          # NaN in a dead column: stays dead
    a[:, 1] = np.nan          # all NaN: dead
    a[7, 2] = np.inf          # inf: alive
    a[:, 4] = -0.0
    for thr in (1e-6, -0.5, 3.0):
        check_mask_and_compaction(to_dev(a, "f32"), a, "f32", thr)


def test_leading_dimension_and_scalar_path():
    """ld > cols through the ABI directly (vector path off because ld is odd)."""
    base = torch.randn(50, 131, device="cuda", dtype=torch.float16)
    base[:, 3:40] = 0
    view = base[:, :100]
    mask = torch.empty(100, dtype=torch.int32, device="cuda")
    idx = torch.empty(100, dtype=torch.int64, device="cuda")
    cnt = torch.empty(1, dtype=torch.int32, device="cuda")
    ws = torch.zeros(_native.load().gw_mask_workspace_bytes(100), dtype=torch.uint8, device="cuda")
    st = _native.load().gw_mask_compact(view.data_ptr(), 0, 50, 100, 131, 1e-6, mask.data_ptr(),
                                        idx.data_ptr(), cnt.data_ptr(), ws.data_ptr(), ws.numel(),
                                        torch.cuda.current_stream().cuda_stream)
    assert st == 0
    ref = O.dead_neuron_mask(view.cpu().numpy(), 1e-6)
    assert np.array_equal(mask.cpu().numpy(), ref)
    assert int(cnt.item()) == ref.sum()
    assert ws.count_nonzero().item() == 0, "workspace must be left zeroed"


def test_workspace_reuse_across_shapes():
    for K in (4096, 64, 1000, 8192, 64):
        a = zero_columns(rand_matrix((17, K), K, "f16"), dead_columns(K, 0.5, K))
        check_mask_and_compaction(to_dev(a, "f16"), a, "f16", 1e-6)
    for ws in _native._ws_cache.values():
        assert ws.count_nonzero().item() == 0


def test_empty_shapes():
    x = torch.zeros(0, 16, device="cuda")
    assert dead_neuron_mask(x).sum().item() == 0
    _, buf, cnt = dead_neuron_mask_compact(torch.zeros(5, 0, device="cuda"))
    assert int(cnt.item()) == 0 and buf.numel() == 0


# ----------------------------------------------------------------- reference-suite known answers
class TestReferenceSuite:
    @pytest.mark.parametrize("M,K", [(1, 128), (4, 256), (128, 768), (1, 3072)])
    def test_output_shape_dtype_device(self, device, M, K):
        m = dead_neuron_mask(torch.randn(M, K, dtype=torch.float16, device=device), threshold=1e-6)
        assert m.shape == (K,) and m.dtype == torch.int32 and m.is_cuda
        assert set(m.unique().tolist()).issubset({0, 1})

    def test_extremes(self, device):
        assert dead_neuron_mask(torch.ones(4, 128, dtype=torch.float16, device=device)).sum() == 128
        assert dead_neuron_mask(torch.zeros(4, 128, dtype=torch.float16, device=device)).sum() == 0
        assert dead_neuron_mask(torch.ones(1, 64, device=device)).sum() == 64
        assert dead_neuron_mask(torch.zeros(1, 64, device=device)).sum() == 0

    def test_threshold_boundary(self, device):
        a = torch.full((4, 64), 0.01, device=device)
        assert dead_neuron_mask(a, threshold=0.01).sum().item() == 0
        a = torch.full((4, 64), 0.01 + 1e-4, device=device)
        assert dead_neuron_mask(a, threshold=0.01).sum().item() == 64
        a = torch.zeros(1, 32, device=device); a[0, :16] = 0.3; a[0, 16:] = 0.7
        m = dead_neuron_mask(a, threshold=0.5)
        assert m[:16].sum().item() == 0 and m[16:].sum().item() == 16

    def test_multirow(self, device):
        a = torch.zeros(8, 64, device=device); a[-1, 0] = 1.0
        m = dead_neuron_mask(a, threshold=1e-6)
        assert m[0].item() == 1 and m[1:].sum().item() == 0

    @pytest.mark.parametrize("K", [3072, 4096, 8192])
    def test_large_k(self, device, K):
        m = dead_neuron_mask(torch.randn(64, K, dtype=torch.float16, device=device))
        assert m.shape == (K,) and m.dtype == torch.int32


# ----------------------------------------------------------------- full-size properties
def test_weight_mask_sharded_mlp_size():
    """W [28672, 8192] bf16 ~ N(0, 1/sqrt(K)) with 44 of 64 128-column blocks zeroed:
    the alive list is exactly the complement (K' = 2560) and equals torch's amax test."""
    K, N = 8192, 28672
    g = torch.Generator(device="cuda").manual_seed(5)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16, generator=g) / K ** 0.5
    dead = dead_columns(K, 0.7, 5, "block", 128)
    w[:, torch.from_numpy(dead).cuda()] = 0
    idx = alive_indices(w, 0.0)
    expect = alive_from_dead(K, dead)
    assert idx.numel() == 2560
    assert np.array_equal(idx.cpu().numpy(), expect)
    ref = (w.abs().float().amax(0) > 0).int()
    assert torch.equal(dead_neuron_mask(w, 0.0), ref)


def test_activation_mask_gemm_sweep_size():
    for pattern in ("random", "block"):
        a = zero_columns(rand_matrix((4096, 4096), 9, "f16"), dead_columns(4096, 0.75, 9, pattern, 64))
        check_mask_and_compaction(to_dev(a, "f16"), a, "f16", 1e-6)
