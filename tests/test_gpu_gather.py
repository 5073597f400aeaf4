"""GPU parity of K2 (gathers, weight packing) through the C ABI: bit-exact.

Golden fixtures hold the reference's own gather outputs (gather.py:19-94);
packing is checked against the oracle in both weight orientations.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from ghostweight_triton_b200 import _native
from ghostweight_triton_b200.kernels import gather_compact
from ghostweight_triton_b200.kernels.gather import pack_weight, pack_weight_kn
from oracle import gw_oracle as O
from tests.golden import gw_golden as G
from tests.golden.gw_inputs import rand_matrix, dead_columns, alive_from_dead

pytestmark = pytest.mark.gpu


def to_dev(a: np.ndarray) -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def to_np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.cpu().view(torch.int16).numpy().view(np.uint16)
    return t.cpu().numpy()


@pytest.mark.parametrize("name", G.names("gather"))
def test_golden_gather(name):
    meta, inp, exp = G.load(name)
    A_c, W_c = gather_compact(to_dev(inp["A"]), to_dev(inp["W"]), to_dev(exp["idx"]))
    G.check_exact(to_np(A_c), exp, "A_c")
    G.check_exact(to_np(W_c), exp, "W_c")
    assert A_c.is_contiguous() and W_c.is_contiguous()


@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("N,K,sp", [(1, 64, 0.5), (10, 128, 0.0), (136, 320, 0.5),
                                    (3072, 768, 0.5), (512, 4096, 0.9), (77, 1000, 0.33)])
def test_pack_weight_both_orientations(dt, N, K, sp):
    w = rand_matrix((N, K), N + K, dt)
    idx = alive_from_dead(K, dead_columns(K, sp, N + K))
    ld = max(-(-len(idx) // 64) * 64, 64)
    ref = O.pack_weight(w, idx, pad_to=ld)
    wd = to_dev(w)
    idd = torch.from_numpy(idx).cuda()
    p1 = pack_weight(wd, idd)                                   # [N, K] row-major: column gather
    p2 = pack_weight_kn(wd.t().contiguous(), idd)               # [K, N]: transposing gather
    for p in (p1, p2):
        assert p.shape == (N, len(idx)) and p.stride() == (ld, 1)
        full = to_np(p.as_strided((N, ld), (ld, 1)))
        assert np.array_equal(full.view(np.uint8), ref.view(np.uint8))


def test_unsorted_repeated_and_reversed_indices():
    A = rand_matrix((9, 300), 1, "f16")
    W = rand_matrix((300, 70), 2, "f16")
    for idx in (np.arange(299, -1, -1), np.array([5, 5, 0, 299, 17, 5]),
                np.random.default_rng(4).permutation(300)[:123]):
        A_c, W_c = gather_compact(to_dev(A), to_dev(W), torch.from_numpy(idx).cuda())
        assert np.array_equal(to_np(A_c), O.gather_columns(A, idx))
        assert np.array_equal(to_np(W_c), O.gather_rows(W, idx))


def test_int32_indices_accepted():
    A = torch.randn(4, 64, device="cuda")
    W = torch.randn(64, 8, device="cuda")
    idx = torch.arange(0, 64, 3, device="cuda", dtype=torch.int32)
    A_c, W_c = gather_compact(A, W, idx)
    assert torch.equal(A_c, A[:, idx.long()]) and torch.equal(W_c, W[idx.long()])


def test_out_of_range_index_reads_zero_and_flags():
    _native.device_error(reset=True)
    A = torch.randn(4, 16, device="cuda")
    W = torch.randn(16, 8, device="cuda")
    idx = torch.tensor([0, 99, 3], device="cuda")
    A_c, W_c = gather_compact(A, W, idx)
    assert torch.equal(A_c[:, 1], torch.zeros(4, device="cuda"))
    assert torch.equal(W_c[1], torch.zeros(8, device="cuda"))
    assert torch.equal(A_c[:, 2], A[:, 3])
    assert _native.device_error(reset=True) & _native.DEVICE_ERR_BAD_INDEX
    assert _native.validate_indices(idx, 16) == 1


# ----------------------------------------------------------------- many-row gathers
# Bit-exact against the oracle over row counts, widths and dead patterns,
# including rows shorter than a 128-byte line, ragged widths and row counts
# that are not a multiple of the CTA's warps.
@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("rows,cols,sp,pattern", [
    (4096, 4096, 0.5, "random"),
    (4096, 4096, 0.0, "random"),
    (1024, 4096, 0.9, "random"),
    (2048, 4096, 0.75, "block"),    # 64-column dead blocks
    (1024, 8192, 0.6875, "block"),  # the sharded-MLP pattern (128-column blocks)
    (1500, 72, 0.5, "random"),
    (1031, 1000, 0.33, "random"),
    (1000, 4096, 0.9, "random"),
    (300, 4096, 0.75, "block"),
    (257, 1000, 0.33, "random"),
    (512, 8192, 0.6875, "block"),
])
def test_window_gather_bit_exact(dt, rows, cols, sp, pattern):
    x = rand_matrix((rows, cols), rows + cols, dt)
    idx = alive_from_dead(cols, dead_columns(cols, sp, rows, pattern, 128 if cols == 8192 else 64))
    xd = to_dev(x)
    idd = torch.from_numpy(idx).cuda()
    ld = max(-(-len(idx) // 64) * 64, 64)
    out = torch.full((rows, ld), 7, dtype=xd.dtype, device="cuda")
    _native.gather_columns(xd, idd, out, pad_to=ld)
    ref = O.gather_columns(x, idx)
    got = to_np(out)
    assert np.array_equal(got[:, :len(idx)].view(np.uint8), np.ascontiguousarray(ref).view(np.uint8))
    assert (got[:, len(idx):] == 0).all()          # padding columns written as zeros


@pytest.mark.parametrize("rows", [512, 1024])
@pytest.mark.parametrize("case", ["unsorted", "repeated", "bad_index", "wide_window"])
def test_irregular_index_lists(case, rows):
    """Unsorted, repeated and out-of-range indices, and a dense run then every 8th column."""
    cols = 4096
    x = rand_matrix((rows, cols), 11, "f16")
    rng = np.random.default_rng(5)
    if case == "unsorted":
        idx = rng.permutation(cols)[:2048]
    elif case == "repeated":
        idx = np.sort(rng.integers(0, cols, 2048))
    elif case == "bad_index":
        idx = np.sort(rng.permutation(cols)[:2048])
        idx[700] = cols + 5
    else:                                          # dense, then every 8th column: windows too wide
        idx = np.concatenate([np.arange(0, 1024), np.arange(1024, cols, 8)])
    _native.device_error(reset=True)
    out = torch.empty(rows, len(idx), dtype=torch.float16, device="cuda")
    _native.gather_columns(to_dev(x), torch.from_numpy(idx).cuda(), out)
    ref = O.gather_columns(x, np.where(idx < cols, idx, 0))
    if case == "bad_index":
        ref[:, 700] = 0
        assert _native.device_error(reset=True) & _native.DEVICE_ERR_BAD_INDEX
    assert np.array_equal(to_np(out), ref)


class TestReferenceSuite:
    """ghostweight_triton tests/test_gather.py:66-216, on B200."""

    @pytest.mark.parametrize("M,K,N,sparsity", [(1, 128, 256, 0.0), (1, 128, 256, 0.5),
                                                (16, 768, 3072, 0.3), (128, 768, 3072, 0.7),
                                                (128, 3072, 768, 0.5)])
    def test_output_shapes(self, device, M, K, N, sparsity):
        A = torch.randn(M, K, dtype=torch.float16, device=device)
        W = torch.randn(K, N, dtype=torch.float16, device=device)
        idx = torch.from_numpy(alive_from_dead(K, dead_columns(K, sparsity, 7))).to(device)
        A_c, W_c = gather_compact(A, W, idx)
        assert A_c.shape == (M, idx.numel()) and W_c.shape == (idx.numel(), N)

    def test_identity_and_single(self, device):
        A = torch.randn(4, 32, device=device)
        W = torch.randn(32, 16, device=device)
        A_c, W_c = gather_compact(A, W, torch.arange(32, device=device))
        assert torch.equal(A_c, A) and torch.equal(W_c, W)
        A = torch.arange(16, dtype=torch.float32, device=device).unsqueeze(0)
        W = torch.eye(16, 8, device=device)
        A_c, W_c = gather_compact(A, W, torch.tensor([5], device=device))
        assert A_c[0, 0].item() == 5.0 and torch.equal(W_c[0], W[5])

    @pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.bfloat16])
    def test_dtype_device_contiguity(self, device, dtype):
        A = torch.randn(4, 64, dtype=dtype, device=device)
        W = torch.randn(64, 32, dtype=dtype, device=device)
        A_c, W_c = gather_compact(A, W, torch.arange(32, device=device))
        assert A_c.dtype == dtype and W_c.dtype == dtype
        assert A_c.is_cuda and W_c.is_cuda and A_c.is_contiguous() and W_c.is_contiguous()


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_gather_unaligned_output_rows(dt):
    # ld_dst = kp + 5 = 1026 (output rows not 16-byte aligned), kp % 8 != 0.
    rows, cols = 1100, 2048
    x = rand_matrix((rows, cols), 21, dt)
    idx = np.sort(np.random.default_rng(6).permutation(cols)[:1021])
    base = torch.full((rows, len(idx) + 5), 9, dtype=torch.float16 if dt == "f16" else torch.bfloat16,
                      device="cuda")
    out = base[:, :len(idx)]
    _native.gather_columns(to_dev(x), torch.from_numpy(idx).cuda(), out)
    assert np.array_equal(to_np(out.contiguous()), O.gather_columns(x, idx))
    assert (base[:, len(idx):].float() == 9).all()        # nothing written past the width


@pytest.mark.parametrize("n", [0, 1, 700, 2048])
def test_gather_device_count(n):
    # The count lives on the device: columns [n, round_up(max(n, 1), 64)) are
    # zero, the ones past that untouched.
    rows, cols = 1024, 4096
    x = rand_matrix((rows, cols), 31, "f16")
    idx = np.sort(np.random.default_rng(7).permutation(cols)[:2048])
    out = torch.full((rows, 2048), 5, dtype=torch.float16, device="cuda")
    n_dev = torch.tensor([n], dtype=torch.int32, device="cuda")
    _native.gather_columns_dev(to_dev(x), torch.from_numpy(idx).cuda(), n_dev, out, pad_to=2048)
    got = to_np(out)
    assert np.array_equal(got[:, :n], O.gather_columns(x, idx[:n]))
    edge = max(-(-max(n, 1) // 64) * 64, 64)
    assert (got[:, n:edge] == 0).all()
    assert (got[:, edge:] == 5).all()


@pytest.mark.parametrize("case", ["offset_runs", "runs_then_scattered", "run_across_chunks", "all"])
def test_gather_runs_and_mixed_chunks(case):
    # Chunks whose lanes' 8 outputs are 8 aligned consecutive columns move
    # 16-byte vectors; the others gather per element. Both must be exact.
    rows, cols = 700, 4096
    x = rand_matrix((rows, cols), 13, "bf16")
    rng = np.random.default_rng(9)
    if case == "offset_runs":                       # runs starting 4 columns past an 8-column boundary
        idx = np.concatenate([np.arange(4 + 128 * b, 4 + 128 * b + 64) for b in range(16)])
    elif case == "runs_then_scattered":
        idx = np.concatenate([np.arange(512, 1024), np.sort(rng.choice(np.arange(1024, cols), 700, replace=False))])
    elif case == "run_across_chunks":               # one run crossing several 256-column chunks, ragged end
        idx = np.arange(1000, 1000 + 1000)
    else:
        idx = np.arange(cols)
    out = torch.full((rows, len(idx)), 3, dtype=torch.bfloat16, device="cuda")
    _native.gather_columns(to_dev(x), torch.from_numpy(idx).cuda(), out)
    assert np.array_equal(to_np(out), O.gather_columns(x, idx))
