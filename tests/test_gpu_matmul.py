"""GPU parity of K3 (tcgen05 gather-GEMM, exact-fp32 gather-GEMM) through the C ABI.

Tolerances are the reference's own (tests/test_matmul.py:68-72): fp16/bf16
atol = rtol = 1e-2, fp32 atol = rtol = 1e-4. Golden fixtures hold the
reference's ghostweight_matmul outputs; the oracle covers bf16, bias and the
GELU epilogues; full-size cases are checked against the dense fp32 product
(dead columns are zero, so the sparse and dense products agree).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from ghostweight_triton_b200 import _native
from ghostweight_triton_b200.kernels import ghostweight_matmul
from ghostweight_triton_b200.kernels.gather import pack_weight
from ghostweight_triton_b200.kernels.matmul import ghost_linear, packed_linear
from oracle import gw_oracle as O
from tests.conftest import tols
from tests.golden import gw_golden as G
from tests.golden.gw_inputs import rand_matrix, dead_columns, alive_from_dead, zero_columns

pytestmark = pytest.mark.gpu

TOL = {"f16": (1e-2, 1e-2), "bf16": (1e-2, 1e-2), "f32": (1e-4, 1e-4)}
DT = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def to_dev(a: np.ndarray) -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def to_np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.cpu().view(torch.int16).numpy().view(np.uint16)
    return t.cpu().numpy()


def as_f32(a: np.ndarray, dt: str) -> np.ndarray:
    return O.to_f32(a, dt)


def assert_close(got: np.ndarray, ref: np.ndarray, dt: str, what: str = ""):
    atol, rtol = TOL[dt]
    g, r = as_f32(got, dt).astype(np.float64), as_f32(ref, dt).astype(np.float64)
    bad = ~(np.abs(g - r) <= atol + rtol * np.abs(r))
    assert not bad.any(), f"{what}: {bad.sum()}/{bad.size} off, max err {np.abs(g - r).max():.3g}"


# ----------------------------------------------------------------- golden (reference outputs)
@pytest.mark.parametrize("name", G.names("matmul"))
def test_golden_matmul(name):
    meta, inp, exp = G.load(name)
    C = ghostweight_matmul(to_dev(inp["A"]), to_dev(inp["W"]), to_dev(exp["idx"]))
    atol, rtol = TOL[meta["dtype"]]
    G.check_close(to_np(C), exp, "C", atol, rtol)


# ----------------------------------------------------------------- oracle sweep (linear form)
@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("M,K,N,sp,pattern", [
    (1, 128, 256, 0.5, "random"), (7, 64, 10, 0.0, "random"), (128, 768, 3072, 0.5, "random"),
    (200, 320, 136, 0.5, "random"), (129, 1000, 520, 0.9, "random"), (300, 4096, 384, 0.75, "block"),
    (1024, 2048, 1024, 0.5, "random"), (16, 4096, 4096, 0.5, "random"), (77, 130, 33, 0.1, "random"),
])
@pytest.mark.parametrize("bias,act", [(False, None), (True, None), (True, "gelu"), (True, "gelu_tanh")])
@pytest.mark.parametrize("strategy", ["overlap", "pregather", "fused"])
def test_ghost_linear_vs_oracle(dt, M, K, N, sp, pattern, bias, act, strategy):
    seed = M + 3 * K + 7 * N
    x = rand_matrix((M, K), seed, dt, 0.5)
    w = rand_matrix((N, K), seed + 1, dt, 1.0 / np.sqrt(K))
    b = rand_matrix((N,), seed + 2, dt, 0.5) if bias else None
    idx = alive_from_dead(K, dead_columns(K, sp, seed, pattern, 64))
    ref = O.ghost_linear(x, w, idx, b, act, dtype=dt)
    xd, wd, idd = to_dev(x), to_dev(w), torch.from_numpy(idx).cuda()
    y = ghost_linear(xd, pack_weight(wd, idd), idd, bias=to_dev(b) if bias else None, activation=act,
                     strategy=strategy)
    assert y.dtype == DT[dt] and y.shape == (M, N)
    assert_close(to_np(y), ref, dt, f"{dt} {M}x{K}x{N} s={sp} bias={bias} act={act}")


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_packed_gemm_tma_operands(dt):
    M, K, N = 333, 512, 264
    a = rand_matrix((M, K), 1, dt)
    w = rand_matrix((N, K), 2, dt, 1 / np.sqrt(K))
    b = rand_matrix((N,), 3, dt)
    ref = O.ghost_linear(a, w, np.arange(K), b, "gelu", dtype=dt)
    wd = pack_weight(to_dev(w), torch.arange(K, device="cuda"))
    y = packed_linear(to_dev(a), wd, bias=to_dev(b), activation="gelu")
    assert_close(to_np(y), ref, dt, "packed")


def test_empty_alive_gives_bias_or_zeros():
    x = torch.randn(5, 64, device="cuda", dtype=torch.float16)
    w = torch.randn(64, 24, device="cuda", dtype=torch.float16)
    C = ghostweight_matmul(x, w, torch.empty(0, dtype=torch.int64, device="cuda"))
    assert C.shape == (5, 24) and torch.count_nonzero(C).item() == 0
    b = torch.randn(24, device="cuda", dtype=torch.float16)
    C = ghostweight_matmul(x, w, torch.empty(0, dtype=torch.int64, device="cuda"), bias=b)
    assert torch.equal(C, b.expand(5, 24))


def test_misaligned_output_leading_dimension():
    """ldy not a multiple of 8 forces the scalar epilogue store path."""
    x = torch.randn(70, 256, device="cuda", dtype=torch.float16)
    w = torch.randn(100, 256, device="cuda", dtype=torch.float16) / 16
    idx = torch.arange(0, 256, 2, device="cuda")
    big = torch.zeros(70, 101, device="cuda", dtype=torch.float16)
    y = big[:, :100]
    _native.gather_gemm(x, pack_weight(w, idx), idx, y)
    ref = (x.float()[:, idx] @ w.float()[:, idx].t()).half()
    torch.testing.assert_close(y, ref, **tols(torch.float16))
    assert torch.count_nonzero(big[:, 100]).item() == 0


def test_repeated_indices_and_out_of_range():
    _native.device_error(reset=True)
    x = torch.randn(20, 64, device="cuda", dtype=torch.float16)
    w = torch.randn(64, 48, device="cuda", dtype=torch.float16) / 8
    idx = torch.tensor([3, 3, 7, 63, 0, 3], device="cuda")
    C = ghostweight_matmul(x, w, idx)
    ref = (x.float()[:, idx] @ w.float()[idx, :]).half()
    torch.testing.assert_close(C, ref, **tols(torch.float16))
    assert _native.device_error(reset=True) == 0
    bad = torch.tensor([3, 64, 7], device="cuda")
    C = ghostweight_matmul(x, w, bad)       # index 64 is out of range: contributes zero
    keep = torch.tensor([3, 7], device="cuda")
    torch.testing.assert_close(C, (x.float()[:, keep] @ w.float()[keep, :]).half(), **tols(torch.float16))
    assert _native.device_error(reset=True) & _native.DEVICE_ERR_BAD_INDEX


@pytest.mark.parametrize("strategy", ["overlap", "pregather"])
def test_workspace_reuse_between_shapes(strategy):
    """One workspace serves successive calls of different K' (stale counters must not leak)."""
    ws = torch.empty(64 << 20, dtype=torch.uint8, device="cuda")
    for M, K, N, kp in [(512, 1024, 384, 1000), (300, 512, 256, 64), (1024, 2048, 512, 1536),
                        (4096, 4096, 4096, 2048), (2500, 1024, 4000, 900), (4096, 4096, 4096, 1024)]:
        x = torch.randn(M, K, device="cuda", dtype=torch.float16)
        w = (torch.randn(N, K, device="cuda") / K ** 0.5).half()
        idx = torch.sort(torch.randperm(K, device="cuda")[:kp]).values
        y = torch.empty(M, N, device="cuda", dtype=torch.float16)
        _native.gather_gemm(x, pack_weight(w, idx), idx, y, strategy=strategy, workspace=ws)
        ref = (x.float()[:, idx] @ w.float()[:, idx].t()).half()
        torch.testing.assert_close(y, ref, **tols(torch.float16))


# ----------------------------------------------------------------- CTA-pair GEMM, TMA-store epilogue
@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("M,K,N,kp,bias,act", [
    (4096, 4096, 4096, 2048, False, None),      # 256 pair tiles: 222 whole, the last 34 as 68 halves
    (2500, 4096, 4000, 2048, True, "gelu"),     # ragged last tile row and column: TMA clips the store
    (4096, 1024, 3900, 512, True, None),        # a last-wave half tile entirely past N is skipped
    (2500, 512, 4000, 100, True, "gelu_tanh"),  # 2 k-blocks, the second one zero-filled past K'
    (4096, 1024, 4608, 1000, True, None),       # 288 tiles, 3.9 waves
])
@pytest.mark.parametrize("strategy", ["pregather", "overlap"])
def test_pair_gemm_ragged_vs_fp32(dt, M, K, N, kp, bias, act, strategy):
    torch_dt = DT[dt]
    g = torch.Generator(device="cuda").manual_seed(M + N + kp)
    x = torch.randn(M, K, device="cuda", dtype=torch_dt, generator=g)
    w = (torch.randn(N, K, device="cuda", generator=g) / kp ** 0.5).to(torch_dt)
    b = torch.randn(N, device="cuda", generator=g).to(torch_dt) if bias else None
    idx = torch.sort(torch.randperm(K, device="cuda", generator=g)[:kp]).values
    wp = pack_weight(w, idx)
    ws = torch.empty(_native.gather_gemm_workspace_bytes(M, kp, torch_dt), dtype=torch.uint8, device="cuda")
    big = torch.full((M, N + 8), float("nan"), device="cuda", dtype=torch_dt)
    y = big[:, :N]                             # ldy = N + 8: still 16-byte rows, columns past N untouched
    _native.gather_gemm(x, wp, idx, y, bias=b, activation=act, strategy=strategy, workspace=ws)
    ref = F.linear(x.float()[:, idx], w.float()[:, idx], None if b is None else b.float())
    if act == "gelu":
        ref = F.gelu(ref)
    elif act == "gelu_tanh":
        ref = F.gelu(ref, approximate="tanh")
    torch.testing.assert_close(y, ref.to(torch_dt), **tols(torch_dt))
    assert torch.isnan(big[:, N:]).all()
    assert _native.device_error(reset=False) & _native.DEVICE_ERR_WAIT_TIMEOUT == 0


# ----------------------------------------------------------------- pair GEMM gathering x' itself
def _overlap_case(M, K, N, kp, seed, dtype=torch.float16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", dtype=dtype, generator=g)
    w = (torch.randn(N, K, device="cuda", generator=g) / kp ** 0.5).to(dtype)
    idx = torch.sort(torch.randperm(K, device="cuda", generator=g)[:kp]).values
    return x, w, idx, pack_weight(w, idx)


def test_overlap_garbage_workspace_and_repeated_calls():
    """The in-kernel gather's flags carry a per-call number kept in the workspace header:
    a workspace full of random bytes works, and successive calls with new inputs in the
    same workspace never read an earlier call's x' (each result matches its own inputs)."""
    M, K, N, kp = 4096, 4096, 4096, 2048
    _, w, idx, wp = _overlap_case(M, K, N, kp, 5)
    nbytes = _native.gather_gemm_workspace_bytes(M, kp, torch.float16)
    ws = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device="cuda")
    y = torch.empty(M, N, device="cuda", dtype=torch.float16)
    g = torch.Generator(device="cuda").manual_seed(9)
    for step in range(4):
        x = torch.randn(M, K, device="cuda", dtype=torch.float16, generator=g)
        _native.gather_gemm(x, wp, idx, y, strategy="overlap", workspace=ws)
        ref = (x.float()[:, idx] @ w.float()[:, idx].t()).half()
        torch.testing.assert_close(y, ref, **tols(torch.float16), msg=f"call {step}")
    assert _native.device_error(reset=True) == 0


def test_overlap_shares_workspace_with_pregather_of_other_shapes():
    """x' of a pregather call of another shape lands where the overlap call keeps its flags."""
    ws = torch.empty(96 << 20, dtype=torch.uint8, device="cuda")
    for M, K, N, kp, strat in [(128, 4096, 4096, 4000, "pregather"), (4096, 4096, 4096, 2048, "overlap"),
                               (512, 8192, 1024, 8000, "pregather"), (4096, 4096, 4096, 1024, "overlap"),
                               (2500, 4096, 4000, 2048, "overlap")]:
        x, w, idx, wp = _overlap_case(M, K, N, kp, M + kp)
        y = torch.empty(M, N, device="cuda", dtype=torch.float16)
        _native.gather_gemm(x, wp, idx, y, strategy=strat, workspace=ws)
        ref = (x.float()[:, idx] @ w.float()[:, idx].t()).half()
        torch.testing.assert_close(y, ref, **tols(torch.float16), msg=f"{strat} {M}x{K}x{N} K'={kp}")
    assert _native.device_error(reset=True) == 0


def test_overlap_replayed_from_a_cuda_graph():
    """Every replay of a captured call reads a new call number from the workspace header."""
    M, K, N, kp = 4096, 2048, 4096, 1536
    x, w, idx, wp = _overlap_case(M, K, N, kp, 21)
    ws = torch.empty(_native.gather_gemm_workspace_bytes(M, kp, torch.float16), dtype=torch.uint8,
                     device="cuda")
    y = torch.empty(M, N, device="cuda", dtype=torch.float16)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        _native.gather_gemm(x, wp, idx, y, strategy="overlap", workspace=ws)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _native.gather_gemm(x, wp, idx, y, strategy="overlap", workspace=ws)
    g = torch.Generator(device="cuda").manual_seed(4)
    for rep in range(3):
        x.copy_(torch.randn(M, K, device="cuda", dtype=torch.float16, generator=g))
        graph.replay()
        torch.cuda.synchronize()
        ref = (x.float()[:, idx] @ w.float()[:, idx].t()).half()
        torch.testing.assert_close(y, ref, **tols(torch.float16), msg=f"replay {rep}")
    del graph
    assert _native.device_error(reset=True) == 0


def test_overlap_bad_index_reads_zero_and_flags():
    M, K, N, kp = 4096, 4096, 4096, 1024
    x, w, idx, wp = _overlap_case(M, K, N, kp, 33)
    bad = idx.clone()
    bad[100] = K + 5                               # outside [0, K)
    _native.device_error(reset=True)
    y = torch.empty(M, N, device="cuda", dtype=torch.float16)
    _native.gather_gemm(x, wp, bad, y, strategy="overlap",
                        workspace=_native.gemm_workspace(x.device, _native.gather_gemm_workspace_bytes(
                            M, kp, torch.float16)))
    xs = x.float()[:, idx]
    xs[:, 100] = 0                                 # the bad column contributes zero
    ref = (xs @ w.float()[:, idx].t()).half()
    torch.testing.assert_close(y, ref, **tols(torch.float16))
    assert _native.device_error(reset=True) == _native.DEVICE_ERR_BAD_INDEX


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("M,K,N,kp,bias,act", [
    (4096, 768, 768, 384, True, None),          # 64 pair tiles of 256 x 192 (GPT-2 projection)
    (8192, 768, 768, 308, True, "gelu"),        # 128 tiles, two rounds (DistilBERT projection)
    (4000, 3072, 760, 1229, False, "gelu_tanh"),  # ragged M and N
])
def test_pair_gemm_192_wide_tiles_vs_fp32(dt, M, K, N, kp, bias, act):
    """Output widths where 192-wide pair tiles fill the SM pairs better than 256-wide ones."""
    torch_dt = DT[dt]
    g = torch.Generator(device="cuda").manual_seed(N + kp)
    x = torch.randn(M, K, device="cuda", dtype=torch_dt, generator=g)
    w = (torch.randn(N, K, device="cuda", generator=g) / kp ** 0.5).to(torch_dt)
    b = torch.randn(N, device="cuda", generator=g).to(torch_dt) if bias else None
    idx = torch.sort(torch.randperm(K, device="cuda", generator=g)[:kp]).values
    y = ghost_linear(x, pack_weight(w, idx), idx, bias=b, activation=act, strategy="pregather")
    rows = torch.arange(0, M, 37, device="cuda")
    ref = F.linear(x[rows].float()[:, idx], w.float()[:, idx], None if b is None else b.float())
    if act == "gelu":
        ref = F.gelu(ref)
    elif act == "gelu_tanh":
        ref = F.gelu(ref, approximate="tanh")
    torch.testing.assert_close(y[rows], ref.to(torch_dt), **tols(torch_dt))


def test_pair_gemm_unaligned_ldy_direct_stores():
    """ldy not a multiple of 8 on a pair-kernel shape: the epilogue falls back to direct stores."""
    M, K, N, kp = 2048, 1024, 2048, 512
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(M, K, device="cuda", dtype=torch.float16, generator=g)
    w = (torch.randn(N, K, device="cuda", generator=g) / kp ** 0.5).half()
    idx = torch.sort(torch.randperm(K, device="cuda", generator=g)[:kp]).values
    big = torch.zeros(M, N + 3, device="cuda", dtype=torch.float16)
    y = big[:, :N]
    ws = torch.empty(_native.gather_gemm_workspace_bytes(M, kp, torch.float16), dtype=torch.uint8, device="cuda")
    _native.gather_gemm(x, pack_weight(w, idx), idx, y, strategy="pregather", workspace=ws)
    ref = (x.float()[:, idx] @ w.float()[:, idx].t()).half()
    torch.testing.assert_close(y, ref, **tols(torch.float16))
    assert torch.count_nonzero(big[:, N:]).item() == 0


def test_chained_layers_pdl():
    """Layer 2's gather reads layer 1's output: the programmatic-dependent launches must order them."""
    M, K = 4096, 4096
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(M, K, device="cuda", dtype=torch.float16, generator=g)
    ws = torch.empty(64 << 20, dtype=torch.uint8, device="cuda")
    h = x
    ref = x.float()
    for layer in range(4):
        w = (torch.randn(K, K, device="cuda", generator=g) / 45.0).half()
        idx = torch.sort(torch.randperm(K, device="cuda", generator=g)[:2048]).values
        out = torch.empty(M, K, device="cuda", dtype=torch.float16)
        _native.gather_gemm(h, pack_weight(w, idx), idx, out, strategy="pregather", workspace=ws)
        h = out
        ref = (ref.half().float()[:, idx] @ w.float()[:, idx].t())
    torch.testing.assert_close(h, ref.half(), **tols(torch.float16))


@pytest.mark.parametrize("M", [16, 64])
def test_chained_decode_pack_then_runs_gemm(M):
    """Each layer packs its weight and runs the GEMM straight after it (runs strategy: no
    gather in between), reading the previous layer's output in place. The decode kernel
    requests weight tiles before waiting for the previous kernel, so the pack must be
    complete when the GEMM starts; its input must still wait for the previous GEMM."""
    K = 4096
    g = torch.Generator(device="cuda").manual_seed(M)
    x = torch.randn(M, K, device="cuda", dtype=torch.float16, generator=g)
    h, ref = x, x.float()
    for layer in range(6):
        w = (torch.randn(K, K, device="cuda", generator=g) / 45.0).half()
        blocks = torch.sort(torch.randperm(K // 64, device="cuda", generator=g)[: K // 128]).values
        idx = (blocks[:, None] * 64 + torch.arange(64, device="cuda")).reshape(-1)
        out = torch.empty(M, K, device="cuda", dtype=torch.float16)
        _native.gather_gemm(h, pack_weight(w, idx), idx, out, strategy="runs")
        h = out
        ref = (ref.half().float()[:, idx] @ w.float()[:, idx].t())
    torch.testing.assert_close(h, ref.half(), **tols(torch.float16))


# ----------------------------------------------------------------- small M (cluster split-K and decode kernels)
@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("M,K,N,kp,bias,act", [
    (16, 4096, 4096, 2048, False, None),        # at most 32 rows: the decode kernel
    (1, 4096, 768, 2048, True, "gelu"),         # decode kernel, one valid row
    (100, 4096, 1000, 1500, True, "gelu_tanh"), # tiles of 64, clusters of 4; ragged last tile
    (128, 1024, 4096, 130, True, None),         # 3 k-blocks: tiles of 64, clusters of 2, uneven ranges
    (256, 4096, 2304, 4096, False, "gelu"),     # 2 m-tiles x 18 n-tiles of 128, clusters of 4
    (33, 768, 3072, 384, True, None),           # GPT-2 MLP-in: tiles of 64, clusters of 2
    (16, 3072, 768, 1536, True, None),          # GPT-2 MLP-out at decode: decode kernel
    (512, 4096, 4096, 2048, True, None),        # 64 tiles of 256, clusters of 2
    (200, 4096, 3072, 3072, True, "gelu"),      # tiles of 256, clusters of 4
    (40, 8192, 2048, 8192, False, None),        # tiles of 256, clusters of 8
    (40, 2048, 1000, 1536, True, "gelu_tanh"),  # tiles of 128, clusters of 8; ragged last tile
    (200, 1024, 3072, 256, True, None),         # tiles of 128, clusters of 2
    (40, 1024, 256, 512, False, None),          # tiles of 64, clusters of 8
])
def test_cluster_split_k_vs_fp32(dt, M, K, N, kp, bias, act):
    torch_dt = DT[dt]
    g = torch.Generator(device="cuda").manual_seed(M * 7 + kp)
    x = torch.randn(M, K, device="cuda", dtype=torch_dt, generator=g)
    w = (torch.randn(N, K, device="cuda", generator=g) / kp ** 0.5).to(torch_dt)
    b = torch.randn(N, device="cuda", generator=g).to(torch_dt) if bias else None
    idx = torch.sort(torch.randperm(K, device="cuda", generator=g)[:kp]).values
    wp = pack_weight(w, idx)
    ws = torch.empty(_native.gather_gemm_workspace_bytes(M, kp, torch_dt), dtype=torch.uint8, device="cuda")
    ys = []
    for _ in range(3):                          # fixed reduction order: bitwise reproducible
        y = torch.full((M, N), float("nan"), device="cuda", dtype=torch_dt)
        _native.gather_gemm(x, wp, idx, y, bias=b, activation=act, strategy="pregather", workspace=ws)
        ys.append(y)
    ref = F.linear(x.float()[:, idx], w.float()[:, idx], None if b is None else b.float())
    if act == "gelu":
        ref = F.gelu(ref)
    elif act == "gelu_tanh":
        ref = F.gelu(ref, approximate="tanh")
    torch.testing.assert_close(ys[0], ref.to(torch_dt), **tols(torch_dt))
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[1], ys[2])


@pytest.mark.parametrize("M,N,K,expect", [
    (4096, 4096, 2048, ("pair", 256, 0)),
    (16, 4096, 2048, ("decode", 0, None)),
    (1, 768, 2048, ("decode", 0, None)),
    (100, 1000, 1500, ("splitk", 64, 4)),
    (128, 4096, 130, ("splitk", 64, 2)),
    (48, 4096, 2048, ("splitk", 128, 4)),
    (512, 4096, 2048, ("splitk", 256, 2)),
    (200, 3072, 3072, ("splitk", 256, 4)),
    (40, 2048, 8192, ("splitk", 256, 8)),
    (40, 1000, 1536, ("splitk", 128, 8)),
    (200, 3072, 256, ("splitk", 128, 2)),
    (40, 256, 512, ("splitk", 64, 8)),
])
def test_gemm_plan_dispatch(M, N, K, expect):
    """The kernel each shape dispatches to (the split-K shapes above rely on it)."""
    kernel, tile_n, split = _native.gemm_plan(M, N, K)
    assert (kernel, tile_n) == expect[:2]
    if expect[2] is None:
        assert split >= 2
    else:
        assert split == expect[2]


# ----------------------------------------------------------------- decode kernel (M <= 32)
@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("M,K,N,kp,bias,act", [
    (8, 1024, 1000, 200, True, "gelu"),         # MP 16; ragged last feature block and k-block
    (17, 2048, 136, 1100, False, None),         # MP 32; two feature blocks, the second ragged
    (32, 4096, 4096, 2048, True, "gelu_tanh"),  # MP 32, every padded row valid
    (16, 3072, 768, 1536, True, None),          # six feature blocks: clusters of 16
    (2, 8192, 3072, 8192, False, None),         # long k range per CTA
    (48, 4096, 4096, 2048, True, None),         # 33..64 rows: cluster split-K instead
])
def test_decode_kernel_vs_fp32(dt, M, K, N, kp, bias, act):
    torch_dt = DT[dt]
    g = torch.Generator(device="cuda").manual_seed(M * 13 + kp)
    x = torch.randn(M, K, device="cuda", dtype=torch_dt, generator=g)
    w = (torch.randn(N, K, device="cuda", generator=g) / kp ** 0.5).to(torch_dt)
    b = torch.randn(N, device="cuda", generator=g).to(torch_dt) if bias else None
    idx = torch.sort(torch.randperm(K, device="cuda", generator=g)[:kp]).values
    wp = pack_weight(w, idx)
    ys = []
    for _ in range(2):                          # fixed reduction order: bitwise reproducible
        y = torch.full((M, N), float("nan"), device="cuda", dtype=torch_dt)
        ghost_linear(x, wp, idx, bias=b, activation=act, out=y)
        ys.append(y)
    ref = F.linear(x.float()[:, idx], w.float()[:, idx], None if b is None else b.float())
    if act == "gelu":
        ref = F.gelu(ref)
    elif act == "gelu_tanh":
        ref = F.gelu(ref, approximate="tanh")
    torch.testing.assert_close(ys[0], ref.to(torch_dt), **tols(torch_dt))
    assert torch.equal(ys[0], ys[1])


@pytest.mark.parametrize("strategy", ["auto", "pregather"])
def test_decode_gather_unaligned_x_unsorted_repeats(strategy):
    """The decode kernel's in-kernel gather (auto) reads x through any leading dimension
    and any index order, repeats included; the two-launch path (pregather) agrees."""
    M, K, N = 3, 1001, 700
    g = torch.Generator(device="cuda").manual_seed(21)
    base = torch.randn(M, K + 3, device="cuda", dtype=torch.float16, generator=g)
    x = base[:, 1:K + 1]                        # row stride 1004, first element 2 bytes in
    w = (torch.randn(N, K, device="cuda", generator=g) / 20).half()
    idx = torch.randint(0, K, (517,), device="cuda", generator=g)
    b = torch.randn(N, device="cuda", generator=g).half()
    wp = pack_weight(w, idx)
    y = torch.empty(M, N, device="cuda", dtype=torch.float16)
    if strategy == "auto":
        _native.gather_gemm(x, wp, idx, y, bias=b, activation="gelu_tanh", strategy="auto")
    else:
        ws = _native.gemm_workspace(x.device, _native.gather_gemm_workspace_bytes(M, idx.numel(), x.dtype))
        _native.gather_gemm(x.contiguous(), wp, idx, y, bias=b, activation="gelu_tanh",
                            strategy="pregather", workspace=ws)
    ref = F.gelu(x.float()[:, idx] @ w.float()[:, idx].t() + b.float(), approximate="tanh")
    torch.testing.assert_close(y, ref.half(), **tols(torch.float16))


@pytest.mark.parametrize("M,N,K", [(16, 4096, 2048), (128, 4096, 1024), (7, 768, 3072), (300, 1000, 640)])
def test_packed_gemm_decode_shapes(M, N, K):
    g = torch.Generator(device="cuda").manual_seed(N + K)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    b = torch.randn(N, device="cuda", generator=g).bfloat16()
    y = packed_linear(a, pack_weight(w, torch.arange(K, device="cuda")), bias=b, activation="gelu")
    ref = F.gelu(F.linear(a.float(), w.float(), b.float())).bfloat16()
    torch.testing.assert_close(y, ref, **tols(torch.bfloat16))


def test_cluster_split_k_unaligned_ldy():
    """ldy odd: the reduce-scatter falls back to 2-byte stores."""
    M, K, N, kp = 16, 2048, 1000, 1024
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(M, K, device="cuda", dtype=torch.float16, generator=g)
    w = (torch.randn(N, K, device="cuda", generator=g) / kp ** 0.5).half()
    idx = torch.sort(torch.randperm(K, device="cuda", generator=g)[:kp]).values
    big = torch.zeros(M, N + 1, device="cuda", dtype=torch.float16)
    y = big[:, :N]
    _native.gather_gemm(x, pack_weight(w, idx), idx, y)
    ref = (x.float()[:, idx] @ w.float()[:, idx].t()).half()
    torch.testing.assert_close(y, ref, **tols(torch.float16))
    assert torch.count_nonzero(big[:, N]).item() == 0


@pytest.mark.parametrize("M,kp", [(100, 1500), (64, 2048)])
def test_cluster_split_k_partial_column_group(M, kp):
    """N = 1002 with ldy = 1004: 8-byte stores are allowed, and the last group of four
    columns straddles N, so it is stored element by element; columns N.. stay untouched."""
    N, K = 1002, 4096
    assert _native.gemm_plan(M, N, kp)[0] == "splitk"
    g = torch.Generator(device="cuda").manual_seed(M + kp)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g)
    w = (torch.randn(N, K, device="cuda", generator=g) / kp ** 0.5).bfloat16()
    b = torch.randn(N, device="cuda", generator=g).bfloat16()
    idx = torch.sort(torch.randperm(K, device="cuda", generator=g)[:kp]).values
    big = torch.zeros(M, N + 2, device="cuda", dtype=torch.bfloat16)
    y = big[:, :N]
    _native.gather_gemm(x, pack_weight(w, idx), idx, y, bias=b, activation="gelu")
    ref = F.gelu(F.linear(x.float()[:, idx], w.float()[:, idx], b.float())).bfloat16()
    torch.testing.assert_close(y, ref, **tols(torch.bfloat16))
    assert torch.count_nonzero(big[:, N:]).item() == 0


def test_no_wait_timeouts_after_suite():
    assert _native.device_error(reset=False) & _native.DEVICE_ERR_WAIT_TIMEOUT == 0


# ----------------------------------------------------------------- reference-suite cases
class TestReferenceSuite:
    """ghostweight_triton tests/test_matmul.py:105-207, on B200."""

    @staticmethod
    def _inputs(M, K, N, dtype, device, sparsity, seed=99):
        torch.manual_seed(seed)
        A = torch.randn(M, K, dtype=dtype, device=device) * 0.1
        W = torch.randn(K, N, dtype=dtype, device=device) * 0.1
        dead = set(torch.randperm(K)[: int(K * sparsity)].tolist())
        idx = torch.tensor(sorted(k for k in range(K) if k not in dead), dtype=torch.int64, device=device)
        return A, W, idx

    @staticmethod
    def _ref(A, W, idx):
        return (A.float()[:, idx] @ W.float()[idx, :]).to(A.dtype)

    @pytest.mark.parametrize("M,K,N", [(1, 128, 256), (1, 768, 3072), (16, 768, 3072),
                                       (128, 768, 3072), (128, 3072, 768)])
    def test_output_shape(self, device, M, K, N):
        A, W, idx = self._inputs(M, K, N, torch.float16, device, 0.5)
        C = ghostweight_matmul(A, W, idx)
        assert C.shape == (M, N) and C.is_cuda and C.is_contiguous()

    @pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.bfloat16])
    @pytest.mark.parametrize("M,K,N,sparsity", [(1, 128, 256, 0.0), (1, 768, 3072, 0.5),
                                                (16, 768, 3072, 0.3), (128, 768, 3072, 0.7),
                                                (128, 3072, 768, 0.5), (16, 256, 128, 0.9)])
    def test_matches_reference(self, device, dtype, M, K, N, sparsity):
        A, W, idx = self._inputs(M, K, N, dtype, device, sparsity)
        C = ghostweight_matmul(A, W, idx)
        assert C.dtype == dtype
        torch.testing.assert_close(C, self._ref(A, W, idx), **tols(dtype))

    def test_dense_equals_matmul(self, device):
        torch.manual_seed(1)
        A = torch.randn(32, 128, device=device) * 0.1
        W = torch.randn(128, 64, device=device) * 0.1
        C = ghostweight_matmul(A, W, torch.arange(128, device=device))
        torch.backends.cuda.matmul.allow_tf32 = False
        torch.testing.assert_close(C, A @ W, atol=1e-4, rtol=1e-4)

    def test_k_alive_one(self, device):
        torch.manual_seed(2)
        A = torch.randn(4, 128, device=device)
        W = torch.randn(128, 16, device=device)
        C = ghostweight_matmul(A, W, torch.tensor([7], device=device))
        torch.testing.assert_close(C, A[:, [7]] * W[[7], :], atol=1e-4, rtol=1e-4)

    def test_unsorted(self, device):
        torch.manual_seed(3)
        A = torch.randn(8, 64, device=device) * 0.1
        W = torch.randn(64, 32, device=device) * 0.1
        idx = torch.randperm(64, device=device)[:32]
        torch.testing.assert_close(ghostweight_matmul(A, W, idx), self._ref(A, W, idx),
                                   atol=1e-4, rtol=1e-4)

    def test_block_kwargs_accepted(self, device):
        A, W, idx = self._inputs(64, 128, 64, torch.float32, device, 0.5)
        ref = self._ref(A, W, idx)
        for bm, bn, bk in [(32, 32, 16), (64, 64, 32), (128, 64, 32)]:
            torch.testing.assert_close(ghostweight_matmul(A, W, idx, BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=bk),
                                       ref, atol=1e-4, rtol=1e-4)

    @pytest.mark.parametrize("M,K,N", [(1, 768, 3072), (128, 768, 3072), (128, 3072, 768), (1, 768, 2304)])
    def test_gpt2_shapes_finite(self, device, M, K, N):
        A, W, idx = self._inputs(M, K, N, torch.float16, device, 0.5)
        C = ghostweight_matmul(A, W, idx)
        assert torch.isfinite(C).all()


# ----------------------------------------------------------------- full-size properties
@pytest.mark.parametrize("M", [4096, 1024, 128, 16])
@pytest.mark.parametrize("sp,pattern", [(0.0, "random"), (0.5, "random"), (0.9, "random"),
                                        (0.75, "block")])
@pytest.mark.parametrize("strategy", ["overlap", "pregather", "fused"])
def test_gemm_sweep_size_vs_dense_fp32(M, sp, pattern, strategy):
    """M x 4096 x 4096 fp16: sparse result equals the dense fp32 product of the zeroed weight."""
    K = N = 4096
    g = torch.Generator(device="cuda").manual_seed(M)
    x = torch.randn(M, K, device="cuda", dtype=torch.float16, generator=g)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).half()
    dead = torch.from_numpy(dead_columns(K, sp, M, pattern, 64)).cuda()
    w[:, dead] = 0
    from ghostweight_triton_b200.kernels.mask import alive_indices

    idx = alive_indices(w, 0.0)
    assert idx.numel() == K - dead.numel()
    y = ghost_linear(x, pack_weight(w, idx), idx, strategy=strategy)
    ref = F.linear(x.float(), w.float()).half()
    torch.testing.assert_close(y, ref, **tols(torch.float16))


def test_sharded_mlp_size_bf16_rows():
    """X [8192, 8192] bf16, W [28672, 8192] with 70% dead 128-blocks: spot-check rows vs fp32."""
    M, K, N = 8192, 8192, 28672
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    dead = torch.from_numpy(dead_columns(K, 0.7, 11, "block", 128)).cuda()
    w[:, dead] = 0
    from ghostweight_triton_b200.kernels.mask import alive_indices

    idx = alive_indices(w, 0.0)
    assert idx.numel() == 2560
    y = ghost_linear(x, pack_weight(w, idx), idx)
    rows = torch.arange(0, M, 257, device="cuda")
    ref = (x[rows].float() @ w.float().t()).bfloat16()
    torch.testing.assert_close(y[rows], ref, **tols(torch.bfloat16))


def test_matmul_packed_cache_follows_weight_storage():
    """ghostweight_matmul's packed-weight cache is rebuilt when the weight is
    rebound to other storage (same object and version), and after
    clear_packed_cache() for in-place writes through .data."""
    from ghostweight_triton_b200.kernels.matmul import clear_packed_cache

    K, N, M = 512, 256, 64
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(K, N, device="cuda", generator=g) * K ** -0.5).half()
    idx = torch.sort(torch.randperm(K, device="cuda", generator=g)[: K // 2]).values

    def check():
        C = ghostweight_matmul(x, w, idx)
        ref = x.float()[:, idx] @ w.float()[idx, :]
        torch.testing.assert_close(C.float(), ref, atol=1e-2, rtol=1e-2)

    check()
    check()                                       # served from the cache
    w.data = w.clone() * 2                        # new storage, same object and version
    check()
    w.data.mul_(0.5)                              # in place through .data: no version bump
    clear_packed_cache()
    check()
