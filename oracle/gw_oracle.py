"""CPU oracle for the column-sparse linear hot path -- TEST INFRASTRUCTURE ONLY.

A plain numpy restatement of what ghostweight-triton computes on this path.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only as the checker / the timed CPU reference; the product
(ghostweight_triton_b200) never calls it.

Parity pins: tests/test_oracle.py checks every function here against the
golden vectors in tests/golden/ (produced by the reference's own Triton
kernels run under the Triton interpreter, tests/golden/make_golden.py) and
against the known-answer cases of the reference's tests.

Dtypes: numpy float16 / float32 arrays as-is; bfloat16 travels as the raw
uint16 bit pattern with ``dtype="bf16"``.
"""

from __future__ import annotations

import numpy as np

F16, BF16, F32 = "f16", "bf16", "f32"


# ---------------------------------------------------------------------------
# dtype helpers
# ---------------------------------------------------------------------------
def dtype_name(a: np.ndarray, dtype: str | None = None) -> str:
    if dtype is not None:
        return dtype
    if a.dtype == np.float16:
        return F16
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.uint16:
        return BF16
    raise TypeError(f"unsupported array dtype {a.dtype}")


def to_f32(a: np.ndarray, dtype: str | None = None) -> np.ndarray:
    """Exact widening to float32 (bf16 given as uint16 bits)."""
    d = dtype_name(a, dtype)
    if d == BF16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


def from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 to the storage dtype, round-to-nearest-even (bf16 -> uint16 bits)."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == F32:
        return x
    if dtype == F16:
        return x.astype(np.float16)
    bits = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = ((bits[nan] >> 16) | 0x0040).astype(np.uint16)   # keep NaN quiet
    return out


# ---------------------------------------------------------------------------
# K1: dead-column mask + compaction
# ---------------------------------------------------------------------------
def dead_neuron_mask(a: np.ndarray, threshold: float = 1e-6, dtype: str | None = None) -> np.ndarray:
    """int32 [K]: 1 where max_r fp32(|a[r, k]|) > fp32(threshold).

    Restates ghostweight_triton/kernels/mask.py:41-59: the running max starts
    at 0.0 (mask.py:46), loads are widened to fp32 (mask.py:53), tl.maximum
    keeps the non-NaN operand (mask.py:55), and the test is a strict fp32
    greater-than against the fp32 scalar threshold (mask.py:58).
    """
    assert a.ndim == 2
    thr = np.float32(threshold)
    f = np.abs(to_f32(a, dtype))
    f = np.where(np.isnan(f), np.float32(0.0), f)
    colmax = f.max(axis=0, initial=np.float32(0.0))
    with np.errstate(invalid="ignore"):
        return (colmax > thr).astype(np.int32)


def alive_indices(mask: np.ndarray) -> np.ndarray:
    """Sorted int64 indices of mask == 1: torch.nonzero(mask).squeeze(-1) (module.py:104)."""
    return np.flatnonzero(mask).astype(np.int64)


# ---------------------------------------------------------------------------
# K2: gathers / packing
# ---------------------------------------------------------------------------
def gather_columns(a: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """a[:, idx] -- ghostweight_triton/kernels/gather.py:19-55."""
    return np.ascontiguousarray(a[:, np.asarray(idx, dtype=np.int64)])


def gather_rows(w: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """w[idx, :] -- ghostweight_triton/kernels/gather.py:58-94."""
    return np.ascontiguousarray(w[np.asarray(idx, dtype=np.int64), :])


def index_runs(idx: np.ndarray, K: int) -> int:
    """Entries of idx that keep x[:, idx] from being whole 64-column slices of x.

    The reference always gathers x through idx (ghostweight_triton/kernels/
    matmul.py:55-63); when every 64-entry group idx[64 j : 64 j + 64] is the
    consecutive run idx[64 j] + (0 .. 63) starting at a multiple of 8, that
    gather is a set of contiguous slices. Counted as bad: entries outside
    [0, K), entries off their run, every entry of a run with a misaligned start,
    and entries of a trailing partial run.
    """
    idx = np.asarray(idx, dtype=np.int64)
    n = len(idx)
    t = np.arange(n)
    r = t & 63
    start = idx[t - r] if n else idx
    bad = (idx < 0) | (idx >= K) | (idx != start + r) | ((start & 7) != 0) | (t - r + 64 > n)
    return int(bad.sum())


def pack_weight(weight_nk: np.ndarray, idx: np.ndarray, pad_to: int | None = None) -> np.ndarray:
    """[N, pad_to] with weight[:, idx] in the first len(idx) columns, zeros after."""
    idx = np.asarray(idx, dtype=np.int64)
    pad = len(idx) if pad_to is None else int(pad_to)
    out = np.zeros((weight_nk.shape[0], pad), dtype=weight_nk.dtype)
    out[:, : len(idx)] = weight_nk[:, idx]
    return out


# ---------------------------------------------------------------------------
# K3: gather-GEMM
# ---------------------------------------------------------------------------
def _gelu(v: np.ndarray, activation: str | None) -> np.ndarray:
    if activation is None:
        return v
    v64 = v.astype(np.float64)
    if activation in ("gelu", "gelu_erf"):
        from math import erf, sqrt

        erf_v = np.vectorize(erf, otypes=[np.float64])
        return (0.5 * v64 * (1.0 + erf_v(v64 / sqrt(2.0)))).astype(np.float32)
    if activation == "gelu_tanh":
        c = np.sqrt(2.0 / np.pi)
        return (0.5 * v64 * (1.0 + np.tanh(c * (v64 + 0.044715 * v64 ** 3)))).astype(np.float32)
    raise ValueError(activation)


def ghostweight_matmul(a: np.ndarray, w_kn: np.ndarray, idx: np.ndarray,
                       dtype: str | None = None, acc: type = np.float32) -> np.ndarray:
    """C = a[:, idx] @ w_kn[idx, :], accumulated in `acc`, rounded to a's dtype.

    Restates the reference's own checker _ref_matmul (tests/test_matmul.py:30-42:
    fp32 upcast, gather, matmul, cast back), which pins ghostweight_matmul
    (ghostweight_triton/kernels/matmul.py:27-82: fp32 accumulator, store cast to
    the activation dtype). Empty idx gives zeros.
    """
    d = dtype_name(a, dtype)
    idx = np.asarray(idx, dtype=np.int64)
    a_f = to_f32(a, d)[:, idx].astype(acc)
    w_f = to_f32(w_kn, d)[idx, :].astype(acc)
    return from_f32((a_f @ w_f).astype(np.float32), d)


def ghost_linear(x: np.ndarray, weight_nk: np.ndarray, idx: np.ndarray,
                 bias: np.ndarray | None = None, activation: str | None = None,
                 dtype: str | None = None, acc: type = np.float64) -> np.ndarray:
    """act(x[:, idx] @ weight_nk[:, idx]^T + bias), one final rounding.

    The GhostLinear forward of ghostweight_triton/module.py:88-119 (ghost path:
    ghostweight_matmul then + bias), with the bias added before the single
    rounding as the fused B200 epilogue does.
    """
    d = dtype_name(x, dtype)
    idx = np.asarray(idx, dtype=np.int64)
    xf = to_f32(x, d)[:, idx].astype(acc)
    wf = to_f32(weight_nk, d)[:, idx].astype(acc)
    y = xf @ wf.T
    if bias is not None:
        y = y + to_f32(bias, d).astype(acc)
    y = y.astype(np.float32)
    return from_f32(_gelu(y, activation), d)
