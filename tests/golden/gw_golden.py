"""Loader for the golden fixtures written by make_golden.py.

``load(name)`` returns (meta, inputs, expected); inputs that were too large to
store are regenerated from the recorded seeds exactly as make_golden.py built
them. ``check_exact`` / ``check_close`` compare a result against an expected
entry, whichever form (full array, sha256 digest, row/column sample) it has.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np

from tests.golden.gw_inputs import rand_matrix, dead_columns, zero_columns

HERE = Path(__file__).resolve().parent


def names(kind: str | None = None) -> list[str]:
    return [p.stem for p in sorted(HERE.glob("*.npz"))
            if kind is None or p.stem.startswith(kind + "_")]


def _regenerate(meta: dict) -> dict[str, np.ndarray]:
    kind, dt, seed = meta["kind"], meta["dtype"], meta["seed"]
    if kind == "mask":
        M, K = meta["M"], meta["K"]
        a = rand_matrix((M, K), seed, dt, scale=meta.get("scale", 1.0))
        if meta.get("zero_dead"):
            a = zero_columns(a, dead_columns(K, meta["sparsity"], seed, meta.get("pattern", "random")))
        return {"a": a}
    if kind == "gather":
        M, K, N = meta["M"], meta["K"], meta["N"]
        return {"A": rand_matrix((M, K), seed, dt), "W": rand_matrix((K, N), seed + 1, dt)}
    if kind == "matmul":
        M, K, N = meta["M"], meta["K"], meta["N"]
        s = meta.get("scale", 1.0)
        return {"A": rand_matrix((M, K), seed, dt, s), "W": rand_matrix((K, N), seed + 1, dt, s)}
    if kind == "chain":
        M, K, N = meta["M"], meta["K"], meta["N"]
        x = zero_columns(rand_matrix((M, K), seed, dt, 0.1),
                         dead_columns(K, meta["sparsity"], seed, meta["pattern"]))
        return {"x": x, "weight": rand_matrix((N, K), seed + 1, dt, 0.1),
                "bias": rand_matrix((N,), seed + 2, dt, 0.1)}
    raise ValueError(kind)


def load(name: str) -> tuple[dict, dict[str, np.ndarray], dict[str, np.ndarray]]:
    with np.load(HERE / f"{name}.npz") as z:
        data = {k: z[k] for k in z.files}
    meta = json.loads(str(data.pop("meta")))
    if meta["inline"]:
        inputs = {k[3:]: v for k, v in data.items() if k.startswith("in_")}
    else:
        inputs = _regenerate(meta)
    expected = {k: v for k, v in data.items() if not k.startswith("in_")}
    return meta, inputs, expected


_UINT = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}


def check_exact(actual: np.ndarray, expected: dict, key: str) -> None:
    """Bit-for-bit comparison (NaN payloads included) against a stored array or digest."""
    actual = np.ascontiguousarray(actual)
    if key in expected:
        ref = np.ascontiguousarray(expected[key])
        assert actual.shape == ref.shape, (key, actual.shape, ref.shape)
        assert actual.dtype == ref.dtype, (key, actual.dtype, ref.dtype)
        u = _UINT[actual.itemsize]
        mism = np.flatnonzero(actual.reshape(-1).view(u) != ref.reshape(-1).view(u))
        assert mism.size == 0, f"{key}: {mism.size} mismatches, first at flat index {mism[:8].tolist()}"
    else:
        shape = tuple(int(v) for v in expected[key + "__shape"])
        assert actual.shape == shape, (key, actual.shape, shape)
        got = hashlib.sha256(actual.tobytes()).hexdigest()
        assert got == str(expected[key + "__sha256"]), f"{key}: digest mismatch"


def expected_float(expected: dict, key: str):
    """(values, rows, cols): rows/cols are None when the full array is stored."""
    if key in expected:
        return expected[key], None, None
    return expected[key + "__sample"], expected[key + "__rows"], expected[key + "__cols"]


def check_close(actual: np.ndarray, expected: dict, key: str, atol: float, rtol: float) -> None:
    ref, rows, cols = expected_float(expected, key)
    act = np.asarray(actual)
    if rows is not None:
        act = act[rows][:, cols]
    a = act.astype(np.float64)
    r = ref.astype(np.float64)
    assert a.shape == r.shape, (key, a.shape, r.shape)
    bad = ~(np.abs(a - r) <= atol + rtol * np.abs(r))
    assert not bad.any(), (
        f"{key}: {int(bad.sum())}/{bad.size} outside atol={atol} rtol={rtol}; "
        f"max abs err {np.nanmax(np.abs(a - r)):.3g}")
