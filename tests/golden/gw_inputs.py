"""Seeded, platform-independent input generators shared by the golden-vector
generator (make_golden.py) and the tests that replay the fixtures.

numpy's PCG64 ``default_rng(seed).standard_normal`` is reproducible across
machines, so large inputs are stored as (seed, shape) and regenerated.
"""

from __future__ import annotations

import numpy as np


def rand_matrix(shape, seed: int, dtype: str = "f32", scale: float = 1.0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)
    if dtype == "f16":
        return x.astype(np.float16)
    if dtype == "bf16":
        bits = x.view(np.uint32).astype(np.uint64)
        return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)
    return x


def dead_columns(K: int, sparsity: float, seed: int, pattern: str = "random", block: int = 64) -> np.ndarray:
    """Sorted dead column indices: int(K*sparsity) random columns, or whole
    `block`-wide blocks (int((K//block)*sparsity) of them) for pattern="block"."""
    rng = np.random.default_rng(seed + 7919)
    if pattern == "random":
        n_dead = int(K * sparsity)
        return np.sort(rng.permutation(K)[:n_dead]).astype(np.int64)
    nb = K // block
    n_dead_blocks = int(nb * sparsity)
    blocks = np.sort(rng.permutation(nb)[:n_dead_blocks])
    cols = (blocks[:, None] * block + np.arange(block)[None, :]).reshape(-1)
    return np.sort(cols).astype(np.int64)


def alive_from_dead(K: int, dead: np.ndarray) -> np.ndarray:
    keep = np.ones(K, dtype=bool)
    keep[dead] = False
    return np.flatnonzero(keep).astype(np.int64)


def zero_columns(x: np.ndarray, cols: np.ndarray) -> np.ndarray:
    y = x.copy()
    y[:, cols] = 0
    return y
