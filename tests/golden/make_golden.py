"""Generate golden vectors from the reference implementation itself.

Runs the reference's own @triton.jit kernels (ghostweight_triton/kernels/
mask.py:21-59, gather.py:19-94, matmul.py:27-82) on CPU tensors under the
Triton interpreter (TRITON_INTERPRET=1), launched with exactly the argument
lists their host wrappers use (mask.py:94-102, gather.py:140-156,
matmul.py:125-140) -- the wrappers themselves assert CUDA tensors. The outputs
are written to tests/golden/*.npz together with their inputs (small cases) or
the seeds that regenerate them (tests/golden/gw_inputs.py).

Needs the reference package: the directory named by GW_REFERENCE_DIR (a
checkout, or any directory holding the ghostweight_triton package), else the
copy installed under baseline/_ref of this repository. Run from anywhere:
  GW_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden.py
The GPU test box never runs this; it only reads the committed .npz files.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent


def _reference_dir() -> Path:
    env = os.environ.get("GW_REFERENCE_DIR")
    if env:
        return Path(env)
    installed = HERE.parents[1] / "baseline" / "_ref"
    if (installed / "ghostweight_triton" / "__init__.py").exists():
        return installed
    raise SystemExit("set GW_REFERENCE_DIR to the reference checkout (or install the reference "
                     "into baseline/_ref) before generating golden vectors")


REF = _reference_dir()
sys.path.insert(0, str(REF))
sys.path.insert(1, str(HERE))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402

import ghostweight_triton  # noqa: E402
from ghostweight_triton.kernels import mask as ref_mask  # noqa: E402
from ghostweight_triton.kernels import gather as ref_gather  # noqa: E402
from ghostweight_triton.kernels import matmul as ref_matmul  # noqa: E402

from gw_inputs import rand_matrix, dead_columns, alive_from_dead, zero_columns  # noqa: E402

assert Path(ghostweight_triton.__file__).resolve().is_relative_to(REF.resolve()), (
    "imported the wrong ghostweight_triton: " + ghostweight_triton.__file__)

INLINE_LIMIT = 96 * 1024   # store inputs inline when they are at most this many bytes
OUTPUT_LIMIT = 64 * 1024   # larger outputs are stored as a digest (exact) or a row/column sample (float)


def t(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x))


# ---------------------------------------------------------------- reference launches
def ref_dead_neuron_mask(a: torch.Tensor, threshold: float) -> torch.Tensor:
    a = a.contiguous()
    M, K = a.shape
    out = torch.empty(K, dtype=torch.int32)
    ref_mask._dead_neuron_mask_kernel[(K,)](a, out, M, K, a.stride(0), a.stride(1), threshold,
                                            BLOCK_M=512)
    return out


def ref_gather_compact(A: torch.Tensor, W: torch.Tensor, idx: torch.Tensor):
    M, K = A.shape
    _, N = W.shape
    idx = idx.contiguous().to(torch.int64)
    ka = idx.shape[0]
    A_c = torch.empty((M, ka), dtype=A.dtype)
    W_c = torch.empty((ka, N), dtype=W.dtype)
    grid_a = (triton.cdiv(M, 64), triton.cdiv(ka, 64))
    ref_gather._gather_columns_kernel[grid_a](A, idx, A_c, M, K, ka, A.stride(0), A.stride(1),
                                              A_c.stride(0), A_c.stride(1), BLOCK_M=64, BLOCK_K=64)
    grid_w = (triton.cdiv(ka, 64), triton.cdiv(N, 64))
    ref_gather._gather_rows_kernel[grid_w](W, idx, W_c, K, N, ka, W.stride(0), W.stride(1),
                                           W_c.stride(0), W_c.stride(1), BLOCK_K=64, BLOCK_N=64)
    return A_c, W_c


def ref_ghostweight_matmul(A: torch.Tensor, W: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    M, K = A.shape
    _, N = W.shape
    idx = idx.contiguous().to(torch.int64)
    C = torch.empty((M, N), dtype=A.dtype)
    grid = (triton.cdiv(M, 64), triton.cdiv(N, 64))
    ref_matmul._ghostweight_matmul_kernel[grid](
        A, W, C, idx, M, N, K, idx.shape[0], A.stride(0), A.stride(1), W.stride(0), W.stride(1),
        C.stride(0), C.stride(1), BLOCK_M=64, BLOCK_N=64, BLOCK_K=32,
        ALLOW_TF32=(A.dtype == torch.float16))
    return C


# ---------------------------------------------------------------- fixture writer
def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def save(name: str, meta: dict, arrays: dict[str, np.ndarray], inputs: dict[str, np.ndarray],
         float_outputs: tuple[str, ...] = ()) -> None:
    """Write one fixture. Exact outputs above OUTPUT_LIMIT become sha256 digests
    (key ``<name>__sha256`` plus ``<name>__shape``); float outputs above it keep
    up to 8 evenly spaced rows and, if still too large, evenly spaced columns
    (``<name>__rows`` / ``<name>__cols`` hold the kept indices)."""
    payload = {}
    for k, v in arrays.items():
        if v.nbytes <= OUTPUT_LIMIT:
            payload[k] = v
        elif k in float_outputs:
            rows = np.unique(np.linspace(0, v.shape[0] - 1, num=min(v.shape[0], 8)).astype(np.int64))
            cols = np.arange(v.shape[1], dtype=np.int64)
            sub = v[rows]
            if sub.nbytes > OUTPUT_LIMIT:
                keep = max(1, OUTPUT_LIMIT // (len(rows) * v.itemsize))
                cols = np.unique(np.linspace(0, v.shape[1] - 1, num=keep).astype(np.int64))
                sub = sub[:, cols]
            payload[k + "__sample"] = np.ascontiguousarray(sub)
            payload[k + "__rows"] = rows
            payload[k + "__cols"] = cols
        else:
            payload[k + "__sha256"] = np.array(digest(v))
            payload[k + "__shape"] = np.array(v.shape, dtype=np.int64)
    inline = sum(v.nbytes for v in inputs.values()) <= INLINE_LIMIT
    meta = dict(meta, inline=inline)
    if inline:
        for k, v in inputs.items():
            payload["in_" + k] = v
    payload["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / f"{name}.npz", **payload)
    print(f"  {name}: {', '.join(f'{k}{list(v.shape)}' for k, v in payload.items() if k != 'meta')}")


# ---------------------------------------------------------------- cases
def mask_cases() -> None:
    # Random activations with constructed dead columns (tests/test_mask.py:47-61, 119-132).
    for dt in ("f16", "f32"):
        for (M, K, sp) in [(1, 128, 0.0), (1, 128, 0.5), (4, 256, 0.3), (32, 768, 0.7),
                           (128, 3072, 0.5), (8, 200, 0.4), (64, 4096, 0.9)]:
            seed = 1000 + M * 7 + K + int(sp * 100)
            a = rand_matrix((M, K), seed, dt)
            dead = dead_columns(K, sp, seed)
            a = zero_columns(a, dead)
            out = ref_dead_neuron_mask(t(a), 1e-6).numpy()
            save(f"mask_{dt}_{M}x{K}_s{int(sp * 100)}",
                 {"kind": "mask", "dtype": dt, "M": M, "K": K, "threshold": 1e-6, "seed": seed,
                  "sparsity": sp, "pattern": "random", "zero_dead": True},
                 {"mask": out}, {"a": a})

    def explicit(name, a, thr, dt):
        out = ref_dead_neuron_mask(t(a), thr).numpy()
        save(name, {"kind": "mask", "dtype": dt, "M": a.shape[0], "K": a.shape[1],
                    "threshold": thr}, {"mask": out}, {"a": a})

    # Known-answer cases of tests/test_mask.py:130-189.
    explicit("mask_exact_threshold_dead", np.full((4, 64), 0.01, np.float32), 0.01, "f32")
    explicit("mask_just_above_alive", np.full((4, 64), 0.01 + 1e-4, np.float32), 0.01, "f32")
    a = np.zeros((1, 32), np.float32); a[0, :16] = 0.3; a[0, 16:] = 0.7
    explicit("mask_split_threshold", a, 0.5, "f32")
    a = np.zeros((8, 64), np.float32); a[-1, 0] = 1.0
    explicit("mask_any_row_alive", a, 1e-6, "f32")
    explicit("mask_all_zero_f16", np.zeros((4, 128), np.float16), 1e-6, "f16")
    explicit("mask_all_ones_f16", np.ones((4, 128), np.float16), 1e-6, "f16")
    # Semantic pins beyond the reference tests: fp32 compare of an fp16 value just
    # above the threshold, NaN handling, negative threshold, infinities, no rows.
    explicit("mask_f16_fp32_compare", np.full((2, 16), 1.0133e-6, np.float16), 1e-6, "f16")
    a = rand_matrix((8, 64), 5, "f32")
    a[:, ::2] = 0.0; a[0, 1] = np.nan; a[:, 3] = np.nan; a[:, 4] = 0.0; a[2, 4] = np.nan
    explicit("mask_nan_ignored", a, 1e-6, "f32")
    explicit("mask_negative_threshold", a, -1.0, "f32")
    a = np.zeros((3, 48), np.float16); a[1, 5] = np.inf; a[2, 7] = -np.inf; a[0, 9] = np.float16(-2.0)
    explicit("mask_inf_f16", a, 1.5, "f16")
    explicit("mask_zero_rows", np.zeros((0, 16), np.float32), 1e-6, "f32")
    explicit("mask_zero_rows_negthr", np.zeros((0, 16), np.float32), -0.5, "f32")
    # Weight-side mask of a single fp32 GhostLinear: W [3072, 768] ~ N(0, 0.02), 384 zeroed columns.
    seed = 11
    w = rand_matrix((3072, 768), seed, "f32", scale=0.02)
    dead = dead_columns(768, 0.5, seed)
    w = zero_columns(w, dead)
    out = ref_dead_neuron_mask(t(w), 0.0).numpy()
    save("mask_linear768x3072_weight_f32",
         {"kind": "mask", "dtype": "f32", "M": 3072, "K": 768, "threshold": 0.0, "seed": seed,
          "sparsity": 0.5, "pattern": "random", "zero_dead": True, "scale": 0.02},
         {"mask": out}, {"a": w})


def gather_cases() -> None:
    # tests/test_gather.py:66-173 shapes, values, identity, reversed, single index.
    for dt in ("f16", "f32"):
        for (M, K, N, sp) in [(1, 64, 128, 0.0), (1, 64, 128, 0.5), (8, 256, 512, 0.3),
                              (32, 768, 3072, 0.6)]:
            seed = 2000 + M + K + N + int(sp * 100)
            A = rand_matrix((M, K), seed, dt)
            W = rand_matrix((K, N), seed + 1, dt)
            idx = alive_from_dead(K, dead_columns(K, sp, seed))
            A_c, W_c = ref_gather_compact(t(A), t(W), t(idx))
            save(f"gather_{dt}_{M}x{K}x{N}_s{int(sp * 100)}",
                 {"kind": "gather", "dtype": dt, "M": M, "K": K, "N": N, "seed": seed, "sparsity": sp},
                 {"A_c": A_c.numpy(), "W_c": W_c.numpy(), "idx": idx}, {"A": A, "W": W})
    A = np.arange(16, dtype=np.float32)[None, :]
    W = np.eye(16, 8, dtype=np.float32)
    idx = np.array([5], np.int64)
    A_c, W_c = ref_gather_compact(t(A), t(W), t(idx))
    save("gather_single_alive", {"kind": "gather", "dtype": "f32", "M": 1, "K": 16, "N": 8},
         {"A_c": A_c.numpy(), "W_c": W_c.numpy(), "idx": idx}, {"A": A, "W": W})
    A = rand_matrix((2, 8), 3, "f32"); W = rand_matrix((8, 4), 4, "f32")
    idx = np.arange(7, -1, -1, dtype=np.int64)
    A_c, W_c = ref_gather_compact(t(A), t(W), t(idx))
    save("gather_reversed", {"kind": "gather", "dtype": "f32", "M": 2, "K": 8, "N": 4},
         {"A_c": A_c.numpy(), "W_c": W_c.numpy(), "idx": idx}, {"A": A, "W": W})


def matmul_cases() -> None:
    # tests/test_matmul.py:105-173 shapes and sparsities, scale 0.1 inputs.
    for dt in ("f16", "f32"):
        for (M, K, N, sp) in [(1, 128, 256, 0.0), (1, 128, 256, 0.5), (1, 768, 3072, 0.5),
                              (16, 768, 3072, 0.3), (128, 768, 3072, 0.7), (128, 3072, 768, 0.5),
                              (16, 256, 128, 0.9), (200, 320, 136, 0.5)]:
            seed = 3000 + M + K + N + int(sp * 100)
            A = rand_matrix((M, K), seed, dt, scale=0.1)
            W = rand_matrix((K, N), seed + 1, dt, scale=0.1)
            idx = alive_from_dead(K, dead_columns(K, sp, seed))
            C = ref_ghostweight_matmul(t(A), t(W), t(idx)).numpy()
            save(f"matmul_{dt}_{M}x{K}x{N}_s{int(sp * 100)}",
                 {"kind": "matmul", "dtype": dt, "M": M, "K": K, "N": N, "seed": seed,
                  "sparsity": sp, "scale": 0.1},
                 {"C": C, "idx": idx}, {"A": A, "W": W}, float_outputs=("C",))
    # Unsorted indices (test_matmul.py:156-165), K'=1 (:145-154), K'=K (:134-143).
    A = rand_matrix((8, 64), 31, "f32", 0.1); W = rand_matrix((64, 32), 32, "f32", 0.1)
    idx = np.random.default_rng(33).permutation(64)[:32].astype(np.int64)
    save("matmul_unsorted", {"kind": "matmul", "dtype": "f32", "M": 8, "K": 64, "N": 32},
         {"C": ref_ghostweight_matmul(t(A), t(W), t(idx)).numpy(), "idx": idx}, {"A": A, "W": W})
    A = rand_matrix((4, 128), 41, "f32"); W = rand_matrix((128, 16), 42, "f32")
    idx = np.array([7], np.int64)
    save("matmul_k1", {"kind": "matmul", "dtype": "f32", "M": 4, "K": 128, "N": 16},
         {"C": ref_ghostweight_matmul(t(A), t(W), t(idx)).numpy(), "idx": idx}, {"A": A, "W": W})
    A = rand_matrix((32, 128), 51, "f32", 0.1); W = rand_matrix((128, 64), 52, "f32", 0.1)
    idx = np.arange(128, dtype=np.int64)
    save("matmul_dense", {"kind": "matmul", "dtype": "f32", "M": 32, "K": 128, "N": 64},
         {"C": ref_ghostweight_matmul(t(A), t(W), t(idx)).numpy(), "idx": idx}, {"A": A, "W": W})


def chain_cases() -> None:
    # mask -> nonzero -> matmul (+ bias): tests/test_end_to_end.py:70-92 and the
    # GhostLinear ghost path (module.py:103-117) on x with zeroed columns.
    for dt, (M, K, N, sp, pattern) in [("f16", (32, 256, 128, 0.5, "random")),
                                       ("f32", (16, 128, 256, 0.5, "random")),
                                       ("f16", (64, 512, 192, 0.75, "block")),
                                       ("f32", (24, 384, 72, 0.9, "random"))]:
        seed = 4000 + M + K + N
        x = zero_columns(rand_matrix((M, K), seed, dt, 0.1), dead_columns(K, sp, seed, pattern))
        weight = rand_matrix((N, K), seed + 1, dt, 0.1)            # nn.Linear.weight [N, K]
        bias = rand_matrix((N,), seed + 2, dt, 0.1)
        mask = ref_dead_neuron_mask(t(x), 1e-6)
        alive = torch.nonzero(mask, as_tuple=False).squeeze(-1).to(torch.int64)
        out = ref_ghostweight_matmul(t(x), t(weight).t().contiguous(), alive)
        y = (out + t(bias)).numpy()
        save(f"chain_{dt}_{M}x{K}x{N}_{pattern}{int(sp * 100)}",
             {"kind": "chain", "dtype": dt, "M": M, "K": K, "N": N, "seed": seed, "sparsity": sp,
              "pattern": pattern},
             {"mask": mask.numpy(), "alive": alive.numpy(), "y": y},
             {"x": x, "weight": weight, "bias": bias}, float_outputs=("y",))


def main() -> None:
    for old in HERE.glob("*.npz"):
        old.unlink()
    print("mask"); mask_cases()
    print("gather"); gather_cases()
    print("matmul"); matmul_cases()
    print("chain"); chain_cases()


if __name__ == "__main__":
    main()
