"""CPU: pin the numpy oracle to the reference's own outputs.

Every golden fixture in tests/golden/ was produced by the reference's Triton
kernels (tests/golden/make_golden.py). Masks, index lists and gathers must
match bit for bit; matmul outputs within the reference's own tolerances
(tests/test_matmul.py:68-72: fp16 1e-2, fp32 1e-4).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import gw_oracle as O
from tests.golden import gw_golden as G
from tests.golden.gw_inputs import rand_matrix, dead_columns, alive_from_dead, zero_columns

TOL = {"f16": (1e-2, 1e-2), "bf16": (1e-2, 1e-2), "f32": (1e-4, 1e-4)}


def test_fixtures_present():
    for kind in ("mask", "gather", "matmul", "chain"):
        assert G.names(kind), f"no golden fixtures of kind {kind}"


@pytest.mark.parametrize("name", G.names("mask"))
def test_mask_matches_reference(name):
    meta, inp, exp = G.load(name)
    G.check_exact(O.dead_neuron_mask(inp["a"], meta["threshold"], meta["dtype"]), exp, "mask")


@pytest.mark.parametrize("name", G.names("gather"))
def test_gather_matches_reference(name):
    meta, inp, exp = G.load(name)
    idx = exp["idx"]
    G.check_exact(O.gather_columns(inp["A"], idx), exp, "A_c")
    G.check_exact(O.gather_rows(inp["W"], idx), exp, "W_c")


@pytest.mark.parametrize("name", G.names("matmul"))
def test_matmul_matches_reference(name):
    meta, inp, exp = G.load(name)
    atol, rtol = TOL[meta["dtype"]]
    C = O.ghostweight_matmul(inp["A"], inp["W"], exp["idx"], meta["dtype"])
    G.check_close(C, exp, "C", atol, rtol)


@pytest.mark.parametrize("name", G.names("chain"))
def test_chain_matches_reference(name):
    meta, inp, exp = G.load(name)
    dt = meta["dtype"]
    mask = O.dead_neuron_mask(inp["x"], 1e-6, dt)
    G.check_exact(mask, exp, "mask")
    alive = O.alive_indices(mask)
    G.check_exact(alive, exp, "alive")
    atol, rtol = TOL[dt]
    y = O.ghost_linear(inp["x"], inp["weight"], alive, inp["bias"], dtype=dt)
    G.check_close(y, exp, "y", atol, rtol)


def test_inline_inputs_match_generator():
    """Inline fixtures were built by the same seeded generator the tests use."""
    for name in G.names("mask"):
        meta, inp, _ = G.load(name)
        if meta.get("inline") and "seed" in meta:
            regen = G._regenerate(meta)["a"]
            assert np.array_equal(regen.view(np.uint8), inp["a"].view(np.uint8)), name


# --------------------------------------------------------------------------
# Known answers from the reference suite, restated against the oracle
# --------------------------------------------------------------------------
def test_known_answers():
    a = np.full((4, 64), 0.01, np.float32)
    assert O.dead_neuron_mask(a, 0.01).sum() == 0                      # test_mask.py:130-140
    a = np.full((4, 64), 0.01 + 1e-4, np.float32)
    assert O.dead_neuron_mask(a, 0.01).sum() == 64                     # :142-148
    a = np.zeros((8, 64), np.float32); a[-1, 0] = 1.0
    m = O.dead_neuron_mask(a, 1e-6)
    assert m[0] == 1 and m[1:].sum() == 0                              # :171-179
    a = rand_matrix((8, 200), 9, "f16")
    a = zero_columns(a, dead_columns(200, 0.4, 9))
    assert O.dead_neuron_mask(a, 1e-6).sum() == 200 - 80               # :218-228


def test_fp32_compare_semantics():
    """fp16 value 1.0133e-6 > fp32(1e-6): alive in the reference kernel (fp32 compare)."""
    a = np.full((2, 16), 1.0133e-6, np.float16)
    assert O.dead_neuron_mask(a, 1e-6).sum() == 16


def test_nan_semantics():
    a = np.zeros((4, 4), np.float32)
    a[0, 0] = np.nan; a[1, 0] = 1.0          # NaN ignored, other row alive
    a[:, 1] = np.nan                          # all NaN: max stays 0 -> dead
    m = O.dead_neuron_mask(a, 1e-6)
    assert m.tolist() == [1, 0, 0, 0]
    assert O.dead_neuron_mask(a, -1.0).tolist() == [1, 1, 1, 1]


def test_bf16_roundtrip_and_matmul():
    x = rand_matrix((8, 32), 1, "bf16")
    f = O.to_f32(x, "bf16")
    assert np.array_equal(O.from_f32(f, "bf16"), x)
    idx = np.arange(0, 32, 2)
    w = rand_matrix((32, 16), 2, "bf16")
    c = O.ghostweight_matmul(x, w, idx, "bf16")
    ref = (f[:, idx] @ O.to_f32(w, "bf16")[idx, :])
    assert np.allclose(O.to_f32(c, "bf16"), ref, atol=1e-2, rtol=1e-2)


def test_empty_index_gives_zeros():
    a = rand_matrix((3, 8), 1, "f32"); w = rand_matrix((8, 5), 2, "f32")
    c = O.ghostweight_matmul(a, w, np.zeros(0, np.int64))
    assert c.shape == (3, 5) and not c.any()


def test_pack_weight_layout():
    w = rand_matrix((6, 10), 3, "f16")
    idx = np.array([1, 4, 9])
    p = O.pack_weight(w, idx, pad_to=8)
    assert p.shape == (6, 8)
    assert np.array_equal(p[:, :3], w[:, idx]) and not p[:, 3:].any()


def test_ghost_linear_equals_dense_when_dead_columns_zero():
    """Dead (all-zero) columns contribute nothing: the identity the path relies on."""
    x = rand_matrix((16, 64), 4, "f32")
    dead = dead_columns(64, 0.5, 4)
    x = zero_columns(x, dead)
    w = rand_matrix((24, 64), 5, "f32")
    alive = alive_from_dead(64, dead)
    y_sparse = O.ghost_linear(x, w, alive, dtype="f32")
    y_dense = O.ghost_linear(x, w, np.arange(64), dtype="f32")
    assert np.allclose(y_sparse, y_dense, atol=1e-5, rtol=1e-5)


def test_index_runs_structure():
    """Lists of whole 64-column runs (starts multiple of 8) have no violations, and
    their gather equals the concatenated 64-column slices of x."""
    K = 1024
    for block in (64, 128):
        idx = alive_from_dead(K, dead_columns(K, 0.5, 3, "block", block))
        assert O.index_runs(idx, K) == 0
        x = rand_matrix((5, K), 4, "f16")
        slices = np.concatenate([x[:, s:s + 64] for s in idx[::64]], axis=1)
        assert np.array_equal(O.gather_columns(x, idx), slices)
    assert O.index_runs(np.arange(8, 8 + 128), K) == 0           # start 8: 16-byte aligned
    assert O.index_runs(np.arange(4, 4 + 64), K) == 64            # start 4: whole run misaligned
    assert O.index_runs(np.arange(0, 96), K) == 32                # trailing partial run
    broken = np.arange(0, 128)
    broken[70] = 500
    assert O.index_runs(broken, K) == 1
    assert O.index_runs(np.arange(K - 32, K + 32), K) == 32       # 32 entries past K
    assert O.index_runs(np.array([], dtype=np.int64), K) == 0
    random_idx = alive_from_dead(K, dead_columns(K, 0.5, 3, "random"))
    assert O.index_runs(random_idx, K) > 0
