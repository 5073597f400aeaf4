"""GPU: the allocation-free mask entry point gives the same answers as the regular one.

gw_mask_compact_static exists for callers that are not allowed to allocate
device memory once they are running (pre-planned serving memory, plugins
whose host owns all allocations, allocator callbacks). It keeps its scratch in
a static device array inside the library instead of taking a workspace. This
file is collected last on purpose, and must pass both on its own in a fresh
process and after the rest of the suite.

Mask and alive-index outputs are integers, so the comparison is exact, the
same standard the other mask tests use.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from ghostweight_triton_b200 import _native

pytestmark = pytest.mark.gpu

MAX_COLS = 1048576   # GW_MASK_STATIC_MAX_COLS in include/ghostweight_b200.h


def _run(entry: str, x: torch.Tensor, threshold: float):
    lib = _native.load()
    rows, cols = x.shape
    mask = torch.full((cols,), -1, dtype=torch.int32, device=x.device)
    idx = torch.full((cols,), -1, dtype=torch.int64, device=x.device)
    cnt = torch.full((1,), -1, dtype=torch.int32, device=x.device)
    stream = torch.cuda.current_stream().cuda_stream
    dt = _native.dtype_code(x.dtype)
    if entry == "static":
        st = lib.gw_mask_compact_static(x.data_ptr(), dt, rows, cols, cols, threshold,
                                        mask.data_ptr(), idx.data_ptr(), cnt.data_ptr(), stream)
    else:
        ws = torch.zeros(lib.gw_mask_workspace_bytes(cols), dtype=torch.uint8, device=x.device)
        st = lib.gw_mask_compact(x.data_ptr(), dt, rows, cols, cols, threshold, mask.data_ptr(),
                                 idx.data_ptr(), cnt.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    assert st == 0, _native.status_string(st)
    n = int(cnt.item())
    return mask.cpu().numpy(), idx[:n].cpu().numpy(), n


def _input(rows: int, cols: int, dtype: torch.dtype, dead_frac: float, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, cols, device="cuda", generator=g).to(dtype)
    dead = torch.randperm(cols, device="cuda", generator=g)[: int(cols * dead_frac)]
    x[:, dead] = 0
    return x


def test_two_calls_in_a_row_match_regular_entry():
    # Second call has fewer columns and a different dtype: whatever the first
    # call left in the shared static array must not leak into it.
    cases = [(_input(300, 8192, torch.bfloat16, 0.7, 1), 0.0),
             (_input(64, 1000, torch.float16, 0.4, 2), 1e-6)]
    for x, thr in cases:
        m_s, i_s, n_s = _run("static", x, thr)
        m_r, i_r, n_r = _run("regular", x, thr)
        assert n_s == n_r
        assert np.array_equal(m_s, m_r)
        assert np.array_equal(i_s, i_r)
        assert n_s == int((x.abs().float().amax(0) > thr).sum().item())


@pytest.mark.parametrize("rows,cols,dtype,thr", [
    (257, 8191, torch.float16, 0.0),       # odd column count: the scalar (one column per thread) kernel
    (33, 4096, torch.bfloat16, -1.0),      # negative threshold: every column alive
    (16, 0, torch.float32, 0.0),           # no columns: nothing launched, the count reads 0
])
def test_scalar_path_negative_threshold_and_empty(rows, cols, dtype, thr):
    # Each case is run twice through the static entry point, so the second
    # run starts from whatever the first left in the shared array.
    x = _input(rows, max(cols, 1), dtype, 0.5, 3)[:, :cols].contiguous()
    ref = _run("regular", x, thr)
    for _ in range(2):
        m_s, i_s, n_s = _run("static", x, thr)
        assert n_s == ref[2]
        assert np.array_equal(m_s, ref[0])
        assert np.array_equal(i_s, ref[1])
    assert n_s == (cols if thr < 0 else int((x.abs().float().amax(0) > thr).sum().item()) if cols else 0)


def test_oversized_request_is_rejected_without_launch():
    lib = _native.load()
    x = torch.zeros(1, 16, device="cuda")
    st = lib.gw_mask_compact_static(x.data_ptr(), 2, 1, MAX_COLS + 1, MAX_COLS + 1, 0.0,
                                    None, None, None, torch.cuda.current_stream().cuda_stream)
    assert st == _native.GW_ERR_WORKSPACE
    torch.cuda.synchronize()
