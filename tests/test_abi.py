"""CPU: the C-ABI library builds, loads and exports every declared symbol.

No compute entry point is called here (there is no GPU); only the pure-host
helpers (status strings, version, workspace sizing) are exercised.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from ghostweight_triton_b200 import _native

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "ghostweight_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^GW_API\s+[\w\s\*]+?\b(gw_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    if not _native.LIB_PATH.exists():
        from ghostweight_triton_b200.csrc import build

        build.build()
    return _native.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    for name in ("gw_mask_compact", "gw_gather_columns", "gw_gather_rows", "gw_gather_rows_t",
                 "gw_gather_gemm", "gw_packed_gemm", "gw_validate_indices"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in {HEADER.name} but not exported"


def test_python_binding_covers_header():
    assert sorted(_native.SIGNATURES) == declared_symbols()


def test_library_is_sm100a_only():
    """The shared object embeds sm_100a code only (cuobjdump-free check: nvcc flags)."""
    from ghostweight_triton_b200.csrc import build

    assert build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_status_strings(lib):
    assert lib.gw_status_string(0) == b"ok"
    for st in range(1, 9):
        assert lib.gw_status_string(st) not in (b"ok", b"unknown status")
    assert lib.gw_status_string(99) == b"unknown status"
    assert lib.gw_version() == b"0.1.0"


def test_mask_workspace_sizing(lib):
    assert lib.gw_mask_workspace_bytes(0) == 256
    assert lib.gw_mask_workspace_bytes(8192) == 1280          # 16 + 256 words * 4, rounded to 256
    assert lib.gw_mask_workspace_bytes(8192) % 256 == 0
    assert lib.gw_mask_workspace_bytes(1) >= 16 + 4


def test_gemm_workspace_sizing(lib):
    # Header (epoch, two counters and one 8-byte flag per 128-row x 64-column
    # unit of x', rounded up to 256 bytes) + x' [M, round_up(K', 64)] 16-bit.
    assert lib.gw_gather_gemm_workspace_bytes(8, 64, 0) == 256 + 8 * 64 * 2
    units = (2 * 4096 // 256) * (2048 // 64)
    hdr = (8 * (4 + units) + 255) // 256 * 256
    assert lib.gw_gather_gemm_workspace_bytes(4096, 2048, 0) == hdr + 4096 * 2048 * 2
    assert lib.gw_gather_gemm_workspace_bytes(4096, 2048, 2) == 0     # fp32 needs none
    assert lib.gw_gather_gemm_workspace_bytes(0, 2048, 0) == 0


def test_no_gpu_reports_unsupported(lib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert lib.gw_device_supported(0) == 0


def test_gemm_plan_without_gpu(lib):
    import ctypes

    import torch

    if torch.cuda.is_available():
        pytest.skip("GPU present")
    k, t, s = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    assert lib.gw_gemm_plan(-1, 4, 4, ctypes.byref(k), None, None) == 1          # GW_ERR_SHAPE
    assert lib.gw_gemm_plan(4, 4, 4, None, None, None) == 4                      # GW_ERR_NULL
    assert lib.gw_gemm_plan(4, 4, 4, ctypes.byref(k), ctypes.byref(t), ctypes.byref(s)) != 0


def test_dtype_and_epilogue_codes():
    import torch

    assert _native.dtype_code(torch.float16) == 0
    assert _native.dtype_code(torch.bfloat16) == 1
    assert _native.dtype_code(torch.float32) == 2
    with pytest.raises(TypeError):
        _native.dtype_code(torch.int8)
    assert _native.epilogue_code(None) == 0 and _native.epilogue_code("gelu_tanh") == 2
    with pytest.raises(ValueError):
        _native.epilogue_code("relu")


def test_load_missing_library_raises(tmp_path):
    with pytest.raises(RuntimeError, match="not built"):
        _native.load(tmp_path / "libghostweight_b200.so")


def test_ctypes_signatures_match_arity(lib):
    text = HEADER.read_text()
    for name, (_, args) in _native.SIGNATURES.items():
        m = re.search(rf"\b{name}\s*\(([^)]*)\)", text, re.S)
        assert m, name
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), f"{name}: header has {len(params)} params, binding {len(args)}"


def test_fast_call_binding_shares_the_library(lib):
    """The CPython fast-call module binds the same library copy ctypes loaded, and
    covers the hot entry points with the same argument lists."""
    import ctypes as C

    api = _native.api()
    assert api.fast, "fast-call module not built or bound to a second library copy"
    from ghostweight_triton_b200 import _gwfast

    assert _gwfast.library_anchor() == C.cast(lib.gw_version, C.c_void_p).value
    for name in _native.FAST_ENTRIES:
        assert name in _native.SIGNATURES and hasattr(_gwfast, name[3:])
        assert len(_native.SIGNATURES[name][1]) >= 3
    # Pure host arithmetic through both bindings agrees.
    for M, n, dt in [(4096, 2048, 0), (8, 64, 1), (0, 10, 0), (300, 77, 2)]:
        assert api.gw_gather_gemm_workspace_bytes(M, n, dt) == lib.gw_gather_gemm_workspace_bytes(M, n, dt)
    import pytest as _pt

    with _pt.raises(TypeError):
        _gwfast.gather_gemm(1, 2, 3)            # wrong argument count is a Python error, not a call
