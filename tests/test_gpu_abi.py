"""GPU: C-ABI status codes and error behaviour, called with raw pointers via ctypes.

Every rejected call returns its status before anything is launched; nothing
here hands a kernel an invalid address.
"""

from __future__ import annotations

import pytest
import torch

from ghostweight_triton_b200 import _native

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    return _native.load()


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def test_device_supported(lib):
    assert lib.gw_device_supported(torch.cuda.current_device()) == 1


def test_shape_dtype_null_errors(lib):
    x = torch.randn(8, 64, device="cuda", dtype=torch.float16)
    w = torch.randn(32, 64, device="cuda", dtype=torch.float16)
    y = torch.empty(8, 32, device="cuda", dtype=torch.float16)
    idx = torch.arange(64, device="cuda")
    s = stream()
    ok = lib.gw_gather_gemm(x.data_ptr(), 0, 8, 64, 64, w.data_ptr(), 32, 64, idx.data_ptr(), 64,
                            None, 0, y.data_ptr(), 32, 1, None, 0, s)
    assert ok == _native.GW_OK
    assert lib.gw_gather_gemm(x.data_ptr(), 7, 8, 64, 64, w.data_ptr(), 32, 64, idx.data_ptr(), 64,
                              None, 0, y.data_ptr(), 32, 1, None, 0, s) == _native.GW_ERR_DTYPE
    assert lib.gw_gather_gemm(x.data_ptr(), 0, 8, 64, 10, w.data_ptr(), 32, 64, idx.data_ptr(), 64,
                              None, 0, y.data_ptr(), 32, 1, None, 0, s) == _native.GW_ERR_SHAPE
    assert lib.gw_gather_gemm(x.data_ptr(), 0, 8, 64, 64, w.data_ptr(), 32, 64, idx.data_ptr(), 64,
                              None, 9, y.data_ptr(), 32, 1, None, 0, s) == _native.GW_ERR_UNSUPPORTED
    assert lib.gw_gather_gemm(x.data_ptr(), 0, 8, 64, 64, w.data_ptr(), 32, 64, None, 64,
                              None, 0, y.data_ptr(), 32, 1, None, 0, s) == _native.GW_ERR_NULL
    # packed weight with ldw % 8 != 0 cannot be a TMA operand
    assert lib.gw_gather_gemm(x.data_ptr(), 0, 8, 64, 64, w.data_ptr(), 32, 65, idx.data_ptr(), 64,
                              None, 0, y.data_ptr(), 32, 1, None, 0, s) == _native.GW_ERR_ALIGN
    assert lib.gw_packed_gemm(x.data_ptr(), 2, 8, 64, 64, w.data_ptr(), 32, 64, None, 0,
                              y.data_ptr(), 32, s) == _native.GW_ERR_DTYPE
    # pregather without a (large enough) workspace
    assert lib.gw_gather_gemm(x.data_ptr(), 0, 8, 64, 64, w.data_ptr(), 32, 64, idx.data_ptr(), 64,
                              None, 0, y.data_ptr(), 32, 2, None, 0, s) == _native.GW_ERR_NULL
    ws = torch.empty(64, dtype=torch.uint8, device="cuda")
    assert lib.gw_gather_gemm(x.data_ptr(), 0, 8, 64, 64, w.data_ptr(), 32, 64, idx.data_ptr(), 64,
                              None, 0, y.data_ptr(), 32, 2, ws.data_ptr(), 64, s) == _native.GW_ERR_WORKSPACE
    assert lib.gw_gather_gemm(x.data_ptr(), 0, 8, 64, 64, w.data_ptr(), 32, 64, idx.data_ptr(), 64,
                              None, 0, y.data_ptr(), 32, 7, None, 0, s) == _native.GW_ERR_UNSUPPORTED
    assert lib.gw_gather_gemm_workspace_bytes(8, 64, 0) == 256 + 1024
    torch.cuda.synchronize()


def test_mask_workspace_errors(lib):
    x = torch.randn(8, 4096, device="cuda")
    m = torch.empty(4096, dtype=torch.int32, device="cuda")
    ws = torch.zeros(64, dtype=torch.uint8, device="cuda")
    s = stream()
    assert lib.gw_mask_compact(x.data_ptr(), 2, 8, 4096, 4096, 0.0, m.data_ptr(), None, None,
                               ws.data_ptr(), ws.numel(), s) == _native.GW_ERR_WORKSPACE
    assert lib.gw_mask_compact(x.data_ptr(), 2, 8, 4096, 4096, 0.0, m.data_ptr(), None, None,
                               None, 0, s) == _native.GW_ERR_NULL
    assert lib.gw_mask_compact(x.data_ptr(), 2, 8, 4096, 100, 0.0, m.data_ptr(), None, None,
                               ws.data_ptr(), ws.numel(), s) == _native.GW_ERR_SHAPE


def test_python_errors_are_raised():
    x = torch.randn(8, 64, device="cuda", dtype=torch.float16)
    w = torch.randn(32, 65, device="cuda", dtype=torch.float16)[:, :64]   # ld 65: misaligned
    y = torch.empty(8, 32, device="cuda", dtype=torch.float16)
    with pytest.raises(_native.GhostweightError, match="aligned"):
        _native.gather_gemm(x, w, torch.arange(64, device="cuda"), y)


def test_device_error_word_roundtrip():
    _native.device_error(reset=True)
    assert _native.device_error(reset=False) == 0


def test_validate_indices():
    idx = torch.tensor([0, 5, -1, 10, 9], device="cuda")
    assert _native.validate_indices(idx, 10) == 2
    assert _native.validate_indices(torch.arange(10, device="cuda"), 10) == 0
