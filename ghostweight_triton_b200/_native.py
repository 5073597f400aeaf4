"""ctypes binding of libghostweight_b200.so (the sm_100a C ABI).

Every function here takes torch CUDA tensors, passes raw device pointers,
sizes and torch's current stream to the C ABI declared in
``include/ghostweight_b200.h`` and turns a non-zero status into an exception.
There is no fallback: if the library is missing or the GPU is not an sm_100
part, calls raise.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_NAME = "libghostweight_b200.so"
LIB_PATH = Path(__file__).resolve().with_name(LIB_NAME)

# gw_dtype / gw_epilogue / gw_status values (include/ghostweight_b200.h).
DTYPE_CODES = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}
EPILOGUES = {None: 0, "none": 0, "gelu": 1, "gelu_erf": 1, "gelu_tanh": 2}
GW_OK = 0
GW_ERR_SHAPE = 1
GW_ERR_DTYPE = 2
GW_ERR_ALIGN = 3
GW_ERR_NULL = 4
GW_ERR_WORKSPACE = 5
GW_ERR_CUDA = 6
GW_ERR_DEVICE = 7
GW_ERR_UNSUPPORTED = 8
GEMM_STRATEGIES = {"auto": 0, "fused": 1, "pregather": 2, "overlap": 3, "runs": 4}
DEVICE_ERR_WAIT_TIMEOUT = 1
DEVICE_ERR_BAD_INDEX = 2

# Exported symbols and their ctypes signatures.
_vp, _i, _i64, _sz, _d = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_double
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "gw_status_string": (ctypes.c_char_p, [_i]),
    "gw_last_cuda_error": (ctypes.c_char_p, []),
    "gw_version": (ctypes.c_char_p, []),
    "gw_device_supported": (_i, [_i]),
    "gw_get_device_error": (_i, [_i, ctypes.POINTER(ctypes.c_uint)]),
    "gw_mask_workspace_bytes": (_sz, [_i64]),
    "gw_mask_compact": (_i, [_vp, _i, _i64, _i64, _i64, _d, _vp, _vp, _vp, _vp, _sz, _vp]),
    "gw_mask_compact_static": (_i, [_vp, _i, _i64, _i64, _i64, _d, _vp, _vp, _vp, _vp]),
    "gw_gather_columns": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _vp]),
    "gw_gather_rows": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _vp]),
    "gw_gather_rows_t": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _vp]),
    "gw_gather_gemm_workspace_bytes": (_sz, [_i64, _i64, _i]),
    "gw_gather_gemm": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _i,
                            _vp, _i64, _i, _vp, _sz, _vp]),
    "gw_gather_gemm_peers": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _i,
                                  _vp, _i64, _vp, _i, _i, _vp, _sz, _vp]),
    "gw_packed_gemm": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i, _vp, _i64, _vp]),
    "gw_validate_indices": (_i, [_vp, _i64, _i64, _vp, _vp]),
    "gw_index_runs": (_i, [_vp, _i64, _i64, _vp, _vp]),
    "gw_gemm_plan": (_i, [_i64, _i64, _i64, ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "gw_selftest_wait_timeout": (_i, [_i64, _vp]),
    "gw_dynamic_linear": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _i64, _i64, _d, _vp, _i, _vp, _i64,
                               _vp, _vp, _vp]),
    "gw_gather_columns_dev": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _vp]),
    "gw_gather_rows_t_dev": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _vp]),
    "gw_gather_gemm_dev": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _vp, _i,
                                _vp, _i64, _vp, _sz, _vp]),
}

_lib: ctypes.CDLL | None = None
_lib_lock = threading.Lock()
_api = None
# Entry points the CPython fast-call module (_gwfast, built from csrc/gw_pyfast.c)
# binds; the same arguments as the ctypes functions, a fraction of the host time.
FAST_ENTRIES = ("gw_gather_gemm", "gw_gather_gemm_dev", "gw_packed_gemm", "gw_gather_columns", "gw_dynamic_linear",
                "gw_gather_rows_t", "gw_gather_columns_dev", "gw_gather_rows_t_dev", "gw_mask_compact",
                "gw_gather_gemm_workspace_bytes")


class _Api:
    """The library's entry points by C name: the fast-call binding where it covers
    them and the one library copy checks out, else the ctypes functions."""

    def __init__(self, lib: ctypes.CDLL):
        for name in SIGNATURES:
            setattr(self, name, getattr(lib, name))
        self.fast = False
        try:
            from ghostweight_triton_b200 import _gwfast
        except ImportError:
            return
        if _gwfast.library_anchor() != ctypes.cast(lib.gw_version, ctypes.c_void_p).value:
            return          # a second copy of the library: keep everything on ctypes
        for name in FAST_ENTRIES:
            setattr(self, name, getattr(_gwfast, name[3:]))
        self.fast = True


def api() -> _Api:
    """Entry points of the loaded library (see _Api); loads it on first use."""
    global _api
    if _api is None:
        lib = load()
        with _lib_lock:
            if _api is None:
                _api = _Api(lib)
    return _api


class GhostweightError(RuntimeError):
    """A C-ABI call of libghostweight_b200.so returned a non-zero status."""

    def __init__(self, status: int, what: str, detail: str = ""):
        self.status = status
        msg = f"{what}: {status_string(status)} (status {status})"
        if detail:
            msg += f" [{detail}]"
        super().__init__(msg)


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and return the native library; raises if it is absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lib_lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p.name} is not built: run `python -m ghostweight_triton_b200.csrc.build` "
                "(nvcc for sm_100a); there is no non-native fallback"
            )
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def status_string(status: int) -> str:
    try:
        return load().gw_status_string(int(status)).decode()
    except Exception:  # library itself unavailable
        return "unknown"


def _check(status: int, what: str) -> None:
    if status != GW_OK:
        detail = load().gw_last_cuda_error().decode() if status == GW_ERR_CUDA else ""
        raise GhostweightError(status, what, detail)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}; expected float16, bfloat16 or float32") from None


def epilogue_code(activation: str | None) -> int:
    try:
        return EPILOGUES[activation]
    except KeyError:
        raise ValueError(f"unsupported activation {activation!r}; expected None, 'gelu' or 'gelu_tanh'") from None


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _rowmajor(*ts: torch.Tensor) -> None:
    """Matrices cross the ABI as (pointer, leading dimension): unit column stride required."""
    for t in ts:
        assert t.ndim == 2 and (t.stride(1) == 1 or t.shape[1] <= 1), (
            f"expected a row-major matrix, got shape {tuple(t.shape)} strides {t.stride()}")


try:  # the raw cudaStream_t of torch's current stream, without building a Stream object
    _raw_stream = torch._C._cuda_getCurrentRawStream
except AttributeError:  # pragma: no cover - older torch
    _raw_stream = None


def _stream(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(idx)
    return torch.cuda.current_stream(device).cuda_stream


class _on_device:
    """Make `device` current for the duration of a C call (cheap when already current)."""

    __slots__ = ("idx", "prev")

    def __init__(self, device: torch.device):
        self.idx = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


# ---------------------------------------------------------------------------
# Mask workspace: zero-initialised once, returned to zero by every call.
# One buffer per (device, stream) so concurrent streams never share one.
# ---------------------------------------------------------------------------
_ws_cache: dict[tuple[int, int], torch.Tensor] = {}
_ws_lock = threading.Lock()


def mask_workspace(device: torch.device, cols: int) -> torch.Tensor:
    need = int(load().gw_mask_workspace_bytes(int(cols)))
    key = (device.index if device.index is not None else torch.cuda.current_device(), _stream(device))
    with _ws_lock:
        ws = _ws_cache.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.zeros(max(need, 4096), dtype=torch.uint8, device=device)
            _ws_cache[key] = ws
    return ws


# ---------------------------------------------------------------------------
# Thin wrappers (tensors in, tensors out; no allocation except where noted)
# ---------------------------------------------------------------------------
def mask_compact(x: torch.Tensor, threshold: float, mask: torch.Tensor | None = None,
                 alive_idx: torch.Tensor | None = None, count: torch.Tensor | None = None) -> None:
    """K1 over a row-major [rows, cols] CUDA matrix (x.stride(1) == 1)."""
    assert x.ndim == 2 and (x.stride(1) == 1 or x.shape[1] <= 1)
    rows, cols = x.shape
    ws = mask_workspace(x.device, cols)
    with _on_device(x.device):
        st = api().gw_mask_compact(
            _ptr(x), dtype_code(x.dtype), rows, cols, max(x.stride(0), cols), float(threshold),
            _ptr(mask), _ptr(alive_idx), _ptr(count), _ptr(ws), ws.numel(), _stream(x.device))
    _check(st, "gw_mask_compact")


def gather_columns(src: torch.Tensor, idx: torch.Tensor, dst: torch.Tensor, pad_to: int | None = None) -> None:
    """dst[r, j] = src[r, idx[j]]; zero columns [len(idx), pad_to)."""
    _rowmajor(src, dst)
    assert idx.dtype == torch.int64
    rows, cols = src.shape
    n = idx.numel()
    pad = n if pad_to is None else int(pad_to)
    with _on_device(src.device):
        st = api().gw_gather_columns(
            _ptr(src), dtype_code(src.dtype), rows, cols, max(src.stride(0), cols), _ptr(idx), n,
            _ptr(dst), max(dst.stride(0), pad), pad, _stream(src.device))
    _check(st, "gw_gather_columns")


def gather_rows(src: torch.Tensor, idx: torch.Tensor, dst: torch.Tensor) -> None:
    """dst[j, :] = src[idx[j], :]."""
    _rowmajor(src, dst)
    assert idx.dtype == torch.int64
    rows, cols = src.shape
    n = idx.numel()
    with _on_device(src.device):
        st = load().gw_gather_rows(
            _ptr(src), dtype_code(src.dtype), rows, cols, max(src.stride(0), cols), _ptr(idx), n,
            _ptr(dst), max(dst.stride(0), cols), _stream(src.device))
    _check(st, "gw_gather_rows")


def gather_rows_t(src: torch.Tensor, idx: torch.Tensor, dst: torch.Tensor, pad_to: int | None = None) -> None:
    """dst[n, j] = src[idx[j], n]; zero columns [len(idx), pad_to)."""
    _rowmajor(src, dst)
    assert idx.dtype == torch.int64
    rows, cols = src.shape
    n = idx.numel()
    pad = n if pad_to is None else int(pad_to)
    with _on_device(src.device):
        st = api().gw_gather_rows_t(
            _ptr(src), dtype_code(src.dtype), rows, cols, max(src.stride(0), cols), _ptr(idx), n,
            _ptr(dst), max(dst.stride(0), pad), pad, _stream(src.device))
    _check(st, "gw_gather_rows_t")


_ws_bytes: dict[tuple[int, int, torch.dtype], int] = {}


def gather_gemm_workspace_bytes(M: int, n_alive: int, dtype: torch.dtype) -> int:
    key = (M, n_alive, dtype)
    n = _ws_bytes.get(key)
    if n is None:
        n = int(api().gw_gather_gemm_workspace_bytes(int(M), int(n_alive), dtype_code(dtype)))
        if len(_ws_bytes) > 4096:
            _ws_bytes.clear()
        _ws_bytes[key] = n
    return n


# GEMM workspaces reused across calls: one per (device, stream), grown as
# needed. Calls on one stream are ordered, so they may share it; under CUDA
# graph capture a fresh buffer is allocated instead (from the graph's pool), so
# a captured graph never refers to a buffer that a later call replaces.
_gemm_ws: dict[tuple[int, int], torch.Tensor] = {}


def gemm_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    if torch.cuda.is_current_stream_capturing():
        return torch.empty(nbytes, dtype=torch.uint8, device=device)
    dev = device.index if device.index is not None else torch.cuda.current_device()
    key = (dev, _stream(device))
    ws = _gemm_ws.get(key)
    if ws is None or ws.numel() < nbytes:
        with _ws_lock:
            ws = _gemm_ws.get(key)
            if ws is None or ws.numel() < nbytes:
                ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
                _gemm_ws[key] = ws
    return ws


def gather_gemm(x: torch.Tensor, w_packed: torch.Tensor, idx: torch.Tensor, y: torch.Tensor,
                bias: torch.Tensor | None = None, activation: str | None = None,
                strategy: str = "auto", workspace: torch.Tensor | None = None) -> None:
    """y = act(x[:, idx] @ w_packed[:, :len(idx)]^T + bias) on the current stream.

    strategy "auto" uses the two-launch pregather path when `workspace` is large
    enough, else the single fused kernel; "fused" / "pregather" force one;
    "runs" loads x directly (idx must be 64-column runs: see index_runs).
    """
    _rowmajor(x, w_packed, y)
    assert idx.dtype == torch.int64 and idx.is_contiguous()
    M, K = x.shape
    N = w_packed.shape[0]
    n = idx.numel()
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel() * workspace.element_size())
    dev = x.get_device()
    cur = torch.cuda.current_device()
    if dev != cur:
        torch.cuda.set_device(dev)
    try:
        st = api().gw_gather_gemm(
            x.data_ptr(), DTYPE_CODES[x.dtype], M, K, max(x.stride(0), K), w_packed.data_ptr(), N,
            max(w_packed.stride(0), n), idx.data_ptr(), n, _ptr(bias), epilogue_code(activation),
            y.data_ptr(), max(y.stride(0), N), GEMM_STRATEGIES[strategy], ws_ptr, ws_bytes,
            _raw_stream(dev) if _raw_stream is not None else torch.cuda.current_stream().cuda_stream)
    finally:
        if dev != cur:
            torch.cuda.set_device(cur)
    if st:
        _check(st, "gw_gather_gemm")


def prepare_gather_gemm(w_packed: torch.Tensor, idx: torch.Tensor, bias: torch.Tensor | None,
                        activation: str | None, strategy: str, dtype: torch.dtype) -> tuple:
    """The arguments of gw_gather_gemm that stay fixed across calls with one packed
    weight, alive list and bias (for :func:`gather_gemm_prepared`). The tensors
    must stay alive and unchanged while the tuple is used."""
    _rowmajor(w_packed)
    assert idx.dtype == torch.int64 and idx.is_contiguous()
    n = idx.numel()
    return (DTYPE_CODES[dtype], w_packed.data_ptr(), w_packed.shape[0], max(w_packed.stride(0), n),
            idx.data_ptr(), n, _ptr(bias), epilogue_code(activation), GEMM_STRATEGIES[strategy])


def gather_gemm_prepared(prep: tuple, x: torch.Tensor, y: torch.Tensor) -> None:
    """gather_gemm(x, ...) with the fixed arguments of :func:`prepare_gather_gemm`.

    x [M, K] must be contiguous and on the current device, y [M, N] contiguous.
    The "runs" strategy falls back to "auto" for x rows that TMA cannot load in
    place (not 16-byte aligned), as gather_gemm does.
    """
    dtc, wptr, N, ldw, iptr, n, bptr, epi, strat = prep
    M, K = x.shape
    if strat == GEMM_STRATEGIES["runs"] and (x.data_ptr() % 16 or K % 8):
        strat = GEMM_STRATEGIES["auto"]
    ws_ptr, ws_bytes = None, 0
    if strat != GEMM_STRATEGIES["runs"] and strat != GEMM_STRATEGIES["fused"] and dtc != 2:
        ws_bytes = gather_gemm_workspace_bytes(M, n, x.dtype)
        if ws_bytes:
            ws = gemm_workspace(x.device, ws_bytes)
            ws_ptr, ws_bytes = ws.data_ptr(), ws.numel()
    dev = x.get_device()
    st = api().gw_gather_gemm(
        x.data_ptr(), dtc, M, K, K, wptr, N, ldw, iptr, n, bptr, epi, y.data_ptr(), N, strat,
        ws_ptr, ws_bytes, _raw_stream(dev) if _raw_stream is not None else torch.cuda.current_stream().cuda_stream)
    if st:
        _check(st, "gw_gather_gemm")


def gather_columns_dev(src: torch.Tensor, idx: torch.Tensor, n_dev: torch.Tensor, dst: torch.Tensor,
                       pad_to: int) -> None:
    """dst[r, j] = src[r, idx[j]] for j < n (n = n_dev[0] on the device, at most len(idx)); zero
    columns [n, round_up(max(n, 1), 64)). No synchronisation."""
    _rowmajor(src, dst)
    assert idx.dtype == torch.int64 and n_dev.dtype == torch.int32
    rows, cols = src.shape
    with _on_device(src.device):
        st = api().gw_gather_columns_dev(
            _ptr(src), dtype_code(src.dtype), rows, cols, max(src.stride(0), cols), _ptr(idx),
            idx.numel(), _ptr(n_dev), _ptr(dst), max(dst.stride(0), pad_to), int(pad_to),
            _stream(src.device))
    _check(st, "gw_gather_columns_dev")


def gather_rows_t_dev(src: torch.Tensor, idx: torch.Tensor, n_dev: torch.Tensor, dst: torch.Tensor,
                      pad_to: int) -> None:
    """dst[n, j] = src[idx[j], n] for j < n_dev[0]; zero up to the next 64-column boundary."""
    _rowmajor(src, dst)
    assert idx.dtype == torch.int64 and n_dev.dtype == torch.int32
    rows, cols = src.shape
    with _on_device(src.device):
        st = api().gw_gather_rows_t_dev(
            _ptr(src), dtype_code(src.dtype), rows, cols, max(src.stride(0), cols), _ptr(idx),
            idx.numel(), _ptr(n_dev), _ptr(dst), max(dst.stride(0), pad_to), int(pad_to),
            _stream(src.device))
    _check(st, "gw_gather_rows_t_dev")


def gather_gemm_dev(x: torch.Tensor, w_packed: torch.Tensor, idx: torch.Tensor, n_dev: torch.Tensor,
                    y: torch.Tensor, bias: torch.Tensor | None = None, activation: str | None = None,
                    workspace: torch.Tensor | None = None) -> None:
    """gather_gemm with K' = n_dev[0] read on the device (len(idx) is its upper bound)."""
    _rowmajor(x, w_packed, y)
    assert idx.dtype == torch.int64 and n_dev.dtype == torch.int32
    M, K = x.shape
    N = w_packed.shape[0]
    n = idx.numel()
    if workspace is None and x.dtype != torch.float32:
        nbytes = gather_gemm_workspace_bytes(M, n, x.dtype)
        workspace = gemm_workspace(x.device, nbytes) if nbytes else None
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel() * workspace.element_size())
    with _on_device(x.device):
        st = api().gw_gather_gemm_dev(
            _ptr(x), dtype_code(x.dtype), M, K, max(x.stride(0), K), _ptr(w_packed), N,
            w_packed.stride(0), _ptr(idx), n, _ptr(n_dev), _ptr(bias), epilogue_code(activation),
            _ptr(y), max(y.stride(0), N), ws_ptr, ws_bytes, _stream(x.device))
    _check(st, "gw_gather_gemm_dev")


def gather_gemm_peers(x: torch.Tensor, w_packed: torch.Tensor, idx: torch.Tensor, y: torch.Tensor,
                      peer_addresses: list[int], bias: torch.Tensor | None = None,
                      activation: str | None = None, workspace: torch.Tensor | None = None,
                      strategy: str = "pregather") -> None:
    """gather_gemm whose output block y also goes to each peer address.

    y is this rank's block of a full output (a column slice view, row stride
    ldy); peer_addresses are device addresses of the same block in the other
    ranks' full outputs (same row stride), valid in this process. strategy is
    "pregather" (gather, then the GEMM) or "runs" (no gather; see index_runs).
    """
    _rowmajor(x, w_packed)
    assert y.ndim == 2 and y.stride(1) == 1
    assert idx.dtype == torch.int64 and idx.is_contiguous()
    M, K = x.shape
    N = y.shape[1]
    n = idx.numel()
    if workspace is None and strategy != "runs":
        nbytes = gather_gemm_workspace_bytes(M, n, x.dtype)
        workspace = gemm_workspace(x.device, nbytes) if nbytes else None
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (workspace.data_ptr(), workspace.numel() * workspace.element_size())
    peers = (ctypes.c_void_p * max(1, len(peer_addresses)))(*[ctypes.c_void_p(a) for a in peer_addresses])
    with _on_device(x.device):
        st = load().gw_gather_gemm_peers(
            _ptr(x), dtype_code(x.dtype), M, K, max(x.stride(0), K), _ptr(w_packed), N,
            max(w_packed.stride(0), n), _ptr(idx), n, _ptr(bias), epilogue_code(activation),
            _ptr(y), y.stride(0), peers, len(peer_addresses), GEMM_STRATEGIES[strategy], ws_ptr,
            ws_bytes, _stream(x.device))
    _check(st, "gw_gather_gemm_peers")


def packed_gemm(a: torch.Tensor, w_packed: torch.Tensor, y: torch.Tensor,
                bias: torch.Tensor | None = None, activation: str | None = None) -> None:
    """y = act(a @ w_packed[:, :K]^T + bias) with both operands loaded by TMA."""
    _rowmajor(a, w_packed, y)
    M, K = a.shape
    N = w_packed.shape[0]
    with _on_device(a.device):
        st = api().gw_packed_gemm(
            _ptr(a), dtype_code(a.dtype), M, K, max(a.stride(0), K), _ptr(w_packed), N,
            max(w_packed.stride(0), K), _ptr(bias), epilogue_code(activation), _ptr(y),
            max(y.stride(0), N), _stream(a.device))
    _check(st, "gw_packed_gemm")


def dynamic_linear(x: torch.Tensor, weight: torch.Tensor, threshold: float, y: torch.Tensor,
                   bias: torch.Tensor | None = None, activation: str | None = None,
                   count: torch.Tensor | None = None, mask: torch.Tensor | None = None) -> int:
    """Mask of x's columns and the sparse layer y = act(x[:, alive] @ weight[:, alive]^T + bias)
    in one launch (gw_dynamic_linear). Returns the gw_status: GW_ERR_UNSUPPORTED for shapes
    or layouts the single launch does not take (the caller then runs the separate kernels);
    raises on any other error."""
    M, K = x.shape
    N = weight.shape[0]
    with _on_device(x.device):
        st = api().gw_dynamic_linear(
            x.data_ptr(), DTYPE_CODES[x.dtype], M, K, x.stride(0), weight.data_ptr(), N,
            weight.stride(0), float(threshold), _ptr(bias), epilogue_code(activation), y.data_ptr(),
            y.stride(0), _ptr(count), _ptr(mask), _stream(x.device))
    if st != GW_OK and st != GW_ERR_UNSUPPORTED:
        _check(st, "gw_dynamic_linear")
    return st


def validate_indices(idx: torch.Tensor, K: int) -> int:
    """Number of entries of idx outside [0, K) (synchronises)."""
    bad = torch.empty(1, dtype=torch.int32, device=idx.device)
    with _on_device(idx.device):
        st = load().gw_validate_indices(_ptr(idx), idx.numel(), int(K), _ptr(bad), _stream(idx.device))
    _check(st, "gw_validate_indices")
    return int(bad.item())


def index_runs(idx: torch.Tensor, K: int) -> int:
    """Entries of idx that break the 64-column-run structure of strategy "runs"
    (0: the list qualifies; synchronises)."""
    bad = torch.empty(1, dtype=torch.int32, device=idx.device)
    with _on_device(idx.device):
        st = load().gw_index_runs(_ptr(idx), idx.numel(), int(K), _ptr(bad), _stream(idx.device))
    _check(st, "gw_index_runs")
    return int(bad.item())


GEMM_KERNELS = {1: "pair", 2: "decode", 3: "splitk", 4: "single"}


def gemm_plan(M: int, N: int, K: int) -> tuple[str, int, int]:
    """(kernel, tile width, cluster size) the dense GEMM runs for an M x N output over K
    columns on the current device (gw_gemm_plan); 0 where the kernel has no such size."""
    kernel, tile_n, split = _i(), _i(), _i()
    _check(load().gw_gemm_plan(int(M), int(N), int(K), ctypes.byref(kernel), ctypes.byref(tile_n),
                               ctypes.byref(split)), "gw_gemm_plan")
    return GEMM_KERNELS[kernel.value], tile_n.value, split.value


def device_error(reset: bool = True, device: torch.device | None = None) -> int:
    """Device error word bits (DEVICE_ERR_*) of `device` (synchronises)."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    out = ctypes.c_uint(0)
    with _on_device(dev):
        st = load().gw_get_device_error(1 if reset else 0, ctypes.byref(out))
    _check(st, "gw_get_device_error")
    return int(out.value)


def selftest_wait_timeout(limit_ns: int = 1_000_000, device: torch.device | None = None) -> None:
    """Launch the bounded-wait self-test kernel on the current stream (its waits
    give up after limit_ns and raise DEVICE_ERR_WAIT_TIMEOUT; no synchronisation)."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    with _on_device(dev):
        st = load().gw_selftest_wait_timeout(int(limit_ns), _stream(dev))
    _check(st, "gw_selftest_wait_timeout")


def device_supported(device: int = 0) -> bool:
    return bool(load().gw_device_supported(int(device)))
