"""Fused gather-GEMM on B200.

``ghostweight_matmul`` mirrors ghostweight_triton/kernels/matmul.py:85-142:
C[M, N] = A[:, alive] @ W[alive, :] with fp32 accumulation, cast to A's dtype;
unsorted or repeated indices are fine and an empty index list gives zeros.
On B200 the weight rows are first packed into the K'-major operand (one
transposing gather) and the product runs on the tcgen05 kernel K3
(csrc/gw_gemm_tc.cu). Two strategies feed its A operand: "pregather" gathers
the alive activation columns into a dense scratch matrix and streams both
operands by TMA (two launches; the default when a workspace is affordable),
"fused" has producer warps gather them straight into shared memory (one
launch, no scratch). fp32 inputs use the exact-fp32 kernel, matching the
reference's TF32-off choice for fp32 (matmul.py:127-130).

``ghost_linear`` is the module-level entry: activations [M, K] times an
already packed weight, with bias and optional GELU fused into the epilogue.
"""

from __future__ import annotations

import torch

from ghostweight_triton_b200 import _native
from ghostweight_triton_b200.kernels.gather import pack_weight


def ghostweight_matmul(
    activations: torch.Tensor,
    weights: torch.Tensor,
    alive_indices: torch.Tensor,
    BLOCK_M: int = 64,
    BLOCK_N: int = 64,
    BLOCK_K: int = 32,
    *,
    bias: torch.Tensor | None = None,
    activation: str | None = None,
    strategy: str = "auto",
) -> torch.Tensor:
    """Sparse matmul that skips dead neurons.

    Parameters
    ----------
    activations   : [M, K]
    weights       : [K, N]
    alive_indices : [K_alive], any integer dtype (converted to int64)
    BLOCK_M, BLOCK_N, BLOCK_K : accepted for signature compatibility; ignored.
    bias          : optional [N], added in the fp32 epilogue (extension).
    activation    : None, "gelu" or "gelu_tanh", applied after the bias (extension).
    strategy      : "auto" | "pregather" | "fused" | "overlap" | "runs" (extension, see
                    module docstring; "runs" needs an alive list of 64-column runs).

    Returns
    -------
    torch.Tensor [M, N], dtype of ``activations``, contiguous.
    """
    assert activations.ndim == 2 and weights.ndim == 2
    assert activations.is_cuda and weights.is_cuda
    M, K = activations.shape
    K_w, N = weights.shape
    assert K == K_w, f"K mismatch: A K={K}, W K={K_w}"

    if not activations.is_contiguous():
        activations = activations.contiguous()
    if not weights.is_contiguous():
        weights = weights.contiguous()
    if alive_indices.dtype != torch.int64 or alive_indices.device != activations.device:
        alive_indices = alive_indices.to(device=activations.device, dtype=torch.int64)
    if not alive_indices.is_contiguous():
        alive_indices = alive_indices.contiguous()
    if (bias is None and activation is None and strategy == "auto" and M and N
            and activations.get_device() == torch.cuda.current_device()):
        # The reference call without the extensions: the cached packed weight
        # comes with gw_gather_gemm's fixed arguments prepared.
        w_packed, prep = _packed_cache.get_prepared(weights, alive_indices, activations.dtype)
        C = activations.new_empty((M, N))
        if prep is not None:
            _native.gather_gemm_prepared(prep, activations, C)
        else:
            _gemm(activations, w_packed, alive_indices, C, None, None, "auto")
        return C
    C = torch.empty((M, N), dtype=activations.dtype, device=activations.device)
    if M == 0 or N == 0:
        return C
    w_packed = _packed_cache.get(weights, alive_indices, activations.dtype)
    if bias is not None and (bias.dtype != activations.dtype or not bias.is_contiguous()):
        bias = bias.contiguous().to(dtype=activations.dtype)
    _gemm(activations, w_packed, alive_indices, C, bias, activation, strategy)
    return C


class _PackedCache:
    """Packed weights of recent ghostweight_matmul calls.

    The reference API passes the weight [K, N] and the alive list on every
    call, and a loop over layers passes the same tensors again and again; the
    packing (a transposing gather of W[alive, :]) is then done once. An entry
    is used only for the very same tensor objects (held by weak reference, so
    an entry never outlives its weight) at the same in-place version counts
    (any in-place update of either tensor, or of a view sharing their storage,
    changes them), on the same storage (``w.data = ...`` keeps the object and
    its version) and for the same output dtype. Writes through ``w.data``
    change neither, so they need :func:`clear_packed_cache`. Small LRU: at
    most `max_entries` entries and `max_bytes` of packed data.
    """

    def __init__(self, max_entries: int = 32, max_bytes: int = 2 << 30):
        import collections
        import weakref

        self._weakref = weakref
        self._entries: "collections.OrderedDict" = collections.OrderedDict()
        self.max_entries = max_entries
        self.max_bytes = max_bytes
        self.bytes = 0

    def get(self, weights: torch.Tensor, idx: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        return self.get_prepared(weights, idx, dtype, prepare=False)[0]

    def get_prepared(self, weights: torch.Tensor, idx: torch.Tensor, dtype: torch.dtype,
                     prepare: bool = True) -> tuple:
        """(packed weight, the fixed gw_gather_gemm arguments for it without bias,
        activation or strategy choice, or None when the entry is not kept)."""
        key = (id(weights), id(idx), dtype)
        e = self._entries.get(key)
        if e is not None:
            w_ref, i_ref, w_ver, i_ver, packed, prep, ptrs = e
            if (w_ref() is weights and i_ref() is idx and w_ver == weights._version
                    and i_ver == idx._version and ptrs == (weights.data_ptr(), idx.data_ptr())
                    and not torch.cuda.is_current_stream_capturing()):
                self._entries.move_to_end(key)
                if prep is None and prepare:
                    prep = e[5] = _native.prepare_gather_gemm(packed, idx, None, None, "auto", dtype)
                return packed, prep
            self._drop(key)
        packed = pack_weight(weights.t(), idx, dtype=dtype)
        if torch.cuda.is_current_stream_capturing():
            return packed, None     # a graph's private pool: do not keep it
        nbytes = packed.untyped_storage().nbytes()
        if nbytes > self.max_bytes:
            return packed, None
        cb = lambda _ref, key=key: self._drop(key)
        prep = _native.prepare_gather_gemm(packed, idx, None, None, "auto", dtype) if prepare else None
        self._entries[key] = [self._weakref.ref(weights, cb), self._weakref.ref(idx, cb),
                              weights._version, idx._version, packed, prep,
                              (weights.data_ptr(), idx.data_ptr())]
        self.bytes += nbytes
        while len(self._entries) > self.max_entries or self.bytes > self.max_bytes:
            self._drop(next(iter(self._entries)))
        if key not in self._entries:
            return packed, None
        return packed, prep

    def _drop(self, key) -> None:
        e = self._entries.pop(key, None)
        if e is not None:
            self.bytes -= e[4].untyped_storage().nbytes()

    def clear(self) -> None:
        self._entries.clear()
        self.bytes = 0


_packed_cache = _PackedCache()


def clear_packed_cache() -> None:
    """Forget every packed weight ghostweight_matmul keeps.

    An entry is rebuilt by itself when the weight or the index list is
    replaced, rebound to other storage (``w.data = ...``) or updated in place
    through autograd-visible operations (optimizer steps, ``copy_`` under
    ``no_grad``), which bump the tensor's version counter. In-place writes
    through ``w.data`` bypass that counter; call this after them.
    """
    _packed_cache.clear()


def _gemm(x, w_packed, idx, y, bias, activation, strategy):
    ws = None
    if strategy == "runs" and (x.data_ptr() % 16 or x.stride(0) % 8):
        strategy = "auto"          # direct TMA of x needs 16-byte aligned rows
    if strategy != "fused" and strategy != "runs" and x.dtype is not torch.float32:
        nbytes = _native.gather_gemm_workspace_bytes(x.shape[0], idx.numel(), x.dtype)
        if nbytes:
            ws = _native.gemm_workspace(x.device, nbytes)
    _native.gather_gemm(x, w_packed, idx, y, bias=bias, activation=activation,
                        strategy=strategy, workspace=ws)


def index_runs(alive_indices: torch.Tensor, K: int) -> int:
    """Entries of the alive list that keep it from being 64-column runs (0: strategy
    "runs" applies). One device pass and one host synchronisation."""
    return _native.index_runs(alive_indices, K)


def ghost_linear(
    x: torch.Tensor,
    w_packed: torch.Tensor,
    alive_indices: torch.Tensor,
    bias: torch.Tensor | None = None,
    activation: str | None = None,
    out: torch.Tensor | None = None,
    strategy: str = "auto",
) -> torch.Tensor:
    """y = act(x[:, alive] @ w_packed^T + bias) for x [M, K], w_packed [N, K_alive]."""
    assert x.ndim == 2 and x.is_cuda
    if not x.is_contiguous():
        x = x.contiguous()
    M = x.shape[0]
    N = w_packed.shape[0]
    y = out if out is not None else torch.empty((M, N), dtype=x.dtype, device=x.device)
    if M and N:
        _gemm(x, w_packed, alive_indices, y, bias, activation, strategy)
    return y


def ghost_linear_dev(
    x: torch.Tensor,
    w_packed: torch.Tensor,
    alive_buffer: torch.Tensor,
    alive_count: torch.Tensor,
    bias: torch.Tensor | None = None,
    activation: str | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """ghost_linear with K' = alive_count[0] read on the device (no host synchronisation).

    w_packed is the [N, round_up(K, 64)] buffer of :func:`pack_weight_dev` for the
    same alive list; alive_buffer's first K' entries are the alive columns.
    """
    assert x.ndim == 2 and x.is_cuda
    x = x.contiguous()
    M = x.shape[0]
    N = w_packed.shape[0]
    y = out if out is not None else torch.empty((M, N), dtype=x.dtype, device=x.device)
    if M and N:
        _native.gather_gemm_dev(x, w_packed, alive_buffer, alive_count, y, bias=bias,
                                activation=activation)
    return y


def packed_linear(
    a: torch.Tensor,
    w_packed: torch.Tensor,
    bias: torch.Tensor | None = None,
    activation: str | None = None,
) -> torch.Tensor:
    """y = act(a @ w_packed^T + bias) for an already compacted a [M, K_alive] (TMA operands)."""
    assert a.ndim == 2 and a.is_cuda
    a = a.contiguous()
    y = torch.empty((a.shape[0], w_packed.shape[0]), dtype=a.dtype, device=a.device)
    if y.numel():
        _native.packed_gemm(a, w_packed, y, bias=bias, activation=activation)
    return y


class _PipeState:
    """Per-device streams, events and x' buffers of ghost_linear_pipelined."""

    def __init__(self, device: torch.device):
        lo, hi = torch.cuda.Stream.priority_range()      # (least, greatest) priority
        self.gemm = torch.cuda.Stream(device, priority=hi)
        self.gather = torch.cuda.Stream(device, priority=lo)
        self.ready = [torch.cuda.Event(), torch.cuda.Event()]
        self.free = [torch.cuda.Event(), torch.cuda.Event()]
        self.bufs: dict = {}

    def xbuf(self, slot: int, dtype: torch.dtype, M: int, ldp: int, device) -> torch.Tensor:
        key = (slot, dtype)
        b = self.bufs.get(key)
        if b is None or b.numel() < M * ldp:
            if b is not None:
                # The gather and GEMM streams may still use the old buffer:
                # the allocator reuses it only after their queued work.
                b.record_stream(self.gather)
                b.record_stream(self.gemm)
            b = self.bufs[key] = torch.empty(M * ldp, dtype=dtype, device=device)
        return b[: M * ldp].view(M, ldp)


_pipe_states: dict = {}


def ghost_linear_pipelined(calls) -> list:
    """Independent gather-GEMM calls with each gather overlapping the previous GEMM.

    ``calls`` is a sequence of ``(x, w_packed, alive_indices, out[, bias[,
    activation]])``, each meaning ``ghost_linear(x, w_packed, alive_indices,
    bias, activation, out=out)``, and the outputs are returned in order. The
    calls must not depend on one another (one call's output is not a later
    call's input): call i+1's gather of x[:, alive] then runs on a
    low-priority stream while call i's GEMM runs on a high-priority one. The
    GEMM keeps the SMs it needs, and the gather fills the registers and issue
    slots it leaves (the GEMM reads only a few percent of HBM bandwidth). x'
    alternates between two buffers, ordered by events. The caller's current
    stream waits for all of it before this returns, and the whole call can be
    captured in a CUDA graph. Calls with at most 4 rows (the decode kernel
    gathers x' itself, one launch), fp32 operands or index lists that are not
    int64 run as ``ghost_linear`` in order on the GEMM stream.
    """
    cur = torch.cuda.current_stream()
    device = cur.device
    st = _pipe_states.get(device.index)
    if st is None:
        st = _pipe_states[device.index] = _PipeState(device)
    norm = []
    for c in calls:
        x, wp, idx, out = c[0], c[1], c[2], c[3]
        bias = c[4] if len(c) > 4 else None
        act = c[5] if len(c) > 5 else None
        assert x.ndim == 2 and x.is_cuda and out is not None
        norm.append((x, wp, idx, out, bias, act))
    st.gemm.wait_stream(cur)
    st.gather.wait_stream(cur)
    # Both slots start free, ordered after the caller's work. Recording them
    # here (not reusing an earlier call's events) also keeps every wait inside
    # a CUDA graph capture that this call may be part of.
    for e in st.free:
        e.record(st.gemm)

    def piped(c):
        x, wp, idx, out, bias, act = c
        return (x.shape[0] > 4 and x.dtype is not torch.float32 and x.is_contiguous()
                and idx.dtype is torch.int64 and idx.numel() > 0)

    def gather(i):
        x, wp, idx, _, _, _ = norm[i]
        b = i % 2
        kp = idx.numel()
        ldp = (kp + 63) // 64 * 64
        xg = st.xbuf(b, x.dtype, x.shape[0], ldp, device)[:, :kp]
        st.gather.wait_event(st.free[b])
        with torch.cuda.stream(st.gather):
            _native.gather_columns(x, idx, xg)
            st.ready[b].record(st.gather)
        return xg

    xgs = {}
    if norm and piped(norm[0]):
        xgs[0] = gather(0)
    for i, c in enumerate(norm):
        if i + 1 < len(norm) and piped(norm[i + 1]):
            xgs[i + 1] = gather(i + 1)
        x, wp, idx, out, bias, act = c
        with torch.cuda.stream(st.gemm):
            if i in xgs:
                b = i % 2
                st.gemm.wait_event(st.ready[b])
                if out.numel():
                    _native.packed_gemm(xgs.pop(i), wp, out, bias=bias, activation=act)
                st.free[b].record(st.gemm)
            else:
                ghost_linear(x, wp, idx, bias=bias, activation=act, out=out)
    cur.wait_stream(st.gemm)
    cur.wait_stream(st.gather)
    return [c[3] for c in norm]
