"""Gathers and the one-time weight compaction on B200.

``gather_compact`` mirrors ghostweight_triton/kernels/gather.py:97-158 (the
two-step path: compacted activations and weights, both contiguous, dtype
preserved). ``pack_weight`` is the weight compaction of the sparse path: it
packs the alive input columns of an nn.Linear weight [N, K] into the dense
[N, K'_pad] K'-major operand that the tcgen05 gather-GEMM streams by TMA.
"""

from __future__ import annotations

import torch

from ghostweight_triton_b200 import _native

# Packed weights keep their row stride a multiple of 64 elements (128 bytes of
# fp16/bf16): every TMA row starts 128-byte aligned. Padding columns are zero.
PACK_ALIGN = 64


def _round_up(v: int, m: int) -> int:
    return (v + m - 1) // m * m


def gather_compact(
    activations: torch.Tensor,
    weights: torch.Tensor,
    alive_indices: torch.Tensor,
    BLOCK_M: int = 64,
    BLOCK_K: int = 64,
    BLOCK_N: int = 64,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Compact activations and weights to alive neurons only.

    Parameters
    ----------
    activations   : [M, K]
    weights       : [K, N]
    alive_indices : [K_alive], any integer dtype (converted to int64)
    BLOCK_* : accepted for signature compatibility; ignored.

    Returns
    -------
    A_compact : [M, K_alive] = activations[:, alive_indices]
    W_compact : [K_alive, N] = weights[alive_indices, :]
    """
    assert activations.ndim == 2 and weights.ndim == 2
    assert activations.is_cuda and weights.is_cuda
    M, K = activations.shape
    K_w, N = weights.shape
    assert K == K_w, f"K mismatch: A K={K}, W K={K_w}"

    activations = activations.contiguous()
    weights = weights.contiguous()
    alive_indices = alive_indices.contiguous().to(device=activations.device, dtype=torch.int64)
    K_alive = alive_indices.shape[0]

    A_compact = torch.empty((M, K_alive), dtype=activations.dtype, device=activations.device)
    W_compact = torch.empty((K_alive, N), dtype=weights.dtype, device=weights.device)
    if M > 0 and K_alive > 0:
        _native.gather_columns(activations, alive_indices, A_compact)
    if K_alive > 0 and N > 0:
        _native.gather_rows(weights, alive_indices.to(weights.device), W_compact)
    return A_compact, W_compact


def pack_weight(weight: torch.Tensor, alive_indices: torch.Tensor,
                dtype: torch.dtype | None = None) -> torch.Tensor:
    """Pack the alive input columns of a linear weight for the gather-GEMM.

    ``weight`` is [N, K] (nn.Linear orientation, any strides: a transposed view
    of a [K, N] buffer such as a transformers Conv1D weight is packed by the
    transposing gather without a copy). Returns W' [N, K_alive], a view of a
    [N, round_up(K_alive, 64)] zero-padded, row-major buffer.
    """
    assert weight.ndim == 2 and weight.is_cuda
    if dtype is not None and weight.dtype != dtype:
        weight = weight.to(dtype)
    idx = alive_indices.contiguous().to(device=weight.device, dtype=torch.int64)
    N, K = weight.shape
    k_alive = idx.numel()
    ld = max(_round_up(k_alive, PACK_ALIGN), PACK_ALIGN)
    buf = torch.empty((N, ld), dtype=weight.dtype, device=weight.device)
    if N > 0:
        if weight.stride(1) == 1:
            _native.gather_columns(weight, idx, buf, pad_to=ld)
        elif weight.stride(0) == 1:
            _native.gather_rows_t(weight.t(), idx, buf, pad_to=ld)
        else:
            _native.gather_columns(weight.contiguous(), idx, buf, pad_to=ld)
    return buf[:, :k_alive]


def pack_weight_dev(weight: torch.Tensor, alive_buffer: torch.Tensor, alive_count: torch.Tensor,
                    dtype: torch.dtype | None = None) -> torch.Tensor:
    """:func:`pack_weight` for an alive list whose length lives on the device.

    ``alive_buffer`` holds the alive columns in its first ``alive_count[0]``
    entries (int32 device scalar, as the mask kernel writes it); nothing is
    synchronised. Returns the whole [N, round_up(K, 64)] buffer: columns
    [K', round_up(max(K', 1), 64)) are zero, the ones past that are not
    written (the device-count GEMM never reads them).
    """
    assert weight.ndim == 2 and weight.is_cuda
    if dtype is not None and weight.dtype != dtype:
        weight = weight.to(dtype)
    idx = alive_buffer.contiguous().to(device=weight.device, dtype=torch.int64)
    N, K = weight.shape
    ld = max(_round_up(idx.numel(), PACK_ALIGN), PACK_ALIGN)
    buf = torch.empty((N, ld), dtype=weight.dtype, device=weight.device)
    if N > 0:
        if weight.stride(1) == 1:
            _native.gather_columns_dev(weight, idx, alive_count, buf, pad_to=ld)
        elif weight.stride(0) == 1:
            _native.gather_rows_t_dev(weight.t(), idx, alive_count, buf, pad_to=ld)
        else:
            _native.gather_columns_dev(weight.contiguous(), idx, alive_count, buf, pad_to=ld)
    return buf


def pack_weight_kn(weights_kn: torch.Tensor, alive_indices: torch.Tensor,
                   dtype: torch.dtype | None = None) -> torch.Tensor:
    """Same as :func:`pack_weight` for a reference-orientation weight [K, N]."""
    return pack_weight(weights_kn.t(), alive_indices, dtype=dtype)
