"""Dead-neuron (dead-column) mask on B200.

Mirrors ghostweight_triton/kernels/mask.py:62-104. A column k of an [M, K]
matrix is alive iff max_m fp32(|A[m, k]|) > fp32(threshold), with the running
max starting at 0 and NaN entries ignored (mask.py:46-58). The work is done by
the sm_100a kernel K1 (csrc/gw_mask.cu), which also emits the sorted alive
index list in the same launch; ``dead_neuron_mask_compact`` exposes that.
"""

from __future__ import annotations

import torch

from ghostweight_triton_b200 import _native


def dead_neuron_mask(
    activations: torch.Tensor,
    threshold: float = 1e-6,
    BLOCK_M: int = 512,
) -> torch.Tensor:
    """Detect dead neurons in an activation matrix.

    Parameters
    ----------
    activations : torch.Tensor
        Shape [M, K]; float16, bfloat16 or float32; on a CUDA (sm_100) device.
    threshold : float
        Neurons whose max |activation| is <= threshold are dead.
    BLOCK_M : int
        Accepted for signature compatibility with the Triton version; the
        B200 kernel picks its own tiling.

    Returns
    -------
    torch.Tensor
        Shape [K], dtype int32: 1 = alive, 0 = dead.
    """
    assert activations.ndim == 2, (
        f"dead_neuron_mask expects [M, K], got shape {activations.shape}"
    )
    assert activations.is_cuda, "activations must be on CUDA"
    activations = activations.contiguous()
    _, K = activations.shape
    mask = torch.empty(K, dtype=torch.int32, device=activations.device)
    _native.mask_compact(activations, threshold, mask=mask)
    return mask


def dead_neuron_mask_compact(
    activations: torch.Tensor,
    threshold: float = 1e-6,
    want_mask: bool = True,
) -> tuple[torch.Tensor | None, torch.Tensor, torch.Tensor]:
    """Mask plus alive-index compaction in one launch.

    Returns ``(mask, alive_buffer, alive_count)``: mask int32 [K] (or None),
    alive_buffer int64 [K] whose first ``alive_count`` entries are the alive
    column indices in ascending order (what ``torch.nonzero(mask)`` gives at
    ghostweight_triton/module.py:104), alive_count an int32 [1] device tensor.
    Nothing is synchronised.
    """
    assert activations.ndim == 2, (
        f"dead_neuron_mask expects [M, K], got shape {activations.shape}"
    )
    assert activations.is_cuda, "activations must be on CUDA"
    activations = activations.contiguous()
    _, K = activations.shape
    dev = activations.device
    mask = torch.empty(K, dtype=torch.int32, device=dev) if want_mask else None
    alive = torch.empty(K, dtype=torch.int64, device=dev)
    count = torch.empty(1, dtype=torch.int32, device=dev)
    _native.mask_compact(activations, threshold, mask=mask, alive_idx=alive, count=count)
    return mask, alive, count


def alive_indices(activations: torch.Tensor, threshold: float = 1e-6) -> torch.Tensor:
    """Sorted int64 alive column indices of an [R, K] matrix (reads the count: synchronises)."""
    _, alive, count = dead_neuron_mask_compact(activations, threshold, want_mask=False)
    return alive[: int(count.item())]
