"""
GhostWeight B200
================
Training-free inference sparsity via dead-neuron masking, on hand-written
sm_100a (B200) CUDA kernels behind a C ABI (include/ghostweight_b200.h).

Same public surface as ghostweight_triton (ghostweight_triton/__init__.py:10-28);
the ``ghostweight_triton`` package in this repository re-exports this one so
existing imports keep working.
"""

from ghostweight_triton_b200.kernels import (
    dead_neuron_mask,
    ghostweight_matmul,
    gather_compact,
)
from ghostweight_triton_b200.module import GhostLinear
from ghostweight_triton_b200.replace import replace_linears, get_sparsity_report

__version__ = "0.1.0"

__all__ = [
    "dead_neuron_mask",
    "ghostweight_matmul",
    "gather_compact",
    "GhostLinear",
    "replace_linears",
    "get_sparsity_report",
]
