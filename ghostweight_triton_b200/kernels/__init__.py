"""B200 kernel wrappers (same import surface as ghostweight_triton.kernels)."""

from ghostweight_triton_b200.kernels.mask import dead_neuron_mask
from ghostweight_triton_b200.kernels.gather import gather_compact
from ghostweight_triton_b200.kernels.matmul import ghostweight_matmul

__all__ = [
    "dead_neuron_mask",
    "gather_compact",
    "ghostweight_matmul",
]
