from ghostweight_triton_b200.utils.sparsity import sparsity_stats, log_sparsity
from ghostweight_triton_b200.utils.compat import check_environment

__all__ = ["sparsity_stats", "log_sparsity", "check_environment"]
