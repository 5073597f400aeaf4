"""Drop-in import name for code written against ghostweight-triton.

``import ghostweight_triton`` (and every submodule the original package has:
kernels, kernels.mask, kernels.gather, kernels.matmul, module, replace, utils,
utils.sparsity, utils.compat) resolves to the B200 implementation in
``ghostweight_triton_b200``; the module objects are shared, so classes such as
GhostLinear are the same objects under both names.
"""

import importlib as _importlib
import sys as _sys

import ghostweight_triton_b200 as _impl
from ghostweight_triton_b200 import *  # noqa: F401,F403
from ghostweight_triton_b200 import __all__, __version__  # noqa: F401

_SUBMODULES = (
    "kernels",
    "kernels.mask",
    "kernels.gather",
    "kernels.matmul",
    "module",
    "replace",
    "utils",
    "utils.sparsity",
    "utils.compat",
)

for _name in _SUBMODULES:
    _mod = _importlib.import_module(f"{_impl.__name__}.{_name}")
    _sys.modules[f"{__name__}.{_name}"] = _mod
    _parent, _, _leaf = _name.rpartition(".")
    setattr(_sys.modules[f"{__name__}.{_parent}"] if _parent else _sys.modules[__name__], _leaf, _mod)
