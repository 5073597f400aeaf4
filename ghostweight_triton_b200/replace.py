"""Model rewriting pass: swap linear layers for GhostLinear in place.

Mirrors ghostweight_triton/replace.py:9-67 (same signature, skip-pattern and
min_features rules, return value {qualified name: in_features}). One addition:
transformers' Conv1D layers (GPT-2's attention and MLP projections, weight
stored [in, out]) are rewritten too -- the reference only matches nn.Linear
(replace.py:35), which leaves GPT-2 dense.
"""

from __future__ import annotations

import torch.nn as nn

from ghostweight_triton_b200.module import GhostLinear


def _conv1d_type():
    try:
        from transformers.pytorch_utils import Conv1D
    except Exception:  # transformers not installed
        return None
    return Conv1D


def _in_features(child: nn.Module, conv1d) -> int | None:
    if isinstance(child, GhostLinear):
        return None
    if isinstance(child, nn.Linear):
        return child.in_features
    if conv1d is not None and isinstance(child, conv1d):
        return int(child.weight.shape[0])
    return None


def replace_linears(
    model: nn.Module,
    threshold: float = 1e-6,
    skip_patterns: list[str] | None = None,
    min_features: int = 128,
    *,
    include_conv1d: bool = True,
    freeze_from_weight: bool = False,
) -> dict[str, int]:
    """Recursively replace nn.Linear (and transformers Conv1D) modules with GhostLinear.

    Args:
        model:              the model to patch (modified in place)
        threshold:          dead-neuron threshold given to every GhostLinear
        skip_patterns:      substrings; a layer whose qualified name contains any is skipped
        min_features:       layers with fewer input features are skipped
        include_conv1d:     also rewrite transformers Conv1D layers (extension)
        freeze_from_weight: freeze each new layer's mask from its weight's dead
                            input columns right away (extension)

    Returns:
        dict mapping replaced module names to their in_features
    """
    skip_patterns = skip_patterns or []
    conv1d = _conv1d_type() if include_conv1d else None
    replaced: dict[str, int] = {}

    for name, module in model.named_modules():
        # Direct children only; deeper levels are visited by named_modules().
        todo: dict[str, nn.Module] = {}
        for child_name, child in module.named_children():
            in_f = _in_features(child, conv1d)
            if in_f is None:
                continue
            full_name = f"{name}.{child_name}" if name else child_name
            if any(pat in full_name for pat in skip_patterns):
                continue
            if in_f < min_features:
                continue
            todo[child_name] = child
            replaced[full_name] = in_f

        for child_name, child in todo.items():
            if isinstance(child, nn.Linear):
                ghost = GhostLinear.from_linear(child, threshold=threshold)
            else:
                ghost = GhostLinear.from_conv1d(child, threshold=threshold)
            if freeze_from_weight:
                ghost.freeze_weight_mask()
            setattr(module, child_name, ghost)

    return replaced


def get_sparsity_report(model: nn.Module) -> dict[str, float]:
    """Current sparsity of every GhostLinear layer, keyed by qualified name."""
    return {
        name: module.current_sparsity
        for name, module in model.named_modules()
        if isinstance(module, GhostLinear)
    }
