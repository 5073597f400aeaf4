"""Host-side sparsity statistics and printing.

Same behaviour as ghostweight_triton/utils/sparsity.py:8-89: ``sparsity_stats``
summarises an int32 alive mask, ``log_sparsity`` pretty-prints either a mask
or a {layer: sparsity} report.
"""

from __future__ import annotations

import torch


def sparsity_stats(mask: torch.Tensor) -> dict:
    """Counts for a [K] dead-neuron mask (1 = alive, 0 = dead).

    Returns a dict with keys total, alive, dead, pct_dead, pct_alive.
    """
    assert mask.ndim == 1, f"Expected 1D mask, got shape {mask.shape}"
    total = mask.numel()
    alive = int(mask.sum().item())
    dead = total - alive
    return {
        "total": total,
        "alive": alive,
        "dead": dead,
        "pct_dead": dead / total if total > 0 else 0.0,
        "pct_alive": alive / total if total > 0 else 0.0,
    }


def log_sparsity(
    report: dict[str, float] | torch.Tensor,
    title: str = "GhostWeight Sparsity Report",
) -> None:
    """Print a mask summary (tensor input) or a per-layer sparsity table (dict input)."""
    if isinstance(report, torch.Tensor):
        s = sparsity_stats(report)
        rule = "-" * 60
        print(f"\n{rule}\n  {title}\n{rule}")
        print(f"  Total neurons : {s['total']}")
        print(f"  Alive         : {s['alive']} ({s['pct_alive']:.1%})")
        print(f"  Dead          : {s['dead']} ({s['pct_dead']:.1%})")
        print(f"{rule}\n")
        return

    if not report:
        print(f"[{title}] No GhostLinear layers found.")
        return

    width = max(20, max(len(n) for n in report))
    bar_w = 40
    rule = "-" * (width + bar_w + 20)
    print(f"\n{rule}\n  {title}\n{rule}")
    print(f"  {'Layer':<{width}}  {'Sparsity':>8}  Dead neurons")
    total = 0.0
    for name, sp in report.items():
        sp = float(sp)
        filled = int(sp * bar_w)
        print(f"  {name:<{width}}  {sp:>7.1%}  {'#' * filled}{'.' * (bar_w - filled)}")
        total += sp
    print(rule)
    print(f"  {'Average':<{width}}  {total / len(report):>7.1%}")
    print(f"{rule}\n")
