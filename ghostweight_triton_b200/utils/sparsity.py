"""Host-side sparsity summaries (not on the hot path).

Keeps the reference's two names and the keys of ``sparsity_stats``'s result
(ghostweight_triton/utils/sparsity.py:8-89) so user code that reads them keeps
working. The counting runs on the mask's device with one host read, and
``log_sparsity`` renders through one small table formatter for both kinds of
input.
"""

from __future__ import annotations

import torch

_BAR = 32


def sparsity_stats(mask: torch.Tensor) -> dict:
    """Counts for a 1-D alive mask (non-zero = alive), e.g. ``dead_neuron_mask``'s output.

    Returns ``{"total", "alive", "dead", "pct_dead", "pct_alive"}``; the
    fractions are 0.0 for an empty mask.
    """
    if mask.ndim != 1:
        raise AssertionError(f"sparsity_stats takes a 1-D mask; got {mask.ndim} dims {tuple(mask.shape)}")
    total = int(mask.numel())
    alive = int(torch.count_nonzero(mask).item()) if total else 0
    frac = (lambda n: n / total) if total else (lambda n: 0.0)
    return {"total": total, "alive": alive, "dead": total - alive,
            "pct_dead": frac(total - alive), "pct_alive": frac(alive)}


def _table(title: str, header: tuple[str, str, str], rows: list[tuple[str, str, str]],
           footer: tuple[str, str, str] | None) -> str:
    w0 = max([len(header[0])] + [len(r[0]) for r in rows] + ([len(footer[0])] if footer else []))
    w1 = max([len(header[1])] + [len(r[1]) for r in rows] + ([len(footer[1])] if footer else []))
    fmt = lambda r: f"  {r[0]:<{w0}}  {r[1]:>{w1}}  {r[2]}".rstrip()
    width = w0 + w1 + _BAR + 6
    out = [f"{title} ".ljust(width, "="), fmt(header), "-" * width]
    out += [fmt(r) for r in rows]
    if footer:
        out += ["-" * width, fmt(footer)]
    return "\n".join(out)


def _bar(frac: float) -> str:
    n = max(0, min(_BAR, round(frac * _BAR)))
    return "|" + "#" * n + " " * (_BAR - n) + "|"


def log_sparsity(report: dict[str, float] | torch.Tensor,
                 title: str = "GhostWeight Sparsity Report") -> None:
    """Print a mask summary (tensor) or a {layer name: dead fraction} table (dict,
    e.g. ``get_sparsity_report``'s result)."""
    if isinstance(report, torch.Tensor):
        s = sparsity_stats(report)
        rows = [("alive", f"{s['alive']}/{s['total']}", f"{s['pct_alive']:.1%}"),
                ("dead", f"{s['dead']}/{s['total']}", f"{s['pct_dead']:.1%} {_bar(s['pct_dead'])}")]
        print(_table(title, ("neurons", "count", "share"), rows, None))
        return
    if not report:
        print(f"{title}: no GhostLinear layers in the report")
        return
    fracs = {name: float(v) for name, v in report.items()}
    rows = [(name, f"{f:.1%}", _bar(f)) for name, f in fracs.items()]
    mean = sum(fracs.values()) / len(fracs)
    print(_table(title, ("layer", "dead", ""), rows, (f"mean of {len(fracs)} layers", f"{mean:.1%}",
                                                       _bar(mean))))
