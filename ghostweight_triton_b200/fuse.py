"""Fused GhostLinear MLP chains: fc -> GELU -> proj without the dead features.

In a transformer MLP the first projection's output goes through an
elementwise activation into the second projection only (GPT-2's
``GPT2MLP``: c_fc -> gelu_new -> c_proj; DistilBERT's ``FFN``: lin1 -> gelu
-> lin2). When both are GhostLinears with frozen masks, the second layer's dead
input features are outputs of the first layer that nothing reads: their
columns of the second weight are zero. The fused chain therefore

* computes only the second layer's alive features in the first GEMM (the rows
  of the first weight restricted to them, packed over the first layer's own
  alive inputs), with the bias and the GELU in its epilogue, so that its output
  already is the second layer's compacted input x'; and
* feeds that straight into the second GEMM (both operands by TMA, no gather).

One gather launch and the dead part of the first GEMM disappear; the result
equals the unfused chain's (the skipped terms are products with zero weights),
up to the one rounding of the intermediate that the fused GELU saves. This is
an extension: the reference replaces the two projections independently
(ghostweight_triton/replace.py:35-56) and keeps the full intermediate.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from ghostweight_triton_b200.kernels.gather import pack_weight
from ghostweight_triton_b200.kernels.matmul import ghost_linear, packed_linear
from ghostweight_triton_b200.module import GhostLinear

# Activation modules (by class name) that the GEMM epilogue reproduces.
_ACT_BY_CLASS = {
    "NewGELUActivation": "gelu_tanh",     # transformers' gelu_new: tanh approximation
    "GELUTanh": "gelu_tanh",
    "GELUActivation": "gelu",             # exact erf GELU
}


def _epilogue_of(act: nn.Module) -> str | None:
    if isinstance(act, nn.GELU):
        return "gelu_tanh" if act.approximate == "tanh" else "gelu"
    return _ACT_BY_CLASS.get(type(act).__name__)


class GhostMLPChain(nn.Module):
    """fc -> activation -> proj (-> dropout) with proj's dead inputs never computed.

    ``fc`` and ``proj`` are GhostLinears with frozen masks (``proj.in_features ==
    fc.out_features``); they stay registered as submodules, so parameters and
    state-dict keys are unchanged. The packed operands are built on first use and
    rebuilt when a weight or a mask changes.
    """

    def __init__(self, fc: GhostLinear, proj: GhostLinear, activation: str,
                 dropout: nn.Module | None = None):
        super().__init__()
        assert proj.in_features == fc.out_features
        self.fc = fc
        self.proj = proj
        self.activation = activation
        self.dropout = dropout
        self._plan: tuple | None = None

    def refresh_packed(self) -> None:
        """Rebuild the fused operands at the next forward: needed after in-place
        writes through ``weight.data`` or ``bias.data``, which bypass the
        version counters the plan is keyed on."""
        self._plan = None

    def _operands(self, dtype: torch.dtype):
        fc, proj = self.fc, self.proj
        a_fc, a_proj = fc._frozen_indices, proj._frozen_indices
        key = (dtype, fc.weight.data_ptr(), fc.weight._version, proj.weight.data_ptr(),
               proj.weight._version, a_fc.data_ptr(), a_fc._version, a_proj.data_ptr(),
               a_proj._version, None if fc.bias is None else (fc.bias.data_ptr(), fc.bias._version))
        if self._plan is not None and self._plan[0] == key:
            return self._plan[1:]
        with torch.no_grad():
            # proj's weight packed over its alive inputs, whole buffer: the fused
            # features padded with zero columns to a multiple of 64 (TMA rows).
            wp = pack_weight(proj.weight.detach(), a_proj, dtype=dtype)
            n_pad = wp.stride(0)
            w_proj = wp.as_strided((wp.shape[0], n_pad), (n_pad, 1))
            # Rows of fc's weight for the features proj reads (zero rows for the
            # padding: their outputs are act(0) = 0), over fc's alive inputs.
            rows = fc.weight.detach().index_select(0, a_proj)
            pad = n_pad - rows.shape[0]
            if pad:
                rows = torch.cat([rows, rows.new_zeros(pad, rows.shape[1])])
            w_fc = pack_weight(rows, a_fc, dtype=dtype)
            b_fc = None
            if fc.bias is not None:
                b_fc = fc.bias.detach().index_select(0, a_proj).to(dtype)
                if pad:
                    b_fc = torch.cat([b_fc, b_fc.new_zeros(pad)])
        self._plan = (key, w_fc, b_fc, w_proj)
        return w_fc, b_fc, w_proj

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.fc.in_features)
        w_fc, b_fc, w_proj = self._operands(x2.dtype)
        h = ghost_linear(x2, w_fc, self.fc._frozen_indices, bias=b_fc, activation=self.activation)
        bias = self.proj.bias
        if bias is not None and bias.dtype != x2.dtype:
            bias = bias.to(x2.dtype)
        y = packed_linear(h, w_proj, bias=bias)
        if self.dropout is not None:
            y = self.dropout(y)
        return y.reshape(*lead, self.proj.out_features)


def _frozen(m: nn.Module) -> bool:
    return isinstance(m, GhostLinear) and m.mask_frozen and m._frozen_indices is not None


def fuse_mlp_chains(model: nn.Module) -> list[str]:
    """Replace every MLP block whose two projections are frozen GhostLinears joined by
    a GELU with a :class:`GhostMLPChain`; returns the names of the replaced blocks.

    Recognised blocks: modules with ``c_fc``, ``c_proj`` and ``act`` (transformers'
    GPT2MLP) or ``lin1``, ``lin2`` and ``activation`` (DistilBERT's FFN), each with
    an optional ``dropout``. Run it after ``replace_linears(...,
    freeze_from_weight=True)`` (or after freezing the masks).
    """
    replaced = []
    for name, parent in list(model.named_modules()):
        for child_name, child in list(parent.named_children()):
            fc = proj = act = None
            if hasattr(child, "c_fc") and hasattr(child, "c_proj") and hasattr(child, "act"):
                fc, proj, act = child.c_fc, child.c_proj, child.act
            elif hasattr(child, "lin1") and hasattr(child, "lin2") and hasattr(child, "activation"):
                fc, proj, act = child.lin1, child.lin2, child.activation
                if getattr(child, "chunk_size_feed_forward", 0):
                    continue
            if fc is None or not (_frozen(fc) and _frozen(proj)) or fc.activation is not None:
                continue
            epi = _epilogue_of(act) if isinstance(act, nn.Module) else None
            if epi is None or proj.in_features != fc.out_features or proj._frozen_indices.numel() == 0:
                continue
            dropout = getattr(child, "dropout", None)
            setattr(parent, child_name, GhostMLPChain(fc, proj, epi, dropout))
            replaced.append(f"{name}.{child_name}" if name else child_name)
    return replaced
