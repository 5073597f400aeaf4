"""GPU: fused GhostLinear MLP chains (fc -> GELU -> proj, proj's dead inputs never computed).

The fused chain must equal the unfused model's output (the skipped terms are
products with zero weights) within the fp16 tolerance of the reference's
tests (tests/test_matmul.py:68-72).
"""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

from ghostweight_triton_b200 import replace_linears
from ghostweight_triton_b200.fuse import GhostMLPChain, fuse_mlp_chains

pytestmark = pytest.mark.gpu


def _zero_dead(model, sparsity, seed):
    import torch.nn as nn
    from transformers.pytorch_utils import Conv1D

    rng = np.random.default_rng(seed)
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, nn.Linear) and mod.in_features >= 128:
                k = mod.in_features
                mod.weight[:, torch.from_numpy(rng.permutation(k)[: int(k * sparsity)])] = 0
            elif isinstance(mod, Conv1D):
                k = mod.weight.shape[0]
                mod.weight[torch.from_numpy(rng.permutation(k)[: int(k * sparsity)]), :] = 0


@pytest.mark.parametrize("which", ["gpt2", "distilbert"])
def test_fused_chains_match_unfused_model(which):
    torch.manual_seed(0)
    if which == "gpt2":
        from transformers import GPT2Config, GPT2Model
        model = GPT2Model(GPT2Config(n_layer=2))
        n_expected = 2
    else:
        from transformers import DistilBertConfig, DistilBertModel
        model = DistilBertModel(DistilBertConfig(n_layers=2))
        n_expected = 2
    _zero_dead(model, 0.6, 1)
    model = model.half().cuda().eval()
    ghost = copy.deepcopy(model)
    replace_linears(ghost, threshold=0.0, include_conv1d=True, freeze_from_weight=True)
    fused = copy.deepcopy(ghost)
    names = fuse_mlp_chains(fused)
    assert len(names) == n_expected
    assert sum(isinstance(m, GhostMLPChain) for m in fused.modules()) == n_expected
    ids = torch.randint(0, 1000, (4, 96), device="cuda")
    with torch.no_grad():
        a = ghost(input_ids=ids).last_hidden_state.float()
        b = fused(input_ids=ids).last_hidden_state.float()
        d = model(input_ids=ids).last_hidden_state.float()
    assert float((b - a).norm() / a.norm()) < 5e-3
    assert float((b - d).norm() / d.norm()) < 5e-3


def test_fused_chain_odd_feature_count_and_weight_update():
    """proj with an alive count that is not a multiple of 8 (padded features), bias on
    both layers, and a weight change after the first call (operands rebuilt)."""
    import torch.nn as nn
    import torch.nn.functional as F

    torch.manual_seed(2)

    class MLP(nn.Module):
        def __init__(self):
            super().__init__()
            self.lin1 = nn.Linear(256, 300)
            self.lin2 = nn.Linear(300, 200)
            self.activation = nn.GELU()
            self.dropout = nn.Dropout(0.0)

        def forward(self, x):
            return self.dropout(self.lin2(self.activation(self.lin1(x))))

    holder = nn.Sequential(MLP()).half().cuda().eval()
    with torch.no_grad():
        holder[0].lin1.weight[:, 7::3] = 0
        holder[0].lin2.weight[:, 5::4] = 0
    replace_linears(holder, threshold=0.0, freeze_from_weight=True, min_features=1)
    assert fuse_mlp_chains(holder) == ["0"]
    x = torch.randn(37, 256, device="cuda", dtype=torch.float16)
    chain = holder[0]

    def reference():
        h = F.gelu(F.linear(x.float(), chain.fc.weight.float(), chain.fc.bias.float()))
        return F.linear(h, chain.proj.weight.float(), chain.proj.bias.float())

    with torch.no_grad():
        torch.testing.assert_close(holder(x).float(), reference(), atol=2e-2, rtol=2e-2)
        chain.proj.weight.mul_(0.5)
        torch.testing.assert_close(holder(x).float(), reference(), atol=2e-2, rtol=2e-2)
