"""CPU: the Python surface is a drop-in for ghostweight_triton and has no CPU fallback.

Signatures and defaults follow the reference (ghostweight_triton/__init__.py:21-28,
kernels/mask.py:62-66, gather.py:97-104, matmul.py:85-92, module.py:34-43,
replace.py:9-14). Model rewriting and state handling need no GPU and are
tested here on CPU modules; forwards are GPU tests.
"""

from __future__ import annotations

import inspect

import pytest
import torch
import torch.nn as nn

import ghostweight_triton
import ghostweight_triton_b200 as gwb
from ghostweight_triton_b200 import GhostLinear, replace_linears, get_sparsity_report


def test_all_names():
    assert gwb.__all__ == ["dead_neuron_mask", "ghostweight_matmul", "gather_compact",
                           "GhostLinear", "replace_linears", "get_sparsity_report"]
    assert gwb.__version__ == "0.1.0"


def test_alias_package_shares_modules():
    from ghostweight_triton.kernels import dead_neuron_mask, gather_compact, ghostweight_matmul
    from ghostweight_triton.module import GhostLinear as GL
    from ghostweight_triton.utils.sparsity import sparsity_stats, log_sparsity  # noqa: F401
    from ghostweight_triton.utils import check_environment  # noqa: F401

    assert GL is GhostLinear
    assert dead_neuron_mask is gwb.dead_neuron_mask
    assert gather_compact is gwb.gather_compact and ghostweight_matmul is gwb.ghostweight_matmul
    assert ghostweight_triton.replace_linears is replace_linears


def _params(fn):
    return [(p.name, p.default) for p in inspect.signature(fn).parameters.values()
            if p.kind is not inspect.Parameter.KEYWORD_ONLY]


def test_signatures_match_reference():
    E = inspect.Parameter.empty
    assert _params(gwb.dead_neuron_mask) == [("activations", E), ("threshold", 1e-6), ("BLOCK_M", 512)]
    assert _params(gwb.gather_compact) == [("activations", E), ("weights", E), ("alive_indices", E),
                                           ("BLOCK_M", 64), ("BLOCK_K", 64), ("BLOCK_N", 64)]
    assert _params(gwb.ghostweight_matmul) == [("activations", E), ("weights", E),
                                               ("alive_indices", E), ("BLOCK_M", 64),
                                               ("BLOCK_N", 64), ("BLOCK_K", 32)]
    assert _params(GhostLinear.__init__)[:8] == [
        ("self", E), ("in_features", E), ("out_features", E), ("bias", True),
        ("threshold", 1e-6), ("min_sparsity_to_activate", 0.1), ("device", None), ("dtype", None)]
    assert _params(replace_linears) == [("model", E), ("threshold", 1e-6), ("skip_patterns", None),
                                        ("min_features", 128)]


@pytest.mark.parametrize("fn,args", [
    (gwb.dead_neuron_mask, (torch.randn(4, 8),)),
    (gwb.gather_compact, (torch.randn(4, 8), torch.randn(8, 3), torch.arange(4))),
    (gwb.ghostweight_matmul, (torch.randn(4, 8), torch.randn(8, 3), torch.arange(4))),
])
def test_cpu_tensors_are_rejected(fn, args):
    """No CPU fallback: the same AssertionError the reference raises (mask.py:87)."""
    with pytest.raises(AssertionError):
        fn(*args)


def test_shape_asserts():
    with pytest.raises(AssertionError):
        gwb.dead_neuron_mask(torch.randn(2, 3, 4))


def test_ghostlinear_forward_on_cpu_rejected():
    gl = GhostLinear(16, 8)
    with pytest.raises(AssertionError):
        gl(torch.randn(2, 16))


def test_from_linear_shares_parameters():
    lin = nn.Linear(32, 16)
    gl = GhostLinear.from_linear(lin, threshold=0.5, min_sparsity_to_activate=0.2)
    assert gl.weight is lin.weight and gl.bias is lin.bias
    assert gl.threshold == 0.5 and gl.min_sparsity_to_activate == 0.2
    assert not gl.mask_frozen and gl.current_sparsity == 0.0
    assert "in=32, out=16" in repr(gl)


def test_from_conv1d_is_a_transposed_view():
    from transformers.pytorch_utils import Conv1D

    conv = Conv1D(12, 20)          # nf=12 outputs, nx=20 inputs: weight [20, 12]
    gl = GhostLinear.from_conv1d(conv)
    assert gl.in_features == 20 and gl.out_features == 12
    assert gl.weight.shape == (12, 20)
    assert gl.weight.data_ptr() == conv.weight.data_ptr()
    assert gl.bias is conv.bias


def test_replace_linears_rules(toy_model_cpu):
    out = replace_linears(toy_model_cpu, min_features=128)
    assert isinstance(toy_model_cpu.fc1, GhostLinear) and isinstance(toy_model_cpu.fc2, GhostLinear)
    assert isinstance(toy_model_cpu.fc3, GhostLinear)          # in_features 128 >= 128
    assert out == {"fc1": 128, "fc2": 512, "fc3": 128}
    assert all(isinstance(v, int) for v in out.values())


def test_replace_min_features_and_skip(toy_model_cpu):
    replace_linears(toy_model_cpu, min_features=512)
    assert not isinstance(toy_model_cpu.fc1, GhostLinear)
    assert isinstance(toy_model_cpu.fc2, GhostLinear)

    class Nested(nn.Module):
        def __init__(self):
            super().__init__()
            self.encoder = nn.Sequential(nn.Linear(128, 256), nn.ReLU(), nn.Linear(256, 128))
            self.head = nn.Module()
            self.head.linear = nn.Linear(128, 10)
            self.lm_head = nn.Linear(10, 5)

    m = Nested()
    replace_linears(m, skip_patterns=["lm_head", "head"], min_features=1, threshold=0.05)
    assert not isinstance(m.lm_head, GhostLinear) and not isinstance(m.head.linear, GhostLinear)
    assert isinstance(m.encoder[0], GhostLinear) and isinstance(m.encoder[2], GhostLinear)
    assert m.encoder[0].threshold == pytest.approx(0.05)
    rep = get_sparsity_report(m)
    assert set(rep) == {"encoder.0", "encoder.2"} and all(isinstance(v, float) for v in rep.values())


def test_replace_is_idempotent(toy_model_cpu):
    replace_linears(toy_model_cpu, min_features=1)
    again = replace_linears(toy_model_cpu, min_features=1)
    assert again == {}


def test_replace_conv1d_gpt2_block():
    from transformers import GPT2Config, GPT2Model

    cfg = GPT2Config(n_layer=2, n_embd=128, n_head=4, n_positions=64, vocab_size=100)
    model = GPT2Model(cfg)
    out = replace_linears(model, min_features=128)
    # per layer: c_attn (128->384), attn.c_proj (128->128), c_fc (128->512), mlp.c_proj (512->128)
    assert len(out) == 8
    assert out["h.0.mlp.c_proj"] == 512
    assert isinstance(model.h[1].attn.c_attn, GhostLinear)
    off = replace_linears(GPT2Model(cfg), include_conv1d=False)
    assert off == {}


def test_empty_report_for_plain_model():
    assert get_sparsity_report(nn.Sequential(nn.ReLU(), nn.Dropout())) == {}


def test_frozen_indices_survive_state_dict():
    gl = GhostLinear(64, 32)
    nn.init.normal_(gl.weight)
    gl._set_frozen(torch.tensor([1, 5, 9], dtype=torch.int64))
    sd = gl.state_dict()
    assert "_frozen_indices" in sd
    fresh = GhostLinear(64, 32)
    fresh.load_state_dict(sd)
    assert fresh.mask_frozen and fresh._frozen_indices.tolist() == [1, 5, 9]
    assert fresh.current_sparsity == pytest.approx(1 - 3 / 64)
    fresh.unfreeze_mask()
    assert not fresh.mask_frozen and fresh._frozen_indices is None


def test_sparsity_utils_cpu(capsys):
    from ghostweight_triton_b200.utils import sparsity_stats, log_sparsity

    m = torch.tensor([1, 0, 1, 1], dtype=torch.int32)
    s = sparsity_stats(m)
    assert s == {"total": 4, "alive": 3, "dead": 1, "pct_dead": 0.25, "pct_alive": 0.75}
    log_sparsity(m)
    out = capsys.readouterr().out
    assert "3/4" in out and "25.0%" in out
    log_sparsity({"a": 0.5, "b": 0.25})
    out = capsys.readouterr().out
    assert "mean of 2 layers" in out and "37.5%" in out
    log_sparsity({})
    assert "no GhostLinear layers" in capsys.readouterr().out
    assert sparsity_stats(torch.zeros(0, dtype=torch.int32))["pct_dead"] == 0.0
    with pytest.raises(AssertionError):
        sparsity_stats(torch.zeros(2, 2))


def test_check_environment_reports_native_library():
    info = gwb.utils.check_environment(verbose=False)
    for k in ("torch_version", "triton_version", "cuda_version", "gpu_name", "compute_cap",
              "arch_list_set", "sm120_ready", "warnings", "sm100_ready", "native_library"):
        assert k in info
