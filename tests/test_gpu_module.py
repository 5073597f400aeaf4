"""GPU: GhostLinear, replace_linears and the end-to-end chain on B200.

Ports the reference's module / replace / end-to-end suites
(ghostweight_triton tests/test_module.py:65-260, test_replace.py:78-246,
test_end_to_end.py:68-267) and replays the golden chain fixtures
(mask -> nonzero -> matmul + bias computed by the reference) through
GhostLinear in dynamic mode.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from ghostweight_triton_b200 import GhostLinear, replace_linears, get_sparsity_report
from ghostweight_triton_b200.kernels import dead_neuron_mask, ghostweight_matmul
from ghostweight_triton_b200.utils.sparsity import sparsity_stats, log_sparsity
from tests.golden import gw_golden as G

pytestmark = pytest.mark.gpu

TOL = {"f16": (1e-2, 1e-2), "f32": (1e-4, 1e-4)}


def _from_linear(in_f, out_f, bias, device, dtype, threshold=1e-6, seed=42):
    torch.manual_seed(seed)
    lin = nn.Linear(in_f, out_f, bias=bias).to(device=device, dtype=dtype)
    return GhostLinear.from_linear(lin, threshold=threshold), lin


@pytest.mark.parametrize("name", G.names("chain"))
def test_golden_chain_through_ghostlinear(name):
    meta, inp, exp = G.load(name)
    dt = {"f16": torch.float16, "f32": torch.float32}[meta["dtype"]]
    N, K = inp["weight"].shape
    gl = GhostLinear(K, N, bias=True, device="cuda", dtype=dt)
    with torch.no_grad():
        gl.weight.copy_(torch.from_numpy(inp["weight"]))
        gl.bias.copy_(torch.from_numpy(inp["bias"]))
        y = gl(torch.from_numpy(inp["x"]).cuda())
    atol, rtol = TOL[meta["dtype"]]
    G.check_close(y.cpu().numpy(), exp, "y", atol, rtol)
    assert gl.current_sparsity == pytest.approx(1 - exp["alive"].shape[0] / K)


class TestConstructionAndForward:
    def test_construction(self, device):
        torch.manual_seed(42)
        gl = GhostLinear(128, 256, device=device, dtype=torch.float16)
        assert gl.weight.shape == (256, 128)
        gl, lin = _from_linear(256, 512, True, device, torch.float16)
        assert gl.weight is lin.weight and gl.bias is lin.bias
        gl, _ = _from_linear(256, 512, False, device, torch.float32)
        assert gl.bias is None

    @pytest.mark.parametrize("M,in_f,out_f", [(1, 128, 256), (1, 768, 3072), (16, 768, 3072),
                                              (128, 768, 3072), (128, 3072, 768)])
    def test_output_shape_2d(self, device, M, in_f, out_f):
        gl, _ = _from_linear(in_f, out_f, True, device, torch.float16)
        assert gl(torch.randn(M, in_f, dtype=torch.float16, device=device)).shape == (M, out_f)

    def test_output_shape_3d(self, device):
        gl, _ = _from_linear(128, 256, True, device, torch.float16)
        assert gl(torch.randn(2, 16, 128, dtype=torch.float16, device=device)).shape == (2, 16, 256)

    @pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.bfloat16])
    def test_output_dtype_finite(self, device, dtype):
        gl, _ = _from_linear(768, 3072, True, device, dtype)
        y = gl(torch.randn(32, 768, dtype=dtype, device=device))
        assert y.dtype == dtype and torch.isfinite(y).all()

    def test_dense_fallback_matches_f_linear(self, device):
        gl, lin = _from_linear(128, 256, True, device, torch.float32)
        x = torch.ones(8, 128, device=device)
        torch.testing.assert_close(gl(x), F.linear(x, lin.weight, lin.bias), atol=1e-4, rtol=1e-4)

    @pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.bfloat16])
    def test_ghost_path_matches_f_linear(self, device, dtype):
        # The output contract: 1e-2 (atol and rtol) for 16-bit outputs, 1e-4
        # for fp32, against the exact product rounded to the output dtype.
        torch.manual_seed(7)
        lin = nn.Linear(256, 512).to(device=device, dtype=dtype)
        gl = GhostLinear.from_linear(lin)
        x = torch.randn(16, 256, dtype=dtype, device=device)
        x[:, ::2] = 0.0
        y = gl(x)
        assert gl.current_sparsity == pytest.approx(0.5)
        ref = F.linear(x.double(), lin.weight.double(), lin.bias.double()).to(dtype)
        tol = 1e-4 if dtype == torch.float32 else 1e-2
        torch.testing.assert_close(y, ref, atol=tol, rtol=tol)

    def test_sparsity_property(self, device):
        gl, _ = _from_linear(128, 256, True, device, torch.float32)
        gl(torch.zeros(4, 128, device=device))
        assert gl.current_sparsity >= 0.99
        gl(torch.ones(4, 128, device=device))
        assert gl.current_sparsity < 0.1
        assert isinstance(gl.current_sparsity, float)

    def test_bias(self, device):
        torch.manual_seed(5)
        lin = nn.Linear(64, 128).to(device=device)
        nn.init.constant_(lin.bias, 1.0)
        gl = GhostLinear.from_linear(lin)
        assert gl(torch.zeros(4, 64, device=device)).abs().sum().item() > 0
        gl, _ = _from_linear(64, 128, False, device, torch.float32)
        assert gl(torch.zeros(4, 64, device=device)).abs().sum().item() == 0.0


@pytest.mark.parametrize("mode", ["dynamic", "dynamic_host_count", "frozen"])
def test_fp32_ghostlinear_8x128x768_to_3072_matches_oracle(mode):
    """The single fp32 GhostLinear workload at its own shape and the fp32 contract.

    X [8, 128, 768] ~ N(0, 1), W [3072, 768] ~ N(0, 0.02), bias [3072] ~ N(0, 0.02);
    384 seeded-random input columns zeroed in W and in X; threshold 0, so the
    activation mask finds exactly the zeroed columns. Checked against the
    oracle's GhostLinear (mask -> alive list -> x[:, idx] @ W[:, idx]^T + b) at
    rtol = atol = 1e-4 (the reference's fp32 tolerance, tests/test_matmul.py:68-72).
    """
    from oracle import gw_oracle as O

    rng = np.random.default_rng(2024)
    x = rng.standard_normal((8, 128, 768), dtype=np.float32)
    w = (rng.standard_normal((3072, 768), dtype=np.float32) * 0.02).astype(np.float32)
    b = (rng.standard_normal(3072, dtype=np.float32) * 0.02).astype(np.float32)
    dead = np.sort(rng.permutation(768)[:384])
    w[:, dead] = 0
    x[..., dead] = 0
    idx = O.alive_indices(O.dead_neuron_mask(x.reshape(-1, 768), 0.0))
    assert np.array_equal(idx, np.setdiff1d(np.arange(768), dead))
    ref = O.ghost_linear(x.reshape(-1, 768), w, idx, b)

    gl = GhostLinear(768, 3072, bias=True, threshold=0.0, device="cuda", dtype=torch.float32)
    with torch.no_grad():
        gl.weight.copy_(torch.from_numpy(w))
        gl.bias.copy_(torch.from_numpy(b))
    xd = torch.from_numpy(x).cuda()
    if mode == "dynamic_host_count":
        gl.sync_free = False
    if mode == "frozen":
        gl.freeze_mask(xd)
        assert np.array_equal(gl._frozen_indices.cpu().numpy(), idx)
    with torch.no_grad():
        for _ in range(2):      # the second forward sees the first one's count
            y = gl(xd)
    assert y.shape == (8, 128, 3072) and y.dtype == torch.float32
    assert gl.current_sparsity == pytest.approx(0.5)
    np.testing.assert_allclose(y.reshape(-1, 3072).cpu().numpy(), ref, rtol=1e-4, atol=1e-4)


class TestFreeze:
    def test_frozen_sparsity_constant(self, device):
        gl, _ = _from_linear(128, 256, True, device, torch.float32)
        cal = torch.zeros(4, 128, device=device)
        cal[:, :64] = 1.0
        gl.freeze_mask(cal)
        sp = gl.current_sparsity
        assert sp == pytest.approx(0.5) and gl.mask_frozen
        gl(torch.ones(4, 128, device=device))
        assert gl.current_sparsity == pytest.approx(sp)

    def test_frozen_forward_matches_reference_semantics(self, device):
        """Frozen mode computes x[:, frozen] @ W[:, frozen]^T + b, whatever x holds."""
        gl, lin = _from_linear(256, 192, True, device, torch.float32)
        cal = torch.randn(8, 256, device=device)
        cal[:, 100:] = 0
        gl.freeze_mask(cal)
        x = torch.randn(10, 256, device=device)
        y = gl(x)
        idx = torch.arange(100, device=device)
        ref = x[:, idx] @ lin.weight[:, idx].t() + lin.bias
        torch.testing.assert_close(y, ref, atol=1e-4, rtol=1e-4)
        for _ in range(3):
            assert gl(torch.randn(8, 256, device=device)).shape == (8, 192)

    def test_weight_mask_freeze_is_exact(self, device):
        torch.manual_seed(1)
        lin = nn.Linear(512, 300).to(device=device, dtype=torch.float16)
        with torch.no_grad():
            lin.weight[:, 64:320] = 0
        gl = GhostLinear.from_linear(lin)
        gl.freeze_weight_mask()
        assert gl.current_sparsity == pytest.approx(0.5)
        x = torch.randn(33, 512, dtype=torch.float16, device=device)
        torch.testing.assert_close(gl(x), F.linear(x, lin.weight, lin.bias), atol=1e-2, rtol=1e-2)

    def test_weight_update_repacks(self, device):
        gl, lin = _from_linear(128, 64, False, device, torch.float32)
        gl.freeze_mask(torch.ones(2, 128, device=device))
        gl.min_sparsity_to_activate = 0.0
        x = torch.randn(4, 128, device=device)
        y1 = gl(x)
        with torch.no_grad():
            lin.weight.mul_(2.0)
        torch.testing.assert_close(gl(x), 2 * y1, atol=1e-4, rtol=1e-4)

    def test_state_dict_roundtrip_on_gpu(self, device):
        gl, lin = _from_linear(128, 64, True, device, torch.float16)
        cal = torch.randn(4, 128, dtype=torch.float16, device=device)
        cal[:, ::4] = 0
        gl.freeze_mask(cal)
        fresh = GhostLinear(128, 64, device=device, dtype=torch.float16)
        fresh.load_state_dict(gl.state_dict())
        x = torch.randn(5, 128, dtype=torch.float16, device=device)
        torch.testing.assert_close(fresh(x), gl(x))


class TestActivationEpilogue:
    @pytest.mark.parametrize("act,approx", [("gelu", "none"), ("gelu_tanh", "tanh")])
    def test_fused_gelu(self, device, act, approx):
        torch.manual_seed(3)
        lin = nn.Linear(256, 384).to(device=device, dtype=torch.float16)
        gl = GhostLinear.from_linear(lin)
        gl.activation = act
        x = torch.randn(40, 256, dtype=torch.float16, device=device)
        x[:, 1::3] = 0
        ref = F.gelu(F.linear(x.float(), lin.weight.float(), lin.bias.float()), approximate=approx)
        torch.testing.assert_close(gl(x).float(), ref, atol=1e-2, rtol=1e-2)


class TestReplaceAndModels:
    def test_qualifying_layers_and_forward(self, device, toy_model):
        replace_linears(toy_model, min_features=128)
        assert isinstance(toy_model.fc1, GhostLinear) and isinstance(toy_model.fc2, GhostLinear)
        with torch.no_grad():
            y = toy_model(torch.randn(4, 128, dtype=torch.float16, device=device))
        assert y.shape == (4, 10)
        rep = get_sparsity_report(toy_model)
        assert set(rep) == {n for n, m in toy_model.named_modules() if isinstance(m, GhostLinear)}
        assert all(0.0 <= v <= 1.0 for v in rep.values())

    def test_zero_input_higher_sparsity(self, device, toy_model):
        replace_linears(toy_model, min_features=128)
        with torch.no_grad():
            toy_model(torch.ones(4, 128, dtype=torch.float16, device=device))
        dense = sum(get_sparsity_report(toy_model).values())
        with torch.no_grad():
            toy_model(torch.zeros(4, 128, dtype=torch.float16, device=device))
        assert sum(get_sparsity_report(toy_model).values()) >= dense

    def test_stacked_and_transformer_layer(self, device):
        layers = nn.Sequential(nn.Linear(256, 1024), nn.ReLU(), nn.Linear(1024, 512), nn.ReLU(),
                               nn.Linear(512, 128)).to(device=device, dtype=torch.float16)
        x = torch.randn(32, 256, dtype=torch.float16, device=device)
        with torch.no_grad():
            ref = layers(x)
        replace_linears(layers, min_features=128)
        with torch.no_grad():
            y = layers(x)
        assert torch.isfinite(y).all()
        torch.testing.assert_close(y, ref, atol=2e-2, rtol=2e-2)

    def test_gpt2_conv1d_forward_matches_dense(self, device):
        from transformers import GPT2Config, GPT2Model

        cfg = GPT2Config(n_layer=2, n_embd=256, n_head=4, n_positions=128, vocab_size=1000)
        torch.manual_seed(0)
        model = GPT2Model(cfg).to(device=device, dtype=torch.float16).eval()
        # Zero half the input columns of every Conv1D weight ([in, out] rows).
        g = torch.Generator().manual_seed(0)
        with torch.no_grad():
            for mod in model.modules():
                if type(mod).__name__ == "Conv1D":
                    n_in = mod.weight.shape[0]
                    dead = torch.randperm(n_in, generator=g)[: n_in // 2].to(device)
                    mod.weight[dead, :] = 0
        ids = torch.randint(0, 1000, (2, 64), device=device)
        with torch.no_grad():
            ref = model(ids).last_hidden_state
        out = replace_linears(model, min_features=128, freeze_from_weight=True)
        assert len(out) == 8
        with torch.no_grad():
            y = model(ids).last_hidden_state
        torch.testing.assert_close(y, ref, atol=3e-2, rtol=3e-2)


class TestEndToEnd:
    def test_mask_to_matmul_pipeline(self, device):
        torch.manual_seed(10)
        A = torch.randn(32, 256, dtype=torch.float16, device=device) * 0.1
        W = torch.randn(256, 128, dtype=torch.float16, device=device) * 0.1
        A[:, ::2] = 0.0
        mask = dead_neuron_mask(A, threshold=1e-6)
        alive = mask.nonzero(as_tuple=True)[0].to(torch.int64)
        C = ghostweight_matmul(A, W, alive)
        ref = (A.float()[:, alive] @ W.float()[alive, :]).half()
        torch.testing.assert_close(C, ref, atol=1e-2, rtol=1e-2)

    def test_sparsity_stats_and_log(self, device, capsys):
        A = torch.zeros(4, 128, dtype=torch.float16, device=device)
        A[:, :64] = 1.0
        s = sparsity_stats(dead_neuron_mask(A))
        assert s["alive"] == 64 and s["dead"] == 64 and s["pct_dead"] == pytest.approx(0.5)
        log_sparsity(dead_neuron_mask(A))
        assert "64/128" in capsys.readouterr().out


def test_packed_weight_follows_weight_updates():
    """The frozen W' is rebuilt when the weight is rebound to other storage or
    updated through a version-bumping in-place op, and after refresh_packed()
    for in-place writes through .data (which bypass the version counter)."""
    K, N, M = 512, 256, 64
    g = torch.Generator(device="cuda").manual_seed(7)
    gl = GhostLinear(K, N, bias=True, device="cuda", dtype=torch.float16)
    dead = torch.randperm(K, device="cuda", generator=g)[: K // 2]
    with torch.no_grad():
        gl.weight.normal_(0.0, K ** -0.5, generator=g)
        gl.weight[:, dead] = 0
        gl.bias.normal_(0.0, 0.1, generator=g)
    gl.freeze_weight_mask()
    x = torch.randn(M, K, device="cuda", generator=g).half()

    def check():
        with torch.no_grad():
            y = gl(x)
        ref = F.linear(x.float(), gl.weight.detach().float(), gl.bias.detach().float())
        torch.testing.assert_close(y.float(), ref, atol=1e-2, rtol=1e-2)

    check()
    gl.weight.data = gl.weight.detach().clone() * 2          # new storage, same object and version
    check()
    with torch.no_grad():
        gl.weight.mul_(0.5)                                  # version-bumping in-place update
    check()
    gl.weight.data.mul_(3)                                   # in place through .data: no version bump
    gl.refresh_packed()
    check()
