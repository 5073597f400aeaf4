"""GPU (single process): the column-parallel layer at world size 1 equals the dense layer.

Multi-rank behaviour of the same host logic is covered on gloo CPU ranks
(tests/test_sharded_cpu.py); this checks the device path end to end.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from ghostweight_triton_b200.sharded import ColumnParallelGhostLinear

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_world1_matches_dense(dtype):
    torch.manual_seed(0)
    N, K, M = 520, 1024, 300
    w = (torch.randn(N, K, device="cuda") / K ** 0.5).to(dtype)
    w[:, 128:768] = 0
    b = torch.randn(N, device="cuda").to(dtype)
    layer = ColumnParallelGhostLinear.from_full_weight(w, b)
    assert layer.k_alive == K - 640
    x = torch.randn(M, K, device="cuda").to(dtype)
    torch.testing.assert_close(layer(x), F.linear(x.float(), w.float(), b.float()).to(dtype),
                               atol=1e-2, rtol=1e-2)


def test_world1_repacks_after_weight_updates():
    """W' follows the shard's weight: a version-bumping in-place update is
    picked up by itself, a write through .data after refresh_packed()."""
    torch.manual_seed(1)
    N, K, M = 512, 1024, 128
    w = (torch.randn(N, K, device="cuda") / K ** 0.5).half()
    w[:, 256:768] = 0
    b = torch.randn(N, device="cuda").half()
    layer = ColumnParallelGhostLinear.from_full_weight(w, b)
    x = torch.randn(M, K, device="cuda").half()

    def check():
        wn = layer.weight.detach()[:N].float()
        ref = F.linear(x.float(), wn, layer.bias.detach()[:N].float())
        torch.testing.assert_close(layer(x).float(), ref, atol=1e-2, rtol=1e-2)

    check()
    with torch.no_grad():
        layer.weight.mul_(2)
    check()
    layer.weight.data.mul_(0.25)
    layer.refresh_packed()
    check()
