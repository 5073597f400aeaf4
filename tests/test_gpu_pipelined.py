"""GPU: ghost_linear_pipelined (each call's gather overlapping the previous GEMM).

Independent gather-GEMM calls run with the gather of call i+1 on a
low-priority stream while call i's GEMM runs on a high-priority one, x'
alternating between two buffers. Every output must equal the same call made
alone through ghost_linear, bit for bit (the same kernels run on the same
operands), for pipelined calls, for the calls that fall back to ghost_linear
(few rows, fp32), with bias and GELU, and with shapes changing from call to
call.
"""

from __future__ import annotations

import pytest
import torch

from ghostweight_triton_b200.kernels.gather import pack_weight
from ghostweight_triton_b200.kernels.matmul import ghost_linear, ghost_linear_pipelined

pytestmark = pytest.mark.gpu


def _layer(M, K, N, kp, dtype, seed, bias=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    w = (torch.randn(N, K, device="cuda", generator=g) / kp ** 0.5).to(dtype)
    idx = torch.sort(torch.randperm(K, device="cuda", generator=g)[:kp]).values
    b = torch.randn(N, device="cuda", generator=g).to(dtype) if bias else None
    return x, pack_weight(w, idx), idx, b


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_pipelined_equals_one_call_at_a_time(dtype):
    specs = [  # (M, K, N, K', bias, activation)
        (4096, 4096, 4096, 2048, False, None),
        (2048, 2048, 3072, 1000, True, "gelu_tanh"),
        (4096, 4096, 4096, 2048, True, "gelu"),
        (100, 1024, 512, 300, True, None),        # split-K GEMM under the pipeline
        (3, 1024, 512, 300, True, None),          # decode rows: ghost_linear on the GEMM stream
        (1024, 3072, 768, 1536, False, None),
        (4096, 4096, 4096, 410, False, None),
    ]
    calls, refs = [], []
    for s, (M, K, N, kp, bias, act) in enumerate(specs):
        x, wp, idx, b = _layer(M, K, N, kp, dtype, 10 + s, bias)
        refs.append(ghost_linear(x, wp, idx, bias=b, activation=act))
        out = torch.full((M, N), float("nan"), device="cuda", dtype=dtype)
        calls.append((x, wp, idx, out, b, act))
    outs = ghost_linear_pipelined(calls)
    torch.cuda.synchronize()
    for o, r, c in zip(outs, refs, calls):
        assert o is c[3]
        assert torch.equal(o, r)


def test_pipelined_repeated_and_fp32_fallback():
    x, wp, idx, _ = _layer(4096, 2048, 2048, 1024, torch.float16, 3)
    x32 = torch.randn(512, 256, device="cuda")
    w32 = torch.randn(384, 256, device="cuda")
    idx32 = torch.arange(0, 256, 2, device="cuda")
    wp32 = pack_weight(w32, idx32)
    ref = ghost_linear(x, wp, idx)
    ref32 = ghost_linear(x32, wp32, idx32)
    # Many calls through the same two x' slots, an fp32 call in between.
    calls = [(x, wp, idx, torch.empty_like(ref)) for _ in range(7)]
    calls.insert(3, (x32, wp32, idx32, torch.empty_like(ref32)))
    outs = ghost_linear_pipelined(calls)
    for i, o in enumerate(outs):
        assert torch.equal(o, ref32 if i == 3 else ref)
    # The caller's stream is ordered after every call: a kernel queued on it
    # right away sees the results.
    assert torch.equal(outs[-1].sum(), ref.sum())


def test_pipelined_captured_in_a_graph():
    x, wp, idx, _ = _layer(4096, 2048, 2048, 1024, torch.float16, 5)
    x2, wp2, idx2, b2 = _layer(2048, 1024, 3072, 700, torch.float16, 6, bias=True)
    ref, ref2 = ghost_linear(x, wp, idx), ghost_linear(x2, wp2, idx2, bias=b2, activation="gelu")
    outs = [torch.empty_like(ref), torch.empty_like(ref2), torch.empty_like(ref)]
    ghost_linear_pipelined([(x, wp, idx, outs[0]), (x2, wp2, idx2, outs[1], b2, "gelu"),
                            (x, wp, idx, outs[2])])          # eager first: events recorded outside
    for o in outs:
        o.zero_()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        ghost_linear_pipelined([(x, wp, idx, outs[0]), (x2, wp2, idx2, outs[1], b2, "gelu"),
                                (x, wp, idx, outs[2])])
    torch.cuda.current_stream().wait_stream(side)
    for o in outs:
        o.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(outs[0], ref) and torch.equal(outs[1], ref2) and torch.equal(outs[2], ref)


def test_pipelined_growing_shapes_reuse_no_stale_buffer():
    # Each call needs a larger x' than the one before, so both slots are
    # replaced while earlier calls are still queued; a tensor allocated in
    # between must not land on a buffer a queued GEMM still reads.
    layers = [_layer(M, 2048, 1024, kp, torch.float16, 40 + i)
              for i, (M, kp) in enumerate(((512, 256), (1024, 512), (2048, 1024), (4096, 2048)))]
    refs = [ghost_linear(x, wp, idx) for x, wp, idx, _ in layers]
    outs = ghost_linear_pipelined([(x, wp, idx, torch.empty_like(r))
                                   for (x, wp, idx, _), r in zip(layers, refs)])
    junk = [torch.full((4096, 4096), 7.0, dtype=torch.float16, device="cuda") for _ in range(4)]
    torch.cuda.synchronize()
    for o, r in zip(outs, refs):
        assert torch.equal(o, r)
    del junk
