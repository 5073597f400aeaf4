"""GPU, 2 ranks over NCCL: the column-parallel layer equals the dense layer on every rank.

Runs only where at least two GPUs are visible (skipped otherwise). Each rank is
a spawned process with a short process-group timeout; the parent joins them
with a deadline and terminates the ones it started if a rank stalls, so a
failure ends the test instead of hanging it. NVLS is off (plain peer
transfers), and no kernel of this package waits on another rank.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q) -> None:
    import datetime

    import torch.distributed as dist
    import torch.nn.functional as F

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    try:
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        from ghostweight_triton_b200.sharded import ColumnParallelGhostLinear

        device = torch.device("cuda", rank)
        results = {}

        def excess(y, ref):
            # How far y is outside the output contract (1e-2 atol + 1e-2 rtol
            # against the fp32 product rounded to y's dtype); <= 0 passes.
            r = ref.to(y.dtype).float()
            return ((y.float() - r).abs() - (1e-2 + 1e-2 * r.abs())).max().item()

        for dtype, (M, N, K) in ((torch.bfloat16, (2048, 4096, 2048)), (torch.float16, (300, 1000, 768))):
            g = torch.Generator(device=device).manual_seed(7)      # identical full tensors on all ranks
            w = (torch.randn(N, K, device=device, generator=g) / K ** 0.5).to(dtype)
            b = torch.randn(N, device=device, generator=g).to(dtype)
            x = torch.randn(M, K, device=device, generator=g).to(dtype)
            perm = torch.randperm(K, device=device, generator=g)
            dead = perm[: K // 2]
            w[:, dead] = 0
            # Column perm[-1] is zero in rank 0's rows only: the union mask keeps it alive
            # on both ranks, so every rank sees K - K/2 alive columns.
            w[: N // 2, perm[-1]] = 0
            layer = ColumnParallelGhostLinear.from_full_weight(w, b, device=device)
            y = layer(x)
            ref = F.linear(x.float(), w.float(), b.float())
            err = excess(y, ref)
            # The all-gather fused into the GEMM (peer stores over NVLink): three
            # calls cycle through both shared buffers; each result equals NCCL's.
            layer.gather_output = "peers"
            errs = []
            for step in range(3):
                xs = x if step != 1 else x * 0.5
                yp = layer(xs).clone()
                refp = ref if step != 1 else F.linear(xs.float(), w.float(), b.float())
                errs.append(excess(yp, refp))
            # A result still referenced is not overwritten: the call that would
            # reuse its buffer raises on every rank before any collective. (The
            # N = 1000 case splits into 500-wide shards, which take the NCCL
            # path: its outputs are fresh tensors and nothing is refused.)
            peer_path = layer.out_features % 8 == 0 and layer.n_local % 8 == 0
            kept = layer(x)
            layer(x)
            try:
                layer(x)
                assert not peer_path, "reusing a referenced peer buffer did not raise"
            except RuntimeError as e:
                assert peer_path and "still referenced" in str(e)
            kept_err = excess(kept, ref)
            del kept
            errs += [kept_err, excess(layer(x).clone(), ref)]
            layer.close()
            results[str(dtype)] = (max(err, *errs), layer.k_alive, tuple(y.shape))
        # Whole 128-column blocks dead: the alive list is 64-column runs, so both
        # output paths run the GEMM on x in place (strategy "runs", no gather).
        M, N, K = 1024, 2048, 2048
        g = torch.Generator(device=device).manual_seed(11)
        w = (torch.randn(N, K, device=device, generator=g) / K ** 0.5).half()
        b = torch.randn(N, device=device, generator=g).half()
        x = torch.randn(M, K, device=device, generator=g).half()
        blocks = torch.randperm(K // 128, device=device, generator=g)[: K // 256]
        w[:, (blocks[:, None] * 128 + torch.arange(128, device=device)).reshape(-1)] = 0
        layer = ColumnParallelGhostLinear.from_full_weight(w, b, device=device)
        ref = F.linear(x.float(), w.float(), b.float())
        errs = [excess(layer(x), ref)]
        layer.gather_output = "peers"
        for _ in range(2):
            errs.append(excess(layer(x), ref))
        layer.close()
        results["runs"] = (max(errs), layer.k_alive, layer.strategy)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, results, None))
    except Exception as e:  # reported to the parent, which fails the test
        import traceback

        q.put((rank, None, repr(e) + "\n" + traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_column_parallel_two_ranks_nccl():
    import torch.multiprocessing as mp

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            rank, res, err = q.get(timeout=240)
            assert err is None, f"rank {rank}: {err}"
            got[rank] = res
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    for rank, res in got.items():
        for dt in ("torch.bfloat16", "torch.float16"):
            err = res[dt][0]
            assert err <= 0.0, f"rank {rank} {dt}: outside atol=rtol=1e-2 by {err}"
        assert res["torch.bfloat16"][1] == 1024 and res["torch.bfloat16"][2] == (2048, 4096)
        assert res["torch.float16"][1] == 384 and res["torch.float16"][2] == (300, 1000)
        assert res["runs"][0] <= 0.0 and res["runs"][1:] == (1024, "runs"), res["runs"]
