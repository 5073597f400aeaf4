"""CPU (gloo ranks): host-side logic of the column-parallel sharded layer.

Covers shard bookkeeping (even and uneven splits), the union of per-shard
dead-column masks (all_reduce MAX) and the all-gather + re-layout of output
shards, with world sizes 2 and 3 spawned as separate processes.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ghostweight_triton_b200.sharded import gather_columns_from_ranks, shard_rows, union_mask


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_rows_cover_exactly():
    for n_total, world in [(28672, 8), (28672, 1), (10, 3), (7, 4), (1, 2)]:
        covered = []
        for r in range(world):
            start, stop, padded = shard_rows(n_total, world, r)
            assert 0 <= stop - start <= padded
            covered.extend(range(start, stop))
        assert covered == list(range(n_total))


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        K, M, N = 40, 5, 11
        torch.manual_seed(0)
        full_w = torch.randn(N, K)
        full_w[:, ::3] = 0                          # globally dead columns
        start, stop, padded = shard_rows(N, world, rank)
        local_w = torch.zeros(padded, K)
        local_w[: stop - start] = full_w[start:stop]
        # per-shard mask, then union
        mask = (local_w.abs().amax(0) > 0).to(torch.int32)
        union_mask(mask)
        expect = (full_w.abs().amax(0) > 0).to(torch.int32)
        ok_mask = torch.equal(mask, expect)
        # local output shard and gathered full output
        x = torch.randn(M, K, generator=torch.Generator().manual_seed(1))
        y_local = x @ local_w.t()
        full = gather_columns_from_ranks(y_local, N)
        ok_y = torch.allclose(full, x @ full_w.t(), atol=1e-5)
        q.put((rank, ok_mask, ok_y, tuple(full.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_union_mask_and_gather(world):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = sorted(q.get() for _ in range(world))
    for rank, ok_mask, ok_y, shape in results:
        assert ok_mask, f"rank {rank}: union mask differs from the full-weight mask"
        assert ok_y, f"rank {rank}: gathered output differs from the dense product"
        assert shape == (5, 11)
