"""Column-parallel GhostLinear: output features split across ranks.

For layers too large for one GPU's share of a job (e.g. an MLP up-projection
x [8192, 8192] -> [8192, 28672]), rank r holds the pre-sharded weight rows
W[r*n : (r+1)*n, :] and bias slice; x is replicated. Each rank:

  1. computes the dead-column mask of its own shard with K1 and takes the
     union over ranks (all_reduce MAX of the int32 [K] mask, K*4 bytes), so
     every rank uses the same alive list -- exactly the list the full weight
     would give (a column is dead in W iff it is dead in every shard);
  2. packs its shard's alive columns once (K2);
  3. runs the tcgen05 gather-GEMM on its rows (K3) -> y_r [M, n] (strategy
     "runs", no gather, when the alive list is made of 64-column runs);
  4. if the next op needs full rows, either all-gathers y (NCCL over NVLink)
     into [world, M, n] and re-lays it out to [M, N] (gather_output=True), or
     (gather_output="peers") lets the GEMM itself store every finished tile
     into all ranks' full [M, N] outputs over NVLink (CUDA IPC mappings of the
     peers' buffers, gw_gather_gemm_peers), followed by one small collective
     that orders every rank's readers after every rank's GEMM.

The reference has no multi-GPU code; this is the sharded configuration of the
same hot path. Uneven splits pad the last shard with zero rows.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist
import torch.nn as nn

from ghostweight_triton_b200.kernels.gather import pack_weight
from ghostweight_triton_b200.kernels.mask import dead_neuron_mask_compact
from ghostweight_triton_b200.kernels.matmul import ghost_linear, index_runs


def shard_rows(n_total: int, world: int, rank: int) -> tuple[int, int, int]:
    """(start, stop, padded) rows owned by `rank`; every rank pads to `padded` rows."""
    padded = -(-n_total // world)
    start = min(rank * padded, n_total)
    stop = min(start + padded, n_total)
    return start, stop, padded


def union_mask(mask: torch.Tensor, group=None) -> torch.Tensor:
    """Element-wise OR of int32 0/1 masks over the group (in place, returns mask)."""
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(mask, op=dist.ReduceOp.MAX, group=group)
    return mask


class PeerOutputs:
    """Full-size [rows, cols] output buffers shared by the ranks of a group.

    Each rank allocates `n_buf` buffers with cudaMalloc (outside torch's
    caching allocator, so that CUDA IPC handles cover exactly one buffer),
    exports their IPC handles, and opens every peer's; rank r then holds the
    device addresses of all ranks' buffer i. Mappings are closed and buffers
    freed by close() (collective: every rank closes its peer mappings, then a
    barrier, then each frees its own).
    """

    def __init__(self, rows: int, cols: int, dtype: torch.dtype, group=None, n_buf: int = 2):
        from cuda.bindings import runtime as rt

        self._rt = rt
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows, self.cols, self.dtype = rows, cols, dtype
        self.device = torch.cuda.current_device()
        self._check(rt.cudaSetDevice(self.device))
        nbytes = rows * cols * torch.empty((), dtype=dtype).element_size()
        self._own: list[int] = []
        self._peers: list[list[int]] = []        # [buf][rank] -> address (own at index rank)
        handles = []
        for _ in range(n_buf):
            ptr = self._check(rt.cudaMalloc(nbytes))
            self._own.append(int(ptr))
            h = self._check(rt.cudaIpcGetMemHandle(ptr))
            handles.append(bytes(h.reserved))
        gathered: list = [None] * self.world
        dist.all_gather_object(gathered, handles, group=group)
        for i in range(n_buf):
            addrs = []
            for r in range(self.world):
                if r == self.rank:
                    addrs.append(self._own[i])
                    continue
                h = rt.cudaIpcMemHandle_t()
                h.reserved = gathered[r][i]
                addrs.append(int(self._check(
                    rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess))))
            self._peers.append(addrs)
        self._views = [self._wrap(ptr, nbytes) for ptr in self._own]

    @staticmethod
    def _check(res):
        err = res[0] if isinstance(res, tuple) else res
        if int(err) != 0:
            raise RuntimeError(f"CUDA runtime error {err}")
        return res[1] if isinstance(res, tuple) and len(res) > 1 else None

    def _wrap(self, ptr: int, nbytes: int) -> torch.Tensor:
        class _Mem:
            __cuda_array_interface__ = {"shape": (nbytes // 2,), "typestr": "<i2",
                                        "data": (ptr, False), "strides": None,
                                        "version": 2}
        t = torch.as_tensor(_Mem(), device=torch.device("cuda", self.device))
        assert t.data_ptr() == ptr and t.numel() == nbytes // 2
        return t.view(self.dtype).view(self.rows, self.cols)

    def local(self, i: int) -> torch.Tensor:
        return self._views[i]

    def peer_addresses(self, i: int, byte_offset: int = 0) -> list[int]:
        """Addresses of the other ranks' buffer i (rank order, own rank left out)."""
        return [a + byte_offset for r, a in enumerate(self._peers[i]) if r != self.rank]

    def close(self) -> None:
        rt = self._rt
        for addrs in self._peers:
            for r, a in enumerate(addrs):
                if r != self.rank:
                    rt.cudaIpcCloseMemHandle(a)
        self._peers = []
        dist.barrier(group=self.group)
        for ptr in self._own:
            rt.cudaFree(ptr)
        self._own = []
        self._views = []


def gather_columns_from_ranks(y_local: torch.Tensor, n_total: int, group=None,
                              out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather row-major [M, n] shards into [M, n_total] (shard r -> columns r*n ..)."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return y_local[:, :n_total]
    M, n = y_local.shape
    buf = torch.empty((world * M, n), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local.contiguous(), group=group)
    full = buf.view(world, M, n).permute(1, 0, 2).reshape(M, world * n)
    if out is None:
        return full[:, :n_total].contiguous()
    out.copy_(full[:, :n_total])
    return out


class ColumnParallelGhostLinear(nn.Module):
    """GhostLinear whose output features are split across the ranks of `group`."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True,
                 threshold: float = 0.0, gather_output: bool | str = True, group=None,
                 device=None, dtype=None):
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.in_features = in_features
        self.out_features = out_features
        self.threshold = threshold
        self.gather_output = gather_output
        self.row_start, self.row_stop, self.n_local = shard_rows(out_features, self.world, self.rank)
        factory = {"device": device, "dtype": dtype}
        self.weight = nn.Parameter(torch.zeros(self.n_local, in_features, **factory))
        self.bias = nn.Parameter(torch.zeros(self.n_local, **factory)) if bias else None
        self.alive: torch.Tensor | None = None
        self.w_packed: torch.Tensor | None = None
        self._packed_key: tuple | None = None   # (weight, version, storage) w_packed was built from
        self.strategy = "auto"       # "runs" when the alive list is 64-column runs
        self._peer_out: PeerOutputs | None = None
        self._peer_step = 0
        self._flag: torch.Tensor | None = None
        # Weak references to the tensor each shared buffer last returned (see
        # _forward_peers): a buffer is not overwritten while it is referenced.
        self._peer_returned: list = [None, None]

    @property
    def k_alive(self) -> int:
        return -1 if self.alive is None else int(self.alive.numel())

    # ------------------------------------------------------------------ construction
    @classmethod
    def from_full_weight(cls, weight: torch.Tensor, bias: torch.Tensor | None = None,
                         threshold: float = 0.0, gather_output: bool = True, group=None,
                         device=None) -> "ColumnParallelGhostLinear":
        """Take this rank's rows of a full [N, K] weight (and bias) and freeze the mask."""
        N, K = weight.shape
        dev = device if device is not None else weight.device
        m = cls(K, N, bias=bias is not None, threshold=threshold, gather_output=gather_output,
                group=group, device=dev, dtype=weight.dtype)
        rows = m.row_stop - m.row_start
        with torch.no_grad():
            m.weight[:rows].copy_(weight[m.row_start:m.row_stop])
            if bias is not None:
                m.bias[:rows].copy_(bias[m.row_start:m.row_stop])
        m.freeze_weight_mask()
        return m

    @classmethod
    def from_full_weight_seed(cls, out_features: int, in_features: int, seed: int,
                              dead: np.ndarray, dtype: torch.dtype, device,
                              group=None) -> "ColumnParallelGhostLinear":
        """Pre-sharded synthetic weight: each rank draws only its rows, N(0, 1/sqrt(K)),
        with the global dead columns zeroed (benchmarks; no full weight is built)."""
        m = cls(in_features, out_features, bias=False, threshold=0.0, group=group,
                device=device, dtype=dtype)
        g = torch.Generator(device=device).manual_seed(seed * 1009 + m.rank)
        rows = m.row_stop - m.row_start
        with torch.no_grad():
            w = torch.randn(rows, in_features, device=device, generator=g) / in_features ** 0.5
            w[:, torch.from_numpy(np.asarray(dead)).to(device)] = 0
            m.weight[:rows].copy_(w.to(dtype))
        m.freeze_weight_mask()
        return m

    # ------------------------------------------------------------------ mask
    def freeze_weight_mask(self) -> None:
        """Alive columns = union over ranks of each shard's |W| column mask."""
        with torch.no_grad():
            mask, _, _ = dead_neuron_mask_compact(self.weight.detach(), self.threshold)
            union_mask(mask, self.group)
            self.alive = torch.nonzero(mask, as_tuple=False).squeeze(-1).to(torch.int64)
            self._packed_key = None
            self._packed_weight()
            # Same list on every rank, so every rank picks the same strategy.
            runs = (self.weight.dtype != torch.float32 and self.alive.numel() > 0
                    and index_runs(self.alive, self.in_features) == 0)
            self.strategy = "runs" if runs else "auto"

    def _packed_weight(self) -> torch.Tensor:
        """This shard's W' over the frozen alive list, packed again when the
        weight was replaced, moved to other storage or updated in place through
        autograd-visible operations (its version counter). The alive list stays
        the frozen union, so repacking is local to the rank."""
        w = self.weight
        key = (w, w._version, w.data_ptr())
        k = self._packed_key
        if k is None or k[0] is not w or k[1:] != key[1:]:
            with torch.no_grad():
                self.w_packed = pack_weight(w.detach(), self.alive)
            self._packed_key = key
        return self.w_packed

    def refresh_packed(self) -> None:
        """Pack W' again at the next forward: needed after in-place writes
        through ``weight.data``, which bypass the version counter."""
        self._packed_key = None

    # ------------------------------------------------------------------ forward
    def local_forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's output columns y[:, start:start+n_local] (padded rows included)."""
        assert self.alive is not None, "call freeze_weight_mask() first"
        x2 = x.reshape(-1, self.in_features)
        return ghost_linear(x2, self._packed_weight(), self.alive, bias=self.bias, out=out,
                            strategy=self.strategy)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        # Peer stores need 16-byte aligned rows and block offsets (multiples of 8
        # elements) on every rank -- the shard width decides it uniformly, so all
        # ranks take the same path and issue the same collectives.
        if (self.gather_output == "peers" and self.world > 1 and self.out_features % 8 == 0
                and self.n_local % 8 == 0):
            return self._forward_peers(x, lead)
        y = self.local_forward(x)
        if not self.gather_output:
            return y.reshape(*lead, self.n_local)
        full = gather_columns_from_ranks(y, self.out_features, self.group)
        return full.reshape(*lead, self.out_features)

    def _forward_peers(self, x: torch.Tensor, lead: tuple = ()) -> torch.Tensor:
        """Full [..., N] output with the all-gather fused into the GEMM (peer stores).

        The result is a view of one of two shared buffers used in turn, which
        every rank's GEMM of the call after the next one writes again. That call
        raises RuntimeError while the tensor returned from that buffer is still
        referenced (keep a ``.clone()`` of outputs you need longer; views derived
        from the returned tensor are not tracked). Every rank must call with the
        same M.
        """
        import weakref

        from ghostweight_triton_b200 import _native

        assert self.alive is not None, "call freeze_weight_mask() first"
        x2 = x.reshape(-1, self.in_features).contiguous()
        M = x2.shape[0]
        po = self._peer_out
        if po is None or po.rows < M:
            if po is not None:
                po.close()
            po = self._peer_out = PeerOutputs(M, self.out_features, x2.dtype, self.group)
            self._flag = torch.zeros(1, dtype=torch.int32, device=x2.device)
        i = self._peer_step % 2
        held = self._peer_returned[i]
        if held is not None and held() is not None:
            # Checked on every rank before any collective of this call, so a
            # refusal leaves the ranks in step (each rank holds its own output).
            raise RuntimeError(
                "the output this layer returned two calls ago is still referenced and its "
                "shared buffer would be overwritten now; clone() outputs kept across calls")
        self._peer_step += 1
        full = po.local(i)[:M]
        n_real = self.row_stop - self.row_start
        esize = full.element_size()
        bias = self.bias[:n_real] if self.bias is not None else None
        runs = self.strategy == "runs" and x2.data_ptr() % 16 == 0 and x2.stride(0) % 8 == 0
        _native.gather_gemm_peers(x2, self._packed_weight()[:n_real], self.alive,
                                  full[:, self.row_start:self.row_stop],
                                  po.peer_addresses(i, self.row_start * esize), bias=bias,
                                  strategy="runs" if runs else "pregather")
        # Orders every rank's readers of `full` after every rank's GEMM (and its
        # peer stores): each rank joins only after its own GEMM on this stream.
        dist.all_reduce(self._flag, group=self.group)
        out = full.reshape(*lead, self.out_features) if lead else full
        self._peer_returned[i] = weakref.ref(out)
        return out

    def close(self) -> None:
        """Release the shared output buffers (collective when gather_output="peers")."""
        if self._peer_out is not None:
            self._peer_out.close()
            self._peer_out = None
