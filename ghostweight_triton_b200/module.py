"""GhostLinear: drop-in nn.Linear with dead-neuron (dead-column) sparsity on B200.

Mirrors ghostweight_triton/module.py:12-157 (same constructor, from_linear,
forward semantics, freeze/unfreeze, current_sparsity, mask_frozen, repr).
What changes underneath:

* no per-call ``weight.t().contiguous()`` (module.py:97): the alive columns of
  ``weight`` [N, K] are packed once into the K'-major operand W' and cached
  (frozen mode) or packed per call from the alive list (dynamic mode, reading
  only N*K' elements instead of transposing all N*K);
* dynamic mode runs the fused mask+compaction kernel K1 instead of
  dead_neuron_mask + torch.nonzero + cast (module.py:103-104), and by default
  (``sync_free = True``) never reads the alive count on the host: the packing,
  the gather and the GEMM read it on the device, so a dynamic-mask forward
  queues without a host synchronisation and can be captured in a CUDA graph.
  The dense-fallback choice (module.py:111-112) then uses the previous
  forward's sparsity once its count has reached the host (read without
  waiting), and ``current_sparsity`` reads the count when it is accessed.
  With ``sync_free = False`` the forward reads the count first, as the
  reference does;
* the bias add (module.py:116-117) is fused into the GEMM epilogue;
* a frozen alive list made of 64-column runs (a mask that kills whole blocks of
  input columns) is detected once, and the GEMM then loads those blocks of x
  directly (strategy "runs": no gather launch, no scratch).

Additions beyond the reference surface: ``freeze_weight_mask()`` freezes the
mask from the per-input-column |W| reduction (the weight-side dead-column
mask), ``from_conv1d`` wraps a transformers Conv1D, ``activation`` fuses a GELU
into the epilogue, and the frozen index list survives state_dict round trips.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ghostweight_triton_b200 import _native
from ghostweight_triton_b200.kernels.gather import pack_weight, pack_weight_dev
from ghostweight_triton_b200.kernels.mask import dead_neuron_mask_compact, alive_indices as _alive
from ghostweight_triton_b200.kernels.matmul import ghost_linear, ghost_linear_dev, index_runs

_ACTIVATIONS = (None, "gelu", "gelu_tanh")


_SM_COUNT: dict[int, int] = {}


def _one_wave(K: int, N: int, device: torch.device) -> bool:
    """Whether gw_dynamic_linear's grid (ceil(N / 128) feature blocks x ceil(K / 512)
    ranks, one CTA per SM) runs in a single wave on this device."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    sms = _SM_COUNT.get(idx)
    if sms is None:
        sms = _SM_COUNT[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return -(-N // 128) * -(-K // 512) <= sms


class _CountReadback:
    """The last dynamic forward's alive count on its way to the host.

    An asynchronous copy into pinned memory and an event: ``ready()`` returns
    the count only if it has already landed (never waits), ``value()`` waits
    for it. Not copied by deepcopy (events and pinned buffers stay per module).
    """

    def __init__(self):
        self.host: torch.Tensor | None = None
        self.event: torch.cuda.Event | None = None
        self.dev: torch.Tensor | None = None

    def __deepcopy__(self, memo):
        return _CountReadback()

    def record(self, count: torch.Tensor) -> None:
        self.dev = count
        if torch.cuda.is_current_stream_capturing():
            self.event = None          # replays rewrite `count`; value() reads it then
            return
        if self.host is None:
            self.host = torch.empty(1, dtype=torch.int32).pin_memory()
            self.event = torch.cuda.Event()
        elif self.event is None:
            self.event = torch.cuda.Event()
        self.host.copy_(count, non_blocking=True)
        self.event.record()

    def ready(self) -> int | None:
        if self.event is None or self.host is None or torch.cuda.is_current_stream_capturing():
            return None
        return int(self.host[0]) if self.event.query() else None

    def value(self) -> int | None:
        if self.dev is None:
            return None
        if self.event is not None:
            self.event.synchronize()
            return int(self.host[0])
        return int(self.dev.item())


class GhostLinear(nn.Module):
    """Drop-in nn.Linear replacement with training-free inference sparsity.

    At inference time:
      1. Detects dead input neurons (|activation| <= threshold across the batch).
      2. If the dead fraction >= min_sparsity_to_activate: tcgen05 gather-GEMM
         over the alive columns only.
      3. Otherwise: dense F.linear (cuBLAS), as the reference does (module.py:111-112).

    Masking modes:
      Dynamic (default): recomputed every forward pass from the input.
      Frozen: computed once by freeze_mask(calibration) or freeze_weight_mask().

    Parameters
    ----------
    in_features, out_features, bias, device, dtype : as nn.Linear
    threshold : float
        Dead-neuron detection threshold (strict: alive iff max |x| > threshold).
    min_sparsity_to_activate : float
        Minimum dead fraction before the sparse path is used.
    activation : None | "gelu" | "gelu_tanh"
        Optional activation fused after the bias (extension; default None).
    """

    def __init__(
        self,
        in_features: int,
        out_features: int,
        bias: bool = True,
        threshold: float = 1e-6,
        min_sparsity_to_activate: float = 0.1,
        device=None,
        dtype=None,
        activation: str | None = None,
    ):
        super().__init__()
        if activation not in _ACTIVATIONS:
            raise ValueError(f"activation must be one of {_ACTIVATIONS}, got {activation!r}")
        self.in_features = in_features
        self.out_features = out_features
        self.threshold = threshold
        self.min_sparsity_to_activate = min_sparsity_to_activate
        self.activation = activation

        factory = {"device": device, "dtype": dtype}
        self.weight = nn.Parameter(torch.empty(out_features, in_features, **factory))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, **factory))
        else:
            self.register_parameter("bias", None)

        self.register_buffer("_frozen_indices", None)
        self._mask_frozen: bool = False
        self._last_sparsity: float = 0.0
        # (key, packed weight) for the frozen index list; rebuilt when the
        # weight, its dtype/device or the index list changes.
        self._packed: tuple[tuple, torch.Tensor] | None = None
        # (key, whether the frozen list is made of 64-column runs), same key rule.
        self._runs: tuple | None = None
        # Dynamic mode without host synchronisation (see the module docstring).
        self.sync_free: bool = True
        self._readback = _CountReadback()
        self._sparsity_pending = False

    # ------------------------------------------------------------------ construction
    @classmethod
    def from_linear(
        cls,
        linear: nn.Linear,
        threshold: float = 1e-6,
        min_sparsity_to_activate: float = 0.1,
    ) -> "GhostLinear":
        """Wrap an existing nn.Linear; weight and bias Parameters are shared, not copied."""
        ghost = cls(
            in_features=linear.in_features,
            out_features=linear.out_features,
            bias=linear.bias is not None,
            threshold=threshold,
            min_sparsity_to_activate=min_sparsity_to_activate,
            device=linear.weight.device,
            dtype=linear.weight.dtype,
        )
        ghost.weight = linear.weight
        if linear.bias is not None:
            ghost.bias = linear.bias
        return ghost

    @classmethod
    def from_conv1d(
        cls,
        conv: nn.Module,
        threshold: float = 1e-6,
        min_sparsity_to_activate: float = 0.1,
    ) -> "GhostLinear":
        """Wrap a transformers Conv1D (weight [in, out], y = x @ W + b).

        The GhostLinear weight is a transposed VIEW of the Conv1D weight (same
        storage, shape [out, in]); packing reads it with the transposing gather.
        """
        w = conv.weight
        in_f, out_f = w.shape
        ghost = cls(
            in_features=in_f,
            out_features=out_f,
            bias=conv.bias is not None,
            threshold=threshold,
            min_sparsity_to_activate=min_sparsity_to_activate,
            device=w.device,
            dtype=w.dtype,
        )
        ghost.weight = nn.Parameter(w.data.t(), requires_grad=w.requires_grad)
        if conv.bias is not None:
            ghost.bias = conv.bias
        return ghost

    # ------------------------------------------------------------------ forward
    def _weight_packed(self, alive: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        """W' for the frozen list, rebuilt when the weight (object, storage or an
        in-place update), the list or the dtype changes. The check is a few
        identity and integer compares, so a frozen forward pays no hashing."""
        w = self.weight
        c = self._packed
        if c is not None:
            k = c[0]
            if (k[0] is w and k[1] == w._version and k[2] == w.data_ptr() and k[3] is alive
                    and k[4] == alive._version and k[5] is dtype):
                return c[1]
        packed = pack_weight(w.detach(), alive, dtype=dtype)
        self._packed = ((w, w._version, w.data_ptr(), alive, alive._version, dtype), packed)
        return packed

    def _alive_runs(self, alive: torch.Tensor) -> bool:
        """Whether the frozen list is made of 64-column runs (checked once per list,
        which reads one count on the host; inside CUDA-graph capture an unchecked
        list takes the gather path instead)."""
        r = self._runs
        if r is None or r[0] is not alive or r[1] != alive._version:
            if torch.cuda.is_current_stream_capturing():
                return False
            r = self._runs = (alive, alive._version, index_runs(alive, self.in_features) == 0)
        return r[2]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x : [..., in_features] -> [..., out_features] (arbitrary batch dims)."""
        # Frozen mask, repeated call: everything the gather-GEMM needs was kept
        # by the last call (_fast), and is used again while the weight, bias
        # and alive list are the same tensors (same in-place versions and
        # storage), the mask is still frozen, and the input dtype, activation
        # and dense-fallback threshold are unchanged. The checks read the
        # module's dicts directly; a frozen small layer otherwise spends more
        # host time in attribute lookups than its kernels take on the GPU.
        d = self.__dict__
        fast = d.get("_fast")
        if fast is not None:
            (dtype, w, wv, wp, b, bv, bp, alive, av, act, min_sp, in_f, out_f,
             w_packed, bias_c, prep, sparsity) = fast
            params = d["_parameters"]
            if (x.dtype is dtype and d["_mask_frozen"] and d["_buffers"]["_frozen_indices"] is alive
                    and alive._version == av and params["weight"] is w and w._version == wv
                    and w.data_ptr() == wp and params.get("bias") is b
                    and (b is None or (b._version == bv and b.data_ptr() == bp))
                    and d.get("activation") == act and d["min_sparsity_to_activate"] == min_sp
                    and x.is_cuda and x.get_device() == torch.cuda.current_device()):
                shape = x.shape
                x_2d = x.reshape(-1, in_f)
                if not x_2d.is_contiguous():
                    x_2d = x_2d.contiguous()
                out = x_2d.new_empty((x_2d.shape[0], out_f))
                if x_2d.shape[0]:
                    _native.gather_gemm_prepared(prep, x_2d, out)
                d["_last_sparsity"] = sparsity
                return out.reshape(*shape[:-1], out_f)
            d["_fast"] = None
        orig_shape = x.shape
        x_2d = x.reshape(-1, self.in_features)
        assert x_2d.is_cuda, "GhostLinear runs on CUDA (sm_100) only"

        frozen = self._mask_frozen and self._frozen_indices is not None
        if not frozen and self.sync_free:
            return self._forward_sync_free(x_2d).reshape(*orig_shape[:-1], self.out_features)
        if frozen:
            alive = self._frozen_indices
            k_alive = alive.shape[0]
        else:
            _, buf, count = dead_neuron_mask_compact(x_2d, self.threshold, want_mask=False)
            k_alive = int(count.item())
            alive = buf[:k_alive]

        sparsity = 1.0 - k_alive / self.in_features
        self._last_sparsity = float(sparsity)

        bias = self.bias
        if bias is not None and bias.dtype is not x_2d.dtype:
            bias = bias.to(x_2d.dtype)
        if sparsity < self.min_sparsity_to_activate or k_alive == 0:
            out = F.linear(x_2d, self.weight.to(x_2d.dtype), bias)
            if self.activation is not None:
                out = F.gelu(out, approximate="tanh" if self.activation == "gelu_tanh" else "none")
        else:
            strategy = "auto"
            if frozen:
                w_packed = self._weight_packed(alive, x_2d.dtype)
                if x_2d.dtype is not torch.float32 and self._alive_runs(alive):
                    strategy = "runs"
            else:
                w_packed = pack_weight(self.weight.detach(), alive, dtype=x_2d.dtype)
            out = ghost_linear(x_2d, w_packed, alive, bias=bias, activation=self.activation,
                               strategy=strategy)
            if (frozen and not torch.cuda.is_current_stream_capturing()
                    and alive.dtype is torch.int64 and alive.is_contiguous()):
                w, b = self.weight, self.bias
                self.__dict__["_fast"] = (
                    x_2d.dtype, w, w._version, w.data_ptr(), b,
                    None if b is None else b._version, None if b is None else b.data_ptr(),
                    alive, alive._version, self.activation, self.min_sparsity_to_activate,
                    self.in_features, self.out_features, w_packed, bias,
                    _native.prepare_gather_gemm(w_packed, alive, bias, self.activation, strategy, x_2d.dtype),
                    float(sparsity))
        return out.reshape(*orig_shape[:-1], self.out_features)

    def _forward_sync_free(self, x_2d: torch.Tensor) -> torch.Tensor:
        """Dynamic-mask forward whose alive count never leaves the device."""
        bias = self.bias
        if bias is not None and bias.dtype != x_2d.dtype:
            bias = bias.to(x_2d.dtype)
        prev = self._readback.ready()           # the previous forward's count, if it has landed
        dense = prev is not None and 1.0 - prev / self.in_features < self.min_sparsity_to_activate
        if (not dense and x_2d.shape[0] <= 32 and x_2d.dtype in (torch.float16, torch.bfloat16)
                and _one_wave(self.in_features, self.out_features, x_2d.device)):
            # At most 32 rows: mask, compaction and the sparse product in one
            # launch (gw_dynamic_linear), reading x and W once. Taken where its
            # clusters run in one wave (every projection of GPT-2 and
            # DistilBERT); larger layers run the separate kernels, which were
            # faster there.
            w = self.weight.detach()
            if w.dtype is x_2d.dtype and w.stride(1) == 1 and x_2d.stride(1) == 1:
                y = torch.empty((x_2d.shape[0], self.out_features), dtype=x_2d.dtype, device=x_2d.device)
                count = torch.empty(1, dtype=torch.int32, device=x_2d.device)
                if _native.dynamic_linear(x_2d, w, self.threshold, y, bias=bias, activation=self.activation,
                                          count=count) == _native.GW_OK:
                    self._readback.record(count)
                    self._sparsity_pending = True
                    return y
        _, buf, count = dead_neuron_mask_compact(x_2d, self.threshold, want_mask=False)
        if dense:
            out = F.linear(x_2d, self.weight.to(x_2d.dtype), bias)
            if self.activation is not None:
                out = F.gelu(out, approximate="tanh" if self.activation == "gelu_tanh" else "none")
        else:
            w_packed = pack_weight_dev(self.weight.detach(), buf, count, dtype=x_2d.dtype)
            out = ghost_linear_dev(x_2d, w_packed, buf, count, bias=bias, activation=self.activation)
        self._readback.record(count)
        self._sparsity_pending = True
        return out

    # ------------------------------------------------------------------ masks
    def freeze_mask(self, calibration_input: torch.Tensor) -> None:
        """Freeze the dead-neuron mask from calibration activations; later calls reuse it."""
        with torch.no_grad():
            x_2d = calibration_input.reshape(-1, self.in_features)
            self._set_frozen(_alive(x_2d, self.threshold))

    def freeze_weight_mask(self) -> None:
        """Freeze the mask from the weight: input column k is dead iff max_n |W[n, k]| <= threshold.

        A dead weight column contributes exactly zero, so the output equals the
        dense layer's for every input.
        """
        with torch.no_grad():
            w = self.weight.detach()
            self._set_frozen(_alive(w if w.stride(1) == 1 else w.contiguous(), self.threshold))

    def _set_frozen(self, idx: torch.Tensor) -> None:
        self._frozen_indices = idx.to(torch.int64)
        self._mask_frozen = True
        self._packed = None
        self._runs = None
        self._sparsity_pending = False
        if (self._frozen_indices.is_cuda and self._frozen_indices.numel()
                and not torch.cuda.is_current_stream_capturing()):
            self._alive_runs(self._frozen_indices)     # decided now, not in the first forward
        k_alive = int(self._frozen_indices.numel())
        self._last_sparsity = float(1.0 - k_alive / self.in_features)

    def refresh_packed(self) -> None:
        """Rebuild the packed weight W' at the next forward.

        W' is kept between forwards and rebuilt by itself when the weight is
        replaced, moved to other storage (``weight.data = ...``) or updated in
        place through autograd-visible operations (optimizer steps, ``copy_``
        under ``no_grad``), which bump its version counter. In-place writes
        through ``weight.data`` bypass that counter; call this after them.
        """
        self._packed = None
        self.__dict__["_fast"] = None

    def unfreeze_mask(self) -> None:
        """Switch back to dynamic per-forward masking."""
        self._mask_frozen = False
        self._frozen_indices = None
        self._packed = None
        self._runs = None

    @property
    def current_sparsity(self) -> float:
        """Sparsity of the frozen mask, or of the most recent forward pass (a
        synchronisation-free forward's count is read here, on access)."""
        if self._sparsity_pending and not (self._mask_frozen and self._frozen_indices is not None):
            n = self._readback.value()
            if n is not None:
                self._last_sparsity = float(1.0 - n / self.in_features)
            # A count recorded during CUDA-graph capture is rewritten by every
            # replay: keep reading it.
            self._sparsity_pending = self._readback.event is None and self._readback.dev is not None
        return self._last_sparsity

    @property
    def mask_frozen(self) -> bool:
        return self._mask_frozen

    # ------------------------------------------------------------------ checkpointing
    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict,
                              missing_keys, unexpected_keys, error_msgs):
        key = prefix + "_frozen_indices"
        if key in state_dict and self._frozen_indices is None:
            idx = state_dict.pop(key)
            super()._load_from_state_dict(state_dict, prefix, local_metadata, strict,
                                          missing_keys, unexpected_keys, error_msgs)
            state_dict[key] = idx
            self._set_frozen(idx.to(self.weight.device))
            return
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict,
                                      missing_keys, unexpected_keys, error_msgs)
        if self._frozen_indices is not None:
            self._mask_frozen = True
            self._packed = None
            self._last_sparsity = float(1.0 - self._frozen_indices.numel() / self.in_features)

    def extra_repr(self) -> str:
        return (
            f"in={self.in_features}, out={self.out_features}, "
            f"bias={self.bias is not None}, "
            f"threshold={self.threshold}, "
            f"frozen={self._mask_frozen}, "
            f"sparsity={self._last_sparsity:.1%}"
        )
