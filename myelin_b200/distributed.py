"""Collectives over packed spikes, API-compatible with ``myelin.distributed``.

One process per GPU with ``torch.distributed`` (NCCL over NVLink on B200,
gloo on CPU for tests). Differences from src/myelin/distributed.py:63-109 that
do not change results:

- the all-gather is one ``all_gather_into_tensor`` into a single
  ``[world, *packed_shape]`` buffer (the returned per-rank objects are views
  of it) instead of a list-form all_gather of separately allocated tensors;
- spike counts travel as int32 when the total cannot overflow it (half the
  bytes of the reference's int64) and are returned as int64 like the
  reference; per-neuron counts over all leading dims come straight out of the
  column-count kernel as int32.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist

from myelin_b200.packing import (
    CountDim,
    PackedSpikes,
    _normalize_count_dims,
    _validate_packed_spikes,
    packed_spike_count,
    packed_spike_counts_over_leading_dims,
)

_INT32_MAX = 2**31 - 1


def distributed_available_and_initialized() -> bool:
    """Whether ``torch.distributed`` can run collectives now."""

    return dist.is_available() and dist.is_initialized()


def _require_distributed_initialized() -> None:
    if not dist.is_available():
        raise RuntimeError("torch.distributed is not available")
    if not dist.is_initialized():
        raise RuntimeError("torch.distributed is not initialized")


def packed_spike_all_gather_into_tensor(
    packed: PackedSpikes,
    *,
    group: Any | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Gather every rank's packed words into one ``[world, *packed_shape]`` int32 tensor.

    ``out`` may be preallocated (e.g. reused across steps); every rank must
    contribute the same packed shape.
    """

    _validate_packed_spikes(packed)
    _require_distributed_initialized()
    world_size = dist.get_world_size(group=group)
    local = packed.data.contiguous()
    shape = (world_size, *local.shape)
    if out is None:
        out = torch.empty(shape, dtype=local.dtype, device=local.device)
    elif tuple(out.shape) != shape or out.dtype != local.dtype or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous int32 tensor of shape {shape}")
    # the concatenated [world * d0, ...] view of the same memory: the form every
    # backend accepts (NCCL also takes the stacked form, gloo does not)
    dist.all_gather_into_tensor(out.view(world_size * local.shape[0], *local.shape[1:]), local,
                                group=group)
    return out


def packed_spike_all_gather(
    packed: PackedSpikes,
    *,
    group: Any | None = None,
) -> list[PackedSpikes]:
    """All-gather packed spikes: one ``PackedSpikes`` per rank (src/myelin/distributed.py:63-80)."""

    gathered = packed_spike_all_gather_into_tensor(packed, group=group)
    return [PackedSpikes(data=gathered[r], original_shape=packed.original_shape)
            for r in range(gathered.shape[0])]


def _count_denominator(packed: PackedSpikes, dim: CountDim) -> int:
    if dim is None:
        return packed.original_numel
    dims = _normalize_count_dims(dim, ndim=len(packed.original_shape))
    denominator = 1
    for index in dims:
        denominator *= packed.original_shape[index]
    return denominator


def _packed_spike_count_for_collective(
    packed: PackedSpikes, dim: CountDim, group: Any | None = None
) -> torch.Tensor:
    """Local counts to be summed across ranks; int32 when every sum fits in int32."""

    world_size = dist.get_world_size(group=group)
    fits_int32 = _count_denominator(packed, dim) * world_size <= _INT32_MAX
    ndim = len(packed.original_shape)
    if dim is not None and fits_int32:
        dims = _normalize_count_dims(dim, ndim=ndim)
        if ndim > 1 and set(dims) == set(range(ndim - 1)):
            return packed_spike_counts_over_leading_dims(packed, dtype=torch.int32)
    counts = packed_spike_count(packed, dim=dim)
    return counts.to(torch.int32) if fits_int32 else counts


def packed_spike_count_all_reduce(
    packed: PackedSpikes,
    dim: CountDim = None,
    *,
    group: Any | None = None,
) -> torch.Tensor:
    """Spike counts summed across all ranks, int64 (src/myelin/distributed.py:83-94)."""

    _require_distributed_initialized()
    counts = _packed_spike_count_for_collective(packed, dim, group).contiguous()
    dist.all_reduce(counts, op=dist.ReduceOp.SUM, group=group)
    return counts.to(torch.int64)


def packed_spike_rate_all_reduce(
    packed: PackedSpikes,
    dim: CountDim = None,
    *,
    group: Any | None = None,
    dtype: torch.dtype = torch.float32,
) -> torch.Tensor:
    """Spike rates averaged over equally shaped ranks (src/myelin/distributed.py:97-109)."""

    counts = packed_spike_count_all_reduce(packed, dim=dim, group=group)
    world_size = dist.get_world_size(group=group)
    return counts.to(dtype) / (_count_denominator(packed, dim) * world_size)


class _DeviceArray:
    """A raw device allocation seen by torch through ``__cuda_array_interface__``."""

    def __init__(self, address: int, shape: tuple[int, ...]) -> None:
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "typestr": "<i4", "data": (address, False),
            "strides": None, "version": 3,
        }


class PackedSpikeExchange:
    """One step of packed-spike exchange fused over NVLink peer memory.

    ``pack_count_all_gather(spikes)`` packs this rank's spikes, counts spikes
    per neuron, and writes the packed words straight into this rank's slot of
    every rank's gather buffer (peer stores over NVLink / NVSwitch, inside the
    packing kernel: the transfers overlap the packing), then all-reduces the
    counts. Returns the gathered words ``[world, *leading, ceil(N/32)]`` (the
    result of ``packed_spike_all_gather_into_tensor`` of every rank's
    ``pack_spikes``) and the summed per-neuron counts (the result of
    ``packed_spike_count_all_reduce(packed, dim=leading dims)``), the step of
    src/myelin/distributed.py:63-98 in one kernel plus one small all-reduce.

    The count all-reduce is also the completion barrier: a rank's all-reduce
    finishes only after every rank has entered it, i.e. after every rank's
    packing kernel (and all its peer stores) has finished. Gather buffers are
    allocated once per object (CUDA IPC, plain peer-to-peer memory, no switch-replicated mapping) and
    used alternately, so reads of a returned buffer that the caller enqueues
    on the current stream before its next call are ordered before any rank
    overwrites it (a rank writes that buffer again only after the next call's
    all-reduce, which waits for this rank's stream). Collective: every rank constructs the
    object with the same local spike shape and calls each method in the same
    order. ``close()`` releases the buffers (collective as well).
    """

    def __init__(self, local_shape: tuple[int, ...], *, device: torch.device | int | None = None,
                 group: Any = None, buffers: int = 2, native: Any = None) -> None:
        _require_distributed_initialized()
        from myelin_b200 import _native

        self._nat = native if native is not None else _native
        if len(local_shape) < 1 or local_shape[-1] <= 0:
            raise ValueError("local_shape must have a non-empty last dimension")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("PackedSpikeExchange supports up to 8 ranks (one NVLink domain)")
        self.local_shape = tuple(int(d) for d in local_shape)
        self.n = self.local_shape[-1]
        self.rows = 1
        for d in self.local_shape[:-1]:
            self.rows *= d
        self.words = (self.n + 31) // 32
        self.slot_bytes = self.rows * self.words * 4
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device) if not isinstance(device, int) else \
            torch.device("cuda", device)
        # the native layer may supply its own device context and raw-memory view
        # (tests run the host logic on CPU ranks with a stand-in)
        self._ctx = getattr(self._nat, "device_context", torch.cuda.device)
        view = getattr(self._nat, "device_view", None)
        self._view = view if view is not None else (
            lambda address, shape, dev: torch.as_tensor(_DeviceArray(address, shape), device=dev))
        self._own: list[int] = []
        self._opened: list[int] = []
        self._slots: list[tuple[int, list[int]]] = []  # (own slot, peer slots) per buffer
        self._views: list[torch.Tensor] = []
        handles = []
        with self._ctx(self.device):
            for _ in range(buffers):
                address, handle = self._nat.ipc_alloc(self.world * self.slot_bytes)
                self._own.append(address)
                handles.append(handle)
        gathered: list[Any] = [None] * self.world
        dist.all_gather_object(gathered, (self.rank, self.local_shape, handles), group=group)
        for r, (rr, shape, _) in enumerate(gathered):
            if rr != r or tuple(shape) != self.local_shape:
                raise ValueError("every rank must build PackedSpikeExchange with the same shape")
        with self._ctx(self.device):
            for i in range(buffers):
                peers = []
                for r in range(self.world):
                    if r != self.rank:
                        base = self._nat.ipc_open(gathered[r][2][i])
                        self._opened.append(base)
                        peers.append(base + self.rank * self.slot_bytes)
                self._slots.append((self._own[i] + self.rank * self.slot_bytes, peers))
                shape = (self.world, *self.local_shape[:-1], self.words)
                self._views.append(self._view(self._own[i], shape, self.device))
        self._step = 0

    def pack_count_all_gather(
        self, spikes: torch.Tensor, *, count_dtype: torch.dtype = torch.int64
    ) -> tuple[torch.Tensor, torch.Tensor]:
        if tuple(spikes.shape) != self.local_shape:
            raise ValueError(f"spikes must be shaped {self.local_shape}; got {tuple(spikes.shape)}")
        if spikes.device != self.device:
            raise ValueError(f"spikes must be on {self.device}")
        if count_dtype not in (torch.int64, torch.int32):
            raise ValueError("count_dtype must be torch.int64 or torch.int32")
        i = self._step % len(self._slots)
        self._step += 1
        wide = self.rows * self.world > _INT32_MAX  # int32 on the wire when the sum fits
        counts = torch.empty((self.n,), dtype=torch.int64 if wide else torch.int32,
                             device=self.device)
        own, peers = self._slots[i]
        self._nat.pack_count_scatter(spikes.contiguous(), own, self.rows, self.n, peers,
                                     counts if wide else None, None if wide else counts)
        dist.all_reduce(counts, op=dist.ReduceOp.SUM, group=self.group)
        return self._views[i], counts.to(count_dtype)

    def lif_forward_packed_spikes(
        self, inputs: torch.Tensor, initial_state: Any, params: Any, *, reset_mode: str = "hard"
    ) -> tuple[Any, torch.Tensor]:
        """``kernels.lif_forward_packed_spikes`` feeding the all-gather directly.

        The scan writes its packed words straight into this rank's slot of
        its own gather buffer and a push kernel stores that slot into every
        peer's buffer over NVLink, all peers at once (src/myelin/kernels.py:96-156 followed by
        distributed.py:63-80, with no staging buffer and no NCCL all-gather).
        Returns the final ``LIFState`` and the gathered words ``[world, T, B,
        ceil(N/32)]``, which equal ``packed_spike_all_gather_into_tensor`` of
        every rank's packed output. A one-word all-reduce after the push
        completes the step (the same ordering argument as
        ``pack_count_all_gather``).
        """

        from myelin_b200 import _native as nat
        from myelin_b200 import kernels as K
        from myelin_b200.neurons import LIFState

        rc = K._reset_code(reset_mode)
        K._validate_scan(inputs, [("membrane", initial_state.membrane)])
        vT = self._scan_scatter(inputs.contiguous(), initial_state.membrane.contiguous(), params,
                                rc, nat.MB_LIF)
        return LIFState(membrane=vT), self._views[(self._step - 1) % len(self._slots)]

    def linear_surrogate_lif_packed_forward(
        self,
        inputs: torch.Tensor,
        weight: torch.Tensor,
        bias: torch.Tensor | None,
        params: Any,
        *,
        surrogate: str = "atan",
        surrogate_slope: float = 10.0,
        hard_forward: bool = True,
        checkpoint_size: Any = 25,
    ) -> tuple[Any, torch.Tensor]:
        """``kernels.linear_surrogate_lif_packed_forward`` feeding the all-gather
        directly: the projection, then the packed scan into this rank's slot
        and the copies to every peer (src/myelin/kernels.py:705-776 followed
        by distributed.py:63-80). Forward only, like the reference's packed
        path. Returns the final ``LIFState`` and the gathered words."""

        from myelin_b200 import _native as nat
        from myelin_b200 import kernels as K
        from myelin_b200.autograd import _project
        from myelin_b200.checkpointing import resolve_checkpoint_size
        from myelin_b200.neurons import LIFState
        from myelin_b200.surrogates import surrogate_id

        surrogate_id(surrogate)
        resolve_checkpoint_size(int(inputs.shape[0]), checkpoint_size)
        K._hard_forward_only(hard_forward, "packed surrogate LIF")
        K._validate_linear(inputs, weight, bias)
        with torch.no_grad():
            T, B, F = inputs.shape
            N = weight.shape[1]
            x2 = inputs.contiguous().reshape(T * B, F)
            currents = _project(x2, weight.contiguous(), bias).view(T, B, N)
            v0 = torch.zeros((B, N), dtype=inputs.dtype, device=inputs.device)
            vT = self._scan_scatter(currents, v0, params, nat.MB_RESET_HARD, nat.MB_LIF)
        return LIFState(membrane=vT), self._views[(self._step - 1) % len(self._slots)]

    def _scan_scatter(self, x: torch.Tensor, v0: torch.Tensor, params: Any, reset_mode: int,
                      neuron: int) -> torch.Tensor:
        if tuple(x.shape) != self.local_shape:
            raise ValueError(f"spikes must be shaped {self.local_shape}; got {tuple(x.shape)}")
        if x.device != self.device:
            raise ValueError(f"inputs must be on {self.device}")
        i = self._step % len(self._slots)
        self._step += 1
        own, peers = self._slots[i]
        vT = torch.empty_like(v0)
        self._nat.scan_forward_packed_scatter(
            neuron=neuron, x=x, v0=v0, a0=None, vT=vT, aT=None, packed=own, peers=peers,
            decay=params.decay, threshold=float(params.threshold), reset=float(params.reset),
            adapt_decay=0.0, beta=0.0, reset_mode=reset_mode,
        )
        # completion: no rank's all-reduce ends before every rank's kernel has
        flag = torch.zeros((1,), dtype=torch.int32, device=self.device)
        dist.all_reduce(flag, group=self.group)
        return vT

    def close(self) -> None:
        """Unmap the peers' buffers, wait for every rank, free this rank's."""

        if not self._own:
            return
        # kernels still queued on this device may be storing into the peer
        # mappings: let them finish before the mappings go away
        sync = getattr(self._nat, "device_synchronize", None)
        if sync is not None:
            sync(self.device)
        else:
            torch.cuda.synchronize(self.device)
        for address in self._opened:
            self._nat.ipc_close(address)
        self._opened = []
        self._views = []
        dist.barrier(group=self.group)
        for address in self._own:
            self._nat.ipc_free(address)
        self._own = []
