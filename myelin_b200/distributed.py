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
