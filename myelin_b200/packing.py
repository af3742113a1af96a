"""Bit-packed spike tensors, API-compatible with ``myelin.packing``.

Same ``PackedSpikes`` dataclass and word format as src/myelin/packing.py:18-273:
int32 words along the last dimension, bit j of word w = element 32*w + j
(LSB first), zero padding, nonzero input = spike. Packing, unpacking and
counting run in the CUDA kernels of ``libmyelin_b200`` (``mb_pack_spikes``,
``mb_unpack_spikes``, ``mb_count_rows``, ``mb_count_columns``); the small
metadata helpers (sizes, byte counts) work on any device.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import TypeAlias

import torch

from myelin_b200 import _native as nat
from myelin_b200 import compile_ops as cops

BITS_PER_WORD = 32
CountDim: TypeAlias = int | Sequence[int] | None


@dataclass(frozen=True)
class PackedSpikes:
    """Spike tensor packed into signed int32 words along the last dimension."""

    data: torch.Tensor
    original_shape: tuple[int, ...]

    @property
    def packed_shape(self) -> tuple[int, ...]:
        return tuple(self.data.shape)

    @property
    def original_numel(self) -> int:
        numel = 1
        for size in self.original_shape:
            numel *= size
        return numel


def packed_last_dim_size(size: int) -> int:
    """Number of int32 words that hold ``size`` spikes."""

    if size < 0:
        raise ValueError("size must be non-negative")
    return (size + BITS_PER_WORD - 1) // BITS_PER_WORD


def _rows(shape: Sequence[int]) -> int:
    rows = 1
    for size in shape[:-1]:
        rows *= size
    return rows


def pack_spikes(spikes: torch.Tensor) -> PackedSpikes:
    """Pack binary spikes into int32 words along the last dimension.

    Inputs may be bool, integer or floating CUDA tensors; nonzero values are
    spikes (src/myelin/packing.py:45-71).
    """

    if spikes.ndim == 0:
        raise ValueError("spikes must have at least one dimension")
    if spikes.shape[-1] == 0:
        raise ValueError("cannot pack an empty last dimension")
    nat.require_cuda(spikes, "spikes")
    original_shape = tuple(spikes.shape)
    n = original_shape[-1]
    words = cops.pack(spikes.contiguous(), _rows(original_shape), n)
    words = words.view(*original_shape[:-1], packed_last_dim_size(n))
    return PackedSpikes(data=words, original_shape=original_shape)


def pack_spikes_with_counts(
    spikes: torch.Tensor, *, dtype: torch.dtype = torch.int64
) -> tuple[PackedSpikes, torch.Tensor]:
    """``pack_spikes(spikes)`` and its per-neuron counts over every leading dimension.

    Equals ``(p, packed_spike_counts_over_leading_dims(p, dtype=dtype))`` for
    ``p = pack_spikes(spikes)``, computed in one pass over the spikes for
    aligned 1-byte inputs (bool / uint8 / int8) whose last dimension is a
    multiple of 32 — the step before a packed all-gather and a count
    all-reduce (src/myelin/distributed.py:63-109). Not in the reference API.
    """

    if spikes.ndim == 0:
        raise ValueError("spikes must have at least one dimension")
    if spikes.shape[-1] == 0:
        raise ValueError("cannot pack an empty last dimension")
    if dtype not in (torch.int64, torch.int32):
        raise ValueError("dtype must be torch.int64 or torch.int32")
    nat.require_cuda(spikes, "spikes")
    original_shape = tuple(spikes.shape)
    n = original_shape[-1]
    words, counts = cops.pack_count(spikes.contiguous(), _rows(original_shape), n,
                                    wide=dtype == torch.int64)
    words = words.view(*original_shape[:-1], packed_last_dim_size(n))
    return PackedSpikes(data=words, original_shape=original_shape), counts


def unpack_spikes(packed: PackedSpikes, *, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Unpack to the original shape with 0/1 values of ``dtype``."""

    _validate_packed_spikes(packed)
    nat.require_cuda(packed.data, "packed.data")
    out = cops.unpack(packed.data.contiguous(), _rows(packed.original_shape),
                      packed.original_shape[-1], dtype)
    return out.view(packed.original_shape)


def _row_counts(packed: PackedSpikes) -> torch.Tensor:
    _validate_packed_spikes(packed)
    nat.require_cuda(packed.data, "packed.data")
    lead = packed.original_shape[:-1]
    counts = cops.count_rows(packed.data.contiguous(), _rows(packed.original_shape),
                             packed.original_shape[-1])
    return counts.view(lead)


def packed_spike_counts_over_leading_dims(
    packed: PackedSpikes, *, dtype: torch.dtype = torch.int64
) -> torch.Tensor:
    """Per-neuron counts over every leading dimension: shape ``[N]``.

    ``dtype`` is ``torch.int64`` (the reference's result type) or
    ``torch.int32`` (the compact form used on the wire for all-reduce).
    """

    _validate_packed_spikes(packed)
    nat.require_cuda(packed.data, "packed.data")
    n = packed.original_shape[-1]
    if dtype not in (torch.int64, torch.int32):
        raise ValueError("dtype must be torch.int64 or torch.int32")
    return cops.count_columns(packed.data.contiguous(), _rows(packed.original_shape), n,
                              wide=dtype == torch.int64)


def packed_spike_count(packed: PackedSpikes, dim: CountDim = None) -> torch.Tensor:
    """Spike counts with dense-like reduction semantics (src/myelin/packing.py:84-107)."""

    if dim is None:
        return packed_spike_counts(packed, dim=None)
    ndim = len(packed.original_shape)
    dims = _normalize_count_dims(dim, ndim=ndim)
    if ndim - 1 not in dims:
        if set(dims) == set(range(ndim - 1)):
            return packed_spike_counts_over_leading_dims(packed)
        dense = unpack_spikes(packed, dtype=torch.float32)
        return dense.sum(dim=tuple(dims)).to(torch.int64)
    return packed_spike_counts(packed, dim=dims)


def packed_spike_counts(packed: PackedSpikes, dim: CountDim = -1) -> torch.Tensor:
    """Counts from packed words; ``dim`` must include the last dimension (or be None)."""

    if dim is None:
        return _row_counts(packed).sum()
    dims = _normalize_count_dims(dim, ndim=len(packed.original_shape))
    last = len(packed.original_shape) - 1
    if last not in dims:
        raise ValueError(
            "packed_spike_counts requires reducing the packed/original last dimension; "
            "use packed_spike_count for dense-like reductions that keep that dimension"
        )
    row_counts = _row_counts(packed)
    remaining = tuple(index for index in dims if index != last)
    if not remaining:
        return row_counts
    return row_counts.sum(dim=remaining)


def packed_spike_rate(
    packed: PackedSpikes, dim: CountDim = None, *, dtype: torch.dtype = torch.float32
) -> torch.Tensor:
    """Mean spike activity (src/myelin/packing.py:145-162)."""

    counts = packed_spike_count(packed, dim=dim)
    dims = (
        tuple(range(len(packed.original_shape)))
        if dim is None
        else _normalize_count_dims(dim, ndim=len(packed.original_shape))
    )
    denominator = 1
    for index in dims:
        denominator *= packed.original_shape[index]
    return counts.to(dtype) / denominator


def _normalize_count_dims(dim: int | Sequence[int], *, ndim: int) -> tuple[int, ...]:
    raw = (dim,) if isinstance(dim, int) else tuple(dim)
    normalized: list[int] = []
    for d in raw:
        actual = d + ndim if d < 0 else d
        if actual < 0 or actual >= ndim:
            raise IndexError(f"dimension out of range: {d}")
        if actual in normalized:
            raise ValueError(f"duplicate reduction dimension: {d}")
        normalized.append(actual)
    return tuple(normalized)


def _validate_packed_spikes(packed: PackedSpikes) -> None:
    if packed.data.dtype != torch.int32:
        raise ValueError("packed.data must have dtype torch.int32")
    if len(packed.original_shape) == 0:
        raise ValueError("packed.original_shape must have at least one dimension")
    if packed.original_shape[-1] <= 0:
        raise ValueError("packed.original_shape must have non-empty last dimension")
    expected = (*packed.original_shape[:-1], packed_last_dim_size(packed.original_shape[-1]))
    if tuple(packed.data.shape) != expected:
        raise ValueError(
            "packed.data shape does not match packed.original_shape; "
            f"got {tuple(packed.data.shape)} and expected {expected}"
        )


def dense_spike_bytes(spikes: torch.Tensor) -> int:
    """Storage bytes of a dense spike tensor."""

    return spikes.numel() * spikes.element_size()


def packed_spike_bytes(packed: PackedSpikes) -> int:
    """Storage bytes of a packed spike tensor."""

    return packed.data.numel() * packed.data.element_size()


def spike_compression_ratio(spikes: torch.Tensor, packed: PackedSpikes) -> float:
    """Dense bytes divided by packed bytes."""

    packed_bytes = packed_spike_bytes(packed)
    if packed_bytes == 0:
        raise ValueError("packed representation has zero bytes")
    return dense_spike_bytes(spikes) / packed_bytes
