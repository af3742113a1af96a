"""Checkpoint-size policy (src/myelin/checkpointing.py:8-60), same names and values.

``checkpoint_size`` bounds how many time steps the backward replays from one
saved state. The CUDA scan always saves a state every ``MB_SCAN_CHUNK`` (16)
steps and replays at most that many in registers, which needs no more memory
than any policy below for T >= 16 and never stores a per-step trace.
"""

from __future__ import annotations

import math
from typing import Literal, TypeAlias

CheckpointPolicy: TypeAlias = Literal["memory", "balanced", "speed"]
CheckpointSize: TypeAlias = int | CheckpointPolicy
_POLICIES = frozenset(("memory", "balanced", "speed"))


def recommended_checkpoint_size(timesteps: int, *, policy: CheckpointPolicy = "balanced") -> int:
    """``memory`` = ceil(sqrt(T)), ``balanced`` = ceil(T/4), ``speed`` = ceil(T/2), clamped to [1, T]."""

    if timesteps <= 0:
        raise ValueError("timesteps must be positive")
    if policy == "memory":
        size = math.ceil(math.sqrt(timesteps))
    elif policy == "balanced":
        size = math.ceil(timesteps / 4)
    elif policy == "speed":
        size = math.ceil(timesteps / 2)
    else:
        raise ValueError("policy must be 'memory', 'balanced', or 'speed'")
    return max(1, min(timesteps, size))


def resolve_checkpoint_size(timesteps: int, checkpoint_size: CheckpointSize) -> int:
    """Concrete chunk size from a positive int or a named policy."""

    if isinstance(checkpoint_size, int):
        if checkpoint_size <= 0:
            raise ValueError("checkpoint_size must be positive")
        return min(checkpoint_size, timesteps)
    return recommended_checkpoint_size(timesteps, policy=checkpoint_size)


def parse_checkpoint_size(value: str) -> CheckpointSize:
    """Parse a positive integer or a policy name."""

    if value in _POLICIES:
        return value  # type: ignore[return-value]
    try:
        size = int(value)
    except ValueError as exc:
        expected = ", ".join(sorted(_POLICIES))
        raise ValueError(
            f"checkpoint_size must be a positive integer or one of: {expected}"
        ) from exc
    if size <= 0:
        raise ValueError("checkpoint_size must be positive")
    return size
