"""Surrogate spike functions: names, primitives and closed-form derivatives.

The six built-in surrogates of src/myelin/surrogates.py:18-152 with the same
public names. The primitives are the smooth functions a user passes to the
modules (``SurrogateLIFCell(surrogate=atan_surrogate)``); the CUDA backward
evaluates the closed-form derivative selected by the surrogate's id (the
numbering of src/myelin/triton/lif.py:356-370).
"""

from __future__ import annotations

import math
from collections.abc import Callable
from typing import Literal

import torch

SurrogateFn = Callable[[torch.Tensor], torch.Tensor]
SurrogateName = Literal[
    "sigmoid",
    "fast_sigmoid",
    "atan",
    "triangular",
    "superspike",
    "multi_gaussian",
]
SURROGATE_NAMES: tuple[SurrogateName, ...] = (
    "sigmoid",
    "fast_sigmoid",
    "atan",
    "triangular",
    "superspike",
    "multi_gaussian",
)
SURROGATE_IDS: dict[str, int] = {name: index for index, name in enumerate(SURROGATE_NAMES)}


def sigmoid_surrogate(centered: torch.Tensor) -> torch.Tensor:
    """Logistic sigmoid."""

    return torch.sigmoid(centered)


def fast_sigmoid_surrogate(centered: torch.Tensor) -> torch.Tensor:
    """Rational sigmoid ``(c / (1 + |c|) + 1) / 2``."""

    return 0.5 * (centered / (1.0 + centered.abs()) + 1.0)


def atan_surrogate(centered: torch.Tensor) -> torch.Tensor:
    """Arctangent sigmoid ``atan(pi c / 2) / pi + 1 / 2``."""

    return torch.atan(math.pi * centered / 2.0) / math.pi + 0.5


def triangular_surrogate(centered: torch.Tensor) -> torch.Tensor:
    """Triangle ``clamp(1 - |c|, 0, 1)``."""

    return (1.0 - centered.abs()).clamp(min=0.0, max=1.0)


def superspike_surrogate(centered: torch.Tensor) -> torch.Tensor:
    """Unclamped primitive ``c / (1 + |c|) + 1/2`` whose slope is ``1 / (1 + |c|)^2``."""

    return centered / (1.0 + centered.abs()) + 0.5


def _gauss_cdf(centered: torch.Tensor, mean: float, sigma: float) -> torch.Tensor:
    return 0.5 * (1.0 + torch.erf((centered - mean) / (math.sqrt(2.0) * sigma)))


def multi_gaussian_surrogate(centered: torch.Tensor) -> torch.Tensor:
    """CDF of the mixture ``0.6 N(0, 0.5) + 0.2 N(1, 1) + 0.2 N(-1, 1)``."""

    return (
        0.6 * _gauss_cdf(centered, 0.0, 0.5)
        + 0.2 * _gauss_cdf(centered, 1.0, 1.0)
        + 0.2 * _gauss_cdf(centered, -1.0, 1.0)
    )


def surrogate_derivative(centered: torch.Tensor, name: SurrogateName) -> torch.Tensor:
    """Derivative of a built-in surrogate with respect to ``centered``."""

    if name == "sigmoid":
        value = torch.sigmoid(centered)
        return value * (1.0 - value)
    if name == "fast_sigmoid":
        return 0.5 / (1.0 + centered.abs()).square()
    if name == "atan":
        return 0.5 / (1.0 + (math.pi / 2.0 * centered).square())
    if name == "triangular":
        return torch.where(centered.abs() < 1.0, -centered.sign(), torch.zeros_like(centered))
    if name == "superspike":
        return 1.0 / (1.0 + centered.abs()).square()
    if name == "multi_gaussian":
        inv_sqrt_2pi = 1.0 / math.sqrt(2.0 * math.pi)
        return (
            0.6 * (inv_sqrt_2pi / 0.5) * torch.exp(-0.5 * (centered / 0.5).square())
            + 0.2 * inv_sqrt_2pi * torch.exp(-0.5 * (centered - 1.0).square())
            + 0.2 * inv_sqrt_2pi * torch.exp(-0.5 * (centered + 1.0).square())
        )
    raise ValueError(f"unknown surrogate: {name}")


def hard_surrogate_spike(centered: torch.Tensor, surrogate: SurrogateFn) -> torch.Tensor:
    """Binary forward spike whose gradient is the surrogate's."""

    hard = (centered >= 0).to(centered.dtype)
    smooth = surrogate(centered)
    return hard + smooth - smooth.detach()


_BY_NAME: dict[str, SurrogateFn] = {
    "sigmoid": sigmoid_surrogate,
    "fast_sigmoid": fast_sigmoid_surrogate,
    "atan": atan_surrogate,
    "triangular": triangular_surrogate,
    "superspike": superspike_surrogate,
    "multi_gaussian": multi_gaussian_surrogate,
}


def surrogate_from_name(name: SurrogateName) -> SurrogateFn:
    """Return a surrogate function by its stable API name."""

    try:
        return _BY_NAME[name]
    except KeyError:
        raise ValueError(f"unknown surrogate: {name!r}; expected one of {SURROGATE_NAMES}") from None


def surrogate_name(surrogate: SurrogateFn) -> SurrogateName:
    """Return the stable API name of a built-in surrogate function."""

    for name, fn in _BY_NAME.items():
        if fn is surrogate:
            return name  # type: ignore[return-value]
    raise ValueError(
        "the CUDA surrogate backward supports only the built-in surrogate functions: "
        "sigmoid_surrogate, fast_sigmoid_surrogate, atan_surrogate, "
        "triangular_surrogate, superspike_surrogate, and multi_gaussian_surrogate."
    )


def surrogate_id(name: SurrogateName) -> int:
    """Kernel id of a surrogate name (src/myelin/triton/lif.py:356-370)."""

    try:
        return SURROGATE_IDS[name]
    except KeyError:
        raise ValueError(f"unknown surrogate: {name!r}; expected one of {SURROGATE_NAMES}") from None
