"""Neuron parameter and state dataclasses, field-for-field as the reference.

Mirrors ``LIFParams``/``LIFState``/``ALIFParams``/``ALIFState`` of
src/myelin/neurons.py:15-71 (same names, fields, defaults and derived decay
properties) so that user code constructing them is unchanged. The dynamics
themselves run in the CUDA scan (``myelin_b200.kernels``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class LIFParams:
    """Leaky integrate-and-fire parameters (src/myelin/neurons.py:15-29)."""

    tau_mem: float = 20.0
    threshold: float = 1.0
    reset: float = 0.0

    @property
    def decay(self) -> float:
        """Per-step membrane decay ``1 - 1 / tau_mem`` (computed in double)."""

        if self.tau_mem <= 0:
            raise ValueError("tau_mem must be positive")
        return 1.0 - (1.0 / self.tau_mem)


@dataclass(frozen=True)
class LIFState:
    """LIF state carried between steps (src/myelin/neurons.py:32-36)."""

    membrane: torch.Tensor


@dataclass(frozen=True)
class ALIFParams:
    """Adaptive LIF parameters (src/myelin/neurons.py:39-63)."""

    tau_mem: float = 20.0
    tau_adaptation: float = 100.0
    threshold: float = 1.0
    reset: float = 0.0
    beta: float = 1.0

    @property
    def decay(self) -> float:
        if self.tau_mem <= 0:
            raise ValueError("tau_mem must be positive")
        return 1.0 - (1.0 / self.tau_mem)

    @property
    def adaptation_decay(self) -> float:
        if self.tau_adaptation <= 0:
            raise ValueError("tau_adaptation must be positive")
        return 1.0 - (1.0 / self.tau_adaptation)


@dataclass(frozen=True)
class ALIFState:
    """ALIF state carried between steps (src/myelin/neurons.py:66-71)."""

    membrane: torch.Tensor
    adaptation: torch.Tensor


@dataclass(frozen=True)
class IzhikevichParams:
    """Izhikevich-style neuron parameters (src/myelin/neurons.py:74-96).

    Defaults are the regular-spiking configuration of the discrete model;
    ``dt`` scales both the voltage and the recovery update.
    """

    recovery_decay: float = 0.02
    recovery_coupling: float = 0.2
    reset_voltage: float = -65.0
    recovery_jump: float = 8.0
    threshold: float = 30.0
    dt: float = 1.0
    voltage_square_coeff: float = 0.04
    voltage_coeff: float = 5.0
    voltage_bias: float = 140.0

    def validate(self) -> None:
        """Validate the scalar parameters (src/myelin/neurons.py:91-95)."""

        if self.dt <= 0:
            raise ValueError("dt must be positive")


@dataclass(frozen=True)
class IzhikevichState:
    """Izhikevich state carried between steps (src/myelin/neurons.py:98-103)."""

    voltage: torch.Tensor
    recovery: torch.Tensor
