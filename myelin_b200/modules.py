"""nn.Module API of the hot path, constructor-compatible with ``myelin.modules``.

Mirrors LinearSynapse, the LIF/ALIF cells, TimeUnroll, LinearLIF,
LinearSurrogateLIF, LinearSurrogateLIFRate, RateReadoutClassifier and
LinearSurrogateLIFPacked of src/myelin/modules.py (same constructor
arguments, parameter names, shapes and default initialisation). Every
time-unrolled forward runs the CUDA scan; a single cell step is a scan of
length one.
"""

from __future__ import annotations

from typing import Literal

import torch
from torch import nn

from myelin_b200.checkpointing import CheckpointSize
from myelin_b200.kernels import (
    izhikevich_step,
    Backend,
    alif_forward,
    linear_surrogate_lif_forward,
    linear_surrogate_lif_packed_forward,
    linear_surrogate_lif_rate_forward,
    lif_forward,
    surrogate_alif_forward,
    surrogate_lif_forward,
)
from myelin_b200.neurons import (
    ALIFParams,
    ALIFState,
    IzhikevichParams,
    IzhikevichState,
    LIFParams,
    LIFState,
)
from myelin_b200.packing import PackedSpikes
from myelin_b200.surrogates import (
    SurrogateFn,
    atan_surrogate,
    fast_sigmoid_surrogate,
    surrogate_name,
)


class LinearSynapse(nn.Module):
    """Trainable dense projection over time-major inputs (src/myelin/modules.py:112-133).

    ``weight`` is ``[in_features, out_features]`` and the projection is
    ``inputs @ weight + bias``.
    """

    def __init__(
        self,
        in_features: int,
        out_features: int,
        params: LIFParams | None = None,
        bias: bool = True,
    ) -> None:
        super().__init__()
        self.weight = nn.Parameter((torch.rand((in_features, out_features)) - 0.5) * 0.02)
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.register_parameter("bias", None)

    def forward(self, inputs: torch.Tensor) -> torch.Tensor:
        output = torch.matmul(inputs, self.weight)
        if self.bias is not None:
            output = output + self.bias
        return output


class LIFCell(nn.Module):
    """Single-step hard-reset LIF population."""

    def __init__(self, params: LIFParams | None = None) -> None:
        super().__init__()
        self.params = params or LIFParams()

    def forward(self, state: LIFState, input_current: torch.Tensor) -> tuple[LIFState, torch.Tensor]:
        if state.membrane.shape != input_current.shape:
            raise ValueError(
                "state.membrane and input_current must have the same shape; "
                f"got {tuple(state.membrane.shape)} and {tuple(input_current.shape)}"
            )
        new_state, spikes = lif_forward(input_current.unsqueeze(0), state, self.params)
        return new_state, spikes[0]


class ALIFCell(nn.Module):
    """Single-step adaptive LIF population."""

    def __init__(self, params: ALIFParams | None = None) -> None:
        super().__init__()
        self.params = params or ALIFParams()

    def forward(
        self, state: ALIFState, input_current: torch.Tensor
    ) -> tuple[ALIFState, torch.Tensor]:
        new_state, spikes = alif_forward(input_current.unsqueeze(0), state, self.params)
        return new_state, spikes[0]


class IzhikevichCell(nn.Module):
    """Single-step Izhikevich-style population (src/myelin/modules.py:175-208)."""

    def __init__(self, params: IzhikevichParams | None = None) -> None:
        super().__init__()
        self.params = params or IzhikevichParams()

    def forward(
        self, state: IzhikevichState, input_current: torch.Tensor
    ) -> tuple[IzhikevichState, torch.Tensor]:
        return izhikevich_step(state, input_current, self.params)


class SurrogateLIFCell(nn.Module):
    """Single-step LIF with hard-forward surrogate-gradient spikes (src/myelin/modules.py:211-239)."""

    def __init__(
        self,
        params: LIFParams | None = None,
        surrogate: SurrogateFn = atan_surrogate,
        surrogate_slope: float = 10.0,
        hard_forward: bool = True,
    ) -> None:
        super().__init__()
        self.params = params or LIFParams()
        self.surrogate = surrogate
        self.surrogate_slope = surrogate_slope
        self.hard_forward = hard_forward

    def forward(self, state: LIFState, input_current: torch.Tensor) -> tuple[LIFState, torch.Tensor]:
        new_state, spikes = surrogate_lif_forward(
            input_current.unsqueeze(0),
            state,
            self.params,
            surrogate=surrogate_name(self.surrogate),
            surrogate_slope=self.surrogate_slope,
            hard_forward=self.hard_forward,
        )
        return new_state, spikes[0]


class SurrogateALIFCell(nn.Module):
    """Single-step ALIF with hard-forward surrogate-gradient spikes (src/myelin/modules.py:242-272)."""

    def __init__(
        self,
        params: ALIFParams | None = None,
        surrogate: SurrogateFn = atan_surrogate,
        surrogate_slope: float = 10.0,
        hard_forward: bool = True,
    ) -> None:
        super().__init__()
        self.params = params or ALIFParams()
        self.surrogate = surrogate
        self.surrogate_slope = surrogate_slope
        self.hard_forward = hard_forward

    def forward(
        self, state: ALIFState, input_current: torch.Tensor
    ) -> tuple[ALIFState, torch.Tensor]:
        new_state, spikes = surrogate_alif_forward(
            input_current.unsqueeze(0),
            state,
            self.params,
            surrogate=surrogate_name(self.surrogate),
            surrogate_slope=self.surrogate_slope,
            hard_forward=self.hard_forward,
        )
        return new_state, spikes[0]


class TimeUnroll(nn.Module):
    """Apply a cell across ``[T, B, N]`` inputs in one fused scan (src/myelin/modules.py:415-582)."""

    def __init__(self, cell: nn.Module, *, backend: Backend = "torch") -> None:
        super().__init__()
        self.cell = cell
        self.backend: Backend = backend

    def forward(
        self,
        inputs: torch.Tensor,
        initial_state: LIFState | ALIFState | None = None,
    ) -> tuple[LIFState | ALIFState, torch.Tensor]:
        cell = self.cell
        alif = isinstance(cell, ALIFCell | SurrogateALIFCell)
        if initial_state is None:
            zeros = torch.zeros(inputs.shape[1:], dtype=inputs.dtype, device=inputs.device)
            if alif:
                initial_state = ALIFState(membrane=zeros, adaptation=torch.zeros_like(zeros))
            else:
                initial_state = LIFState(membrane=zeros)
        if isinstance(cell, LIFCell):
            if not isinstance(initial_state, LIFState):
                raise TypeError("LIFCell requires LIFState")
            return lif_forward(inputs, initial_state, cell.params, backend=self.backend)
        if isinstance(cell, ALIFCell):
            if not isinstance(initial_state, ALIFState):
                raise TypeError("ALIFCell requires ALIFState")
            return alif_forward(inputs, initial_state, cell.params, backend=self.backend)
        if isinstance(cell, SurrogateALIFCell):
            if not isinstance(initial_state, ALIFState):
                raise TypeError("SurrogateALIFCell requires ALIFState")
            return surrogate_alif_forward(
                inputs,
                initial_state,
                cell.params,
                surrogate=surrogate_name(cell.surrogate),
                surrogate_slope=cell.surrogate_slope,
                hard_forward=cell.hard_forward,
                backend=self.backend,
            )
        if isinstance(cell, SurrogateLIFCell):
            if not isinstance(initial_state, LIFState):
                raise TypeError("SurrogateLIFCell requires LIFState")
            return surrogate_lif_forward(
                inputs,
                initial_state,
                cell.params,
                surrogate=surrogate_name(cell.surrogate),
                surrogate_slope=cell.surrogate_slope,
                hard_forward=cell.hard_forward,
                backend=self.backend,
            )
        raise TypeError(f"TimeUnroll does not support cell type {type(cell).__name__}")


class LinearLIF(nn.Module):
    """``LinearSynapse`` followed by ``TimeUnroll(LIFCell)``."""

    def __init__(self, in_features: int, out_features: int, params: LIFParams | None = None) -> None:
        super().__init__()
        self.synapse = LinearSynapse(in_features, out_features)
        self.unroll = TimeUnroll(LIFCell(params))

    def forward(self, inputs: torch.Tensor) -> tuple[LIFState, torch.Tensor]:
        return self.unroll(self.synapse(inputs))


class LinearSurrogateLIF(nn.Module):
    """Dense projection plus surrogate LIF unroll (src/myelin/modules.py:706-750)."""

    def __init__(
        self,
        in_features: int,
        out_features: int,
        params: LIFParams | None = None,
        surrogate: SurrogateFn = atan_surrogate,
        surrogate_slope: float = 10.0,
        hard_forward: bool = True,
        bias: bool = True,
        backend: Backend = "torch",
        stream_synapse: bool = False,
        checkpoint_size: CheckpointSize | None = None,
    ) -> None:
        super().__init__()
        self.synapse = LinearSynapse(in_features, out_features, bias=bias)
        self.stream_synapse = stream_synapse
        self.checkpoint_size: CheckpointSize | None = checkpoint_size
        self.unroll = TimeUnroll(
            SurrogateLIFCell(params, surrogate, surrogate_slope, hard_forward), backend=backend
        )

    def forward(self, inputs: torch.Tensor) -> torch.Tensor:
        cell = self.unroll.cell
        if self.stream_synapse:
            _state, spikes = linear_surrogate_lif_forward(
                inputs,
                self.synapse.weight,
                self.synapse.bias,
                cell.params,
                surrogate=surrogate_name(cell.surrogate),
                surrogate_slope=cell.surrogate_slope,
                hard_forward=cell.hard_forward,
                backend=self.unroll.backend,
                checkpoint_size=self.checkpoint_size,
            )
            return spikes
        _state, spikes = self.unroll(self.synapse(inputs))
        return spikes


class LinearSurrogateLIFRate(nn.Module):
    """Dense projection plus surrogate LIF returning spike rates (src/myelin/modules.py:803-845)."""

    def __init__(
        self,
        in_features: int,
        out_features: int,
        params: LIFParams | None = None,
        surrogate: SurrogateFn = atan_surrogate,
        surrogate_slope: float = 10.0,
        hard_forward: bool = True,
        bias: bool = True,
        backend: Backend = "torch",
        checkpoint_size: CheckpointSize = 25,
        reduction: Literal["mean", "none"] = "none",
    ) -> None:
        super().__init__()
        self.synapse = LinearSynapse(in_features, out_features, bias=bias)
        self.cell = SurrogateLIFCell(params, surrogate, surrogate_slope, hard_forward)
        self.backend: Backend = backend
        self.checkpoint_size: CheckpointSize = checkpoint_size
        self.reduction: Literal["mean", "none"] = reduction

    def forward(self, inputs: torch.Tensor) -> torch.Tensor:
        _state, rates = linear_surrogate_lif_rate_forward(
            inputs,
            self.synapse.weight,
            self.synapse.bias,
            self.cell.params,
            surrogate=surrogate_name(self.cell.surrogate),
            surrogate_slope=self.cell.surrogate_slope,
            hard_forward=self.cell.hard_forward,
            backend=self.backend,
            checkpoint_size=self.checkpoint_size,
            reduction=self.reduction,
        )
        return rates


class RateReadoutClassifier(nn.Module):
    """Hidden streamed LIF layer plus a rate readout (src/myelin/modules.py:848-903)."""

    def __init__(
        self,
        in_features: int,
        hidden_features: int,
        out_features: int,
        params: LIFParams | None = None,
        *,
        surrogate: SurrogateFn = fast_sigmoid_surrogate,
        surrogate_slope: float = 5.0,
        hard_forward: bool = True,
        bias: bool = True,
        backend: Backend = "torch",
        checkpoint_size: CheckpointSize = 25,
        dropout: float = 0.0,
    ) -> None:
        super().__init__()
        self.hidden = LinearSurrogateLIF(
            in_features,
            hidden_features,
            params,
            surrogate=surrogate,
            surrogate_slope=surrogate_slope,
            hard_forward=hard_forward,
            bias=bias,
            backend=backend,
            stream_synapse=True,
            checkpoint_size=checkpoint_size,
        )
        self.dropout = nn.Dropout(dropout)
        self.output = LinearSurrogateLIFRate(
            hidden_features,
            out_features,
            params,
            surrogate=surrogate,
            surrogate_slope=surrogate_slope,
            hard_forward=hard_forward,
            bias=bias,
            backend=backend,
            checkpoint_size=checkpoint_size,
            reduction="none",
        )

    def forward(self, inputs: torch.Tensor) -> torch.Tensor:
        hidden_spikes = self.dropout(self.hidden(inputs))
        return self.output(hidden_spikes)


class LinearSurrogateLIFPacked(nn.Module):
    """Dense projection plus LIF returning bit-packed spikes, forward only (src/myelin/modules.py:906-943)."""

    def __init__(
        self,
        in_features: int,
        out_features: int,
        params: LIFParams | None = None,
        surrogate: SurrogateFn = atan_surrogate,
        surrogate_slope: float = 10.0,
        hard_forward: bool = True,
        bias: bool = True,
        backend: Backend = "torch",
        checkpoint_size: CheckpointSize = 25,
    ) -> None:
        super().__init__()
        self.synapse = LinearSynapse(in_features, out_features, bias=bias)
        self.cell = SurrogateLIFCell(params, surrogate, surrogate_slope, hard_forward)
        self.backend: Backend = backend
        self.checkpoint_size: CheckpointSize = checkpoint_size

    def forward(self, inputs: torch.Tensor) -> PackedSpikes:
        _state, packed = linear_surrogate_lif_packed_forward(
            inputs,
            self.synapse.weight,
            self.synapse.bias,
            self.cell.params,
            surrogate=surrogate_name(self.cell.surrogate),
            surrogate_slope=self.cell.surrogate_slope,
            hard_forward=self.cell.hard_forward,
            backend=self.backend,
            checkpoint_size=self.checkpoint_size,
        )
        return packed
