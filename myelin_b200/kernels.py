"""Public fused-kernel entry points, signature-compatible with ``myelin.kernels``.

Every function keeps the reference's positional/keyword names and defaults
(src/myelin/kernels.py:52-865). ``backend`` and the Triton tile arguments
(``block_size``, ``block_b``, ``block_n``, ``block_f``) are accepted for
drop-in compatibility; every backend name the reference defines selects the
same hand-written sm_100a kernels. Tensors must be on a CUDA device: there is
no CPU fallback.

Extensions over the reference: ``reset_mode="subtract"`` (membrane minus the
(adaptive) threshold after a spike instead of a hard reset) on the LIF/ALIF
scans, ``checkpoint_size`` on ``surrogate_alif_forward``, and a backward for
``surrogate_alif_forward`` / ``alif_forward`` on the GPU.
"""

from __future__ import annotations

from typing import Literal

import torch

from myelin_b200 import _native as nat
from myelin_b200 import compile_ops as cops
from myelin_b200.autograd import (
    ALIFScanFunction,
    LIFScanFunction,
    LinearScanFunction,
    TwoLayerPackedHiddenRateFunction,
    _project,
)
from myelin_b200.checkpointing import CheckpointSize, resolve_checkpoint_size
from myelin_b200.neurons import (
    ALIFParams,
    ALIFState,
    IzhikevichParams,
    IzhikevichState,
    LIFParams,
    LIFState,
)
from myelin_b200.packing import PackedSpikes
from myelin_b200.surrogates import SurrogateName, surrogate_id

Backend = Literal["auto", "torch", "triton", "triton_generated", "triton_compile", "cuda"]
_BACKENDS = frozenset(("auto", "torch", "triton", "triton_generated", "triton_compile", "cuda"))
ResetMode = Literal["hard", "subtract"]


def _check_backend(backend: str) -> None:
    if backend not in _BACKENDS:
        raise ValueError(f"unsupported backend: {backend}")


def _reset_code(reset_mode: str) -> int:
    if reset_mode == "hard":
        return nat.MB_RESET_HARD
    if reset_mode == "subtract":
        return nat.MB_RESET_SUBTRACT
    raise ValueError("reset_mode must be 'hard' or 'subtract'")


def _validate_scan(inputs: torch.Tensor, states: list[tuple[str, torch.Tensor]]) -> None:
    """Validation order and messages of src/myelin/triton/lif.py:340-353."""

    if inputs.ndim != 3:
        raise ValueError(f"inputs must be shaped [T, B, N]; got {tuple(inputs.shape)}")
    for name, tensor in states:
        if tensor.shape != inputs.shape[1:]:
            raise ValueError(
                f"initial_state.{name} must match inputs.shape[1:]; "
                f"got {tuple(tensor.shape)} and {tuple(inputs.shape[1:])}"
            )
    nat.require_cuda(inputs)
    for name, tensor in states:
        if tensor.device != inputs.device:
            raise ValueError(f"initial_state.{name} must be on the same device as inputs")
        if tensor.dtype != inputs.dtype:
            raise ValueError(f"initial_state.{name} must have the same dtype as inputs")
    if inputs.dtype not in nat.SCAN_DTYPES:
        raise ValueError(
            f"inputs must be float32, bfloat16 or float16 for the CUDA scan; got {inputs.dtype}"
        )


def _hard_forward_only(hard_forward: bool, what: str) -> None:
    if not hard_forward:
        raise ValueError(f"{what} currently supports only hard_forward=True")


def lif_forward(
    inputs: torch.Tensor,
    initial_state: LIFState,
    params: LIFParams,
    *,
    backend: Backend = "auto",
    block_size: int = 256,
    reset_mode: ResetMode = "hard",
) -> tuple[LIFState, torch.Tensor]:
    """Fused-time LIF forward over ``[T, B, N]`` (src/myelin/kernels.py:52-93).

    Spikes are bit-exact with the reference's ``lif_unroll``. The backward
    supports gradients of the final membrane only, like the reference's fused
    path (src/myelin/autograd.py:44-101).
    """

    _check_backend(backend)
    rc = _reset_code(reset_mode)
    _validate_scan(inputs, [("membrane", initial_state.membrane)])
    vT, spikes = LIFScanFunction.apply(
        inputs.contiguous(),
        initial_state.membrane.contiguous(),
        params.decay,
        float(params.threshold),
        float(params.reset),
        rc,
        nat.MB_SURR_NONE,
        0.0,
        True,
    )
    return LIFState(membrane=vT), spikes


def fused_lif_unroll(
    inputs: torch.Tensor,
    initial_state: LIFState,
    params: LIFParams,
    *,
    backend: Backend = "auto",
    block_size: int = 256,
) -> tuple[LIFState, torch.Tensor]:
    """Compatibility alias for ``lif_forward`` (src/myelin/kernels.py:849-865)."""

    return lif_forward(inputs, initial_state, params, backend=backend, block_size=block_size)


def lif_forward_packed_spikes(
    inputs: torch.Tensor,
    initial_state: LIFState,
    params: LIFParams,
    *,
    backend: Backend = "auto",
    block_b: int = 8,
    reset_mode: ResetMode = "hard",
) -> tuple[LIFState, PackedSpikes]:
    """LIF forward writing int32 spike words directly (src/myelin/kernels.py:96-156).

    Forward-only, like the reference's fused packed path.
    """

    _check_backend(backend)
    rc = _reset_code(reset_mode)
    _validate_scan(inputs, [("membrane", initial_state.membrane)])
    x = inputs.contiguous()
    v0 = initial_state.membrane.contiguous()
    vT, _, _, words, _, _, _ = cops.scan_forward(
        x, v0, None, nat.MB_LIF, params.decay, float(params.threshold), float(params.reset),
        0.0, 0.0, rc, packed=True,
    )
    return LIFState(membrane=vT), PackedSpikes(data=words, original_shape=tuple(x.shape))


def alif_forward(
    inputs: torch.Tensor,
    initial_state: ALIFState,
    params: ALIFParams,
    *,
    backend: Backend = "auto",
    block_size: int = 256,
    reset_mode: ResetMode = "hard",
) -> tuple[ALIFState, torch.Tensor]:
    """Fused-time ALIF forward (src/myelin/kernels.py:159-199).

    Spikes are bit-exact with ``alif_unroll``. Like the reference's torch
    path, spikes carry no gradient; final-state gradients flow through the
    membrane and adaptation recurrences.
    """

    _check_backend(backend)
    rc = _reset_code(reset_mode)
    _validate_scan(
        inputs,
        [("membrane", initial_state.membrane), ("adaptation", initial_state.adaptation)],
    )
    vT, aT, spikes = ALIFScanFunction.apply(
        inputs.contiguous(),
        initial_state.membrane.contiguous(),
        initial_state.adaptation.contiguous(),
        params.decay,
        float(params.threshold),
        float(params.reset),
        params.adaptation_decay,
        float(params.beta),
        rc,
        nat.MB_SURR_NONE,
        0.0,
    )
    return ALIFState(membrane=vT, adaptation=aT), spikes.detach()


def surrogate_lif_forward(
    inputs: torch.Tensor,
    initial_state: LIFState,
    params: LIFParams,
    *,
    surrogate: SurrogateName = "atan",
    surrogate_slope: float = 10.0,
    hard_forward: bool = True,
    backend: Backend = "auto",
    block_size: int = 256,
    checkpoint_size: CheckpointSize | None = None,
    reset_mode: ResetMode = "hard",
) -> tuple[LIFState, torch.Tensor]:
    """Hard-forward LIF with a surrogate-gradient backward (src/myelin/kernels.py:249-337)."""

    sid = surrogate_id(surrogate)
    _check_backend(backend)
    _hard_forward_only(hard_forward, "CUDA surrogate LIF")
    rc = _reset_code(reset_mode)
    _validate_scan(inputs, [("membrane", initial_state.membrane)])
    if checkpoint_size is not None:
        resolve_checkpoint_size(int(inputs.shape[0]) or 1, checkpoint_size)
    vT, spikes = LIFScanFunction.apply(
        inputs.contiguous(),
        initial_state.membrane.contiguous(),
        params.decay,
        float(params.threshold),
        float(params.reset),
        rc,
        sid,
        float(surrogate_slope),
        False,
    )
    return LIFState(membrane=vT), spikes


def surrogate_alif_forward(
    inputs: torch.Tensor,
    initial_state: ALIFState,
    params: ALIFParams,
    *,
    surrogate: SurrogateName = "atan",
    surrogate_slope: float = 10.0,
    hard_forward: bool = True,
    backend: Backend = "auto",
    checkpoint_size: CheckpointSize | None = None,
    reset_mode: ResetMode = "hard",
) -> tuple[ALIFState, torch.Tensor]:
    """Hard-forward ALIF with a surrogate-gradient backward on the GPU.

    The reference runs this only through torch autograd of
    ``surrogate_alif_unroll`` (src/myelin/kernels.py:340-392,
    src/myelin/functional.py:149-189); its adjoint is computed here in closed
    form with chunked replay.
    """

    sid = surrogate_id(surrogate)
    _check_backend(backend)
    _hard_forward_only(hard_forward, "CUDA surrogate ALIF")
    rc = _reset_code(reset_mode)
    _validate_scan(
        inputs,
        [("membrane", initial_state.membrane), ("adaptation", initial_state.adaptation)],
    )
    if checkpoint_size is not None:
        resolve_checkpoint_size(int(inputs.shape[0]) or 1, checkpoint_size)
    vT, aT, spikes = ALIFScanFunction.apply(
        inputs.contiguous(),
        initial_state.membrane.contiguous(),
        initial_state.adaptation.contiguous(),
        params.decay,
        float(params.threshold),
        float(params.reset),
        params.adaptation_decay,
        float(params.beta),
        rc,
        sid,
        float(surrogate_slope),
    )
    return ALIFState(membrane=vT, adaptation=aT), spikes


def _validate_linear(
    inputs: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None
) -> None:
    if inputs.ndim != 3:
        raise ValueError(f"inputs must be shaped [T, B, F]; got {tuple(inputs.shape)}")
    if weight.ndim != 2:
        raise ValueError(f"weight must be shaped [F, N]; got {tuple(weight.shape)}")
    if inputs.shape[2] != weight.shape[0]:
        raise ValueError("inputs.shape[2] must match weight.shape[0]")
    nat.require_cuda(inputs)
    if weight.device != inputs.device or weight.dtype != inputs.dtype:
        raise ValueError("weight must have the same device and dtype as inputs")
    if bias is not None:
        if bias.shape != (weight.shape[1],):
            raise ValueError("bias must be shaped [N]")
        if bias.device != inputs.device or bias.dtype != inputs.dtype:
            raise ValueError("bias must have the same device and dtype as inputs")
    if inputs.dtype not in nat.SCAN_DTYPES:
        raise ValueError(
            f"inputs must be float32, bfloat16 or float16 for the CUDA scan; got {inputs.dtype}"
        )


def linear_surrogate_lif_forward(
    inputs: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    params: LIFParams,
    *,
    surrogate: SurrogateName = "atan",
    surrogate_slope: float = 10.0,
    hard_forward: bool = True,
    backend: Backend = "auto",
    checkpoint_size: CheckpointSize | None = None,
    block_b: int = 16,
    block_n: int = 32,
    block_f: int = 32,
) -> tuple[LIFState, torch.Tensor]:
    """Dense projection + surrogate LIF (src/myelin/kernels.py:395-562).

    The membrane starts at zero (src/myelin/autograd.py:469-473). Gradients
    flow to inputs, weight and bias.
    """

    sid = surrogate_id(surrogate)
    _check_backend(backend)
    _hard_forward_only(hard_forward, "streamed LinearSurrogateLIF")
    if checkpoint_size is not None:
        resolve_checkpoint_size(int(inputs.shape[0]), checkpoint_size)
    _validate_linear(inputs, weight, bias)
    vT, spikes = LinearScanFunction.apply(
        inputs.contiguous(),
        weight.contiguous(),
        None if bias is None else bias.contiguous(),
        params.decay,
        float(params.threshold),
        float(params.reset),
        sid,
        float(surrogate_slope),
        False,
    )
    return LIFState(membrane=vT), spikes


def linear_surrogate_lif_rate_forward(
    inputs: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    params: LIFParams,
    *,
    surrogate: SurrogateName = "atan",
    surrogate_slope: float = 10.0,
    hard_forward: bool = True,
    backend: Backend = "auto",
    checkpoint_size: CheckpointSize = 25,
    block_b: int = 16,
    block_n: int = 32,
    block_f: int = 32,
    reduction: Literal["mean", "none"] = "mean",
) -> tuple[LIFState, torch.Tensor]:
    """Dense projection + surrogate LIF returning spike rates ``count / T``.

    Never materialises dense spikes (src/myelin/kernels.py:565-702).
    """

    sid = surrogate_id(surrogate)
    _check_backend(backend)
    resolve_checkpoint_size(int(inputs.shape[0]), checkpoint_size)
    _hard_forward_only(hard_forward, "checkpointed spike-rate LIF")
    if reduction not in {"mean", "none"}:
        raise ValueError("reduction must be 'mean' or 'none'")
    _validate_linear(inputs, weight, bias)
    vT, rates = LinearScanFunction.apply(
        inputs.contiguous(),
        weight.contiguous(),
        None if bias is None else bias.contiguous(),
        params.decay,
        float(params.threshold),
        float(params.reset),
        sid,
        float(surrogate_slope),
        True,
    )
    if reduction == "mean":
        return LIFState(membrane=vT), rates.mean()
    return LIFState(membrane=vT), rates


def _izhikevich_params(params: IzhikevichParams) -> list[float]:
    params.validate()
    return [float(getattr(params, k)) for k in cops.IZH_FIELDS]


def izhikevich_forward(
    inputs: torch.Tensor,
    initial_state: IzhikevichState,
    params: IzhikevichParams,
    *,
    backend: Backend = "auto",
    block_size: int = 256,
) -> tuple[IzhikevichState, torch.Tensor]:
    """Fused-time Izhikevich forward (src/myelin/kernels.py:202-246).

    Spikes and final states are bit-exact with ``izhikevich_unroll`` for
    fp32 inputs. Forward only, like the reference's generated kernel: no
    gradient flows through it. Every ``backend`` runs the CUDA kernel.
    """

    _check_backend(backend)
    values = _izhikevich_params(params)
    if inputs.ndim != 3:
        raise ValueError(f"inputs must be shaped [T, B, N]; got {tuple(inputs.shape)}")
    expected = inputs.shape[1:]
    for name, t in (("voltage", initial_state.voltage), ("recovery", initial_state.recovery)):
        if t.shape != expected:
            raise ValueError(
                f"initial_state.{name} must match inputs.shape[1:]; "
                f"got {tuple(t.shape)} and {tuple(expected)}"
            )
    nat.require_cuda(inputs)
    for name, t in (("voltage", initial_state.voltage), ("recovery", initial_state.recovery)):
        if t.device != inputs.device or t.dtype != inputs.dtype:
            raise ValueError(f"initial_state.{name} must have the same device and dtype as inputs")
    if inputs.dtype not in nat.SCAN_DTYPES:
        raise ValueError(
            f"inputs must be float32, bfloat16 or float16 for the CUDA scan; got {inputs.dtype}"
        )
    with torch.no_grad():
        vT, uT, spikes = cops.izhikevich_forward(
            inputs.contiguous(), initial_state.voltage.contiguous(),
            initial_state.recovery.contiguous(), values,
        )
    return IzhikevichState(voltage=vT, recovery=uT), spikes


def izhikevich_step(
    state: IzhikevichState, input_current: torch.Tensor, params: IzhikevichParams
) -> tuple[IzhikevichState, torch.Tensor]:
    """Advance one Izhikevich step (src/myelin/neurons.py:204-230), as a T=1 scan."""

    params.validate()
    for name, t in (("voltage", state.voltage), ("recovery", state.recovery)):
        if t.shape != input_current.shape:
            raise ValueError(
                f"state.{name} and input_current must have the same shape; "
                f"got {tuple(t.shape)} and {tuple(input_current.shape)}"
            )
    shape = input_current.shape
    flat = (1, 1, input_current.numel())
    new_state, spikes = izhikevich_forward(
        input_current.reshape(flat),
        IzhikevichState(state.voltage.reshape(flat[1:]), state.recovery.reshape(flat[1:])),
        params,
    )
    return (IzhikevichState(new_state.voltage.reshape(shape), new_state.recovery.reshape(shape)),
            spikes.reshape(shape))


def _two_layer_validate(inputs, hidden_weight, hidden_bias, output_weight, output_bias):
    _validate_linear(inputs, hidden_weight, hidden_bias)
    if output_weight.ndim != 2 or output_weight.shape[0] != hidden_weight.shape[1]:
        raise ValueError("output_weight must be shaped [hidden_features, output_features]")
    if output_bias is not None and tuple(output_bias.shape) != (output_weight.shape[1],):
        raise ValueError("output_bias must be shaped [output_features]")
    if output_weight.dtype != inputs.dtype or output_weight.device != inputs.device:
        raise ValueError("output_weight must match the inputs' dtype and device")


def two_layer_surrogate_lif_rate_recompute_forward(
    inputs: torch.Tensor,
    hidden_weight: torch.Tensor,
    hidden_bias: torch.Tensor | None,
    output_weight: torch.Tensor,
    output_bias: torch.Tensor | None,
    params: LIFParams,
    *,
    surrogate: SurrogateName = "fast_sigmoid",
    surrogate_slope: float = 5.0,
    hard_forward: bool = True,
    checkpoint_size: CheckpointSize = 25,
) -> torch.Tensor:
    """Two-layer LIF rate model with whole-model backward recompute.

    Same rates and gradients as the packed-hidden variant; between forward and
    backward only the inputs, parameters and the layers' fp32 chunk
    checkpoints are kept, and the backward regenerates the hidden spikes
    (src/myelin/kernels.py:779-808, src/myelin/autograd.py:926-1126).
    """

    sid = surrogate_id(surrogate)
    resolve_checkpoint_size(int(inputs.shape[0]), checkpoint_size)  # validates like the reference
    if not hard_forward:
        raise ValueError("two-layer recompute rate training supports only hard_forward=True")
    _two_layer_validate(inputs, hidden_weight, hidden_bias, output_weight, output_bias)
    return TwoLayerPackedHiddenRateFunction.apply(
        inputs.contiguous(),
        hidden_weight.contiguous(),
        None if hidden_bias is None else hidden_bias.contiguous(),
        output_weight.contiguous(),
        None if output_bias is None else output_bias.contiguous(),
        params.decay,
        float(params.threshold),
        float(params.reset),
        sid,
        float(surrogate_slope),
        False,
    )


def two_layer_surrogate_lif_rate_packed_hidden_forward(
    inputs: torch.Tensor,
    hidden_weight: torch.Tensor,
    hidden_bias: torch.Tensor | None,
    output_weight: torch.Tensor,
    output_bias: torch.Tensor | None,
    params: LIFParams,
    *,
    surrogate: SurrogateName = "fast_sigmoid",
    surrogate_slope: float = 5.0,
    hard_forward: bool = True,
    checkpoint_size: CheckpointSize = 25,
    block_b: int = 16,
    block_n: int = 32,
    block_f: int = 32,
) -> torch.Tensor:
    """Two-layer LIF rate model storing the hidden spikes bit-packed.

    Rates ``[B, O]`` of ``linear_surrogate_lif_rate_forward`` applied to the
    spikes of ``linear_surrogate_lif_forward``; between forward and backward
    the hidden spikes are kept as packed words (src/myelin/kernels.py:811-846,
    src/myelin/autograd.py:1129-1387). Tile arguments are accepted and ignored.
    """

    sid = surrogate_id(surrogate)
    resolve_checkpoint_size(int(inputs.shape[0]), checkpoint_size)
    if not hard_forward:
        raise ValueError("packed-hidden two-layer rate training supports only hard_forward=True")
    _two_layer_validate(inputs, hidden_weight, hidden_bias, output_weight, output_bias)
    return TwoLayerPackedHiddenRateFunction.apply(
        inputs.contiguous(),
        hidden_weight.contiguous(),
        None if hidden_bias is None else hidden_bias.contiguous(),
        output_weight.contiguous(),
        None if output_bias is None else output_bias.contiguous(),
        params.decay,
        float(params.threshold),
        float(params.reset),
        sid,
        float(surrogate_slope),
        True,
    )


def linear_surrogate_lif_packed_forward(
    inputs: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    params: LIFParams,
    *,
    surrogate: SurrogateName = "atan",
    surrogate_slope: float = 10.0,
    hard_forward: bool = True,
    backend: Backend = "auto",
    checkpoint_size: CheckpointSize = 25,
    block_b: int = 16,
    block_f: int = 32,
) -> tuple[LIFState, PackedSpikes]:
    """Forward-only dense projection + LIF with packed int32 spike output.

    src/myelin/kernels.py:705-776. Not differentiable.
    """

    surrogate_id(surrogate)
    _check_backend(backend)
    resolve_checkpoint_size(int(inputs.shape[0]), checkpoint_size)
    _hard_forward_only(hard_forward, "packed surrogate LIF")
    _validate_linear(inputs, weight, bias)
    with torch.no_grad():
        T, B, F = inputs.shape
        N = weight.shape[1]
        x2 = inputs.contiguous().reshape(T * B, F)
        currents = _project(x2, weight.contiguous(), bias).view(T, B, N)
        v0 = torch.zeros((B, N), dtype=inputs.dtype, device=inputs.device)
        vT, _, _, words, _, _, _ = cops.scan_forward(
            currents, v0, None, nat.MB_LIF, params.decay, float(params.threshold),
            float(params.reset), 0.0, 0.0, nat.MB_RESET_HARD, packed=True,
        )
    return LIFState(membrane=vT), PackedSpikes(data=words, original_shape=(T, B, N))
