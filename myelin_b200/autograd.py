"""torch.autograd boundaries around the CUDA scan (no Triton, no CPU path).

Forward saves only the inputs and one fp32 state per 16-step chunk; backward
replays each chunk in registers and walks it in reverse (``mb_scan_backward``).
The reference saves the whole pre-reset membrane trace instead
(src/myelin/autograd.py:130-201) or recomputes chunks on the host
(src/myelin/triton/lif.py:2070-2247).
"""

from __future__ import annotations

from typing import Any

import torch

from myelin_b200 import _native as nat
from myelin_b200 import compile_ops as cops


def _scan_forward(ctx: Any, x, v0, a0, neuron, decay, threshold, reset, adapt_decay, beta,
                  reset_mode, surrogate, slope, reject_spike_grad):
    save = any(ctx.needs_input_grad[:3])
    vT, aT, spikes, _, _, ckpt_v, ckpt_a = cops.scan_forward(
        x, v0, a0, neuron, decay, threshold, reset, adapt_decay, beta, reset_mode,
        dense=True, checkpoints=save,
    )
    ctx.set_materialize_grads(False)
    ctx.save_for_backward(x, ckpt_v, ckpt_a)
    ctx.cfg = (neuron, decay, threshold, reset, adapt_decay, beta, reset_mode, surrogate, slope)
    ctx.reject_spike_grad = reject_spike_grad
    return vT, aT, spikes


def _scan_backward(ctx: Any, g_vT, g_aT, g_spikes):
    """Returns (grad_x, grad_v0, grad_a0) or None when no gradient flows."""

    if g_vT is None and g_aT is None and g_spikes is None:
        return None
    x, ckpt_v, ckpt_a = ctx.saved_tensors
    neuron, decay, threshold, reset, adapt_decay, beta, reset_mode, surrogate, slope = ctx.cfg
    need_x, need_v0, need_a0 = ctx.needs_input_grad[:3]
    grad_x, grad_v0, grad_a0 = cops.scan_backward(
        x, ckpt_v, ckpt_a, grad_spikes=g_spikes, grad_vT=g_vT,
        grad_aT=g_aT if neuron == nat.MB_ALIF else None, neuron=neuron, decay=decay,
        threshold=threshold, reset=reset, adapt_decay=adapt_decay, beta=beta,
        reset_mode=reset_mode, surrogate=surrogate, slope=slope, need_v0=need_v0,
        need_a0=need_a0, reject_spike_grad=ctx.reject_spike_grad,
    )
    return (grad_x if need_x else None), grad_v0, grad_a0


class LIFScanFunction(torch.autograd.Function):
    """Fused-time LIF scan: (inputs, v0) -> (final membrane, spikes).

    ``surrogate`` is a kernel id (0..5), or ``MB_SURR_NONE`` (6) for the exact
    gradient of the hard threshold (the plain ``lif_forward`` boundary, which
    like src/myelin/autograd.py:46-53 refuses nonzero spike gradients when
    ``reject_spike_grad`` is set).
    """

    @staticmethod
    def forward(ctx: Any, x, v0, decay, threshold, reset, reset_mode, surrogate, slope,
                reject_spike_grad):
        vT, _, spikes = _scan_forward(ctx, x, v0, None, nat.MB_LIF, decay, threshold, reset,
                                      0.0, 0.0, reset_mode, surrogate, slope, reject_spike_grad)
        return vT, spikes

    @staticmethod
    def backward(ctx: Any, g_vT, g_spikes):
        grads = _scan_backward(ctx, g_vT, None, g_spikes)
        tail = (None,) * 7
        if grads is None:
            return (None, None, *tail)
        return (grads[0], grads[1], *tail)


class ALIFScanFunction(torch.autograd.Function):
    """Fused-time ALIF scan: (inputs, v0, a0) -> (final membrane, final adaptation, spikes)."""

    @staticmethod
    def forward(ctx: Any, x, v0, a0, decay, threshold, reset, adapt_decay, beta, reset_mode,
                surrogate, slope):
        return _scan_forward(ctx, x, v0, a0, nat.MB_ALIF, decay, threshold, reset, adapt_decay,
                             beta, reset_mode, surrogate, slope, False)

    @staticmethod
    def backward(ctx: Any, g_vT, g_aT, g_spikes):
        grads = _scan_backward(ctx, g_vT, g_aT, g_spikes)
        tail = (None,) * 8
        if grads is None:
            return (None, None, None, *tail)
        return (*grads, *tail)


def _project(x2: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """currents[T*B, N] = x2[T*B, F] @ weight[F, N] (+ bias).

    16-bit inputs run on the tcgen05 GEMM (fp32 accumulation, bias added in
    fp32, one rounding to the input type). fp32 inputs keep fp32 arithmetic
    (cuBLAS SGEMM): the tensor cores have no fp32-exact mode, and spike
    parity with the fp32 reference needs fp32 products.
    """

    wt = weight.t().contiguous()  # [N, F]: K-major B operand
    if cops.gemm_tn_dtype_ok(x2, wt):
        return cops.gemm_tn(x2, wt, bias)
    if bias is not None:
        return torch.addmm(bias, x2, weight)
    return torch.mm(x2, weight)


def _input_grad(g2: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """dX[T*B, F] = G[T*B, N] @ weight[F, N]^T."""

    if cops.gemm_tn_dtype_ok(g2, weight):
        return cops.gemm_tn(g2, weight)
    return torch.mm(g2, weight.t())


class LinearScanFunction(torch.autograd.Function):
    """Dense projection ``x_t @ W + b`` feeding the LIF scan from a zero membrane.

    Outputs (final membrane, spikes [T,B,N]) when ``rate_output`` is False,
    else (final membrane, rates [B,N] = count / T). The projected currents are
    kept resident for the backward (no GEMM recompute); the backward runs the
    reverse scan to get dL/dcurrents, then the two weight-side GEMMs.
    Reference semantics: src/myelin/autograd.py:445-885.
    """

    @staticmethod
    def forward(
        ctx: Any,
        inputs: torch.Tensor,
        weight: torch.Tensor,
        bias: torch.Tensor | None,
        decay: float,
        threshold: float,
        reset: float,
        surrogate: int,
        slope: float,
        rate_output: bool,
    ):
        T, B, F = inputs.shape
        N = weight.shape[1]
        x2 = inputs.reshape(T * B, F)
        currents = _project(x2, weight, bias).view(T, B, N)
        save = any(ctx.needs_input_grad[:3])
        v0 = torch.zeros((B, N), dtype=inputs.dtype, device=inputs.device)
        vT, _, spikes, _, rates, ckpt_v, _ = cops.scan_forward(
            currents, v0, None, nat.MB_LIF, decay, threshold, reset, 0.0, 0.0,
            nat.MB_RESET_HARD, dense=not rate_output, rates=rate_output, checkpoints=save,
        )
        out = rates if rate_output else spikes
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(inputs, weight, currents, ckpt_v)
        ctx.has_bias = bias is not None
        ctx.cfg = (decay, threshold, reset, surrogate, slope, rate_output)
        return vT, out

    @staticmethod
    def backward(ctx: Any, g_vT, g_out):
        tail = (None,) * 6
        if g_vT is None and g_out is None:
            return (None, None, None, *tail)
        inputs, weight, currents, ckpt_v = ctx.saved_tensors
        decay, threshold, reset, surrogate, slope, rate_output = ctx.cfg
        need_x, need_w, need_b = ctx.needs_input_grad[:3]
        T, B, F = inputs.shape
        N = weight.shape[1]
        grad_currents, _, _ = cops.scan_backward(
            currents, ckpt_v, None, grad_spikes=None if rate_output else g_out,
            grad_rates=g_out if rate_output else None, grad_vT=g_vT, neuron=nat.MB_LIF,
            decay=decay, threshold=threshold, reset=reset, adapt_decay=0.0, beta=0.0,
            reset_mode=nat.MB_RESET_HARD, surrogate=surrogate, slope=slope, need_v0=False,
            need_a0=False,
        )
        g2 = grad_currents.view(T * B, N)
        grad_inputs = _input_grad(g2, weight).view(T, B, F) if need_x else None
        grad_weight = torch.mm(inputs.reshape(T * B, F).t(), g2) if need_w else None
        grad_bias = g2.sum(dim=0) if (need_b and ctx.has_bias) else None
        return (grad_inputs, grad_weight, grad_bias, *tail)
