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


def _scan_scratch(x: torch.Tensor, alif: bool, save: bool):
    T, B, N = x.shape
    if not save or T == 0:
        return None, None
    K = nat.num_checkpoints(T)
    ckpt_v = torch.empty((K, B, N), dtype=torch.float32, device=x.device)
    ckpt_a = torch.empty_like(ckpt_v) if alif else None
    return ckpt_v, ckpt_a


def _scan_forward(ctx: Any, x, v0, a0, neuron, decay, threshold, reset, adapt_decay, beta,
                  reset_mode, surrogate, slope, reject_spike_grad):
    alif = neuron == nat.MB_ALIF
    save = any(ctx.needs_input_grad[:3])
    ckpt_v, ckpt_a = _scan_scratch(x, alif, save)
    vT = torch.empty_like(v0)
    aT = torch.empty_like(a0) if alif else None
    spikes = torch.empty_like(x)
    nat.scan_forward(
        neuron=neuron, x=x, v0=v0, a0=a0, vT=vT, aT=aT, spikes=spikes, packed=None,
        rates=None, ckpt_v=ckpt_v, ckpt_a=ckpt_a, decay=decay, threshold=threshold,
        reset=reset, adapt_decay=adapt_decay, beta=beta, reset_mode=reset_mode,
    )
    ctx.set_materialize_grads(False)
    ctx.save_for_backward(x, ckpt_v, ckpt_a)
    ctx.cfg = (neuron, decay, threshold, reset, adapt_decay, beta, reset_mode, surrogate, slope)
    ctx.reject_spike_grad = reject_spike_grad
    return vT, aT, spikes


def _scan_backward(ctx: Any, g_vT, g_aT, g_spikes):
    """Returns (grad_x, grad_v0, grad_a0) or None when no gradient flows."""

    if ctx.reject_spike_grad:
        if g_spikes is not None and bool(torch.any(g_spikes != 0)):
            raise NotImplementedError(
                "spike-output backward of the hard LIF forward is not defined; use "
                "surrogate_lif_forward for surrogate-gradient training."
            )
        g_spikes = None
    if g_vT is None and g_aT is None and g_spikes is None:
        return None
    x, ckpt_v, ckpt_a = ctx.saved_tensors
    neuron, decay, threshold, reset, adapt_decay, beta, reset_mode, surrogate, slope = ctx.cfg
    alif = neuron == nat.MB_ALIF
    need_x, need_v0, need_a0 = ctx.needs_input_grad[:3]
    grad_x = torch.empty_like(x)
    grad_v0 = torch.empty(x.shape[1:], dtype=x.dtype, device=x.device) if need_v0 else None
    grad_a0 = torch.empty(x.shape[1:], dtype=x.dtype, device=x.device) if alif and need_a0 else None
    nat.scan_backward(
        neuron=neuron, x=x, ckpt_v=ckpt_v, ckpt_a=ckpt_a,
        grad_spikes=None if g_spikes is None else g_spikes.contiguous(),
        grad_rates=None,
        grad_vT=None if g_vT is None else g_vT.contiguous(),
        grad_aT=None if (g_aT is None or not alif) else g_aT.contiguous(),
        grad_x=grad_x, grad_v0=grad_v0, grad_a0=grad_a0, decay=decay, threshold=threshold,
        reset=reset, adapt_decay=adapt_decay, beta=beta, reset_mode=reset_mode,
        surrogate=surrogate, slope=slope,
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
    if nat.gemm_tn_supported(x2, wt):
        out = torch.empty((x2.shape[0], wt.shape[0]), dtype=x2.dtype, device=x2.device)
        return nat.gemm_tn(x2, wt, bias, out)
    if bias is not None:
        return torch.addmm(bias, x2, weight)
    return torch.mm(x2, weight)


def _input_grad(g2: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """dX[T*B, F] = G[T*B, N] @ weight[F, N]^T."""

    if nat.gemm_tn_supported(g2, weight):
        out = torch.empty((g2.shape[0], weight.shape[0]), dtype=g2.dtype, device=g2.device)
        return nat.gemm_tn(g2, weight, None, out)
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
        ckpt_v, _ = _scan_scratch(currents, False, save)
        v0 = torch.zeros((B, N), dtype=inputs.dtype, device=inputs.device)
        vT = torch.empty_like(v0)
        out = torch.empty_like(v0) if rate_output else torch.empty_like(currents)
        nat.scan_forward(
            neuron=nat.MB_LIF, x=currents, v0=v0, a0=None, vT=vT, aT=None,
            spikes=None if rate_output else out, packed=None,
            rates=out if rate_output else None, ckpt_v=ckpt_v, ckpt_a=None, decay=decay,
            threshold=threshold, reset=reset, adapt_decay=0.0, beta=0.0,
            reset_mode=nat.MB_RESET_HARD,
        )
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
        grad_currents = torch.empty_like(currents)
        g = None if g_out is None else g_out.contiguous()
        nat.scan_backward(
            neuron=nat.MB_LIF, x=currents, ckpt_v=ckpt_v, ckpt_a=None,
            grad_spikes=None if rate_output else g, grad_rates=g if rate_output else None,
            grad_vT=None if g_vT is None else g_vT.contiguous(), grad_aT=None,
            grad_x=grad_currents, grad_v0=None, grad_a0=None, decay=decay, threshold=threshold,
            reset=reset, adapt_decay=0.0, beta=0.0, reset_mode=nat.MB_RESET_HARD,
            surrogate=surrogate, slope=slope,
        )
        g2 = grad_currents.view(T * B, N)
        grad_inputs = _input_grad(g2, weight).view(T, B, F) if need_x else None
        grad_weight = torch.mm(inputs.reshape(T * B, F).t(), g2) if need_w else None
        grad_bias = g2.sum(dim=0) if (need_b and ctx.has_bias) else None
        return (grad_inputs, grad_weight, grad_bias, *tail)
