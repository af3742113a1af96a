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
    """currents[T*B, N] = x2[T*B, F] @ weight[F, N] (+ bias) on the library's
    tensor-core GEMM: 16-bit operands read in place (weight as an N-major
    operand, no transposed copy), fp32 operands as exact 3-way bf16 splits
    (fp32 products, see ``myelin_b200.projection``); fp32 accumulation, bias
    added in fp32, one rounding to the input type."""

    return cops.linear_project(x2, weight, bias)


def _input_grad(g2: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """dX[T*B, F] = G[T*B, N] @ weight[F, N]^T (tensor cores, as ``_project``)."""

    return cops.linear_input_grad(g2, weight)


def _weight_bias_grads(x2: torch.Tensor, g2: torch.Tensor, weight: torch.Tensor,
                       bias: torch.Tensor | None, need_w: bool, need_b: bool):
    """(dW = x2^T G on the tensor cores, x2 read as an M-major operand; db =
    fixed-order column sums of G), each None when not needed."""

    if not (need_w or need_b):
        return None, None
    gw, gb = cops.linear_weight_grad(x2, g2, weight, bias if need_b else None)
    return (gw if need_w else None), gb


class LinearScanFunction(torch.autograd.Function):
    """Dense projection ``x_t @ W + b`` feeding the LIF scan from a zero membrane.

    Outputs (final membrane, spikes [T,B,N]) when ``rate_output`` is False,
    else (final membrane, rates [B,N] = count / T). The projected currents are
    kept resident for the backward (no GEMM recompute); the backward runs the
    reverse scan to get dL/dcurrents, then dX and dW on the tensor cores and
    db as a fixed-order column sum (no library GEMM, no float atomics).
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
        # dtype / device carrier for the bias gradient (no data kept)
        ctx.bias_like = bias.new_empty(0) if bias is not None else None
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
        need_bias = need_b and ctx.has_bias
        # with a bias, the reverse scan also sums dL/dcurrents over t per neuron
        # as it stores it; db is then the sum of those over the batch rows
        outs = cops.scan_backward(
            currents, ckpt_v, None, grad_spikes=None if rate_output else g_out,
            grad_rates=g_out if rate_output else None, grad_vT=g_vT, neuron=nat.MB_LIF,
            decay=decay, threshold=threshold, reset=reset, adapt_decay=0.0, beta=0.0,
            reset_mode=nat.MB_RESET_HARD, surrogate=surrogate, slope=slope, need_v0=False,
            need_a0=False, need_sum=need_bias,
        )
        g2 = outs[0].view(T * B, N)
        grad_inputs = _input_grad(g2, weight).view(T, B, F) if need_x else None
        grad_weight, _ = _weight_bias_grads(inputs.reshape(T * B, F), g2, weight, None, need_w,
                                            False)
        grad_bias = cops.bias_grad(outs[3].view(B, N), ctx.bias_like) if need_bias else None
        return (grad_inputs, grad_weight, grad_bias, *tail)


class TwoLayerPackedHiddenRateFunction(torch.autograd.Function):
    """Two stream-synapse LIF layers: hidden spikes, then output spike rates,
    with the hidden spikes kept bit-packed between forward and backward
    (``save_hidden``) or not kept at all and regenerated in the backward by
    re-running the layer-1 scan from its checkpoints (whole-model recompute,
    src/myelin/autograd.py:926-1126).

    Forward: currents1 = X W1 + b1 -> scan writing packed hidden words (and
    checkpoints) -> hidden = unpack(words), transient -> currents2 = hidden W2
    + b2 -> rate scan. Saved: inputs, weights, biases, the two layers'
    checkpoints and the packed words (1 bit per hidden spike instead of a
    dense [T, B, H] tensor and two current tensors). Backward recomputes both
    projections (same deterministic kernels, so the same bits) and runs the
    two reverse scans. Reference: src/myelin/autograd.py:1129-1387.
    """

    @staticmethod
    def forward(ctx: Any, inputs, hidden_weight, hidden_bias, output_weight, output_bias,
                decay: float, threshold: float, reset: float, surrogate: int, slope: float,
                save_hidden: bool = True):
        T, B, F = inputs.shape
        H = hidden_weight.shape[1]
        O = output_weight.shape[1]
        save = any(ctx.needs_input_grad[:5])
        cur1 = _project(inputs.reshape(T * B, F), hidden_weight, hidden_bias).view(T, B, H)
        v0 = torch.zeros((B, H), dtype=inputs.dtype, device=inputs.device)
        _, _, _, words, _, ckpt1, _ = cops.scan_forward(
            cur1, v0, None, nat.MB_LIF, decay, threshold, reset, 0.0, 0.0, nat.MB_RESET_HARD,
            packed=True, checkpoints=save,
        )
        del cur1
        hidden = cops.unpack(words, T * B, H, inputs.dtype)
        cur2 = _project(hidden, output_weight, output_bias).view(T, B, O)
        del hidden
        vo = torch.zeros((B, O), dtype=inputs.dtype, device=inputs.device)
        _, _, _, _, rates, ckpt2, _ = cops.scan_forward(
            cur2, vo, None, nat.MB_LIF, decay, threshold, reset, 0.0, 0.0, nat.MB_RESET_HARD,
            rates=True, checkpoints=save,
        )
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(inputs, hidden_weight, hidden_bias, output_weight, output_bias,
                              ckpt1, ckpt2, words if save_hidden else None)
        ctx.cfg = (decay, threshold, reset, surrogate, slope)
        return rates

    @staticmethod
    def backward(ctx: Any, g_rates):
        tail = (None,) * 6
        if g_rates is None:
            return (None,) * 5 + tail
        inputs, w1, b1, w2, b2, ckpt1, ckpt2, words = ctx.saved_tensors
        decay, threshold, reset, surrogate, slope = ctx.cfg
        need_x, need_w1, need_b1, need_w2, need_b2 = ctx.needs_input_grad[:5]
        T, B, F = inputs.shape
        H, O = w1.shape[1], w2.shape[1]
        scan_kw = dict(neuron=nat.MB_LIF, decay=decay, threshold=threshold, reset=reset,
                       adapt_decay=0.0, beta=0.0, reset_mode=nat.MB_RESET_HARD,
                       surrogate=surrogate, slope=slope, need_v0=False, need_a0=False)

        x2 = inputs.reshape(T * B, F)
        cur1 = None
        if words is None:  # whole-model recompute: regenerate the hidden spikes
            cur1 = _project(x2, w1, b1).view(T, B, H)
            v0 = torch.zeros((B, H), dtype=inputs.dtype, device=inputs.device)
            words = cops.scan_forward(cur1, v0, None, nat.MB_LIF, decay, threshold, reset, 0.0,
                                      0.0, nat.MB_RESET_HARD, packed=True)[3]
        hidden = cops.unpack(words, T * B, H, inputs.dtype)  # [T*B, H]
        cur2 = _project(hidden, w2, b2).view(T, B, O)
        # the bias gradients as in LinearScanFunction: sums over t formed by the
        # reverse scan, then over the batch rows (the same bits as the dense path)
        sum2 = need_b2 and b2 is not None
        outs2 = cops.scan_backward(cur2, ckpt2, None, grad_rates=g_rates, need_sum=sum2,
                                   **scan_kw)
        del cur2
        g2 = outs2[0].view(T * B, O)
        grad_w2, _ = _weight_bias_grads(hidden, g2, w2, None, need_w2, False)
        grad_b2 = cops.bias_grad(outs2[3].view(B, O), b2) if sum2 else None
        del hidden

        grad_x = grad_w1 = grad_b1 = None
        if need_x or need_w1 or need_b1:
            g_hidden = _input_grad(g2, w2).view(T, B, H)
            if cur1 is None:
                cur1 = _project(x2, w1, b1).view(T, B, H)
            sum1 = need_b1 and b1 is not None
            outs1 = cops.scan_backward(cur1, ckpt1, None, grad_spikes=g_hidden, need_sum=sum1,
                                       **scan_kw)
            del cur1, g_hidden
            g1 = outs1[0].view(T * B, H)
            grad_x = _input_grad(g1, w1).view(T, B, F) if need_x else None
            grad_w1, _ = _weight_bias_grads(x2, g1, w1, None, need_w1, False)
            grad_b1 = cops.bias_grad(outs1[3].view(B, H), b1) if sum1 else None
        return (grad_x, grad_w1, grad_b1, grad_w2, grad_b2, *tail)
