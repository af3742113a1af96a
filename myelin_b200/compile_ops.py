"""Compile-visible operators: the C-ABI entry points as ``torch.library`` ops.

``torch.compile`` cannot trace through the ctypes calls of ``_native``; each
entry point is therefore registered as a custom op (``myelin_b200::*``) with a
fake implementation that only computes output shapes, so a compiled model
sees opaque operators instead of graph breaks. The autograd functions call the
ops' backward counterparts explicitly (``myelin_b200::scan_backward``), so
forward and backward both stay in the graph.

The reference registers a narrower set the same way
(src/myelin/triton/compile_ops.py:23-560: the checkpointed rate forward and
its gradients as ``myelin::*`` ops with ``register_fake`` /
``register_autograd``). Here every hot-path kernel is covered.

Eager calls skip the dispatcher (about 12 us per call) and run the same
implementation directly; while ``torch.compile`` traces, the registered op is
called. Both run the same CUDA kernels.
"""

from __future__ import annotations

import torch

from myelin_b200 import _native as nat

_NS = "myelin_b200"


def _tracing() -> bool:
    """Whether a tracer is recording: dynamo (``torch.compile``) or any active
    dispatch mode (AOTAutograd, ``make_fx``, fake-tensor propagation)."""

    return torch.compiler.is_compiling() or torch._C._len_torch_dispatch_stack() > 0


def _none0(t: torch.Tensor | None) -> torch.Tensor | None:
    """Zero-element placeholders (outputs that were not requested) read as None."""

    return None if t is None or t.numel() == 0 and t.dim() == 1 else t


# ---------------------------------------------------------------------------
# scan forward
# ---------------------------------------------------------------------------
def _scan_forward_shapes(x, neuron, dense, packed, rates, checkpoints):
    T, B, N = x.shape
    alif = neuron == nat.MB_ALIF
    checkpoints = checkpoints and T > 0
    K = (T + nat.SCAN_CHUNK - 1) // nat.SCAN_CHUNK if checkpoints else 0
    return {
        "vT": ((B, N), x.dtype),
        "aT": ((B, N) if alif else (0,), x.dtype),
        "spikes": ((T, B, N) if dense else (0,), x.dtype),
        "packed": ((T, B, (N + 31) // 32) if packed else (0,), torch.int32),
        "rates": ((B, N) if rates else (0,), x.dtype),
        "ckpt_v": ((K, B, N) if checkpoints else (0,), torch.float32),
        "ckpt_a": ((K, B, N) if checkpoints and alif else (0,), torch.float32),
    }


def _scan_forward_eager(x, v0, a0, neuron, decay, threshold, reset, adapt_decay, beta,
                        reset_mode, dense, packed, rates, checkpoints):
    """Allocates only the requested outputs; the others are None."""

    shapes = _scan_forward_shapes(x, neuron, dense, packed, rates, checkpoints)
    out = {k: (torch.empty(s, dtype=d, device=x.device) if len(s) > 1 else None)
           for k, (s, d) in shapes.items()}
    nat.scan_forward(
        neuron=neuron, x=x, v0=v0, a0=a0 if neuron == nat.MB_ALIF else None, vT=out["vT"],
        aT=out["aT"], spikes=out["spikes"], packed=out["packed"], rates=out["rates"],
        ckpt_v=out["ckpt_v"], ckpt_a=out["ckpt_a"], decay=decay, threshold=threshold,
        reset=reset, adapt_decay=adapt_decay, beta=beta, reset_mode=reset_mode,
    )
    return tuple(out.values())


def _scan_forward_impl(
    x: torch.Tensor, v0: torch.Tensor, a0: torch.Tensor | None, neuron: int, decay: float,
    threshold: float, reset: float, adapt_decay: float, beta: float, reset_mode: int,
    dense: bool, packed: bool, rates: bool, checkpoints: bool,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
           torch.Tensor]:
    outs = _scan_forward_eager(x, v0, a0, neuron, decay, threshold, reset, adapt_decay, beta,
                               reset_mode, dense, packed, rates, checkpoints)
    # an op returns tensors only: zero-element placeholders for the unrequested ones
    return tuple(x.new_empty(0) if t is None else t for t in outs)  # type: ignore[return-value]


scan_forward_op = torch.library.custom_op(f"{_NS}::scan_forward", _scan_forward_impl,
                                          mutates_args=())


@scan_forward_op.register_fake
def _scan_forward_fake(x, v0, a0, neuron, decay, threshold, reset, adapt_decay, beta,
                       reset_mode, dense, packed, rates, checkpoints):
    shapes = _scan_forward_shapes(x, neuron, dense, packed, rates, checkpoints)
    return tuple(x.new_empty(s, dtype=d) for s, d in shapes.values())


def scan_forward(x, v0, a0, neuron, decay, threshold, reset, adapt_decay, beta, reset_mode, *,
                 dense=False, packed=False, rates=False, checkpoints=False):
    """Fused-time LIF/ALIF forward (``mb_scan_forward``).

    Returns ``(vT, aT, spikes, packed, rates, ckpt_v, ckpt_a)``; outputs that
    were not requested (and aT / ckpt_a for LIF) are None.
    """

    args = (x, v0, a0, int(neuron), float(decay), float(threshold), float(reset),
            float(adapt_decay), float(beta), int(reset_mode), bool(dense), bool(packed),
            bool(rates), bool(checkpoints))
    if _tracing():
        return tuple(_none0(t) for t in scan_forward_op(*args))
    return _scan_forward_eager(*args)


# ---------------------------------------------------------------------------
# scan backward
# ---------------------------------------------------------------------------
def _scan_backward_eager(x, ckpt_v, ckpt_a, grad_spikes, grad_rates, grad_vT, grad_aT, neuron,
                         decay, threshold, reset, adapt_decay, beta, reset_mode, surrogate,
                         slope, need_v0, need_a0, reject_spike_grad, need_sum=False):
    """Allocates only the requested gradients; the others are None."""

    if reject_spike_grad and grad_spikes is not None:
        # the hard forward's spike output has no gradient (src/myelin/autograd.py:46-53)
        if bool(torch.any(grad_spikes != 0)):
            raise NotImplementedError(
                "spike-output backward of the hard LIF forward is not defined; use "
                "surrogate_lif_forward for surrogate-gradient training."
            )
        grad_spikes = None
    T, B, N = x.shape
    alif = neuron == nat.MB_ALIF
    grad_x = torch.empty_like(x)
    grad_v0 = torch.empty((B, N), dtype=x.dtype, device=x.device) if need_v0 else None
    grad_a0 = torch.empty((B, N), dtype=x.dtype, device=x.device) if alif and need_a0 else None
    grad_sum = torch.empty((B * N,), dtype=torch.float32, device=x.device) if need_sum else None
    nat.scan_backward(
        neuron=neuron, x=x, ckpt_v=ckpt_v, ckpt_a=ckpt_a if alif else None,
        grad_spikes=None if grad_spikes is None else grad_spikes.contiguous(),
        grad_rates=None if grad_rates is None else grad_rates.contiguous(),
        grad_vT=None if grad_vT is None else grad_vT.contiguous(),
        grad_aT=None if (grad_aT is None or not alif) else grad_aT.contiguous(),
        grad_x=grad_x, grad_v0=grad_v0, grad_a0=grad_a0, decay=decay, threshold=threshold,
        reset=reset, adapt_decay=adapt_decay, beta=beta, reset_mode=reset_mode,
        surrogate=surrogate, slope=slope, grad_sum=grad_sum,
    )
    return grad_x, grad_v0, grad_a0, grad_sum


def _scan_backward_impl(
    x: torch.Tensor, ckpt_v: torch.Tensor | None, ckpt_a: torch.Tensor | None,
    grad_spikes: torch.Tensor | None, grad_rates: torch.Tensor | None,
    grad_vT: torch.Tensor | None, grad_aT: torch.Tensor | None, neuron: int, decay: float,
    threshold: float, reset: float, adapt_decay: float, beta: float, reset_mode: int,
    surrogate: int, slope: float, need_v0: bool, need_a0: bool, reject_spike_grad: bool,
    need_sum: bool = False,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    outs = _scan_backward_eager(x, ckpt_v, ckpt_a, grad_spikes, grad_rates, grad_vT, grad_aT,
                                neuron, decay, threshold, reset, adapt_decay, beta, reset_mode,
                                surrogate, slope, need_v0, need_a0, reject_spike_grad, need_sum)
    empty = (x.new_empty(0), x.new_empty(0), x.new_empty(0), x.new_empty(0, dtype=torch.float32))
    return tuple(e if t is None else t for t, e in zip(outs, empty))  # type: ignore[return-value]


scan_backward_op = torch.library.custom_op(f"{_NS}::scan_backward", _scan_backward_impl,
                                           mutates_args=())


@scan_backward_op.register_fake
def _scan_backward_fake(x, ckpt_v, ckpt_a, grad_spikes, grad_rates, grad_vT, grad_aT, neuron,
                        decay, threshold, reset, adapt_decay, beta, reset_mode, surrogate, slope,
                        need_v0, need_a0, reject_spike_grad, need_sum=False):
    B, N = x.shape[1], x.shape[2]
    alif = neuron == nat.MB_ALIF
    return (torch.empty_like(x), x.new_empty((B, N) if need_v0 else (0,)),
            x.new_empty((B, N) if alif and need_a0 else (0,)),
            x.new_empty((B * N,) if need_sum else (0,), dtype=torch.float32))


def scan_backward(x, ckpt_v, ckpt_a, *, grad_spikes=None, grad_rates=None, grad_vT=None,
                  grad_aT=None, neuron, decay, threshold, reset, adapt_decay, beta, reset_mode,
                  surrogate, slope, need_v0=True, need_a0=True, reject_spike_grad=False,
                  need_sum=False):
    """Reverse-time surrogate backward (``mb_scan_backward``).

    Returns ``(grad_x, grad_v0, grad_a0)``; gradients that were not requested
    are None. With ``need_sum`` a fourth value: the fp32 sum over t of grad_x
    per neuron, [B*N] (``mb_scan_backward_sum``; formed inside the LIF
    backward kernel as it stores grad_x).
    """

    args = (x, ckpt_v, ckpt_a, grad_spikes, grad_rates, grad_vT, grad_aT, int(neuron),
            float(decay), float(threshold), float(reset), float(adapt_decay), float(beta),
            int(reset_mode), int(surrogate), float(slope), bool(need_v0), bool(need_a0),
            bool(reject_spike_grad), bool(need_sum))
    if _tracing():
        outs = tuple(_none0(t) for t in scan_backward_op(*args))
    else:
        outs = _scan_backward_eager(*args)
    return outs if need_sum else outs[:3]


# ---------------------------------------------------------------------------
# projection GEMM
# ---------------------------------------------------------------------------
def _gemm_tn_impl(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    out = torch.empty((a.shape[0], b.shape[0]), dtype=a.dtype, device=a.device)
    if not nat.gemm_tn_supported(a, b):
        # 16-byte row alignment is a property of the storage, invisible while
        # tracing: such operands are made contiguous first
        a, b = a.contiguous(), b.contiguous()
    return nat.gemm_tn(a, b, bias, out)


gemm_tn_op = torch.library.custom_op(f"{_NS}::gemm_tn", _gemm_tn_impl, mutates_args=())


@gemm_tn_op.register_fake
def _gemm_tn_fake(a, b, bias):
    return a.new_empty((a.shape[0], b.shape[0]))


def gemm_tn(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``a[M, K] @ b[N, K]^T (+ bias)`` on the tcgen05 GEMM (16-bit, K % 8 == 0)."""

    return gemm_tn_op(a, b, bias) if _tracing() else _gemm_tn_impl(a, b, bias)


def gemm_tn_dtype_ok(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Shape/dtype part of the GEMM's operand rules (what tracing can see)."""

    return (a.dtype in nat.GEMM_DTYPES and b.dtype == a.dtype and a.dim() == 2 and b.dim() == 2
            and a.shape[1] == b.shape[1] and a.shape[1] % 8 == 0)


# ---------------------------------------------------------------------------
# stream-synapse projections (myelin_b200.projection: mb_gemm, mb_split_bf16,
# mb_column_sums)
# ---------------------------------------------------------------------------
def _linear_project_impl(x2: torch.Tensor, weight: torch.Tensor,
                         bias: torch.Tensor | None) -> torch.Tensor:
    from myelin_b200 import projection

    return projection.project(x2, weight, bias)


linear_project_op = torch.library.custom_op(f"{_NS}::linear_project", _linear_project_impl,
                                            mutates_args=())


@linear_project_op.register_fake
def _linear_project_fake(x2, weight, bias):
    return x2.new_empty((x2.shape[0], weight.shape[1]))


def linear_project(x2: torch.Tensor, weight: torch.Tensor,
                   bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x2[M, F] @ weight[F, N] (+ bias)`` on the tensor cores (16-bit or fp32)."""

    if _tracing():
        return linear_project_op(x2, weight, bias)
    return _linear_project_impl(x2, weight, bias)


def _linear_input_grad_impl(g2: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    from myelin_b200 import projection

    return projection.input_grad(g2, weight)


linear_input_grad_op = torch.library.custom_op(f"{_NS}::linear_input_grad",
                                               _linear_input_grad_impl, mutates_args=())


@linear_input_grad_op.register_fake
def _linear_input_grad_fake(g2, weight):
    return g2.new_empty((g2.shape[0], weight.shape[0]))


def linear_input_grad(g2: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """``g2[M, N] @ weight[F, N]^T`` on the tensor cores."""

    if _tracing():
        return linear_input_grad_op(g2, weight)
    return _linear_input_grad_impl(g2, weight)


def _linear_weight_grad_impl(x2: torch.Tensor, g2: torch.Tensor, weight_like: torch.Tensor,
                             bias_like: torch.Tensor | None) -> tuple[torch.Tensor, torch.Tensor]:
    from myelin_b200 import projection

    gw = projection.weight_grad(x2, g2, weight_like.dtype)
    gb = (projection.bias_grad(g2, bias_like.dtype) if bias_like is not None
          else g2.new_empty(0))
    return gw, gb


linear_weight_grad_op = torch.library.custom_op(f"{_NS}::linear_weight_grad",
                                                _linear_weight_grad_impl, mutates_args=())


@linear_weight_grad_op.register_fake
def _linear_weight_grad_fake(x2, g2, weight_like, bias_like):
    gw = weight_like.new_empty((x2.shape[1], g2.shape[1]))
    gb = bias_like.new_empty((g2.shape[1],)) if bias_like is not None else g2.new_empty(0)
    return gw, gb


def linear_weight_grad(x2: torch.Tensor, g2: torch.Tensor, weight_like: torch.Tensor,
                       bias_like: torch.Tensor | None
                       ) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``(x2^T @ g2, column sums of g2)`` in the weight's / bias's dtypes; the
    bias gradient is None when ``bias_like`` is None."""

    if _tracing():
        gw, gb = linear_weight_grad_op(x2, g2, weight_like, bias_like)
    else:
        gw, gb = _linear_weight_grad_impl(x2, g2, weight_like, bias_like)
    return gw, (gb if bias_like is not None else None)


def _bias_grad_impl(rows: torch.Tensor, bias_like: torch.Tensor) -> torch.Tensor:
    from myelin_b200 import projection

    return projection.bias_grad(rows, bias_like.dtype)


bias_grad_op = torch.library.custom_op(f"{_NS}::bias_grad", _bias_grad_impl, mutates_args=())


@bias_grad_op.register_fake
def _bias_grad_fake(rows, bias_like):
    return bias_like.new_empty((rows.shape[1],))


def bias_grad(rows: torch.Tensor, bias_like: torch.Tensor) -> torch.Tensor:
    """Column sums of ``rows`` [R, N] in a fixed order, in the bias's dtype
    (``mb_column_sums``): the bias gradient from per-neuron sums over t."""

    if _tracing():
        return bias_grad_op(rows, bias_like)
    return _bias_grad_impl(rows, bias_like)


# ---------------------------------------------------------------------------
# packing
# ---------------------------------------------------------------------------
def _pack_impl(spikes: torch.Tensor, rows: int, n: int) -> torch.Tensor:
    words = torch.empty((rows, (n + 31) // 32), dtype=torch.int32, device=spikes.device)
    nat.pack(spikes, words, rows, n)
    return words


pack_op = torch.library.custom_op(f"{_NS}::pack_spikes", _pack_impl, mutates_args=())


@pack_op.register_fake
def _pack_fake(spikes, rows, n):
    return spikes.new_empty((rows, (n + 31) // 32), dtype=torch.int32)


def pack(spikes: torch.Tensor, rows: int, n: int) -> torch.Tensor:
    """Packed words ``[rows, ceil(n/32)]`` of contiguous ``spikes[rows, n]``."""

    return pack_op(spikes, rows, n) if _tracing() else _pack_impl(spikes, rows, n)


def _unpack_impl(words: torch.Tensor, rows: int, n: int, dtype: torch.dtype) -> torch.Tensor:
    out = torch.empty((rows, n), dtype=dtype, device=words.device)
    nat.unpack(words, out, rows, n)
    return out


unpack_op = torch.library.custom_op(f"{_NS}::unpack_spikes", _unpack_impl, mutates_args=())


@unpack_op.register_fake
def _unpack_fake(words, rows, n, dtype):
    return words.new_empty((rows, n), dtype=dtype)


def unpack(words: torch.Tensor, rows: int, n: int, dtype: torch.dtype) -> torch.Tensor:
    """Dense ``[rows, n]`` 0/1 values of ``dtype`` from contiguous packed words."""

    return unpack_op(words, rows, n, dtype) if _tracing() else _unpack_impl(words, rows, n, dtype)


def _count_rows_impl(words: torch.Tensor, rows: int, n: int) -> torch.Tensor:
    counts = torch.empty((rows,), dtype=torch.int64, device=words.device)
    nat.count_rows(words, counts, rows, n)
    return counts


count_rows_op = torch.library.custom_op(f"{_NS}::count_rows", _count_rows_impl, mutates_args=())


@count_rows_op.register_fake
def _count_rows_fake(words, rows, n):
    return words.new_empty((rows,), dtype=torch.int64)


def count_rows(words: torch.Tensor, rows: int, n: int) -> torch.Tensor:
    """int64 spike count of each packed row."""

    return count_rows_op(words, rows, n) if _tracing() else _count_rows_impl(words, rows, n)


def _count_columns_impl(words: torch.Tensor, rows: int, n: int, wide: bool) -> torch.Tensor:
    counts = torch.empty((n,), dtype=torch.int64 if wide else torch.int32, device=words.device)
    nat.count_columns(words, rows, n, counts if wide else None, None if wide else counts)
    return counts


count_columns_op = torch.library.custom_op(f"{_NS}::count_columns", _count_columns_impl,
                                           mutates_args=())


@count_columns_op.register_fake
def _count_columns_fake(words, rows, n, wide):
    return words.new_empty((n,), dtype=torch.int64 if wide else torch.int32)


def count_columns(words: torch.Tensor, rows: int, n: int, wide: bool = True) -> torch.Tensor:
    """Per-neuron spike counts over all rows: int64 (``wide``) or int32."""

    if _tracing():
        return count_columns_op(words, rows, n, wide)
    return _count_columns_impl(words, rows, n, wide)


def _pack_count_impl(spikes: torch.Tensor, rows: int, n: int,
                     wide: bool) -> tuple[torch.Tensor, torch.Tensor]:
    words = torch.empty((rows, (n + 31) // 32), dtype=torch.int32, device=spikes.device)
    counts = torch.empty((n,), dtype=torch.int64 if wide else torch.int32, device=spikes.device)
    nat.pack_count(spikes, words, rows, n, counts if wide else None, None if wide else counts)
    return words, counts


pack_count_op = torch.library.custom_op(f"{_NS}::pack_count_spikes", _pack_count_impl,
                                        mutates_args=())


@pack_count_op.register_fake
def _pack_count_fake(spikes, rows, n, wide):
    return (spikes.new_empty((rows, (n + 31) // 32), dtype=torch.int32),
            spikes.new_empty((n,), dtype=torch.int64 if wide else torch.int32))


def pack_count(spikes: torch.Tensor, rows: int, n: int,
               wide: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """Packed words ``[rows, ceil(n/32)]`` and per-neuron counts ``[n]`` in one call."""

    if _tracing():
        return pack_count_op(spikes, rows, n, wide)
    return _pack_count_impl(spikes, rows, n, wide)


IZH_FIELDS = ("recovery_decay", "recovery_coupling", "reset_voltage", "recovery_jump",
              "threshold", "dt", "voltage_square_coeff", "voltage_coeff", "voltage_bias")


def _izhikevich_impl(x: torch.Tensor, v0: torch.Tensor, u0: torch.Tensor,
                     params: list[float]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    vT = torch.empty_like(v0)
    uT = torch.empty_like(u0)
    spikes = torch.empty_like(x)
    nat.izhikevich_forward(x, v0, u0, vT, uT, spikes,
                           nat.IzhikevichParamsC(*[float(p) for p in params]))
    return vT, uT, spikes


izhikevich_op = torch.library.custom_op(f"{_NS}::izhikevich_forward", _izhikevich_impl,
                                        mutates_args=())


@izhikevich_op.register_fake
def _izhikevich_fake(x, v0, u0, params):
    return torch.empty_like(v0), torch.empty_like(u0), torch.empty_like(x)


def izhikevich_forward(x: torch.Tensor, v0: torch.Tensor, u0: torch.Tensor,
                       params: list[float]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Fused-time Izhikevich forward: (vT, uT, spikes); ``params`` in IZH_FIELDS order."""

    if _tracing():
        return izhikevich_op(x, v0, u0, list(params))
    return _izhikevich_impl(x, v0, u0, list(params))


OPS = (scan_forward_op, scan_backward_op, gemm_tn_op, linear_project_op, linear_input_grad_op,
       linear_weight_grad_op, bias_grad_op, pack_op, unpack_op, count_rows_op, count_columns_op,
       pack_count_op, izhikevich_op)
