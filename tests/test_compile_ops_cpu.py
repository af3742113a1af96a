"""Compile visibility of the CUDA path (``myelin_b200.compile_ops``), without a GPU.

Fake CUDA tensors carry shapes and dtypes only, so ``make_fx`` in fake mode
records which operators a compiled graph would contain. Every public hot-path
function must reach the ``myelin_b200::*`` custom ops (never a ctypes call,
which a tracer cannot see), and the fake implementations must give the shapes
and dtypes the kernels write. The reference registers its compile-visible
ops the same way (src/myelin/triton/compile_ops.py:23-560).
"""

from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.proxy_tensor import make_fx

import myelin_b200 as mb
from myelin_b200 import _native as nat
from myelin_b200 import compile_ops as cops

OP_NAMES = ("scan_forward", "scan_backward", "gemm_tn", "linear_project", "linear_input_grad",
            "linear_weight_grad", "bias_grad", "pack_spikes", "unpack_spikes",
            "count_rows", "count_columns", "pack_count_spikes", "izhikevich_forward")


def _traced_ops(fn, *args):
    gm = make_fx(fn, tracing_mode="fake")(*args)
    ops = {str(n.target) for n in gm.graph.nodes if n.op == "call_function"}
    return gm, {o.split(".")[1] for o in ops if o.startswith("myelin_b200.")}


def _fake(*shapes_dtypes):
    with FakeTensorMode():
        return [torch.empty(s, dtype=d, device="cuda") for s, d in shapes_dtypes]


def test_ops_are_registered():
    for name in OP_NAMES:
        assert hasattr(torch.ops.myelin_b200, name), name


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_surrogate_alif_forward_traces_to_scan_op(dtype):
    params = mb.ALIFParams(tau_mem=10.0, tau_adaptation=50.0, beta=1.8)

    def f(x, v0, a0):
        st, spikes = mb.surrogate_alif_forward(x, mb.ALIFState(v0, a0), params,
                                               surrogate="atan", reset_mode="subtract")
        return st.membrane, st.adaptation, spikes

    x, v0, a0 = _fake(((33, 4, 64), dtype), ((4, 64), dtype), ((4, 64), dtype))
    gm, ops = _traced_ops(f, x, v0, a0)
    assert ops == {"scan_forward"}
    with FakeTensorMode(allow_non_fake_inputs=True):
        vT, aT, spikes = gm(x, v0, a0)
    assert vT.shape == (4, 64) and aT.shape == (4, 64) and spikes.shape == (33, 4, 64)
    assert spikes.dtype == dtype


def test_packed_forward_and_packing_trace_to_ops():
    params = mb.LIFParams(tau_mem=10.0)

    def f(x, v0, s):
        st, packed = mb.lif_forward_packed_spikes(x, mb.LIFState(v0), params)
        p2 = mb.pack_spikes(s)
        return (packed.data, mb.unpack_spikes(p2), mb.packed_spike_count(p2),
                mb.packed_spike_count(p2, dim=(0, 1)))

    x, v0, s = _fake(((20, 3, 96), torch.float32), ((3, 96), torch.float32),
                     ((5, 3, 70), torch.bool))
    gm, ops = _traced_ops(f, x, v0, s)
    assert ops == {"scan_forward", "pack_spikes", "unpack_spikes", "count_rows", "count_columns"}
    with FakeTensorMode(allow_non_fake_inputs=True):
        words, dense, rows, cols = gm(x, v0, s)
    assert words.shape == (20, 3, 3) and words.dtype == torch.int32
    assert dense.shape == (5, 3, 70) and dense.dtype == torch.float32
    assert rows.shape == () and rows.dtype == torch.int64  # dim=None: total count
    assert cols.shape == (70,) and cols.dtype == torch.int64


def test_linear_stream_forward_traces_to_gemm_and_scan():
    params = mb.LIFParams(tau_mem=20.0)

    def f(x, w, b):
        st, spikes = mb.linear_surrogate_lif_forward(x, w, b, params, surrogate="superspike")
        return st.membrane, spikes

    x, w, b = _fake(((8, 4, 32), torch.bfloat16), ((32, 48), torch.bfloat16),
                    ((48,), torch.bfloat16))
    gm, ops = _traced_ops(f, x, w, b)
    assert ops == {"linear_project", "scan_forward"}


def test_fp32_linear_traces_to_tensor_core_projection():
    params = mb.LIFParams(tau_mem=20.0)

    def f(x, w, b):
        return mb.linear_surrogate_lif_forward(x, w, b, params)[1]

    x, w, b = _fake(((8, 4, 32), torch.float32), ((32, 48), torch.float32),
                    ((48,), torch.float32))
    _, ops = _traced_ops(f, x, w, b)
    # fp32 projection: exact 3-way bf16 splits on the library's GEMM, no torch matmul
    assert ops == {"linear_project", "scan_forward"}


@pytest.mark.parametrize("neuron", [nat.MB_LIF, nat.MB_ALIF])
def test_scan_backward_fake_shapes(neuron):
    def f(x, cv, ca, gs, gv):
        return cops.scan_backward(
            x, cv, ca, grad_spikes=gs, grad_vT=gv, neuron=neuron, decay=0.9, threshold=1.0,
            reset=0.0, adapt_decay=0.98, beta=1.8, reset_mode=nat.MB_RESET_SUBTRACT,
            surrogate=2, slope=10.0, need_v0=True, need_a0=True,
        )

    x, cv, ca, gs, gv = _fake(((40, 2, 64), torch.bfloat16), ((3, 2, 64), torch.float32),
                              ((3, 2, 64), torch.float32), ((40, 2, 64), torch.bfloat16),
                              ((2, 64), torch.bfloat16))
    gm, ops = _traced_ops(f, x, cv, ca, gs, gv)
    assert ops == {"scan_backward"}
    with FakeTensorMode(allow_non_fake_inputs=True):
        gx, gv0, ga0 = gm(x, cv, ca, gs, gv)
    assert gx.shape == x.shape and gx.dtype == x.dtype and gv0.shape == (2, 64)
    if neuron == nat.MB_ALIF:
        assert ga0.shape == (2, 64)
    else:
        assert ga0 is None  # LIF has no adaptation gradient


def test_scan_forward_fake_placeholders():
    """Outputs that were not requested come back as None from the wrapper."""

    def f(x, v0):
        return cops.scan_forward(x, v0, None, nat.MB_LIF, 0.9, 1.0, 0.0, 0.0, 0.0, 0,
                                 rates=True, checkpoints=True)

    x, v0 = _fake(((17, 2, 32), torch.float32), ((2, 32), torch.float32))
    with FakeTensorMode(allow_non_fake_inputs=True):
        vT, aT, spikes, packed, rates, ckpt_v, ckpt_a = f(x, v0)
    assert aT is None and spikes is None and packed is None and ckpt_a is None
    assert rates.shape == (2, 32) and ckpt_v.shape == (2, 2, 32)
    assert ckpt_v.dtype == torch.float32


def test_izhikevich_and_fused_pack_trace_to_ops():
    def f(x, v0, u0, s):
        st, spikes = mb.izhikevich_forward(x, mb.IzhikevichState(v0, u0), mb.IzhikevichParams())
        packed, counts = mb.pack_spikes_with_counts(s, dtype=torch.int32)
        return st.voltage, st.recovery, spikes, packed.data, counts

    x, v0, u0, s = _fake(((9, 2, 40), torch.float32), ((2, 40), torch.float32),
                         ((2, 40), torch.float32), ((3, 4, 64), torch.bool))
    gm, ops = _traced_ops(f, x, v0, u0, s)
    assert ops == {"izhikevich_forward", "pack_count_spikes"}
    with FakeTensorMode(allow_non_fake_inputs=True):
        vT, uT, spikes, words, counts = gm(x, v0, u0, s)
    assert vT.shape == (2, 40) and spikes.shape == (9, 2, 40)
    assert words.shape == (3, 4, 2) and counts.shape == (64,) and counts.dtype == torch.int32
