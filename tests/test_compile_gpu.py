"""torch.compile over the CUDA path: the ``myelin_b200::*`` ops on a B200.

``torch.library.opcheck`` validates each op's schema, fake implementation and
AOT dispatch on real CUDA inputs; compiled models (``fullgraph=True``: no graph
breaks) must give the eager results, forward and backward. The reference
offers compile visibility for its rate-training ops the same way
(src/myelin/triton/compile_ops.py:23-560, tests/test_baselines.py:12-33).
"""

from __future__ import annotations

import pytest
import torch

import myelin_b200 as mb
from myelin_b200 import _native as nat
from myelin_b200 import compile_ops as cops

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _gen(seed: int) -> torch.Generator:
    return torch.Generator(device=DEV).manual_seed(seed)


def test_opcheck_scan_ops():
    g = _gen(1)
    x = torch.randn((33, 3, 64), generator=g, device=DEV).to(torch.bfloat16)
    v0 = torch.zeros((3, 64), device=DEV, dtype=torch.bfloat16)
    a0 = torch.zeros_like(v0)
    fwd_args = (x, v0, a0, nat.MB_ALIF, 0.9, 1.0, 0.0, 0.98, 1.8, nat.MB_RESET_SUBTRACT,
                True, True, True, True)
    torch.library.opcheck(cops.scan_forward_op, fwd_args)
    outs = cops.scan_forward_op(*fwd_args)
    gs = torch.randn(x.shape, generator=g, device=DEV).to(torch.bfloat16)
    bwd_args = (x, outs[5], outs[6], gs, None, None, None, nat.MB_ALIF, 0.9, 1.0, 0.0, 0.98, 1.8,
                nat.MB_RESET_SUBTRACT, 2, 10.0, True, True, False)
    torch.library.opcheck(cops.scan_backward_op, bwd_args)


def test_opcheck_gemm_and_packing_ops():
    g = _gen(2)
    a = torch.randn((96, 64), generator=g, device=DEV).to(torch.bfloat16)
    b = torch.randn((80, 64), generator=g, device=DEV).to(torch.bfloat16)
    bias = torch.randn((80,), generator=g, device=DEV).to(torch.bfloat16)
    torch.library.opcheck(cops.gemm_tn_op, (a, b, bias))
    s = torch.rand((6, 70), generator=g, device=DEV) < 0.3
    torch.library.opcheck(cops.pack_op, (s, 6, 70))
    words = cops.pack_op(s, 6, 70)
    torch.library.opcheck(cops.unpack_op, (words, 6, 70, torch.float32))
    torch.library.opcheck(cops.count_rows_op, (words, 6, 70))
    torch.library.opcheck(cops.count_columns_op, (words, 6, 70, True))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_compiled_alif_forward_backward_matches_eager(dtype):
    params = mb.ALIFParams(tau_mem=10.0, tau_adaptation=50.0, beta=1.8)
    g = _gen(3)
    x0 = (0.2 + 0.6 * torch.randn((40, 4, 128), generator=g, device=DEV)).to(dtype)
    gs = torch.randn(x0.shape, generator=g, device=DEV).to(dtype)
    v0 = torch.zeros((4, 128), device=DEV, dtype=dtype)

    def step(x):
        st, spikes = mb.surrogate_alif_forward(x, mb.ALIFState(v0, torch.zeros_like(v0)), params,
                                               surrogate="atan", reset_mode="subtract")
        return (spikes * gs).sum() + st.membrane.float().sum(), spikes

    results = []
    for fn in (step, torch.compile(step, fullgraph=True)):
        x = x0.clone().requires_grad_(True)
        loss, spikes = fn(x)
        loss.backward()
        results.append((spikes.detach(), x.grad.detach()))
    assert torch.equal(results[0][0], results[1][0])
    assert torch.equal(results[0][1], results[1][1])  # same kernels, same bits


def test_compiled_linear_module_training_step_matches_eager():
    torch.manual_seed(4)
    layer = mb.LinearSurrogateLIF(64, 96, mb.LIFParams(tau_mem=20.0),
                                  surrogate=mb.superspike_surrogate, surrogate_slope=10.0,
                                  stream_synapse=True).to(DEV, torch.bfloat16)
    g = _gen(5)
    x = (torch.rand((12, 8, 64), generator=g, device=DEV) < 0.3).to(torch.bfloat16)

    def step(mod):
        spikes = mod(x)
        loss = spikes.float().mean(dim=0).pow(2).sum()
        loss.backward()
        return spikes.detach()

    eager_spikes = step(layer)
    eager_grads = [p.grad.clone() for p in layer.parameters()]
    layer.zero_grad(set_to_none=True)
    compiled_spikes = step(torch.compile(layer, fullgraph=True))
    assert torch.equal(eager_spikes, compiled_spikes)
    for ge, p in zip(eager_grads, layer.parameters()):
        # dW / db come from the same deterministic kernels (tensor-core GEMM,
        # fixed-order column sums) compiled or not: identical
        assert torch.equal(p.grad, ge)


def test_compiled_pack_and_count_match_eager():
    g = _gen(6)
    s = torch.rand((16, 8, 300), generator=g, device=DEV) < 0.05

    def f(spikes):
        p = mb.pack_spikes(spikes)
        return p.data, mb.packed_spike_count(p, dim=(0, 1)), mb.unpack_spikes(p, dtype=torch.bfloat16)

    for a, b in zip(f(s), torch.compile(f, fullgraph=True)(s)):
        assert torch.equal(a, b)
