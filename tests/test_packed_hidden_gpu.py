"""Two-layer rate models: bit-packed hidden spikes and
whole-model backward recompute.

The reference checks its packed-hidden function against the composition of
the dense layers (tests/test_triton_lif.py:2427-2505, same shapes and
parameters here). The packed-hidden backward recomputes both projections
with the same deterministic kernels, so here the results equal the
composition bit for bit; the saved state holds no dense hidden tensor.
"""

from __future__ import annotations

import pytest
import torch

import myelin_b200 as mb

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _leaves(dtype, T, B, F, H, O, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.rand((T, B, F), generator=g, device=DEV).to(dtype)
    w1 = ((torch.rand((F, H), generator=g, device=DEV) - 0.5) * 0.04 * 20 / F ** 0.5).to(dtype)
    b1 = ((torch.rand((H,), generator=g, device=DEV) - 0.5) * 0.01).to(dtype)
    w2 = ((torch.rand((H, O), generator=g, device=DEV) - 0.5) * 0.04 * 20 / H ** 0.5).to(dtype)
    b2 = ((torch.rand((O,), generator=g, device=DEV) - 0.5) * 0.01).to(dtype)
    return [t.requires_grad_(True) for t in (x, w1, b1, w2, b2)]


def _run(fn, leaves, target):
    rates = fn(*leaves)
    loss = (rates.float() - target).square().mean()
    loss.backward()
    return rates.detach(), [None if t.grad is None else t.grad.detach() for t in leaves]


@pytest.mark.parametrize("dtype,shape", [
    (torch.float32, (6, 3, 13, 35, 5)),      # the reference test's shapes
    (torch.float32, (40, 8, 64, 96, 10)),
    (torch.bfloat16, (50, 16, 128, 256, 10)),
])
@pytest.mark.parametrize("with_bias", [True, False])
def test_packed_hidden_matches_dense_composition(dtype, shape, with_bias):
    T, B, F, H, O = shape
    params = mb.LIFParams(tau_mem=8.0, threshold=0.7, reset=-0.2)
    kw = dict(surrogate="fast_sigmoid", surrogate_slope=5.0, checkpoint_size=3)
    target = torch.linspace(0.05, 0.45, steps=B * O, device=DEV).reshape(B, O)

    def composed(x, w1, b1, w2, b2):
        _, hidden = mb.linear_surrogate_lif_forward(x, w1, b1 if with_bias else None, params, **kw)
        _, rates = mb.linear_surrogate_lif_rate_forward(hidden, w2, b2 if with_bias else None,
                                                        params, reduction="none", **kw)
        return rates

    def packed(x, w1, b1, w2, b2):
        return mb.two_layer_surrogate_lif_rate_packed_hidden_forward(
            x, w1, b1 if with_bias else None, w2, b2 if with_bias else None, params, **kw)

    def recompute(x, w1, b1, w2, b2):
        return mb.two_layer_surrogate_lif_rate_recompute_forward(
            x, w1, b1 if with_bias else None, w2, b2 if with_bias else None, params, **kw)

    leaves = _leaves(dtype, T, B, F, H, O, seed=151 + T)
    r_ref, g_ref = _run(composed, leaves, target)
    names = ("inputs", "hidden_weight", "hidden_bias", "output_weight", "output_bias")
    for fn in (packed, recompute):
        leaves2 = [t.detach().clone().requires_grad_(True) for t in leaves]
        r_act, g_act = _run(fn, leaves2, target)
        assert torch.equal(r_act, r_ref), fn.__name__
        for name, a, b in zip(names, g_act, g_ref):
            if not with_bias and name.endswith("bias"):
                continue
            assert torch.equal(a, b), (fn.__name__, name)


def test_packed_hidden_saves_bits_not_dense_hidden():
    T, B, F, H, O = 32, 8, 64, 256, 10
    params = mb.LIFParams(tau_mem=10.0, threshold=0.5)
    leaves = _leaves(torch.float32, T, B, F, H, O, seed=7)
    saved = []

    def pack_hook(t):
        saved.append((tuple(t.shape), t.dtype))
        return t

    with torch.autograd.graph.saved_tensors_hooks(pack_hook, lambda t: t):
        mb.two_layer_surrogate_lif_rate_packed_hidden_forward(*leaves, params)
    shapes = {s for s, _ in saved}
    assert (T, B, H // 32) in shapes                     # the packed words
    assert (T, B, H) not in shapes                       # no dense hidden spikes / currents
    assert (T * B, H) not in shapes
    assert all(not (len(s) == 3 and s[-1] == O and s[0] == T) for s in shapes)  # no output currents


def test_packed_hidden_rejects_soft_forward_and_bad_shapes():
    params = mb.LIFParams()
    x, w1, b1, w2, b2 = _leaves(torch.float32, 4, 2, 8, 16, 3, seed=1)
    with pytest.raises(ValueError, match="hard_forward=True"):
        mb.two_layer_surrogate_lif_rate_packed_hidden_forward(x, w1, b1, w2, b2, params,
                                                              hard_forward=False)
    with pytest.raises(ValueError, match="output_weight"):
        mb.two_layer_surrogate_lif_rate_packed_hidden_forward(x, w1, b1, w2[:5], b2, params)


def test_recompute_saves_no_hidden_spikes():
    T, B, F, H, O = 32, 8, 64, 256, 10
    params = mb.LIFParams(tau_mem=10.0, threshold=0.5)
    leaves = _leaves(torch.float32, T, B, F, H, O, seed=9)
    saved = []
    with torch.autograd.graph.saved_tensors_hooks(lambda t: saved.append(tuple(t.shape)) or t,
                                                  lambda t: t):
        mb.two_layer_surrogate_lif_rate_recompute_forward(*leaves, params)
    assert (T, B, H // 32) not in saved and (T, B, H) not in saved
