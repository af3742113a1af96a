"""GPU parity of the stream-synapse path (projection GEMM + scan) and the modules.

Golden vectors come from the reference's torch autograd functions. The
projection's fp32 summation order differs from torch's CPU matmul, so spikes
are compared by flip rate (<= 1e-6, exact at these sizes) and
gradients with the scaled fp32 tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import myelin_b200 as mb
from tests.conftest import assert_close_scaled, load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def dev(a):
    return torch.as_tensor(np.asarray(a)).to(DEV, torch.float32)


def host(t):
    return t.detach().float().cpu().numpy()


def test_linear_stream_matches_reference_golden(oracle):
    g = load_golden("linear_stream")
    x = dev(g["x"]).requires_grad_(True)
    w = dev(g["w"]).requires_grad_(True)
    b = dev(g["b"]).requires_grad_(True)
    params = mb.LIFParams(tau_mem=float(g["tau"]), threshold=float(g["thr"]), reset=float(g["reset"]))
    state, spikes = mb.linear_surrogate_lif_forward(
        x, w, b, params, surrogate="fast_sigmoid", surrogate_slope=float(g["slope"]))
    assert np.array_equal(host(spikes).astype(np.uint8), oracle.unpack(g["packed"], g["w"].shape[1]))
    np.testing.assert_allclose(host(state.membrane), g["vT"], rtol=1e-5, atol=1e-5)
    ((spikes * dev(g["grad_spikes"])).sum() + (state.membrane * dev(g["grad_vT"])).sum()).backward()
    assert_close_scaled(host(x.grad), g["grad_x"], what="grad_x")
    assert_close_scaled(host(w.grad), g["grad_w"], what="grad_w")
    assert_close_scaled(host(b.grad), g["grad_b"], what="grad_b")


def test_linear_rate_matches_reference_golden():
    g = load_golden("linear_checkpoint_rate")
    x = dev(g["x"]).requires_grad_(True)
    w = dev(g["w"]).requires_grad_(True)
    b = dev(g["b"]).requires_grad_(True)
    params = mb.LIFParams(tau_mem=float(g["tau"]), threshold=float(g["thr"]), reset=float(g["reset"]))
    state, rates = mb.linear_surrogate_lif_rate_forward(
        x, w, b, params, surrogate="superspike", surrogate_slope=float(g["slope"]),
        checkpoint_size=3, reduction="none")
    assert np.array_equal(host(rates), g["rates"])
    (rates * dev(g["grad_rates"])).sum().backward()
    assert_close_scaled(host(x.grad), g["grad_x"], what="grad_x")
    assert_close_scaled(host(w.grad), g["grad_w"], what="grad_w")
    assert_close_scaled(host(b.grad), g["grad_b"], what="grad_b")


def test_config2_shape_flip_rate_and_gradients(oracle):
    """BASELINE config 2 layer 1: Bernoulli(0.2) [25, 256, 784] @ W[784, 1024], fast_sigmoid 25."""

    T, B, F, N = 25, 256, 784, 1024
    gen = torch.Generator().manual_seed(2)
    x = (torch.rand((T, B, F), generator=gen) < 0.2).float()
    w_out_in = torch.empty((N, F))
    torch.nn.init.kaiming_uniform_(w_out_in, a=5 ** 0.5, generator=gen)
    w = w_out_in.t().contiguous()
    b = (torch.rand((N,), generator=gen) * 2 - 1) / F ** 0.5
    params = mb.LIFParams(tau_mem=20.0, threshold=1.0, reset=0.0)
    xd, wd, bd = x.to(DEV).requires_grad_(True), w.to(DEV).requires_grad_(True), b.to(DEV).requires_grad_(True)
    state, spikes = mb.linear_surrogate_lif_forward(xd, wd, bd, params, surrogate="fast_sigmoid",
                                                    surrogate_slope=25.0)
    # oracle on the GPU's own currents: the scan must be bit-exact on identical inputs
    from myelin_b200.autograd import _project

    cur = _project(xd.detach().reshape(T * B, F), wd.detach(), bd.detach()).reshape(T, B, N)
    kw = dict(decay=np.float32(1 - 1 / 20.0), threshold=np.float32(1.0), reset=np.float32(0.0))
    ref = oracle.scan_forward(host(cur), np.zeros((B, N), np.float32), **kw)
    assert np.array_equal(host(spikes).astype(np.uint8), ref["spikes"])
    # against an independent CPU projection: flip rate bar
    cur_cpu = oracle.linear_currents(x.numpy(), w.numpy(), b.numpy())
    ref_cpu = oracle.scan_forward(cur_cpu, np.zeros((B, N), np.float32), **kw)
    flips = int(np.sum(host(spikes).astype(np.uint8) != ref_cpu["spikes"]))
    assert flips / spikes.numel() <= 1e-6, f"{flips} flipped spikes of {spikes.numel()}"
    gs = torch.randn((T, B, N), generator=gen)
    (spikes * gs.to(DEV)).sum().backward()
    bwd = oracle.scan_backward(host(cur), np.zeros((B, N), np.float32), grad_spikes=gs.numpy(),
                               surrogate="fast_sigmoid", slope=25.0, **kw)
    dx, dw, db = oracle.linear_backward(x.numpy(), w.numpy(), bwd["grad_x"])
    # the north star's fp32 bar (1e-5), with the scaled floor of assert_close_scaled
    assert_close_scaled(host(xd.grad), dx, rtol=1e-5, what="grad_x")
    assert_close_scaled(host(wd.grad), dw, rtol=1e-5, what="grad_w")
    assert_close_scaled(host(bd.grad), db, rtol=1e-5, what="grad_b")
    # and the plain elementwise rtol 1e-5 pass rate, reported next to it
    for name, got, want in (("grad_x", host(xd.grad), dx), ("grad_w", host(wd.grad), dw)):
        rate = float(np.mean(np.abs(got - want) <= 1e-5 * np.abs(want) + 1e-30))
        print(f"{name}: plain rtol 1e-5 pass rate {rate:.6f}")


def test_packed_forward_matches_dense_forward():
    gen = torch.Generator().manual_seed(8)
    x = (torch.rand((12, 6, 50), generator=gen) < 0.3).float().to(DEV)
    w = (torch.randn((50, 45), generator=gen) * 0.5).to(DEV)
    b = (torch.randn((45,), generator=gen) * 0.1).to(DEV)
    params = mb.LIFParams(tau_mem=10.0)
    s1, spikes = mb.linear_surrogate_lif_forward(x, w, b, params)
    s2, packed = mb.linear_surrogate_lif_packed_forward(x, w, b, params)
    assert torch.equal(mb.unpack_spikes(packed), spikes.detach())
    assert torch.equal(s1.membrane.detach(), s2.membrane)


def test_modules_train_and_match_functional():
    torch.manual_seed(0)
    model = mb.RateReadoutClassifier(40, 64, 10, mb.LIFParams(tau_mem=10.0),
                                     backend="triton").to(DEV)
    for p in model.parameters():
        torch.nn.init.normal_(p, std=0.3)
    x = (torch.rand((20, 16, 40), device=DEV) < 0.3).float()
    target = torch.randint(0, 10, (16,), device=DEV)
    opt = torch.optim.SGD(model.parameters(), lr=0.5)
    losses = []
    for _ in range(5):
        opt.zero_grad()
        rates = model(x)
        assert rates.shape == (16, 10)
        loss = torch.nn.functional.cross_entropy(rates * 10, target)
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert all(np.isfinite(losses))
    layer = mb.LinearSurrogateLIF(40, 30, stream_synapse=True).to(DEV)
    spikes = layer(x)
    _, ref = mb.linear_surrogate_lif_forward(x, layer.synapse.weight, layer.synapse.bias,
                                             layer.unroll.cell.params)
    assert torch.equal(spikes, ref)
    unrolled = mb.LinearSurrogateLIF(40, 30, stream_synapse=False).to(DEV)
    unrolled.load_state_dict(layer.state_dict())
    assert (unrolled(x) != spikes).float().mean().item() <= 1e-3


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_16bit_stream_synapse_uses_tensor_core_projection(oracle, dtype):
    """bf16/f16 layer: projection on the tcgen05 GEMM, scan bit-exact on its currents,
    currents and gradients against an fp32 torch reference of the same op."""

    from myelin_b200.autograd import _input_grad, _project

    T, B, F, N = 12, 64, 256, 320
    gen = torch.Generator().manual_seed(5)
    x = (torch.rand((T, B, F), generator=gen) < 0.2).to(dtype)
    w = (torch.randn((F, N), generator=gen) * 0.15).to(dtype)
    b = (torch.randn((N,), generator=gen) * 0.1).to(dtype)
    xd, wd, bd = (t.to(DEV).requires_grad_(True) for t in (x, w, b))
    params = mb.LIFParams(tau_mem=20.0, threshold=1.0, reset=0.0)
    state, spikes = mb.linear_surrogate_lif_forward(xd, wd, bd, params, surrogate="fast_sigmoid",
                                                    surrogate_slope=25.0)
    cur = _project(xd.detach().reshape(T * B, F), wd.detach(), bd.detach())
    ref_cur = (x.float().reshape(T * B, F) @ w.float() + b.float()).to(dtype)
    assert_close_scaled(host(cur), ref_cur.float().numpy(), rtol=1e-2, what="currents")
    kw = dict(decay=np.float32(1 - 1 / 20.0), threshold=np.float32(1.0), reset=np.float32(0.0))
    ref = oracle.scan_forward(host(cur).reshape(T, B, N), np.zeros((B, N), np.float32), **kw)
    assert np.array_equal(host(spikes).astype(np.uint8), ref["spikes"])
    gs = torch.randn((T, B, N), generator=gen).to(dtype)
    (spikes * gs.to(DEV)).sum().backward()
    bwd = oracle.scan_backward(host(cur).reshape(T, B, N), np.zeros((B, N), np.float32),
                               grad_spikes=gs.float().numpy(), surrogate="fast_sigmoid",
                               slope=25.0, **kw)
    g_ref = torch.from_numpy(bwd["grad_x"]).to(dtype).float().reshape(T * B, N)
    dx_ref = (g_ref @ w.float().t()).reshape(T, B, F)
    dw_ref = x.float().reshape(T * B, F).t() @ g_ref
    assert_close_scaled(host(xd.grad), dx_ref.numpy(), rtol=3e-2, what="grad_x")
    assert_close_scaled(host(wd.grad), dw_ref.numpy(), rtol=3e-2, what="grad_w")
    assert_close_scaled(host(bd.grad), g_ref.sum(0).numpy(), rtol=3e-2, what="grad_b")
    g2 = torch.randn((T * B, N), device=DEV).to(dtype)
    assert_close_scaled(host(_input_grad(g2, wd.detach())),
                        (g2.float() @ wd.detach().float().t()).cpu().numpy(), rtol=1e-2)
