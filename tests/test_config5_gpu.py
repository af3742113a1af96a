"""BASELINE config 5 layers on the GPU path, checked piece by piece.

Config 5 is a bf16 rate network: Bernoulli(0.1) input spikes [T=100, B, 2048],
hidden stream-synapse LIF layers 2048 -> 4096 and 4096 -> 4096 (superspike
surrogate, slope 10, tau_mem 20), then a 4096 -> 10 rate readout
(src/myelin/modules.py:706-845; autograd semantics src/myelin/autograd.py:445-885).
The batch is reduced from 512 to 64 per layer (M = T*B = 6400 rows) so the
fp32 references finish in seconds; the layer widths are the config's, so every
projection runs on the two-SM pair kernel exactly as in the benchmarked step.

Per layer:
- currents against an fp32 torch product of the same bf16 operands (one bf16
  rounding, 2e-2 scaled);
- spikes (or rates) bit-exact against the C oracle's scan of the GPU's own
  currents (identical inputs: the scan is exact);
- dX, dW and db against fp32 torch products of the oracle's dL/dcurrents
  (rounded to bf16, as the GPU stores them), within the bf16 bar 2e-2 (scaled).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import myelin_b200 as mb
from myelin_b200.autograd import _project
from tests.conftest import assert_close_scaled

pytestmark = pytest.mark.gpu
DEV = "cuda"
T, B = 100, 64
KW = dict(decay=np.float32(1 - 1 / 20.0), threshold=np.float32(1.0), reset=np.float32(0.0))


def host(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def _layer_params(F: int, N: int, seed: int):
    gen = torch.Generator().manual_seed(seed)
    w = torch.empty((N, F))
    torch.nn.init.kaiming_uniform_(w, a=5 ** 0.5, generator=gen)
    b = (torch.rand((N,), generator=gen) * 2 - 1) / F ** 0.5
    return w.t().contiguous().bfloat16(), b.bfloat16(), gen


def _check_layer(oracle, x: torch.Tensor, F: int, N: int, seed: int, rate: bool):
    w, b, gen = _layer_params(F, N, seed)
    xd = x.to(DEV).requires_grad_(True)
    wd, bd = w.to(DEV).requires_grad_(True), b.to(DEV).requires_grad_(True)
    params = mb.LIFParams(tau_mem=20.0, threshold=1.0, reset=0.0)
    if rate:
        _, out = mb.linear_surrogate_lif_rate_forward(
            xd, wd, bd, params, surrogate="superspike", surrogate_slope=10.0, reduction="none")
    else:
        _, out = mb.linear_surrogate_lif_forward(xd, wd, bd, params, surrogate="superspike",
                                                 surrogate_slope=10.0)
    cur = _project(xd.detach().reshape(T * B, F), wd.detach(), bd.detach())
    ref_cur = (x.float().reshape(T * B, F) @ w.float() + b.float()).bfloat16()
    assert_close_scaled(host(cur), ref_cur.float().numpy(), rtol=2e-2, what="currents")
    cur3 = host(cur).reshape(T, B, N)
    fwd = oracle.scan_forward(cur3, np.zeros((B, N), np.float32), **KW)
    if rate:
        want = (fwd["counts"].astype(np.float32) / np.float32(T))
        assert np.array_equal(host(out), torch.from_numpy(want).bfloat16().float().numpy())
        g_out = torch.randn((B, N), generator=gen).bfloat16()
        bwd = oracle.scan_backward(cur3, np.zeros((B, N), np.float32),
                                   grad_rates=g_out.float().numpy(), surrogate="superspike",
                                   slope=10.0, **KW)
    else:
        assert np.array_equal(host(out).astype(np.uint8), fwd["spikes"])
        g_out = torch.randn((T, B, N), generator=gen).bfloat16()
        bwd = oracle.scan_backward(cur3, np.zeros((B, N), np.float32),
                                   grad_spikes=g_out.float().numpy(), surrogate="superspike",
                                   slope=10.0, **KW)
    (out * g_out.to(DEV)).sum().backward()
    g_ref = torch.from_numpy(bwd["grad_x"]).bfloat16().float().reshape(T * B, N)
    dx_ref = (g_ref @ w.float().t()).reshape(T, B, F)
    dw_ref = x.float().reshape(T * B, F).t() @ g_ref
    db_ref = g_ref.sum(0)
    assert_close_scaled(host(xd.grad), dx_ref.numpy(), rtol=2e-2, what="grad_x")
    assert_close_scaled(host(wd.grad), dw_ref.numpy(), rtol=2e-2, what="grad_w")
    assert_close_scaled(host(bd.grad), db_ref.numpy(), rtol=2e-2, what="grad_b")
    return out.detach()


def test_config5_hidden_layers_and_readout(oracle):
    gen = torch.Generator().manual_seed(55)
    x = (torch.rand((T, B, 2048), generator=gen) < 0.1).bfloat16()
    h1 = _check_layer(oracle, x, 2048, 4096, 1, rate=False)
    assert 0.0 < float(h1.float().mean()) < 0.5, "layer 1 must spike, and not everywhere"
    h2 = _check_layer(oracle, h1.cpu(), 4096, 4096, 2, rate=False)
    _check_layer(oracle, h2.cpu(), 4096, 10, 3, rate=True)
