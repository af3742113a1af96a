"""Izhikevich forward on the GPU through the C ABI.

Bit-exact against the reference's own golden vectors (functional.izhikevich_unroll,
src/myelin/functional.py:81-112) and against the float32 oracle on seeded
inputs: the pair path (even B*N, aligned) and the scalar path (odd B*N),
T not a multiple of the kernel's unroll, and 16-bit inputs (fp32 carry, so
the oracle runs on the upcast inputs and the states are compared after the
same rounding).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import myelin_b200 as mb
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda"
FIELDS = ("recovery_decay", "recovery_coupling", "reset_voltage", "recovery_jump", "threshold",
          "dt", "voltage_square_coeff", "voltage_coeff", "voltage_bias")


@pytest.mark.parametrize("name", ["izhikevich_a", "izhikevich_b"])
def test_izhikevich_matches_reference_golden(oracle, name):
    g = load_golden(name)
    params = mb.IzhikevichParams(**{k: float(g[k]) for k in FIELDS})
    state, spikes = mb.izhikevich_forward(
        torch.from_numpy(g["x"]).to(DEV),
        mb.IzhikevichState(torch.from_numpy(g["v0"]).to(DEV), torch.from_numpy(g["u0"]).to(DEV)),
        params,
    )
    assert spikes.dtype == torch.float32
    assert np.array_equal(oracle.pack(spikes.cpu().numpy()), g["packed"])
    assert np.array_equal(state.voltage.cpu().numpy(), g["vT"])
    assert np.array_equal(state.recovery.cpu().numpy(), g["uT"])


def _inputs(shape, seed, dtype):
    gen = torch.Generator().manual_seed(seed)
    T, B, N = shape
    x = (torch.randn(shape, generator=gen) * 5.0 + 9.0).to(dtype)
    v0 = (-65.0 + torch.rand((B, N), generator=gen) * 20.0).to(dtype)
    u0 = (0.2 * v0.float() + torch.rand((B, N), generator=gen)).to(dtype)
    return x, v0, u0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(1, 1, 1), (13, 3, 5), (64, 4, 96), (101, 2, 4096),
                                   (37, 7, 33), (0, 2, 8)])
def test_izhikevich_matches_oracle(oracle, dtype, shape):
    x, v0, u0 = _inputs(shape, hash((shape, str(dtype))) % 1000, dtype)
    params = mb.IzhikevichParams(dt=0.5, threshold=28.0)
    state, spikes = mb.izhikevich_forward(
        x.to(DEV), mb.IzhikevichState(v0.to(DEV), u0.to(DEV)), params)
    pdict = {k: getattr(params, k) for k in FIELDS}
    es, ev, eu = oracle.izhikevich_forward(x.float().numpy(), v0.float().numpy(),
                                           u0.float().numpy(), pdict)
    assert spikes.dtype == dtype and spikes.shape == x.shape
    assert np.array_equal(spikes.float().cpu().numpy(), es)
    # fp32 carry: final states equal the oracle's after one rounding to dtype
    assert torch.equal(state.voltage.cpu(), torch.from_numpy(ev).to(dtype))
    assert torch.equal(state.recovery.cpu(), torch.from_numpy(eu).to(dtype))


def test_izhikevich_step_and_cell_match_oracle(oracle):
    x, v0, u0 = _inputs((1, 6, 50), 3, torch.float32)
    params = mb.IzhikevichParams()
    pdict = {k: getattr(params, k) for k in FIELDS}
    es, ev, eu = oracle.izhikevich_forward(x.numpy(), v0.numpy(), u0.numpy(), pdict)
    st = mb.IzhikevichState(v0.to(DEV), u0.to(DEV))
    for new_state, spike in (mb.izhikevich_step(st, x[0].to(DEV), params),
                             mb.IzhikevichCell(params)(st, x[0].to(DEV))):
        assert np.array_equal(spike.cpu().numpy(), es[0])
        assert np.array_equal(new_state.voltage.cpu().numpy(), ev)
        assert np.array_equal(new_state.recovery.cpu().numpy(), eu)


def test_izhikevich_errors():
    x, v0, u0 = _inputs((4, 2, 3), 1, torch.float32)
    state = mb.IzhikevichState(v0.to(DEV), u0.to(DEV))
    with pytest.raises(ValueError, match="dt must be positive"):
        mb.izhikevich_forward(x.to(DEV), state, mb.IzhikevichParams(dt=0.0))
    with pytest.raises(ValueError, match=r"\[T, B, N\]"):
        mb.izhikevich_forward(x[0].to(DEV), state, mb.IzhikevichParams())
    with pytest.raises(ValueError, match="initial_state.recovery must match"):
        mb.izhikevich_forward(x.to(DEV), mb.IzhikevichState(v0.to(DEV), u0[:1].to(DEV)),
                              mb.IzhikevichParams())
    with pytest.raises(ValueError):
        mb.izhikevich_forward(x, mb.IzhikevichState(v0, u0), mb.IzhikevichParams())  # CPU
    with pytest.raises(ValueError, match="same shape"):
        mb.izhikevich_step(state, x[0, :1].to(DEV), mb.IzhikevichParams())


def test_izhikevich_config_size_throughput_sanity():
    """Full north-star shape (T=256, B=128, N=4096, fp32): runs, spikes some,
    and keeps the device status clean."""

    from myelin_b200 import _native as nat

    g = torch.Generator(device=DEV).manual_seed(0)
    x = torch.randn((256, 128, 4096), generator=g, device=DEV) * 5.0 + 9.0
    v0 = torch.full((128, 4096), -65.0, device=DEV)
    state, spikes = mb.izhikevich_forward(x, mb.IzhikevichState(v0, 0.2 * v0),
                                          mb.IzhikevichParams())
    torch.cuda.synchronize()
    assert 0 < float(spikes.mean()) < 0.5
    assert nat.device_status(clear=True) == 0
