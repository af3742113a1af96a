"""Pin the CPU oracle against golden vectors produced by the reference itself.

Fixtures come from ``tests/golden/make_golden.py`` (the reference's own torch
functions). Forward spikes and plain-forward final states must be bit-exact;
surrogate gradients (torch autograd in the reference, closed form here) agree
to rtol 1e-5 with an absolute floor of 1e-5 x max|grad| (``assert_close_scaled``).
"""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest
import torch

from tests.conftest import GOLDEN, assert_close_scaled, load_golden

SURROGATES = ("sigmoid", "fast_sigmoid", "atan", "triangular", "superspike", "multi_gaussian")


def f32(v) -> np.float32:
    return np.float32(float(v))


def lif_decay(tau: float) -> np.float32:
    return np.float32(1.0 - 1.0 / float(tau))


@pytest.mark.parametrize("name", ["lif_fwd_a", "lif_fwd_b"])
def test_lif_forward_bit_exact(oracle, name):
    g = load_golden(name)
    out = oracle.scan_forward(g["x"], g["v0"], decay=lif_decay(g["tau"]), threshold=f32(g["thr"]),
                              reset=f32(g["reset"]))
    assert np.array_equal(oracle.pack(out["spikes"]), g["packed"])
    assert np.array_equal(out["vT"], g["vT"])


@pytest.mark.parametrize("name", ["alif_fwd_a", "alif_fwd_b"])
def test_alif_forward_bit_exact(oracle, name):
    g = load_golden(name)
    out = oracle.scan_forward(
        g["x"], g["v0"], g["a0"], neuron=oracle.ALIF, decay=lif_decay(g["tau_mem"]),
        threshold=f32(g["threshold"]), reset=f32(g["reset"]),
        adapt_decay=lif_decay(g["tau_adaptation"]), beta=f32(g["beta"]),
    )
    assert np.array_equal(oracle.pack(out["spikes"]), g["packed"])
    assert np.array_equal(out["vT"], g["vT"])
    assert np.array_equal(out["aT"], g["aT"])


@pytest.mark.parametrize("name", ["alif_subtract_dsl_a", "alif_subtract_dsl_b"])
def test_alif_subtract_forward_bit_exact_with_reference_dsl(oracle, name):
    """The subtractive-reset forward (the headline workload's reset rule)
    against the reference's own custom-neuron evaluator
    (src/myelin/dsl.py:457-511) on an ALIF IR with
    ``where(spike, pre_reset - adaptive_threshold, pre_reset)``."""

    g = load_golden(name)
    out = oracle.scan_forward(
        g["x"], g["v0"], g["a0"], neuron=oracle.ALIF, reset_mode=oracle.SUBTRACT,
        decay=lif_decay(g["tau_mem"]), threshold=f32(g["threshold"]), reset=f32(g["reset"]),
        adapt_decay=lif_decay(g["tau_adaptation"]), beta=f32(g["beta"]),
    )
    assert int(out["spikes"].sum()) == int(g["spike_count"]) > 0
    assert np.array_equal(oracle.pack(out["spikes"]), g["packed"])
    assert np.array_equal(out["vT"], g["vT"])
    assert np.array_equal(out["aT"], g["aT"])


@pytest.mark.parametrize("surrogate", SURROGATES)
@pytest.mark.parametrize("chunk", [1, 5, 16])
def test_surrogate_lif_backward_matches_reference_autograd(oracle, surrogate, chunk):
    g = load_golden(f"surrogate_lif_{surrogate}")
    kw = dict(decay=lif_decay(g["tau"]), threshold=f32(g["thr"]), reset=f32(g["reset"]))
    fwd = oracle.scan_forward(g["x"], g["v0"], **kw)
    assert np.array_equal(oracle.pack(fwd["spikes"]), g["packed"])
    # reference surrogate spikes are {0, 1 - 1ulp}; membranes differ by <= 2.4e-7 (hard reset)
    np.testing.assert_allclose(fwd["vT"], g["vT"], rtol=0, atol=1e-6)
    bwd = oracle.scan_backward(
        g["x"], g["v0"], grad_spikes=g["grad_spikes"], grad_vT=g["grad_vT"],
        surrogate=surrogate, slope=float(g["slope"]), chunk=chunk, **kw,
    )
    assert_close_scaled(bwd["grad_x"], g["grad_x"], what="grad_x")
    assert_close_scaled(bwd["grad_v0"], g["grad_v0"], what="grad_v0")


def _alif_kw(oracle, g, reset_mode):
    return dict(
        neuron=oracle.ALIF, reset_mode=reset_mode, decay=lif_decay(g["tau_mem"]),
        threshold=f32(g["threshold"]), reset=f32(g["reset"]),
        adapt_decay=lif_decay(g["tau_adaptation"]), beta=f32(g["beta"]),
    )


@pytest.mark.parametrize("name", [f"surrogate_alif_{s}" for s in SURROGATES] + ["alif_subtract_atan"])
def test_surrogate_alif_backward_matches_autograd(oracle, name):
    g = load_golden(name)
    reset_mode = oracle.SUBTRACT if "subtract" in name else oracle.HARD
    surrogate = name.rsplit("_", 1)[-1] if "subtract" in name else name[len("surrogate_alif_"):]
    kw = _alif_kw(oracle, g, reset_mode)
    fwd = oracle.scan_forward(g["x"], g["v0"], g["a0"], **kw)
    assert np.array_equal(oracle.pack(fwd["spikes"]), g["packed"])
    np.testing.assert_allclose(fwd["vT"], g["vT"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(fwd["aT"], g["aT"], rtol=0, atol=1e-5)
    bwd = oracle.scan_backward(
        g["x"], g["v0"], g["a0"], grad_spikes=g["grad_spikes"], grad_vT=g["grad_vT"],
        grad_aT=g["grad_aT"], surrogate=surrogate, slope=float(g["slope"]), **kw,
    )
    assert_close_scaled(bwd["grad_x"], g["grad_x"], what="grad_x")
    assert_close_scaled(bwd["grad_v0"], g["grad_v0"], what="grad_v0")
    assert_close_scaled(bwd["grad_a0"], g["grad_a0"], what="grad_a0")


def test_linear_stream_matches_reference(oracle):
    g = load_golden("linear_stream")
    kw = dict(decay=lif_decay(g["tau"]), threshold=f32(g["thr"]), reset=f32(g["reset"]))
    cur = oracle.linear_currents(g["x"], g["w"], g["b"])
    T, B, _ = g["x"].shape
    v0 = np.zeros((B, g["w"].shape[1]), np.float32)
    fwd = oracle.scan_forward(cur, v0, **kw)
    assert np.array_equal(oracle.pack(fwd["spikes"]), g["packed"])
    np.testing.assert_allclose(fwd["vT"], g["vT"], rtol=1e-5, atol=1e-5)
    bwd = oracle.scan_backward(cur, v0, grad_spikes=g["grad_spikes"], grad_vT=g["grad_vT"],
                               surrogate="fast_sigmoid", slope=float(g["slope"]), **kw)
    dx, dw, db = oracle.linear_backward(g["x"], g["w"], bwd["grad_x"])
    np.testing.assert_allclose(dx, g["grad_x"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(dw, g["grad_w"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(db, g["grad_b"], rtol=1e-4, atol=1e-5)


def test_linear_checkpoint_rate_matches_reference(oracle):
    g = load_golden("linear_checkpoint_rate")
    kw = dict(decay=lif_decay(g["tau"]), threshold=f32(g["thr"]), reset=f32(g["reset"]))
    cur = oracle.linear_currents(g["x"], g["w"], g["b"])
    T, B, _ = g["x"].shape
    v0 = np.zeros((B, g["w"].shape[1]), np.float32)
    fwd = oracle.scan_forward(cur, v0, **kw)
    rates = (fwd["counts"].astype(np.float32) / np.float32(T)).astype(np.float32)
    np.testing.assert_array_equal(rates, g["rates"])
    bwd = oracle.scan_backward(cur, v0, grad_rates=g["grad_rates"], surrogate="superspike",
                               slope=float(g["slope"]), **kw)
    dx, dw, db = oracle.linear_backward(g["x"], g["w"], bwd["grad_x"])
    np.testing.assert_allclose(dx, g["grad_x"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(dw, g["grad_w"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(db, g["grad_b"], rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("n", [1, 31, 32, 33, 65, 100])
def test_packing_matches_reference(oracle, n):
    g = load_golden("packing")
    words = oracle.pack(g[f"spikes_{n}"])
    assert words.dtype == np.int32
    assert np.array_equal(words, g[f"packed_{n}"])
    assert np.array_equal(oracle.count_rows(words, n), g[f"rows_{n}"])
    assert np.array_equal(oracle.count_columns(words, n), g[f"cols_{n}"])
    assert int(oracle.count_rows(words, n).sum()) == int(g[f"total_{n}"])
    assert np.array_equal(oracle.unpack(words, n), (g[f"spikes_{n}"] != 0).astype(np.uint8))


def test_packing_high_bit_is_negative(oracle):
    g = load_golden("packing")
    spikes = np.zeros((1, 32), np.float32)
    spikes[0, -1] = 1.0
    assert oracle.pack(spikes)[0, 0] == -(1 << 31) == g["high_bit_word"][0, 0]


def c1_input() -> torch.Tensor:
    gen = torch.Generator()
    gen.manual_seed(0)
    return torch.randn((64, 32, 1024), generator=gen) * 0.5 + 0.3


def test_c1_full_size_checksum(oracle):
    """BASELINE config 1 at full size: oracle spikes and membrane hash-identical to lif_unroll."""

    record = json.loads((GOLDEN / "c1_checksum.json").read_text())
    x = c1_input().numpy()
    if hashlib.sha256(x.tobytes()).hexdigest() != record["input_sha256"]:
        pytest.skip("torch.randn stream differs from the one the checksum was made with")
    out = oracle.scan_forward(x, np.zeros((32, 1024), np.float32), decay=lif_decay(10.0),
                              threshold=np.float32(1.0), reset=np.float32(0.0))
    assert hashlib.sha256(oracle.pack(out["spikes"]).tobytes()).hexdigest() == record["packed_sha256"]
    assert hashlib.sha256(out["vT"].tobytes()).hexdigest() == record["vT_sha256"]
    assert int(out["spikes"].sum()) == record["spike_count"]


# Known answers of the reference's own unit tests (tests/test_lif_reference.py:15-113).
def test_known_answer_lif_step_hard_reset(oracle):
    x = np.array([[[0.6, 0.2]]], np.float32)
    out = oracle.scan_forward(x, np.array([[0.5, 0.0]], np.float32), decay=lif_decay(10.0),
                              threshold=np.float32(1.0), reset=np.float32(-0.25))
    assert out["spikes"].tolist() == [[[1, 0]]]
    np.testing.assert_allclose(out["vT"], [[-0.25, 0.2]], rtol=1e-6)


def test_known_answer_alif_adaptation(oracle):
    kw = dict(neuron=oracle.ALIF, decay=lif_decay(10.0), threshold=np.float32(1.0),
              reset=np.float32(-0.25), adapt_decay=lif_decay(5.0), beta=np.float32(1.0))
    out = oracle.scan_forward(np.array([[[0.7, 0.8]]], np.float32), np.array([[0.5, 0.0]], np.float32),
                              np.array([[0.2, 0.0]], np.float32), **kw)
    assert out["spikes"].tolist() == [[[0, 0]]]
    np.testing.assert_allclose(out["vT"], [[1.15, 0.8]], rtol=1e-6)
    np.testing.assert_allclose(out["aT"], [[0.16, 0.0]], rtol=1e-6)
    kw.update(reset=np.float32(0.0), beta=np.float32(0.5))
    out = oracle.scan_forward(np.array([[[0.7, 1.1]]], np.float32), np.array([[0.5, 0.0]], np.float32),
                              np.array([[0.1, 0.0]], np.float32), **kw)
    assert out["spikes"].tolist() == [[[1, 1]]]
    assert np.array_equal(out["vT"], np.zeros((1, 2), np.float32))
    np.testing.assert_allclose(out["aT"], [[1.08, 1.0]], rtol=1e-6)


def test_oracle_chunk_size_does_not_change_gradients(oracle):
    rng = np.random.default_rng(7)
    x = rng.normal(0.3, 0.5, (37, 2, 29)).astype(np.float32)
    v0 = np.zeros((2, 29), np.float32)
    gs = rng.normal(0, 1, x.shape).astype(np.float32)
    kw = dict(decay=lif_decay(10.0), threshold=np.float32(1.0), reset=np.float32(0.0),
              grad_spikes=gs, surrogate="atan", slope=10.0)
    a = oracle.scan_backward(x, v0, chunk=1, **kw)["grad_x"]
    b = oracle.scan_backward(x, v0, chunk=16, **kw)["grad_x"]
    assert np.array_equal(a, b)


@pytest.mark.parametrize("name", ["izhikevich_a", "izhikevich_b"])
def test_izhikevich_oracle_matches_reference_golden(oracle, name):
    g = load_golden(name)
    params = {k: float(g[k]) for k in oracle.IZHIKEVICH_FIELDS}
    spikes, vT, uT = oracle.izhikevich_forward(g["x"], g["v0"], g["u0"], params)
    assert np.array_equal(oracle.pack(spikes), g["packed"])
    assert np.array_equal(vT, g["vT"])
    assert np.array_equal(uT, g["uT"])


def test_torch_path_port_matches_reference_fixture():
    """The torch restatement that bench.py times as myelin's torch CPU path
    (oracle/torch_path.py) computes what the reference's loop computes: same
    spikes, final state and autograd gradients as the fixture made with the
    reference's own ``hard_surrogate_spike`` and atan surrogate."""

    from oracle import torch_path

    g = load_golden("alif_subtract_atan")
    x = torch.from_numpy(g["x"]).requires_grad_(True)
    v0 = torch.from_numpy(g["v0"]).requires_grad_(True)
    a0 = torch.from_numpy(g["a0"]).requires_grad_(True)
    m, a, spikes = torch_path.alif_atan_unroll(
        x, v0, a0, decay=1.0 - 1.0 / float(g["tau_mem"]), threshold=float(g["threshold"]),
        beta=float(g["beta"]), adaptation_decay=1.0 - 1.0 / float(g["tau_adaptation"]),
        reset=float(g["reset"]), slope=float(g["slope"]), subtract=True)
    from oracle import oracle as o

    assert np.array_equal(o.pack(spikes.detach().numpy()), g["packed"])
    np.testing.assert_allclose(m.detach().numpy(), g["vT"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(a.detach().numpy(), g["aT"], rtol=0, atol=1e-6)
    loss = ((spikes * torch.from_numpy(g["grad_spikes"])).sum()
            + (m * torch.from_numpy(g["grad_vT"])).sum() + (a * torch.from_numpy(g["grad_aT"])).sum())
    gx, gv0, ga0 = torch.autograd.grad(loss, (x, v0, a0))
    assert_close_scaled(gx.numpy(), g["grad_x"], what="grad_x")
    assert_close_scaled(gv0.numpy(), g["grad_v0"], what="grad_v0")
    assert_close_scaled(ga0.numpy(), g["grad_a0"], what="grad_a0")
