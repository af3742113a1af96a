"""GPU parity of the LIF/ALIF scan (forward and surrogate backward) through the C ABI.

Bars: spikes and packed words bit-exact; fp32 final states bit-exact for the
plain forward; fp32 gradients within rtol 1e-5 (scaled, see
``assert_close_scaled``); 16-bit I/O compared with the fp32-carry oracle run on
the upcast inputs, outputs within 2e-2 (the bf16 bar).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import myelin_b200 as mb
from myelin_b200 import _native as nat
from tests.conftest import assert_close_scaled, load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda"
SURROGATES = ("sigmoid", "fast_sigmoid", "atan", "triangular", "superspike", "multi_gaussian")


@pytest.fixture(autouse=True)
def _device_status_clean():
    nat.device_status(clear=True)
    yield
    torch.cuda.synchronize()
    assert nat.device_status(clear=True) == 0, "a bounded wait in a scan kernel ran out"


def dev(a, dtype=torch.float32):
    return torch.as_tensor(np.asarray(a)).to(DEV, dtype)


def host(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def dec(tau) -> np.float32:
    return np.float32(1.0 - 1.0 / float(tau))


# ---------------------------------------------------------------------------
# golden vectors from the reference
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("name", ["lif_fwd_a", "lif_fwd_b"])
def test_lif_forward_matches_reference_golden(oracle, name):
    g = load_golden(name)
    params = mb.LIFParams(tau_mem=float(g["tau"]), threshold=float(g["thr"]), reset=float(g["reset"]))
    state, spikes = mb.lif_forward(dev(g["x"]), mb.LIFState(dev(g["v0"])), params)
    n = g["x"].shape[-1]
    assert np.array_equal(host(spikes).astype(np.uint8), oracle.unpack(g["packed"], n))
    assert np.array_equal(host(state.membrane), g["vT"])
    state2, packed = mb.lif_forward_packed_spikes(dev(g["x"]), mb.LIFState(dev(g["v0"])), params)
    assert np.array_equal(packed.data.cpu().numpy(), g["packed"])
    assert np.array_equal(host(state2.membrane), g["vT"])


@pytest.mark.parametrize("name", ["alif_fwd_a", "alif_fwd_b"])
def test_alif_forward_matches_reference_golden(oracle, name):
    g = load_golden(name)
    params = mb.ALIFParams(tau_mem=float(g["tau_mem"]), tau_adaptation=float(g["tau_adaptation"]),
                           threshold=float(g["threshold"]), reset=float(g["reset"]),
                           beta=float(g["beta"]))
    state, spikes = mb.alif_forward(dev(g["x"]), mb.ALIFState(dev(g["v0"]), dev(g["a0"])), params)
    assert np.array_equal(host(spikes).astype(np.uint8), oracle.unpack(g["packed"], g["x"].shape[-1]))
    assert np.array_equal(host(state.membrane), g["vT"])
    assert np.array_equal(host(state.adaptation), g["aT"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("name", ["alif_subtract_dsl_a", "alif_subtract_dsl_b"])
def test_alif_subtract_forward_matches_reference_dsl(oracle, name, dtype):
    """Subtractive reset (the headline workload's reset rule) against the
    reference's own custom-neuron evaluator (src/myelin/dsl.py:457-511) on an
    ALIF IR with ``where(spike, pre_reset - adaptive_threshold, pre_reset)``.
    Spikes bit-exact; final states bit-exact in fp32 and equal to the rounded
    fp32 result in bf16 (fp32 carry). Case ``b`` (T=96) holds bf16-representable
    inputs; case ``a`` runs in fp32 only."""

    g = load_golden(name)
    if dtype == torch.bfloat16 and not name.endswith("_b"):
        pytest.skip("inputs of this case are not bf16-representable")
    params = mb.ALIFParams(tau_mem=float(g["tau_mem"]), tau_adaptation=float(g["tau_adaptation"]),
                           threshold=float(g["threshold"]), reset=float(g["reset"]),
                           beta=float(g["beta"]))
    n = g["x"].shape[-1]
    state0 = mb.ALIFState(dev(g["v0"], dtype), dev(g["a0"], dtype))
    runs = {
        "alif_forward": lambda: mb.alif_forward(dev(g["x"], dtype), state0, params,
                                                reset_mode="subtract"),
        "surrogate_alif_forward": lambda: mb.surrogate_alif_forward(
            dev(g["x"], dtype), state0, params, surrogate="atan", checkpoint_size="memory",
            reset_mode="subtract"),
    }
    for what, run in runs.items():
        state, spikes = run()
        assert np.array_equal(host(spikes).astype(np.uint8), oracle.unpack(g["packed"], n)), what
        want_v = torch.from_numpy(g["vT"]).to(dtype).float().numpy()
        want_a = torch.from_numpy(g["aT"]).to(dtype).float().numpy()
        assert np.array_equal(host(state.membrane), want_v), what
        assert np.array_equal(host(state.adaptation), want_a), what


@pytest.mark.parametrize("surrogate", SURROGATES)
def test_surrogate_lif_gradients_match_reference_golden(oracle, surrogate):
    g = load_golden(f"surrogate_lif_{surrogate}")
    x = dev(g["x"]).requires_grad_(True)
    v0 = dev(g["v0"]).requires_grad_(True)
    params = mb.LIFParams(tau_mem=float(g["tau"]), threshold=float(g["thr"]), reset=float(g["reset"]))
    state, spikes = mb.surrogate_lif_forward(x, mb.LIFState(v0), params, surrogate=surrogate,
                                             surrogate_slope=float(g["slope"]))
    assert np.array_equal(host(spikes).astype(np.uint8), oracle.unpack(g["packed"], g["x"].shape[-1]))
    # reference surrogate spikes are {0, 1 - 1 ulp}
    np.testing.assert_allclose(host(spikes), g["spikes"], rtol=0, atol=1.2e-7)
    np.testing.assert_allclose(host(state.membrane), g["vT"], rtol=0, atol=1e-6)
    loss = (spikes * dev(g["grad_spikes"])).sum() + (state.membrane * dev(g["grad_vT"])).sum()
    loss.backward()
    assert_close_scaled(host(x.grad), g["grad_x"], what="grad_x")
    assert_close_scaled(host(v0.grad), g["grad_v0"], what="grad_v0")


@pytest.mark.parametrize("name", [f"surrogate_alif_{s}" for s in SURROGATES] + ["alif_subtract_atan"])
def test_surrogate_alif_gradients_match_golden(oracle, name):
    g = load_golden(name)
    subtract = "subtract" in name
    surrogate = "atan" if subtract else name[len("surrogate_alif_"):]
    x = dev(g["x"]).requires_grad_(True)
    v0 = dev(g["v0"]).requires_grad_(True)
    a0 = dev(g["a0"]).requires_grad_(True)
    params = mb.ALIFParams(tau_mem=float(g["tau_mem"]), tau_adaptation=float(g["tau_adaptation"]),
                           threshold=float(g["threshold"]), reset=float(g["reset"]),
                           beta=float(g["beta"]))
    state, spikes = mb.surrogate_alif_forward(
        x, mb.ALIFState(v0, a0), params, surrogate=surrogate, surrogate_slope=float(g["slope"]),
        reset_mode="subtract" if subtract else "hard", checkpoint_size="memory",
    )
    assert np.array_equal(host(spikes).astype(np.uint8), oracle.unpack(g["packed"], g["x"].shape[-1]))
    loss = ((spikes * dev(g["grad_spikes"])).sum() + (state.membrane * dev(g["grad_vT"])).sum()
            + (state.adaptation * dev(g["grad_aT"])).sum())
    loss.backward()
    assert_close_scaled(host(x.grad), g["grad_x"], what="grad_x")
    assert_close_scaled(host(v0.grad), g["grad_v0"], what="grad_v0")
    assert_close_scaled(host(a0.grad), g["grad_a0"], what="grad_a0")


def test_c1_full_size_matches_reference_checksum(oracle):
    import hashlib
    import json

    from tests.conftest import GOLDEN

    record = json.loads((GOLDEN / "c1_checksum.json").read_text())
    gen = torch.Generator()
    gen.manual_seed(0)
    x = torch.randn((64, 32, 1024), generator=gen) * 0.5 + 0.3
    if hashlib.sha256(x.numpy().tobytes()).hexdigest() != record["input_sha256"]:
        pytest.skip("torch.randn stream differs from the checksum's")
    params = mb.LIFParams(tau_mem=10.0, threshold=1.0, reset=0.0)
    v0 = torch.zeros((32, 1024), device=DEV)
    state, packed = mb.lif_forward_packed_spikes(x.to(DEV), mb.LIFState(v0), params)
    assert hashlib.sha256(packed.data.cpu().numpy().tobytes()).hexdigest() == record["packed_sha256"]
    assert hashlib.sha256(host(state.membrane).tobytes()).hexdigest() == record["vT_sha256"]
    state, spikes = mb.lif_forward(x.to(DEV), mb.LIFState(v0), params)
    assert int(spikes.sum().item()) == record["spike_count"]


# ---------------------------------------------------------------------------
# oracle sweeps: shapes, dtypes, neuron models, reset modes, code paths
# ---------------------------------------------------------------------------

SHAPES = [(1, 1, 1), (7, 3, 19), (5, 2, 35), (16, 4, 32), (33, 5, 64), (17, 3, 4100), (40, 8, 96)]
DTYPES = [torch.float32, torch.bfloat16, torch.float16]


def _inputs(shape, dtype, seed, alif):
    gen = torch.Generator().manual_seed(seed)
    T, B, N = shape
    x = (torch.randn(shape, generator=gen) * 0.6 + 0.25).to(dtype)
    v0 = (torch.rand((B, N), generator=gen) * 0.3).to(dtype)
    a0 = (torch.rand((B, N), generator=gen) * 0.3).to(dtype) if alif else None
    return x, v0, a0


def _round(a: np.ndarray, dtype) -> np.ndarray:
    return torch.from_numpy(a).to(dtype).float().numpy()


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("neuron", ["lif", "alif"])
@pytest.mark.parametrize("reset_mode", ["hard", "subtract"])
def test_forward_bit_exact_vs_oracle(oracle, shape, dtype, neuron, reset_mode):
    alif = neuron == "alif"
    x, v0, a0 = _inputs(shape, dtype, hash((shape, neuron)) % 1000, alif)
    okw = dict(neuron=oracle.ALIF if alif else oracle.LIF,
               reset_mode=oracle.SUBTRACT if reset_mode == "subtract" else oracle.HARD,
               decay=dec(10.0), threshold=np.float32(1.0), reset=np.float32(-0.1))
    if alif:
        params = mb.ALIFParams(tau_mem=10.0, tau_adaptation=50.0, threshold=1.0, reset=-0.1, beta=1.8)
        okw.update(adapt_decay=dec(50.0), beta=np.float32(1.8))
        ref = oracle.scan_forward(x.float().numpy(), v0.float().numpy(), a0.float().numpy(), **okw)
        state, spikes = mb.alif_forward(x.to(DEV), mb.ALIFState(v0.to(DEV), a0.to(DEV)), params,
                                        reset_mode=reset_mode)
        assert np.array_equal(host(state.adaptation), _round(ref["aT"], dtype))
    else:
        params = mb.LIFParams(tau_mem=10.0, threshold=1.0, reset=-0.1)
        ref = oracle.scan_forward(x.float().numpy(), v0.float().numpy(), **okw)
        state, spikes = mb.lif_forward(x.to(DEV), mb.LIFState(v0.to(DEV)), params,
                                       reset_mode=reset_mode)
        _, packed = mb.lif_forward_packed_spikes(x.to(DEV), mb.LIFState(v0.to(DEV)), params,
                                                 reset_mode=reset_mode)
        assert np.array_equal(packed.data.cpu().numpy(), oracle.pack(ref["spikes"]))
    assert spikes.dtype == dtype
    assert np.array_equal(host(spikes).astype(np.uint8), ref["spikes"])
    assert np.array_equal(host(state.membrane), _round(ref["vT"], dtype))


def test_forward_misaligned_base_pointer_takes_fallback_path(oracle):
    T, B, N = 20, 4, 64
    storage = torch.randn(T * B * N + 1, device=DEV) * 0.6 + 0.3
    x = storage[1:].view(T, B, N)  # contiguous, base not 16-byte aligned
    params = mb.LIFParams(tau_mem=10.0, threshold=1.0, reset=0.0)
    state, spikes = mb.lif_forward(x, mb.LIFState(torch.zeros((B, N), device=DEV)), params)
    ref = oracle.scan_forward(host(x), np.zeros((B, N), np.float32), decay=dec(10.0),
                              threshold=np.float32(1.0), reset=np.float32(0.0))
    assert np.array_equal(host(spikes).astype(np.uint8), ref["spikes"])
    assert np.array_equal(host(state.membrane), ref["vT"])


@pytest.mark.parametrize("shape", [(1, 2, 3), (7, 3, 19), (16, 4, 32), (37, 5, 96), (50, 8, 300)])
@pytest.mark.parametrize("neuron", ["lif", "alif"])
@pytest.mark.parametrize("reset_mode", ["hard", "subtract"])
@pytest.mark.parametrize("surrogate", ["atan", "sigmoid", "multi_gaussian"])
def test_fp32_gradients_vs_oracle(oracle, shape, neuron, reset_mode, surrogate):
    alif = neuron == "alif"
    x, v0, a0 = _inputs(shape, torch.float32, 11, alif)
    gen = torch.Generator().manual_seed(12)
    gs = torch.randn(shape, generator=gen)
    gv = torch.randn(shape[1:], generator=gen)
    ga = torch.randn(shape[1:], generator=gen)
    okw = dict(neuron=oracle.ALIF if alif else oracle.LIF,
               reset_mode=oracle.SUBTRACT if reset_mode == "subtract" else oracle.HARD,
               decay=dec(10.0), threshold=np.float32(1.0), reset=np.float32(0.0),
               surrogate=surrogate, slope=10.0)
    xd = x.to(DEV).requires_grad_(True)
    vd = v0.to(DEV).requires_grad_(True)
    if alif:
        ad = a0.to(DEV).requires_grad_(True)
        params = mb.ALIFParams(tau_mem=10.0, tau_adaptation=50.0, threshold=1.0, reset=0.0, beta=1.8)
        okw.update(adapt_decay=dec(50.0), beta=np.float32(1.8))
        state, spikes = mb.surrogate_alif_forward(xd, mb.ALIFState(vd, ad), params, surrogate=surrogate,
                                                  reset_mode=reset_mode)
        loss = ((spikes * gs.to(DEV)).sum() + (state.membrane * gv.to(DEV)).sum()
                + (state.adaptation * ga.to(DEV)).sum())
        ref = oracle.scan_backward(x.numpy(), v0.numpy(), a0.numpy(), grad_spikes=gs.numpy(),
                                   grad_vT=gv.numpy(), grad_aT=ga.numpy(), **okw)
    else:
        params = mb.LIFParams(tau_mem=10.0, threshold=1.0, reset=0.0)
        state, spikes = mb.surrogate_lif_forward(xd, mb.LIFState(vd), params, surrogate=surrogate,
                                                 reset_mode=reset_mode)
        loss = (spikes * gs.to(DEV)).sum() + (state.membrane * gv.to(DEV)).sum()
        ref = oracle.scan_backward(x.numpy(), v0.numpy(), grad_spikes=gs.numpy(),
                                   grad_vT=gv.numpy(), **okw)
    loss.backward()
    assert_close_scaled(host(xd.grad), ref["grad_x"], what="grad_x")
    assert_close_scaled(host(vd.grad), ref["grad_v0"], what="grad_v0")
    if alif:
        assert_close_scaled(host(ad.grad), ref["grad_a0"], what="grad_a0")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("neuron", ["lif", "alif"])
def test_16bit_io_gradients_vs_fp32_carry_oracle(oracle, dtype, neuron):
    alif = neuron == "alif"
    shape = (48, 6, 160)
    x, v0, a0 = _inputs(shape, dtype, 21, alif)
    gen = torch.Generator().manual_seed(22)
    gs = torch.randn(shape, generator=gen).to(dtype)
    okw = dict(neuron=oracle.ALIF if alif else oracle.LIF, decay=dec(10.0),
               threshold=np.float32(1.0), reset=np.float32(0.0), surrogate="atan", slope=10.0)
    xd = x.to(DEV).requires_grad_(True)
    if alif:
        params = mb.ALIFParams(tau_mem=10.0, tau_adaptation=50.0, threshold=1.0, reset=0.0, beta=1.8)
        okw.update(adapt_decay=dec(50.0), beta=np.float32(1.8))
        _, spikes = mb.surrogate_alif_forward(xd, mb.ALIFState(v0.to(DEV), a0.to(DEV)), params)
        ref = oracle.scan_backward(x.float().numpy(), v0.float().numpy(), a0.float().numpy(),
                                   grad_spikes=gs.float().numpy(), **okw)
        fwd = oracle.scan_forward(x.float().numpy(), v0.float().numpy(), a0.float().numpy(),
                                  **{k: v for k, v in okw.items() if k not in ("surrogate", "slope")})
    else:
        params = mb.LIFParams(tau_mem=10.0, threshold=1.0, reset=0.0)
        _, spikes = mb.surrogate_lif_forward(xd, mb.LIFState(v0.to(DEV)), params)
        ref = oracle.scan_backward(x.float().numpy(), v0.float().numpy(),
                                   grad_spikes=gs.float().numpy(), **okw)
        fwd = oracle.scan_forward(x.float().numpy(), v0.float().numpy(),
                                  **{k: v for k, v in okw.items() if k not in ("surrogate", "slope")})
    assert np.array_equal(host(spikes).astype(np.uint8), fwd["spikes"])
    (spikes * gs.to(DEV)).sum().backward()
    assert xd.grad.dtype == dtype
    got = host(xd.grad)
    # gradients beyond the 16-bit range round to +-inf, exactly where the fp32 result does
    expected = _round(ref["grad_x"], dtype)
    overflow = ~np.isfinite(expected)
    assert np.array_equal(~np.isfinite(got), overflow)
    assert_close_scaled(np.where(overflow, 0, got), np.where(overflow, 0, ref["grad_x"]),
                        rtol=2e-2, what="grad_x")


def test_time_lengths_not_multiple_of_chunk_and_zero(oracle):
    params = mb.LIFParams(tau_mem=10.0, threshold=1.0, reset=0.0)
    for T in (0, 1, 15, 16, 17, 31, 33):
        x, v0, _ = _inputs((T, 3, 40), torch.float32, T, False)
        xd = x.to(DEV).requires_grad_(True)
        vd = v0.to(DEV).requires_grad_(True)
        state, spikes = mb.surrogate_lif_forward(xd, mb.LIFState(vd), params)
        assert spikes.shape == (T, 3, 40)
        (state.membrane.sum() + spikes.sum()).backward()
        if T == 0:
            assert torch.equal(state.membrane, vd.detach())
            assert torch.equal(vd.grad, torch.ones_like(vd))
            continue
        ref = oracle.scan_backward(x.numpy(), v0.numpy(), grad_spikes=np.ones(x.shape, np.float32),
                                   grad_vT=np.ones((3, 40), np.float32), decay=dec(10.0),
                                   threshold=np.float32(1.0), reset=np.float32(0.0),
                                   surrogate="atan", slope=10.0)
        assert_close_scaled(host(xd.grad), ref["grad_x"], what=f"T={T}")


def test_lif_forward_rejects_spike_gradients_like_reference():
    x = torch.rand((4, 2, 5), device=DEV, requires_grad=True)
    _, spikes = mb.lif_forward(x, mb.LIFState(torch.zeros((2, 5), device=DEV)), mb.LIFParams())
    with pytest.raises(NotImplementedError):
        spikes.sum().backward()


def test_lif_forward_final_membrane_gradient_vs_oracle(oracle):
    x, v0, _ = _inputs((30, 4, 50), torch.float32, 5, False)
    xd = x.to(DEV).requires_grad_(True)
    vd = v0.to(DEV).requires_grad_(True)
    state, _ = mb.lif_forward(xd, mb.LIFState(vd), mb.LIFParams(tau_mem=10.0))
    gv = torch.randn((4, 50))
    (state.membrane * gv.to(DEV)).sum().backward()
    ref = oracle.scan_backward(x.numpy(), v0.numpy(), grad_vT=gv.numpy(), surrogate=nat.MB_SURR_NONE,
                               decay=dec(10.0), threshold=np.float32(1.0), reset=np.float32(0.0))
    assert_close_scaled(host(xd.grad), ref["grad_x"], what="grad_x")
    assert_close_scaled(host(vd.grad), ref["grad_v0"], what="grad_v0")


def test_north_star_alif_bf16_full_size(oracle):
    """BASELINE config 3 at full size: T=256, B=128, N=4096 bf16, atan, subtractive reset."""

    T, B, N = 256, 128, 4096
    gen = torch.Generator().manual_seed(3)
    x = (torch.randn((T, B, N), generator=gen) * 0.6 + 0.2).to(torch.bfloat16)
    gs = torch.randn((T, B, N), generator=gen).to(torch.bfloat16)
    params = mb.ALIFParams(tau_mem=10.0, tau_adaptation=50.0, threshold=1.0, reset=0.0, beta=1.8)
    zeros = torch.zeros((B, N), dtype=torch.bfloat16, device=DEV)
    xd = x.to(DEV).requires_grad_(True)
    state, spikes = mb.surrogate_alif_forward(xd, mb.ALIFState(zeros, zeros), params,
                                              surrogate="atan", checkpoint_size="memory",
                                              reset_mode="subtract")
    (spikes * gs.to(DEV)).sum().backward()
    okw = dict(neuron=oracle.ALIF, reset_mode=oracle.SUBTRACT, decay=dec(10.0),
               threshold=np.float32(1.0), reset=np.float32(0.0), adapt_decay=dec(50.0),
               beta=np.float32(1.8))
    xf = x.float().numpy()
    z = np.zeros((B, N), np.float32)
    fwd = oracle.scan_forward(xf, z, z, **okw)
    assert np.array_equal(host(spikes).astype(np.uint8), fwd["spikes"])
    ref = oracle.scan_backward(xf, z, z, grad_spikes=gs.float().numpy(), surrogate="atan",
                               slope=10.0, **okw)
    assert_close_scaled(host(xd.grad), ref["grad_x"], rtol=2e-2, what="grad_x")


@pytest.mark.parametrize("shape,dtype,neuron", [
    ((40, 3, 64), torch.float32, nat.MB_LIF),     # fast LIF kernel, fp32 I/O
    ((33, 4, 96), torch.bfloat16, nat.MB_LIF),    # fast LIF kernel, bf16 I/O, partial chunk
    ((21, 3, 5), torch.float32, nat.MB_LIF),      # rows not 16-byte aligned: general kernel
    ((40, 3, 64), torch.bfloat16, nat.MB_ALIF),   # ALIF: summed after the kernel
])
def test_backward_sum_over_t_of_stored_gradient(shape, dtype, neuron):
    """``mb_scan_backward_sum``: per neuron, the fp32 sum over t of grad_x as
    stored, from the last step to the first: bit for bit against the same
    additions on the host, with grad_x itself unchanged."""

    from myelin_b200 import compile_ops as cops

    T, B, N = shape
    g = torch.Generator(device=DEV).manual_seed(T + B + N + neuron)
    x = (torch.randn(shape, generator=g, device=DEV) * 0.6 + 0.3).to(dtype)
    gs = torch.randn(shape, generator=g, device=DEV).to(dtype)
    z = torch.zeros((B, N), dtype=dtype, device=DEV)
    alif = neuron == nat.MB_ALIF
    kw = dict(neuron=neuron, decay=0.9, threshold=1.0, reset=0.0,
              adapt_decay=0.98 if alif else 0.0, beta=1.8 if alif else 0.0,
              reset_mode=nat.MB_RESET_HARD)
    fwd = cops.scan_forward(x, z, z if alif else None, kw["neuron"], kw["decay"], kw["threshold"],
                            kw["reset"], kw["adapt_decay"], kw["beta"], kw["reset_mode"],
                            dense=True, checkpoints=True)
    args = dict(grad_spikes=gs, surrogate=1, slope=25.0, need_v0=False,  # fast_sigmoid
                need_a0=False, **kw)
    plain = cops.scan_backward(x, fwd[5], fwd[6], **args)
    gx, _, _, gsum = cops.scan_backward(x, fwd[5], fwd[6], need_sum=True, **args)
    torch.cuda.synchronize()
    assert torch.equal(gx, plain[0])
    want = torch.zeros((B * N,), dtype=torch.float32)
    host = gx.float().cpu().reshape(T, B * N)
    for t in range(T - 1, -1, -1):
        want = want + host[t]
    assert torch.equal(gsum.cpu(), want)
