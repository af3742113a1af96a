"""Generate golden vectors for the oracle from the reference implementation itself.

Run in a container where the reference (djsaunde/myelin) source tree is
available:

    python tests/golden/make_golden.py --reference-src <path to myelin>/src

It imports the reference's own torch functions (the correctness oracle the
reference names in src/myelin/neurons.py:1-5) and writes small ``.npz``
fixtures next to this script. The fixtures are committed; tests never import
the reference. Cases:

- lif_fwd_*.npz / alif_fwd_*.npz: ``functional.lif_unroll`` / ``alif_unroll``
  (src/myelin/functional.py:21-78) spikes (packed words) and final state;
- surrogate_lif_<surrogate>.npz / surrogate_alif_<surrogate>.npz: spikes, final
  state and torch-autograd gradients of ``surrogate_lif_unroll`` /
  ``surrogate_alif_unroll`` (functional.py:115-189) for every surrogate;
- alif_subtract_atan.npz: the same for the subtractive-reset extension, from a
  torch restatement of ``surrogate_alif_unroll`` with ``m = p - theta * s``
  (the gradient of this case has no reference counterpart and stays unpinned);
- alif_subtract_dsl_*.npz: the subtractive-reset ALIF forward evaluated by the
  reference's own custom-neuron oracle, ``dsl.evaluate_neuron_unroll``
  (src/myelin/dsl.py:457-511), on an ALIF ``NeuronIR`` built like ``alif_ir``
  (dsl.py:1064-1089) whose membrane update is
  ``where(spike, pre_reset - adaptive_threshold, pre_reset)``: spikes (packed
  words) and final membrane / adaptation. Case ``b`` uses bf16-representable
  inputs and states so the bf16-I/O kernel can be checked against it too;
- linear_stream.npz / linear_checkpoint_rate.npz: the torch autograd functions
  ``LinearSurrogateLIFStreamFunction`` / ``LinearSurrogateLIFCheckpointRateFunction``
  (src/myelin/autograd.py:445-885);
- packing.npz: ``pack_spikes`` / ``packed_spike_counts`` / ``packed_spike_count``
  (src/myelin/packing.py:45-216) on ragged widths;
- izhikevich_*.npz: ``functional.izhikevich_unroll`` (functional.py:81-112)
  spikes (packed words) and final voltage / recovery, default and custom
  parameters;
- c1_checksum.json: SHA-256 of the packed spikes and final membrane of
  ``lif_unroll`` at BASELINE config 1 (T=64, B=32, N=1024, x ~ N(0.3, 0.5),
  torch.Generator seed 0), for a full-size bit-exact check without storing it.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def _gen(seed: int) -> torch.Generator:
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def _pack_np(spikes: torch.Tensor) -> np.ndarray:
    from myelin.packing import pack_spikes

    return pack_spikes((spikes != 0).to(torch.float32)).data.numpy()


def c1_input(seed: int = 0) -> torch.Tensor:
    """BASELINE config 1 input: x ~ N(0.3, 0.5), [64, 32, 1024] float32."""

    return torch.randn((64, 32, 1024), generator=_gen(seed)) * 0.5 + 0.3


def lif_forward_cases() -> None:
    from myelin.functional import alif_unroll, lif_unroll
    from myelin.neurons import ALIFParams, ALIFState, LIFParams, LIFState

    for name, (T, B, N), tau, thr, reset, mean, std, seed in [
        ("lif_fwd_a", (40, 3, 67), 10.0, 1.0, -0.25, 0.3, 0.5, 1),
        ("lif_fwd_b", (33, 5, 32), 20.0, 0.8, 0.0, 0.2, 0.6, 2),
    ]:
        g = _gen(seed)
        x = torch.randn((T, B, N), generator=g) * std + mean
        v0 = torch.rand((B, N), generator=g) * 0.2
        params = LIFParams(tau_mem=tau, threshold=thr, reset=reset)
        state, spikes = lif_unroll(x, LIFState(membrane=v0), params)
        np.savez_compressed(
            OUT / f"{name}.npz", x=x.numpy(), v0=v0.numpy(), tau=tau, thr=thr, reset=reset,
            packed=_pack_np(spikes), vT=state.membrane.numpy(),
        )

    for name, (T, B, N), p, mean, std, seed in [
        ("alif_fwd_a", (40, 3, 67), dict(tau_mem=10.0, tau_adaptation=50.0, threshold=1.0,
                                           reset=0.0, beta=1.8), 0.2, 0.6, 3),
        ("alif_fwd_b", (29, 4, 45), dict(tau_mem=10.0, tau_adaptation=5.0, threshold=1.0,
                                           reset=-0.25, beta=1.0), 0.4, 0.5, 4),
    ]:
        g = _gen(seed)
        x = torch.randn((T, B, N), generator=g) * std + mean
        v0 = torch.rand((B, N), generator=g) * 0.2
        a0 = torch.rand((B, N), generator=g) * 0.2
        params = ALIFParams(**p)
        state, spikes = alif_unroll(x, ALIFState(membrane=v0, adaptation=a0), params)
        np.savez_compressed(
            OUT / f"{name}.npz", x=x.numpy(), v0=v0.numpy(), a0=a0.numpy(),
            packed=_pack_np(spikes), vT=state.membrane.numpy(), aT=state.adaptation.numpy(),
            **{k: v for k, v in p.items()},
        )


def izhikevich_cases() -> None:
    """``functional.izhikevich_unroll`` (src/myelin/functional.py:81-112) in float32."""

    from myelin.functional import izhikevich_unroll
    from myelin.neurons import IzhikevichParams, IzhikevichState

    for name, (T, B, N), p, mean, std, seed in [
        ("izhikevich_a", (60, 3, 67), {}, 10.0, 4.0, 5),
        ("izhikevich_b", (50, 4, 64), dict(recovery_decay=0.1, recovery_coupling=0.25,
                                           reset_voltage=-60.0, recovery_jump=2.0, threshold=25.0,
                                           dt=0.5, voltage_square_coeff=0.05,
                                           voltage_coeff=4.5, voltage_bias=130.0), 8.0, 6.0, 6),
    ]:
        g = _gen(seed)
        x = torch.randn((T, B, N), generator=g) * std + mean
        v0 = -65.0 + torch.rand((B, N), generator=g) * 10.0
        u0 = 0.2 * v0 + torch.rand((B, N), generator=g)
        params = IzhikevichParams(**p)
        state, spikes = izhikevich_unroll(x, IzhikevichState(voltage=v0, recovery=u0), params)
        fields = {k: getattr(params, k) for k in (
            "recovery_decay", "recovery_coupling", "reset_voltage", "recovery_jump", "threshold",
            "dt", "voltage_square_coeff", "voltage_coeff", "voltage_bias")}
        np.savez_compressed(
            OUT / f"{name}.npz", x=x.numpy(), v0=v0.numpy(), u0=u0.numpy(),
            packed=_pack_np(spikes), vT=state.voltage.numpy(), uT=state.recovery.numpy(),
            **fields,
        )


def _surrogate_alif_subtract(x, v0, a0, params, surrogate_fn, slope):
    """Restatement of surrogate_alif_unroll with m = p - theta * s (extension)."""

    from myelin.surrogates import hard_surrogate_spike

    membrane, adaptation, spikes = v0, a0, []
    for xt in x.unbind(0):
        membrane = membrane * params.decay + xt
        theta = params.threshold + params.beta * adaptation
        spike = hard_surrogate_spike(slope * (membrane - theta), surrogate_fn)
        membrane = membrane - theta * spike
        adaptation = adaptation * params.adaptation_decay + spike
        spikes.append(spike)
    return membrane, adaptation, torch.stack(spikes)


def surrogate_cases() -> None:
    from myelin.functional import surrogate_alif_unroll, surrogate_lif_unroll
    from myelin.neurons import ALIFParams, ALIFState, LIFParams, LIFState
    from myelin.surrogates import SURROGATE_NAMES, surrogate_from_name

    T, B, N = 24, 3, 37
    for index, surrogate in enumerate(SURROGATE_NAMES):
        fn = surrogate_from_name(surrogate)
        g = _gen(100 + index)
        x = (torch.randn((T, B, N), generator=g) * 0.5 + 0.3).requires_grad_(True)
        v0 = (torch.rand((B, N), generator=g) * 0.2).requires_grad_(True)
        gs = torch.randn((T, B, N), generator=g)
        gv = torch.randn((B, N), generator=g)
        params = LIFParams(tau_mem=10.0, threshold=1.0, reset=-0.1)
        state, spikes = surrogate_lif_unroll(
            x, LIFState(membrane=v0), params, surrogate=fn, surrogate_slope=5.0
        )
        gx, gv0 = torch.autograd.grad((spikes * gs).sum() + (state.membrane * gv).sum(), (x, v0))
        np.savez_compressed(
            OUT / f"surrogate_lif_{surrogate}.npz", x=x.detach().numpy(),
            v0=v0.detach().numpy(), grad_spikes=gs.numpy(), grad_vT=gv.numpy(), slope=5.0,
            tau=10.0, thr=1.0, reset=-0.1, packed=_pack_np(spikes.detach()),
            spikes=spikes.detach().numpy(), vT=state.membrane.detach().numpy(),
            grad_x=gx.numpy(), grad_v0=gv0.numpy(),
        )

        g = _gen(200 + index)
        x = (torch.randn((T, B, N), generator=g) * 0.6 + 0.2).requires_grad_(True)
        v0 = (torch.rand((B, N), generator=g) * 0.2).requires_grad_(True)
        a0 = (torch.rand((B, N), generator=g) * 0.2).requires_grad_(True)
        gs = torch.randn((T, B, N), generator=g)
        gv = torch.randn((B, N), generator=g)
        ga = torch.randn((B, N), generator=g)
        p = dict(tau_mem=10.0, tau_adaptation=50.0, threshold=1.0, reset=0.0, beta=1.8)
        params = ALIFParams(**p)
        state, spikes = surrogate_alif_unroll(
            x, ALIFState(membrane=v0, adaptation=a0), params, surrogate=fn, surrogate_slope=10.0
        )
        loss = (spikes * gs).sum() + (state.membrane * gv).sum() + (state.adaptation * ga).sum()
        gx, gv0, ga0 = torch.autograd.grad(loss, (x, v0, a0))
        np.savez_compressed(
            OUT / f"surrogate_alif_{surrogate}.npz", x=x.detach().numpy(),
            v0=v0.detach().numpy(), a0=a0.detach().numpy(), grad_spikes=gs.numpy(),
            grad_vT=gv.numpy(), grad_aT=ga.numpy(), slope=10.0,
            packed=_pack_np(spikes.detach()), vT=state.membrane.detach().numpy(),
            aT=state.adaptation.detach().numpy(), grad_x=gx.numpy(), grad_v0=gv0.numpy(),
            grad_a0=ga0.numpy(), **p,
        )

    fn = surrogate_from_name("atan")
    g = _gen(300)
    x = (torch.randn((T, B, N), generator=g) * 0.6 + 0.2).requires_grad_(True)
    v0 = (torch.rand((B, N), generator=g) * 0.2).requires_grad_(True)
    a0 = (torch.rand((B, N), generator=g) * 0.2).requires_grad_(True)
    gs = torch.randn((T, B, N), generator=g)
    gv = torch.randn((B, N), generator=g)
    ga = torch.randn((B, N), generator=g)
    p = dict(tau_mem=10.0, tau_adaptation=50.0, threshold=1.0, reset=0.0, beta=1.8)
    m, a, spikes = _surrogate_alif_subtract(x, v0, a0, ALIFParams(**p), fn, 10.0)
    loss = (spikes * gs).sum() + (m * gv).sum() + (a * ga).sum()
    gx, gv0, ga0 = torch.autograd.grad(loss, (x, v0, a0))
    np.savez_compressed(
        OUT / "alif_subtract_atan.npz", x=x.detach().numpy(), v0=v0.detach().numpy(),
        a0=a0.detach().numpy(), grad_spikes=gs.numpy(), grad_vT=gv.numpy(), grad_aT=ga.numpy(),
        slope=10.0, packed=_pack_np(spikes.detach()), vT=m.detach().numpy(),
        aT=a.detach().numpy(), grad_x=gx.numpy(), grad_v0=gv0.numpy(), grad_a0=ga0.numpy(), **p,
    )


def alif_subtract_ir():
    """ALIF NeuronIR with subtractive reset, from the reference DSL's own
    builders (dsl.py:1064-1089 shows the hard-reset original)."""

    from myelin.dsl import NeuronIR, input_, param, state, where

    membrane = state("membrane")
    adaptation = state("adaptation")
    current = input_("input_current")
    decay = param("decay")
    adaptation_decay = param("adaptation_decay")
    threshold = param("threshold")
    beta = param("beta")
    pre_reset = membrane * decay + current
    adaptive_threshold = threshold + beta * adaptation
    spike = pre_reset.ge(adaptive_threshold)
    spike_float = where(spike, 1.0, 0.0)
    return NeuronIR(
        name="alif_subtract",
        state=("membrane", "adaptation"),
        params=("decay", "adaptation_decay", "threshold", "beta"),
        inputs=("input_current",),
        next_state={
            "membrane": where(spike, pre_reset - adaptive_threshold, pre_reset),
            "adaptation": adaptation * adaptation_decay + spike_float,
        },
        outputs={"spike": spike_float},
    )


def alif_subtract_dsl_cases() -> None:
    from myelin.dsl import evaluate_neuron_unroll
    from myelin.neurons import ALIFParams

    ir = alif_subtract_ir()
    for name, (T, B, N), seed, bf16 in [
        ("alif_subtract_dsl_a", (24, 3, 37), 600, False),
        ("alif_subtract_dsl_b", (96, 4, 160), 601, True),  # T >= 64, bf16-representable
    ]:
        g = _gen(seed)
        x = torch.randn((T, B, N), generator=g) * 0.6 + 0.2
        v0 = torch.rand((B, N), generator=g) * 0.4
        a0 = torch.rand((B, N), generator=g) * 0.3
        if bf16:
            x, v0, a0 = (t.to(torch.bfloat16).to(torch.float32) for t in (x, v0, a0))
        p = dict(tau_mem=10.0, tau_adaptation=50.0, threshold=1.0, reset=0.0, beta=1.8)
        params = ALIFParams(**p)
        values = {"decay": params.decay, "adaptation_decay": params.adaptation_decay,
                  "threshold": params.threshold, "beta": params.beta}
        final, spikes = evaluate_neuron_unroll(
            ir, x, {"membrane": v0, "adaptation": a0}, values)
        np.savez_compressed(
            OUT / f"{name}.npz", x=x.numpy(), v0=v0.numpy(), a0=a0.numpy(),
            packed=_pack_np(spikes), vT=final["membrane"].numpy(),
            aT=final["adaptation"].numpy(), spike_count=np.asarray(int(spikes.sum().item())),
            **p,
        )


def linear_cases() -> None:
    from myelin.autograd import (
        linear_surrogate_lif_checkpoint_rate_function,
        linear_surrogate_lif_stream_function,
    )
    from myelin.neurons import LIFParams

    T, B, F, N = 8, 4, 40, 33
    g = _gen(400)
    x = (torch.rand((T, B, F), generator=g) < 0.2).to(torch.float32).requires_grad_(True)
    bound = 1.0 / np.sqrt(F)
    w = ((torch.rand((F, N), generator=g) * 2 - 1) * bound * 4).requires_grad_(True)
    b = ((torch.rand((N,), generator=g) * 2 - 1) * bound).requires_grad_(True)
    gs = torch.randn((T, B, N), generator=g)
    gv = torch.randn((B, N), generator=g)
    params = LIFParams(tau_mem=20.0, threshold=1.0, reset=0.0)
    state, spikes = linear_surrogate_lif_stream_function(
        x, w, b, params, surrogate="fast_sigmoid", surrogate_slope=25.0
    )
    loss = (spikes * gs).sum() + (state.membrane * gv).sum()
    gx, gw, gb = torch.autograd.grad(loss, (x, w, b))
    np.savez_compressed(
        OUT / "linear_stream.npz", x=x.detach().numpy(), w=w.detach().numpy(),
        b=b.detach().numpy(), grad_spikes=gs.numpy(), grad_vT=gv.numpy(), tau=20.0, thr=1.0,
        reset=0.0, slope=25.0, packed=_pack_np(spikes.detach()),
        vT=state.membrane.detach().numpy(), grad_x=gx.numpy(), grad_w=gw.numpy(),
        grad_b=gb.numpy(),
    )

    g = _gen(401)
    x = (torch.rand((T, B, F), generator=g) < 0.3).to(torch.float32).requires_grad_(True)
    w = ((torch.rand((F, N), generator=g) * 2 - 1) * bound * 4).requires_grad_(True)
    b = ((torch.rand((N,), generator=g) * 2 - 1) * bound).requires_grad_(True)
    gr = torch.randn((B, N), generator=g)
    state, rates = linear_surrogate_lif_checkpoint_rate_function(
        x, w, b, params, surrogate="superspike", surrogate_slope=10.0, checkpoint_size=3,
        reduction="none",
    )
    gx, gw, gb = torch.autograd.grad((rates * gr).sum(), (x, w, b))
    np.savez_compressed(
        OUT / "linear_checkpoint_rate.npz", x=x.detach().numpy(), w=w.detach().numpy(),
        b=b.detach().numpy(), grad_rates=gr.numpy(), tau=20.0, thr=1.0, reset=0.0, slope=10.0,
        rates=rates.detach().numpy(), vT=state.membrane.detach().numpy(), grad_x=gx.numpy(),
        grad_w=gw.numpy(), grad_b=gb.numpy(),
    )


def packing_cases() -> None:
    from myelin.packing import pack_spikes, packed_spike_count, packed_spike_counts

    arrays: dict[str, np.ndarray] = {}
    g = _gen(500)
    for n in (1, 31, 32, 33, 65, 100):
        vals = torch.randn((3, 2, n), generator=g)
        keep = torch.rand((3, 2, n), generator=g) < 0.4
        spikes = torch.where(keep, vals, torch.zeros_like(vals))
        spikes[0, 0, 0] = -0.0
        packed = pack_spikes(spikes)
        arrays[f"spikes_{n}"] = spikes.numpy()
        arrays[f"packed_{n}"] = packed.data.numpy()
        arrays[f"rows_{n}"] = packed_spike_counts(packed, dim=-1).numpy()
        arrays[f"cols_{n}"] = packed_spike_count(packed, dim=(0, 1)).numpy()
        arrays[f"total_{n}"] = np.asarray(packed_spike_count(packed).item())
    high = torch.zeros((1, 32))
    high[0, -1] = 1.0
    arrays["high_bit_word"] = pack_spikes(high).data.numpy()
    np.savez_compressed(OUT / "packing.npz", **arrays)


def c1_checksum() -> None:
    from myelin.functional import lif_unroll
    from myelin.neurons import LIFParams, LIFState

    x = c1_input(0)
    state, spikes = lif_unroll(x, LIFState(membrane=torch.zeros((32, 1024))),
                               LIFParams(tau_mem=10.0, threshold=1.0, reset=0.0))
    packed = _pack_np(spikes)
    record = {
        "config": "BASELINE config 1: T=64 B=32 N=1024, x ~ N(0.3,0.5) torch.Generator seed 0, "
                  "tau_mem=10 (beta=0.9), threshold=1, reset=0, v0=0",
        "packed_sha256": hashlib.sha256(packed.tobytes()).hexdigest(),
        "vT_sha256": hashlib.sha256(state.membrane.numpy().tobytes()).hexdigest(),
        "spike_count": int(spikes.sum().item()),
        "input_sha256": hashlib.sha256(x.numpy().tobytes()).hexdigest(),
        "torch": torch.__version__,
    }
    (OUT / "c1_checksum.json").write_text(json.dumps(record, indent=2) + "\n")


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference-src", required=True, help="path to the reference's src/")
    cases = {"lif": lif_forward_cases, "surrogate": surrogate_cases, "linear": linear_cases,
             "packing": packing_cases, "c1": c1_checksum, "izhikevich": izhikevich_cases,
             "subtract_dsl": alif_subtract_dsl_cases}
    parser.add_argument("--cases", nargs="*", choices=sorted(cases), default=sorted(cases),
                        help="which fixture groups to (re)write (default: all)")
    args = parser.parse_args()
    sys.path.insert(0, args.reference_src)
    torch.set_num_threads(1)
    for name in args.cases:
        cases[name]()
    for f in sorted(OUT.glob("*.npz")) + sorted(OUT.glob("*.json")):
        print(f"{f.name:40s} {f.stat().st_size:8d} B")


if __name__ == "__main__":
    main()
