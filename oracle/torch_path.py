"""TEST INFRASTRUCTURE ONLY: the reference's torch CPU path for the ALIF scan, restated for timing.

The reference's CPU implementation of ``surrogate_alif_forward`` (backend
"torch", src/myelin/kernels.py:340-392) is a per-timestep Python loop of torch
tensor ops, ``functional.surrogate_alif_unroll`` (src/myelin/functional.py:149-189),
with the hard forward spike ``hard + smooth - smooth.detach()``
(src/myelin/surrogates.py:105-110) and, for BASELINE config 3, the atan
surrogate (surrogates.py:41-44); its backward is torch autograd through that
loop. ``alif_atan_unroll`` below follows the same operations in the same
order, plus the subtractive reset ``m = p - theta * s`` that config 3 asks for
(the reference only hard-resets). ``bench.py`` times it on the GPU box's host
cores as "myelin's torch CPU path" (the reference itself does not travel to
that box); ``tests/test_oracle_golden.py`` checks it against the C oracle.
Only ``tests/`` and ``bench.py``'s CPU legs use this module.
"""

from __future__ import annotations

import math
import os
import time

import torch


def alif_atan_unroll(x, m0, a0, *, decay, threshold, beta, adaptation_decay, reset, slope,
                     subtract):
    """Returns (final membrane, final adaptation, spikes [T, B, N]), differentiable."""

    spikes = []
    membrane, adaptation = m0, a0
    for current in x.unbind(dim=0):
        membrane = membrane * decay + current
        adaptive_threshold = threshold + beta * adaptation
        centered = slope * (membrane - adaptive_threshold)
        hard = (centered >= 0).to(centered.dtype)
        smooth = torch.atan(math.pi * centered / 2.0) / math.pi + 0.5
        spike = hard + smooth - smooth.detach()
        if subtract:
            membrane = membrane - adaptive_threshold * spike
        else:
            membrane = membrane * (1.0 - spike) + reset * spike
        adaptation = adaptation * adaptation_decay + spike
        spikes.append(spike)
    return membrane, adaptation, torch.stack(spikes, dim=0)


def host_threads() -> int:
    return len(os.sched_getaffinity(0))


def time_config3(*, T: int = 256, B: int = 128, N: int = 4096, dtype=torch.bfloat16,
                 seconds: float = 10.0, min_steps: int = 2, threads: int | None = None,
                 steps: int | None = None, warmup: int = 1) -> dict:
    """Time forward + autograd backward at BASELINE config 3 on CPU.

    x ~ N(0.2, 0.6), grad ~ N(0, 1) (seeded), tau_mem 10, tau_adaptation 50,
    beta 1.8, threshold 1, subtractive reset, atan slope 10, in ``dtype``
    (the config's bf16: the reference's torch path computes in the input dtype).
    Runs ``steps`` timed steps if given, else steps until ``seconds`` have
    passed (at least ``min_steps``). Returns per-step times and the thread count.
    """

    threads = threads or host_threads()
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(99)
    x = (torch.randn((T, B, N), generator=gen) * 0.6 + 0.2).to(dtype).requires_grad_(True)
    grad = torch.randn((T, B, N), generator=gen).to(dtype)
    zeros = torch.zeros((B, N), dtype=dtype)
    kw = dict(decay=1.0 - 1.0 / 10.0, threshold=1.0, beta=1.8, adaptation_decay=1.0 - 1.0 / 50.0,
              reset=0.0, slope=10.0, subtract=True)

    def step():
        _, _, spikes = alif_atan_unroll(x, zeros, zeros, **kw)
        (gx,) = torch.autograd.grad(spikes, x, grad)
        return gx

    for _ in range(warmup):
        step()
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if steps is not None:
            if len(times) >= steps:
                break
        elif len(times) >= min_steps and time.perf_counter() - t_start >= seconds:
            break
    return {"times": times, "threads": threads, "units": T * B * N, "shape": (T, B, N),
            "dtype": str(dtype).replace("torch.", "")}
