"""Packed collectives over NCCL on 2 GPUs (skipped with fewer devices).

Each rank packs its own seeded Bernoulli spikes with the CUDA kernel; the
all-gather must return every rank's words bit for bit in rank order, and the
count all-reduce must equal the per-neuron counts of all ranks' spikes.
"""

from __future__ import annotations

import multiprocessing
import os
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rank_spikes(rank: int) -> torch.Tensor:
    gen = torch.Generator().manual_seed(900 + rank)
    return torch.rand((16, 8, 256), generator=gen) < 0.1


def _worker(rank: int, world: int, init: str, queue) -> None:
    from datetime import timedelta

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=init, rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        import myelin_b200 as mb

        packed = mb.pack_spikes(_rank_spikes(rank).cuda())
        gathered = mb.packed_spike_all_gather(packed)
        ok = len(gathered) == world
        for r, item in enumerate(gathered):
            ref = mb.pack_spikes(_rank_spikes(r).cuda())
            ok = ok and torch.equal(item.data, ref.data) and item.original_shape == ref.original_shape
        counts = mb.packed_spike_count_all_reduce(packed, dim=(0, 1))
        expected = sum(_rank_spikes(r).sum(dim=(0, 1)) for r in range(world)).cuda()
        ok = ok and counts.dtype == torch.int64 and torch.equal(counts, expected)
        rows = mb.packed_spike_count_all_reduce(packed, dim=-1)
        ok = ok and torch.equal(rows, sum(_rank_spikes(r).sum(-1) for r in range(world)).cuda())
        rate = mb.packed_spike_rate_all_reduce(packed)
        total = float(sum(_rank_spikes(r).sum() for r in range(world)))
        ok = ok and abs(rate.item() - total / (16 * 8 * 256 * world)) < 1e-7
        torch.cuda.synchronize()
        queue.put((rank, bool(ok), ""))
    except Exception as exc:
        queue.put((rank, False, f"{type(exc).__name__}: {exc}"))
    finally:
        dist.destroy_process_group()


def test_packed_collectives_over_nccl(tmp_path: Path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = multiprocessing.get_context("spawn")
    queue = ctx.Queue()
    init = f"file://{tmp_path / 'rdzv'}"
    procs = [ctx.Process(target=_worker, args=(r, world, init, queue)) for r in range(world)]
    for p in procs:
        p.start()
    failures = []
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.terminate()
            failures.append(f"rank {p.pid} timed out")
    results = []
    while not queue.empty():
        results.append(queue.get(timeout=1))
    failures += [m for _, ok, m in results if not ok]
    if len(results) != world:
        failures.append(f"expected {world} results, got {len(results)}")
    assert not failures, failures


def _exchange_spikes(rank: int, step: int, shape) -> torch.Tensor:
    gen = torch.Generator().manual_seed(1000 * step + 7 * rank + shape[-1])
    return torch.rand(shape, generator=gen) < 0.1


def _exchange_currents(rank: int, step: int, shape) -> torch.Tensor:
    gen = torch.Generator(device="cuda").manual_seed(500 * step + 11 * rank + shape[-1])
    return 0.3 + 0.5 * torch.randn(shape, generator=gen, device="cuda")


def _exchange_worker(rank: int, world: int, init: str, queue) -> None:
    from datetime import timedelta

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=init, rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        import myelin_b200 as mb

        ok, msg = True, ""
        # (16, 8, 256): fused kernel with peer stores; (6, 5, 70): pack then copy
        for shape in ((16, 8, 256), (6, 5, 70)):
            ex = mb.PackedSpikeExchange(shape)
            for step in range(3):  # both buffers, then the first again
                view, counts = ex.pack_count_all_gather(_exchange_spikes(rank, step, shape).cuda())
                torch.cuda.synchronize()
                for r in range(world):
                    ref = mb.pack_spikes(_exchange_spikes(r, step, shape).cuda()).data
                    if not torch.equal(view[r], ref):
                        ok, msg = False, f"words of rank {r}, shape {shape}, step {step}"
                expected = sum(_exchange_spikes(r, step, shape).sum(dim=(0, 1)).to(torch.int64)
                               for r in range(world)).cuda()
                if counts.dtype != torch.int64 or not torch.equal(counts, expected):
                    ok, msg = False, f"counts, shape {shape}, step {step}"
            # the packed scan feeding the same buffers (fused forward / fallback)
            params = mb.LIFParams(tau_mem=8.0)
            for step in range(2):
                xs = [_exchange_currents(r, step, shape) for r in range(world)]
                v0 = torch.full(shape[1:], 0.25, device="cuda")
                st, view = ex.lif_forward_packed_spikes(xs[rank], mb.LIFState(v0), params,
                                                        reset_mode="subtract")
                torch.cuda.synchronize()
                for r in range(world):
                    ref_st, ref = mb.lif_forward_packed_spikes(xs[r], mb.LIFState(v0), params,
                                                               reset_mode="subtract")
                    if not torch.equal(view[r], ref.data):
                        ok, msg = False, f"scan words of rank {r}, shape {shape}, step {step}"
                    if r == rank and not torch.equal(st.membrane, ref_st.membrane):
                        ok, msg = False, f"scan state, shape {shape}, step {step}"
            ex.close()
        # projection + packed scan (bf16, tcgen05 GEMM) feeding the buffers
        T, B, F, N = 12, 8, 64, 256
        ex = mb.PackedSpikeExchange((T, B, N))
        g = torch.Generator(device="cuda").manual_seed(5)
        w = (0.2 * torch.randn((F, N), generator=g, device="cuda")).to(torch.bfloat16)
        b = (0.1 * torch.randn((N,), generator=g, device="cuda")).to(torch.bfloat16)
        xs = [(torch.rand((T, B, F), generator=torch.Generator(device="cuda").manual_seed(40 + r),
                          device="cuda") < 0.3).to(torch.bfloat16) for r in range(world)]
        params = mb.LIFParams(tau_mem=20.0)
        st, view = ex.linear_surrogate_lif_packed_forward(xs[rank], w, b, params)
        torch.cuda.synchronize()
        for r in range(world):
            ref_st, ref = mb.linear_surrogate_lif_packed_forward(xs[r], w, b, params)
            if not torch.equal(view[r], ref.data):
                ok, msg = False, f"linear packed words of rank {r}"
            if r == rank and not torch.equal(st.membrane, ref_st.membrane):
                ok, msg = False, "linear packed state"
        ex.close()
        torch.cuda.synchronize()
        queue.put((rank, bool(ok), msg))
    except Exception as exc:
        queue.put((rank, False, f"{type(exc).__name__}: {exc}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_packed_spike_exchange_over_nvlink(tmp_path: Path, world: int):
    """Fused pack + peer-store all-gather + count all-reduce on 2-8 GPUs equals
    every rank's pack_spikes and the summed counts, bit for bit; the packed
    scans feeding the same buffers equal every rank's packed forward."""

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = multiprocessing.get_context("spawn")
    queue = ctx.Queue()
    init = f"file://{tmp_path / 'rdzv_exchange'}"
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, init, queue))
             for r in range(world)]
    for p in procs:
        p.start()
    failures = []
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.terminate()
            failures.append(f"rank {p.pid} timed out")
    results = []
    while not queue.empty():
        results.append(queue.get(timeout=1))
    failures += [m for _, ok, m in results if not ok]
    if len(results) != world:
        failures.append(f"expected {world} results, got {len(results)}")
    assert not failures, failures
