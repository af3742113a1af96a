"""Host logic of the packed-spike collectives, on CPU.

A fake ``torch.distributed`` (as in the reference's tests/test_distributed.py:86-124)
checks the call pattern; a real 2-rank gloo process group (spawned processes,
file:// rendezvous, bounded joins) checks the all-gather layout, the int32
wire format and the int64 results. Counting on CPU uses the numpy oracle in
place of the CUDA count kernels (which the GPU tests cover).
"""

from __future__ import annotations

import multiprocessing
from pathlib import Path
from typing import Any

import numpy as np
import pytest
import torch
import torch.distributed as torch_dist

import myelin_b200.distributed as mbd
import myelin_b200.neurons as mbd_neurons
from myelin_b200.packing import PackedSpikes, _normalize_count_dims


def oracle_packed(spikes: np.ndarray) -> PackedSpikes:
    from oracle import oracle

    return PackedSpikes(data=torch.from_numpy(oracle.pack(spikes)), original_shape=spikes.shape)


def oracle_count(packed: PackedSpikes, dim=None) -> torch.Tensor:
    """Dense-like counts from the oracle's unpack (CPU stand-in for the CUDA counts)."""

    from oracle import oracle

    bits = torch.from_numpy(oracle.unpack(packed.data.numpy(), packed.original_shape[-1])).to(torch.int64)
    if dim is None:
        return bits.sum()
    return bits.sum(dim=_normalize_count_dims(dim, ndim=bits.ndim))


def oracle_leading(packed: PackedSpikes, *, dtype=torch.int64) -> torch.Tensor:
    return oracle_count(packed, tuple(range(len(packed.original_shape) - 1))).to(dtype)


class FakeDist:
    class ReduceOp:
        SUM = "sum"

    def __init__(self, world_size: int = 2, initialized: bool = True) -> None:
        self.world_size = world_size
        self.initialized = initialized
        self.reduced_dtype: torch.dtype | None = None

    def is_available(self) -> bool:
        return True

    def is_initialized(self) -> bool:
        return self.initialized

    def get_world_size(self, group: Any | None = None) -> int:
        return self.world_size

    def all_gather_into_tensor(self, out: torch.Tensor, local: torch.Tensor, group=None) -> None:
        assert out.shape[0] == self.world_size * local.shape[0]  # concatenated form
        blocks = out.view(self.world_size, *local.shape)
        for rank in range(self.world_size):
            blocks[rank].copy_(local + rank)

    def all_reduce(self, tensor: torch.Tensor, op=None, group=None) -> None:
        assert op == self.ReduceOp.SUM
        self.reduced_dtype = tensor.dtype
        tensor.mul_(self.world_size)


@pytest.fixture
def fake(monkeypatch):
    fd = FakeDist(world_size=3)
    monkeypatch.setattr(mbd, "dist", fd)
    monkeypatch.setattr(mbd, "packed_spike_count", oracle_count)
    monkeypatch.setattr(mbd, "packed_spike_counts_over_leading_dims", oracle_leading)
    return fd


def test_all_gather_keeps_metadata_and_rank_order(fake):
    spikes = np.zeros((2, 3, 35), np.float32)
    spikes[..., 0] = 1.0
    packed = oracle_packed(spikes)
    gathered = mbd.packed_spike_all_gather(packed)
    assert len(gathered) == 3
    for rank, item in enumerate(gathered):
        assert item.original_shape == packed.original_shape
        assert torch.equal(item.data, packed.data + rank)
    buf = mbd.packed_spike_all_gather_into_tensor(packed)
    assert buf.shape == (3, *packed.data.shape)


def test_count_all_reduce_uses_int32_wire_and_returns_int64(fake):
    spikes = np.zeros((2, 3, 35), np.float32)
    spikes[0, :, 0] = 1.0
    spikes[1, :, 1] = 1.0
    packed = oracle_packed(spikes)
    counts = mbd.packed_spike_count_all_reduce(packed, dim=-1)
    assert fake.reduced_dtype == torch.int32
    assert counts.dtype == torch.int64
    assert torch.equal(counts, torch.from_numpy(spikes.sum(-1).astype(np.int64)) * 3)
    per_neuron = mbd.packed_spike_count_all_reduce(packed, dim=(0, 1))
    assert torch.equal(per_neuron, torch.from_numpy(spikes.sum((0, 1)).astype(np.int64)) * 3)
    rates = mbd.packed_spike_rate_all_reduce(packed, dim=-1)
    assert torch.allclose(rates, torch.from_numpy(spikes.mean(-1)))


def test_count_all_reduce_falls_back_to_int64_when_int32_could_overflow(fake, monkeypatch):
    monkeypatch.setattr(mbd, "_INT32_MAX", 10)
    packed = oracle_packed(np.ones((2, 3, 35), np.float32))
    counts = mbd.packed_spike_count_all_reduce(packed)
    assert fake.reduced_dtype == torch.int64
    assert counts.item() == 2 * 3 * 35 * 3


def test_collectives_require_initialized_process_group(monkeypatch):
    monkeypatch.setattr(mbd, "dist", FakeDist(initialized=False))
    packed = PackedSpikes(data=torch.zeros((1, 1), dtype=torch.int32), original_shape=(1, 32))
    with pytest.raises(RuntimeError, match="not initialized"):
        mbd.packed_spike_all_gather(packed)
    with pytest.raises(RuntimeError, match="not initialized"):
        mbd.packed_spike_count_all_reduce(packed)
    assert not mbd.distributed_available_and_initialized() or torch_dist.is_initialized()


def _rank_spikes(rank: int) -> np.ndarray:
    spikes = np.zeros((4, 3, 70), np.float32)
    spikes[..., rank] = 1.0
    spikes[rank, 1, 40 + rank] = 1.0
    return spikes


def _gloo_worker(rank: int, world: int, init: str, queue) -> None:
    torch_dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        mbd.packed_spike_count = oracle_count
        mbd.packed_spike_counts_over_leading_dims = oracle_leading
        packed = oracle_packed(_rank_spikes(rank))
        gathered = mbd.packed_spike_all_gather(packed)
        ok = all(torch.equal(g.data, oracle_packed(_rank_spikes(r)).data) for r, g in enumerate(gathered))
        total = sum(_rank_spikes(r) for r in range(world))
        cols = mbd.packed_spike_count_all_reduce(packed, dim=(0, 1))
        ok = ok and torch.equal(cols, torch.from_numpy(total.sum((0, 1)).astype(np.int64)))
        rows = mbd.packed_spike_count_all_reduce(packed, dim=-1)
        ok = ok and torch.equal(rows, torch.from_numpy(total.sum(-1).astype(np.int64)))
        rate = mbd.packed_spike_rate_all_reduce(packed)
        ok = ok and torch.allclose(rate, torch.tensor(float(total.sum()) / (total.size * world)))
        queue.put((rank, bool(ok), ""))
    except Exception as exc:  # the parent reports child failures
        queue.put((rank, False, f"{type(exc).__name__}: {exc}"))
    finally:
        torch_dist.destroy_process_group()


def test_collectives_on_two_gloo_ranks(tmp_path: Path):
    if not torch_dist.is_available() or not torch_dist.is_gloo_available():
        pytest.skip("gloo unavailable")
    world = 2
    ctx = multiprocessing.get_context("spawn")
    queue = ctx.Queue()
    init = f"file://{tmp_path / 'rendezvous'}"
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, init, queue)) for r in range(world)]
    for p in procs:
        p.start()
    failures = []
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.terminate()
            failures.append(f"rank process {p.pid} timed out")
        elif p.exitcode != 0:
            failures.append(f"rank process {p.pid} exited with {p.exitcode}")
    results = []
    while not queue.empty():
        results.append(queue.get(timeout=1))
    failures += [msg for _, ok, msg in results if not ok]
    if len(results) != world:
        failures.append(f"expected {world} results, got {len(results)}")
    assert not failures, failures


class _FakeIpc:
    """Stand-in for the CUDA IPC / scatter-kernel layer of PackedSpikeExchange
    on CPU ranks: addresses encode (owner rank, buffer); 'opening' a peer's
    handle yields a distinct importer address; the scatter records its
    destinations and counts spikes with torch."""

    IMPORT = 1 << 50

    def __init__(self, rank: int) -> None:
        self.rank = rank
        self.calls: list[tuple] = []
        self.n_alloc = 0

    def device_context(self, device):
        import contextlib

        return contextlib.nullcontext()

    def device_view(self, address, shape, device):
        return torch.zeros(shape, dtype=torch.int32)

    def ipc_alloc(self, nbytes):
        address = ((self.rank + 1) << 40) | (self.n_alloc << 32)
        self.n_alloc += 1
        self.calls.append(("alloc", address, nbytes))
        return address, repr((address, nbytes)).encode()

    def ipc_open(self, handle):
        address, _ = eval(handle.decode())  # noqa: S307 - test-local repr round trip
        self.calls.append(("open", address))
        return address | self.IMPORT

    def pack_count_scatter(self, spikes, words, rows, n, peers, c64, c32):
        self.calls.append(("scatter", words, tuple(peers)))
        out = c64 if c64 is not None else c32
        out.copy_((spikes.reshape(rows, n) != 0).sum(0).to(out.dtype))

    def scan_forward_packed_scatter(self, *, x, v0, vT, packed, peers, decay, threshold,
                                    reset_mode, **_):
        self.calls.append(("scan", packed, tuple(peers), decay, threshold, reset_mode))
        vT.copy_(v0)

    def device_synchronize(self, device):
        self.calls.append(("sync",))

    def ipc_close(self, address):
        self.calls.append(("close", address))

    def ipc_free(self, address):
        self.calls.append(("free", address))


def _exchange_worker(rank: int, world: int, init: str, queue) -> None:
    torch_dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        shape = (4, 3, 70)
        fake = _FakeIpc(rank)
        ex = mbd.PackedSpikeExchange(shape, device=torch.device("cpu"), native=fake)
        slot = 4 * 3 * 3 * 4  # rows x words x 4 bytes
        ok = ex.slot_bytes == slot
        own = [c[1] for c in fake.calls if c[0] == "alloc"]
        ok = ok and all(c[2] == world * slot for c in fake.calls if c[0] == "alloc")

        def expected_slots(i):
            peers = [((((d + 1) << 40) | (i << 32)) | _FakeIpc.IMPORT) + rank * slot
                     for d in range(world) if d != rank]
            return own[i] + rank * slot, tuple(peers)

        totals = []
        for step in range(3):
            spikes = torch.rand(shape, generator=torch.Generator().manual_seed(10 * step + rank)) < 0.3
            view, counts = ex.pack_count_all_gather(spikes)
            ok = ok and view.shape == (world, 4, 3, 3) and counts.dtype == torch.int64
            totals.append(counts)
            scatter = [c for c in fake.calls if c[0] == "scatter"][-1]
            ok = ok and scatter[1:] == expected_slots(step % 2)  # two buffers, used alternately
        expect = [sum((torch.rand(shape, generator=torch.Generator().manual_seed(10 * s + r)) < 0.3)
                      .sum((0, 1)).to(torch.int64) for r in range(world)) for s in range(3)]
        ok = ok and all(torch.equal(a, b) for a, b in zip(totals, expect))
        # the packed scan path shares the buffer rotation (step 3 uses buffer 1)
        # and completes with a one-word all-reduce that every rank joins
        params = mbd_neurons.LIFParams(tau_mem=4.0)
        x = torch.zeros(shape)
        v0 = torch.full(shape[1:], 0.5)
        vT = ex._scan_scatter(x, v0, params, 1, 0)
        scan = [c for c in fake.calls if c[0] == "scan"][-1]
        ok = ok and scan[1:3] == expected_slots(1) and scan[3] == params.decay and scan[5] == 1
        ok = ok and torch.equal(vT, v0)
        try:
            ex._scan_scatter(torch.zeros((4, 3, 71)), v0, params, 0, 0)
            ok = False  # a shape other than the exchange's must be refused
        except ValueError:
            pass
        ex.close()
        kinds = [c[0] for c in fake.calls]
        # peers' mappings are closed before this rank's buffers are freed
        ok = ok and kinds.count("close") == 2 * (world - 1) and kinds.count("free") == 2
        ok = ok and max(i for i, k in enumerate(kinds) if k == "close") < kinds.index("free")
        # the device is synchronised before any peer mapping goes away
        ok = ok and "sync" in kinds and kinds.index("sync") < kinds.index("close")
        queue.put((rank, bool(ok), ""))
    except Exception as exc:  # pragma: no cover - reported through the queue
        queue.put((rank, False, f"{type(exc).__name__}: {exc}"))
    finally:
        torch_dist.destroy_process_group()


def test_packed_spike_exchange_host_logic_on_two_gloo_ranks(tmp_path: Path):
    world = 2
    ctx = multiprocessing.get_context("spawn")
    queue = ctx.Queue()
    init = f"file://{tmp_path / 'rendezvous_exchange'}"
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, init, queue)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    results = [queue.get(timeout=1) for _ in range(world)]
    assert all(ok for _, ok, _ in results), results
