"""GPU parity of pack / unpack / counts through the C ABI: bit-exact against the
reference's golden vectors and the numpy oracle, for every input dtype, ragged
widths, the high bit, and size-independent properties at config-4 shard size.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import myelin_b200 as mb
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda"

WIDTHS = [1, 31, 32, 33, 65, 100]
DTYPES = [torch.float32, torch.bfloat16, torch.float16, torch.float64, torch.bool, torch.uint8,
          torch.int8, torch.int16, torch.int32, torch.int64]


@pytest.mark.parametrize("n", WIDTHS)
def test_pack_counts_match_reference_golden(n):
    g = load_golden("packing")
    spikes = torch.from_numpy(g[f"spikes_{n}"]).to(DEV)
    packed = mb.pack_spikes(spikes)
    assert packed.data.dtype == torch.int32
    assert packed.original_shape == tuple(spikes.shape)
    assert np.array_equal(packed.data.cpu().numpy(), g[f"packed_{n}"])
    assert np.array_equal(mb.packed_spike_counts(packed, dim=-1).cpu().numpy(), g[f"rows_{n}"])
    assert np.array_equal(mb.packed_spike_count(packed, dim=(0, 1)).cpu().numpy(), g[f"cols_{n}"])
    assert mb.packed_spike_count(packed).item() == int(g[f"total_{n}"])
    assert mb.packed_spike_count(packed).dtype == torch.int64


def _random_spikes(shape, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    keep = torch.rand(shape, generator=gen) < 0.3
    if dtype.is_floating_point:
        vals = torch.randn(shape, generator=gen)
        x = torch.where(keep, vals, torch.zeros_like(vals))
        x.view(-1)[0] = -0.0
        return x.to(dtype)
    if dtype == torch.bool:
        return keep
    vals = torch.randint(-5, 6, shape, generator=gen)
    return torch.where(keep, vals, torch.zeros_like(vals)).to(dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(3, 2, 1), (4, 5, 31), (2, 3, 64), (7, 3, 96), (5, 257), (9, 2, 4096)])
def test_pack_unpack_round_trip_all_dtypes(oracle, dtype, shape):
    spikes = _random_spikes(shape, dtype, hash((shape, str(dtype))) % 997)
    packed = mb.pack_spikes(spikes.to(DEV))
    expected = oracle.pack(spikes.float().numpy() if dtype == torch.bfloat16 else spikes.numpy())
    assert np.array_equal(packed.data.cpu().numpy(), expected)
    out = mb.unpack_spikes(packed, dtype=dtype)
    assert out.dtype == dtype
    assert torch.equal(out.cpu(), (spikes != 0).to(dtype))
    assert torch.equal(mb.unpack_spikes(packed).cpu(), (spikes != 0).float())


def test_high_bit_and_padding_words():
    high = torch.zeros((1, 32), device=DEV)
    high[0, -1] = 1.0
    assert mb.pack_spikes(high).data.item() == -(1 << 31)
    padded = mb.PackedSpikes(data=torch.tensor([[[-1, -1]]], dtype=torch.int32, device=DEV),
                             original_shape=(1, 1, 35))
    assert mb.packed_spike_counts(padded).tolist() == [[35]]
    assert mb.packed_spike_count(padded).item() == 35
    assert mb.packed_spike_count(padded, dim=(0, 1)).sum().item() == 35
    assert torch.allclose(mb.packed_spike_rate(padded).cpu(), torch.tensor(1.0))


def test_dense_like_count_dims_match_dense_sums():
    spikes = _random_spikes((6, 5, 70), torch.float32, 3).to(DEV)
    dense = (spikes != 0).float()
    packed = mb.pack_spikes(spikes)
    for dim in [0, 1, -1, (0, 1), (1, 0), (0, -1), (1, -1)]:
        assert torch.equal(mb.packed_spike_count(packed, dim=dim), dense.sum(dim=dim).to(torch.int64)), dim
    assert torch.allclose(mb.packed_spike_rate(packed, dim=(0, -1)), dense.mean(dim=(0, 2)))


def test_config4_shard_properties(oracle):
    """BASELINE config 4, one shard of 8: Bernoulli(0.05) bool [128, 128, 8192]."""

    T, B, N = 128, 128, 8192
    gen = torch.Generator(device=DEV).manual_seed(4)
    spikes = torch.rand((T, B, N), generator=gen, device=DEV) < 0.05
    packed = mb.pack_spikes(spikes)
    # round trip and idempotence
    assert torch.equal(mb.unpack_spikes(packed, dtype=torch.bool), spikes)
    assert torch.equal(mb.pack_spikes(mb.unpack_spikes(packed, dtype=torch.bfloat16)).data, packed.data)
    # counts agree with dense reductions, in every form
    cols = mb.packed_spike_count(packed, dim=(0, 1))
    assert torch.equal(cols, spikes.sum(dim=(0, 1)))
    cols32 = mb.packed_spike_counts_over_leading_dims(packed, dtype=torch.int32)
    assert torch.equal(cols32.to(torch.int64), cols)
    rows = mb.packed_spike_counts(packed, dim=-1)
    assert torch.equal(rows, spikes.sum(dim=-1))
    assert mb.packed_spike_count(packed).item() == int(spikes.sum().item()) == int(cols.sum().item())
    # one slice against the oracle bit for bit
    sl = spikes[:4].cpu().numpy()
    assert np.array_equal(packed.data[:4].cpu().numpy(), oracle.pack(sl))


@pytest.mark.parametrize("n", WIDTHS)
def test_pack_with_counts_matches_reference_golden(n):
    g = load_golden("packing")
    spikes = torch.from_numpy(g[f"spikes_{n}"]).to(DEV)
    packed, counts = mb.pack_spikes_with_counts(spikes)
    assert np.array_equal(packed.data.cpu().numpy(), g[f"packed_{n}"])
    assert counts.dtype == torch.int64
    assert np.array_equal(counts.cpu().numpy(), g[f"cols_{n}"])


@pytest.mark.parametrize("dtype", [torch.bool, torch.uint8, torch.int8, torch.float32,
                                   torch.bfloat16])
@pytest.mark.parametrize("shape", [(3, 1, 32), (5, 7, 64), (300, 96), (37, 3, 256),
                                   (1000, 8192), (6, 5, 33), (2, 513)])
@pytest.mark.parametrize("count_dtype", [torch.int64, torch.int32])
def test_pack_with_counts_matches_oracle(oracle, dtype, shape, count_dtype):
    """Fused path (1-byte, n % 32 == 0) and the pack-then-count path agree
    bit for bit with the oracle, including 1-byte values other than 0/1."""

    spikes = _random_spikes(shape, dtype, hash((shape, str(dtype), "pc")) % 991)
    if dtype in (torch.uint8, torch.int8):
        spikes.view(-1)[:7] = torch.tensor([1, 2, 127, -128 if dtype == torch.int8 else 128, 255
                                            if dtype == torch.uint8 else -1, 0, 64]).to(dtype)
    host = spikes.float().numpy() if dtype == torch.bfloat16 else spikes.numpy()
    packed, counts = mb.pack_spikes_with_counts(spikes.to(DEV), dtype=count_dtype)
    assert np.array_equal(packed.data.cpu().numpy(), oracle.pack(host))
    n = shape[-1]
    expected = (host.reshape(-1, n) != 0).sum(axis=0)
    assert counts.dtype == count_dtype
    assert np.array_equal(counts.cpu().numpy().astype(np.int64), expected)


@pytest.mark.parametrize("rows,n", [(70000, 64), (160000, 4096)])
def test_pack_with_counts_long_columns_flush(rows, n):
    """More rows per block than the 8-bit counters hold between flushes (255),
    all ones, on the per-word-column kernel (n = 64) and the whole-row kernel
    (n = 4096: blocks of 272 rows): every column count equals the row
    count."""

    spikes = torch.ones((rows, n), dtype=torch.bool, device=DEV)
    packed, counts = mb.pack_spikes_with_counts(spikes)
    assert bool(torch.all(counts == rows))
    assert bool(torch.all(packed.data == -1))
