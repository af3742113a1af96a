"""The allocation-free column count, called through the C ABI.

``mb_count_columns_noalloc`` serves callers that cannot allocate device memory
when they count (a host runtime that owns all device memory in its own arena,
or a loop where an allocation would block on the device): its scratch is a
fixed array inside the library instead of a caller-provided workspace. It must
give exactly the counts of ``mb_count_columns`` (integers: bit-exact), also on
the second of two calls in a row, when the shared array still holds the first
call's partial sums. This file is collected last so that a run stopping at the
first failure has already run every other test.
"""

from __future__ import annotations

import pytest
import torch

from myelin_b200 import _native as nat

pytestmark = pytest.mark.gpu
DEV = "cuda"
MAX_BYTES = 4 << 20  # MB_COUNT_COLUMNS_NOALLOC_MAX_BYTES


def _words(shape, p, seed):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    spikes = torch.rand(shape, generator=gen, device=DEV) < p
    import myelin_b200 as mb

    return mb.pack_spikes(spikes).data.contiguous(), spikes


def _count_with_workspace(words, rows, n):
    c64 = torch.empty(n, dtype=torch.int64, device=DEV)
    c32 = torch.empty(n, dtype=torch.int32, device=DEV)
    nat.count_columns(words, rows, n, c64, c32)
    return c64, c32


def _count_noalloc(words, rows, n):
    lib = nat.lib()
    c64 = torch.full((n,), -7, dtype=torch.int64, device=DEV)
    c32 = torch.full((n,), -7, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    status = lib.mb_count_columns_noalloc(words.data_ptr(), rows, n, c64.data_ptr(),
                                          c32.data_ptr(), stream)
    assert status == 0, lib.mb_last_error().decode()
    return c64, c32


@pytest.mark.parametrize(
    "shapes",
    [
        [((128, 128, 8192), 0.05, 1), ((64, 96, 8192), 0.3, 2)],  # config-4 shard, then a denser one
        [((7, 3, 45), 0.4, 3), ((300, 5, 70), 0.1, 4)],            # ragged widths, many rows
        # 74 row slices, then 2: the second call must not read the partial
        # sums the first call left in slices 2..73
        [((128, 128, 8192), 0.05, 5), ((2, 64, 8192), 0.2, 6)],
    ],
)
def test_noalloc_counts_match_workspace_counts_on_consecutive_calls(shapes):
    for shape, p, seed in shapes:
        words, spikes = _words(shape, p, seed)
        rows = words.numel() // words.shape[-1]
        n = shape[-1]
        need = nat.lib().mb_count_columns_workspace_bytes(rows, n)
        assert need <= MAX_BYTES
        ref64, ref32 = _count_with_workspace(words, rows, n)
        got64, got32 = _count_noalloc(words, rows, n)
        torch.cuda.synchronize()
        assert torch.equal(got64, ref64)
        assert torch.equal(got32, ref32)
        assert torch.equal(got64, spikes.reshape(-1, n).sum(dim=0))


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = nat.lib()
    n = 1 << 22  # 4M neurons: the partial sums alone exceed the built-in scratch
    rows = 1 << 12
    assert lib.mb_count_columns_workspace_bytes(rows, n) > MAX_BYTES
    out = torch.empty(1, dtype=torch.int64, device=DEV)
    status = lib.mb_count_columns_noalloc(out.data_ptr(), rows, n, out.data_ptr(), None,
                                          torch.cuda.current_stream().cuda_stream)
    assert status != 0
    assert "scratch" in lib.mb_last_error().decode()
