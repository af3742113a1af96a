"""Peer-scatter entry points on one GPU, with other buffers of the same GPU
standing in for the peers' gather slots.

``mb_scan_forward_packed_scatter`` and ``mb_pack_count_scatter`` store this
rank's words into its own slot and into every peer slot. Any device pointer
is a valid destination, so one GPU checks the kernels' indexing and the
push kernel's 16-byte and 4-byte paths; the NVLink case itself runs in
tests/test_distributed_gpu.py. Every destination must equal the ordinary
packed output bit for bit (src/myelin/kernels.py:96-156, packing.py:45-71).
"""

from __future__ import annotations

import pytest
import torch

import myelin_b200 as mb
from myelin_b200 import _native as nat

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.mark.parametrize("shape,peers", [
    ((33, 4, 96), 1),       # 33*4*3 words: 1584 B, 16-byte pushes
    ((33, 5, 96), 3),       # 1980 B: 4-byte pushes
    ((256, 64, 1024), 7),   # 2 MiB: several grid-stride passes
    ((7, 3, 70), 2),        # ragged N: the general forward, then the push
])
def test_scan_forward_packed_scatter_local_peers(shape, peers):
    T, B, N = shape
    g = torch.Generator(device=DEV).manual_seed(T + B + N)
    x = 0.3 + 0.5 * torch.randn(shape, generator=g, device=DEV)
    v0 = torch.full((B, N), 0.1, device=DEV)
    params = mb.LIFParams(tau_mem=7.0)
    ref_state, ref = mb.lif_forward_packed_spikes(x, mb.LIFState(v0), params)
    W = (N + 31) // 32
    own = torch.full((T, B, W), -1, dtype=torch.int32, device=DEV)
    slots = [torch.full((T, B, W), -1, dtype=torch.int32, device=DEV) for _ in range(peers)]
    vT = torch.empty_like(v0)
    for _ in range(2):  # the same result on a second call into the same slots
        nat.scan_forward_packed_scatter(
            neuron=nat.MB_LIF, x=x, v0=v0, a0=None, vT=vT, aT=None, packed=own.data_ptr(),
            peers=[s.data_ptr() for s in slots], decay=params.decay,
            threshold=float(params.threshold), reset=float(params.reset), adapt_decay=0.0,
            beta=0.0, reset_mode=nat.MB_RESET_HARD,
        )
        torch.cuda.synchronize()
        assert torch.equal(own, ref.data)
        assert torch.equal(vT, ref_state.membrane)
        for s in slots:
            assert torch.equal(s, ref.data)
    assert nat.device_status(clear=True) == 0


@pytest.mark.parametrize("shape,peers", [
    ((16, 8, 256), 7),     # fused pack kernel storing to 7 peer slots
    ((6, 5, 70), 3),       # ragged N: pack + count, then the push
    ((16, 8, 8192), 7),    # whole-row blocks (256 words), bulk copies to 8 slots
    ((37, 5, 4096), 2),    # whole-row blocks (128 words), a ragged last group
    ((128, 64, 8192), 1),  # many groups per block: both staging buffers reused
    ((3, 1, 8192), 0),     # own slot only, fewer rows than one group
])
def test_pack_count_scatter_local_peers(shape, peers):
    rows, n = shape[0] * shape[1], shape[2]
    g = torch.Generator(device=DEV).manual_seed(n)
    spikes = torch.rand(shape, generator=g, device=DEV) < 0.2
    ref = mb.pack_spikes(spikes).data
    W = (n + 31) // 32
    own = torch.full((shape[0], shape[1], W), -1, dtype=torch.int32, device=DEV)
    slots = [torch.full_like(own, -1) for _ in range(peers)]
    counts = torch.empty((n,), dtype=torch.int64, device=DEV)
    for _ in range(2):
        nat.pack_count_scatter(spikes, own.data_ptr(), rows, n, [s.data_ptr() for s in slots],
                               counts, None)
        torch.cuda.synchronize()
        assert torch.equal(own, ref)
        for s in slots:
            assert torch.equal(s, ref)
        assert torch.equal(counts, spikes.sum(dim=(0, 1)).to(torch.int64))
    assert nat.device_status(clear=True) == 0
