"""A bounded wait that runs out is reported, in every code unit that has one.

Each unit (the general scan kernels, the fast scan kernels, the tensor-core
GEMMs) keeps its own device status word; ``mb_device_status`` reads and
clears all of them. A diagnostic kernel in each unit waits on a barrier that
nothing arrives at with a small poll budget, so its wait runs out through the
same code path as the real kernels' waits. Nothing faults and nothing spins
without bound: the probe returns after its polls.
"""

from __future__ import annotations

import pytest
import torch

from myelin_b200 import _native as nat

UNITS = {"scan": nat.MB_UNIT_SCAN, "scan_fast": nat.MB_UNIT_SCAN_FAST, "gemm": nat.MB_UNIT_GEMM}


@pytest.mark.gpu
@pytest.mark.parametrize("unit", sorted(UNITS))
def test_wait_timeout_is_reported_and_cleared(unit):
    assert nat.device_status(clear=True) == 0
    nat.debug_wait_timeout(UNITS[unit], polls=64)
    torch.cuda.synchronize()
    # read without clearing, then read and clear, then clean
    assert nat.device_status(clear=False) == 1
    assert nat.device_status(clear=True) == 1
    assert nat.device_status(clear=True) == 0


@pytest.mark.gpu
def test_every_unit_reports_at_once():
    for code in UNITS.values():
        nat.debug_wait_timeout(code, polls=16)
    torch.cuda.synchronize()
    assert nat.device_status(clear=True) == 1
    assert nat.device_status(clear=True) == 0


def test_probe_argument_checks():
    lib = nat.lib()
    assert lib.mb_debug_wait_timeout(nat.MB_UNIT_SCAN, 0, None) != 0
    assert "polls" in lib.mb_last_error().decode()
    assert lib.mb_debug_wait_timeout(nat.MB_UNIT_SCAN, 1 << 20, None) != 0
    assert lib.mb_debug_wait_timeout(9, 16, None) != 0
    assert "unknown unit" in lib.mb_last_error().decode()
