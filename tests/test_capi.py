"""The C-ABI library loads, exports every symbol include/myelin_b200.h declares,
and its host-side argument checks report errors (no device work needed)."""

from __future__ import annotations

import ctypes
import re

import pytest

from myelin_b200 import _native as nat
from tests.conftest import ROOT

HEADER = ROOT / "include" / "myelin_b200.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(mb_[a-z0-9_]+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    lib = nat.lib()
    declared = declared_symbols()
    assert {"mb_scan_forward", "mb_scan_backward", "mb_pack_spikes", "mb_count_columns"} <= declared
    missing = [name for name in sorted(declared) if not hasattr(lib, name)]
    assert not missing, missing
    assert declared == set(nat.EXPORTED_SYMBOLS), "ctypes signatures out of sync with the header"


def test_host_side_queries():
    lib = nat.lib()
    assert nat.version().startswith("myelin_b200")
    assert lib.mb_scan_num_checkpoints(0) == 0
    assert lib.mb_scan_num_checkpoints(1) == 1
    assert lib.mb_scan_num_checkpoints(256) == 256 // nat.SCAN_CHUNK
    assert lib.mb_scan_num_checkpoints(257) == 256 // nat.SCAN_CHUNK + 1
    assert lib.mb_count_columns_workspace_bytes(0, 10) == 0
    ws = lib.mb_count_columns_workspace_bytes(16384, 8192)
    assert ws > 0 and ws % (4 * 8192) == 0


@pytest.mark.parametrize(
    "call, fragment",
    [
        (lambda l: l.mb_scan_forward(0, 99, None, None, None, None, None, None, None, None, None,
                                     None, 1, 1, 1, 0.9, 1.0, 0.0, 0.0, 0.0, 0, None),
         "unsupported dtype"),
        (lambda l: l.mb_scan_forward(5, 0, None, None, None, None, None, None, None, None, None,
                                     None, 1, 1, 1, 0.9, 1.0, 0.0, 0.0, 0.0, 0, None),
         "unknown neuron"),
        (lambda l: l.mb_scan_forward(0, 0, None, None, None, None, None, None, None, None, None,
                                     None, 1, 1, 1, 0.9, 1.0, 0.0, 0.0, 0.0, 7, None),
         "reset mode"),
        (lambda l: l.mb_scan_backward(0, 0, None, None, None, None, None, None, None, None, None,
                                      None, 1, 1, 1, 0.9, 1.0, 0.0, 0.0, 0.0, 0, 42, 1.0, None),
         "surrogate"),
        (lambda l: l.mb_pack_spikes(0, None, None, 3, 0, None), "empty last dimension"),
        (lambda l: l.mb_unpack_spikes(None, 0, None, 3, 0, None), "non-empty last dimension"),
        (lambda l: l.mb_count_columns(None, 4, 64, None, None, None, 0, None), "no output"),
    ],
)
def test_argument_errors_are_reported(call, fragment):
    lib = nat.lib()
    assert call(lib) != 0
    assert fragment in lib.mb_last_error().decode()


def test_empty_problem_is_a_no_op():
    lib = nat.lib()
    # B*N == 0: nothing to launch, success without touching the device
    assert lib.mb_scan_forward(0, 0, None, None, None, None, None, None, None, None, None, None,
                               4, 0, 8, 0.9, 1.0, 0.0, 0.0, 0.0, 0, None) == 0
    assert lib.mb_pack_spikes(0, None, None, 0, 8, None) == 0
    assert lib.mb_last_error().decode() == ""


def test_library_is_a_plain_shared_object():
    handle = ctypes.CDLL(str(nat.LIB_PATH))
    assert handle.mb_version.restype is not None or True


def test_gemm_work_plan_sizes():
    """Host-side K-slice plans of mb_gemm, through the workspace each needs
    (with no GPU visible the library plans for the B200's 148 SMs, 74 SM pairs).

    - K < 8192 with many tiles: no slicing, no workspace;
    - config-5 weight gradient (4096 x 4096 outputs, K = T*B = 51200, bf16):
      256 pair tiles = 3 whole waves of 74 + 34 tail tiles, sliced in 2; the
      fp32 partials cover only the tail tiles' rows, 3328 .. 4095;
    - fp32 output from 3-part split operands (config-2 layer-1 weight
      gradient, 784 x 1024, K = 6400): accuracy slices of at most 2048 of K,
      4 of them over the whole output;
    - a 10-wide output with long K: sliced until the units fill the SMs."""

    lib = nat.lib()
    ws = lib.mb_gemm_workspace_bytes
    assert ws(51200, 4096, 4096, 1, 1, nat.MB_BF16) == 0
    tail = 2 * (4096 - 13 * 256) * 4096 * 4
    assert ws(4096, 4096, 51200, 1, 1, nat.MB_BF16) == tail
    assert ws(4096, 4096, 8192, 1, 1, nat.MB_BF16) == tail
    assert ws(4096, 4096, 51200, 1, 1, nat.MB_F32) == tail
    assert ws(784, 1024, 6400, 3, 3, nat.MB_F32) == 4 * 784 * 1024 * 4
    narrow = ws(4096, 10, 51200, 1, 1, nat.MB_BF16)
    assert narrow > 0 and narrow % (4096 * 12 * 4) == 0  # slices x M x pitch(10 -> 12) x fp32
    assert ws(0, 10, 10, 1, 1, nat.MB_BF16) == 0
