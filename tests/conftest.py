"""Test configuration: the ``gpu`` marker and shared helpers.

``-m "not gpu"`` runs on CPU (oracle vs golden vectors, host logic, C-ABI
loading); ``-m gpu`` needs a CUDA device and compares the CUDA kernels, called
through the C ABI, with the oracle.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def assert_close_scaled(actual, expected, rtol: float = 1e-5, what: str = "") -> None:
    """|a - b| <= rtol * |b| + rtol * max|b| elementwise.

    The gradient bar for fp32: relative 1e-5, with an absolute floor of 1e-5
    times the tensor's largest magnitude. The reverse-time adjoint multiplies
    through many steps, and on the few elements where two terms nearly cancel
    two fp32 orderings of the same formula (the reference's own autograd vs
    its closed form) already differ by more than 1e-5 relative.
    """

    a = np.asarray(actual, dtype=np.float64)
    b = np.asarray(expected, dtype=np.float64)
    assert a.shape == b.shape, (what, a.shape, b.shape)
    scale = float(np.max(np.abs(b))) if b.size else 0.0
    tol = rtol * np.abs(b) + rtol * scale
    bad = np.abs(a - b) > tol
    if np.any(bad):
        idx = np.argwhere(bad)[0]
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{b.size} elements exceed rtol={rtol} (scaled); "
            f"first at {tuple(idx)}: {a[tuple(idx)]} vs {b[tuple(idx)]}, max|b|={scale}"
        )


def load_golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    o.build()
    return o
