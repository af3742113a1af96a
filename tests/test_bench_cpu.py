"""The reference arm of bench.py (myelin's own CPU path of the headline step,
timed on this host) prints one JSON line in the contract's shape: the same
metric, unit and direction as the GPU arm, `impl: reference`, a cpu_baseline
describing the run and an end-to-end figure with no host<->device bytes."""

from __future__ import annotations

import json
import subprocess
import sys

from tests.conftest import ROOT


def test_reference_arm_json_line():
    proc = subprocess.run(
        [sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
        cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, proc.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "LIF/ALIF fwd+bwd neuron-timesteps/s"
    assert d["unit"] == "neuron-steps/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] >= 3
    assert d["vs_baseline"] is None and d["dtype"] == "bf16"
    assert d["config"]["workload"] == "alif_bf16"
    assert (d["config"]["T"], d["config"]["B_per_gpu"], d["config"]["N"]) == (256, 128, 4096)
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1 and cb["kind"] in ("port", "reference")
    assert cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
