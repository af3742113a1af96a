"""Benchmark of the myelin_b200 hot path (one JSON line on stdout, rank 0).

Workload (default ``alif_bf16``, BASELINE config 3, the shape the north-star
metric is quoted on): ALIF forward + atan-surrogate backward, T=256, B=128,
N=4096, bf16 currents ~ N(0.2, 0.6), tau_mem=10 (decay 0.9), tau_adaptation=50
(rho 0.98), beta=1.8, threshold 1, subtractive reset, checkpoint_size="memory",
upstream spike gradient ~ N(0, 1). A step is one forward + backward pass through
the public API (``surrogate_alif_forward`` + autograd) over one batch.
Other workloads: ``lif_fp32`` (same shape, LIF, fp32, hard reset),
``pack_count`` (config 4 shard: Bernoulli(0.05) bool [128, 1024/N, 8192] ->
packed words + per-neuron int32 counts), ``mlp_fp32`` (config 2: one training
step of the 784 -> 1024 -> 10 stream-synapse LIF MLP, fp32) and ``rate_net``
(config 5: one training step of 4 x 4096 hidden stream-synapse LIF layers and
a 4096 -> 10 rate readout, bf16, T=100, B=512 per GPU, with the gradient
all-reduce across ranks), ``izhikevich_fp32`` (Izhikevich forward at the
north-star shape) and ``lif_packed`` (LIF forward with packed words only at
the north-star shape, plus the packed all-gather at N > 1).

Multi-GPU (torchrun, one process per GPU): the scan workloads run one batch
shard of the same size per rank (weak scaling, no collective on the data
path); ``pack_count`` splits config 4's batch of 1024 over the ranks (strong
scaling) and all-gathers the packed words and all-reduces the counts, through
the peer-mapped exchange by default (``--allgather fused``) or NCCL
(``--allgather nccl``). The value is all ranks' units divided by the
max-over-ranks device time. At N > 1 the default run also times BASELINE
config 4's packed reductions on the same ranks (the ``collective`` key: the
fused peer-store exchange and pack + NCCL, each with an in-run bit-exact
parity check against every rank's regenerated shard).

CPU figures: ``--impl reference`` (and the GPU arm's ``cpu_baseline`` at N = 1)
time myelin's own CPU implementation of the path, its torch per-timestep loop
+ autograd (restated in ``oracle/torch_path.py``), at the full config-3 step
on all host threads, next to the C restatement of the same scan
(``oracle/scan_oracle.c``, OpenMP) on a 32-row sample, both by the same
per-step timing method.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
FALLBACK_HBM_GBS = 6650.0

# ---------------------------------------------------------------------------
# workload definitions
# ---------------------------------------------------------------------------
T_STEPS, BATCH, NEURONS = 256, 128, 4096

# algorithmic bytes per neuron-step, from the API's inputs and outputs plus the fp32
# chunk checkpoints (4 B per state every 16 steps)
#   forward : read x, write dense spikes, write fp32 checkpoints (s states / 16 steps)
#   backward: read x, read grad_spikes, write grad_x, read checkpoints
ALGO_BYTES = {
    "alif_bf16": {"fwd": 2 + 2 + 4 * 2 / 16, "bwd": 2 + 2 + 2 + 4 * 2 / 16},
    "lif_fp32": {"fwd": 4 + 4 + 4 * 1 / 16, "bwd": 4 + 4 + 4 + 4 * 1 / 16},
}


def load_peak_hbm() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(name: str) -> float | None:
    """DRAM bytes per launch from a committed ncu summary, if one exists."""

    path = ROOT / "profiles" / f"{name}.json"
    if not path.exists():
        return None
    try:
        return float(json.loads(path.read_text())["dram_bytes_per_launch"])
    except (KeyError, ValueError):
        return None


# ---------------------------------------------------------------------------
# clocks sampled during the timed region (NVML reads only)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "hw_slowdown": 0x0000000000000008,
        "sw_thermal_slowdown": 0x0000000000000020,
        "hw_thermal_slowdown": 0x0000000000000040,
        "sw_power_cap": 0x0000000000000004,
        "hw_power_brake_slowdown": 0x0000000000000080,
    }

    def __init__(self, device_index: int, period_s: float = 0.005) -> None:
        self.samples: list[tuple[float, int, int]] = []
        self.period = period_s
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML missing: report no clocks rather than fail the bench
            self._nvml = None

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def _run(self) -> None:
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                self.samples.append((time.perf_counter(), mhz, reasons))
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *exc) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self) -> dict | None:
        if self._nvml is None or not self.samples:
            return None
        mhz = [s[1] for s in self.samples]
        reasons = set()
        for _, _, r in self.samples:
            for name, bit in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": float(statistics.median(mhz)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(mhz)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def scan_workload(name: str, rank: int):
    """Two seeded input sets (x, grad_spikes) of the workload and its forward.
    Steps alternate between the sets: each set is larger than L2, so no step
    reads inputs the step before left in L2 (the forward -> backward reuse
    inside a step is real, a step -> step reuse of the same inputs would not
    be)."""

    import myelin_b200 as mb

    shape = (T_STEPS, BATCH, NEURONS)
    sets = []
    for k in range(2):
        gen = torch.Generator(device="cuda").manual_seed(1234 + rank + 1000 * k)
        if name == "alif_bf16":
            x = (torch.randn(shape, generator=gen, device="cuda") * 0.6 + 0.2).to(torch.bfloat16)
            gs = torch.randn(shape, generator=gen, device="cuda").to(torch.bfloat16)
        else:
            x = torch.randn(shape, generator=gen, device="cuda") * 0.5 + 0.3
            gs = torch.randn(shape, generator=gen, device="cuda")
        sets.append((x, gs))
    if name == "alif_bf16":
        dtype = torch.bfloat16
        params = mb.ALIFParams(tau_mem=10.0, tau_adaptation=50.0, threshold=1.0, reset=0.0,
                               beta=1.8)
        zeros = torch.zeros((BATCH, NEURONS), dtype=dtype, device="cuda")

        def forward(xin):
            state, spikes = mb.surrogate_alif_forward(
                xin, mb.ALIFState(zeros, zeros), params, surrogate="atan",
                checkpoint_size="memory", reset_mode="subtract")
            return spikes
    else:
        dtype = torch.float32
        params = mb.LIFParams(tau_mem=10.0, threshold=1.0, reset=0.0)
        zeros = torch.zeros((BATCH, NEURONS), dtype=dtype, device="cuda")

        def forward(xin):
            state, spikes = mb.surrogate_lif_forward(xin, mb.LIFState(zeros), params,
                                                     surrogate="atan", checkpoint_size="memory")
            return spikes
    return sets, forward


def run_gpu(args) -> None:
    world, rank, local = dist_setup(args.gpus)
    from myelin_b200 import _native as nat

    name = args.workload
    if name == "pack_count":
        return run_pack_count(args, world, rank, local)
    if name in ("mlp_fp32", "rate_net"):
        return run_network(args, world, rank, local)
    if name == "izhikevich_fp32":
        return run_izhikevich(args, world, rank, local)
    if name == "lif_packed":
        return run_lif_packed(args, world, rank, local)
    sets, forward = scan_workload(name, rank)
    for xs, _ in sets:
        xs.requires_grad_(True)
    x, gs = sets[0]
    stream = torch.cuda.current_stream()
    units = T_STEPS * BATCH * NEURONS  # neuron-steps per rank per step

    def step(xin, g):
        spikes = forward(xin)
        (gx,) = torch.autograd.grad(spikes, xin, g)
        return gx

    # warm up like the timed loop below: the previous step's spikes (and the
    # checkpoints they hold) stay alive while the next forward allocates, so
    # the allocator has cached every block before timing starts
    for k in range(args.warmup):
        xs, g = sets[k % 2]
        spikes = forward(xs)
        torch.autograd.grad(spikes, xs, g)
    torch.cuda.synchronize()

    # eager: the public API called step by step, per-kernel events on the
    # launching stream (these include the host's per-call gaps when the host
    # falls behind the device)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record(stream)
    t_host = time.perf_counter()
    for k in range(args.steps):
        e0, e1, e2 = ev[k]
        xs, g = sets[k % 2]
        e0.record(stream)
        spikes = forward(xs)
        e1.record(stream)
        torch.autograd.grad(spikes, xs, g)
        e2.record(stream)
    stop.record(stream)
    # host time to issue the steps: at or above the device time per step,
    # the eager step is bound by the host's per-call work
    host_ms = (time.perf_counter() - t_host) * 1e3 / args.steps
    torch.cuda.synchronize()
    barrier(world)
    eager_ms = max_over_ranks(start.elapsed_time(stop), world) / args.steps
    eager_fwd_ms = statistics.mean(a.elapsed_time(b) for a, b, _ in ev)
    eager_bwd_ms = statistics.mean(b.elapsed_time(c) for _, b, c in ev)

    # headline: the same public-API step (forward + autograd backward) captured
    # once in a CUDA graph and replayed, so the device runs the step's kernels
    # back to back without waiting on the host between launches
    # (a fresh leaf: autograd binds a leaf's gradient sink to the stream it
    # was first used on, and the eager loop above used the legacy stream)
    # One graph per input set; the timed loop alternates them.
    leaves = [(xs.detach().requires_grad_(True), g) for xs, g in sets]
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.stream(cap):
        for _ in range(2):
            for xg, g in leaves:
                torch.autograd.grad(forward(xg), xg, g)
    stream.wait_stream(cap)
    torch.cuda.synchronize()
    step_graphs = []
    for xg, g in leaves:
        graph_k = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_k, stream=cap):
            torch.autograd.grad(forward(xg), xg, g)
        step_graphs.append(graph_k)
    for k in range(args.warmup):
        step_graphs[k % 2].replay()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record(stream)
        for k in range(args.steps):
            step_graphs[k % 2].replay()
        stop.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    total_ms = max_over_ranks(start.elapsed_time(stop), world)
    ms_per_step = total_ms / args.steps
    value = units * world / (ms_per_step / 1e3)
    del step_graphs, leaves
    status = nat.device_status(clear=True)
    # per-kernel device times for the roofline: the step's two kernels, each
    # replayed from its own graph with events between them
    graph = graph_replay_diagnostic(name, sets, stream, args.steps, world)
    timing = graph.get("in_graph", graph)
    fwd_ms, bwd_ms = timing["fwd_launch_ms"], timing["bwd_launch_ms"]
    launch_times = ("CUDA events recorded as nodes of one graph holding the step's two kernels"
                    if "in_graph" in graph else
                    "CUDA events between graph replays of the step's kernels")

    # end to end through the public API with host buffers
    pinned_x = x.detach().cpu().pin_memory()
    pinned_g = gs.cpu().pin_memory()
    out_host = torch.empty(x.shape, dtype=x.dtype).pin_memory()
    e2e_steps = max(1, min(args.steps, 20))
    # The result read of step i runs on a second stream, ordered after the
    # step's kernels by an event, so it overlaps the next step's host-to-device
    # copies (PCIe is full duplex); everything else is the plain public API.
    copy_stream = torch.cuda.Stream()

    def e2e_step():
        xd = pinned_x.to("cuda", non_blocking=True).requires_grad_(True)
        gd = pinned_g.to("cuda", non_blocking=True)
        gx = step(xd, gd)
        done = torch.cuda.Event()
        done.record(stream)
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(done)
            out_host.copy_(gx, non_blocking=True)
        gx.record_stream(copy_stream)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    s2, t2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    stream.wait_stream(copy_stream)
    t2.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s2.elapsed_time(t2), world) / e2e_steps
    elt = x.element_size()

    peak, peak_kind = load_peak_hbm()
    bytes_fwd = ALGO_BYTES[name]["fwd"] * units
    bytes_bwd = ALGO_BYTES[name]["bwd"] * units

    def roof(bytes_per_launch: float, ms: float, profile: str) -> dict:
        achieved = bytes_per_launch / (ms / 1e3) / 1e9
        return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "traffic": profile_traffic(profile),
                "algorithmic_bytes": int(bytes_per_launch), "avg_launch_ms": round(ms, 4),
                "launch_times": launch_times}

    def step_roof(step_bytes: float, ms: float, peak: float, peak_kind: str) -> dict:
        # the forward leaves up to an L2's worth of dirty output lines whose
        # write-back falls into the backward; per kernel that shifts time from
        # the forward to the backward, for the step it nets out
        achieved = step_bytes / (ms / 1e3) / 1e9
        return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "algorithmic_bytes": int(step_bytes), "ms": round(ms, 4),
                "what": "both scan kernels of the step: forward + backward algorithmic bytes over "
                        "the headline step time (the graph replays, everything in the step)"}

    result = {
        "metric": "LIF/ALIF fwd+bwd neuron-timesteps/s",
        "value": value,
        "unit": "neuron-steps/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16" if name == "alif_bf16" else "f32",
        "data": "synthetic (seeded on device; shapes/distributions of BASELINE config 3)",
        "config": {
            "workload": name + (" (BASELINE config 3: ALIF fwd + atan bwd, checkpoint_size=memory,"
                                " subtractive reset)" if name == "alif_bf16" else
                                " (LIF fwd + atan bwd at the config-3 shape)"),
            "T": T_STEPS, "B_per_gpu": BATCH, "N": NEURONS, "global_batch": BATCH * world,
            "parallelism": f"dp{world} (batch-sharded, no data-path collective)",
            "l2": "inputs larger than L2 (x and grad_spikes are T*B*N*elt = "
                  f"{units * elt / 1e6:.0f} MB each), no flush; two input sets, "
                  "steps alternate between them, so no step reads inputs the previous "
                  "step left in L2",
            "cuda_graph": "the public-API step (forward + autograd backward) captured once "
                          "and replayed; the eager figure is under 'eager'",
        },
        "roofline": roof(bytes_bwd, bwd_ms, f"scan_bwd_{name}"),
        "roofline_fwd": roof(bytes_fwd, fwd_ms, f"scan_fwd_{name}"),
        "roofline_step": step_roof(bytes_fwd + bytes_bwd, ms_per_step, peak, peak_kind),
        "e2e": {"value": units * world / (e2e_ms / 1e3), "unit": "neuron-steps/s",
                "h2d_bytes_per_step": 2 * units * elt, "d2h_bytes_per_step": units * elt,
                "ms_per_step": e2e_ms},
        "gpu_launches": 2 * args.steps,
        "device_status": status,
        "kernels_graph_replay": graph,
        "eager": {"ms_per_step": round(eager_ms, 4),
                  "value": units * world / (eager_ms / 1e3),
                  "fwd_launch_ms": round(eager_fwd_ms, 4), "bwd_launch_ms": round(eager_bwd_ms, 4),
                  "host_issue_ms_per_step": round(host_ms, 4),
                  "note": "the public API called step by step without a graph"},
    }
    clk = clocks.summary()
    if clk is not None:
        result["clocks"] = clk
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(name, seconds=args.cpu_seconds)
    if world > 1:
        import torch.distributed as dist

        # the packed reductions on the same ranks, after the
        # scan's own numbers are final: every rank takes part
        result["collective"] = collective_leg(world, rank, local, args.steps, args.warmup)
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def graph_replay_diagnostic(name: str, sets, stream, steps: int, world: int) -> dict:
    """The step's two kernels (the scan forward and backward the public API
    launches, called here through the same ops with the workload's
    parameters) captured in CUDA graphs and replayed, alternating between the
    two input sets like the timed step: the kernels' device time without the
    host's per-launch work (Python, autograd) in between. A gap between this
    and the eager step says how much of the eager time is the host's."""

    from myelin_b200 import _native as nat
    from myelin_b200 import compile_ops as cops

    alif = name == "alif_bf16"
    kw = dict(neuron=nat.MB_ALIF if alif else nat.MB_LIF, decay=0.9, threshold=1.0, reset=0.0,
              adapt_decay=(1.0 - 1.0 / 50.0) if alif else 0.0, beta=1.8 if alif else 0.0,
              reset_mode=nat.MB_RESET_SUBTRACT if alif else nat.MB_RESET_HARD)
    x0 = sets[0][0]
    B, N = x0.shape[1], x0.shape[2]
    zeros = torch.zeros((B, N), dtype=x0.dtype, device=x0.device)
    inputs = [(xs.detach(), g) for xs, g in sets]

    def fwd(k):
        out = cops.scan_forward(inputs[k][0], zeros, zeros if alif else None, kw["neuron"],
                                kw["decay"], kw["threshold"], kw["reset"], kw["adapt_decay"],
                                kw["beta"], kw["reset_mode"], dense=True, checkpoints=True)
        return out[5], out[6]

    def bwd(k, ckpt_v, ckpt_a):
        return cops.scan_backward(inputs[k][0], ckpt_v, ckpt_a, grad_spikes=inputs[k][1],
                                  grad_vT=None, grad_aT=None, surrogate=2, slope=10.0,
                                  need_v0=False, need_a0=False, **kw)[0]

    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.stream(cap):
        for _ in range(2):
            for k in range(2):
                bwd(k, *fwd(k))
    stream.wait_stream(cap)
    torch.cuda.synchronize()
    graphs = []
    for k in range(2):
        g_fwd, g_bwd = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_fwd, stream=cap):
            ckpts = fwd(k)
        with torch.cuda.graph(g_bwd, pool=g_fwd.pool(), stream=cap):
            bwd(k, *ckpts)
        graphs.append((g_fwd, g_bwd))
    for _ in range(3):
        for g_fwd, g_bwd in graphs:
            g_fwd.replay()
            g_bwd.replay()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    for i, (e0, e1, e2) in enumerate(ev):
        g_fwd, g_bwd = graphs[i % 2]
        e0.record(stream)
        g_fwd.replay()
        e1.record(stream)
        g_bwd.replay()
        e2.record(stream)
    torch.cuda.synchronize()
    total = max_over_ranks(ev[0][0].elapsed_time(ev[-1][2]), world) / steps
    fwd_ms = statistics.mean(a.elapsed_time(b) for a, b, _ in ev)
    bwd_ms = statistics.mean(b.elapsed_time(c) for _, b, c in ev)
    del graphs

    # Both sets' kernels in ONE graph with event-record nodes before, between
    # and after them: each kernel's device time as it runs inside the
    # alternating steps, with no graph launch (and its host round trip)
    # between kernels. Every rank takes the same collective steps whether or
    # not this works here.
    in_fwd = in_bwd = in_over = -1.0
    try:
        evs = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(6)]
        g_one = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_one, stream=cap):
            for k in range(2):
                evs[2 * k].record(cap)
                ckpts = fwd(k)
                evs[2 * k + 1].record(cap)
                bwd(k, *ckpts)
            evs[4].record(cap)
            evs[5].record(cap)  # an empty interval: what one event node itself adds
        for _ in range(3):
            g_one.replay()
        torch.cuda.synchronize()
        f_list, b_list, o_list = [], [], []
        for _ in range(max(1, steps // 2)):
            g_one.replay()
            torch.cuda.synchronize()
            f_list += [evs[0].elapsed_time(evs[1]), evs[2].elapsed_time(evs[3])]
            b_list += [evs[1].elapsed_time(evs[2]), evs[3].elapsed_time(evs[4])]
            o_list.append(evs[4].elapsed_time(evs[5]))
        del g_one
        in_fwd, in_bwd = statistics.mean(f_list), statistics.mean(b_list)
        in_over = statistics.mean(o_list)
    except RuntimeError as exc:  # event nodes in a graph not supported: keep the two-graph times
        print(f"in-graph kernel events unavailable: {exc}", file=sys.stderr)
    in_fwd = max_over_ranks(in_fwd, world)
    in_bwd = max_over_ranks(in_bwd, world)
    in_over = max_over_ranks(in_over, world)
    out = {"ms_per_step": round(total, 4), "fwd_launch_ms": round(fwd_ms, 4),
           "bwd_launch_ms": round(bwd_ms, 4),
           "note": "the step's forward and backward scan kernels, each captured once in a "
                   "CUDA graph and replayed (same kernels, same parameters); diagnostic, not "
                   "the headline"}
    if in_fwd > 0 and in_bwd > 0:
        out["in_graph"] = {"fwd_launch_ms": round(in_fwd, 4), "bwd_launch_ms": round(in_bwd, 4),
                           "empty_interval_ms": round(in_over, 4),
                           "note": "both kernels in one graph, CUDA events recorded as graph "
                                   "nodes before, between and after them (max over ranks); "
                                   "each interval includes what an event node adds (the "
                                   "empty interval), not subtracted"}
    return out


PEER_GBS = 770.0  # measured NVLink peer-copy bandwidth per direction on this pool's B200s


def collective_leg(world: int, rank: int, local: int, steps: int, warmup: int) -> dict:
    """BASELINE config 4's packed reductions on ``world`` ranks, with a parity check.

    Spikes: Bernoulli(0.05) bool [T=128, B=1024, N=8192], the batch split over
    the ranks (rank r holds rows r*B/w .. (r+1)*B/w, seeded 77 + r). A step
    packs this rank's shard into int32 words, counts spikes per neuron over T
    and the local batch, all-gathers every rank's words and all-reduces the
    counts (src/myelin/distributed.py:63-109). Timed two ways on the same
    shards: ``fused`` (PackedSpikeExchange: one kernel packs, counts and
    stores every word into each rank's gather buffer over NVLink, then an
    int32 NCCL all-reduce) and ``nccl`` (pack + count kernel, NCCL
    all_gather_into_tensor, NCCL all-reduce). CUDA events on the launching
    stream, max over ranks.

    Parity (bit-exact, checked inside this run after each timing): every rank
    regenerates every rank's seeded shard, packs it with ``pack_spikes`` and
    compares the words with that rank's slot of the gathered buffer, and
    compares the all-reduced counts with the per-neuron sum of all shards'
    spikes (torch, int64). A MIN all-reduce of the per-rank results gives one
    verdict for the job.
    """

    import torch.distributed as dist

    import myelin_b200 as mb

    T, B_TOTAL, N = 128, 1024, 8192
    B = B_TOTAL // world
    stream = torch.cuda.current_stream()

    def shard(r: int) -> torch.Tensor:
        gen = torch.Generator(device="cuda").manual_seed(77 + r)
        return torch.rand((T, B, N), generator=gen, device="cuda") < 0.05

    spikes = shard(rank)
    exchange = mb.PackedSpikeExchange((T, B, N))
    gather_buf = torch.empty((world, T, B, N // 32), dtype=torch.int32, device="cuda")

    def fused_step():
        return exchange.pack_count_all_gather(spikes, count_dtype=torch.int32)

    def nccl_step():
        packed, counts = mb.pack_spikes_with_counts(spikes, dtype=torch.int32)
        mb.packed_spike_all_gather_into_tensor(packed, out=gather_buf)
        dist.all_reduce(counts, op=dist.ReduceOp.SUM)
        return gather_buf, counts

    def timed(step_fn):
        for _ in range(warmup):
            step_fn()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            out = step_fn()
        stop.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        return max_over_ranks(start.elapsed_time(stop), world) / steps, out

    def parity(gathered: torch.Tensor, counts: torch.Tensor) -> bool:
        ok = tuple(gathered.shape) == (world, T, B, N // 32)
        want_counts = torch.zeros(N, dtype=torch.int64, device="cuda")
        for r in range(world):
            s = shard(r)
            ok = ok and torch.equal(mb.pack_spikes(s).data, gathered[r])
            want_counts += s.sum(dim=(0, 1))
            del s
        ok = ok and torch.equal(counts.to(torch.int64), want_counts)
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        return bool(flag.item())

    words_bytes = T * B_TOTAL * (N // 32) * 4
    received = words_bytes * (world - 1) / world  # per rank, whatever the path
    bound_ms = received / (PEER_GBS * 1e9) * 1e3
    units = T * B_TOTAL * N
    out = {"workload": "pack_count (BASELINE config 4: Bernoulli(0.05) bool [128, 1024, 8192], "
                       f"batch sharded over {world} ranks: [128, {B}, 8192] per rank)",
           "spikes_per_step": units, "words_bytes_per_step": words_bytes,
           "received_bytes_per_rank": int(received),
           "receive_bound_ms": round(bound_ms, 4),
           "receive_bound_note": f"(w-1)/w of the packed words reach every rank over NVLink; "
                                 f"{PEER_GBS:.0f} GB/s measured peer bandwidth per direction"}
    for name, step_fn in (("fused", fused_step), ("nccl", nccl_step)):
        ms, (gathered, counts) = timed(step_fn)
        out[name] = {
            "ms_per_step": round(ms, 4),
            "spikes_per_s": units / (ms / 1e3),
            "allgather_busbw_gbs": round(received / (ms / 1e3) / 1e9, 1),
            "vs_receive_bound": round(ms / bound_ms, 3),
            "parity_ok": parity(gathered, counts),
        }
    out["parity_ok"] = out["fused"]["parity_ok"] and out["nccl"]["parity_ok"]
    out["limit"] = ("the all-gather's receive side: every rank takes in "
                    f"{received / 1e6:.0f} MB of other ranks' words per step while its own "
                    f"packing work shrinks as 1/w; fused step = "
                    f"{out['fused']['vs_receive_bound']}x the receive bound")
    exchange.close()
    return out


def build_network(name: str, device: str, seed: int):
    """Config-2 / config-5 models with seeded Kaiming-uniform weights ([in, out] layout)."""

    import myelin_b200 as mb

    torch.manual_seed(seed)
    if name == "mlp_fp32":
        params = mb.LIFParams(tau_mem=20.0, threshold=1.0, reset=0.0)
        layers = [mb.LinearSurrogateLIF(784, 1024, params, surrogate=mb.fast_sigmoid_surrogate,
                                        surrogate_slope=25.0, stream_synapse=True),
                  mb.LinearSurrogateLIF(1024, 10, params, surrogate=mb.fast_sigmoid_surrogate,
                                        surrogate_slope=25.0, stream_synapse=True)]
        dtype = torch.float32
    else:
        params = mb.LIFParams(tau_mem=20.0, threshold=1.0, reset=0.0)
        layers = [mb.LinearSurrogateLIF(f, 4096, params, surrogate=mb.superspike_surrogate,
                                        surrogate_slope=10.0, stream_synapse=True)
                  for f in (2048, 4096, 4096, 4096)]
        layers.append(mb.LinearSurrogateLIFRate(4096, 10, params, surrogate=mb.superspike_surrogate,
                                                surrogate_slope=10.0, reduction="none"))
        dtype = torch.bfloat16
    model = torch.nn.Sequential(*layers)
    for layer in layers:
        w = torch.empty(layer.synapse.weight.shape[::-1])
        torch.nn.init.kaiming_uniform_(w, a=5 ** 0.5)
        fan_in = w.shape[1]
        with torch.no_grad():
            layer.synapse.weight.copy_(w.t())
            layer.synapse.bias.uniform_(-1 / fan_in ** 0.5, 1 / fan_in ** 0.5)
    return model.to(device=device, dtype=dtype), dtype


def run_network(args, world, rank, local) -> None:
    """One training step of config 2 (fp32 MLP) or config 5 (bf16 rate network)."""

    from myelin_b200 import _native as nat

    name = args.workload
    model, dtype = build_network(name, "cuda", 0)
    gen = torch.Generator(device="cuda").manual_seed(100 + rank)
    if name == "mlp_fp32":
        T, B, F = 25, args.batch or 256, 784
        x = (torch.rand((T, B, F), generator=gen, device="cuda") < 0.2).to(dtype)
        labels = torch.randint(0, 10, (B,), generator=gen, device="cuda")

        def loss_fn():
            counts = model(x).sum(dim=0)
            return torch.nn.functional.cross_entropy(counts, labels)

        neurons = 1024 + 10
    else:
        T, B, F = 100, args.batch or 512, 2048
        x = (torch.rand((T, B, F), generator=gen, device="cuda") < 0.1).to(dtype)
        target = torch.rand((B, 10), generator=gen, device="cuda").mul(0.3).to(dtype)

        def loss_fn():
            return torch.nn.functional.mse_loss(model(x).float(), target.float())

        neurons = 4 * 4096 + 10
    params = [p for p in model.parameters()]
    flat = torch.empty(sum(p.numel() for p in params), dtype=torch.float32, device="cuda")
    opt = torch.optim.SGD(params, lr=1e-3)

    def step():
        opt.zero_grad(set_to_none=True)
        loss = loss_fn()
        loss.backward()
        if world > 1:
            import torch.distributed as dist

            torch.cat([p.grad.reshape(-1).float() for p in params], out=flat)
            dist.all_reduce(flat, op=dist.ReduceOp.SUM)
            flat.div_(world)
            offset = 0
            for p in params:
                n = p.numel()
                p.grad.copy_(flat[offset:offset + n].view_as(p))
                offset += n
        opt.step()
        return loss

    # On one GPU the whole training step (forward, backward, SGD update) is
    # captured once in a CUDA graph and replayed: the same kernels on the same
    # buffers every step, without the per-launch host latency of a step made of
    # many short kernels. With several ranks the step stays eager (its NCCL
    # all-reduce is issued from the host each step).
    graph = None
    if world == 1:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(args.warmup):
                step()
        torch.cuda.current_stream().wait_stream(side)
        opt.zero_grad(set_to_none=True)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_loss = step()
        for _ in range(args.warmup):
            graph.replay()
    else:
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            if graph is not None:
                graph.replay()
                loss = static_loss
            else:
                loss = step()
        stop.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(start.elapsed_time(stop), world) / args.steps
    units = T * B * neurons
    flops = 0
    for index, layer in enumerate(model):
        fi, fo = layer.synapse.weight.shape
        # forward projection and weight gradient; the input gradient except for
        # the first layer, whose input (the data) needs none
        flops += 2 * T * B * fi * fo * (3 if index > 0 else 2)
    result = {
        "metric": "LIF/ALIF fwd+bwd neuron-timesteps/s (training step)",
        "value": units * world / (ms / 1e3), "unit": "neuron-steps/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if name == "mlp_fp32" else "bf16", "data": "synthetic Bernoulli spikes",
        "config": {"workload": name + (" (BASELINE config 2)" if name == "mlp_fp32" else
                                       " (BASELINE config 5)"),
                   "T": T, "B_per_gpu": B, "global_batch": B * world, "F": F,
                   "parallelism": f"dp{world} (gradient all-reduce, NCCL)" if world > 1 else "dp1",
                   "cuda_graph": graph is not None},
        "tflops_per_gpu": round(flops / (ms / 1e3) / 1e12, 1),
        "loss": float(loss.item()),
        "device_status": nat.device_status(clear=True),
    }
    clk = clocks.summary()
    if clk is not None:
        result["clocks"] = clk
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_izhikevich(args, world, rank, local) -> None:
    """Izhikevich fused-time forward (forward only, like the reference's
    generated kernel) at the north-star shape T=256, B=128, N=4096, fp32,
    currents ~ N(9, 5), regular-spiking defaults, v0 = -65, u0 = 0.2 v0."""

    import myelin_b200 as mb
    from myelin_b200 import _native as nat

    gen = torch.Generator(device="cuda").manual_seed(31 + rank)
    x = torch.randn((T_STEPS, BATCH, NEURONS), generator=gen, device="cuda") * 5.0 + 9.0
    v0 = torch.full((BATCH, NEURONS), -65.0, device="cuda")
    state0 = mb.IzhikevichState(v0, 0.2 * v0)
    params = mb.IzhikevichParams()
    stream = torch.cuda.current_stream()
    # warm up exactly like the timed loop: the previous output stays alive while
    # the next is allocated, so both blocks are cached before timing starts
    for _ in range(args.warmup):
        _, spikes = mb.izhikevich_forward(x, state0, params)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            _, spikes = mb.izhikevich_forward(x, state0, params)
        stop.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(start.elapsed_time(stop), world) / args.steps
    units = T_STEPS * BATCH * NEURONS
    algo = units * 8  # read x (4 B) + write spikes (4 B) per neuron-step
    peak, peak_kind = load_peak_hbm()
    achieved = algo / (ms / 1e3) / 1e9
    result = {
        "metric": "Izhikevich forward neuron-timesteps/s", "value": units * world / (ms / 1e3),
        "unit": "neuron-steps/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic currents ~ N(9, 5)",
        "config": {"workload": "izhikevich_fp32 (north-star shape, forward only)", "T": T_STEPS,
                   "B_per_gpu": BATCH, "N": NEURONS,
                   "l2": "x and spikes are 537 MB each (larger than L2), no flush"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": profile_traffic("scan_fwd_izhikevich_fp32")},
        "spike_rate": float(spikes.mean()),
        "gpu_launches": args.steps, "device_status": nat.device_status(clear=True),
    }
    clk = clocks.summary()
    if clk is not None:
        result["clocks"] = clk
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_lif_packed(args, world, rank, local) -> None:
    """LIF forward with packed spike output at the north-star shape (T=256,
    B=128 per GPU, N=4096, fp32, x ~ N(0.3, 0.5)), followed at N > 1 by the
    packed all-gather of every rank's words: the forward-only communication
    path of the packed modules. ``--allgather fused`` writes the words into
    this rank's slot of a peer-mapped gather buffer and a push kernel stores
    the slot into every peer's (``PackedSpikeExchange.lif_forward_packed_spikes``); ``nccl``
    runs ``lif_forward_packed_spikes`` then ``all_gather_into_tensor``."""

    import myelin_b200 as mb
    from myelin_b200 import _native as nat

    T, B, N = T_STEPS, BATCH, NEURONS
    gen = torch.Generator(device="cuda").manual_seed(41 + rank)
    x = torch.randn((T, B, N), generator=gen, device="cuda") * 0.5 + 0.3
    state0 = mb.LIFState(torch.zeros((B, N), device="cuda"))
    params = mb.LIFParams(tau_mem=10.0)
    stream = torch.cuda.current_stream()
    fused = world > 1 and args.allgather == "fused"
    exchange = mb.PackedSpikeExchange((T, B, N)) if fused else None
    gather_buf = torch.empty((world, T, B, N // 32), dtype=torch.int32, device="cuda")

    def step():
        if fused:
            return exchange.lif_forward_packed_spikes(x, state0, params)[1]
        _, packed = mb.lif_forward_packed_spikes(x, state0, params)
        if world > 1:
            mb.packed_spike_all_gather_into_tensor(packed, out=gather_buf)
        return packed.data

    for _ in range(args.warmup):
        words = step()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            words = step()
        stop.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(start.elapsed_time(stop), world) / args.steps
    units = T * B * N
    algo = units * (4 + 0.125)  # read x (4 B) + write packed words (1/8 B) per neuron-step
    peak, peak_kind = load_peak_hbm()
    achieved = algo / (ms / 1e3) / 1e9
    result = {
        "metric": "LIF packed forward neuron-timesteps/s (+ packed all-gather at N > 1)",
        "value": units * world / (ms / 1e3), "unit": "neuron-steps/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic currents ~ N(0.3, 0.5)",
        "config": {"workload": "lif_packed (north-star shape, forward only)", "T": T,
                   "B_per_gpu": B, "N": N,
                   "allgather": ("peer-mapped slot + push kernel over NVLink" if fused else
                                 "NCCL all_gather_into_tensor" if world > 1 else None),
                   "l2": "x is 537 MB (larger than L2), no flush"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": profile_traffic("scan_fwd_lif_packed_fp32") if world == 1 else None,
                     "note": "scan bytes over the whole step (all-gather included at N > 1)"},
        "words_checksum": int(words.sum().item()),
        "gpu_launches": args.steps, "device_status": nat.device_status(clear=True),
    }
    clk = clocks.summary()
    if clk is not None:
        result["clocks"] = clk
    if exchange is not None:
        exchange.close()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_pack_count(args, world, rank, local) -> None:
    """Bernoulli(0.05) spikes [128, 1024, 8192], batch sharded over ranks.

    A step packs this rank's [128, 1024/world, 8192] spikes into int32 words,
    counts spikes per neuron (int32, summed over T and the local batch), then
    all-gathers the packed words and all-reduces the counts (NCCL over NVLink).
    """

    import myelin_b200 as mb
    from myelin_b200 import _native as nat

    T, B, N = 128, 1024 // world, 8192
    gen = torch.Generator(device="cuda").manual_seed(77 + rank)
    spikes = torch.rand((T, B, N), generator=gen, device="cuda") < 0.05
    stream = torch.cuda.current_stream()
    gather_buf = torch.empty((world, T, B, N // 32), dtype=torch.int32, device="cuda")
    fused = world > 1 and args.allgather == "fused"
    exchange = mb.PackedSpikeExchange((T, B, N)) if fused else None
    if world > 1:
        import torch.distributed as dist

    def step():
        if fused:
            # one kernel packs, counts and stores the words into every rank's
            # gather buffer over NVLink; the count all-reduce completes the step
            _, counts = exchange.pack_count_all_gather(spikes, count_dtype=torch.int32)
            return counts
        packed, counts = mb.pack_spikes_with_counts(spikes, dtype=torch.int32)
        if world > 1:
            mb.packed_spike_all_gather_into_tensor(packed, out=gather_buf)
            dist.all_reduce(counts, op=dist.ReduceOp.SUM)
        return counts

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            counts = step()
        stop.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(start.elapsed_time(stop), world) / args.steps
    total = int(counts.sum().item())
    units = T * B * N
    peak, peak_kind = load_peak_hbm()
    # one pass: read 1 B bool + write 1/8 B of words per spike (per-neuron
    # partial counts: a few MB per step, not counted)
    algo = units * (1 + 0.125)
    words_bytes = units // 8
    result = {
        "metric": "spikes/s (pack + per-neuron count + packed all-gather + count all-reduce)",
        "value": units * world / (ms / 1e3), "unit": "spikes/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic Bernoulli(0.05)",
        "config": {"workload": "pack_count (BASELINE config 4)", "T": T, "B_total": B * world,
                   "B_per_gpu": B, "N": N, "parallelism": f"dp{world} (batch-sharded)",
                   "allgather": ("fused pack + peer stores over NVLink" if fused else
                                 "NCCL all_gather_into_tensor" if world > 1 else None)},
        "allgather_busbw_gbs": (round(words_bytes * world * (world - 1) / world / (ms / 1e3) / 1e9, 1)
                                if world > 1 else None),
        "roofline": {"bound": "hbm", "achieved": round(algo / (ms / 1e3) / 1e9, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(algo / (ms / 1e3) / 1e9 / peak, 4),
                     "peak_kind": peak_kind,
                     "traffic": profile_traffic("pack_count_rows_config4") if world == 1 else None,
                     "note": "fused pack+count bytes over the whole step (collectives included)"},
        "spike_count_check": total,
        # one packing kernel per step (the totals are zeroed by a memset)
        "gpu_launches": args.steps, "device_status": nat.device_status(clear=True),
    }
    clk = clocks.summary()
    if clk is not None:
        result["clocks"] = clk
    if exchange is not None:
        exchange.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


# ---------------------------------------------------------------------------
# CPU arms: myelin's torch CPU path (restated in oracle/torch_path.py) and the
# C restatement of the same scan (oracle/scan_oracle.c), on the host's cores
# ---------------------------------------------------------------------------
C_PORT_ROWS = 32  # C-port sample: 32 of 128 rows, 134 MB per fp32 array (beyond the host LLC)


def _oracle_sample(name: str, rows: int, threads: int):
    from oracle import oracle

    rng = np.random.default_rng(99)
    shape = (T_STEPS, rows, NEURONS)
    if name == "alif_bf16":
        x = torch.from_numpy(rng.normal(0.2, 0.6, shape).astype(np.float32)).to(torch.bfloat16)
        x = x.float().numpy()
        gs = torch.from_numpy(rng.normal(0, 1, shape).astype(np.float32)).to(torch.bfloat16)
        gs = gs.float().numpy()
        kw = dict(neuron=oracle.ALIF, reset_mode=oracle.SUBTRACT, decay=np.float32(0.9),
                  threshold=np.float32(1.0), reset=np.float32(0.0),
                  adapt_decay=np.float32(1 - 1 / 50), beta=np.float32(1.8))
    else:
        x = rng.normal(0.3, 0.5, shape).astype(np.float32)
        gs = rng.normal(0, 1, shape).astype(np.float32)
        kw = dict(neuron=oracle.LIF, decay=np.float32(0.9), threshold=np.float32(1.0),
                  reset=np.float32(0.0))
    z = np.zeros((rows, NEURONS), np.float32)

    def step():
        oracle.scan_forward(x, z, z, threads=threads, **kw)
        oracle.scan_backward(x, z, z, grad_spikes=gs, surrogate="atan", slope=10.0,
                             threads=threads, **kw)

    return step, T_STEPS * rows * NEURONS


def _timed_steps(step, *, warmup: int, steps: int | None = None, seconds: float = 10.0,
                 min_steps: int = 3) -> list[float]:
    """Per-step wall times (perf_counter), after ``warmup`` untimed steps: exactly
    ``steps`` if given, else until ``seconds`` have passed (at least ``min_steps``).
    Both CPU arms use this one method, so their figures are comparable."""

    for _ in range(warmup):
        step()
    times: list[float] = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if steps is not None and len(times) >= steps:
            break
        if steps is None and len(times) >= min_steps and time.perf_counter() - t_start >= seconds:
            break
    return times


def c_port_figure(name: str, *, threads: int, warmup: int = 2, steps: int | None = None,
                  seconds: float = 5.0) -> dict:
    step, units = _oracle_sample(name, C_PORT_ROWS, threads)
    times = _timed_steps(step, warmup=warmup, steps=steps, seconds=seconds)
    med = statistics.median(times)
    return {"value": units / med, "unit": "neuron-steps/s", "cores": threads, "kind": "port",
            "sample": f"{name}: T={T_STEPS}, B={C_PORT_ROWS} of {BATCH}, N={NEURONS} "
                      f"(134 MB per fp32 array, beyond the host's last-level cache); median of "
                      f"{len(times)} fwd+bwd passes of the C restatement (OpenMP, {threads} "
                      "threads)"}


def torch_path_figure(*, threads: int, warmup: int = 1, steps: int | None = None,
                      seconds: float = 10.0) -> dict:
    from oracle import torch_path

    r = torch_path.time_config3(threads=threads, warmup=warmup, steps=steps, seconds=seconds,
                                min_steps=2)
    med = statistics.median(r["times"])
    T, B, N = r["shape"]
    return {"value": r["units"] / med, "unit": "neuron-steps/s", "cores": r["threads"],
            "kind": "port",
            "sample": f"myelin's torch CPU path (surrogate_alif_unroll + autograd, restated in "
                      f"torch): the full config-3 step T={T}, B={B}, N={N}, {r['dtype']}, "
                      f"median of {len(r['times'])} fwd+bwd steps, torch on {r['threads']} "
                      "host threads"}


def cpu_baseline(name: str, seconds: float = 10.0) -> dict:
    threads = len(os.sched_getaffinity(0))
    if name == "alif_bf16":
        base = torch_path_figure(threads=threads, seconds=seconds)
        base["c_port"] = c_port_figure(name, threads=threads, seconds=seconds / 2)
        return base
    return c_port_figure(name, threads=threads, seconds=seconds)


def run_reference(args) -> None:
    """The reference arm: myelin's own CPU implementation of the path (its
    torch per-timestep loop + autograd, restated in oracle/torch_path.py; the
    reference tree does not travel to the GPU box) on all of the host's
    cores, at the GPU arm's config. Under torchrun rank 0 alone runs it (with
    every host thread, whatever OMP_NUM_THREADS torchrun set) and the value
    is whole-host throughput, comparable to the GPU arm's whole-job value."""

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = len(os.sched_getaffinity(0))
    name = args.workload if args.workload in ("alif_bf16", "lif_fp32") else "alif_bf16"
    if name == "alif_bf16":
        fig = torch_path_figure(threads=threads, warmup=min(args.warmup, 3), steps=args.steps)
        fig["c_port"] = c_port_figure(name, threads=threads, seconds=5.0)
    else:
        fig = c_port_figure(name, threads=threads, warmup=args.warmup, steps=args.steps)
    value = fig["value"]
    ms = (T_STEPS * BATCH * NEURONS if name == "alif_bf16" else T_STEPS * C_PORT_ROWS * NEURONS) \
        / value * 1e3
    result = {
        "impl": "reference",
        "metric": "LIF/ALIF fwd+bwd neuron-timesteps/s", "value": value, "unit": "neuron-steps/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if name == "alif_bf16" else "f32", "data": "synthetic",
        "config": {"workload": name, "T": T_STEPS, "B_per_gpu": BATCH, "N": NEURONS,
                   "host_threads": threads},
        "cpu_baseline": fig,
        "e2e": {"value": value, "unit": "neuron-steps/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(result), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__,
                                     formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=50)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("mine", "reference"), default="mine")
    parser.add_argument("--workload",
                        choices=("alif_bf16", "lif_fp32", "pack_count", "mlp_fp32", "rate_net",
                                 "izhikevich_fp32", "lif_packed"),
                        default="alif_bf16")
    parser.add_argument("--cpu-seconds", type=float, default=10.0)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--allgather", choices=("fused", "nccl"), default="fused",
                        help="pack_count / lif_packed at N > 1: the peer-mapped exchange "
                             "(PackedSpikeExchange), or NCCL all_gather_into_tensor")
    parser.add_argument("--batch", type=int, default=None,
                        help="per-GPU batch of the network workloads (default: the BASELINE "
                             "config's); smaller values are for profiling captures")
    args = parser.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    sys.path.insert(0, str(ROOT))
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
