"""TEST INFRASTRUCTURE ONLY: CPU oracle for myelin_b200 parity tests and the CPU baseline.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs use this module, as the checker or the timed CPU reference; the product
(``myelin_b200``) never imports it.

- Scan forward/backward: ``scan_oracle.c`` (plain C, float32, no FMA,
  OpenMP over neurons), a restatement of the reference's LIF/ALIF scan and
  adjoint; see that file's header for the reference lines it follows.
- Packing and counts: numpy restatement of src/myelin/packing.py:45-216
  (LSB-first int32 words, zero padding, nonzero = spike).
- Linear stream-synapse path: numpy restatement of
  src/myelin/autograd.py:445-556 (currents = x_t @ W + b, scan from a zero
  membrane, dX = G W^T, dW = sum_t x_t^T G_t, db = sum G).

Pinned against golden vectors generated from the reference itself
(``tests/golden/make_golden.py``), checked by ``tests/test_oracle_golden.py``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
SOURCE = ORACLE_DIR / "scan_oracle.c"
BUILD_DIR = ORACLE_DIR / "_build"
LIB = BUILD_DIR / "liboracle_scan.so"
CFLAGS = ["-O3", "-march=x86-64-v2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp",
          "-fPIC", "-shared", "-std=c11"]

LIF, ALIF = 0, 1
HARD, SUBTRACT = 0, 1
SURROGATES = ("sigmoid", "fast_sigmoid", "atan", "triangular", "superspike", "multi_gaussian")
SURR_NONE = 6

_lib = None
_lock = threading.Lock()


def build(force: bool = False) -> Path:
    """Compile ``scan_oracle.c`` with gcc into ``oracle/_build/liboracle_scan.so``."""

    BUILD_DIR.mkdir(exist_ok=True)
    if force or not LIB.exists() or LIB.stat().st_mtime < SOURCE.stat().st_mtime:
        tmp = LIB.with_suffix(f".{os.getpid()}.tmp")
        subprocess.run(["gcc", *CFLAGS, str(SOURCE), "-o", str(tmp), "-lm"], check=True)
        tmp.replace(LIB)
    return LIB


def _load():
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                lib = ctypes.CDLL(str(build()))
                vp, i64, i32, f = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
                lib.oracle_scan_forward.restype = None
                lib.oracle_scan_forward.argtypes = [
                    i32, i32, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, f, f, f, f, f, i32]
                lib.oracle_scan_backward.restype = None
                lib.oracle_scan_backward.argtypes = [
                    i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64,
                    f, f, f, f, f, f, i64, i32]
                lib.oracle_num_threads.restype = i32
                _lib = lib
    return _lib


def num_threads() -> int:
    return int(_load().oracle_num_threads())


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def _p(a):
    return None if a is None else a.ctypes.data


def scan_forward(x, v0, a0=None, *, neuron=LIF, reset_mode=HARD, decay, threshold, reset,
                 adapt_decay=0.0, beta=0.0, threads=0):
    """Returns dict(spikes=uint8 [T,B,N], vT, aT, counts int64 [B,N])."""

    x = _f32(x)
    v0 = _f32(v0)
    a0 = _f32(a0) if neuron == ALIF else None
    T, B, N = x.shape
    vT = np.empty((B, N), np.float32)
    aT = np.empty((B, N), np.float32) if neuron == ALIF else None
    spikes = np.empty((T, B, N), np.uint8)
    counts = np.empty((B, N), np.int64)
    _load().oracle_scan_forward(neuron, reset_mode, _p(x), _p(v0), _p(a0), _p(vT), _p(aT),
                                _p(spikes), _p(counts), T, B, N, decay, threshold, reset,
                                adapt_decay, beta, threads)
    return {"spikes": spikes, "vT": vT, "aT": aT, "counts": counts}


def scan_backward(x, v0, a0=None, *, grad_spikes=None, grad_rates=None, grad_vT=None,
                  grad_aT=None, neuron=LIF, reset_mode=HARD, surrogate=2, slope=10.0, decay,
                  threshold, reset, adapt_decay=0.0, beta=0.0, chunk=16, threads=0):
    """Returns dict(grad_x [T,B,N], grad_v0 [B,N], grad_a0 [B,N] | None)."""

    x = _f32(x)
    v0 = _f32(v0)
    a0 = _f32(a0) if neuron == ALIF else None
    T, B, N = x.shape
    gx = np.empty((T, B, N), np.float32)
    gv0 = np.empty((B, N), np.float32)
    ga0 = np.empty((B, N), np.float32) if neuron == ALIF else None
    sid = SURROGATES.index(surrogate) if isinstance(surrogate, str) else int(surrogate)
    _load().oracle_scan_backward(
        neuron, reset_mode, sid, _p(x), _p(v0), _p(a0), _p(_f32(grad_spikes)),
        _p(_f32(grad_rates)), _p(_f32(grad_vT)), _p(_f32(grad_aT)), _p(gx), _p(gv0), _p(ga0),
        T, B, N, decay, threshold, reset, adapt_decay, beta, slope, chunk, threads)
    return {"grad_x": gx, "grad_v0": gv0, "grad_a0": ga0}


# ---------------------------------------------------------------------------
# Packing (numpy), src/myelin/packing.py:45-216
# ---------------------------------------------------------------------------

def pack(spikes: np.ndarray) -> np.ndarray:
    """Nonzero -> bit, LSB-first int32 words along the last axis, zero padding."""

    spikes = np.asarray(spikes)
    n = spikes.shape[-1]
    words = (n + 31) // 32
    nz = spikes != 0
    padded = np.zeros((*spikes.shape[:-1], words * 32), dtype=bool)
    padded[..., :n] = nz
    bytes_ = np.packbits(padded.reshape(*spikes.shape[:-1], words, 32), axis=-1, bitorder="little")
    return np.ascontiguousarray(bytes_).view("<u4").reshape(*spikes.shape[:-1], words).view(np.int32)


def unpack(words: np.ndarray, n: int) -> np.ndarray:
    """Bits back to 0/1 uint8 of length ``n`` along the last axis."""

    words = np.ascontiguousarray(words, dtype=np.int32)
    bytes_ = words.view(np.uint8).reshape(*words.shape, 4)
    bits = np.unpackbits(bytes_, axis=-1, bitorder="little").reshape(*words.shape[:-1], -1)
    return bits[..., :n]


def count_rows(words: np.ndarray, n: int) -> np.ndarray:
    return unpack(words, n).sum(axis=-1, dtype=np.int64)


def count_columns(words: np.ndarray, n: int) -> np.ndarray:
    bits = unpack(words, n)
    return bits.reshape(-1, n).sum(axis=0, dtype=np.int64)


# ---------------------------------------------------------------------------
# Linear stream-synapse path (numpy + C scan), src/myelin/autograd.py:445-556
# ---------------------------------------------------------------------------

def linear_currents(x, w, b=None):
    T, B, F = x.shape
    cur = (np.asarray(x, np.float32).reshape(T * B, F) @ np.asarray(w, np.float32))
    if b is not None:
        cur = cur + np.asarray(b, np.float32)
    return cur.reshape(T, B, -1).astype(np.float32)


def linear_backward(x, w, grad_currents):
    """dX, dW, db from dL/dcurrents (float64 accumulation, returned as float32)."""

    T, B, F = x.shape
    g = np.asarray(grad_currents, np.float64).reshape(T * B, -1)
    x2 = np.asarray(x, np.float64).reshape(T * B, F)
    dx = (g @ np.asarray(w, np.float64).T).reshape(T, B, F)
    dw = x2.T @ g
    db = g.sum(axis=0)
    return dx.astype(np.float32), dw.astype(np.float32), db.astype(np.float32)


IZHIKEVICH_FIELDS = ("recovery_decay", "recovery_coupling", "reset_voltage", "recovery_jump",
                     "threshold", "dt", "voltage_square_coeff", "voltage_coeff", "voltage_bias")


def izhikevich_forward(x, v0, u0, params: dict):
    """Izhikevich forward, restated from src/myelin/neurons.py:131-156 /
    functional.py:81-112 in float32 with one rounding per operation, in the
    reference's evaluation order (Python scalars rounded to float32 first):

        dv  = ((c2 * v) * v + c1 * v) + bias - u + I
        p_v = v + dt * dv
        p_u = u + dt * (a * (b * v - u))
        s   = p_v >= threshold
        v'  = s ? reset_voltage : p_v;   u' = s ? p_u + jump : p_u

    Returns (spikes [T,B,N] 0/1 float32, vT, uT).
    """

    f = np.float32
    x = _f32(x)
    v = _f32(v0).copy()
    u = _f32(u0).copy()
    a, b, rv, jump, thr, dt, c2, c1, bias = (f(params[k]) for k in IZHIKEVICH_FIELDS)
    spikes = np.empty_like(x)
    with np.errstate(over="ignore", invalid="ignore"):
        for t in range(x.shape[0]):
            dv = (c2 * v) * v
            dv = dv + c1 * v
            dv = dv + bias
            dv = dv - u
            dv = dv + x[t]
            pv = v + dt * dv
            pu = u + dt * (a * (b * v - u))
            s = pv >= thr
            spikes[t] = s
            v = np.where(s, rv, pv).astype(np.float32)
            u = np.where(s, pu + jump, pu).astype(np.float32)
    return spikes, v, u
