"""ctypes binding of the myelin_b200 C ABI (``include/myelin_b200.h``).

This module is the only place that talks to ``libmyelin_b200.so``. It loads
the in-tree library (built by ``python -m myelin_b200.build``), declares the
C signatures, and offers thin helpers that pass torch tensors as raw device
pointers on the current CUDA stream. There is no fallback: if the library is
missing, or a tensor is not on a CUDA device, the call raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libmyelin_b200.so"

# enum mb_dtype
MB_F32, MB_BF16, MB_F16, MB_F64, MB_U8, MB_I16, MB_I32, MB_I64 = range(8)
# enum mb_neuron / mb_reset
MB_LIF, MB_ALIF = 0, 1
MB_RESET_HARD, MB_RESET_SUBTRACT = 0, 1
MB_SURR_NONE = 6
SCAN_CHUNK = 16  # MB_SCAN_CHUNK

_DTYPE_CODES: dict[torch.dtype, int] = {
    torch.float32: MB_F32,
    torch.bfloat16: MB_BF16,
    torch.float16: MB_F16,
    torch.float64: MB_F64,
    torch.bool: MB_U8,
    torch.uint8: MB_U8,
    torch.int8: MB_U8,
    torch.int16: MB_I16,
    torch.int32: MB_I32,
    torch.int64: MB_I64,
}
SCAN_DTYPES = (torch.float32, torch.bfloat16, torch.float16)

_lib: ctypes.CDLL | None = None
_lock = threading.Lock()

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f = ctypes.c_float

_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "mb_last_error": (ctypes.c_char_p, []),
    "mb_version": (ctypes.c_char_p, []),
    "mb_device_status": (_int, [_int]),
    "mb_debug_wait_timeout": (_int, [_int, _int, _vp]),
    "mb_scan_num_checkpoints": (_i64, [_i64]),
    "mb_scan_forward": (
        _int,
        [_int, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
         _i64, _i64, _i64, _f, _f, _f, _f, _f, _int, _vp],
    ),
    "mb_scan_backward": (
        _int,
        [_int, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
         _i64, _i64, _i64, _f, _f, _f, _f, _f, _int, _int, _f, _vp],
    ),
    "mb_scan_backward_sum": (
        _int,
        [_int, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
         _i64, _i64, _i64, _f, _f, _f, _f, _f, _int, _int, _f, _vp],
    ),
    "mb_gemm_tn": (
        _int, [_int, _vp, _i64, _vp, _i64, _vp, _int, _int, _vp, _i64, _i64, _i64, _i64, _vp]
    ),
    "mb_gemm": (
        _int, [_int, _vp, _int, _i64, _i64, _int, _vp, _vp, _int, _i64, _i64, _int, _vp, _vp,
               _int, _int, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _vp]
    ),
    "mb_gemm_workspace_bytes": (_i64, [_i64, _i64, _i64, _int, _int, _int]),
    "mb_split_bf16": (
        _int, [_int, _vp, _i64, _i64, _i64, _i64, _int, _vp, _i64, _i64, _i64, _i64, _vp, _vp]
    ),
    "mb_gemm_small_k": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp]),
    "mb_column_sums_workspace_bytes": (_i64, [_i64, _i64]),
    "mb_column_sums": (_int, [_int, _vp, _i64, _i64, _i64, _int, _vp, _vp, _i64, _vp]),
    "mb_pack_spikes": (_int, [_int, _vp, _vp, _i64, _i64, _vp]),
    "mb_unpack_spikes": (_int, [_vp, _int, _vp, _i64, _i64, _vp]),
    "mb_count_rows": (_int, [_vp, _i64, _i64, _vp, _vp]),
    "mb_count_columns_workspace_bytes": (_i64, [_i64, _i64]),
    "mb_count_columns": (_int, [_vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp]),
    "mb_count_columns_noalloc": (_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "mb_pack_count_workspace_bytes": (_i64, [_i64, _i64]),
    "mb_pack_count_spikes": (_int, [_int, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp]),
    "mb_izhikevich_forward": (
        _int, [_int, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp]
    ),
    "mb_scan_forward_packed_scatter": (
        _int, [_int, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _i64, _i64, _i64, _f, _f, _f,
               _f, _f, _int, _vp]
    ),
    "mb_pack_count_scatter": (
        _int, [_int, _vp, _vp, _i64, _i64, _vp, _int, _vp, _vp, _vp, _i64, _vp]
    ),
    "mb_ipc_handle_bytes": (_int, []),
    "mb_ipc_alloc": (_int, [_i64, _vp, _vp]),
    "mb_ipc_open": (_int, [_vp, _vp]),
    "mb_ipc_close": (_int, [_vp]),
    "mb_ipc_free": (_int, [_vp]),
}

EXPORTED_SYMBOLS = tuple(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it is not built."""

    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"myelin_b200 native library not found at {LIB_PATH}; build it with "
                    "`python -m myelin_b200.build` (nvcc, sm_100a)"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
    return _lib


def version() -> str:
    return lib().mb_version().decode()


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype for myelin_b200 kernels: {dtype}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def check(status: int, what: str) -> None:
    if status != 0:
        message = lib().mb_last_error().decode() or "unknown error"
        raise RuntimeError(f"{what} failed: {message}")


def require_cuda(tensor: torch.Tensor, what: str = "inputs") -> None:
    if not tensor.is_cuda:
        raise ValueError(
            f"myelin_b200 runs on CUDA devices only; {what} is on {tensor.device}. "
            "Move the tensors to a CUDA device (there is no CPU fallback)."
        )


def device_status(clear: bool = True) -> int:
    """Return (and by default clear) the device status of every kernel with
    bounded waits (scan forward/backward, both tensor-core GEMMs)."""

    return int(lib().mb_device_status(1 if clear else 0))


# enum mb_unit: the code units whose status words mb_device_status combines
MB_UNIT_SCAN, MB_UNIT_SCAN_FAST, MB_UNIT_GEMM = 0, 1, 2


def debug_wait_timeout(unit: int, polls: int = 256, device: torch.device | None = None) -> None:
    """Launch a kernel in ``unit`` whose one bounded wait is on a barrier that
    nothing arrives at: the wait runs out, the unit records status 1 and the
    kernel returns (diagnostic for tests of the timeout path)."""

    device = device or torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(device):
        status = lib().mb_debug_wait_timeout(unit, polls, stream_handle(device))
    check(status, "mb_debug_wait_timeout")


def scan_forward(
    *,
    neuron: int,
    x: torch.Tensor,
    v0: torch.Tensor,
    a0: torch.Tensor | None,
    vT: torch.Tensor | None,
    aT: torch.Tensor | None,
    spikes: torch.Tensor | None,
    packed: torch.Tensor | None,
    rates: torch.Tensor | None,
    ckpt_v: torch.Tensor | None,
    ckpt_a: torch.Tensor | None,
    decay: float,
    threshold: float,
    reset: float,
    adapt_decay: float,
    beta: float,
    reset_mode: int,
) -> None:
    T, B, N = x.shape
    with torch.cuda.device(x.device):
        status = lib().mb_scan_forward(
            neuron, dtype_code(x.dtype), ptr(x), ptr(v0), ptr(a0), ptr(vT), ptr(aT),
            ptr(spikes), ptr(packed), ptr(rates), ptr(ckpt_v), ptr(ckpt_a),
            T, B, N, decay, threshold, reset, adapt_decay, beta, reset_mode,
            stream_handle(x.device),
        )
    check(status, "mb_scan_forward")


def scan_backward(
    *,
    neuron: int,
    x: torch.Tensor,
    ckpt_v: torch.Tensor,
    ckpt_a: torch.Tensor | None,
    grad_spikes: torch.Tensor | None,
    grad_rates: torch.Tensor | None,
    grad_vT: torch.Tensor | None,
    grad_aT: torch.Tensor | None,
    grad_x: torch.Tensor,
    grad_v0: torch.Tensor | None,
    grad_a0: torch.Tensor | None,
    decay: float,
    threshold: float,
    reset: float,
    adapt_decay: float,
    beta: float,
    reset_mode: int,
    surrogate: int,
    slope: float,
    grad_sum: torch.Tensor | None = None,
) -> None:
    """Reverse scan; ``grad_sum`` (fp32 [B*N], optional) receives the sum over
    t of grad_x, last step first (``mb_scan_backward_sum``)."""

    T, B, N = x.shape
    with torch.cuda.device(x.device):
        if grad_sum is None:
            status = lib().mb_scan_backward(
                neuron, dtype_code(x.dtype), ptr(x), ptr(ckpt_v), ptr(ckpt_a),
                ptr(grad_spikes), ptr(grad_rates), ptr(grad_vT), ptr(grad_aT),
                ptr(grad_x), ptr(grad_v0), ptr(grad_a0),
                T, B, N, decay, threshold, reset, adapt_decay, beta, reset_mode,
                surrogate, slope, stream_handle(x.device),
            )
        else:
            status = lib().mb_scan_backward_sum(
                neuron, dtype_code(x.dtype), ptr(x), ptr(ckpt_v), ptr(ckpt_a),
                ptr(grad_spikes), ptr(grad_rates), ptr(grad_vT), ptr(grad_aT),
                ptr(grad_x), ptr(grad_v0), ptr(grad_a0), ptr(grad_sum),
                T, B, N, decay, threshold, reset, adapt_decay, beta, reset_mode,
                surrogate, slope, stream_handle(x.device),
            )
    check(status, "mb_scan_backward")


GEMM_DTYPES = (torch.bfloat16, torch.float16)


def gemm_tn_supported(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Whether mb_gemm_tn takes these operands (16-bit, 16-byte rows and bases)."""

    return (
        a.dtype in GEMM_DTYPES and b.dtype == a.dtype and a.dim() == 2 and b.dim() == 2
        and a.shape[1] == b.shape[1] and a.shape[1] % 8 == 0
        and a.stride(1) == 1 and b.stride(1) == 1
        and a.stride(0) % 8 == 0 and b.stride(0) % 8 == 0
        and a.data_ptr() % 16 == 0 and b.data_ptr() % 16 == 0
    )


def gemm_tn(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None,
            out: torch.Tensor) -> torch.Tensor:
    """out[M, N] = a[M, K] @ b[N, K]^T (+ bias) on the tcgen05 tensor cores."""

    M, K = a.shape
    N = b.shape[0]
    with torch.cuda.device(a.device):
        status = lib().mb_gemm_tn(
            dtype_code(a.dtype), ptr(a), a.stride(0), ptr(b), b.stride(0), ptr(bias),
            dtype_code(bias.dtype) if bias is not None else 0, dtype_code(out.dtype), ptr(out),
            out.stride(0), M, N, K, stream_handle(a.device),
        )
    check(status, "mb_gemm_tn")
    return out


MB_KMAJOR, MB_MNMAJOR = 0, 1  # enum mb_major


class GemmOperand:
    """One mb_gemm operand: ``parts`` matrices of 16-bit elements stored from
    ``tensor``'s first element, ``part_stride`` elements apart, each K-major
    (element (r, k) at r * ld + k) or MN-major (element (r, k) at k * ld + r).
    ``nonzero`` (int32 per part, from ``split_bf16``) lets the kernel skip
    all-zero parts."""

    def __init__(self, tensor: torch.Tensor, major: int, ld: int, *, parts: int = 1,
                 part_stride: int = 0, nonzero: torch.Tensor | None = None) -> None:
        self.tensor, self.major, self.ld = tensor, major, ld
        self.parts, self.part_stride, self.nonzero = parts, part_stride, nonzero


def gemm(a: GemmOperand, b: GemmOperand, M: int, N: int, K: int, out: torch.Tensor,
         bias: torch.Tensor | None = None) -> torch.Tensor:
    """out[M, N] = sum over kept part pairs of A_i[M, K] B_j[N, K]^T (+ bias) (``mb_gemm``)."""

    dev = a.tensor.device
    need = int(lib().mb_gemm_workspace_bytes(M, N, K, a.parts, b.parts, dtype_code(out.dtype)))
    ws = torch.empty(need // 4, dtype=torch.float32, device=dev) if need > 0 else None
    with torch.cuda.device(dev):
        status = lib().mb_gemm(
            dtype_code(a.tensor.dtype), ptr(a.tensor), a.major, a.ld, a.part_stride, a.parts,
            ptr(a.nonzero), ptr(b.tensor), b.major, b.ld, b.part_stride, b.parts,
            ptr(b.nonzero), ptr(bias), dtype_code(bias.dtype) if bias is not None else 0,
            dtype_code(out.dtype), ptr(out), out.stride(0), M, N, K, ptr(ws), need,
            stream_handle(dev),
        )
    check(status, "mb_gemm")
    return out


def split_bf16(src: torch.Tensor, rows: int, cols: int, row_stride: int, col_stride: int,
               parts: int, dst: torch.Tensor, dst_rows: int, dst_cols: int, dst_ld: int,
               dst_part_stride: int, nonzero: torch.Tensor | None = None) -> None:
    """``mb_split_bf16``: element (r, c) of ``src`` (at r * row_stride + c *
    col_stride from its first element) split into ``parts`` bf16 parts of
    ``dst`` (or copied, for a 16-bit source), zeros outside the source."""

    with torch.cuda.device(src.device):
        status = lib().mb_split_bf16(
            dtype_code(src.dtype), ptr(src), rows, cols, row_stride, col_stride, parts, ptr(dst),
            dst_rows, dst_cols, dst_ld, dst_part_stride, ptr(nonzero), stream_handle(src.device),
        )
    check(status, "mb_split_bf16")


def gemm_small_k(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out[M, N] = a[M, K] @ b[N, K]^T in fp32 FMAs, K <= 32 (``mb_gemm_small_k``)."""

    M, K = a.shape
    N = b.shape[0]
    with torch.cuda.device(a.device):
        status = lib().mb_gemm_small_k(ptr(a), a.stride(0), ptr(b), b.stride(0), ptr(out),
                                       out.stride(0), M, N, K, stream_handle(a.device))
    check(status, "mb_gemm_small_k")
    return out


def column_sums(src: torch.Tensor, rows: int, cols: int, ld: int, out: torch.Tensor) -> None:
    """out[c] = sum over r of src[r * ld + c] in a fixed order (``mb_column_sums``)."""

    need = int(lib().mb_column_sums_workspace_bytes(rows, cols))
    ws = torch.empty(max(need // 4, 1), dtype=torch.float32, device=src.device)
    with torch.cuda.device(src.device):
        status = lib().mb_column_sums(
            dtype_code(src.dtype), ptr(src), rows, cols, ld, dtype_code(out.dtype), ptr(out),
            ptr(ws), ws.numel() * 4, stream_handle(src.device),
        )
    check(status, "mb_column_sums")


def num_checkpoints(T: int) -> int:
    return int(lib().mb_scan_num_checkpoints(T))


def pack(spikes: torch.Tensor, words: torch.Tensor, rows: int, n: int) -> None:
    with torch.cuda.device(spikes.device):
        status = lib().mb_pack_spikes(
            dtype_code(spikes.dtype), ptr(spikes), ptr(words), rows, n,
            stream_handle(spikes.device),
        )
    check(status, "mb_pack_spikes")


def unpack(words: torch.Tensor, out: torch.Tensor, rows: int, n: int) -> None:
    with torch.cuda.device(words.device):
        status = lib().mb_unpack_spikes(
            ptr(words), dtype_code(out.dtype), ptr(out), rows, n, stream_handle(words.device)
        )
    check(status, "mb_unpack_spikes")


def count_rows(words: torch.Tensor, counts: torch.Tensor, rows: int, n: int) -> None:
    with torch.cuda.device(words.device):
        status = lib().mb_count_rows(ptr(words), rows, n, ptr(counts), stream_handle(words.device))
    check(status, "mb_count_rows")


def count_columns(
    words: torch.Tensor,
    rows: int,
    n: int,
    counts64: torch.Tensor | None,
    counts32: torch.Tensor | None,
) -> None:
    need = int(lib().mb_count_columns_workspace_bytes(rows, n))
    workspace = torch.empty(max(need, 4), dtype=torch.uint8, device=words.device)
    with torch.cuda.device(words.device):
        status = lib().mb_count_columns(
            ptr(words), rows, n, ptr(counts64), ptr(counts32), ptr(workspace), need,
            stream_handle(words.device),
        )
    check(status, "mb_count_columns")


def pack_count(
    spikes: torch.Tensor,
    words: torch.Tensor,
    rows: int,
    n: int,
    counts64: torch.Tensor | None,
    counts32: torch.Tensor | None,
) -> None:
    """Pack ``spikes[rows, n]`` into ``words`` and count spikes per neuron in one call."""

    need = int(lib().mb_pack_count_workspace_bytes(rows, n))
    workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=spikes.device)
    with torch.cuda.device(spikes.device):
        status = lib().mb_pack_count_spikes(
            dtype_code(spikes.dtype), ptr(spikes), ptr(words), rows, n, ptr(counts64),
            ptr(counts32), ptr(workspace), need, stream_handle(spikes.device),
        )
    check(status, "mb_pack_count_spikes")


class IzhikevichParamsC(ctypes.Structure):
    """``mb_izhikevich_params`` (include/myelin_b200.h)."""

    _fields_ = [(name, ctypes.c_float) for name in (
        "recovery_decay", "recovery_coupling", "reset_voltage", "recovery_jump", "threshold",
        "dt", "voltage_square_coeff", "voltage_coeff", "voltage_bias")]


def izhikevich_forward(
    x: torch.Tensor,
    v0: torch.Tensor,
    u0: torch.Tensor,
    vT: torch.Tensor | None,
    uT: torch.Tensor | None,
    spikes: torch.Tensor | None,
    params: IzhikevichParamsC,
) -> None:
    T, B, N = x.shape
    with torch.cuda.device(x.device):
        status = lib().mb_izhikevich_forward(
            dtype_code(x.dtype), ptr(x), ptr(v0), ptr(u0), ptr(vT), ptr(uT), ptr(spikes),
            T, B, N, ctypes.addressof(params), stream_handle(x.device),
        )
    check(status, "mb_izhikevich_forward")


def scan_forward_packed_scatter(
    *,
    neuron: int,
    x: torch.Tensor,
    v0: torch.Tensor,
    a0: torch.Tensor | None,
    vT: torch.Tensor | None,
    aT: torch.Tensor | None,
    packed: int,
    peers: list[int],
    decay: float,
    threshold: float,
    reset: float,
    adapt_decay: float,
    beta: float,
    reset_mode: int,
) -> None:
    """Packed-only forward whose words go to device address ``packed`` and to
    every address in ``peers`` (this rank's slot in the other ranks' buffers)."""

    T, B, N = x.shape
    arr = (ctypes.c_void_p * max(len(peers), 1))(*peers)
    with torch.cuda.device(x.device):
        status = lib().mb_scan_forward_packed_scatter(
            neuron, dtype_code(x.dtype), ptr(x), ptr(v0), ptr(a0), ptr(vT), ptr(aT), packed, arr,
            len(peers), T, B, N, decay, threshold, reset, adapt_decay, beta, reset_mode,
            stream_handle(x.device),
        )
    check(status, "mb_scan_forward_packed_scatter")


def pack_count_scatter(
    spikes: torch.Tensor,
    words: int,
    rows: int,
    n: int,
    peers: list[int],
    counts64: torch.Tensor | None,
    counts32: torch.Tensor | None,
) -> None:
    """Pack + count ``spikes[rows, n]``, storing the words at device address
    ``words`` (this rank's slot of its own gather buffer) and at every address
    in ``peers`` (this rank's slot in the other ranks' gather buffers)."""

    need = int(lib().mb_pack_count_workspace_bytes(rows, n))
    workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=spikes.device)
    arr = (ctypes.c_void_p * max(len(peers), 1))(*peers)
    with torch.cuda.device(spikes.device):
        status = lib().mb_pack_count_scatter(
            dtype_code(spikes.dtype), ptr(spikes), words, rows, n, arr, len(peers),
            ptr(counts64), ptr(counts32), ptr(workspace), need, stream_handle(spikes.device),
        )
    check(status, "mb_pack_count_scatter")


def ipc_alloc(nbytes: int) -> tuple[int, bytes]:
    """cudaMalloc + IPC handle on the current device: (device pointer, handle bytes)."""

    size = int(lib().mb_ipc_handle_bytes())
    handle = ctypes.create_string_buffer(size)
    out = ctypes.c_void_p()
    check(lib().mb_ipc_alloc(nbytes, ctypes.byref(out), handle), "mb_ipc_alloc")
    return int(out.value), handle.raw


def ipc_open(handle: bytes) -> int:
    out = ctypes.c_void_p()
    check(lib().mb_ipc_open(handle, ctypes.byref(out)), "mb_ipc_open")
    return int(out.value)


def ipc_close(address: int) -> None:
    check(lib().mb_ipc_close(address), "mb_ipc_close")


def ipc_free(address: int) -> None:
    check(lib().mb_ipc_free(address), "mb_ipc_free")
