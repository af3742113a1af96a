"""Stream-synapse projections on the library's tensor-core GEMM (``mb_gemm``).

For a layer with weight W [F, N] (the reference's [in, out] layout,
src/myelin/modules.py:123) and inputs x [M = T*B, F]:

    currents = x W + b,   dX = G W^T,   dW = x^T G,   db = sum over rows of G

(G = dL/dcurrents from the reverse scan). The reference computes these with
``torch.matmul`` per time step (src/myelin/autograd.py:445-556) or with
``tl.dot`` inside its Triton kernels (src/myelin/triton/lif.py:554-612,
1136-1258, float atomics for dW and db). Here:

- 16-bit operands (bf16 / f16) are read where they lie, with no transposed
  copies: x is the K-major A of the forward and the M-major A of dW; W is the
  N-major B of the forward and the K-major B of dX; G is the K-major A of dX
  and the N-major B of dW. An operand whose row pitch is not a multiple of 16
  bytes (the 10-wide readout layer) is first copied into a padded buffer
  (``mb_split_bf16`` with one part).
- fp32 operands are split into three bf16 parts whose sum is exact
  (``mb_split_bf16``), and ``mb_gemm`` sums the six significant part products
  with fp32 accumulation: fp32 products to within 2^-24 relative, on the
  16-bit tensor cores. x's parts carry nonzero flags, so for 0/1 spike inputs
  (exact in one part) the kernel runs only the three products of x's leading
  part.
- db is a fixed-order column sum (``mb_column_sums``), deterministic like dW
  (the reference's Triton kernels use float atomics for both).
- the fp32 input gradient of a narrow layer (N <= 32, the 10-wide readout)
  is a plain fp32-FMA kernel (``mb_gemm_small_k``): its tensor-core tiles
  would be mostly padding.
"""

from __future__ import annotations

import torch

from myelin_b200 import _native as nat

HALF_DTYPES = (torch.bfloat16, torch.float16)
SPLIT_PARTS = 3
SMALL_K = 32  # mb_gemm_small_k: fp32 contractions this short skip the tensor cores


def _round8(n: int) -> int:
    return (n + 7) // 8 * 8


def _pitch_ok(t: torch.Tensor) -> bool:
    """Rows readable by the tensor-map copies: unit inner stride, 16-byte row
    pitch and base."""

    return (t.dim() == 2 and t.stride(1) == 1 and t.stride(0) % 8 == 0
            and t.stride(0) >= t.shape[1] and t.data_ptr() % 16 == 0)


def _operand16(t: torch.Tensor, *, rows_out: int, cols_out: int, zero_fill: bool
               ) -> tuple[torch.Tensor, int]:
    """A 16-bit [rows, cols] matrix as a row-major operand: itself when its
    layout is legal and no padding is asked for, else a copy into a buffer of
    pitch round8(cols_out). ``zero_fill`` writes zeros in the padded region
    (needed where the GEMM reads it: padded K)."""

    rows, cols = t.shape
    if _pitch_ok(t) and rows_out == rows and cols_out == cols:
        return t, t.stride(0)
    ld = _round8(cols_out)
    buf = torch.empty((rows_out, ld), dtype=t.dtype, device=t.device)
    nat.split_bf16(t, rows, cols, t.stride(0), t.stride(1), 1, buf, rows_out if zero_fill else rows,
                   cols_out if zero_fill else cols, ld, 0)
    return buf, ld


def _split3(t: torch.Tensor, *, rows_out: int, cols_out: int, flags: bool
            ) -> tuple[torch.Tensor, int, torch.Tensor | None]:
    """An fp32 [rows, cols] matrix as three bf16 parts [3, rows_out, ld] (zeros
    outside the source), with per-part nonzero flags when asked."""

    rows, cols = t.shape
    ld = _round8(cols_out)
    buf = torch.empty((SPLIT_PARTS, rows_out, ld), dtype=torch.bfloat16, device=t.device)
    nz = torch.empty((SPLIT_PARTS,), dtype=torch.int32, device=t.device) if flags else None
    nat.split_bf16(t, rows, cols, t.stride(0), t.stride(1), SPLIT_PARTS, buf, rows_out, cols_out,
                   ld, rows_out * ld, nz)
    return buf, ld, nz


def project(x2: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """currents[M, N] = x2[M, F] @ weight[F, N] (+ bias), in x2's dtype."""

    M, F = x2.shape
    N = weight.shape[1]
    out = torch.empty((M, N), dtype=x2.dtype, device=x2.device)
    if M == 0 or N == 0:
        return out
    if x2.dtype in HALF_DTYPES:
        K = _round8(F)
        a, lda = _operand16(x2, rows_out=M, cols_out=K, zero_fill=True)
        b, ldb = _operand16(weight, rows_out=K, cols_out=N, zero_fill=True)
        return nat.gemm(nat.GemmOperand(a, nat.MB_KMAJOR, lda),
                        nat.GemmOperand(b, nat.MB_MNMAJOR, ldb), M, N, K, out, bias)
    K = _round8(F)
    a, lda, a_nz = _split3(x2, rows_out=M, cols_out=K, flags=True)
    b, ldb, _ = _split3(weight, rows_out=K, cols_out=N, flags=False)
    return nat.gemm(
        nat.GemmOperand(a, nat.MB_KMAJOR, lda, parts=SPLIT_PARTS, part_stride=M * lda,
                        nonzero=a_nz),
        nat.GemmOperand(b, nat.MB_MNMAJOR, ldb, parts=SPLIT_PARTS, part_stride=K * ldb),
        M, N, K, out, bias)


def input_grad(g2: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """dX[M, F] = g2[M, N] @ weight[F, N]^T, in g2's dtype."""

    M, N = g2.shape
    F = weight.shape[0]
    out = torch.empty((M, F), dtype=g2.dtype, device=g2.device)
    if M == 0 or F == 0:
        return out
    if g2.dtype == torch.float32 and N <= SMALL_K and g2.stride(1) == 1 and weight.stride(1) == 1:
        # a narrow fp32 layer: a 10-deep contraction in plain fp32 FMAs
        return nat.gemm_small_k(g2, weight, out)
    K = _round8(N)
    if g2.dtype in HALF_DTYPES:
        a, lda = _operand16(g2, rows_out=M, cols_out=K, zero_fill=True)
        b, ldb = _operand16(weight, rows_out=F, cols_out=K, zero_fill=True)
        return nat.gemm(nat.GemmOperand(a, nat.MB_KMAJOR, lda),
                        nat.GemmOperand(b, nat.MB_KMAJOR, ldb), M, F, K, out)
    a, lda, a_nz = _split3(g2, rows_out=M, cols_out=K, flags=True)
    b, ldb, _ = _split3(weight, rows_out=F, cols_out=K, flags=False)
    return nat.gemm(
        nat.GemmOperand(a, nat.MB_KMAJOR, lda, parts=SPLIT_PARTS, part_stride=M * lda,
                        nonzero=a_nz),
        nat.GemmOperand(b, nat.MB_KMAJOR, ldb, parts=SPLIT_PARTS, part_stride=F * ldb),
        M, F, K, out)


def weight_grad(x2: torch.Tensor, g2: torch.Tensor, weight_dtype: torch.dtype) -> torch.Tensor:
    """dW[F, N] = x2[M, F]^T @ g2[M, N] in ``weight_dtype`` (fp32 accumulation,
    one rounding)."""

    M, F = x2.shape
    N = g2.shape[1]
    out = torch.empty((F, N), dtype=weight_dtype, device=x2.device)
    if F == 0 or N == 0:
        return out
    if M == 0:
        return out.zero_()
    if x2.dtype in HALF_DTYPES:
        a, lda = _operand16(x2, rows_out=M, cols_out=F, zero_fill=False)
        b, ldb = _operand16(g2, rows_out=M, cols_out=N, zero_fill=False)
        return nat.gemm(nat.GemmOperand(a, nat.MB_MNMAJOR, lda),
                        nat.GemmOperand(b, nat.MB_MNMAJOR, ldb), F, N, M, out)
    a, lda, a_nz = _split3(x2, rows_out=M, cols_out=F, flags=True)
    b, ldb, _ = _split3(g2, rows_out=M, cols_out=N, flags=False)
    return nat.gemm(
        nat.GemmOperand(a, nat.MB_MNMAJOR, lda, parts=SPLIT_PARTS, part_stride=M * lda,
                        nonzero=a_nz),
        nat.GemmOperand(b, nat.MB_MNMAJOR, ldb, parts=SPLIT_PARTS, part_stride=M * ldb),
        F, N, M, out)


def bias_grad(g2: torch.Tensor, bias_dtype: torch.dtype) -> torch.Tensor:
    """db[N] = sum over rows of g2[M, N] (fixed order, fp32 accumulation)."""

    M, N = g2.shape
    out = torch.empty((N,), dtype=bias_dtype, device=g2.device)
    if N == 0:
        return out
    src = g2 if g2.stride(1) == 1 else g2.contiguous()
    nat.column_sums(src, M, N, src.stride(0), out)
    return out
