"""The stream-synapse projections on the tensor-core GEMM (``mb_gemm``) against
plain PyTorch references (fp32 for 16-bit operands, float64 for fp32 operands).

Covers every operand layout the projections use (K-major / N-major / M-major,
no transposed copies), ragged M, N and K tails on the one-SM and two-SM
kernels, operands copied into padded buffers (rows not a multiple of 16 bytes:
the 10-wide readout), and fp32 operands split into three bf16 parts (fp32
products on the 16-bit tensor cores), with and without the skip of all-zero
parts that 0/1 spike inputs allow.

Bars: 16-bit operands with fp32 output within rtol 1e-4 of the fp32 product
of the same operands, scaled by max|C| (summation order); 16-bit output within
one rounding (rtol 1e-2); fp32 operands within 1e-5 scaled of the float64
product (the fp32 bar of the north star).
"""

from __future__ import annotations

import pytest
import torch

from myelin_b200 import _native as nat
from myelin_b200 import projection
from tests.conftest import assert_close_scaled

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rand(shape, gen, dtype=torch.float32, scale=1.0):
    return (torch.randn(shape, generator=gen, device=DEV) * scale).to(dtype)


def _spikes(shape, gen, p, dtype):
    return (torch.rand(shape, generator=gen, device=DEV) < p).to(dtype)


def _check(got, ref, rtol, what):
    torch.cuda.synchronize()
    assert torch.isfinite(got).all(), what
    assert_close_scaled(got.double().cpu().numpy(), ref.double().cpu().numpy(), rtol=rtol, what=what)


SHAPES = [
    # (M = T*B, F, N)
    (64, 32, 48),          # one tile, K < one block
    (300, 784, 10),        # config-2 readout-like widths: padded N, ragged F
    (257, 72, 129),        # ragged everywhere
    (6400, 784, 1024),     # config-2 layer 1 (pair kernel at 16 bits)
    (4999, 520, 3001),     # many pair tiles, ragged tails
    (2048, 2048, 4096),    # config-5 layer width, K = 2048
]


@pytest.mark.parametrize("M,F,N", SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_16bit_projections_match_fp32_products(M, F, N, dtype):
    gen = torch.Generator(device=DEV).manual_seed(M + F + N)
    x = _spikes((M, F), gen, 0.2, dtype)
    w = _rand((F, N), gen, dtype, scale=F ** -0.5)
    b = _rand((N,), gen, dtype, scale=0.1)
    g = _rand((M, N), gen, dtype, scale=0.01)
    xf, wf, bf, gf = x.float(), w.float(), b.float(), g.float()
    cur = projection.project(x, w, b)
    assert cur.dtype == dtype and cur.shape == (M, N)
    _check(cur.float(), (xf @ wf + bf).to(dtype).float(), 1e-2, "currents")
    dx = projection.input_grad(g, w)
    _check(dx.float(), (gf @ wf.t()).to(dtype).float(), 1e-2, "dX")
    dw = projection.weight_grad(x, g, torch.float32)
    _check(dw, xf.t() @ gf, 1e-4, "dW fp32 out")
    dw16 = projection.weight_grad(x, g, dtype)
    _check(dw16.float(), (xf.t() @ gf).to(dtype).float(), 1e-2, "dW 16-bit out")
    db = projection.bias_grad(g, torch.float32)
    _check(db, gf.sum(0), 1e-5, "db")


@pytest.mark.parametrize("M,F,N", SHAPES[:4])
def test_fp32_projections_split_into_bf16_parts(M, F, N):
    gen = torch.Generator(device=DEV).manual_seed(7 * M + F + N)
    x = _spikes((M, F), gen, 0.2, torch.float32)
    w = _rand((F, N), gen, scale=F ** -0.5)
    b = _rand((N,), gen, scale=0.1)
    g = _rand((M, N), gen, scale=0.01)
    xd, wd, bd, gd = x.double(), w.double(), b.double(), g.double()
    _check(projection.project(x, w, b), xd @ wd + bd, 1e-5, "currents (spike input)")
    _check(projection.input_grad(g, w), gd @ wd.t(), 1e-5, "dX")
    _check(projection.weight_grad(x, g, torch.float32), xd.t() @ gd, 1e-5, "dW")
    _check(projection.bias_grad(g, torch.float32), gd.sum(0), 1e-5, "db")
    # a real-valued input needs all three parts of x: the part-skip flags must
    # enable them
    xr = _rand((M, F), gen)
    _check(projection.project(xr, w, b), xr.double() @ wd + bd, 1e-5, "currents (real input)")
    _check(projection.weight_grad(xr, g, torch.float32), xr.double().t() @ gd, 1e-5,
           "dW (real input)")


def test_fp32_weight_gradient_over_long_k_runs_in_slices():
    """K = T*B = 51200 (config-5 rows) in fp32: 25 K slices summed in order;
    the bar is the same 1e-5 (scaled) against float64."""

    lib = nat.lib()
    M, F, N = 51200, 64, 96
    assert lib.mb_gemm_workspace_bytes(F, N, M, 3, 3, nat.MB_F32) > 0
    # a large 16-bit problem of moderate K runs unsliced; a small one is sliced
    # to occupy the SMs; a long-K one to even out the last wave
    assert lib.mb_gemm_workspace_bytes(4096, 4096, 4096, 1, 1, nat.MB_BF16) == 0
    assert lib.mb_gemm_workspace_bytes(F, N, M, 1, 1, nat.MB_BF16) > 0
    assert lib.mb_gemm_workspace_bytes(4096, 4096, M, 1, 1, nat.MB_BF16) > 0
    gen = torch.Generator(device=DEV).manual_seed(13)
    x = _rand((M, F), gen)
    g = _rand((M, N), gen, scale=0.01)
    _check(projection.weight_grad(x, g, torch.float32), x.double().t() @ g.double(), 1e-5,
           "dW over K = 51200")


def test_long_k_tail_slicing_matches_fp32_products():
    """K >= 8192 with more two-SM tiles than SM pairs: the whole waves of tiles
    run unsliced and only the last wave's tiles are split into K slices whose
    fp32 partial sums a second kernel adds (+ bias). Weight gradients
    (M-major x, N-major G, 16-bit and fp32 output) and a forward with bias and
    ragged M and N, against fp32 products of the same operands."""

    lib = nat.lib()
    assert lib.mb_gemm_workspace_bytes(4096, 4096, 8192, 1, 1, nat.MB_BF16) > 0
    assert lib.mb_gemm_workspace_bytes(4096, 4096, 4096, 1, 1, nat.MB_BF16) == 0
    gen = torch.Generator(device=DEV).manual_seed(21)
    rows, F, N = 8192, 4096, 4096
    x = _spikes((rows, F), gen, 0.1, torch.bfloat16)
    g = _rand((rows, N), gen, torch.bfloat16, scale=0.01)
    ref = x.float().t() @ g.float()
    _check(projection.weight_grad(x, g, torch.bfloat16).float(), ref.bfloat16().float(), 1e-2,
           "dW bf16, tail-sliced")
    _check(projection.weight_grad(x, g, torch.float32), ref, 1e-4, "dW fp32 out, tail-sliced")
    del x, g, ref
    M, K, N2 = 4000, 8192, 4000
    xf = _spikes((M, K), gen, 0.2, torch.bfloat16)
    w = _rand((K, N2), gen, torch.bfloat16, scale=K ** -0.5)
    b = _rand((N2,), gen, torch.bfloat16, scale=0.1)
    cur = projection.project(xf, w, b)
    _check(cur.float(), (xf.float() @ w.float() + b.float()).bfloat16().float(), 1e-2,
           "forward with bias, tail-sliced, ragged")
    assert nat.device_status(clear=True) == 0


@pytest.mark.parametrize("rows,cols,ld", [(37, 45, 48), (64, 96, 96), (6400, 784, 784)])
def test_split_parts_match_successive_bf16_roundings(rows, cols, ld):
    """Each part is the bf16 rounding of what the parts before it left, for
    the scalar kernel (45 columns) and the 4-column vector kernel (96, 784):
    bit for bit against the same roundings in torch, zero padding outside
    the source, inf/nan kept whole in the leading part."""

    gen = torch.Generator(device=DEV).manual_seed(rows + cols)
    src = torch.randn((rows, cols), generator=gen, device=DEV) * 3.0
    src[0, 0] = float("inf")
    src[1, 2] = float("nan")
    src[2, 3] = 0.0
    src[3, 1] = 1e-30
    dst_rows = rows + 3
    parts = torch.full((3, dst_rows, ld), 7.0, dtype=torch.bfloat16, device=DEV)
    nz = torch.empty(3, dtype=torch.int32, device=DEV)
    nat.split_bf16(src, rows, cols, cols, 1, 3, parts, dst_rows, ld, ld, dst_rows * ld, nz)
    torch.cuda.synchronize()
    finite = torch.isfinite(src)
    rest = torch.where(finite, src, torch.zeros_like(src))
    want = []
    for p in range(3):
        h = rest.bfloat16()
        want.append(h)
        rest = rest - h.float()
    for p in range(3):
        got = parts[p, :rows, :cols]
        assert torch.equal(got.view(torch.int16)[finite], want[p].view(torch.int16)[finite]), p
        if p == 0:
            lead = got.float()
            assert torch.isinf(lead[0, 0]) and lead[0, 0] > 0 and torch.isnan(lead[1, 2])
        else:
            assert torch.count_nonzero(got.float()[~finite]) == 0
        assert torch.count_nonzero(parts[p, rows:, :]) == 0
        assert torch.count_nonzero(parts[p, :, cols:]) == 0
    assert nz.tolist() == [1, 1, 1]


def test_split_parts_sum_exactly_and_flag_nonzero_parts():
    gen = torch.Generator(device=DEV).manual_seed(11)
    src = torch.randn((37, 45), generator=gen, device=DEV) * 3.0
    src[0, 0] = float("inf")
    src[1, 1] = 0.0
    parts = torch.empty((3, 40, 48), dtype=torch.bfloat16, device=DEV)
    nz = torch.empty(3, dtype=torch.int32, device=DEV)
    nat.split_bf16(src, 37, 45, 45, 1, 3, parts, 40, 48, 48, 40 * 48, nz)
    torch.cuda.synchronize()
    total = parts[0].float() + parts[1].float() + parts[2].float()
    finite = torch.isfinite(src)
    assert torch.equal(total[:37, :45][finite], src[finite])
    assert torch.isinf(total[0, 0])
    assert torch.count_nonzero(parts[:, 37:, :]) == 0 and torch.count_nonzero(parts[:, :, 45:]) == 0
    assert nz.tolist() == [1, 1, 1]
    spikes = (torch.rand((33, 20), generator=gen, device=DEV) < 0.5).float()
    nat.split_bf16(spikes, 33, 20, 20, 1, 3, parts, 33, 20, 48, 40 * 48, nz)
    torch.cuda.synchronize()
    assert nz.tolist() == [1, 0, 0]


def test_transposed_and_strided_operands_are_relaid_out():
    gen = torch.Generator(device=DEV).manual_seed(5)
    base = _rand((200, 130), gen, torch.bfloat16)
    w = base.t()[:, :100]  # [130, 100] view with unit row stride: not row-major
    x = _spikes((96, 130), gen, 0.3, torch.bfloat16)
    cur = projection.project(x, w, None)
    _check(cur.float(), (x.float() @ w.float()).bfloat16().float(), 1e-2, "transposed weight")


@pytest.mark.parametrize("K", [1, 7, 8, 10, 16, 17, 32])
def test_small_k_fp32_kernel_within_k_roundings(K):
    """``mb_gemm_small_k`` (narrow fp32 layers' input gradient) for K in every
    padding bucket (8, 16, 32) and ragged M and N, against float64 products:
    an in-order fmaf sum of K terms is within K * 2^-23 of the sum of the
    products' magnitudes."""

    gen = torch.Generator(device=DEV).manual_seed(40 + K)
    M, N = 70, 300
    a = _rand((M, K), gen)
    b = _rand((N, K), gen)
    out = torch.full((M, N), float("nan"), device=DEV)
    nat.gemm_small_k(a, b, out)
    torch.cuda.synchronize()
    ref = a.double() @ b.double().t()
    mag = a.double().abs() @ b.double().abs().t()
    assert torch.isfinite(out).all()
    assert ((out.double() - ref).abs() <= mag * (K * 2.0 ** -23) + 1e-30).all()


def test_mb_gemm_rejects_m_major_a_with_k_major_b():
    lib = nat.lib()
    a = torch.zeros((64, 64), dtype=torch.bfloat16, device=DEV)
    c = torch.zeros((64, 64), dtype=torch.float32, device=DEV)
    rc = lib.mb_gemm(nat.MB_BF16, a.data_ptr(), nat.MB_MNMAJOR, 64, 0, 1, None, a.data_ptr(),
                     nat.MB_KMAJOR, 64, 0, 1, None, None, 0, nat.MB_F32, c.data_ptr(), 64, 64, 64,
                     64, None, 0, None)
    assert rc != 0 and "M-major A" in lib.mb_last_error().decode()


def test_gemm_device_status_clean_after_projections():
    assert nat.device_status(clear=True) == 0
