"""The tcgen05 projection GEMM against a plain PyTorch fp32 reference.

C = A @ B^T (+ bias) with bf16/f16 operands and fp32 accumulation, on the
one-SM kernel (small problems) and the two-SM pair kernel. The fp32
reference multiplies the same (upcast) operands; fp32 outputs agree to
rtol 1e-4 scaled by max|C| (summation order), 16-bit outputs to one rounding
of the output type.
"""

from __future__ import annotations

import pytest
import torch

from myelin_b200 import _native as nat
from tests.conftest import assert_close_scaled

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(M, N, K, dtype, seed, bias_dtype):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    a = torch.randn((M, K), generator=gen, device=DEV).to(dtype)
    b = (torch.randn((N, K), generator=gen, device=DEV) / K ** 0.5).to(dtype)
    bias = None if bias_dtype is None else torch.randn((N,), generator=gen, device=DEV).to(bias_dtype)
    ref = a.float() @ b.float().t()
    if bias is not None:
        ref = ref + bias.float()
    return a, b, bias, ref


@pytest.mark.parametrize("M,N,K", [(1, 8, 8), (128, 256, 64), (129, 257, 72), (300, 10, 784),
                                   (1000, 1000, 1024), (6400, 1024, 784), (2048, 4096, 2048),
                                   # two-SM pair tiles (>= 74 tiles of 256 x 256) with ragged
                                   # M, N and K tails; the last pair tile's second half lies
                                   # wholly past M in (562, 8192, 64)
                                   (4999, 3001, 520), (562, 8192, 64)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("out_f32", [True, False])
def test_gemm_matches_fp32_reference(M, N, K, dtype, out_f32):
    for bias_dtype in (None, torch.float32, dtype):
        a, b, bias, ref = _case(M, N, K, dtype, M + N + K, bias_dtype)
        out = torch.full((M, N), float("nan"), device=DEV,
                         dtype=torch.float32 if out_f32 else dtype)
        nat.gemm_tn(a, b, bias, out)
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        got = out.float().cpu().numpy()
        if out_f32:
            assert_close_scaled(got, ref.cpu().numpy(), rtol=1e-4, what=f"{M}x{N}x{K}")
        else:
            assert_close_scaled(got, ref.to(dtype).float().cpu().numpy(), rtol=1e-2,
                                what=f"{M}x{N}x{K} 16-bit out")


def test_gemm_strided_operands_and_output():
    a_full = torch.randn((500, 200), device=DEV).bfloat16()
    b_full = torch.randn((300, 200), device=DEV).bfloat16()
    a, b = a_full[:, :128], b_full[:, :128]  # leading dimension 200, K = 128
    out_full = torch.zeros((500, 320), device=DEV)
    out = out_full[:, :300]
    nat.gemm_tn(a, b, None, out)
    ref = a.float() @ b.float().t()
    assert_close_scaled(out.cpu().numpy(), ref.cpu().numpy(), rtol=1e-4)
    assert torch.equal(out_full[:, 300:], torch.zeros_like(out_full[:, 300:]))


def test_gemm_device_status_clean():
    assert nat.device_status(clear=True) == 0
