"""Tensor-core bring-up: one 128xNx128 bf16 UMMA per operand configuration the
attention and qmm kernels use, compared with an fp32 torch matmul of the same
bf16 inputs (exact products, f32 accumulation: tolerance 1e-3 relative)."""
import pytest
import torch

from aestrix_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,n", [(0, 128), (0, 256), (1, 128), (2, 128), (2, 256)])
def test_umma_modes(cuda_ctx, mode, n):
    g = torch.Generator(device="cpu").manual_seed(100 + mode * 7 + n)
    a = torch.randn(128, 128, generator=g).to(torch.bfloat16).cuda()
    if mode == 0:
        b = torch.randn(n, 128, generator=g).to(torch.bfloat16).cuda()
        ref = a.float() @ b.float().t()
    else:
        b = torch.randn(128, n, generator=g).to(torch.bfloat16).cuda()
        ref = a.float() @ b.float()
    d = torch.full((128, n), float("nan"), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    cuda_ctx.check(_lib.lib().aex_selftest_umma(cuda_ctx.handle, mode, a.data_ptr(), b.data_ptr(), n,
                                                d.data_ptr(), stream))
    cuda_ctx.sync(stream)
    assert torch.isfinite(d).all()
    err = (d - ref).abs().max().item()
    assert err <= 1e-3 * ref.abs().max().item(), f"mode {mode} n {n}: max abs err {err}"
