"""spx_rmsnorm (the model loop's RMSNorm, residual add fused in front) against the
float32 PyTorch expression of the same arithmetic: ``h = x + residual`` in the dtype
(bit-exact), ``dtype(h * rsqrt(mean(h^2) + eps)) * weight`` within two units in the last
place of the dtype (the mean's summation order and the reciprocal square root differ)."""
import pytest
import torch

from conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


def _ref(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rows,dim", [(8, 4096), (3, 512), (1, 8192), (257, 1032), (33, 8)])
@pytest.mark.parametrize("fused", [False, True])
def test_rmsnorm_matches_torch(dtype, rows, dim, fused):
    from unsloth_spectral import _ops
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + dim)
    x = (torch.randn(rows, dim, generator=g, device="cuda") * 3).to(dtype)
    r = (torch.randn(rows, dim, generator=g, device="cuda") * 3).to(dtype)
    w = (1 + 0.1 * torch.randn(dim, generator=g, device="cuda")).to(dtype)
    eps = 1e-5
    if fused:
        out, h = _ops.rmsnorm(x, w, eps, residual=r)
        hr = r + x
        assert torch.equal(h, hr)
        ref = _ref(hr, w, eps)
    else:
        out = _ops.rmsnorm(x, w, eps)
        ref = _ref(x, w, eps)
    ulp = 2.0 ** (-10 if dtype == torch.float16 else -7)
    err = ((out.float() - ref.float()).abs() / ref.float().abs().clamp_min(1e-3)).max().item()
    assert err <= 2 * ulp, err


def test_rmsnorm_leading_dims_and_zero_rows():
    from unsloth_spectral import _ops
    x = torch.randn(2, 5, 256, device="cuda").to(torch.bfloat16)
    w = torch.ones(256, device="cuda", dtype=torch.bfloat16)
    out = _ops.rmsnorm(x, w, 1e-6)
    assert out.shape == x.shape
    torch.testing.assert_close(out.float(), _ref(x, w, 1e-6).float(), rtol=2 ** -6, atol=0)
    empty = torch.empty(0, 256, device="cuda", dtype=torch.bfloat16)
    assert _ops.rmsnorm(empty, w, 1e-6).shape == (0, 256)
