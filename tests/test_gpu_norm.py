"""The decode loop's small kernels against the PyTorch expressions they replace:
spx_rmsnorm (RMSNorm with the residual add fused in front): ``h = x + residual`` in the
dtype (bit-exact), ``dtype(h * rsqrt(mean(h^2) + eps)) * weight`` within two units in the
last place of the dtype (the mean's summation order and the reciprocal square root
differ); spx_rope_rows (the new token's query RoPE): bit-exact with ``apply_rope`` in
float32, for positions per sequence, one position for all, and a host position."""
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


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("fused_qkv", [False, True])
def test_rope_rows_matches_apply_rope(dtype, fused_qkv):
    from unsloth_spectral import _ops
    from unsloth_spectral import synthetic as syn
    from unsloth_spectral.spectral_attention import apply_rope
    B, nh, hd = 5, 8, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    width = nh * hd + (2 * 2 * hd if fused_qkv else 0)   # q rows inside a [q | k | v] projection
    full = torch.randn(B, 1, width, generator=g, device="cuda").to(dtype)
    qp = full[..., :nh * hd]
    cos, sin = syn.rope_tables(40000, hd, 1e6, device="cuda")
    q = qp.view(B, 1, nh, hd).transpose(1, 2)
    pos_rows = torch.tensor([[3], [900], [32767], [0], [12345]], device="cuda")
    ref = apply_rope(q.float(), cos[pos_rows][:, None], sin[pos_rows][:, None]).to(dtype)
    assert torch.equal(_ops.rope_rows(qp, nh, hd, cos, sin, pos_rows), ref)
    wide = torch.arange(10, device="cuda").repeat(B, 1) * 7 + 100     # positions as the last column of [B, L]
    pid = wide.reshape(-1, wide.shape[-1])[:, -1:]
    ref = apply_rope(q.float(), cos[pid][:, None], sin[pid][:, None]).to(dtype)
    assert torch.equal(_ops.rope_rows(qp, nh, hd, cos, sin, pid), ref)
    one = torch.tensor([[777]], device="cuda")
    ref = apply_rope(q.float(), cos[one][:, None], sin[one][:, None]).to(dtype)
    assert torch.equal(_ops.rope_rows(qp, nh, hd, cos, sin, one), ref)
    ref = apply_rope(q.float(), cos[4321], sin[4321]).to(dtype)
    assert torch.equal(_ops.rope_rows(qp, nh, hd, cos, sin, None, 4321), ref)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_hot_append_matches_index_copy(dtype):
    """spx_hot_append (the cache's single-token append, one launch) against the
    index_copy_ formulation: three tokens appended from strided views of a fused
    projection, rows / positions / device length identical; at full capacity it writes
    nothing and leaves the length."""
    from unsloth_spectral import _ops
    B, H, D, cap = 3, 4, 128, 6
    g = torch.Generator(device="cuda").manual_seed(5)
    hk = torch.randn(B, H, cap, D, generator=g, device="cuda").to(dtype)
    hv = torch.randn(B, H, cap, D, generator=g, device="cuda").to(dtype)
    hp = torch.arange(cap, device="cuda") * 11
    hl = torch.tensor(2, dtype=torch.int32, device="cuda")
    rk, rv, rp = hk.clone(), hv.clone(), hp.clone()
    for step in range(3):
        full = torch.randn(B, 1, (2 + 2) * H * D // 2, generator=g, device="cuda").to(dtype)
        k = full[..., :H * D].view(B, 1, H, D).transpose(1, 2)
        v = full[..., H * D:2 * H * D].view(B, 1, H, D).transpose(1, 2)
        pos = torch.tensor([1000 + step], device="cuda")
        idx = torch.tensor([2 + step], device="cuda")
        rk.index_copy_(2, idx, k)
        rv.index_copy_(2, idx, v)
        rp.index_copy_(0, idx, pos)
        _ops.hot_append(k, v, hk, hv, hp, hl, pos)
    assert torch.equal(hk, rk) and torch.equal(hv, rv) and torch.equal(hp, rp) and int(hl) == 5
    k = torch.zeros(B, H, 1, D, device="cuda", dtype=dtype)
    _ops.hot_append(k, k, hk, hv, hp, hl, torch.tensor([7], device="cuda"))
    assert int(hl) == 6 and torch.equal(hk[:, :, :5], rk[:, :, :5])
    _ops.hot_append(k, k, hk, hv, hp, hl, torch.tensor([8], device="cuda"))   # full: nothing written
    assert int(hl) == 6 and int(hp[5]) == 7
