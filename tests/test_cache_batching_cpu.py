"""Host-side check of SpectralCache's prompt compression on the CPU: the batched path
(one compression call for all full blocks of a prompt) must place every output in the
same tier slot as the block-by-block path.  The compression call is replaced by a
stand-in that reads and writes each operand through the pointer, strides and matrix
count it is given - as the C library does - and computes a deterministic function of
each matrix and its sketch, so that any mix-up of matrices, sketches or slots shows."""
import pytest
import torch

from unsloth_spectral import SpectralCache, _ops
import unsloth_spectral.spectral_cache as sc_mod

B, H, T, D, KK, KV = 2, 3, 64, 32, 5, 9


def fake_rsvd(M, omega, k, n_iter, *, want_factors=True, codes=None, codes_strides=None, rank_pad=None,
              qscale=None, scale_stride=1, qminmax=None, minmax_stride=2, basis=None, basis_stride=0,
              M_mat_stride=0, num_mats=None, m=None, n=None, codes_tiled=False):
    assert not want_factors
    kp = rank_pad
    Mm = torch.as_strided(M, (num_mats, m, n), (M_mat_stride or m * n, n, 1), M.storage_offset()).float()
    om = omega.float()
    row = Mm.sum(-1)                                   # [mats, m]
    sk = om.sum((1, 2))                                # [mats]
    vals = (row[:, :, None] * (torch.arange(kp) + 1) + sk[:, None, None]).round().clamp(-127, 127)
    vals[:, :, k:] = 0
    cs = codes_strides
    if codes_tiled:
        dst = torch.as_strided(codes, (num_mats, kp * m), (cs[0], 1), codes.storage_offset())
        dst.copy_(vals.transpose(1, 2).reshape(num_mats, -1).to(torch.int8))
    else:
        dst = torch.as_strided(codes, (num_mats, m, kp), cs, codes.storage_offset())
        dst.copy_(vals.to(torch.int8))
    torch.as_strided(qscale, (num_mats,), (scale_stride,), qscale.storage_offset()).copy_(sk + Mm.mean((1, 2)))
    torch.as_strided(qminmax, (num_mats, 2), (minmax_stride, 1), qminmax.storage_offset()).copy_(
        torch.stack([Mm.amin((1, 2)), Mm.amax((1, 2))], 1))
    bas = (om[:, :, :1].transpose(1, 2) * (torch.arange(kp)[None, :, None] + 1)).expand(num_mats, kp, n).clone()
    bas[:, k:] = 0
    torch.as_strided(basis, (num_mats, kp, n), (basis_stride, n, 1), basis.storage_offset()).copy_(bas)
    return None, None, None


@pytest.mark.parametrize("nfull,extra", [(3, 10), (2, 0), (5, 63)])
def test_batched_prompt_compression_matches_blockwise(monkeypatch, nfull, extra):
    monkeypatch.setattr(_ops, "rsvd", fake_rsvd)
    monkeypatch.setattr(sc_mod._ops, "rsvd", fake_rsvd)
    g = torch.Generator().manual_seed(nfull)
    Ttot = nfull * T + extra
    K = torch.randn(B, H, Ttot, D, generator=g).half()
    V = torch.randn(B, H, Ttot, D, generator=g).half()

    def build(chunks):
        cache = SpectralCache(H, D, block_size=T, k_rank_keys=KK, k_rank_values=KV, device="cpu",
                              dtype=torch.float16, oversampling=4)
        torch.manual_seed(11)
        for c0, c1 in chunks:
            cache.append(K[:, :, c0:c1], V[:, :, c0:c1])
        return cache

    whole = build([(0, Ttot)])
    blockwise = build([(c0, min(c0 + T, Ttot)) for c0 in range(0, Ttot, T)])
    assert whole.num_cold_blocks == blockwise.num_cold_blocks == nfull
    a, b = whole.tiers, blockwise.tiers
    for name in SpectralCache._COLD:
        assert torch.equal(getattr(a, name)[:, :, :nfull], getattr(b, name)[:, :, :nfull]), name
    assert torch.equal(a.block_pos[:nfull], b.block_pos[:nfull])
    assert a.block_pos[:nfull].tolist() == [i * T for i in range(nfull)]
    assert whole.hot_len == blockwise.hot_len == extra
    if extra:
        assert torch.equal(whole.hot_K, blockwise.hot_K)
        assert torch.equal(whole.hot_K, K[:, :, nfull * T:])
    # distinct blocks got distinct outputs (the stand-in is not constant)
    assert not torch.equal(a.scale_k[:, :, 0], a.scale_k[:, :, 1])
