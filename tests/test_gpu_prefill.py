"""spx_prefill_attn (the multi-query / prefill attention over the compressed cache) against
a float32 PyTorch evaluation of the reference's dense path (integration.py:292-346):
reconstructed K and V (get_kv), keys rotated at their cached positions with the first
half of the tables, softmax(Q K^T / sqrt(D) + mask) V.  Tolerance: cosine >= 0.9999 and
max-abs <= 1e-2 per (sequence, head) output."""
import math

import pytest
import torch

from conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

COS_MIN, ABS_MAX = 0.9999, 1e-2


def _cache(B, H, n_tok, dtype, kk=16, kv=32, seed=0):
    from unsloth_spectral import SpectralCache
    from unsloth_spectral import synthetic as syn
    dev = torch.device("cuda")
    K, V = syn.kv_layer_batched(1, seed, B, H, n_tok, 128, 24, 0.85, dev, dtype=dtype)
    c = SpectralCache(H, 128, block_size=512, k_rank_keys=kk, k_rank_values=kv, device=dev, dtype=dtype)
    c.append(K, V, torch.arange(n_tok, device=dev)[None])
    return c


def _reference(q, cache, cos, sin, q_pos, mask=None, causal=False):
    from unsloth_spectral.spectral_attention import apply_rope
    K, V = cache.get_kv()
    pos = cache.get_all_positions()
    Kr = apply_rope(K.float(), cos[pos][None, None], sin[pos][None, None]).to(K.dtype).float()
    n_rep = q.shape[1] // K.shape[1]
    Kr = Kr.repeat_interleave(n_rep, dim=1)
    Vr = V.float().repeat_interleave(n_rep, dim=1)
    S = q.float() @ Kr.transpose(-1, -2) / math.sqrt(q.shape[-1])
    if mask is not None:
        S = S + mask.float()
    if causal:
        S = S.masked_fill(pos[None, :] > q_pos[:, None], float("-inf"))
    return torch.softmax(S, dim=-1) @ Vr


def _close(got, ref):
    g, r = got.double().flatten(2), ref.double().flatten(2)
    cs = (g * r).sum(-1) / (g.norm(dim=-1) * r.norm(dim=-1))
    assert cs.min().item() >= COS_MIN, cs.min().item()
    assert (g - r).abs().max().item() <= ABS_MAX, (g - r).abs().max().item()


@pytest.mark.parametrize("dtype,H,nrep,n_tok,Tq,kk,kv", [
    (torch.float16, 8, 4, 1636, 200, 16, 32),     # 3 blocks + 100 hot, queries straddle block 2 and the hot tier
    (torch.bfloat16, 8, 4, 1636, 200, 16, 32),
    (torch.float16, 4, 1, 1100, 130, 32, 16),     # n_rep 1, last query tile partial
    (torch.float16, 2, 8, 700, 64, 16, 16),       # n_rep 8
    (torch.float16, 4, 2, 1024, 1024, 16, 32),    # whole prompt, no hot tier
    (torch.float16, 8, 4, 300, 300, 16, 32),      # hot tier only
])
def test_prefill_causal_matches_dense_reference(dtype, H, nrep, n_tok, Tq, kk, kv):
    from unsloth_spectral import _ops
    from unsloth_spectral import synthetic as syn
    dev = torch.device("cuda")
    B = 2
    cache = _cache(B, H, n_tok, dtype, kk, kv)
    cos, sin = syn.rope_tables(n_tok + 8, 128, 1e6, device=dev)
    g = torch.Generator(device=dev).manual_seed(3)
    q = (torch.randn(B, H * nrep, Tq, 128, generator=g, device=dev) / math.sqrt(128) * 4).to(dtype)
    q_pos = torch.arange(n_tok - Tq, n_tok, device=dev)
    got = _ops.prefill(q, cache.tiers, cos, sin, q_pos, causal=True)
    _close(got, _reference(q, cache, cos, sin, q_pos, causal=True))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_prefill_additive_mask_and_non_causal(dtype):
    """An arbitrary additive mask (finite values, -inf entries, per-head rows) over all keys
    in cache order, without the causal rule; and no mask at all."""
    from unsloth_spectral import _ops
    from unsloth_spectral import synthetic as syn
    dev = torch.device("cuda")
    B, H, nrep, n_tok, Tq = 2, 4, 2, 1200, 96
    cache = _cache(B, H, n_tok, dtype, seed=5)
    cos, sin = syn.rope_tables(n_tok + 8, 128, 1e6, device=dev)
    g = torch.Generator(device=dev).manual_seed(9)
    q = (torch.randn(B, H * nrep, Tq, 128, generator=g, device=dev) / math.sqrt(128) * 4).to(dtype)
    q_pos = torch.arange(n_tok - Tq, n_tok, device=dev)
    mask = torch.randn(B, H * nrep, Tq, n_tok, generator=g, device=dev)
    mask = mask.masked_fill(torch.rand(B, H * nrep, Tq, n_tok, generator=g, device=dev) < 0.3, float("-inf"))
    mask[..., 0] = 0.0   # every row keeps a key
    _close(_ops.prefill(q, cache.tiers, cos, sin, q_pos, mask=mask), _reference(q, cache, cos, sin, q_pos, mask=mask))
    m_dt = mask[:, :1].to(dtype)   # broadcast over heads, the attention dtype
    _close(_ops.prefill(q, cache.tiers, cos, sin, q_pos, mask=m_dt), _reference(q, cache, cos, sin, q_pos, mask=m_dt))
    _close(_ops.prefill(q, cache.tiers, cos, sin, q_pos), _reference(q, cache, cos, sin, q_pos))


def test_patched_prefill_uses_kernel_and_matches_eager_path():
    """The integration layer's prompt path: a causal HF-style mask is recognised and
    applied as the causal rule; the kernel's output equals the eager reconstruct-and-
    multiply path on the same cache."""
    from unsloth_spectral import integration as I
    from unsloth_spectral import synthetic as syn
    dev = torch.device("cuda")
    B, H, nrep, n_tok = 1, 8, 4, 1100
    cache = _cache(B, H, n_tok, torch.float16, seed=7)
    cos, sin = syn.rope_tables(n_tok + 8, 128, 1e6, device=dev)
    g = torch.Generator(device=dev).manual_seed(4)
    q = (torch.randn(B, H * nrep, n_tok, 128, generator=g, device=dev) / math.sqrt(128) * 4).half()
    mask = torch.full((n_tok, n_tok), float("-inf"), device=dev).triu_(1)[None, None].half()
    pos = torch.arange(n_tok, device=dev)[None]
    assert I._mask_is_causal(mask, pos[0], cache.get_all_positions())
    got = I._dense_attention(q, cache, cos, sin, nrep, 128, mask, q.dtype, pos)
    eager = I._dense_attention(q, cache, cos, sin, nrep, 128, mask, q.dtype, None)
    _close(got, eager.float())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_prefill_tcgen05_and_mma_kernels_agree(monkeypatch, dtype):
    """The tcgen05 kernel (SPX_PREFILL_PATH=tc: 128-token key tiles, S and O in tensor
    memory) and the mma.sync kernel (the default) on the same prompt, both against the
    float32 reference; causal, with a partial last query tile and a partial hot tile."""
    from unsloth_spectral import _ops
    from unsloth_spectral import synthetic as syn
    dev = torch.device("cuda")
    B, H, nrep, n_tok, Tq = 2, 4, 4, 1700, 300
    cache = _cache(B, H, n_tok, dtype, 32, 16, seed=11)
    cos, sin = syn.rope_tables(n_tok + 8, 128, 1e6, device=dev)
    q = (torch.randn(B, H * nrep, Tq, 128, generator=torch.Generator(device=dev).manual_seed(2), device=dev)
         / math.sqrt(128) * 4).to(dtype)
    q_pos = torch.arange(n_tok - Tq, n_tok, device=dev)
    ref = _reference(q, cache, cos, sin, q_pos, causal=True)
    mma = _ops.prefill(q, cache.tiers, cos, sin, q_pos, causal=True)
    monkeypatch.setenv("SPX_PREFILL_PATH", "tc")
    tc = _ops.prefill(q, cache.tiers, cos, sin, q_pos, causal=True)
    monkeypatch.delenv("SPX_PREFILL_PATH")
    _close(tc, ref)
    _close(mma, ref)
    _close(tc, mma.float())
