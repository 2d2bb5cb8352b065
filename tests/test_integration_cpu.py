"""Host logic of the integration layer, no GPU: the recognition of causal additive masks
(so that the prompt kernel can apply the causal rule and skip future tiles) and the
layout of the in-repo Llama model that patch_unsloth_attention walks."""
import pytest
import torch


def test_mask_is_causal_recognises_the_causal_rule():
    from unsloth_spectral.integration import _mask_is_causal
    T = 40
    pos = torch.arange(T)
    for fill, dt in ((float("-inf"), torch.float32), (torch.finfo(torch.float16).min, torch.float16),
                     (torch.finfo(torch.bfloat16).min, torch.bfloat16)):
        m = torch.full((T, T), fill, dtype=torch.float32).triu_(1).to(dt)[None, None]
        assert _mask_is_causal(m, pos, pos)
    # queries at the end of a longer cache (a prompt appended to earlier tokens)
    q = torch.arange(30, 40)
    m = torch.where(pos[None, :] > q[:, None], float("-inf"), 0.0)[None, None]
    assert _mask_is_causal(m, q, pos)
    # not causal: a padding column, a finite penalty, a wrong shape
    bad = m.clone()
    bad[..., 0] = float("-inf")
    assert not _mask_is_causal(bad, q, pos)
    soft = torch.where(pos[None, :] > q[:, None], -10.0, 0.0)[None, None]
    assert not _mask_is_causal(soft, q, pos)
    assert not _mask_is_causal(m[..., :-1], q, pos)


def test_llama_layout_matches_what_the_patch_walks():
    from unsloth_spectral.llama_loop import MISTRAL_7B, LlamaShape, SpectralLlama
    assert (MISTRAL_7B.layers, MISTRAL_7B.hidden, MISTRAL_7B.heads, MISTRAL_7B.kv_heads, MISTRAL_7B.head_dim,
            MISTRAL_7B.ffn, MISTRAL_7B.vocab, MISTRAL_7B.rope_theta) == (32, 4096, 32, 8, 128, 14336, 32768, 1e6)
    s = LlamaShape(layers=2, hidden=64, heads=4, kv_heads=2, head_dim=16, ffn=96, vocab=50)
    m = SpectralLlama(s, device="cpu", dtype=torch.float32, seed=0)
    attn = m.model.layers[1].self_attn
    cfg = attn.config
    assert (cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.hidden_size, cfg.rope_theta) == (
        4, 2, 16, 64, 1e6)
    assert attn.q_proj.weight.shape == (64, 64) and attn.k_proj.weight.shape == (32, 64)
    assert m.lm_head.weight.shape == (50, 64) and m.model.embed_tokens.weight.shape == (50, 64)
    assert abs(float(attn.q_proj.weight.std()) - 0.02) < 0.005
    with pytest.raises(RuntimeError):
        attn(torch.zeros(1, 1, 64))


def test_attention_importance_and_landmarks_follow_the_reference_rules():
    """spectral_cache.py:710-852: the importance is an EMA (alpha 0.1) of the attention
    averaged over batch, heads and queries, grown with zero padding; block weights are
    slices of it; landmarks concatenate along the token axis and come first in
    get_kv_with_landmarks."""
    from unsloth_spectral import SpectralCache
    off = SpectralCache(2, 16, block_size=4, device="cpu", dtype=torch.float32)
    off.update_attention_importance(torch.rand(1, 2, 1, 8), 8)
    assert off.attention_importance is None and off.get_block_attention_weights(0) is None
    c = SpectralCache(2, 16, block_size=4, device="cpu", dtype=torch.float32, use_attention_weighted_svd=True)
    a1 = torch.rand(2, 2, 1, 6)
    c.update_attention_importance(a1, 6)
    m1 = a1.mean(dim=(0, 1, 2))
    assert torch.allclose(c.attention_importance, m1)
    a2 = torch.rand(2, 2, 1, 9)
    c.update_attention_importance(a2, 9)
    m2 = a2.mean(dim=(0, 1, 2))
    want = torch.cat([m1, torch.zeros(3)]) * 0.9 + 0.1 * m2
    assert torch.allclose(c.attention_importance, want)
    assert torch.allclose(c.get_block_attention_weights(1), want[4:8])
    assert c.get_block_attention_weights(2) is None   # tokens 8..11 not all tracked
    K1, V1 = torch.randn(1, 2, 3, 16), torch.randn(1, 2, 3, 16)
    K2, V2 = torch.randn(1, 2, 2, 16), torch.randn(1, 2, 2, 16)
    c.add_landmarks(K1, V1, torch.tensor([[0, 1, 2]]))
    c.add_landmarks(K2, V2, torch.tensor([[7, 9]]))
    K, V, P = c.get_kv_with_landmarks()
    assert torch.equal(K, torch.cat([K1, K2], 2)) and torch.equal(V, torch.cat([V1, V2], 2))
    assert P.tolist() == [[0, 1, 2, 7, 9]]
    c.reset()
    assert c.landmark_K is None and c.attention_importance is None and c.get_kv_with_landmarks() == (None, None, None)
