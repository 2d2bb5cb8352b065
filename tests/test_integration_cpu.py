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
