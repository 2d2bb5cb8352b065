"""The integration layer (the callers of the decode path) on the GPU: an HF-shaped
Llama attention stack patched with ``patch_unsloth_attention`` (integration.py:728),
prefilled with a prompt that fills two compression blocks, then decoded token by token
through both patched entry points:

* ``self_attn.forward`` -- the per-layer replacement (integration.py:43-425): dense
  attention over the reconstructed cache for the prompt, ``spectral_attention_forward``
  (distance-indexed cold RoPE) for single decode tokens;
* ``self_attn._spx_inference`` -- Unsloth's single-token decode signature
  (integration.py:481-725), routed to ``kernels.spectral_attention_decode``
  (absolute-indexed cold RoPE) as the reference routes it when its kernels load.

Every decode output is compared with the float32 oracle evaluated over the very cache
the layer holds, followed by the same output projection; ``get_cache_stats``
(integration.py:892-938) is checked against the caches' own statistics; and a decode
step with device position ids runs without a host-device synchronisation."""
import math
from types import SimpleNamespace

import pytest
import torch

from conftest import cuda_ok
from oracle import spectral_oracle as so

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

COS_MIN, ABS_MAX = 0.9999, 1e-2


class ToyAttention(torch.nn.Module):
    """The attributes the patched forwards read from an HF Llama attention module."""

    def __init__(self, hidden, nh, nkv, hd, theta, gen):
        super().__init__()
        self.config = SimpleNamespace(num_attention_heads=nh, num_key_value_heads=nkv, head_dim=hd, hidden_size=hidden,
                                      rope_theta=theta)
        self.head_dim = hd
        mk = lambda o, i: torch.nn.Parameter(torch.randn(o, i, generator=gen) * (1.0 / math.sqrt(i)))
        self.q_proj = torch.nn.Linear(hidden, nh * hd, bias=False)
        self.k_proj = torch.nn.Linear(hidden, nkv * hd, bias=False)
        self.v_proj = torch.nn.Linear(hidden, nkv * hd, bias=False)
        self.o_proj = torch.nn.Linear(nh * hd, hidden, bias=False)
        self.q_proj.weight, self.k_proj.weight = mk(nh * hd, hidden), mk(nkv * hd, hidden)
        self.v_proj.weight, self.o_proj.weight = mk(nkv * hd, hidden), mk(hidden, nh * hd)


class ToyModel(torch.nn.Module):
    def __init__(self, layers, **kw):
        super().__init__()
        gen = torch.Generator().manual_seed(5)
        self.model = SimpleNamespace(layers=[SimpleNamespace(self_attn=ToyAttention(gen=gen, **kw))
                                             for _ in range(layers)])


def _rope(x, cos, sin):
    h = x.shape[-1] // 2
    return torch.cat([x[..., :h] * cos[..., :h] - x[..., h:] * sin[..., :h],
                      x[..., h:] * cos[..., :h] + x[..., :h] * sin[..., :h]], dim=-1)


def _expected(attn, cache, x, qpos, mode):
    """The layer's decode output from the oracle over the cache the layer holds: the
    query projected and RoPE'd exactly as the patched forward does, attention by the
    float32 restatement of the reference, then the output projection."""
    from unsloth_spectral.integration import rope_tables_for
    nh, hd = attn.config.num_attention_heads, attn.head_dim
    cos, sin = rope_tables_for(attn, qpos + 2, x.device)
    q = attn.q_proj(x).view(1, 1, nh, hd).transpose(1, 2)
    q = _rope(q.float(), cos[qpos], sin[qpos]).to(q.dtype)
    blocks = [so.Block(b.coeffs_K.float().cpu().numpy(), b.basis_K.float().cpu().numpy(),
                       b.coeffs_V.float().cpu().numpy(), b.basis_V.float().cpu().numpy(), b.start_position)
              for b in cache.cold_blocks]
    fn = so.spectral_attention_forward if mode == "forward" else so.spectral_attention_decode
    out = fn(q.float().cpu().numpy(), blocks, cache.hot_K.float().cpu().numpy(), cache.hot_V.float().cpu().numpy(),
             cache.hot_position_ids.cpu().numpy(), cos.cpu().numpy(), sin.cpu().numpy(), qpos,
             scale=1.0 / math.sqrt(hd))
    o = torch.from_numpy(out).to(x.device).to(x.dtype).transpose(1, 2).reshape(1, 1, nh * hd)
    return attn.o_proj(o).float()


def _close(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    c = float(a @ b / (a.norm() * b.norm()))
    assert c >= COS_MIN, c
    assert float((a - b).abs().max()) <= ABS_MAX * max(1.0, float(b.abs().max())), float((a - b).abs().max())


@pytest.mark.parametrize("entry", ["forward", "inference"])
def test_patched_attention_prefill_then_decode_matches_oracle(entry):
    from unsloth_spectral import SpectralCache, get_cache_stats, patch_unsloth_attention
    dev = torch.device("cuda")
    torch.manual_seed(0)
    hidden, nh, nkv, hd = 512, 32, 8, 128
    model = ToyModel(2, hidden=hidden, nh=nh, nkv=nkv, hd=hd, theta=1e6)
    for layer in model.model.layers:
        layer.self_attn.to(dev, torch.float16)
    patch_unsloth_attention(model, block_size=512, k_rank_keys=16, k_rank_values=16, verbose=False)
    gen = torch.Generator(device=dev).manual_seed(1)
    T0 = 1100
    x = torch.randn(1, T0, hidden, generator=gen, device=dev).half() * 0.5
    caches = []
    with torch.no_grad():
        for layer in model.model.layers:
            out, _, cache = layer.self_attn.forward(x, position_ids=torch.arange(T0, device=dev)[None], use_cache=True)
            assert out.shape == (1, T0, hidden) and torch.isfinite(out).all()
            assert isinstance(cache, SpectralCache) and cache.num_cold_blocks == 2 and cache.hot_len == T0 - 1024
            caches.append(cache)
        for step in range(8):
            qpos = T0 + step
            xt = torch.randn(1, 1, hidden, generator=gen, device=dev).half() * 0.5
            for li, layer in enumerate(model.model.layers):
                attn = layer.self_attn
                pid = torch.tensor([[qpos]], device=dev)
                if entry == "forward":
                    got, _, c = attn.forward(xt, position_ids=pid, past_key_value=caches[li], use_cache=True)
                else:
                    got, c = attn._spx_inference(xt, caches[li], pid)
                assert c is caches[li] and c.total_tokens == qpos + 1
                mode = "forward" if entry == "forward" else "decode"
                _close(got.float(), _expected(attn, c, xt, qpos, mode))
    stats = get_cache_stats(model)
    per = [c.get_memory_stats() for c in caches]
    # the prefill stored each layer's cache on the module; both entry points extend it in place
    assert stats["layers_with_cache"] == 2
    assert stats["total_tokens"] == sum(s["total_tokens"] for s in per) == 2 * (T0 + 8)
    assert stats["total_blocks"] == sum(s["num_blocks"] for s in per) == 4
    assert stats["total_original_bytes"] == sum(s["original_bytes"] for s in per)
    assert stats["total_compressed_bytes"] == sum(s["compressed_bytes"] for s in per)
    assert stats["compression_ratio"] == pytest.approx(stats["total_original_bytes"] / stats["total_compressed_bytes"])
    assert [p["layer_idx"] for p in stats["per_layer_stats"]] == [0, 1]


def test_decode_step_with_device_positions_does_not_synchronise():
    """One single-token decode through the patched inference entry point, after a warm
    call (which builds and caches the RoPE tables and their frequencies), runs with
    torch's sync debug mode set to raise on any device-to-host synchronisation."""
    from unsloth_spectral import patch_unsloth_attention
    dev = torch.device("cuda")
    hidden, nh, nkv, hd = 512, 32, 8, 128
    model = ToyModel(1, hidden=hidden, nh=nh, nkv=nkv, hd=hd, theta=1e6)
    attn = model.model.layers[0].self_attn
    attn.to(dev, torch.float16)
    patch_unsloth_attention(model, block_size=512, k_rank_keys=16, k_rank_values=16, verbose=False)
    gen = torch.Generator(device=dev).manual_seed(2)
    with torch.no_grad():
        x = torch.randn(1, 600, hidden, generator=gen, device=dev).half() * 0.5
        _, _, cache = attn.forward(x, position_ids=torch.arange(600, device=dev)[None], use_cache=True)
        for step in range(3):
            xt = torch.randn(1, 1, hidden, generator=gen, device=dev).half() * 0.5
            pid = torch.tensor([[600 + step]], device=dev)
            if step == 2:
                torch.cuda.synchronize()
                torch.cuda.set_sync_debug_mode("error")
            try:
                out, cache = attn._spx_inference(xt, cache, pid)
            finally:
                torch.cuda.set_sync_debug_mode("default")
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()


def test_get_kv_with_landmarks_on_a_compressed_cache():
    """Landmarks first, then the reconstructed cold blocks and the hot tier, with their
    positions (spectral_cache.py:808-852)."""
    from unsloth_spectral import SpectralCache
    from unsloth_spectral import synthetic as syn
    dev = torch.device("cuda")
    K, V = syn.kv_layer_batched(1, 3, 1, 4, 600, 128, 24, 0.85, dev)
    c = SpectralCache(4, 128, block_size=512, k_rank_keys=16, k_rank_values=16, device=dev, dtype=torch.float16)
    c.append(K, V, torch.arange(600, device=dev)[None])
    lk, lv = K[:, :, :5].clone(), V[:, :, :5].clone()
    c.add_landmarks(lk, lv, torch.arange(5, device=dev)[None])
    Kw, Vw, P = c.get_kv_with_landmarks()
    Kc, Vc = c.get_kv()
    assert torch.equal(Kw, torch.cat([lk, Kc], 2)) and torch.equal(Vw, torch.cat([lv, Vc], 2))
    assert P.shape == (1, 605) and P[0, :5].tolist() == list(range(5)) and P[0, 5:].tolist() == list(range(600))
