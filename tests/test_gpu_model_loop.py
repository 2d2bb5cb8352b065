"""The in-repo greedy token loop (unsloth_spectral.llama_loop) on a reduced
Llama-architecture model patched with ``patch_unsloth_attention``: the prompt runs
through the patched prefill forward (compression of its full blocks), every new token
through the patched single-token forward (spectral decode kernel).  Checks: the loop is
deterministic for a seeded sketch generator (a second generation resets the caches as a
new generation must, spectral_cache.py:176-186), cache statistics count every prompt and
generated token, and a decode step after warm-up makes no host-device synchronisation."""
import pytest
import torch

from conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_greedy_loop_through_patched_layers(dtype):
    from unsloth_spectral import get_cache_stats
    from unsloth_spectral.llama_loop import LlamaShape, SpectralLlama
    dev = torch.device("cuda")
    shape = LlamaShape(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, ffn=1024, vocab=1000)
    model = SpectralLlama(shape, device=dev, dtype=dtype, seed=3)
    model.patch(block_size=512, k_rank_keys=16, k_rank_values=16, hot_buffer_size=64)
    B, T, NEW = 2, 600, 12
    prompt = torch.randint(0, shape.vocab, (B, T), generator=torch.Generator(device=dev).manual_seed(4), device=dev)
    # the rSVD sketch comes from the global generator (rsvd.py:95): seed it for each run
    torch.manual_seed(11)
    a = model.generate(prompt, NEW)
    torch.manual_seed(11)
    b = model.generate(prompt, NEW)
    assert a.shape == (B, NEW) and a.dtype == torch.long
    assert int(a.min()) >= 0 and int(a.max()) < shape.vocab
    assert torch.equal(a, b)
    st = get_cache_stats(model)
    assert st["layers_with_cache"] == 2
    assert st["total_tokens"] == 2 * (T + NEW - 1)
    assert st["total_blocks"] == 2
    for cache in model._caches:
        assert cache.num_cold_blocks == 1 and cache.hot_len == T + NEW - 1 - 512


def test_decode_step_has_no_host_sync():
    from unsloth_spectral.llama_loop import LlamaShape, SpectralLlama
    dev = torch.device("cuda")
    shape = LlamaShape(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, ffn=1024, vocab=1000)
    model = SpectralLlama(shape, device=dev, dtype=torch.float16, seed=5)
    model.patch(block_size=512, k_rank_keys=16, k_rank_values=16, hot_buffer_size=64)
    prompt = torch.randint(0, shape.vocab, (2, 560), generator=torch.Generator(device=dev).manual_seed(6), device=dev)
    with torch.no_grad():
        logits, caches = model.prefill(prompt)
        tok = logits.argmax(-1)
        pos = torch.full((1, 1), 560, dtype=torch.long, device=dev)
        logits = model.decode_step(tok, pos, caches)   # warm: RoPE tables and frequencies cached
        tok = logits.argmax(-1)
        pos += 1
        torch.cuda.synchronize()
        torch.cuda.set_sync_debug_mode("error")
        try:
            logits = model.decode_step(tok, pos, caches)
        finally:
            torch.cuda.set_sync_debug_mode("default")
        torch.cuda.synchronize()
    assert torch.isfinite(logits.float()).all()


def test_cuda_graph_decode_matches_eager():
    """The decode loop replayed from CUDA graphs (hot tier grown through its device
    length, one capture per segment between block compressions) produces exactly the
    eager loop's tokens and cache state, across a compression (600-token prompt: 88 hot
    tokens after the prefill, the 424th new token fills a block)."""
    from unsloth_spectral.llama_loop import LlamaShape, SpectralLlama
    dev = torch.device("cuda")
    shape = LlamaShape(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, ffn=1024, vocab=1000)
    model = SpectralLlama(shape, device=dev, dtype=torch.float16, seed=8)
    model.patch(block_size=512, k_rank_keys=16, k_rank_values=16, hot_buffer_size=64)
    prompt = torch.randint(0, shape.vocab, (2, 600), generator=torch.Generator(device=dev).manual_seed(9), device=dev)
    torch.manual_seed(12)
    eager = model.generate(prompt, 480)
    st_e = [(c.total_tokens, c.num_cold_blocks, c.hot_len) for c in model._caches]
    hot_e = model._caches[1].hot_K.clone()
    torch.manual_seed(12)
    graphed = model.generate(prompt, 480, cuda_graphs=True)
    st_g = [(c.total_tokens, c.num_cold_blocks, c.hot_len) for c in model._caches]
    assert st_e == st_g == [(600 + 479, 2, 600 + 479 - 1024)] * 2
    assert torch.equal(eager, graphed)
    assert torch.equal(hot_e, model._caches[1].hot_K)
    assert int(model._caches[0].tiers.hot_len_device()) == model._caches[0].hot_len
