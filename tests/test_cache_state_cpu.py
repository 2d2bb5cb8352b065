"""SpectralCache.state_dict / load_state_dict on the CPU: a filled cache (cold tier set
from integer codes, hot tier, counters) survives a torch.save / torch.load round trip
into a fresh cache, and a cache of another geometry refuses the state."""
import io

import pytest
import torch

from unsloth_spectral import SpectralCache

B, H, T, D, NB, HOT = 2, 4, 128, 64, 3, 37


def _filled(seed: int) -> SpectralCache:
    g = torch.Generator().manual_seed(seed)
    cache = SpectralCache(H, D, block_size=T, k_rank_keys=16, k_rank_values=16, device="cpu",
                          dtype=torch.float16)
    codes = lambda: torch.randint(-127, 128, (B, H, NB, T, 16), generator=g).to(torch.int8)
    scale = lambda: torch.rand(B, H, NB, generator=g) * 0.02 + 0.001
    basis = lambda: torch.randn(B, H, NB, 16, D, generator=g)
    mm = lambda: torch.randn(B, H, NB, 2, generator=g)
    cache.set_cold(codes(), scale(), basis(), codes(), scale(), basis(), [i * T for i in range(NB)],
                   minmax_K=mm(), minmax_V=mm())
    cache.set_hot(torch.randn(B, H, HOT, D, generator=g).half(), torch.randn(B, H, HOT, D, generator=g).half(),
                  torch.arange(NB * T, NB * T + HOT))
    cache.current_position = cache.total_tokens = NB * T + HOT
    cache.compression_count = NB
    return cache


def test_state_dict_round_trip():
    src = _filled(3)
    buf = io.BytesIO()
    torch.save(src.state_dict(), buf)
    buf.seek(0)
    dst = SpectralCache(H, D, block_size=T, k_rank_keys=16, k_rank_values=16, device="cpu", dtype=torch.float16)
    dst.load_state_dict(torch.load(buf))
    a, b = src.tiers, dst.tiers
    assert b.num_blocks == NB and b.hot_len == HOT
    for name in SpectralCache._COLD:
        assert torch.equal(getattr(a, name)[:, :, :NB], getattr(b, name)[:, :, :NB]), name
    assert torch.equal(a.block_pos[:NB], b.block_pos[:NB])
    assert torch.equal(src.hot_K, dst.hot_K) and torch.equal(src.hot_V, dst.hot_V)
    assert torch.equal(src.hot_position_ids, dst.hot_position_ids)
    assert (dst.current_position, dst.total_tokens, dst.compression_count) == (NB * T + HOT, NB * T + HOT, NB)


def test_state_dict_replaces_contents_and_batch():
    dst = _filled(4)
    src = SpectralCache(H, D, block_size=T, k_rank_keys=16, k_rank_values=16, device="cpu", dtype=torch.float16)
    src.set_hot(torch.ones(1, H, 5, D).half(), torch.ones(1, H, 5, D).half(), torch.arange(5))
    dst.load_state_dict(src.state_dict())
    assert dst.tiers.batch == 1 and dst.num_cold_blocks == 0 and dst.hot_len == 5


@pytest.mark.parametrize("field,value", [("head_dim", 128), ("block_size", 256), ("k_rank_values", 32)])
def test_state_dict_geometry_mismatch(field, value):
    sd = _filled(5).state_dict()
    kw = dict(block_size=T, k_rank_keys=16, k_rank_values=16)
    args = [H, D]
    if field == "head_dim":
        args[1] = value
    else:
        kw[field] = value
    other = SpectralCache(*args, device="cpu", dtype=torch.float16, **kw)
    with pytest.raises(ValueError):
        other.load_state_dict(sd)
