"""spx_decode_attn_noalloc: the decode entry point for callers that cannot allocate
device memory (e.g. an FFI host with no CUDA allocator of its own, or a serving loop that
must not call cudaMalloc/cudaFree on the decode path).  Its scratch is a fixed array
inside the library, so these tests call it through the C ABI with no workspace and
compare it with spx_decode_attn, which uses a caller-provided workspace.

This file is named to be collected last: the entry point's scratch array stays reserved
on the device for the rest of the process."""
import numpy as np
import pytest
import torch

from conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


def _cache_and_inputs(seed):
    """A small FP16 cache (3 cold blocks at k=32 + 40 hot tokens, 8 KV / 32 query heads)."""
    from unsloth_spectral import SpectralCache
    from unsloth_spectral import synthetic as syn
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(seed)
    B, H, Hq, D, T, nb, k, hot = 2, 8, 32, 128, 512, 3, 32, 40
    cache = SpectralCache(H, D, block_size=T, k_rank_keys=k, k_rank_values=k, device=dev, dtype=torch.float16)
    codes = lambda: torch.randint(-127, 128, (B, H, nb, T, k), generator=g, dtype=torch.int8).to(dev)
    scale = lambda: (torch.rand(B, H, nb, generator=g) * 0.02 + 0.005).to(dev)
    basis = lambda: torch.linalg.qr(torch.randn(B, H, nb, D, k, generator=g))[0].transpose(-1, -2).to(dev)
    cache.set_cold(codes(), scale(), basis(), codes(), scale(), basis(), [i * T for i in range(nb)])
    cache.set_hot(torch.randn(B, H, hot, D, generator=g).half().to(dev),
                  torch.randn(B, H, hot, D, generator=g).half().to(dev))
    qpos = nb * T + hot
    cos, sin = syn.rope_tables(qpos + 8, D, 1e6, device=dev)
    return cache, cos, sin, qpos, B, Hq, D, g


def _close(out, ref):
    a = out.double().flatten()
    b = ref.double().flatten()
    cosv = float(a @ b / (a.norm() * b.norm()))
    assert cosv >= 0.9999, cosv
    assert float((a - b).abs().max()) <= 1e-2


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    from unsloth_spectral import _native as N, _ops
    cache, cos, sin, qpos, B, Hq, D, g = _cache_and_inputs(3)
    dev = torch.device("cuda")
    lib = N.lib_for(dev)
    stream = N.stream_handle(dev)
    for call in range(2):   # two calls in a row: the shared scratch keeps the previous contents
        q = (torch.randn(1, B, Hq, D, generator=g) / D ** 0.5).half().to(dev)
        ref = _ops.decode(q, cache.tiers, cos, sin, qpos, rope_mode=N.SPX_ROPE_ABSOLUTE)
        args, out, keep = _ops.decode_args(q, cache.tiers, cos, sin, qpos, rope_mode=N.SPX_ROPE_ABSOLUTE)
        args.workspace, args.workspace_bytes = None, 0
        rc = lib.spx_decode_attn_noalloc(args, stream)
        assert rc == N.SPX_OK, lib.spx_last_error()
        torch.cuda.synchronize()
        _close(out, ref)
        assert torch.isfinite(out).all()
        del keep


def test_noalloc_rejects_requests_beyond_its_scratch():
    from unsloth_spectral import _native as N, _ops
    cache, cos, sin, qpos, B, Hq, D, g = _cache_and_inputs(4)
    dev = torch.device("cuda")
    lib = N.lib_for(dev)
    q = torch.zeros(1, B, Hq, D, dtype=torch.float16, device=dev)
    args, out, keep = _ops.decode_args(q, cache.tiers, cos, sin, qpos, rope_mode=N.SPX_ROPE_ABSOLUTE)
    args.num_layers = 4096          # scratch need far above the built-in array (nothing launches)
    assert lib.spx_decode_workspace_size(args) > N.NOALLOC_SCRATCH_BYTES
    assert lib.spx_decode_attn_noalloc(args, N.stream_handle(dev)) == N.SPX_ERR_WORKSPACE
    assert b"scratch" in lib.spx_last_error()
