"""KV-head sharding of decode across ranks, checked on CPU with gloo ranks: each rank
takes its head slice with the product's sharding helpers (unsloth_spectral.sharding),
computes it with the oracle, and the product's HeadShardGather all-gathers and
reassembles the single-rank output exactly."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import spectral_oracle as so


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case(seed=0, H=4, nrep=2, D=32, T=32, nblk=3, k=8, hot=5):
    rng = np.random.default_rng(seed)
    codes_K = rng.integers(-127, 128, size=(nblk, H, T, k), dtype=np.int8)
    codes_V = rng.integers(-127, 128, size=(nblk, H, T, k), dtype=np.int8)
    scale = (rng.random((nblk, H)) * 0.01 + 0.01).astype(np.float32)
    basis = rng.standard_normal((nblk, H, k, D)).astype(np.float32) / math.sqrt(D)
    hot_K = rng.standard_normal((1, H, hot, D)).astype(np.float32)
    hot_V = rng.standard_normal((1, H, hot, D)).astype(np.float32)
    Q = rng.standard_normal((1, H * nrep, 1, D)).astype(np.float32)
    qpos = nblk * T + hot
    cos, sin = so.rope_tables(qpos + 4, D, 1e4)
    return dict(codes_K=codes_K, codes_V=codes_V, scale=scale, basis=basis, hot_K=hot_K, hot_V=hot_V, Q=Q,
                qpos=qpos, cos=cos, sin=sin, H=H, nrep=nrep, T=T, nblk=nblk, hot=hot)


def _decode_slice(c, h0, h1):
    """Oracle decode of KV heads [h0, h1) and their query heads."""
    nrep = c["nrep"]
    sl = slice(h0, h1)
    blocks = so.blocks_from_codes(c["codes_K"][:, sl], c["scale"][:, sl], c["basis"][:, sl], c["codes_V"][:, sl],
                                  c["scale"][:, sl], c["basis"][:, sl], np.arange(c["nblk"]) * c["T"])
    Q = c["Q"][:, h0 * nrep:h1 * nrep]
    hp = np.arange(c["nblk"] * c["T"], c["nblk"] * c["T"] + c["hot"])
    return so.spectral_attention_decode(Q, blocks, c["hot_K"][:, sl], c["hot_V"][:, sl], hp, c["cos"], c["sin"],
                                        c["qpos"])


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from unsloth_spectral.sharding import HeadShardGather, head_slice, shard_heads, shard_query_heads
        c = _case()
        h0, h1 = head_slice(c["H"], world, rank)
        # the product helpers pick this rank's slice of the cache and of the queries
        kv = torch.arange(c["H"]).view(1, c["H"])
        assert shard_heads(kv, world, rank).flatten().tolist() == list(range(h0, h1))
        qh = torch.arange(c["H"] * c["nrep"]).view(1, 1, -1)
        assert shard_query_heads(qh, c["H"], world, rank).flatten().tolist() == \
            list(range(h0 * c["nrep"], h1 * c["nrep"]))
        part = torch.from_numpy(_decode_slice(c, h0, h1))            # [1, Hl*nrep, 1, D]
        local = part.permute(2, 0, 1, 3).contiguous()                 # [L=1, B=1, Hl*nrep, D]
        g = HeadShardGather(local, world)
        g.start(local)
        g.wait()
        full = g.assembled()                                          # [1, 1, H*nrep, D]
        if rank == 0:
            q.put(full.permute(1, 2, 0, 3).numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_head_sharded_decode_reassembles_single_rank_output(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    c = _case()
    ref = _decode_slice(c, 0, c["H"])
    np.testing.assert_array_equal(out, ref.astype(np.float32))


def test_bench_shard_byte_accounting():
    """The per-rank algorithmic bytes of bench.py add up to the single-GPU figure."""
    import bench
    c = dict(bench.CFG)
    total = bench.algorithmic_bytes_per_step(c, c["kv_heads"])
    for world in (2, 4, 8):
        assert bench.algorithmic_bytes_per_step(c, c["kv_heads"] // world) * world == total
    assert abs(total - 26.06e9) < 0.01e9


def test_bench_rsvd_sweep_grid_and_roofline():
    """The config-3 sweep covers Nb {8, 128, 4096} x k {16, 32} x q {0, 2}, every Nb
    splits evenly over 1/2/4/8 ranks, and the rSVD roofline counts the algorithmic bytes
    (M read, sketch read, INT8 codes + FP16 basis + scale written) and product FLOPs."""
    import bench
    assert sorted(bench.SWEEP) == sorted((nb, k, q) for nb in (8, 128, 4096) for k in (16, 32) for q in (0, 2))
    assert all(nb % w == 0 for nb, _, _ in bench.SWEEP for w in (1, 2, 4, 8))
    r = bench.rsvd_roofline(4096, 32, 2, 1.0, (6502.2, 1658.6))
    per_block = 512 * 128 * 2 + 128 * 40 * 4 + 512 * 32 + 32 * 128 * 2 + 4
    assert r["algorithmic_bytes"] == 4096 * per_block
    assert r["product_flops"] == 4096 * 2.0 * 512 * 128 * 40 * 6
    assert abs(r["achieved"] - 4096 * per_block / 1e-3 / 1e9) < 1e-6
    assert r["bound"] == "hbm" and abs(r["frac"] - r["achieved"] / 6502.2) < 1e-12
