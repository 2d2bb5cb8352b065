"""Seeded synthetic workloads for the compressed-KV decode path.

K/V blocks are low-rank-plus-noise: ``X = A diag(sigma) G^T + N(0, noise^2)`` with
``A ~ N(0,1)[T, r]``, ``G ~ N(0,1)[D, r]`` and ``sigma_i = rho^i``.  Two seedings are
provided:

* ``kv_per_head`` -- one ``torch.Generator`` per (config, layer, batch row, KV head),
  seeded ``1_000_003*cfg + 10_007*layer + 101*b + h`` (V uses a separate stream).
  Used for the small parity cases, where every head must be reproducible on its own.
* ``kv_layer_batched`` -- one generator per (config, layer, tensor) drawing all
  (b, h) at once on the target device.  Same distribution; used for the large
  benchmark cases, where a per-head Python loop would dominate set-up time.

No public dataset is involved; everything is drawn from fixed seeds.
"""
from __future__ import annotations

import math

import torch

V_STREAM_OFFSET = 7_777_777


def head_seed(cfg: int, layer: int, b: int, h: int) -> int:
    return 1_000_003 * cfg + 10_007 * layer + 101 * b + h


def low_rank_block(gen: torch.Generator, T: int, D: int, rank: int, rho: float,
                   noise: float = 0.05) -> torch.Tensor:
    """One [T, D] float32 low-rank-plus-noise matrix drawn on the generator's device."""
    dev = gen.device
    A = torch.randn(T, rank, generator=gen, device=dev, dtype=torch.float32)
    G = torch.randn(D, rank, generator=gen, device=dev, dtype=torch.float32)
    sig = rho ** torch.arange(rank, device=dev, dtype=torch.float32)
    X = (A * sig) @ G.T
    X += noise * torch.randn(T, D, generator=gen, device=dev, dtype=torch.float32)
    return X


def kv_per_head(cfg: int, layer: int, B: int, H: int, T: int, D: int, rank: int, rho: float,
                noise: float = 0.05):
    """Pre-RoPE K and V ``[B, H, T, D]`` float32 on CPU, one generator per head."""
    K = torch.empty(B, H, T, D)
    V = torch.empty(B, H, T, D)
    for b in range(B):
        for h in range(H):
            s = head_seed(cfg, layer, b, h)
            K[b, h] = low_rank_block(torch.Generator().manual_seed(s), T, D, rank, rho, noise)
            V[b, h] = low_rank_block(torch.Generator().manual_seed(s + V_STREAM_OFFSET), T, D, rank,
                                     rho, noise)
    return K, V


def kv_layer_batched(cfg: int, layer: int, B: int, H: int, T: int, D: int, rank: int, rho: float,
                     device, dtype=torch.float16, noise: float = 0.05):
    """Pre-RoPE K and V ``[B, H, T, D]`` in ``dtype`` on ``device``, one generator per
    (layer, tensor); draws every (b, h) at once."""
    out = []
    for t, off in (("K", 0), ("V", V_STREAM_OFFSET)):
        gen = torch.Generator(device=device).manual_seed(head_seed(cfg, layer, 0, 0) + off)
        A = torch.randn(B, H, T, rank, generator=gen, device=device, dtype=torch.float32)
        G = torch.randn(B, H, D, rank, generator=gen, device=device, dtype=torch.float32)
        sig = rho ** torch.arange(rank, device=device, dtype=torch.float32)
        X = torch.matmul(A * sig, G.transpose(-1, -2))
        del A, G
        X += noise * torch.randn(B, H, T, D, generator=gen, device=device, dtype=torch.float32)
        out.append(X.to(dtype))
        del X
    return out[0], out[1]


def query(cfg: int, step: int, B: int, H_q: int, D: int, device="cpu") -> torch.Tensor:
    """Decode query ``Q ~ N(0,1)/sqrt(D)`` of shape ``[B, H_q, 1, D]`` (pre-RoPE)."""
    gen = torch.Generator(device=device).manual_seed(7 * step + cfg)
    return torch.randn(B, H_q, 1, D, generator=gen, device=device) / math.sqrt(D)


def rope_tables(seq_len: int, head_dim: int, theta: float = 1e6, device="cpu"):
    """HF half-split RoPE tables ``cat(freqs, freqs)`` as float32 ``[seq_len, D]``."""
    inv = theta ** (-2.0 * torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim)
    pos = torch.arange(seq_len, dtype=torch.float64)
    freqs = torch.outer(pos, inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().float().to(device), emb.sin().float().to(device)


def rope_rotate(x: torch.Tensor, cos_rows: torch.Tensor, sin_rows: torch.Tensor) -> torch.Tensor:
    """Half-split RoPE of ``x [..., D]`` with rows broadcast over the leading dims."""
    d = x.shape[-1] // 2
    x1, x2 = x[..., :d], x[..., d:]
    return torch.cat([x1 * cos_rows[..., :d] - x2 * sin_rows[..., :d],
                      x2 * cos_rows[..., d:] + x1 * sin_rows[..., d:]], dim=-1)
