"""Spectral decode attention over the three-tier cache.

``spectral_attention_forward`` keeps the reference's signature and semantics
(unsloth_spectral/spectral_attention.py:117-349): cold-tier RoPE indexed by the
clamped distance ``query_position - key_position``, hot tier RoPE'd at absolute
positions, keep-mask (``mask == 0`` -> -inf), float32 softmax, output in ``Q.dtype``.
The whole computation is one ``spx_decode_attn`` call (fused CUDA kernels); nothing
here has a CPU path.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import _native as N
from . import _ops
from .spectral_cache import SpectralBlock, SpectralCache


def repeat_kv(hidden_states: torch.Tensor, n_rep: int) -> torch.Tensor:
    """``[B, H_kv, T, D]`` -> ``[B, H_kv * n_rep, T, D]``; q-head h reads KV head h // n_rep."""
    if n_rep == 1:
        return hidden_states
    return torch.repeat_interleave(hidden_states, n_rep, dim=1)


def repeat_kv_spectral(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """``[H_kv, ...]`` -> ``[H_kv * n_rep, ...]`` with the same head mapping."""
    if n_rep == 1:
        return x
    return torch.repeat_interleave(x, n_rep, dim=0)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Half-split RoPE using the first half of ``cos``/``sin`` for both halves
    (the convention of spectral_attention.py:80-114)."""
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    c, s = cos[..., :h], sin[..., :h]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def _as_device_cache(cache, device) -> SpectralCache:
    """Copy a reference-style cache (``cold_blocks`` list + hot tensors) into device tiers."""
    blocks = list(getattr(cache, "cold_blocks", []) or [])
    hot_K = getattr(cache, "hot_K", None)
    dtype = blocks[0].basis_K.dtype if blocks else (hot_K.dtype if hot_K is not None else torch.float16)
    if blocks:
        kK, kV, T = blocks[0].coeffs_K.shape[-1], blocks[0].coeffs_V.shape[-1], blocks[0].block_size
    else:
        kK, kV, T = 16, 16, getattr(cache, "block_size", 512)
    dc = SpectralCache(cache.num_heads, cache.head_dim, block_size=T, k_rank_keys=kK, k_rank_values=kV,
                       device=device, dtype=dtype)
    if blocks:
        dc.cold_blocks = [SpectralBlock(b.coeffs_K.to(device), b.basis_K.to(device), b.coeffs_V.to(device),
                                        b.basis_V.to(device), b.scales_K.to(device), b.scales_V.to(device),
                                        b.block_size, b.start_position) for b in blocks]
    if hot_K is not None and hot_K.shape[2] > 0:
        hp = getattr(cache, "hot_position_ids", None)
        dc.set_hot(hot_K.to(device), cache.hot_V.to(device), None if hp is None else hp.to(device))
    return dc


def spectral_decode(Q: torch.Tensor, cache, cos: torch.Tensor, sin: torch.Tensor, query_position: int,
                    attention_mask: Optional[torch.Tensor], scale: Optional[float], rope_mode: int) -> torch.Tensor:
    """One fused decode over ``cache`` for ``Q [B, H_q, 1, D]`` (already RoPE'd)."""
    if not isinstance(cache, SpectralCache):
        cache = _as_device_cache(cache, Q.device)
    t = cache.tiers
    if t is None or (t.num_blocks == 0 and t.hot_len == 0):
        raise ValueError("Empty cache - no keys available")
    B, Hq, Tq, D = Q.shape
    if Tq != 1:
        raise ValueError(f"decode attention takes one query token, got {Tq}")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    q = Q.reshape(1, B, Hq, D).to(device=t.device, dtype=cache.dtype).contiguous()
    out = _ops.decode(q, t, cos, sin, int(query_position), rope_mode=rope_mode, mask=attention_mask, scale=scale)
    return out.reshape(B, Hq, 1, D).to(Q.dtype)


def spectral_attention_forward(Q: torch.Tensor, cache, cos: torch.Tensor, sin: torch.Tensor, query_position: int,
                               attention_mask: Optional[torch.Tensor] = None,
                               scale: Optional[float] = None) -> torch.Tensor:
    """Decode attention with distance-indexed cold-tier RoPE
    (spectral_attention.py:117-349).  Returns ``[B, H_q, 1, D]`` in ``Q.dtype``."""
    return spectral_decode(Q, cache, cos, sin, query_position, attention_mask, scale, N.SPX_ROPE_DISTANCE)


def validate_spectral_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, cache, rtol: float = 1e-2,
                                atol: float = 1e-2, cos: Optional[torch.Tensor] = None,
                                sin: Optional[torch.Tensor] = None,
                                query_position: Optional[int] = None) -> Tuple[bool, dict]:
    """Compare spectral attention with dense attention on the uncompressed K/V
    (spectral_attention.py:352-414).  The reference calls the attention without RoPE
    tables and crashes; here identity tables are used unless ``cos``/``sin`` are given,
    which is the comparison the reference intends."""
    B, H, _, D = Q.shape
    scale = 1.0 / math.sqrt(D)
    T = K.shape[2]
    if cos is None:
        cos = torch.ones(T + 1, D, device=Q.device)
        sin = torch.zeros(T + 1, D, device=Q.device)
    qpos = T if query_position is None else query_position
    n_rep = H // K.shape[1]
    Kr, Vr = repeat_kv(K, n_rep), repeat_kv(V, n_rep)
    s_ref = torch.matmul(Q.float(), Kr.float().transpose(-2, -1)) * scale
    out_ref = torch.matmul(torch.softmax(s_ref, dim=-1), Vr.float())
    out = spectral_attention_forward(Q, cache, cos, sin, qpos, scale=scale).float()
    abs_err = (out_ref - out).abs().max().item()
    rel_err = abs_err / (out_ref.abs().max().item() + 1e-8)
    Krec, _ = (cache.get_kv() if isinstance(cache, SpectralCache) else _as_device_cache(cache, Q.device).get_kv())
    s_sp = torch.matmul(Q.float(), repeat_kv(Krec, n_rep).float().transpose(-2, -1)) * scale
    corr = torch.corrcoef(torch.stack([s_ref.flatten(), s_sp.flatten()]))[0, 1].item()
    ok = (abs_err < atol) or (rel_err < rtol)
    return ok, {"max_abs_error": abs_err, "max_rel_error": rel_err,
                "mean_abs_error": (out_ref - out).abs().mean().item(), "attention_correlation": corr,
                "is_valid": ok}
