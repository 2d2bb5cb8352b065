"""CPU oracle for the compressed-KV decode path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import it.  The product path (``unsloth_spectral``) never imports
anything from ``oracle/`` and fails loudly when its CUDA library is missing.

It restates, in float32 numpy and op by op, the reference implementation of
nyssaleo/unsloth-spectral (paths below are relative to that project):

* ``quantize_int8_batched``   <- unsloth_spectral/spectral_cache.py:481-516
* ``batched_randomized_svd``  <- unsloth_spectral/rsvd.py:74-157
* ``compress_tensor``         <- unsloth_spectral/spectral_cache.py:345-407
* ``apply_rope_forward``      <- unsloth_spectral/spectral_attention.py:80-114
* ``apply_rope_kernels``      <- unsloth_spectral/kernels/spectral_attention.py:340-372
* ``spectral_attention_forward``  <- unsloth_spectral/spectral_attention.py:117-349
  (cold-tier RoPE indexed by the clamped *distance* query_position - key_position)
* ``spectral_attention_decode``   <- unsloth_spectral/kernels/spectral_attention.py:684-857
  with ``spectral_score_forward_pytorch`` (:375-453) and
  ``spectral_value_forward_pytorch`` (:544-601)
  (cold-tier RoPE indexed by the *absolute* key position)
* ``get_kv``                  <- unsloth_spectral/spectral_cache.py:557-612

Parity pin: ``tests/golden/make_golden.py`` imports the reference package itself
(only where it is mounted) and records its outputs on seeded inputs into
``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks this module against
those vectors.  The reference has no golden vectors of its own (its tests only print
shapes or thresholds), so the recorded outputs of the reference are the pin.

Cold blocks are passed in the layout the reference keeps (``SpectralBlock``):
``coeffs_K [H_kv, T_blk, k]`` (dequantised values), ``basis_K [H_kv, k, D]``, same for
V, and ``start_position``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

F32 = np.float32


# ---------------------------------------------------------------------------
# INT8 quantisation  (spectral_cache.py:481-516)
# ---------------------------------------------------------------------------
def quantize_int8_batched(C):
    """Per-leading-index symmetric INT8 quantisation.

    Returns ``(quantized, scales_minmax, codes, scale)``:
    ``quantized = round(C / scale) * scale`` (round half to even, IEEE float32
    division), ``scales_minmax [N, 2] = (min, max)`` as the reference stores them,
    plus the integer ``codes`` and the per-index ``scale = max(|C|max, 1e-8) / 127``
    that the reference uses but does not store.
    """
    C = np.asarray(C, dtype=F32)
    axes = tuple(range(1, C.ndim))
    t_min = C.min(axis=axes, keepdims=True)
    t_max = C.max(axis=axes, keepdims=True)
    abs_max = np.maximum(np.abs(C).max(axis=axes, keepdims=True), F32(1e-8))
    scale = (abs_max / F32(127.0)).astype(F32)
    codes = np.rint(C / scale).astype(F32)
    quantized = (codes * scale).astype(F32)
    scales = np.concatenate([t_min.reshape(C.shape[0], 1), t_max.reshape(C.shape[0], 1)], axis=1)
    return quantized, scales.astype(F32), codes.astype(np.int8), scale.reshape(C.shape[0])


def scale_from_minmax(scales_minmax):
    """Recover the quantisation scale from the stored (min, max): the reference's
    ``abs_max`` equals ``max(-min, max)`` (spectral_cache.py:497-505)."""
    mm = np.asarray(scales_minmax, dtype=F32)
    abs_max = np.maximum(np.maximum(-mm[:, 0], mm[:, 1]), F32(1e-8))
    return (abs_max / F32(127.0)).astype(F32)


# ---------------------------------------------------------------------------
# Randomised SVD  (rsvd.py:74-157)
# ---------------------------------------------------------------------------
def batched_randomized_svd(M, k: int, n_iter: int, oversampling: int, Omega=None,
                           dtype=np.float64):
    """Halko rSVD exactly as the reference orders it, with the Gaussian sketch
    ``Omega [B, n, r]`` supplied by the caller (the reference draws it from the
    torch global RNG at rsvd.py:95).

    ``dtype`` is the working precision.  The default, float64, evaluates the
    reference's algorithm essentially in exact arithmetic; that is the parity
    target, because the reference's own float32 run of the un-normalised power
    iterations (rsvd.py:111-113) loses the trailing subspace to rounding once the
    sketch is ill-conditioned (k=32, q=2 on the rank-48 generator: 0.0404 vs 0.0334
    relative error, the optimum being 0.0334).  Pass ``np.float32`` to reproduce the
    reference's float32 run.  Results are returned as float32."""
    M = np.asarray(M, dtype=dtype)
    B, m, n = M.shape
    r = min(k + oversampling, min(m, n))
    if r >= min(m, n) - 1:  # rsvd.py:84-87
        U, S, Vh = np.linalg.svd(M, full_matrices=False)
        return U[:, :, :k].astype(F32), S[:, :k].astype(F32), Vh[:, :k, :].astype(F32)
    Omega = np.asarray(Omega, dtype=dtype)
    assert Omega.shape == (B, n, r), (Omega.shape, (B, n, r))
    Y = np.matmul(M, Omega)                                   # :100
    Mt = np.ascontiguousarray(np.transpose(M, (0, 2, 1)))
    for _ in range(n_iter):                                   # :111-113
        Y = np.matmul(M, np.matmul(Mt, Y))
    Q, _ = np.linalg.qr(Y)                                    # :122 (Householder)
    Q = Q.astype(dtype)
    Bp = np.matmul(np.transpose(Q, (0, 2, 1)), M)             # :132
    Ut, S, Vh = np.linalg.svd(Bp, full_matrices=False)        # :141
    U = np.matmul(Q, Ut.astype(dtype))                        # :149
    return U[:, :, :k].astype(F32), S[:, :k].astype(F32), Vh[:, :k, :].astype(F32)


def relative_reconstruction_error(M, U, S, Vh):
    """Per-matrix ||M - U diag(S) Vh||_F / ||M||_F (float64 accumulation)."""
    M = np.asarray(M, dtype=np.float64)
    R = np.matmul(np.asarray(U, np.float64) * np.asarray(S, np.float64)[:, None, :], np.asarray(Vh, np.float64))
    num = np.sqrt(((M - R) ** 2).sum(axis=(1, 2)))
    den = np.sqrt((M ** 2).sum(axis=(1, 2)))
    return num / den


def compress_tensor(X, rank: int, Omega, n_iter: int = 2, oversampling: int = 5,
                    dtype=np.float64):
    """``SpectralCache._compress_tensor`` (spectral_cache.py:345-407) for one block
    ``X [H, T, D]``: rSVD, C = U*S, per-head INT8 quantisation.

    Returns ``(coeffs_dequantised [H,T,k], basis [H,k,D], scales_minmax [H,2],
    codes [H,T,k] int8, scale [H])`` in float32 (the reference then casts coeffs and
    basis to the model dtype)."""
    X = np.asarray(X, dtype=F32)
    U, S, Vh = batched_randomized_svd(X, rank, n_iter, oversampling, Omega, dtype=dtype)
    coeffs = (U * S[:, None, :]).astype(F32)                  # :387
    q, mm, codes, scale = quantize_int8_batched(coeffs)       # :398
    return q, Vh, mm, codes, scale


# ---------------------------------------------------------------------------
# RoPE helpers
# ---------------------------------------------------------------------------
def apply_rope_forward(x, cos, sin):
    """spectral_attention.py:80-114 -- uses the FIRST half of cos/sin for both halves."""
    d = x.shape[-1]
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    c1, s1 = cos[..., : d // 2], sin[..., : d // 2]
    return np.concatenate([x1 * c1 - x2 * s1, x2 * c1 + x1 * s1], axis=-1).astype(F32)


def apply_rope_kernels(x, cos, sin):
    """kernels/spectral_attention.py:340-366 -- second half uses cos/sin second half."""
    d = x.shape[-1]
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    c1, c2 = cos[..., : d // 2], cos[..., d // 2:]
    s1, s2 = sin[..., : d // 2], sin[..., d // 2:]
    return np.concatenate([x1 * c1 - x2 * s1, x2 * c2 + x1 * s2], axis=-1).astype(F32)


def rope_tables(seq_len: int, head_dim: int, theta: float = 1e6):
    """HF half-split RoPE tables ``cat(freqs, freqs)`` (same construction as the
    reference's test helper, test_phase1_simple.py:15-21), float32."""
    inv = theta ** (-2.0 * np.arange(0, head_dim, 2, dtype=np.float64) / head_dim)
    inv = inv.astype(F32)
    pos = np.arange(seq_len, dtype=F32)
    freqs = np.outer(pos, inv).astype(F32)
    emb = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(emb).astype(F32), np.sin(emb).astype(F32)


# ---------------------------------------------------------------------------
# Cache description
# ---------------------------------------------------------------------------
@dataclass
class Block:
    """One cold block in the reference's layout (spectral_cache.py:20-46)."""
    coeffs_K: np.ndarray   # [H_kv, T, k_K] dequantised
    basis_K: np.ndarray    # [H_kv, k_K, D]
    coeffs_V: np.ndarray   # [H_kv, T, k_V]
    basis_V: np.ndarray    # [H_kv, k_V, D]
    start_position: int

    @property
    def block_size(self) -> int:
        return int(self.coeffs_K.shape[1])


def _repeat_heads(x, n_rep):
    """repeat_kv_spectral (spectral_attention.py:50-77) / repeat_interleave
    (kernels/spectral_attention.py:428-432): q-head h reads KV head h // n_rep."""
    return np.repeat(x, n_rep, axis=0) if n_rep > 1 else x


def _softmax_f32(scores):
    m = np.max(scores, axis=-1, keepdims=True)
    e = np.exp((scores - m).astype(F32))
    return (e / e.sum(axis=-1, keepdims=True)).astype(F32)


def _decode(Q, blocks: Sequence[Block], hot_K, hot_V, hot_pos, cos, sin, query_position,
            attention_mask, scale, mode: str):
    Q = np.asarray(Q, dtype=F32)
    B, H_q, _, D = Q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if blocks:
        H_kv = blocks[0].coeffs_K.shape[0]
    elif hot_K is not None and hot_K.shape[2] > 0:
        H_kv = hot_K.shape[1]
    else:
        raise ValueError("Empty cache - no keys available")  # spectral_attention.py:277-278
    n_rep = H_q // H_kv
    cos = np.asarray(cos, dtype=F32)
    sin = np.asarray(sin, dtype=F32)
    parts = []
    for blk in blocks:
        T = blk.block_size
        ck = _repeat_heads(np.asarray(blk.coeffs_K, F32), n_rep)   # [H_q, T, k]
        bk = _repeat_heads(np.asarray(blk.basis_K, F32), n_rep)    # [H_q, k, D]
        key_pos = np.arange(blk.start_position, blk.start_position + T, dtype=np.int64)
        if mode == "distance":
            idx = np.clip(query_position - key_pos, 0, None)          # spectral_attention.py:198
            c, s = cos[idx][None, None], sin[idx][None, None]
            Qa = apply_rope_forward(np.broadcast_to(Q, (B, H_q, T, D)), c, -s)   # :212-219
        else:
            c, s = cos[key_pos][None, None], sin[key_pos][None, None]          # kernels :411-425
            Qa = apply_rope_kernels(np.broadcast_to(Q, (B, H_q, T, D)), c, -s)
        Ql = np.einsum("bhtd,hkd->bhtk", Qa, bk, dtype=F32)                      # :228-232
        sc = np.sum(Ql * ck[None], axis=-1, dtype=F32)                            # :236-237
        parts.append(sc[:, :, None, :])
    has_hot = hot_K is not None and hot_K.shape[2] > 0
    if has_hot:
        hk = np.asarray(hot_K, F32)
        hp = np.asarray(hot_pos, np.int64).reshape(-1)
        c, s = cos[hp][None, None], sin[hp][None, None]
        rope = apply_rope_forward if mode == "distance" else apply_rope_kernels
        hk_rot = np.repeat(rope(hk, c, s), n_rep, axis=1) if n_rep > 1 else rope(hk, c, s)
        parts.append(np.matmul(Q, hk_rot.transpose(0, 1, 3, 2)))                  # :273
    if not parts:
        raise ValueError("Empty cache - no keys available")
    scores = np.concatenate(parts, axis=-1).astype(F32) * F32(scale)
    if attention_mask is not None:
        scores = np.where(np.asarray(attention_mask) == 0, F32(-np.inf), scores)
    with np.errstate(invalid="ignore", over="ignore"):
        attn = _softmax_f32(scores)
    out = np.zeros((B, H_q, 1, D), dtype=F32)
    pos = 0
    for blk in blocks:
        T = blk.block_size
        cv = _repeat_heads(np.asarray(blk.coeffs_V, F32), n_rep)
        bv = _repeat_heads(np.asarray(blk.basis_V, F32), n_rep)
        a = attn[:, :, :, pos:pos + T]
        pos += T
        vp = np.matmul(a, cv[None])                                              # :322-323
        out += np.matmul(vp, bv[None])                                           # :327-328
    if has_hot:
        T = hot_V.shape[2]
        hv = np.repeat(np.asarray(hot_V, F32), n_rep, axis=1) if n_rep > 1 else np.asarray(hot_V, F32)
        out += np.matmul(attn[:, :, :, pos:pos + T], hv)                          # :343
    return out


def spectral_attention_forward(Q, blocks, hot_K, hot_V, hot_pos, cos, sin, query_position,
                               attention_mask=None, scale=None):
    """spectral_attention.py:117-349 in float32 (distance-indexed cold RoPE)."""
    return _decode(Q, blocks, hot_K, hot_V, hot_pos, cos, sin, query_position,
                   attention_mask, scale, "distance")


def spectral_attention_decode(Q, blocks, hot_K, hot_V, hot_pos, cos, sin, query_position,
                              attention_mask=None, scale=None):
    """kernels/spectral_attention.py:684-857 in float32 (absolute-indexed cold RoPE)."""
    return _decode(Q, blocks, hot_K, hot_V, hot_pos, cos, sin, query_position,
                   attention_mask, scale, "absolute")


def spectral_score_forward(Q, coeffs_K, basis_K, cos, sin, start_position):
    """kernels/spectral_attention.py:375-453: scores [B, H_q, 1, T] for one block."""
    Q = np.asarray(Q, F32)
    B, H_q, _, D = Q.shape
    H_kv, T, _ = coeffs_K.shape
    n_rep = H_q // H_kv
    kp = np.arange(start_position, start_position + T)
    Qa = apply_rope_kernels(np.broadcast_to(Q, (B, H_q, T, D)), cos[kp][None, None], -sin[kp][None, None])
    bk = _repeat_heads(np.asarray(basis_K, F32), n_rep)
    ck = _repeat_heads(np.asarray(coeffs_K, F32), n_rep)
    Ql = np.einsum("bhtd,hkd->bhtk", Qa, bk, dtype=F32)
    return np.sum(Ql * ck[None], axis=-1, dtype=F32)[:, :, None, :]


def spectral_value_forward(attn, coeffs_V, basis_V):
    """kernels/spectral_attention.py:544-601: (attn @ C_V) @ B_V per q-head."""
    attn = np.asarray(attn, F32)
    H_q = attn.shape[1]
    n_rep = H_q // coeffs_V.shape[0]
    cv = _repeat_heads(np.asarray(coeffs_V, F32), n_rep)
    bv = _repeat_heads(np.asarray(basis_V, F32), n_rep)
    return np.matmul(np.matmul(attn, cv[None]), bv[None])


def get_kv(blocks: List[Block], hot_K=None, hot_V=None):
    """spectral_cache.py:557-612 for batch 1: per block bmm(C, B), then hot; returns
    ``[1, H, T_total, D]`` pre-RoPE K and V, or (None, None) for an empty cache."""
    K_parts, V_parts = [], []
    for blk in blocks:
        K_parts.append(np.matmul(np.asarray(blk.coeffs_K, F32), np.asarray(blk.basis_K, F32))[None])
        V_parts.append(np.matmul(np.asarray(blk.coeffs_V, F32), np.asarray(blk.basis_V, F32))[None])
    if hot_K is not None:
        K_parts.append(np.asarray(hot_K, F32))
        V_parts.append(np.asarray(hot_V, F32))
    if not K_parts:
        return None, None
    return np.concatenate(K_parts, axis=2), np.concatenate(V_parts, axis=2)


def blocks_from_codes(codes_K, scale_K, basis_K, codes_V, scale_V, basis_V, start_positions):
    """Build reference-layout blocks from integer codes ``[nblk, H, T, k]`` and
    per-(block, head) scales ``[nblk, H]``: coeffs = codes * scale, as the reference
    stores them (spectral_cache.py:508)."""
    out = []
    for j, p0 in enumerate(start_positions):
        ck = (codes_K[j].astype(F32) * np.asarray(scale_K[j], F32)[:, None, None]).astype(F32)
        cv = (codes_V[j].astype(F32) * np.asarray(scale_V[j], F32)[:, None, None]).astype(F32)
        out.append(Block(ck, np.asarray(basis_K[j], F32), cv, np.asarray(basis_V[j], F32), int(p0)))
    return out
