"""Decode-attention entry points of the reference's ``kernels`` module, backed by the
sm_100a library instead of Triton (unsloth_spectral/kernels/spectral_attention.py).

* ``spectral_attention_decode`` (:684-857): cold-tier RoPE at ABSOLUTE key positions,
  hot tier at absolute positions, keep-mask, float32 softmax -- one fused launch.
* ``spectral_score_forward`` (:456-541) / ``spectral_value_forward`` (:604-677): the
  per-block helpers, on float coefficients.
* ``TritonSpectralConfig`` (:50-64): accepted for compatibility; tile fields do not
  apply to these kernels, ``enable_logging`` turns on debug logging.
"""
from __future__ import annotations

import logging
import math
from dataclasses import dataclass
from typing import Optional

import torch

from .. import _native as N
from .. import _ops
from ..spectral_attention import spectral_attention_forward, spectral_decode

logger = logging.getLogger("unsloth_spectral.kernels.spectral_attention")


@dataclass
class TritonSpectralConfig:
    """Kernel configuration kept for API compatibility (same fields and checks)."""
    BLOCK_T: int = 64
    BLOCK_K: int = 32
    BLOCK_D: int = 64
    num_warps: int = 4
    num_stages: int = 2
    enable_logging: bool = True

    def __post_init__(self):
        assert self.BLOCK_T >= 16, "BLOCK_T must be at least 16"
        assert self.BLOCK_K >= 8, "BLOCK_K must be at least 8"
        assert self.BLOCK_D >= 32, "BLOCK_D must be at least 32"


def spectral_score_forward(Q: torch.Tensor, coeffs_K: torch.Tensor, basis_K: torch.Tensor, cos: torch.Tensor,
                           sin: torch.Tensor, start_position: int, query_position: int,
                           config: Optional[TritonSpectralConfig] = None, use_triton: bool = False) -> torch.Tensor:
    """Scores ``[B, H_q, 1, T_block]`` (in ``Q.dtype``) of one cold block with
    absolute-position RoPE; ``use_triton`` is ignored (one implementation)."""
    s = _ops.block_scores(Q, coeffs_K, basis_K, cos, sin, int(start_position))
    if config is not None and config.enable_logging:
        logger.debug("[SCORE] Q=%s coeffs_K=%s start=%d", tuple(Q.shape), tuple(coeffs_K.shape), start_position)
    return s.unsqueeze(2).to(Q.dtype)


def spectral_value_forward(attn: torch.Tensor, coeffs_V: torch.Tensor, basis_V: torch.Tensor, D: int,
                           config: Optional[TritonSpectralConfig] = None, use_triton: bool = False) -> torch.Tensor:
    """``(attn @ C_V) @ B_V`` -> ``[B, H_q, 1, D]`` in ``attn.dtype``."""
    out = _ops.block_values(attn, coeffs_V, basis_V)
    return out.unsqueeze(2).to(attn.dtype)


def spectral_attention_decode(Q: torch.Tensor, cache, cos: torch.Tensor, sin: torch.Tensor, query_position: int,
                              attention_mask: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                              config: Optional[TritonSpectralConfig] = None) -> torch.Tensor:
    """Full decode over the spectral cache, absolute-position cold RoPE.  Returns
    ``[B, H_q, 1, D]`` in ``Q.dtype``; raises ``ValueError`` on an empty cache."""
    if config is not None and config.enable_logging:
        logger.info("[SPECTRAL_DECODE] Q=%s query_pos=%d", tuple(Q.shape), query_position)
    return spectral_decode(Q, cache, cos, sin, query_position, attention_mask, scale, N.SPX_ROPE_ABSOLUTE)


def spectral_attention_decode_pytorch(Q, cache, cos, sin, query_position, attention_mask=None, scale=None):
    """Same interface as ``spectral_attention_decode``, distance-indexed RoPE (the
    reference routes this name to ``spectral_attention_forward``, :864-879)."""
    return spectral_attention_forward(Q, cache, cos, sin, query_position, attention_mask, scale)
