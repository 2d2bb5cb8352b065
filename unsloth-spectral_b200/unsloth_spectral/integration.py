"""Attention patching for HF/Unsloth Llama-family models (the caller of the decode path).

Mirrors unsloth_spectral/integration.py:43-938:
* ``create_spectral_forward`` -- per-layer ``self_attn.forward`` replacement: projects
  Q/K/V, appends PRE-RoPE keys to the layer's ``SpectralCache`` and, for one query
  token past one block of context, runs the fused spectral decode
  (``spectral_attention_forward``, distance RoPE, :273-291); otherwise (prefill or
  short context) reconstructs K/V and runs dense attention (:292-402).
* ``create_spectral_forward_inference`` -- Unsloth's single-token decode signature
  (:481-725), routed to ``kernels.spectral_attention_decode`` (absolute RoPE) when the
  CUDA library loads, as the reference routes to its kernels module.
* ``patch_unsloth_attention`` / ``get_cache_stats`` -- same arguments and results.

RoPE tables: the reference reads them from ``self.rotary_emb``; modules without one
(current ``transformers``) get float32 tables built from ``config.rope_theta``.
"""
from __future__ import annotations

import logging
import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from . import _ops
from .spectral_attention import apply_rope, spectral_attention_forward
from .spectral_cache import SpectralCache

logger = logging.getLogger("unsloth_spectral.integration")

TRITON_KERNELS_AVAILABLE = False
try:
    from .kernels import TRITON_AVAILABLE
    if TRITON_AVAILABLE:
        from .kernels import TritonSpectralConfig, spectral_attention_decode
        TRITON_KERNELS_AVAILABLE = True
except ImportError:  # pragma: no cover
    TRITON_AVAILABLE = False


def apply_rotary_pos_emb(q, k, cos, sin, position_ids=None):
    """HF-style RoPE (``rotate_half``) with ``cos``/``sin`` broadcast over heads."""
    if cos.dim() == 2:
        cos, sin = cos[None, None], sin[None, None]
    elif cos.dim() == 3:
        cos, sin = cos[:, None], sin[:, None]

    def rotate_half(x):
        h = x.shape[-1] // 2
        return torch.cat((-x[..., h:], x[..., :h]), dim=-1)

    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


def repeat_kv(hidden_states: torch.Tensor, n_rep: int) -> torch.Tensor:
    if n_rep == 1:
        return hidden_states
    return torch.repeat_interleave(hidden_states, n_rep, dim=1)


def _attn_dims(self):
    cfg = getattr(self, "config", None)
    if cfg is not None:
        nh = cfg.num_attention_heads
        nkv = getattr(cfg, "num_key_value_heads", nh)
        hd = getattr(self, "head_dim", None) or getattr(cfg, "head_dim", None) or cfg.hidden_size // nh
        return nh, nkv, hd
    return self.num_heads, self.num_key_value_heads, self.head_dim


def rope_tables_for(self, seq_len: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
    """Float32 ``[len, D]`` RoPE tables for module ``self``: from ``rotary_emb`` when it
    caches tables (Unsloth), else built from the config's rope theta and memoised."""
    rot = getattr(self, "rotary_emb", None)
    if rot is not None and hasattr(rot, "extend_rope_embedding"):
        rot.extend_rope_embedding(None, seq_len=seq_len)
        return rot.get_cached(seq_len, device.index)
    _, _, hd = _attn_dims(self)
    cached = getattr(self, "_spx_rope", None)
    if cached is not None and cached[0].shape[0] >= seq_len and cached[0].device == device:
        return cached
    cfg = getattr(self, "config", None)
    theta = getattr(cfg, "rope_theta", None)
    if theta is None:
        theta = (getattr(cfg, "rope_parameters", None) or {}).get("rope_theta", 10000.0)
    n = max(seq_len, 2 * (cached[0].shape[0] if cached is not None else 2048))
    inv = float(theta) ** (-torch.arange(0, hd, 2, dtype=torch.float64, device=device) / hd)
    freqs = torch.outer(torch.arange(n, dtype=torch.float64, device=device), inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    tabs = (emb.cos().float(), emb.sin().float())
    self._spx_rope = tabs
    return tabs


def _qkv(self, hidden_states):
    """The query, key and value projections of ``hidden_states``.  A module that keeps its
    three weights as row blocks of one tensor, ``spx_qkv_weight`` (the in-repo loop does),
    gets them from one GEMM (one read of the input, one larger weight stream, which at the
    decode step's batch of a few rows runs much closer to the bandwidth than three); any
    other module runs its own ``q_proj`` / ``k_proj`` / ``v_proj`` as the reference does."""
    w = getattr(self, "spx_qkv_weight", None)
    if w is None:
        return self.q_proj(hidden_states), self.k_proj(hidden_states), self.v_proj(hidden_states)
    nq, nk = self.q_proj.weight.shape[0], self.k_proj.weight.shape[0]
    qkv = torch.nn.functional.linear(hidden_states, w)
    return qkv[..., :nq], qkv[..., nq:nq + nk], qkv[..., nq + nk:]


def _mask_is_causal(mask: torch.Tensor, q_pos: torch.Tensor, k_pos: torch.Tensor) -> bool:
    """True when the additive ``mask`` (broadcastable to ``[.., T_q, T_k]``) is 0 where the
    key position is at most the query position and effectively -inf (<= -1e4) where it is
    larger: adding it then equals the causal rule.  One device read (prefill only)."""
    if mask.shape[-2] != q_pos.numel() or mask.shape[-1] != k_pos.numel():
        return False
    future = k_pos.reshape(1, -1) > q_pos.reshape(-1, 1)
    m = mask.float()
    ok = torch.where(future, m <= -1e4, m == 0).all()
    return bool(ok.item())


def _dense_attention(q, cache: SpectralCache, cos, sin, n_rep, head_dim, attention_mask, dtype, q_pos=None):
    """Attention of a multi-token query over the whole cache (integration.py:292-346, the
    prefill / short-context path): softmax(Q RoPE(K)^T / sqrt(D) + mask) V with the keys
    rotated at their cached positions.  Runs ``spx_prefill_attn`` (K and V rebuilt tile by
    tile from the codes inside the kernel); a mask that is exactly the causal rule is
    applied as that rule, so the kernel skips the future tiles.  Shapes the kernel does not
    cover (head_dim != 128, float32 caches, n_rep > 8) reconstruct K/V and run the dense
    product as the reference does."""
    t = cache.tiers
    if q_pos is not None and _ops.prefill_supported(q, t):
        qp = q_pos.reshape(-1)[-q.shape[2]:].to(q.device)
        causal = False
        mask = attention_mask
        if mask is not None and q.shape[2] > 1 and _mask_is_causal(mask, qp, cache.get_all_positions()):
            causal, mask = True, None
        return _ops.prefill(q, t, cos, sin, qp, mask=mask, causal=causal, scale=1.0 / math.sqrt(head_dim)).to(dtype)
    K, V = cache.get_kv()
    pos = cache.get_all_positions()
    K = apply_rope(K, cos[pos][None, None], sin[pos][None, None]).to(dtype)
    K, V = repeat_kv(K, n_rep), repeat_kv(V, n_rep)
    w = torch.matmul(q, K.transpose(2, 3)) / math.sqrt(head_dim)
    if attention_mask is not None:
        w = w + attention_mask
    w = F.softmax(w, dim=-1, dtype=torch.float32).to(q.dtype)
    return torch.matmul(w, V)


def create_spectral_forward(original_forward, block_size: int = 512, k_rank_keys: int = 16,
                            k_rank_values: int = 32, hot_buffer_size: int = 64, use_spectral_attention: bool = True,
                            debug_logging: bool = False, use_attention_weighted_svd: bool = False,
                            landmark_count: int = 0):
    """Per-layer attention forward with a spectral cache (integration.py:43-425)."""

    def spectral_forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_value=None,
                         output_attentions=False, use_cache=False, cache_position=None, **kwargs):
        nh, nkv, hd = _attn_dims(self)
        bsz, q_len, _ = hidden_states.size()
        qp, kp, vp = _qkv(self, hidden_states)
        q = qp.view(bsz, q_len, nh, hd).transpose(1, 2)
        k_pre = kp.view(bsz, q_len, nkv, hd).transpose(1, 2)
        v = vp.view(bsz, q_len, nkv, hd).transpose(1, 2)
        if past_key_value is None:
            past_key_value = getattr(self, "_spectral_cache", None) if use_cache else None
        if not isinstance(past_key_value, SpectralCache):
            cache = SpectralCache(nkv, hd, block_size, k_rank_keys, k_rank_values, hot_buffer_size,
                                  device=hidden_states.device, dtype=hidden_states.dtype,
                                  debug_logging=debug_logging, use_attention_weighted_svd=use_attention_weighted_svd,
                                  landmark_count=landmark_count)
            if isinstance(past_key_value, (tuple, list)) and len(past_key_value) == 2:
                cache.append(past_key_value[0], past_key_value[1])
            past_key_value = cache
        kv_seq_len = q_len + past_key_value.total_tokens
        cos, sin = rope_tables_for(self, kv_seq_len + 1, hidden_states.device)
        if position_ids is None:
            position_ids = torch.arange(past_key_value.total_tokens, kv_seq_len,
                                        device=hidden_states.device)[None]
        cq, sq = cos[position_ids][:, None], sin[position_ids][:, None]
        q = apply_rope(q.float(), cq, sq).to(q.dtype)
        past_key_value.append(k_pre, v, position_ids)
        if use_spectral_attention and past_key_value.total_tokens > block_size and q_len == 1:
            out = spectral_attention_forward(q, past_key_value, cos, sin, kv_seq_len - 1, attention_mask,
                                             1.0 / math.sqrt(hd))
        else:
            out = _dense_attention(q, past_key_value, cos, sin, nh // nkv, hd, attention_mask, q.dtype, position_ids)
        out = out.transpose(1, 2).reshape(bsz, q_len, nh * hd)
        out = self.o_proj(out)
        if use_cache:
            self._spectral_cache = past_key_value
        return out, None, past_key_value if use_cache else None

    return spectral_forward


def create_spectral_forward_inference(block_size: int = 512, k_rank_keys: int = 16, k_rank_values: int = 32,
                                      hot_buffer_size: int = 64, use_spectral_attention: bool = True,
                                      debug_logging: bool = False, use_triton_kernel: bool = True,
                                      use_attention_weighted_svd: bool = False, landmark_count: int = 0):
    """Unsloth-signature single-token decode forward (integration.py:481-725)."""
    use_kernels = use_triton_kernel and TRITON_KERNELS_AVAILABLE

    def spectral_forward_inference(self, hidden_states, past_key_value, position_ids, do_prefill=False,
                                   attention_mask=None):
        bsz, q_len, _ = hidden_states.size()
        assert q_len == 1, f"Inference path expects q_len=1, got {q_len}"
        nh, nkv, hd = _attn_dims(self)
        qp, kp, vp = _qkv(self, hidden_states)
        q = qp.view(bsz, 1, nh, hd).transpose(1, 2)
        k_pre = kp.view(bsz, 1, nkv, hd).transpose(1, 2)
        v = vp.view(bsz, 1, nkv, hd).transpose(1, 2)
        if not isinstance(past_key_value, SpectralCache):
            past_key_value = SpectralCache(nkv, hd, block_size, k_rank_keys, k_rank_values, hot_buffer_size,
                                           device=hidden_states.device, dtype=hidden_states.dtype,
                                           debug_logging=debug_logging,
                                           use_attention_weighted_svd=use_attention_weighted_svd,
                                           landmark_count=landmark_count)
        kv_seq_len = 1 + past_key_value.total_tokens
        cos, sin = rope_tables_for(self, kv_seq_len + 1, hidden_states.device)
        qpos = kv_seq_len - 1
        # the query is rotated at position_ids, as the reference's decode path does
        # (integration.py:600-612); without them, at the next cache position
        pid = None
        if position_ids is not None:
            pid = position_ids.reshape(-1, position_ids.shape[-1])[:, -1:].to(hidden_states.device)
        if (hidden_states.is_cuda and cos.dtype == torch.float32 and cos.is_contiguous() and sin.is_contiguous()
                and qp.stride(-1) == 1 and (pid is None or pid.shape[0] in (1, bsz))):
            # one launch (spx_rope_rows), the same float32 arithmetic as apply_rope below
            q = _ops.rope_rows(qp, nh, hd, cos, sin, pid, qpos)
        elif pid is not None:
            q = apply_rope(q.float(), cos[pid][:, None], sin[pid][:, None]).to(q.dtype)
        else:
            q = apply_rope(q.float(), cos[qpos], sin[qpos]).to(q.dtype)
        past_key_value.append(k_pre, v, position_ids)
        if use_spectral_attention and past_key_value.total_tokens > block_size:
            if use_kernels:
                out = spectral_attention_decode(q, past_key_value, cos, sin, qpos, attention_mask,
                                                1.0 / math.sqrt(hd), TritonSpectralConfig(enable_logging=debug_logging))
            else:
                out = spectral_attention_forward(q, past_key_value, cos, sin, qpos, attention_mask,
                                                 1.0 / math.sqrt(hd))
        else:
            out = _dense_attention(q, past_key_value, cos, sin, nh // nkv, hd, attention_mask, q.dtype,
                                   torch.full((1,), qpos, dtype=torch.long, device=hidden_states.device))
        out = self.o_proj(out.transpose(1, 2).reshape(bsz, 1, nh * hd))
        return out, past_key_value

    return spectral_forward_inference


def patch_unsloth_attention(model, block_size: int = 512, k_rank_keys: int = 16, k_rank_values: int = 32,
                            hot_buffer_size: int = 64, use_spectral_attention: bool = True, verbose: bool = True,
                            debug_logging: bool = False, use_triton_kernel: bool = True,
                            use_attention_weighted_svd: bool = False, landmark_count: int = 0):
    """Patch every ``model.model.layers[i].self_attn`` in place (integration.py:728-889)."""
    num_patched = 0
    for layer in model.model.layers:
        if hasattr(layer, "self_attn"):
            fwd = create_spectral_forward(layer.self_attn.forward, block_size, k_rank_keys, k_rank_values,
                                          hot_buffer_size, use_spectral_attention, debug_logging,
                                          use_attention_weighted_svd, landmark_count)
            layer.self_attn.forward = fwd.__get__(layer.self_attn, type(layer.self_attn))
            layer.self_attn._spx_inference = create_spectral_forward_inference(
                block_size, k_rank_keys, k_rank_values, hot_buffer_size, use_spectral_attention, debug_logging,
                use_triton_kernel, use_attention_weighted_svd, landmark_count).__get__(
                    layer.self_attn, type(layer.self_attn))
            num_patched += 1
    try:
        import unsloth.models.llama as llama_module  # noqa: F401
        fn = create_spectral_forward_inference(block_size, k_rank_keys, k_rank_values, hot_buffer_size,
                                               use_spectral_attention, debug_logging, use_triton_kernel,
                                               use_attention_weighted_svd, landmark_count)
        llama_module.LlamaAttention_fast_forward_inference = fn
        if hasattr(llama_module, "_LlamaModel_fast_forward_inference"):
            llama_module.LlamaModel_fast_forward_inference = llama_module._LlamaModel_fast_forward_inference(
                attention_fast_forward_inference=fn)
        if verbose:
            print("Patched decode inference path (LlamaAttention + LlamaModel)")
    except Exception as e:  # unsloth absent: per-layer patch only, as the reference
        if verbose:
            print(f"Warning: Could not patch inference function: {e}")
    if verbose:
        print(f"Patched {num_patched} attention layers with SpectralCache")
        print(f"   Config: block_size={block_size}, k_K={k_rank_keys}, k_V={k_rank_values}")
    return model


def get_cache_stats(model):
    """Aggregate ``get_memory_stats`` over the patched layers (integration.py:892-938)."""
    tot_tok = tot_blk = orig = comp = 0
    per_layer = []
    for i, layer in enumerate(model.model.layers):
        cache = getattr(getattr(layer, "self_attn", None), "_spectral_cache", None)
        if isinstance(cache, SpectralCache):
            s = cache.get_memory_stats()
            tot_tok += s["total_tokens"]
            tot_blk += s["num_blocks"]
            orig += s["original_bytes"]
            comp += s["compressed_bytes"]
            per_layer.append({"layer_idx": i, "tokens": s["total_tokens"], "blocks": s["num_blocks"],
                              "compression": s["compression_ratio"]})
    return {"total_tokens": tot_tok, "total_blocks": tot_blk, "total_original_bytes": orig,
            "total_compressed_bytes": comp, "compression_ratio": orig / comp if comp > 0 else 1.0,
            "layers_with_cache": len(per_layer), "per_layer_stats": per_layer}
