"""In-repo Llama/Mistral-architecture decoder and greedy token loop driven through the
patched attention layers -- the caller of the decode path without Unsloth.

The reference runs inside Unsloth: ``patch_unsloth_attention`` replaces every layer's
``self_attn.forward`` and Unsloth's ``LlamaAttention_fast_forward_inference``, and its
rebuilt ``LlamaModel_fast_forward_inference`` (integration.py:808-878) walks the layers
for one new token: RMSNorm, the single-token attention with the layer's
``SpectralCache``, residual, RMSNorm, SwiGLU MLP, residual; final norm and LM head.
This module is that loop for a model whose attention modules carry the attributes the
patched forwards read (``config`` with head counts / ``head_dim`` / ``rope_theta``,
``q_proj`` .. ``o_proj``):

* prompt: ``self_attn.forward`` per layer (the patched prefill: pre-RoPE keys go into
  the layer's cache, full blocks are compressed in one batched rSVD launch, attention
  over the reconstructed cache with a causal mask);
* each new token: ``self_attn._spx_inference`` per layer (the patched single-token
  forward, routed to ``kernels.spectral_attention_decode``), greedy argmax.

On the GPU the loop's own small operations are single launches of the library: each
RMSNorm with the residual add in front of it (``spx_rmsnorm``), and the attention
modules hold their q / k / v weights as one tensor so that the patched forwards project
with one GEMM (the forwards' query RoPE and cache append are library kernels too).

Weights are random (``N(0, std^2)``, the architecture only), created directly on the
device.  ``MISTRAL_7B`` is the 32-layer, hidden-4096, 32/8-head, FFN-14336, vocab-32768,
RoPE-theta-1e6 shape.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from types import SimpleNamespace
from typing import List, Optional

import torch
import torch.nn.functional as F

from . import _ops
from .integration import patch_unsloth_attention, rope_tables_for


@dataclass
class LlamaShape:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 32768
    rope_theta: float = 1e6
    eps: float = 1e-5


MISTRAL_7B = LlamaShape()


class RMSNorm(torch.nn.Module):
    """``T(x * rsqrt(mean(x^2) + eps)) * weight``; on the GPU one ``spx_rmsnorm`` launch per
    call (with ``add``, the residual add fused in front), the arithmetic of the float32
    expression below, which runs only for CPU tensors (the layout tests)."""

    def __init__(self, dim: int, eps: float, device, dtype):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(dim, device=device, dtype=dtype))
        self.eps = eps

    def forward(self, x):
        if x.is_cuda:
            return _ops.rmsnorm(x, self.weight, self.eps)
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype) * self.weight

    def add(self, h, a):
        """``h + a`` (the residual stream, in the dtype) and its norm, in one launch."""
        if h.is_cuda:
            out, hn = _ops.rmsnorm(a, self.weight, self.eps, residual=h)
            return hn, out
        hn = h + a
        return hn, self.forward(hn)


def _linear(i: int, o: int, device, dtype, std: float, gen) -> torch.nn.Linear:
    lin = torch.nn.Linear(i, o, bias=False, device="meta")
    lin.weight = torch.nn.Parameter(torch.empty(o, i, device=device, dtype=dtype).normal_(0.0, std, generator=gen))
    return lin


def _linear_of(weight: torch.Tensor) -> torch.nn.Linear:
    lin = torch.nn.Linear(weight.shape[1], weight.shape[0], bias=False, device="meta")
    lin.weight = torch.nn.Parameter(weight)
    return lin


class Attention(torch.nn.Module):
    """Projections and the config attributes of an HF Llama attention module; its
    ``forward`` is replaced by ``patch_unsloth_attention``."""

    def __init__(self, s: LlamaShape, device, dtype, std, gen):
        super().__init__()
        self.config = SimpleNamespace(num_attention_heads=s.heads, num_key_value_heads=s.kv_heads, head_dim=s.head_dim,
                                      hidden_size=s.hidden, rope_theta=s.rope_theta)
        self.head_dim = s.head_dim
        # q / k / v weights are row blocks of one tensor (`spx_qkv_weight`, not saved: it
        # shares their storage), so the patched forwards project with one GEMM
        nq, nk = s.heads * s.head_dim, s.kv_heads * s.head_dim
        w = torch.empty(nq + 2 * nk, s.hidden, device=device, dtype=dtype).normal_(0.0, std, generator=gen)
        self.q_proj = _linear_of(w[:nq])
        self.k_proj = _linear_of(w[nq:nq + nk])
        self.v_proj = _linear_of(w[nq + nk:])
        self.register_buffer("spx_qkv_weight", w, persistent=False)
        self.o_proj = _linear(s.heads * s.head_dim, s.hidden, device, dtype, std, gen)

    def forward(self, *a, **k):  # pragma: no cover - replaced by the patch
        raise RuntimeError("call patch_unsloth_attention(model) first")


class MLP(torch.nn.Module):
    def __init__(self, s: LlamaShape, device, dtype, std, gen):
        super().__init__()
        self.gate_proj = _linear(s.hidden, s.ffn, device, dtype, std, gen)
        self.up_proj = _linear(s.hidden, s.ffn, device, dtype, std, gen)
        self.down_proj = _linear(s.ffn, s.hidden, device, dtype, std, gen)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DecoderLayer(torch.nn.Module):
    def __init__(self, s: LlamaShape, device, dtype, std, gen):
        super().__init__()
        self.input_layernorm = RMSNorm(s.hidden, s.eps, device, dtype)
        self.self_attn = Attention(s, device, dtype, std, gen)
        self.post_attention_layernorm = RMSNorm(s.hidden, s.eps, device, dtype)
        self.mlp = MLP(s, device, dtype, std, gen)


class SpectralLlama(torch.nn.Module):
    """``model.model.layers[i].self_attn`` as HF lays it out, so ``patch_unsloth_attention``
    and ``get_cache_stats`` apply unchanged."""

    def __init__(self, shape: LlamaShape = MISTRAL_7B, device="cuda", dtype=torch.bfloat16, std: float = 0.02,
                 seed: int = 0):
        super().__init__()
        device = torch.device(device)
        gen = torch.Generator(device=device).manual_seed(seed)
        self.shape = shape
        self.model = torch.nn.Module()
        self.model.embed_tokens = torch.nn.Embedding(shape.vocab, shape.hidden, device="meta")
        self.model.embed_tokens.weight = torch.nn.Parameter(
            torch.empty(shape.vocab, shape.hidden, device=device, dtype=dtype).normal_(0.0, std, generator=gen))
        self.model.layers = torch.nn.ModuleList(DecoderLayer(shape, device, dtype, std, gen)
                                                for _ in range(shape.layers))
        self.model.norm = RMSNorm(shape.hidden, shape.eps, device, dtype)
        self.lm_head = _linear(shape.hidden, shape.vocab, device, dtype, std, gen)

    def patch(self, **kw):
        """``patch_unsloth_attention`` with this model (integration.py:728)."""
        kw.setdefault("verbose", False)
        return patch_unsloth_attention(self, **kw)

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor):
        """Run the prompt ``[B, T]`` through the patched ``forward`` of every layer (causal
        mask); returns (logits of the last position ``[B, vocab]``, per-layer caches)."""
        B, T = input_ids.shape
        dev = input_ids.device
        h = self.model.embed_tokens(input_ids)
        pos = torch.arange(T, device=dev)[None]
        mask = torch.full((T, T), float("-inf"), device=dev, dtype=h.dtype).triu_(1)[None, None]
        caches: List = []
        layers = self.model.layers
        x = layers[0].input_layernorm(h)
        for i, layer in enumerate(layers):
            a, _, cache = layer.self_attn.forward(x, attention_mask=mask, position_ids=pos,
                                                  past_key_value=None, use_cache=True)
            caches.append(cache)
            h, x = layer.post_attention_layernorm.add(h, a)       # h + attention, its norm
            nxt = layers[i + 1].input_layernorm if i + 1 < len(layers) else self.model.norm
            h, x = nxt.add(h, layer.mlp(x))                      # h + MLP, the next norm
        return self.lm_head(x[:, -1]), caches

    @torch.no_grad()
    def decode_step(self, token: torch.Tensor, position: torch.Tensor, caches: List):
        """One new token ``[B]`` at device position ``position`` (``[1, 1]`` int64) through
        the patched single-token forward of every layer; returns logits ``[B, vocab]``."""
        h = self.model.embed_tokens(token[:, None])
        layers = self.model.layers
        x = layers[0].input_layernorm(h)
        for i, layer in enumerate(layers):
            a, caches[i] = layer.self_attn._spx_inference(x, caches[i], position)
            h, x = layer.post_attention_layernorm.add(h, a)
            nxt = layers[i + 1].input_layernorm if i + 1 < len(layers) else self.model.norm
            h, x = nxt.add(h, layer.mlp(x))
        return self.lm_head(x[:, -1])

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int, timer=None, cuda_graphs: bool = False):
        """Greedy decoding: the prompt, then ``max_new_tokens`` tokens, each the argmax of
        the previous step's logits.  Positions stay on the device (no host reads inside
        the loop).  ``cuda_graphs``: replay the decode step from a CUDA graph between block
        compressions (``_decode_graphed``).  ``timer(name)``, if given, is called after
        the prefill ("prefill") and at the end ("decode").  Returns the new tokens
        ``[B, max_new_tokens]``."""
        B, T = input_ids.shape
        logits, caches = self.prefill(input_ids)
        if timer is not None:
            timer("prefill")
        out = torch.empty(B, max_new_tokens, dtype=torch.long, device=input_ids.device)
        tok = logits.argmax(-1)
        pos = torch.full((1, 1), T, dtype=torch.long, device=input_ids.device)
        if cuda_graphs:
            self._decode_graphed(tok, pos, caches, out)
        else:
            for s in range(max_new_tokens):
                out[:, s] = tok
                if s + 1 == max_new_tokens:
                    break
                logits = self.decode_step(tok, pos, caches)
                tok = logits.argmax(-1)
                pos += 1
        if timer is not None:
            timer("decode")
        self._caches = caches
        return out

    @torch.no_grad()
    def _decode_graphed(self, tok: torch.Tensor, pos: torch.Tensor, caches: List, out: torch.Tensor):
        """The decode loop with the step captured in a CUDA graph.  One step's kernels
        depend on the host only through the cold-tier block count and the tensors'
        addresses; the hot tier grows through its device length (single-token appends
        write at it and advance it on the device, the merge kernel reads it).  So between
        two block compressions the step is captured once and replayed, the caches' host
        counters advanced per replay; the step whose append fills a block (compression,
        host-side) and the first step of a segment (warm-up of the capture stream) run
        eagerly.  Same kernels and results as the eager loop."""
        n = out.shape[1]
        dev = tok.device
        stream = torch.cuda.Stream(device=dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        tok, s = tok.clone(), 0
        out[:, 0] = tok
        with torch.cuda.stream(stream):
            while s + 1 < n:
                t0 = caches[0].tiers
                room = caches[0].block_size - 1 - t0.hot_len   # appends before one fills a block
                if room < 3 or n - 1 - s < 3:
                    logits = self.decode_step(tok, pos, caches)
                    tok.copy_(logits.argmax(-1))
                    pos.add_(1)
                    s += 1
                    out[:, s] = tok
                    continue
                k = min(room, n - 1 - s)
                # everything the step caches on first use is created here, eagerly and outside
                # the graph's memory pool: hot-tier buffers of full size, RoPE tables long
                # enough for the segment, and (by one eager step on the capture stream) the
                # stream's decode workspace and cuBLAS state
                for c in caches:
                    c.tiers.ensure_hot(c.block_size)
                    c.tiers.hot_bound = c.block_size
                for layer in self.model.layers:
                    rope_tables_for(layer.self_attn, caches[0].total_tokens + k + 2, dev)
                logits = self.decode_step(tok, pos, caches)
                tok.copy_(logits.argmax(-1))
                pos.add_(1)
                s += 1
                out[:, s] = tok
                for c in caches:
                    c.tiers.hot_len_device()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    g_logits = self.decode_step(tok, pos, caches)
                    tok.copy_(g_logits.argmax(-1))
                    pos.add_(1)
                for r in range(k - 1):
                    if r:
                        for c in caches:
                            c.note_replayed_tokens(1)
                    graph.replay()
                    s += 1
                    out[:, s] = tok
                del graph, g_logits
                for c in caches:
                    c.tiers.hot_bound = None
        torch.cuda.current_stream(dev).wait_stream(stream)
