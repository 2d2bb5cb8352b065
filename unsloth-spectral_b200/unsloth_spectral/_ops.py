"""Tensor-level wrappers over the spx C ABI.  Every function here launches CUDA work
through ``libspx.so``; none has a CPU or pure-torch fallback."""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _native as N

_rope_cache = {}


def _key(t: torch.Tensor):
    return (t.data_ptr(), tuple(t.shape), tuple(t.stride()), t.dtype, t._version)


_vtile_cache = {}


def vtile_index(T: int, R: int, device) -> torch.Tensor:
    """``idx`` with ``stored[..., p] = natural[..., idx[p]]`` for one block of value codes:
    natural = rank-major ``[R][T]`` flattened, stored = the value-tile layout of
    ``include/spx.h`` (16-token tiles of ``[R][16]`` bytes, rows XOR (tile & 7), tokens
    ordered 0,1,8,9,2,3,10,11,...)."""
    key = (T, R, str(device))
    idx = _vtile_cache.get(key)
    if idx is None:
        r = torch.arange(R).view(R, 1).expand(R, T)
        t = torch.arange(T).view(1, T).expand(R, T)
        tt, x = t // 16, t % 16
        pos = 4 * ((x % 8) // 2) + (x % 2) + 2 * (x // 8)
        stored = (tt * R + (r ^ (tt % 8))) * 16 + pos
        idx = torch.empty(R * T, dtype=torch.long)
        idx[stored.reshape(-1)] = (r * T + t).reshape(-1)
        idx = idx.to(device)
        _vtile_cache[key] = idx
    return idx


def rope_table_f32(t: torch.Tensor, device) -> torch.Tensor:
    """``t`` as a contiguous float32 ``[rope_len, D]`` table on ``device``."""
    if t.dim() == 3 and t.shape[0] == 1:
        t = t[0]
    if t.dim() != 2:
        raise ValueError(f"cos/sin must be [max_len, head_dim] tables, got shape {tuple(t.shape)}")
    return t.to(device=device, dtype=torch.float32).contiguous()


def rope_tied(cos: torch.Tensor, sin: torch.Tensor) -> bool:
    """True when both tables repeat their first half (HF ``cat(freqs, freqs)`` layout).
    Memoised per tensor version, so the device comparison runs once per table."""
    k = (_key(cos), _key(sin))
    v = _rope_cache.get(k)
    if v is None:
        h = cos.shape[-1] // 2
        v = bool(torch.equal(cos[..., :h], cos[..., h:]) and torch.equal(sin[..., :h], sin[..., h:]))
        if len(_rope_cache) > 64:
            _rope_cache.clear()
        _rope_cache[k] = v
    return v


_freq_cache = {}


def rope_freq(cos: torch.Tensor, sin: torch.Tensor):
    """The RoPE frequencies ``theta_i`` of HF-style tables (first half of each row
    ``cos/sin(position * theta_i)``, times one common magnitude), as a float32 CPU tensor
    of ``D/2`` values, or None when the tables are not of that form.  ``theta`` is read
    from rows 1 and ``len - 1`` in float64 and every row is checked against it, with the
    tolerance of float32 tables whose angles were formed in float32
    (``|dx| <= 4e-6 + 3e-7 * position * theta``).  Memoised per tensor version, so the
    device-to-host copy runs once per table."""
    k = (_key(cos), _key(sin))
    v = _freq_cache.get(k, False)
    if v is not False:
        return v
    c = cos.detach().to("cpu", torch.float64)
    s = sin.detach().to("cpu", torch.float64)
    if c.dim() == 3 and c.shape[0] == 1:
        c, s = c[0], s[0]
    out = None
    if c.dim() == 2 and c.shape[0] >= 2 and c.shape[1] % 2 == 0:
        h = c.shape[1] // 2
        c, s = c[:, :h], s[:, :h]
        n = c.shape[0]
        mag = torch.sqrt(c[0] ** 2 + s[0] ** 2)
        th = torch.atan2(s[1], c[1])
        if n > 2:
            p = n - 1
            ph = torch.atan2(s[p], c[p])
            turns = torch.round((p * th - ph) / (2 * math.pi))
            th = (ph + 2 * math.pi * turns) / p
        pos = torch.arange(n, dtype=torch.float64)[:, None]
        ang = pos * th[None]
        tol = 4e-6 + 3e-7 * pos * th.abs()[None]
        ok = bool(((c - mag * torch.cos(ang)).abs() <= tol * (1 + mag)).all()
                  and ((s - mag * torch.sin(ang)).abs() <= tol * (1 + mag)).all()
                  and bool((s[0].abs() <= 1e-6).all()))
        if ok:
            out = th.to(torch.float32).contiguous()
    if len(_freq_cache) > 64:
        _freq_cache.clear()
    _freq_cache[k] = out
    return out


def rope_rows(x: torch.Tensor, heads: int, head_dim: int, cos: torch.Tensor, sin: torch.Tensor,
              pos: Optional[torch.Tensor] = None, pos_host: int = 0) -> torch.Tensor:
    """``spx_rope_rows``: the rows of ``x`` (``[rows, ..., heads * head_dim]``, last
    dimension contiguous, one token per row) rotated at ``pos`` (int64 device tensor of
    one position per row, a strided column is fine, or one position for all) or at
    ``pos_host``; returns ``[rows, heads, 1, head_dim]`` in the dtype of ``x``."""
    lib = N.lib_for(x.device)
    rows = x.shape[0]
    assert x.stride(-1) == 1 and x.shape[-1] == heads * head_dim
    out = torch.empty(rows, heads, 1, head_dim, dtype=x.dtype, device=x.device)
    dt = {torch.float32: N.SPX_F32, torch.float16: N.SPX_F16, torch.bfloat16: N.SPX_BF16}[x.dtype]
    pstride = 0
    if pos is not None and pos.numel() > 1:
        pstride = pos.stride(0)
    N.check(lib, lib.spx_rope_rows(N.ptr(x), x.stride(0), N.ptr(cos), N.ptr(sin), cos.shape[0], N.ptr(pos),
                                   pstride, int(pos_host), N.ptr(out), rows, heads, head_dim, dt,
                                   N.stream_handle(x.device)), "spx_rope_rows")
    return out


def hot_append(k: torch.Tensor, v: torch.Tensor, hot_k: torch.Tensor, hot_v: torch.Tensor, hot_pos: torch.Tensor,
               hot_len: torch.Tensor, pos: torch.Tensor):
    """``spx_hot_append``: one token's key/value rows ``[B, H, 1, D]`` (any strides, the
    last dimension contiguous) written into the hot tier at the device length ``hot_len``
    (int32 scalar), its position (int64 device scalar) into ``hot_pos``, the length
    advanced by one -- one launch."""
    lib = N.lib_for(k.device)
    B, H, _, D = k.shape
    assert k.stride(-1) == 1 and v.stride(-1) == 1 and hot_k.is_contiguous() and hot_v.is_contiguous()
    dt = {torch.float32: N.SPX_F32, torch.float16: N.SPX_F16, torch.bfloat16: N.SPX_BF16}[k.dtype]
    N.check(lib, lib.spx_hot_append(N.ptr(k), N.ptr(v), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
                                    N.ptr(hot_k), N.ptr(hot_v), N.ptr(hot_pos), N.ptr(hot_len), N.ptr(pos), B, H, D,
                                    hot_k.shape[2], dt, N.stream_handle(k.device)), "spx_hot_append")


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None):
    """``spx_rmsnorm`` over the last dimension of FP16/BF16 ``x``: returns
    ``dtype(h * rsqrt(mean(h^2) + eps)) * weight`` with ``h = x`` or, when ``residual`` is
    given, ``h = x + residual`` (rounded to the dtype), returned as a second value."""
    lib = N.lib_for(x.device)
    dim = x.shape[-1]
    xc = x.contiguous()
    rows = xc.numel() // dim if dim else 0
    out = torch.empty_like(xc)
    rc = residual.contiguous() if residual is not None else None
    h = torch.empty_like(xc) if residual is not None else None
    dt = N.SPX_BF16 if x.dtype == torch.bfloat16 else N.SPX_F16 if x.dtype == torch.float16 else -1
    if rows == 0:
        return out if residual is None else (out, h)
    N.check(lib, lib.spx_rmsnorm(N.ptr(xc), N.ptr(rc) if rc is not None else None, N.ptr(weight.contiguous()),
                                 N.ptr(out), N.ptr(h) if h is not None else None, rows, dim, float(eps), dt,
                                 N.stream_handle(x.device)), "spx_rmsnorm")
    return out if residual is None else (out, h)


def quantize_int8(x: torch.Tensor):
    """Per-leading-index INT8 quantisation; returns (codes int8, scale f32 [N],
    minmax f32 [N, 2], dequantised f32) -- bit-exact with the reference's
    ``_quantize_int8_batched``."""
    lib = N.lib_for(x.device)
    xf = x.to(torch.float32).contiguous()
    N_ = xf.shape[0]
    codes = torch.empty(xf.shape, dtype=torch.int8, device=x.device)
    scale = torch.empty(N_, dtype=torch.float32, device=x.device)
    minmax = torch.empty(N_, 2, dtype=torch.float32, device=x.device)
    deq = torch.empty_like(xf)
    a = N.QuantArgs(num_groups=N_, group_elems=xf[0].numel() if N_ else 1, x=N.ptr(xf), codes=N.ptr(codes),
                    scale=N.ptr(scale), minmax=N.ptr(minmax), dequant=N.ptr(deq))
    N.check(lib, lib.spx_quantize_int8(a, N.stream_handle(x.device)), "spx_quantize_int8")
    return codes, scale, minmax, deq


def rsvd(M: torch.Tensor, omega: torch.Tensor, k: int, n_iter: int, *, want_factors: bool = True,
         codes: Optional[torch.Tensor] = None, codes_strides=None, rank_pad: Optional[int] = None,
         qscale: Optional[torch.Tensor] = None, scale_stride: int = 1, qminmax: Optional[torch.Tensor] = None,
         minmax_stride: int = 2, basis: Optional[torch.Tensor] = None, basis_stride: int = 0,
         M_mat_stride: int = 0, num_mats: Optional[int] = None, m: Optional[int] = None,
         n: Optional[int] = None, codes_tiled: bool = False):
    """Run ``spx_rsvd_compress``.  ``M`` is ``[Nb, m, n]`` (or a strided view described by
    ``num_mats``/``m``/``n``/``M_mat_stride``); ``omega`` is ``[Nb, n, r]`` float32.
    Returns (U, S, Vh) float32 when ``want_factors``; compressed outputs are written in
    place into ``codes``/``qscale``/``qminmax``/``basis``."""
    lib = N.lib_for(M.device)
    if num_mats is None:
        num_mats, m, n = M.shape
    r = omega.shape[-1]
    omega = omega.to(torch.float32).contiguous()
    dev = M.device
    U = S = Vh = None
    if want_factors:
        U = torch.empty(num_mats, m, k, dtype=torch.float32, device=dev)
        S = torch.empty(num_mats, k, dtype=torch.float32, device=dev)
        Vh = torch.empty(num_mats, k, n, dtype=torch.float32, device=dev)
    cs = codes_strides or (0, 0, 0)
    a = N.RsvdArgs(num_mats=num_mats, m=m, n=n, k=k, r=r, n_iter=n_iter, in_dtype=N.dtype_code(M.dtype),
                   M=N.ptr(M), omega=N.ptr(omega), U=N.ptr(U), S=N.ptr(S), Vh=N.ptr(Vh),
                   M_mat_stride=M_mat_stride, codes=N.ptr(codes), codes_mat_stride=cs[0], codes_t_stride=cs[1],
                   codes_j_stride=cs[2], codes_rank_pad=rank_pad or k, codes_tiled=int(bool(codes_tiled)),
                   qscale=N.ptr(qscale),
                   scale_mat_stride=scale_stride, qminmax=N.ptr(qminmax), minmax_mat_stride=minmax_stride,
                   basis=N.ptr(basis), basis_dtype=N.dtype_code(basis.dtype) if basis is not None else 0,
                   basis_mat_stride=basis_stride)
    need = lib.spx_rsvd_workspace_size(a)
    if need == 0 and num_mats > 0:
        N.check(lib, lib.spx_rsvd_compress(a, N.stream_handle(dev)), "spx_rsvd_compress")
    ws = N.workspace(dev, need)
    a.workspace, a.workspace_bytes = N.ptr(ws), ws.numel()
    N.check(lib, lib.spx_rsvd_compress(a, N.stream_handle(dev)), "spx_rsvd_compress")
    return U, S, Vh


def decode_args(q: torch.Tensor, tiers, cos: torch.Tensor, sin: torch.Tensor, query_position: int, *,
                rope_mode: int, mask: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                out: Optional[torch.Tensor] = None, tied: Optional[bool] = None):
    """Build the ``spx_decode_args`` of a decode over ``tiers`` (no workspace set).
    Returns ``(args, out, keepalive)``; ``keepalive`` holds the temporaries the pointers
    refer to and must outlive the call."""
    dev = q.device
    L, B, Hq, D = q.shape
    t = tiers
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    cos32 = rope_table_f32(cos, dev)
    sin32 = rope_table_f32(sin, dev)
    if tied is None:
        tied = rope_tied(cos32, sin32)
    freq = rope_freq(cos32, sin32) if (tied or rope_mode == N.SPX_ROPE_DISTANCE) else None
    if out is None:
        out = torch.empty(L, B, Hq, D, dtype=t.dtype, device=dev)
    mask_u8 = None
    mask_stride = 0
    if mask is not None:
        T_total = t.num_blocks * t.block_size + t.hot_len
        mk = mask
        if mk.dim() == 4:
            mk = mk[:, :, -1, :]            # [B, H, T] for a single query row
        mk = mk.expand(B, Hq, mk.shape[-1])
        if mk.shape[-1] < T_total:
            raise ValueError(f"attention_mask covers {mk.shape[-1]} keys, cache holds {T_total}")
        mask_u8 = (mk != 0).to(device=dev, dtype=torch.uint8).contiguous()
        mask_stride = mask_u8.shape[-1]
    a = N.DecodeArgs(
        num_layers=L, batch=B, num_q_heads=Hq, num_kv_heads=t.num_heads, head_dim=D,
        block_size=t.block_size, num_blocks=t.num_blocks, block_capacity=t.block_capacity,
        rank_k=t.rank_k_pad, rank_v=t.rank_v_pad,
        hot_len=t.hot_len if getattr(t, "hot_bound", None) is None else min(max(t.hot_len, t.hot_bound),
                                                                              t.hot_capacity),
        hot_capacity=t.hot_capacity,
        dtype=N.dtype_code(t.dtype), rope_mode=rope_mode, rope_tied=int(bool(tied)), rope_len=cos32.shape[0],
        query_position=int(query_position), scale=float(scale), mask_stride=mask_stride,
        q=N.ptr(q), codes_k=N.ptr(t.codes_k), codes_v=N.ptr(t.codes_v), scale_k=N.ptr(t.scale_k),
        scale_v=N.ptr(t.scale_v), basis_k=N.ptr(t.basis_k), basis_v=N.ptr(t.basis_v),
        block_pos=N.ptr(t.block_pos), hot_k=N.ptr(t.hot_k), hot_v=N.ptr(t.hot_v), hot_pos=N.ptr(t.hot_pos),
        cos_table=N.ptr(cos32), sin_table=N.ptr(sin32), mask=N.ptr(mask_u8), out=N.ptr(out),
        rope_freq=N.ptr(freq),
        hot_len_device=N.ptr(t.hot_len_device()) if hasattr(t, "hot_len_device") else None)
    return a, out, (q, cos32, sin32, mask_u8, freq)


def decode(q: torch.Tensor, tiers, cos: torch.Tensor, sin: torch.Tensor, query_position: int, *,
           rope_mode: int, mask: Optional[torch.Tensor] = None, scale: Optional[float] = None,
           out: Optional[torch.Tensor] = None, tied: Optional[bool] = None) -> torch.Tensor:
    """Run ``spx_decode_attn`` over ``tiers`` (a ``DeviceTiers``).  ``q`` is
    ``[L, B, H_q, D]`` in the tiers' dtype; returns ``[L, B, H_q, D]``."""
    dev = q.device
    lib = N.lib_for(dev)
    a, out, keep = decode_args(q, tiers, cos, sin, query_position, rope_mode=rope_mode, mask=mask, scale=scale,
                               out=out, tied=tied)
    need = lib.spx_decode_workspace_size(a)
    ws = N.workspace(dev, need)
    a.workspace, a.workspace_bytes = N.ptr(ws), ws.numel()
    N.check(lib, lib.spx_decode_attn(a, N.stream_handle(dev)), "spx_decode_attn")
    del keep
    return out


def prefill_supported(q: torch.Tensor, tiers) -> bool:
    """Shapes ``spx_prefill_attn`` covers: head_dim 128, f16/bf16, n_rep in {1,2,4,8},
    blocks a multiple of 64 tokens, stored ranks up to 64."""
    t = tiers
    if t is None or q.dim() != 4 or q.shape[-1] != 128 or t.dtype not in (torch.float16, torch.bfloat16):
        return False
    if q.dtype != t.dtype or q.shape[1] % t.num_heads or q.shape[1] // t.num_heads not in (1, 2, 4, 8):
        return False
    if t.num_blocks and (t.block_size % 64 or t.rank_k_pad > 64 or t.rank_v_pad > 64):
        return False
    return t.num_blocks > 0 or t.hot_len > 0


def prefill(q: torch.Tensor, tiers, cos: torch.Tensor, sin: torch.Tensor, q_pos: torch.Tensor, *,
            mask: Optional[torch.Tensor] = None, causal: bool = False, scale: Optional[float] = None) -> torch.Tensor:
    """``softmax(Q K^T * scale + mask) V`` over the compressed cache by ``spx_prefill_attn``
    (keys rebuilt from codes and bases, rotated at their cached positions inside the
    kernel).  ``q`` ``[B, H_q, T_q, D]`` (RoPE applied), ``q_pos`` ``[T_q]`` int64 positions,
    ``mask`` an optional additive mask broadcastable to ``[B, H_q, T_q, T_keys]`` over the
    keys in cache order; ``causal`` masks keys past each query's position.  Returns
    ``[B, H_q, T_q, D]`` in the cache dtype."""
    dev = q.device
    lib = N.lib_for(dev)
    t = tiers
    B, Hq, Tq, D = q.shape
    q = q.contiguous()
    cos32 = rope_table_f32(cos, dev)
    sin32 = rope_table_f32(sin, dev)
    qp = q_pos.reshape(-1).to(device=dev, dtype=torch.int64).contiguous()
    if qp.numel() != Tq:
        raise ValueError(f"q_pos has {qp.numel()} positions for {Tq} queries")
    out = torch.empty(B, Hq, Tq, D, dtype=t.dtype, device=dev)
    mk, mdt, strides = None, N.SPX_F32, (0, 0, 0)
    if mask is not None:
        T_total = t.num_blocks * t.block_size + t.hot_len
        if mask.shape[-1] != T_total:
            raise ValueError(f"attention_mask covers {mask.shape[-1]} keys, cache holds {T_total}")
        mk = mask.to(dev)
        if mk.dtype not in (torch.float32, t.dtype):
            mk = mk.float()
        while mk.dim() < 4:
            mk = mk.unsqueeze(0)
        mk = mk.expand(B, Hq, Tq, T_total)
        if mk.stride(-1) != 1:
            mk = mk.contiguous()
        mdt = N.SPX_F32 if mk.dtype == torch.float32 else N.dtype_code(mk.dtype)
        strides = (mk.stride(0), mk.stride(1), mk.stride(2))
    a = N.PrefillArgs(
        batch=B, num_q_heads=Hq, num_kv_heads=t.num_heads, head_dim=D, q_len=Tq, block_size=t.block_size,
        num_blocks=t.num_blocks, block_capacity=t.block_capacity, rank_k=t.rank_k_pad, rank_v=t.rank_v_pad,
        hot_len=t.hot_len, hot_capacity=t.hot_capacity, dtype=N.dtype_code(t.dtype), rope_len=cos32.shape[0],
        causal=int(bool(causal)), mask_dtype=mdt, scale=float(1.0 / math.sqrt(D) if scale is None else scale),
        q=N.ptr(q), q_pos=N.ptr(qp), codes_k=N.ptr(t.codes_k), codes_v=N.ptr(t.codes_v), scale_k=N.ptr(t.scale_k),
        scale_v=N.ptr(t.scale_v), basis_k=N.ptr(t.basis_k), basis_v=N.ptr(t.basis_v), block_pos=N.ptr(t.block_pos),
        hot_k=N.ptr(t.hot_k), hot_v=N.ptr(t.hot_v), hot_pos=N.ptr(t.hot_pos), cos_table=N.ptr(cos32),
        sin_table=N.ptr(sin32), mask=N.ptr(mk), mask_stride_b=strides[0], mask_stride_h=strides[1],
        mask_stride_q=strides[2], out=N.ptr(out))
    N.check(lib, lib.spx_prefill_attn(a, N.stream_handle(dev)), "spx_prefill_attn")
    del mk, qp, cos32, sin32
    return out


def reconstruct(codes, scale, basis, *, batch, num_heads, head_dim, block_size, num_blocks, block_capacity, rank,
                rank_major, out, out_tokens):
    lib = N.lib_for(out.device)
    a = N.ReconstructArgs(batch=batch, num_kv_heads=num_heads, head_dim=head_dim, block_size=block_size,
                          num_blocks=num_blocks, block_capacity=block_capacity, rank=rank,
                          rank_major=int(rank_major), dtype=N.dtype_code(out.dtype), out_tokens=out_tokens,
                          codes=N.ptr(codes), scale=N.ptr(scale), basis=N.ptr(basis), out=N.ptr(out))
    N.check(lib, lib.spx_reconstruct(a, N.stream_handle(out.device)), "spx_reconstruct")
    return out


def block_scores(q, coeffs, basis, cos, sin, start_position: int) -> torch.Tensor:
    """[B, H_q, T] float32 scores of one block (absolute-position RoPE)."""
    dev = q.device
    lib = N.lib_for(dev)
    B, Hq, _, D = q.shape
    H, T, R = coeffs.shape
    qf = q.reshape(B, Hq, D).to(torch.float32).contiguous()
    cf = coeffs.to(device=dev, dtype=torch.float32).contiguous()
    bf = basis.to(device=dev, dtype=torch.float32).contiguous()
    c32, s32 = rope_table_f32(cos, dev), rope_table_f32(sin, dev)
    out = torch.empty(B, Hq, T, dtype=torch.float32, device=dev)
    a = N.BlockScoreArgs(batch=B, num_q_heads=Hq, num_kv_heads=H, head_dim=D, block_size=T, rank=R,
                         rope_len=c32.shape[0], start_position=int(start_position), q=N.ptr(qf),
                         coeffs=N.ptr(cf), basis=N.ptr(bf), cos_table=N.ptr(c32), sin_table=N.ptr(s32),
                         scores=N.ptr(out))
    N.check(lib, lib.spx_block_scores(a, N.stream_handle(dev)), "spx_block_scores")
    return out


def block_values(attn, coeffs, basis) -> torch.Tensor:
    """[B, H_q, D] float32 values of one block."""
    dev = attn.device
    lib = N.lib_for(dev)
    B, Hq, _, T = attn.shape
    H, _, R = coeffs.shape
    D = basis.shape[-1]
    af = attn.reshape(B, Hq, T).to(torch.float32).contiguous()
    cf = coeffs.to(device=dev, dtype=torch.float32).contiguous()
    bf = basis.to(device=dev, dtype=torch.float32).contiguous()
    out = torch.empty(B, Hq, D, dtype=torch.float32, device=dev)
    a = N.BlockValueArgs(batch=B, num_q_heads=Hq, num_kv_heads=H, head_dim=D, block_size=T, rank=R,
                         attn=N.ptr(af), coeffs=N.ptr(cf), basis=N.ptr(bf), out=N.ptr(out))
    N.check(lib, lib.spx_block_values(a, N.stream_handle(dev)), "spx_block_values")
    return out
