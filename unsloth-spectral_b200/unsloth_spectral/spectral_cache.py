"""Three-tier KV cache with device-resident tiers.

Same constructor, attributes and methods as the reference's ``SpectralCache``
(unsloth_spectral/spectral_cache.py:49-705), with a different storage model:

* hot tier: preallocated ``[B, H, HC, D]`` K/V buffers in the cache dtype plus an int64
  position buffer; ``append`` copies into them (no ``torch.cat`` reallocation);
* cold tier: preallocated INT8 codes (keys token-major ``[B, H, NBc, T, RK]``, values in
  the value-tile layout ``[B, H, NBc, RV*T]`` of ``include/spx.h``), one float32 scale and (min, max) per
  (sequence, head, block), bases ``[B, H, NBc, R, D]`` in the cache dtype, and the
  blocks' start positions.  Stored ranks are padded to multiples of 16 with zeros;
* compression runs the batched rSVD + INT8 kernels of ``libspx`` and writes straight
  into the next cold slot (spectral_cache.py:243-407).

``cold_blocks``, ``hot_K``, ``hot_V`` and ``hot_position_ids`` remain available as
reference-layout views (``cold_blocks`` dequantises on access).  Batch sizes above 1
are supported; positions are shared by the batch (the reference reads row 0 too).
Attention-importance tracking and landmark tokens keep the reference's behaviour as
cache state; as in the reference, no entry point consumes them.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch

from . import _native as N
from . import _ops


@dataclass
class SpectralBlock:
    """One compressed block in the reference's layout (spectral_cache.py:20-46):
    ``K ~= coeffs_K @ basis_K``, ``V ~= coeffs_V @ basis_V``; coeffs are dequantised
    INT8 values in the cache dtype, scales are ``(min, max)`` per head."""
    coeffs_K: torch.Tensor
    basis_K: torch.Tensor
    coeffs_V: torch.Tensor
    basis_V: torch.Tensor
    scales_K: torch.Tensor
    scales_V: torch.Tensor
    block_size: int
    start_position: int


def _pad16(k: int) -> int:
    return max(16, (k + 15) // 16 * 16)


class DeviceTiers:
    """Storage of one cache (one layer): the pointers ``spx_decode_attn`` consumes."""

    def __init__(self, batch, num_heads, head_dim, block_size, rank_k, rank_v, dtype, device,
                 block_capacity=4, hot_capacity=None):
        self.batch, self.num_heads, self.head_dim = batch, num_heads, head_dim
        self.block_size, self.dtype, self.device = block_size, dtype, torch.device(device)
        self.rank_k, self.rank_v = rank_k, rank_v
        self.rank_k_pad, self.rank_v_pad = _pad16(rank_k), _pad16(rank_v)
        self.num_blocks = 0
        # hot-tier length: a host int and a device int32 copy the decode kernels read (so
        # a decode step can be replayed from a CUDA graph while the tier grows).  Host-side
        # assignments mark the device copy stale; hot_len_device() refreshes it, and
        # advance_hot() moves both by device arithmetic only.
        self._hot_len = 0
        self._hot_stale = False
        self._hot_len_dev = torch.zeros((), dtype=torch.int32, device=self.device)
        self.hot_bound = None   # launch bound for the hot tier while a CUDA graph replays steps
        self.block_capacity = 0
        self.hot_capacity = 0
        self._alloc_cold(block_capacity)
        self._alloc_hot(hot_capacity or (block_size + 64))

    @property
    def hot_len(self) -> int:
        return self._hot_len

    @hot_len.setter
    def hot_len(self, n: int):
        self._hot_len = int(n)
        self._hot_stale = True

    def hot_len_device(self) -> torch.Tensor:
        """Device int32 copy of the hot length, refreshed after host-side changes."""
        if self._hot_stale:
            self._hot_len_dev.fill_(self._hot_len)
            self._hot_stale = False
        return self._hot_len_dev

    def advance_hot(self, n: int):
        """Grow the hot length by n on the host and, by a device add, on the device."""
        self.hot_len_device().add_(n)
        self._hot_len += n

    # -- allocation --------------------------------------------------------------
    def _alloc_cold(self, cap):
        B, H, T, D = self.batch, self.num_heads, self.block_size, self.head_dim
        dev, dt = self.device, self.dtype
        new = dict(
            codes_k=torch.zeros(B, H, cap, T, self.rank_k_pad, dtype=torch.int8, device=dev),
            codes_v=torch.zeros(B, H, cap, self.rank_v_pad * T, dtype=torch.int8, device=dev),
            scale_k=torch.zeros(B, H, cap, dtype=torch.float32, device=dev),
            scale_v=torch.zeros(B, H, cap, dtype=torch.float32, device=dev),
            minmax_k=torch.zeros(B, H, cap, 2, dtype=torch.float32, device=dev),
            minmax_v=torch.zeros(B, H, cap, 2, dtype=torch.float32, device=dev),
            basis_k=torch.zeros(B, H, cap, self.rank_k_pad, D, dtype=dt, device=dev),
            basis_v=torch.zeros(B, H, cap, self.rank_v_pad, D, dtype=dt, device=dev),
            block_pos=torch.zeros(cap, dtype=torch.int64, device=dev),
        )
        n = self.num_blocks
        if n:
            for name, t in new.items():
                old = getattr(self, name)
                if name == "block_pos":
                    t[:n] = old[:n]
                else:
                    t[:, :, :n] = old[:, :, :n]
        for name, t in new.items():
            setattr(self, name, t)
        self.block_capacity = cap

    def _alloc_hot(self, cap):
        B, H, D = self.batch, self.num_heads, self.head_dim
        hk = torch.zeros(B, H, cap, D, dtype=self.dtype, device=self.device)
        hv = torch.zeros(B, H, cap, D, dtype=self.dtype, device=self.device)
        hp = torch.zeros(cap, dtype=torch.int64, device=self.device)
        n = self.hot_len
        if n:
            hk[:, :, :n] = self.hot_k[:, :, :n]
            hv[:, :, :n] = self.hot_v[:, :, :n]
            hp[:n] = self.hot_pos[:n]
        self.hot_k, self.hot_v, self.hot_pos = hk, hv, hp
        self.hot_capacity = cap

    def ensure_blocks(self, n):
        if n > self.block_capacity:
            self._alloc_cold(max(n, 2 * self.block_capacity))

    def ensure_hot(self, n):
        if n > self.hot_capacity:
            self._alloc_hot(max(n, 2 * self.hot_capacity))

    def nbytes(self) -> int:
        names = ("codes_k", "codes_v", "scale_k", "scale_v", "minmax_k", "minmax_v", "basis_k", "basis_v",
                 "block_pos", "hot_k", "hot_v", "hot_pos")
        return sum(getattr(self, n).numel() * getattr(self, n).element_size() for n in names)


class SpectralCache:
    """Three-tier KV cache with automatic spectral compression (see module docstring).

    Args (as the reference's, spectral_cache.py:72-87):
        num_heads: KV heads; head_dim; block_size: tokens per compressed block;
        k_rank_keys / k_rank_values: spectral ranks; hot_buffer_size: kept for API
        compatibility (the reference stores it without using it); device; dtype of the
        uncompressed tiers and bases; debug_logging.
    Extensions: ``oversampling`` and ``n_iter`` of the rSVD (the reference hard-codes
    5 and 2 at spectral_cache.py:374), ``block_capacity`` preallocated cold slots.
    """

    def __init__(self, num_heads: int, head_dim: int, block_size: int = 512, k_rank_keys: int = 16,
                 k_rank_values: int = 32, hot_buffer_size: int = 64, device="cuda",
                 dtype: torch.dtype = torch.float16, debug_logging: bool = False,
                 use_attention_weighted_svd: bool = False, landmark_positions: Optional[List[int]] = None,
                 landmark_count: int = 0, *, oversampling: int = 5, n_iter: int = 2, block_capacity: int = 4):
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.k_rank_keys = k_rank_keys
        self.k_rank_values = k_rank_values
        self.hot_buffer_size = hot_buffer_size
        self.device = device
        self.dtype = dtype
        self.debug_logging = debug_logging
        self.use_attention_weighted_svd = use_attention_weighted_svd
        self.landmark_positions = set(landmark_positions) if landmark_positions else set()
        self.landmark_count = landmark_count
        self.landmark_K = self.landmark_V = self.landmark_position_ids = None
        self.attention_importance = None
        self.oversampling = oversampling
        self.n_iter = n_iter
        self._block_capacity = block_capacity
        self.tiers: Optional[DeviceTiers] = None
        self.current_position = 0
        self.total_tokens = 0
        self.compression_count = 0
        self.cache_id = id(self)
        self._blocks_view = None
        if debug_logging:
            print(f"[SpectralCache.__init__] id={self.cache_id} H={num_heads} D={head_dim} "
                  f"block={block_size} kK={k_rank_keys} kV={k_rank_values}")

    # -- storage ---------------------------------------------------------------------
    def _tiers_for(self, batch: int, device) -> DeviceTiers:
        if self.tiers is None:
            self.tiers = DeviceTiers(batch, self.num_heads, self.head_dim, self.block_size, self.k_rank_keys,
                                     self.k_rank_values, self.dtype, device, self._block_capacity)
        elif self.tiers.batch != batch:
            raise ValueError(f"cache holds batch {self.tiers.batch}, got {batch}")
        return self.tiers

    @property
    def num_cold_blocks(self) -> int:
        return 0 if self.tiers is None else self.tiers.num_blocks

    @property
    def hot_len(self) -> int:
        return 0 if self.tiers is None else self.tiers.hot_len

    def reset(self):
        """Start a new generation (spectral_cache.py:137-162); buffers are kept."""
        if self.tiers is not None:
            self.tiers.num_blocks = 0
            self.tiers.hot_len = 0
        self.landmark_K = self.landmark_V = self.landmark_position_ids = None
        self.attention_importance = None
        self.current_position = 0
        self.total_tokens = 0
        self.compression_count = 0
        self._blocks_view = None

    # -- serialisation -----------------------------------------------------------------
    _COLD = ("codes_k", "codes_v", "scale_k", "scale_v", "minmax_k", "minmax_v", "basis_k", "basis_v")
    _GEOMETRY = ("num_heads", "head_dim", "block_size", "k_rank_keys", "k_rank_values")

    def state_dict(self) -> dict:
        """The cache's contents as tensors and numbers, for checkpointing a compressed
        cache (e.g. with ``torch.save``): the used part of every tier - INT8 codes (value
        codes in their stored tile layout), scales, min/max, bases and start positions of
        the cold blocks, the hot tier's K, V and positions - plus the geometry and the
        counters.  The tensors are copies on the cache's device.  The reference keeps its
        cache in memory only (spectral_cache.py:49-705 has no serialisation)."""
        sd = {name: getattr(self, name) for name in self._GEOMETRY}
        sd.update(version=1, dtype=str(self.dtype), oversampling=self.oversampling, n_iter=self.n_iter,
                  current_position=self.current_position, total_tokens=self.total_tokens,
                  compression_count=self.compression_count, batch=0)
        t = self.tiers
        if t is not None:
            n, h = t.num_blocks, t.hot_len
            sd["batch"] = t.batch
            for name in self._COLD:
                sd[name] = getattr(t, name)[:, :, :n].clone()
            sd["block_pos"] = t.block_pos[:n].clone()
            sd["hot_k"] = t.hot_k[:, :, :h].clone()
            sd["hot_v"] = t.hot_v[:, :, :h].clone()
            sd["hot_pos"] = t.hot_pos[:h].clone()
        return sd

    def load_state_dict(self, sd: dict):
        """Restore what ``state_dict`` returned.  The geometry (heads, head dim, block size,
        ranks) and dtype must match this cache's (ValueError otherwise); the tensors are
        copied to the cache's device, replacing its contents."""
        for name in self._GEOMETRY:
            if sd[name] != getattr(self, name):
                raise ValueError(f"state has {name}={sd[name]}, cache has {getattr(self, name)}")
        if sd["dtype"] != str(self.dtype):
            raise ValueError(f"state has dtype {sd['dtype']}, cache has {self.dtype}")
        self.reset()
        if self.tiers is not None and self.tiers.batch != sd["batch"]:
            self.tiers = None
        if sd["batch"]:
            t = self._tiers_for(sd["batch"], self.device)
            n, h = sd["block_pos"].shape[0], sd["hot_pos"].shape[0]
            t.ensure_blocks(n)
            for name in self._COLD:
                getattr(t, name)[:, :, :n].copy_(sd[name])
            t.block_pos[:n].copy_(sd["block_pos"])
            t.num_blocks = n
            t.ensure_hot(h)
            t.hot_k[:, :, :h].copy_(sd["hot_k"])
            t.hot_v[:, :, :h].copy_(sd["hot_v"])
            t.hot_pos[:h].copy_(sd["hot_pos"])
            t.hot_len = h
        self.oversampling, self.n_iter = sd["oversampling"], sd["n_iter"]
        self.current_position, self.total_tokens = sd["current_position"], sd["total_tokens"]
        self.compression_count = sd["compression_count"]
        self._blocks_view = None

    # -- append / compression ------------------------------------------------------
    def append(self, K_new: torch.Tensor, V_new: torch.Tensor, position_ids: Optional[torch.Tensor] = None):
        """Append pre-RoPE ``K_new``/``V_new`` ``[B, H, T_new, D]`` (spectral_cache.py:164-241).

        A new generation (first position below ``current_position``) resets the cache,
        as in the reference (spectral_cache.py:176-186).  The reference reads that first
        position with ``.item()`` on every append; here it is read only when it costs no
        device sync on the decode path: CPU ``position_ids`` are always checked, device
        ``position_ids`` only for a multi-token append (a prompt).  A single-token append
        with device positions continues the sequence, so a new generation must start
        with a prompt, with CPU positions or with ``reset()``."""
        B, H, T_new, D = K_new.shape
        if position_ids is not None and self.total_tokens > 0 and (position_ids.device.type == "cpu" or T_new > 1):
            first = int(position_ids.reshape(-1)[0].item())
            if first < self.current_position:
                if self.debug_logging:
                    print(f"[SpectralCache.append] new generation at {first} < {self.current_position}: reset")
                self.reset()
        if H != self.num_heads or D != self.head_dim:
            raise ValueError(f"expected [B, {self.num_heads}, T, {self.head_dim}], got {tuple(K_new.shape)}")
        t = self._tiers_for(B, K_new.device)
        n0 = t.hot_len
        t.ensure_hot(n0 + T_new)
        pid = None
        if position_ids is not None:
            pid = position_ids.reshape(-1, position_ids.shape[-1])[0] if position_ids.dim() > 1 else position_ids
        if T_new == 1 and pid is not None and pid.device == t.device:
            # a decode token: written at the device hot length, which advances on the
            # device, so the step has no host-dependent addresses (CUDA-graph safe)
            if (t.device.type == "cuda" and K_new.dtype == t.dtype and V_new.dtype == t.dtype
                    and K_new.stride(-1) == 1 and V_new.stride(-1) == 1):
                # one launch (spx_hot_append): rows, position and the length advance
                _ops.hot_append(K_new, V_new, t.hot_k, t.hot_v, t.hot_pos, t.hot_len_device(),
                                pid.reshape(1).to(torch.int64))
                t._hot_len += 1
            else:
                idx = t.hot_len_device().view(1).long()
                t.hot_k.index_copy_(2, idx, K_new.to(t.dtype))
                t.hot_v.index_copy_(2, idx, V_new.to(t.dtype))
                t.hot_pos.index_copy_(0, idx, pid.reshape(1).to(torch.int64))
                t.advance_hot(1)
        else:
            t.hot_k[:, :, n0:n0 + T_new].copy_(K_new)
            t.hot_v[:, :, n0:n0 + T_new].copy_(V_new)
            if pid is None:
                t.hot_pos[n0:n0 + T_new] = torch.arange(self.current_position, self.current_position + T_new,
                                                        device=t.device)
            else:
                t.hot_pos[n0:n0 + T_new].copy_(pid.to(torch.int64), non_blocking=True)
            t.hot_len = n0 + T_new
        self.total_tokens += T_new
        self.current_position += T_new
        self._blocks_view = None
        if t.hot_len >= self.block_size:
            self._compress_hot_cache()

    def _compress_hot_cache(self):
        """Compress every full block at the front of the hot tier into the cold tier
        (spectral_cache.py:243-319): K then V per block, as the reference orders its
        sketch draws, then move the remainder to the front."""
        t = self.tiers
        T = self.block_size
        nfull = t.hot_len // T
        if nfull == 0:
            return
        t.ensure_blocks(t.num_blocks + nfull)
        j0 = t.num_blocks
        if nfull == 1:
            self._compress_into(t.hot_k, 0, j0, keys=True)
            self._compress_into(t.hot_v, 0, j0, keys=False)
        else:
            self._compress_blocks(nfull, j0)
        t.block_pos[j0:j0 + nfull] = t.hot_pos[0:nfull * T:T]
        t.num_blocks += nfull
        self.compression_count += nfull
        rem = t.hot_len - nfull * T
        if rem:
            t.hot_k[:, :, :rem] = t.hot_k[:, :, nfull * T:nfull * T + rem].clone()
            t.hot_v[:, :, :rem] = t.hot_v[:, :, nfull * T:nfull * T + rem].clone()
            t.hot_pos[:rem] = t.hot_pos[nfull * T:nfull * T + rem].clone()
        t.hot_len = rem
        self._blocks_view = None

    def _compress_into(self, hot: torch.Tensor, t0: int, j: int, keys: bool):
        t = self.tiers
        B, H, HC, D = hot.shape
        T = self.block_size
        k = self.k_rank_keys if keys else self.k_rank_values
        r = min(k + self.oversampling, min(T, D))
        nm = B * H
        # sketch drawn as rsvd.py:95 does: float32 randn of [mats, n, r] from the global RNG
        omega = torch.randn(nm, D, r, device=hot.device, dtype=torch.float32)
        Mview = hot[:, :, t0:t0 + T]
        if keys:
            codes, kp = t.codes_k, t.rank_k_pad
            cstr = (t.block_capacity * T * kp, kp, 1)     # token-major
            basis, scale, mm = t.basis_k, t.scale_k, t.minmax_k
        else:
            codes, kp = t.codes_v, t.rank_v_pad
            cstr = (t.block_capacity * kp * T, 0, 0)      # value-tile layout
            basis, scale, mm = t.basis_v, t.scale_v, t.minmax_v
        if r >= min(T, D) - 1:
            raise ValueError(f"rank {k} + oversampling {self.oversampling} too large for {T}x{D} blocks")
        _ops.rsvd(Mview, omega, k, self.n_iter, want_factors=False,
                  codes=codes[:, :, j], codes_strides=cstr, rank_pad=kp,
                  qscale=scale[:, :, j], scale_stride=t.block_capacity,
                  qminmax=mm[:, :, j], minmax_stride=2 * t.block_capacity,
                  basis=basis[:, :, j], basis_stride=t.block_capacity * kp * D,
                  M_mat_stride=HC * D, num_mats=nm, m=T, n=D, codes_tiled=not keys)

    def _compress_blocks(self, nfull: int, j0: int):
        """Compress the first ``nfull`` blocks of the hot tier (a long prompt) with one
        rSVD launch for the keys and one for the values, instead of two per block.  The
        sketches are drawn first, in the order of the per-block path (K then V of each
        block, as the reference draws them), and every matrix is computed independently
        of the others in its launch, so the cold tier comes out bit-identical to
        compressing block by block.  The blocks are staged contiguously (one copy of the
        prompt's K and V) and the outputs go to contiguous buffers that are then copied
        into block slots ``j0 .. j0 + nfull - 1``."""
        t = self.tiers
        B, H, HC, D = t.hot_k.shape
        T = self.block_size
        nm = B * H
        dev = t.hot_k.device
        spec = []
        for keys in (True, False):
            k = self.k_rank_keys if keys else self.k_rank_values
            r = min(k + self.oversampling, min(T, D))
            if r >= min(T, D) - 1:
                raise ValueError(f"rank {k} + oversampling {self.oversampling} too large for {T}x{D} blocks")
            spec.append((keys, k, r))
        omegas = {True: [], False: []}
        for _ in range(nfull):
            for keys, _k, r in spec:
                # drawn as rsvd.py:95 does: float32 randn of [mats, n, r] from the global RNG
                omegas[keys].append(torch.randn(nm, D, r, device=dev, dtype=torch.float32))
        for keys, k, r in spec:
            hot = t.hot_k if keys else t.hot_v
            X = hot[:, :, :nfull * T].reshape(B, H, nfull, T, D).permute(2, 0, 1, 3, 4).contiguous()
            omega = torch.cat(omegas[keys], dim=0)   # matrices ordered (block, sequence, head)
            kp = t.rank_k_pad if keys else t.rank_v_pad
            if keys:
                codes = torch.empty(nfull, B, H, T, kp, dtype=torch.int8, device=dev)
                cstr = (T * kp, kp, 1)                 # token-major
            else:
                codes = torch.empty(nfull, B, H, kp * T, dtype=torch.int8, device=dev)
                cstr = (kp * T, 0, 0)                  # value-tile layout
            scale = torch.empty(nfull, B, H, dtype=torch.float32, device=dev)
            mm = torch.empty(nfull, B, H, 2, dtype=torch.float32, device=dev)
            basis = torch.empty(nfull, B, H, kp, D, dtype=t.dtype, device=dev)
            _ops.rsvd(X, omega, k, self.n_iter, want_factors=False,
                      codes=codes, codes_strides=cstr, rank_pad=kp,
                      qscale=scale, scale_stride=1, qminmax=mm, minmax_stride=2,
                      basis=basis, basis_stride=kp * D,
                      M_mat_stride=T * D, num_mats=nfull * nm, m=T, n=D, codes_tiled=not keys)
            dst = slice(j0, j0 + nfull)
            if keys:
                t.codes_k[:, :, dst] = codes.permute(1, 2, 0, 3, 4)
                t.scale_k[:, :, dst] = scale.permute(1, 2, 0)
                t.minmax_k[:, :, dst] = mm.permute(1, 2, 0, 3)
                t.basis_k[:, :, dst] = basis.permute(1, 2, 0, 3, 4)
            else:
                t.codes_v[:, :, dst] = codes.permute(1, 2, 0, 3)
                t.scale_v[:, :, dst] = scale.permute(1, 2, 0)
                t.minmax_v[:, :, dst] = mm.permute(1, 2, 0, 3)
                t.basis_v[:, :, dst] = basis.permute(1, 2, 0, 3, 4)

    def note_replayed_tokens(self, n: int = 1):
        """Host bookkeeping of ``n`` single-token appends that a replayed CUDA graph made
        on the device (the graph re-runs the kernels, not this Python): the counters
        ``append`` would have advanced.  The caller guarantees that none of these appends
        filled a block (no compression happened)."""
        t = self.tiers
        t._hot_len += n
        self.total_tokens += n
        self.current_position += n
        self._blocks_view = None

    # -- reference-layout views -------------------------------------------------------
    @property
    def hot_K(self) -> Optional[torch.Tensor]:
        return None if self.hot_len == 0 else self.tiers.hot_k[:, :, :self.hot_len]

    @property
    def hot_V(self) -> Optional[torch.Tensor]:
        return None if self.hot_len == 0 else self.tiers.hot_v[:, :, :self.hot_len]

    @property
    def hot_position_ids(self) -> Optional[torch.Tensor]:
        return None if self.hot_len == 0 else self.tiers.hot_pos[:self.hot_len].unsqueeze(0)

    def set_hot(self, K: Optional[torch.Tensor], V: Optional[torch.Tensor],
                position_ids: Optional[torch.Tensor] = None):
        """Replace the hot tier (K/V ``[B, H, T, D]``, positions ``[T]`` or ``[1, T]``)."""
        if K is None:
            if self.tiers is not None:
                self.tiers.hot_len = 0
            return
        B, H, T, D = K.shape
        t = self._tiers_for(B, K.device)
        t.ensure_hot(T)
        t.hot_k[:, :, :T].copy_(K)
        t.hot_v[:, :, :T].copy_(V)
        if position_ids is None:
            start = t.num_blocks * self.block_size
            t.hot_pos[:T] = torch.arange(start, start + T, device=t.device)
        else:
            t.hot_pos[:T].copy_(position_ids.reshape(-1)[-T:].to(torch.int64))
        t.hot_len = T
        self._blocks_view = None

    def set_cold(self, codes_K, scale_K, basis_K, codes_V, scale_V, basis_V, start_positions,
                 minmax_K=None, minmax_V=None):
        """Replace the cold tier from integer codes.  Shapes (per sequence batch B):
        codes_K ``[B, H, nblk, T, k_K]``, codes_V ``[B, H, nblk, T, k_V]`` (token-major,
        as the reference's coeffs), scale ``[B, H, nblk]``, basis ``[B, H, nblk, k, D]``,
        start_positions ``[nblk]``."""
        B, H, nb, T, kK = codes_K.shape
        kV = codes_V.shape[-1]
        if T != self.block_size or kK > _pad16(self.k_rank_keys) or kV > _pad16(self.k_rank_values):
            raise ValueError("cold tier does not match the cache geometry")
        t = self._tiers_for(B, codes_K.device)
        t.ensure_blocks(nb)
        t.codes_k.zero_()
        t.codes_v.zero_()
        t.basis_k.zero_()
        t.basis_v.zero_()
        t.codes_k[:, :, :nb, :, :kK] = codes_K
        nat = torch.zeros(B, H, nb, t.rank_v_pad, T, dtype=torch.int8, device=t.device)
        nat[:, :, :, :kV, :] = codes_V.transpose(-1, -2)
        t.codes_v[:, :, :nb] = nat.reshape(B, H, nb, -1)[..., _ops.vtile_index(T, t.rank_v_pad, t.device)]
        t.scale_k[:, :, :nb] = scale_K
        t.scale_v[:, :, :nb] = scale_V
        t.basis_k[:, :, :nb, :kK] = basis_K.to(self.dtype)
        t.basis_v[:, :, :nb, :kV] = basis_V.to(self.dtype)
        if minmax_K is not None:
            t.minmax_k[:, :, :nb] = minmax_K
            t.minmax_v[:, :, :nb] = minmax_V
        t.block_pos[:nb] = torch.as_tensor(start_positions, dtype=torch.int64).to(t.device)
        t.num_blocks = nb
        self._blocks_view = None

    @hot_K.setter
    def hot_K(self, value):
        """Assigning ``hot_K`` replaces the hot keys and sets the hot length; positions
        default to the tokens right after the cold tier until ``hot_position_ids`` is
        assigned."""
        if value is None or value.shape[2] == 0:
            if self.tiers is not None:
                self.tiers.hot_len = 0
            return
        self.set_hot(value, torch.zeros_like(value), None)

    @hot_V.setter
    def hot_V(self, value):
        if value is None or value.shape[2] == 0:
            return
        t = self.tiers
        if t is None or t.hot_len != value.shape[2]:
            raise ValueError("assign hot_K before hot_V, with the same token count")
        t.hot_v[:, :, :t.hot_len].copy_(value)

    @hot_position_ids.setter
    def hot_position_ids(self, value):
        if value is None:
            return
        t = self.tiers
        v = value.reshape(-1)
        if t is None or t.hot_len != v.numel():
            raise ValueError("assign hot_K before hot_position_ids, with the same token count")
        t.hot_pos[:t.hot_len].copy_(v.to(torch.int64))

    @property
    def cold_blocks(self) -> List[SpectralBlock]:
        """The cold tier as reference ``SpectralBlock`` records (dequantised on access)."""
        if self._blocks_view is not None:
            return self._blocks_view
        t = self.tiers
        out = []
        if t is not None and t.num_blocks:
            starts = t.block_pos[:t.num_blocks].tolist()
            kK, kV = self.k_rank_keys, self.k_rank_values
            for j in range(t.num_blocks):
                ck = (t.codes_k[:, :, j, :, :kK].float() * t.scale_k[:, :, j, None, None]).to(self.dtype)
                nat = torch.empty_like(t.codes_v[:, :, j])
                nat[..., _ops.vtile_index(self.block_size, t.rank_v_pad, t.device)] = t.codes_v[:, :, j]
                nat = nat.view(t.batch, t.num_heads, t.rank_v_pad, self.block_size)
                cv = (nat[:, :, :kV, :].transpose(-1, -2).float()
                      * t.scale_v[:, :, j, None, None]).to(self.dtype)
                bk = t.basis_k[:, :, j, :kK]
                bv = t.basis_v[:, :, j, :kV]
                mk, mv = t.minmax_k[:, :, j], t.minmax_v[:, :, j]
                if t.batch == 1:
                    ck, cv, bk, bv, mk, mv = ck[0], cv[0], bk[0], bv[0], mk[0], mv[0]
                out.append(SpectralBlock(ck, bk, cv, bv, mk, mv, self.block_size, int(starts[j])))
        self._blocks_view = out
        return out

    @cold_blocks.setter
    def cold_blocks(self, blocks: List[SpectralBlock]):
        """Load reference-style blocks (batch 1, coeffs ``[H, T, k]`` = code * scale)."""
        if not blocks:
            if self.tiers is not None:
                self.tiers.num_blocks = 0
            self._blocks_view = None
            return
        dev = blocks[0].coeffs_K.device if blocks[0].coeffs_K.is_cuda else torch.device(self.device)

        def codes_of(c, mm):
            mm = mm.to(dev, torch.float32)
            s = torch.clamp(torch.maximum(-mm[:, 0], mm[:, 1]), min=1e-8) / 127.0
            return torch.round(c.to(dev, torch.float32) / s[:, None, None]).to(torch.int8), s

        ck, sk, cv, sv = [], [], [], []
        for b in blocks:
            c, s = codes_of(b.coeffs_K, b.scales_K)
            ck.append(c)
            sk.append(s)
            c, s = codes_of(b.coeffs_V, b.scales_V)
            cv.append(c)
            sv.append(s)
        self.set_cold(torch.stack(ck, 1)[None], torch.stack(sk, 1)[None],
                      torch.stack([b.basis_K.to(dev) for b in blocks], 1)[None],
                      torch.stack(cv, 1)[None], torch.stack(sv, 1)[None],
                      torch.stack([b.basis_V.to(dev) for b in blocks], 1)[None],
                      [b.start_position for b in blocks],
                      torch.stack([b.scales_K.to(dev) for b in blocks], 1)[None],
                      torch.stack([b.scales_V.to(dev) for b in blocks], 1)[None])

    def get_spectral_components(self) -> Tuple[List[SpectralBlock], Optional[torch.Tensor], Optional[torch.Tensor]]:
        return self.cold_blocks, self.hot_K, self.hot_V

    def get_all_positions(self) -> torch.Tensor:
        """Positions of every cached token, cold blocks first (spectral_cache.py:529-555)."""
        t = self.tiers
        if t is None or (t.num_blocks == 0 and t.hot_len == 0):
            return torch.empty(0, dtype=torch.long, device=self.device)
        parts = []
        if t.num_blocks:
            ar = torch.arange(self.block_size, device=t.device)
            parts.append((t.block_pos[:t.num_blocks, None] + ar[None]).reshape(-1))
        if t.hot_len:
            parts.append(t.hot_pos[:t.hot_len])
        return torch.cat(parts)

    def get_kv(self) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
        """Reconstruct pre-RoPE K and V ``[B, H, T_total, D]`` (spectral_cache.py:557-612)."""
        t = self.tiers
        if t is None or (t.num_blocks == 0 and t.hot_len == 0):
            return None, None
        T = self.block_size
        nb = t.num_blocks
        total = nb * T + t.hot_len
        K = torch.empty(t.batch, t.num_heads, total, t.head_dim, dtype=self.dtype, device=t.device)
        V = torch.empty_like(K)
        if nb:
            common = dict(batch=t.batch, num_heads=t.num_heads, head_dim=t.head_dim, block_size=T, num_blocks=nb,
                          block_capacity=t.block_capacity, out_tokens=total)
            _ops.reconstruct(t.codes_k, t.scale_k, t.basis_k, rank=t.rank_k_pad, rank_major=False, out=K, **common)
            _ops.reconstruct(t.codes_v, t.scale_v, t.basis_v, rank=t.rank_v_pad, rank_major=True, out=V, **common)
        if t.hot_len:
            K[:, :, nb * T:] = t.hot_k[:, :, :t.hot_len]
            V[:, :, nb * T:] = t.hot_v[:, :, :t.hot_len]
        return K, V

    def get_memory_stats(self) -> dict:
        """Byte accounting with the reference's formula (spectral_cache.py:614-655), plus
        ``device_bytes``: what the preallocated tiers actually hold on the device."""
        B = self.tiers.batch if self.tiers is not None else 1
        original = self.total_tokens * self.num_heads * self.head_dim * 2 * 2 * B
        compressed = 0
        nb = self.num_cold_blocks
        H, T, D = self.num_heads, self.block_size, self.head_dim
        per_block = (H * T * self.k_rank_keys + H * T * self.k_rank_values
                     + (H * self.k_rank_keys * D + H * self.k_rank_values * D) * 2 + 2 * H * 2 * 4)
        compressed += nb * per_block * B
        compressed += 2 * B * H * self.hot_len * D * 2
        return {
            "original_bytes": original,
            "compressed_bytes": compressed,
            "compression_ratio": original / compressed if compressed > 0 else 1.0,
            "num_blocks": nb,
            "total_tokens": self.total_tokens,
            "device_bytes": self.tiers.nbytes() if self.tiers is not None else 0,
        }

    # -- container protocol -------------------------------------------------------------
    def __len__(self):
        return self.total_tokens

    def __getitem__(self, index):
        if index == 0:
            return self.get_kv()[0]
        if index == 1:
            return self.get_kv()[1]
        raise IndexError(f"SpectralCache subscript index out of range: {index} (expected 0 or 1)")

    def __iter__(self):
        K, V = self.get_kv()
        yield K
        yield V

    def __repr__(self):
        s = self.get_memory_stats()
        return (f"SpectralCache(tokens={self.total_tokens}, blocks={s['num_blocks']}, "
                f"compression={s['compression_ratio']:.2f}x)")

    # -- attention importance and landmark tokens (spectral_cache.py:706-852) ------------
    # The reference keeps these as cache state that no entry point of its own consumes:
    # nothing calls update_attention_importance, compression does not read the weights,
    # and the attention paths read get_kv, not get_kv_with_landmarks.  They are kept with
    # the same behaviour for callers that use them directly.
    def update_attention_importance(self, attention_weights: torch.Tensor, query_position: int):
        """Exponential moving average (alpha 0.1) of the attention ``[B, H, 1, T_kv]`` a
        query paid to each cached token, averaged over batch, heads and queries; grows with
        the cache (spectral_cache.py:710-750).  No-op unless use_attention_weighted_svd."""
        if not self.use_attention_weighted_svd:
            return
        avg = attention_weights.mean(dim=(0, 1, 2))
        if self.attention_importance is None:
            self.attention_importance = avg.clone()
            return
        alpha = 0.1
        if self.attention_importance.shape[0] < avg.shape[0]:
            pad = torch.zeros(avg.shape[0] - self.attention_importance.shape[0], device=avg.device, dtype=avg.dtype)
            self.attention_importance = torch.cat([self.attention_importance, pad])
        n = avg.shape[0]
        self.attention_importance[:n] = (1 - alpha) * self.attention_importance[:n] + alpha * avg

    def get_block_attention_weights(self, block_idx: int) -> Optional[torch.Tensor]:
        """Importance of the tokens of block ``block_idx`` ``[block_size]``, or None when
        not tracked (or not yet covering the block) (spectral_cache.py:752-775)."""
        if self.attention_importance is None:
            return None
        start = block_idx * self.block_size
        end = start + self.block_size
        if end > self.attention_importance.shape[0]:
            return None
        return self.attention_importance[start:end]

    def add_landmarks(self, K: torch.Tensor, V: torch.Tensor, position_ids: torch.Tensor):
        """Keep tokens ``[B, H, T, D]`` uncompressed as landmarks (spectral_cache.py:781-806)."""
        if self.landmark_K is None:
            self.landmark_K, self.landmark_V = K.clone(), V.clone()
            self.landmark_position_ids = position_ids.clone()
        else:
            self.landmark_K = torch.cat([self.landmark_K, K], dim=2)
            self.landmark_V = torch.cat([self.landmark_V, V], dim=2)
            self.landmark_position_ids = torch.cat([self.landmark_position_ids, position_ids], dim=1)
        if self.debug_logging:
            print(f"[SpectralCache] Added {K.shape[2]} landmark tokens; total {self.landmark_K.shape[2]}")

    def get_kv_with_landmarks(self) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor], Optional[torch.Tensor]]:
        """Landmarks, then the cold blocks (reconstructed), then the hot tier:
        ``(K [B, H, T, D], V, position_ids [B, T])`` (spectral_cache.py:808-852)."""
        K, V = self.get_kv()
        pos = self.get_all_positions()
        Ks, Vs, Ps = [], [], []
        if self.landmark_K is not None:
            Ks.append(self.landmark_K)
            Vs.append(self.landmark_V)
            if self.landmark_position_ids is not None:
                Ps.append(self.landmark_position_ids.to(pos.device if pos.numel() else self.landmark_K.device))
        if K is not None:
            Ks.append(K.to(self.landmark_K.dtype) if self.landmark_K is not None else K)
            Vs.append(V.to(self.landmark_V.dtype) if self.landmark_V is not None else V)
            Ps.append(pos[None].expand(K.shape[0], -1))
        if not Ks:
            return None, None, None
        B = Ks[0].shape[0]
        Ps = [p.expand(B, -1) if p.shape[0] == 1 else p for p in Ps]
        return torch.cat(Ks, dim=2), torch.cat(Vs, dim=2), (torch.cat(Ps, dim=1) if Ps else None)
