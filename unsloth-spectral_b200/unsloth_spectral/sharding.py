"""Decode sharded by KV head across the GPUs of one node.

Attention is independent per KV head, so rank ``r`` of ``world`` owns KV heads
``[r*H/world, (r+1)*H/world)`` of every layer's cache (codes, scales, bases, hot tier)
and the ``n_rep`` query heads of each; it decodes that slice on its own GPU with no
communication.  The only collective is one all-gather of the per-rank attention
outputs ``[L, B, H_q/world, D]`` (NCCL over NVLink on GPUs, gloo on CPU), assembled in
the global head order so that the gathered tensor equals the single-GPU output.  The
reference decodes on one device (kernels/spectral_attention.py:684-857); this module
is the multi-GPU layout of the same computation.

``HeadShardGather`` runs the all-gather on a side stream: the gather of step ``i``
overlaps the decode of step ``i + 1``, which writes the other of two output buffers.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def head_slice(num_kv_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """KV heads ``[h0, h1)`` owned by ``rank``; ``num_kv_heads`` must divide evenly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads do not split across {world} ranks")
    n = num_kv_heads // world
    return rank * n, (rank + 1) * n


def shard_heads(x: torch.Tensor, world: int, rank: int, dim: int = 1) -> torch.Tensor:
    """The slice of ``x`` along its KV-head dimension ``dim`` that ``rank`` owns."""
    h0, h1 = head_slice(x.shape[dim], world, rank)
    return x.narrow(dim, h0, h1 - h0)


def shard_query_heads(q: torch.Tensor, num_kv_heads: int, world: int, rank: int, dim: int = 2) -> torch.Tensor:
    """The query heads of ``rank``'s KV heads: q-head ``h`` reads KV head ``h // n_rep``,
    so the owned query heads are ``[h0*n_rep, h1*n_rep)``."""
    nrep = q.shape[dim] // num_kv_heads
    h0, h1 = head_slice(num_kv_heads, world, rank)
    return q.narrow(dim, h0 * nrep, (h1 - h0) * nrep)


def assemble(gathered: torch.Tensor) -> torch.Tensor:
    """``[world, L, B, Hq_local, D]`` (rank-major, as an all-gather lays it out) ->
    ``[L, B, world * Hq_local, D]`` in the global query-head order."""
    w, L, B, Hl, D = gathered.shape
    return gathered.permute(1, 2, 0, 3, 4).reshape(L, B, w * Hl, D)


class HeadShardGather:
    """All-gather of this rank's decode outputs ``[L, B, Hq_local, D]`` into the full
    ``[L, B, H_q, D]`` layout.

    ``start(src)`` enqueues the gather of ``src`` (on a side stream for CUDA tensors, after
    the work already queued on the current stream); ``wait()`` makes the current stream
    wait for the last gather; ``assembled()`` returns the full output of the last gather
    (after ``wait()``).  Before the current stream overwrites a buffer that an earlier
    ``start`` is still reading, call ``wait()`` (or alternate two buffers and call
    ``release(src)``, which waits only for a gather that reads ``src``)."""

    def __init__(self, like: torch.Tensor, world: int, group: Optional[dist.ProcessGroup] = None):
        self.world = world
        self.group = group
        self.buf = torch.empty((world,) + tuple(like.shape), dtype=like.dtype, device=like.device)
        self.cuda = like.is_cuda
        self.side = torch.cuda.Stream(device=like.device) if self.cuda else None
        self.done = None
        self._reading = {}   # data_ptr of a source -> event after its gather

    def start(self, src: torch.Tensor):
        if not self.cuda:
            self._gather(src)
            return
        cur = torch.cuda.current_stream(src.device)
        self.side.wait_stream(cur)
        with torch.cuda.stream(self.side):
            self._gather(src)
            ev = torch.cuda.Event()
            ev.record(self.side)
        src.record_stream(self.side)
        self.done = ev
        self._reading[src.data_ptr()] = ev

    def _gather(self, src):
        # the output as ranks concatenated along the leading dimension, the form every
        # backend accepts (gloo rejects a separate rank dimension)
        flat = self.buf.view((self.world * self.buf.shape[1],) + tuple(self.buf.shape[2:]))
        dist.all_gather_into_tensor(flat, src.contiguous(), group=self.group)

    def release(self, src: torch.Tensor):
        """Make the current stream wait until no gather still reads ``src``."""
        ev = self._reading.pop(src.data_ptr(), None)
        if ev is not None:
            torch.cuda.current_stream(src.device).wait_event(ev)

    def wait(self):
        if self.cuda and self.done is not None:
            torch.cuda.current_stream(self.buf.device).wait_event(self.done)
            self._reading.clear()

    def assembled(self) -> torch.Tensor:
        return assemble(self.buf)

    def close(self):
        if self.cuda:
            self.side.synchronize()
        self._reading.clear()
        self.done = None
