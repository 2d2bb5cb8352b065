"""Batched randomized SVD on the device (``spx_rsvd_compress``).

Same signature and outputs as the reference (unsloth_spectral/rsvd.py:28-157):
``U [B, m, k]``, ``S [B, k]``, ``Vh [B, k, n]`` in the input dtype.  The Gaussian sketch
is drawn exactly as the reference draws it -- ``torch.randn(B, n, r)`` in float32 on
the input's device from the global generator -- so a caller that seeds torch gets the
same sketch the reference would use.  The subspace iteration re-orthonormalises every
power step (same subspace in exact arithmetic, no float32 blow-up).
"""
from __future__ import annotations

import torch

from . import _ops


def batched_randomized_svd(M: torch.Tensor, k: int, n_iter: int = 2, oversampling: int = 5):
    B, m, n = M.shape
    r = min(k + oversampling, min(m, n))
    original_dtype = M.dtype
    if r >= min(m, n) - 1:
        # rsvd.py:84-87: full SVD for ranks close to the matrix size (device library call)
        U, S, Vh = torch.linalg.svd(M.float(), full_matrices=False)
        return U[:, :, :k].to(original_dtype), S[:, :k].to(original_dtype), Vh[:, :k, :].to(original_dtype)
    omega = torch.randn(B, n, r, device=M.device, dtype=torch.float32 if M.dtype != torch.float64 else M.dtype)
    Mc = M if M.dtype in (torch.float32, torch.float16, torch.bfloat16) else M.float()
    U, S, Vh = _ops.rsvd(Mc.contiguous(), omega, k, n_iter)
    return U.to(original_dtype), S.to(original_dtype), Vh.to(original_dtype)
