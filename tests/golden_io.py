"""Helpers to turn the recorded golden cases into oracle / product inputs."""
from __future__ import annotations

import os

import numpy as np
import torch

from oracle import spectral_oracle as so
from unsloth_spectral import synthetic as syn

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def decode_case(name):
    """Inputs of a recorded decode case: codes, scales, bases, hot tier, tables."""
    z = load(name)
    D = int(z["D"])
    qpos = int(z["qpos"])
    if int(z["untied"]):
        cos, sin = z["cos"], z["sin"]
    else:
        c, s = syn.rope_tables(qpos + 16, D, float(z["theta"]))
        cos, sin = c.numpy(), s.numpy()
    scale_K = np.stack([so.scale_from_minmax(m) for m in z["mmk"]])   # [nblk, H]
    scale_V = np.stack([so.scale_from_minmax(m) for m in z["mmv"]])
    blocks = so.blocks_from_codes(z["ck"], scale_K, z["bk"], z["cv"], scale_V, z["bv"],
                                  z["start_pos"])
    z.update(cos=cos, sin=sin, scale_K=scale_K, scale_V=scale_V, blocks=blocks)
    return z


def rsvd_inputs(z, i):
    """Regenerate the fp16 rSVD input of golden case ``i`` and its sketch."""
    rank = int(z[f"c{i}_rank"])
    rho = float(z[f"c{i}_rho"])
    Ms = []
    for h in range(8):
        gen = torch.Generator().manual_seed(syn.head_seed(3, 0, 0, h) + rank)
        Ms.append(syn.low_rank_block(gen, 512, 128, rank, rho))
    M16 = torch.stack(Ms).to(torch.float16)
    k = int(z[f"c{i}_k"])
    torch.manual_seed(int(z[f"c{i}_seed"]))
    Omega = torch.randn(8, 128, k + 8)
    return M16, Omega
