"""Generate golden vectors by running the reference implementation itself.

Run in a container where the reference project (nyssaleo/unsloth-spectral) is
mounted; pass its root with ``--reference`` (or the ``SPX_REFERENCE_ROOT``
environment variable).  The script imports the reference's own Python package,
feeds it seeded inputs, and records inputs + outputs as small ``.npz`` files next to
this script.  The tests read only these files; they never import the reference.

Reference entry points exercised (paths relative to the reference project):
  unsloth_spectral/spectral_cache.py:481  SpectralCache._quantize_int8_batched
  unsloth_spectral/rsvd.py:28             batched_randomized_svd
  unsloth_spectral/spectral_attention.py:117  spectral_attention_forward
  unsloth_spectral/kernels/spectral_attention.py:684  spectral_attention_decode
  unsloth_spectral/kernels/spectral_attention.py:456  spectral_score_forward
  unsloth_spectral/kernels/spectral_attention.py:604  spectral_value_forward
  unsloth_spectral/spectral_cache.py:557  SpectralCache.get_kv

Usage:  python tests/golden/make_golden.py --reference <path to reference root>
"""
from __future__ import annotations

import argparse
import hashlib
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "unsloth-spectral_b200"))


def _import_reference(root):
    os.environ.setdefault("UNSLOTH_SPECTRAL_QUIET", "1")
    sys.dont_write_bytecode = True
    sys.path.insert(0, root)
    import importlib
    sc = importlib.import_module("unsloth_spectral.spectral_cache")
    sa = importlib.import_module("unsloth_spectral.spectral_attention")
    rs = importlib.import_module("unsloth_spectral.rsvd")
    ka = importlib.import_module("unsloth_spectral.kernels.spectral_attention")
    sys.path.pop(0)
    return sc, sa, rs, ka


def _load_synthetic():
    # The repo's generator lives in a package that shares the reference's import
    # name, so load the one file directly under a private name.
    import importlib.util
    path = os.path.join(REPO, "unsloth-spectral_b200", "unsloth_spectral", "synthetic.py")
    spec = importlib.util.spec_from_file_location("_spx_synthetic", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def digest(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]


def make_quant(sc, torch, out):
    g = torch.Generator().manual_seed(1234)
    C = torch.randn(6, 512, 16, generator=g)
    C[0] *= 1e-3
    C[2] *= 30.0
    C[3] *= 1e4
    C[4] = 0.0                       # all-zero head: exercises the 1e-8 floor
    s = 2.0 ** -3                    # exact scale => exact .5 ties after division
    C[5] = 0.0
    C[5, 0, 0] = 127 * s
    C[5, 1, 0:6] = torch.tensor([2.5, -3.5, 0.5, -0.5, 1.5, 126.5]) * s
    cache = sc.SpectralCache(num_heads=6, head_dim=16, device="cpu", dtype=torch.float32)
    q, mm = sc.SpectralCache._quantize_int8_batched(cache, C)
    np.savez_compressed(os.path.join(out, "quant.npz"), C=C.numpy(), quantized=q.numpy(),
                        scales=mm.numpy())
    print("quant.npz", C.shape)


def make_rsvd(rs, syn, torch, out):
    cases = []
    for (rank, rho, k, q, seed) in [(24, 0.85, 16, 2, 4242), (24, 0.85, 16, 0, 4243),
                                    (48, 0.9, 32, 2, 4244), (48, 0.9, 32, 0, 4245)]:
        Ms = []
        for h in range(8):
            gen = torch.Generator().manual_seed(syn.head_seed(3, 0, 0, h) + rank)
            Ms.append(syn.low_rank_block(gen, 512, 128, rank, rho))
        M16 = torch.stack(Ms).to(torch.float16)
        torch.manual_seed(seed)
        U, S, Vh = rs.batched_randomized_svd(M16.float(), k, n_iter=q, oversampling=8)
        Mf = M16.float()
        err = (torch.linalg.norm(Mf - (U * S[:, None, :]) @ Vh, dim=(1, 2))
               / torch.linalg.norm(Mf, dim=(1, 2)))
        # The same reference code path in float64 with the very same sketch values: the
        # reference draws its sketch in the input dtype (rsvd.py:95), so hand it the
        # float32 draw upcast to float64 for the duration of the call.
        torch.manual_seed(seed)
        omega64 = torch.randn(8, 128, k + 8).double()
        real_randn = torch.randn
        torch.randn = lambda *a, **kw: omega64.clone()
        try:
            U2, S2, Vh2 = rs.batched_randomized_svd(Mf.double(), k, n_iter=q, oversampling=8)
        finally:
            torch.randn = real_randn
        Md = Mf.double()
        err64 = (torch.linalg.norm(Md - (U2 * S2[:, None, :]) @ Vh2, dim=(1, 2))
                 / torch.linalg.norm(Md, dim=(1, 2)))
        cases.append(dict(rank=rank, rho=rho, k=k, q=q, seed=seed, M_digest=digest(M16.numpy()),
                          S=S.numpy(), err=err.numpy(), S64=S2.numpy(), err64=err64.numpy()))
        print(f"rsvd case k={k} q={q} rank={rank}: err(fp32)={err.mean():.6f} "
              f"err(fp64)={err64.mean():.6f}")
    arr = {}
    for i, c in enumerate(cases):
        for key, v in c.items():
            arr[f"c{i}_{key}"] = np.asarray(v)
    arr["ncases"] = np.asarray(len(cases))
    np.savez_compressed(os.path.join(out, "rsvd.npz"), **arr)


def _compress(rs, sc_mod, cache, X, k, p, q, seed, torch):
    """The reference's _compress_tensor steps (spectral_cache.py:349-405) with the
    oversampling the configs ask for (the class hard-codes 5)."""
    torch.manual_seed(seed)
    U, S, Vh = rs.batched_randomized_svd(X.float(), k=k, n_iter=q, oversampling=p)
    coeffs = U * S.unsqueeze(1)
    cq, mm = sc_mod.SpectralCache._quantize_int8_batched(cache, coeffs)
    return cq, Vh, mm


def _codes(coeffs_q, minmax):
    """Integer codes of reference-dequantised coefficients; asserts that codes * scale
    reproduces the reference's stored values bit for bit."""
    mm = minmax.numpy().astype(np.float32)
    abs_max = np.maximum(np.maximum(-mm[:, 0], mm[:, 1]), np.float32(1e-8))
    scale = (abs_max / np.float32(127.0)).astype(np.float32)
    c = coeffs_q.numpy().astype(np.float32)
    codes = np.rint(c / scale[:, None, None])
    assert np.array_equal((codes.astype(np.float32) * scale[:, None, None]).astype(np.float32), c)
    assert np.abs(codes).max() <= 127
    return codes.astype(np.int8)


def make_decode(name, sc, sa, rs, ka, syn, torch, out, *, cfg, B, H_q, H_kv, D, T_blk, nblk,
                kK, kV, T_hot, rank, rho, p, q, theta, untied=False, with_mask=True):
    assert B == 1
    T_cold = nblk * T_blk
    T_all = T_cold + T_hot
    K, V = syn.kv_per_head(cfg, 0, B, H_kv, T_all, D, rank, rho)
    cache = sc.SpectralCache(num_heads=H_kv, head_dim=D, block_size=T_blk, k_rank_keys=kK,
                             k_rank_values=kV, device="cpu", dtype=torch.float32)
    blocks = []
    rec = {k_: [] for k_ in ("ck", "bk", "mmk", "cv", "bv", "mmv")}
    for j in range(nblk):
        Kb = K[0, :, j * T_blk:(j + 1) * T_blk]
        Vb = V[0, :, j * T_blk:(j + 1) * T_blk]
        ckq, bk, mmk = _compress(rs, sc, cache, Kb, kK, p, q, 9000 + 2 * j, torch)
        cvq, bv, mmv = _compress(rs, sc, cache, Vb, kV, p, q, 9001 + 2 * j, torch)
        blocks.append(sc.SpectralBlock(coeffs_K=ckq, basis_K=bk, coeffs_V=cvq, basis_V=bv,
                                       scales_K=mmk, scales_V=mmv, block_size=T_blk,
                                       start_position=j * T_blk))
        for key, v in (("ck", _codes(ckq, mmk)), ("bk", bk.numpy()), ("mmk", mmk.numpy()),
                       ("cv", _codes(cvq, mmv)), ("bv", bv.numpy()), ("mmv", mmv.numpy())):
            rec[key].append(v)
    hot_K = K[:, :, T_cold:].contiguous()
    hot_V = V[:, :, T_cold:].contiguous()
    hot_pos = torch.arange(T_cold, T_all).unsqueeze(0)
    cache.cold_blocks = blocks
    cache.hot_K, cache.hot_V, cache.hot_position_ids = hot_K, hot_V, hot_pos
    cache.total_tokens = T_all
    cache.current_position = T_all
    qpos = T_all
    cos, sin = syn.rope_tables(qpos + 16, D, theta)
    if untied:
        g = torch.Generator().manual_seed(77)
        cos = torch.rand(qpos + 16, D, generator=g) * 2 - 1
        sin = torch.rand(qpos + 16, D, generator=g) * 2 - 1
    Qpre = syn.query(cfg, 0, B, H_q, D)
    Q = syn.rope_rotate(Qpre, cos[qpos], sin[qpos])
    scale = 1.0 / math.sqrt(D)
    res = {}
    res["out_forward"] = sa.spectral_attention_forward(Q, cache, cos, sin, qpos, scale=scale)
    res["out_decode"] = ka.spectral_attention_decode(
        Q, cache, cos, sin, qpos, scale=scale, config=ka.TritonSpectralConfig(enable_logging=False))
    mask = None
    if with_mask:
        g = torch.Generator().manual_seed(99)
        mask = (torch.rand(B, H_q, 1, T_all, generator=g) > 0.1).to(torch.int64)
        res["out_forward_mask"] = sa.spectral_attention_forward(Q, cache, cos, sin, qpos,
                                                                attention_mask=mask, scale=scale)
        res["out_decode_mask"] = ka.spectral_attention_decode(
            Q, cache, cos, sin, qpos, attention_mask=mask, scale=scale,
            config=ka.TritonSpectralConfig(enable_logging=False))
    res["scores_block0"] = ka.spectral_score_forward(
        Q, blocks[0].coeffs_K, blocks[0].basis_K, cos, sin, blocks[0].start_position, qpos,
        config=ka.TritonSpectralConfig(enable_logging=False))
    attn0 = torch.softmax(res["scores_block0"] * scale, dim=-1)
    res["attn_block0"] = attn0
    res["values_block0"] = ka.spectral_value_forward(
        attn0, blocks[0].coeffs_V, blocks[0].basis_V, D, config=ka.TritonSpectralConfig(enable_logging=False))
    Kf, Vf = cache.get_kv()
    arr = dict(
        cfg=cfg, H_q=H_q, H_kv=H_kv, D=D, T_blk=T_blk, nblk=nblk, kK=kK, kV=kV, T_hot=T_hot,
        qpos=qpos, theta=theta, untied=int(untied), scale=scale,
        ck=np.stack(rec["ck"]), bk=np.stack(rec["bk"]), mmk=np.stack(rec["mmk"]),
        cv=np.stack(rec["cv"]), bv=np.stack(rec["bv"]), mmv=np.stack(rec["mmv"]),
        start_pos=np.arange(nblk) * T_blk, hot_K=hot_K.numpy(), hot_V=hot_V.numpy(),
        hot_pos=hot_pos.numpy(), Q=Q.numpy(), Qpre=Qpre.numpy(),
        getkv_K_digest=np.asarray(digest(Kf.numpy())),
        getkv_K_sum=np.asarray(Kf.double().sum().item()), getkv_V_sum=np.asarray(Vf.double().sum().item()),
    )
    if untied:
        arr["cos"] = cos.numpy()
        arr["sin"] = sin.numpy()
    if mask is not None:
        arr["mask"] = mask.numpy().astype(np.int8)
    for key, v in res.items():
        arr[key] = v.numpy()
    np.savez_compressed(os.path.join(out, f"{name}.npz"), **arr)
    o1, o2 = res["out_forward"].flatten(), res["out_decode"].flatten()
    cosv = float(torch.dot(o1, o2) / (o1.norm() * o2.norm()))
    print(f"{name}.npz: forward-vs-decode cosine {cosv:.6f}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SPX_REFERENCE_ROOT"))
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        sys.exit("pass --reference <root of the reference project>")
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    sc, sa, rs, ka = _import_reference(args.reference)
    import logging
    logging.getLogger("unsloth_spectral").setLevel(logging.WARNING)
    syn = _load_synthetic()
    make_quant(sc, torch, args.out)
    make_rsvd(rs, syn, torch, args.out)
    # config 0: Mistral GQA layout, 4 cold blocks of 512 at k=16 (p=8, q=2) + 64 hot, FP32
    make_decode("decode_cfg0", sc, sa, rs, ka, syn, torch, args.out, cfg=0, B=1, H_q=32, H_kv=8,
                D=128, T_blk=512, nblk=4, kK=16, kV=16, T_hot=64, rank=24, rho=0.85, p=8, q=2,
                theta=1e6)
    # the reference's own GQA test shape (test_gqa_fix.py:31-46): 8/2 heads, D=64, block 256,
    # with the reference defaults k_K=16, k_V=32 and a ragged hot tier
    make_decode("decode_gqa_small", sc, sa, rs, ka, syn, torch, args.out, cfg=5, B=1, H_q=8,
                H_kv=2, D=64, T_blk=256, nblk=2, kK=16, kV=32, T_hot=37, rank=24, rho=0.85, p=5,
                q=2, theta=10000.0)
    # arbitrary (untied) cos/sin tables, as the reference's Colab kernel test feeds
    make_decode("decode_untied", sc, sa, rs, ka, syn, torch, args.out, cfg=6, B=1, H_q=4, H_kv=1,
                D=64, T_blk=256, nblk=2, kK=16, kV=16, T_hot=5, rank=24, rho=0.85, p=8, q=2,
                theta=10000.0, untied=True, with_mask=False)


if __name__ == "__main__":
    main()
