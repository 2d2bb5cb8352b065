"""Parity of the CUDA path (through the C ABI) with the CPU oracle and with outputs
recorded from the reference implementation.

Tolerances (from the path's specification):
  * INT8 codes: bit-exact given the same float32 coefficients;
  * rSVD: relative reconstruction error within 1e-3 absolute of the reference's
    algorithm on the same sketch;
  * attention: cosine >= 0.9999 and max-abs error <= 1e-2 against the float32 oracle
    over the same compressed cache (float32 caches are also held to 2e-4).
"""
import math

import numpy as np
import pytest
import torch

from conftest import cuda_ok
from oracle import spectral_oracle as so
import golden_io as gio

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

COS_MIN = 0.9999
ABS_MAX = 1e-2


def _cos(a, b):
    a, b = np.ravel(a).astype(np.float64), np.ravel(b).astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def _close(out, ref, abs_tol=ABS_MAX):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    assert _cos(out, ref) >= COS_MIN, _cos(out, ref)
    assert np.abs(out - ref).max() <= abs_tol, np.abs(out - ref).max()


def _to_dtype_np(x, dtype):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dtype)
    return t.float().numpy()


def cache_from_arrays(H, D, T, kK, kV, codes_K, scale_K, basis_K, codes_V, scale_V, basis_V, start_pos,
                      hot_K, hot_V, hot_pos, dtype, B=1):
    """Our device cache from per-block arrays in the reference's layout
    (codes [nblk, H, T, k] or [B, nblk, H, T, k])."""
    from unsloth_spectral import SpectralCache
    dev = torch.device("cuda")
    cache = SpectralCache(H, D, block_size=T, k_rank_keys=kK, k_rank_values=kV, device=dev, dtype=dtype)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    if codes_K is not None and len(codes_K):
        if codes_K.ndim == 4:
            codes_K, codes_V, scale_K, scale_V, basis_K, basis_V = (
                x[None] for x in (codes_K, codes_V, scale_K, scale_V, basis_K, basis_V))
        perm5 = lambda a: t(a).permute(0, 2, 1, 3, 4)
        cache.set_cold(perm5(codes_K), t(scale_K).permute(0, 2, 1), perm5(basis_K), perm5(codes_V),
                       t(scale_V).permute(0, 2, 1), perm5(basis_V), list(start_pos))
    if hot_K is not None and hot_K.shape[2] > 0:
        cache.set_hot(t(hot_K).to(dtype), t(hot_V).to(dtype), t(np.asarray(hot_pos).reshape(-1)))
    return cache


# ----------------------------------------------------------------------- quantiser
def test_quantize_matches_reference_bit_exact():
    from unsloth_spectral import _ops
    z = gio.load("quant")
    C = torch.from_numpy(z["C"]).cuda()
    codes, scale, minmax, deq = _ops.quantize_int8(C)
    assert np.array_equal(deq.cpu().numpy(), z["quantized"])
    assert np.array_equal(minmax.cpu().numpy(), z["scales"])


@pytest.mark.parametrize("shape", [(8, 512, 16), (64, 512, 32), (3, 17, 5), (1, 1, 1)])
def test_quantize_random_bit_exact(shape):
    from unsloth_spectral import _ops
    g = torch.Generator().manual_seed(sum(shape))
    C = torch.randn(*shape, generator=g) * torch.logspace(-4, 4, shape[0])[:, None, None]
    codes, scale, minmax, deq = _ops.quantize_int8(C.cuda())
    q, mm, ocodes, oscale = so.quantize_int8_batched(C.numpy())
    assert np.array_equal(codes.cpu().numpy(), ocodes)
    assert np.array_equal(scale.cpu().numpy(), oscale)
    assert np.array_equal(minmax.cpu().numpy(), mm)
    assert np.array_equal(deq.cpu().numpy(), q)


# ------------------------------------------------------------------- decode (golden)
def _golden_cache(c, dtype):
    return cache_from_arrays(int(c["H_kv"]), int(c["D"]), int(c["T_blk"]), int(c["kK"]), int(c["kV"]),
                             c["ck"], c["scale_K"], c["bk"], c["cv"], c["scale_V"], c["bv"], c["start_pos"],
                             c["hot_K"], c["hot_V"], c["hot_pos"], dtype)


@pytest.mark.parametrize("name", ["decode_cfg0", "decode_gqa_small", "decode_untied"])
@pytest.mark.parametrize("masked", [False, True])
def test_decode_matches_reference_fp32(name, masked):
    from unsloth_spectral import spectral_attention_forward
    from unsloth_spectral.kernels import spectral_attention_decode
    c = gio.decode_case(name)
    if masked and "mask" not in c:
        pytest.skip("no mask recorded for this case")
    cache = _golden_cache(c, torch.float32)
    Q = torch.from_numpy(c["Q"]).cuda()
    cos, sin = torch.from_numpy(c["cos"]).cuda(), torch.from_numpy(c["sin"]).cuda()
    mask = torch.from_numpy(c["mask"]).cuda() if masked else None
    qpos, scale = int(c["qpos"]), float(c["scale"])
    fwd = spectral_attention_forward(Q, cache, cos, sin, qpos, attention_mask=mask, scale=scale).cpu().numpy()
    dec = spectral_attention_decode(Q, cache, cos, sin, qpos, attention_mask=mask, scale=scale).cpu().numpy()
    sfx = "_mask" if masked else ""
    _close(fwd, c["out_forward" + sfx], 2e-4)
    _close(dec, c["out_decode" + sfx], 2e-4)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("mode", ["forward", "decode"])
def test_decode_half_precision_vs_oracle(dtype, mode):
    from unsloth_spectral import spectral_attention_forward
    from unsloth_spectral.kernels import spectral_attention_decode
    c = gio.decode_case("decode_cfg0")
    cache = _golden_cache(c, dtype)
    Q = torch.from_numpy(c["Q"]).cuda().to(dtype)
    cos, sin = torch.from_numpy(c["cos"]).cuda(), torch.from_numpy(c["sin"]).cuda()
    fn = spectral_attention_forward if mode == "forward" else spectral_attention_decode
    out = fn(Q, cache, cos, sin, int(c["qpos"]), scale=float(c["scale"])).float().cpu().numpy()
    blocks = so.blocks_from_codes(c["ck"], c["scale_K"], _to_dtype_np(c["bk"], dtype), c["cv"], c["scale_V"],
                                  _to_dtype_np(c["bv"], dtype), c["start_pos"])
    ofn = so.spectral_attention_forward if mode == "forward" else so.spectral_attention_decode
    ref = ofn(_to_dtype_np(c["Q"], dtype), blocks, _to_dtype_np(c["hot_K"], dtype), _to_dtype_np(c["hot_V"], dtype),
              c["hot_pos"], c["cos"], c["sin"], int(c["qpos"]), scale=float(c["scale"]))
    _close(out, ref)


# ------------------------------------------------------------------ decode (random)
def _random_case(seed, B, H, nrep, D, T, nblk, kK, kV, hot, masked, qpos_extra=0, untied=False):
    rng = np.random.default_rng(seed)
    codes_K = rng.integers(-127, 128, size=(B, nblk, H, T, kK), dtype=np.int8)
    codes_V = rng.integers(-127, 128, size=(B, nblk, H, T, kV), dtype=np.int8)
    scale_K = (rng.random((B, nblk, H)) * 0.02 + 0.005).astype(np.float32)
    scale_V = (rng.random((B, nblk, H)) * 0.02 + 0.005).astype(np.float32)
    def basis(k):
        if nblk == 0:
            return np.zeros((B, 0, H, k, D), np.float32)
        Qm = np.linalg.qr(rng.standard_normal((B, nblk, H, D, k)))[0]
        return np.ascontiguousarray(np.swapaxes(Qm, -1, -2)).astype(np.float32)
    basis_K, basis_V = basis(kK), basis(kV)
    hot_K = rng.standard_normal((B, H, hot, D)).astype(np.float32)
    hot_V = rng.standard_normal((B, H, hot, D)).astype(np.float32)
    start = np.arange(nblk) * T
    hot_pos = np.arange(nblk * T, nblk * T + hot)
    qpos = nblk * T + hot + qpos_extra
    L = max(qpos, nblk * T + hot) + 8
    if untied:
        cos = (rng.random((L, D)) * 2 - 1).astype(np.float32)
        sin = (rng.random((L, D)) * 2 - 1).astype(np.float32)
    else:
        cc, ss = so.rope_tables(L, D, 1e6)
        cos, sin = cc, ss
    Q = (rng.standard_normal((B, H * nrep, 1, D)) / math.sqrt(D)).astype(np.float32)
    mask = None
    if masked:
        mask = (rng.random((B, H * nrep, 1, nblk * T + hot)) > 0.2).astype(np.int64)
    return dict(codes_K=codes_K, codes_V=codes_V, scale_K=scale_K, scale_V=scale_V, basis_K=basis_K,
                basis_V=basis_V, hot_K=hot_K, hot_V=hot_V, start=start, hot_pos=hot_pos, qpos=qpos, cos=cos,
                sin=sin, Q=Q, mask=mask, B=B, H=H, D=D, T=T, kK=kK, kV=kV, nblk=nblk)


def _run_random(r, dtype, mode):
    from unsloth_spectral import spectral_attention_forward
    from unsloth_spectral.kernels import spectral_attention_decode
    B, H, D, T = r["B"], r["H"], r["D"], r["T"]
    cache = cache_from_arrays(H, D, T, r["kK"], r["kV"], r["codes_K"] if r["nblk"] else None, r["scale_K"],
                              r["basis_K"], r["codes_V"], r["scale_V"], r["basis_V"], r["start"], r["hot_K"],
                              r["hot_V"], r["hot_pos"], dtype, B=B)
    Q = torch.from_numpy(r["Q"]).cuda().to(dtype)
    cos, sin = torch.from_numpy(r["cos"]).cuda(), torch.from_numpy(r["sin"]).cuda()
    mask = None if r["mask"] is None else torch.from_numpy(r["mask"]).cuda()
    fn = spectral_attention_forward if mode == "forward" else spectral_attention_decode
    out = fn(Q, cache, cos, sin, r["qpos"], attention_mask=mask).float().cpu().numpy()
    ofn = so.spectral_attention_forward if mode == "forward" else so.spectral_attention_decode
    refs = []
    for b in range(B):
        blocks = so.blocks_from_codes(r["codes_K"][b], r["scale_K"][b], _to_dtype_np(r["basis_K"][b], dtype),
                                      r["codes_V"][b], r["scale_V"][b], _to_dtype_np(r["basis_V"][b], dtype),
                                      r["start"]) if r["nblk"] else []
        refs.append(ofn(_to_dtype_np(r["Q"][b:b + 1], dtype), blocks, _to_dtype_np(r["hot_K"][b:b + 1], dtype),
                        _to_dtype_np(r["hot_V"][b:b + 1], dtype), r["hot_pos"], r["cos"], r["sin"], r["qpos"],
                        attention_mask=None if r["mask"] is None else r["mask"][b:b + 1]))
    return out, np.concatenate(refs, 0)


CASES = [
    # seed, B, H, nrep, D, T, nblk, kK, kV, hot, masked
    (1, 2, 8, 4, 128, 512, 3, 32, 32, 64, False),
    (2, 1, 8, 4, 128, 512, 2, 16, 32, 0, False),      # no hot tier
    (3, 3, 2, 1, 64, 256, 2, 48, 16, 17, True),       # MHA, ragged hot tier, mask
    (4, 1, 4, 8, 128, 128, 5, 64, 64, 200, False),
    (5, 2, 8, 4, 128, 512, 0, 16, 16, 130, False),    # hot tier only
    (6, 1, 2, 4, 64, 64, 7, 16, 16, 3, True),
    (7, 2, 1, 16, 128, 256, 1, 32, 48, 1, False),
]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("mode", ["forward", "decode"])
def test_decode_random_shapes_fp32(case, mode):
    r = _random_case(*case)
    out, ref = _run_random(r, torch.float32, mode)
    _close(out, ref, 5e-4)


# a 300-token hot tier (a warm buffer plus the hot tail) is too large to stage in shared
# memory: the merge reads it directly from global memory
@pytest.mark.parametrize("case", CASES[:3] + [(8, 2, 4, 4, 128, 512, 2, 16, 16, 300, False)])
def test_decode_random_shapes_fp16(case):
    r = _random_case(*case)
    out, ref = _run_random(r, torch.float16, "decode")
    _close(out, ref)


def test_decode_untied_tables_and_late_query():
    r = _random_case(11, 1, 2, 4, 64, 128, 3, 16, 16, 9, False, qpos_extra=-200, untied=True)
    for mode in ("forward", "decode"):
        out, ref = _run_random(r, torch.float32, mode)
        _close(out, ref, 5e-4)


def test_empty_cache_raises_value_error():
    from unsloth_spectral import SpectralCache, spectral_attention_forward
    cache = SpectralCache(8, 128, device="cuda", dtype=torch.float16)
    Q = torch.zeros(1, 32, 1, 128, device="cuda", dtype=torch.float16)
    cos = torch.ones(16, 128, device="cuda")
    with pytest.raises(ValueError, match="Empty cache"):
        spectral_attention_forward(Q, cache, cos, cos * 0, 3)


def test_fully_masked_row_is_nan_like_reference():
    r = _random_case(21, 1, 2, 2, 64, 64, 1, 16, 16, 4, True)
    r["mask"][:, 0] = 0
    out, ref = _run_random(r, torch.float32, "decode")
    assert np.isnan(ref[:, 0]).all() and np.isnan(out[:, 0]).all()
    _close(out[:, 1:], ref[:, 1:], 5e-4)


# -------------------------------------------------------------- per-block helpers
def test_block_score_and_value_match_reference():
    from unsloth_spectral.kernels import spectral_score_forward, spectral_value_forward
    c = gio.decode_case("decode_cfg0")
    b0 = c["blocks"][0]
    Q = torch.from_numpy(c["Q"]).cuda()
    cos, sin = torch.from_numpy(c["cos"]).cuda(), torch.from_numpy(c["sin"]).cuda()
    s = spectral_score_forward(Q, torch.from_numpy(b0.coeffs_K).cuda(), torch.from_numpy(b0.basis_K).cuda(), cos,
                               sin, b0.start_position, int(c["qpos"]))
    np.testing.assert_allclose(s.cpu().numpy(), c["scores_block0"], atol=2e-4, rtol=1e-4)
    v = spectral_value_forward(torch.from_numpy(c["attn_block0"]).cuda(), torch.from_numpy(b0.coeffs_V).cuda(),
                               torch.from_numpy(b0.basis_V).cuda(), 128)
    np.testing.assert_allclose(v.cpu().numpy(), c["values_block0"], atol=1e-5, rtol=1e-4)


def test_get_kv_matches_reference():
    c = gio.decode_case("decode_cfg0")
    cache = _golden_cache(c, torch.float32)
    K, V = cache.get_kv()
    assert abs(K.double().sum().item() - float(c["getkv_K_sum"])) < 1e-2
    assert abs(V.double().sum().item() - float(c["getkv_V_sum"])) < 1e-2
    Ko, Vo = so.get_kv(c["blocks"], c["hot_K"], c["hot_V"])
    np.testing.assert_allclose(K.cpu().numpy(), Ko, atol=1e-4)
    np.testing.assert_allclose(V.cpu().numpy(), Vo, atol=1e-4)
    blocks = cache.cold_blocks
    np.testing.assert_array_equal(blocks[1].coeffs_K.cpu().numpy(), c["blocks"][1].coeffs_K)
    assert blocks[2].start_position == 1024


# ------------------------------------------------------------------------------ rSVD
@pytest.mark.parametrize("i", range(4))
def test_rsvd_matches_reference_error(i):
    from unsloth_spectral import _ops
    z = gio.load("rsvd")
    M16, Omega = gio.rsvd_inputs(z, i)
    k, q = int(z[f"c{i}_k"]), int(z[f"c{i}_q"])
    U, S, Vh = _ops.rsvd(M16.cuda(), Omega.cuda(), k, q)
    M = M16.float().numpy()
    err = so.relative_reconstruction_error(M, U.cpu().numpy(), S.cpu().numpy(), Vh.cpu().numpy())
    assert np.abs(err - z[f"c{i}_err64"]).max() <= 1e-3
    # where the reference's float32 run is not rounding-dominated, match it as well
    stable = np.abs(z[f"c{i}_err"] - z[f"c{i}_err64"]) < 1e-4
    assert np.abs(err - z[f"c{i}_err"])[stable].max(initial=0) <= 1e-3
    np.testing.assert_allclose(S.cpu().numpy(), z[f"c{i}_S64"], rtol=2e-3)
    # orthonormal factors
    Uc, Vc = U.double(), Vh.double()
    assert torch.allclose(Uc.transpose(1, 2) @ Uc, torch.eye(k, dtype=torch.float64, device="cuda")[None], atol=1e-4)
    assert torch.allclose(Vc @ Vc.transpose(1, 2), torch.eye(k, dtype=torch.float64, device="cuda")[None], atol=1e-4)


@pytest.mark.parametrize("case", ["rank6", "steep", "rank6_q0"])
def test_rsvd_ill_conditioned_sketches(case):
    """Sketches the orthonormalisation has to work for: an exactly rank-6 block (r = 24
    sketch columns, so Cholesky-QR meets zero pivots and leaves zero columns) and a
    spectrum decaying as 0.5^i (pivot spreads far beyond 1e12, so the extra passes run).
    The reconstruction error must match the reference algorithm's float64 run on the
    same sketch within 1e-3, as for the golden cases."""
    from unsloth_spectral import _ops
    g = torch.Generator().manual_seed(11)
    k, q = 16, 0 if case == "rank6_q0" else 2
    if case.startswith("rank6"):
        A = torch.randn(6, 512, 6, generator=g)
        Bm = torch.randn(6, 6, 128, generator=g)
        M16 = (A @ Bm).to(torch.float16)
    else:
        sig = 0.5 ** torch.arange(48, dtype=torch.float32)
        A = torch.randn(6, 512, 48, generator=g) * sig
        M16 = (A @ torch.randn(6, 48, 128, generator=g)).to(torch.float16)
    Omega = torch.randn(6, 128, k + 8, generator=g)
    U, S, Vh = _ops.rsvd(M16.cuda(), Omega.cuda(), k, q)
    for x in (U, S, Vh):
        assert torch.isfinite(x).all()
    M = M16.float().numpy()
    err = so.relative_reconstruction_error(M, U.cpu().numpy(), S.cpu().numpy(), Vh.cpu().numpy())
    U64, S64, Vh64 = so.batched_randomized_svd(M, k, q, 8, Omega.numpy())
    err64 = so.relative_reconstruction_error(M, U64, S64, Vh64)
    assert np.abs(err - err64).max() <= 1e-3, (err, err64)
    S_np = S.cpu().numpy()
    big = S64 >= 1e-3 * S64[:, :1]
    np.testing.assert_allclose(S_np[big], S64[big], rtol=2e-3)
    if case.startswith("rank6"):   # nothing beyond the rank
        assert (S_np[:, 6:] <= 1e-4 * S_np[:, :1]).all()


@pytest.mark.parametrize("m,n,k,dtype", [(200, 96, 13, torch.float16), (384, 128, 10, torch.float32),
                                         (256, 128, 13, torch.bfloat16)])
def test_rsvd_odd_shapes(m, n, k, dtype):
    """Shapes off the tensor-core fast path: m not a multiple of 128, n != 128, float32
    input (CUDA-core products), and r = k + 8 not a multiple of 4 (the scalar branches of
    the Gram, solve and lift kernels).  Error parity with the float64 reference algorithm
    on the same sketch, within 1e-3."""
    from unsloth_spectral import _ops
    g = torch.Generator().manual_seed(21)
    sig = 0.85 ** torch.arange(24, dtype=torch.float32)
    M = ((torch.randn(5, m, 24, generator=g) * sig) @ torch.randn(5, 24, n, generator=g)
         + 0.05 * torch.randn(5, m, n, generator=g)).to(dtype)
    Omega = torch.randn(5, n, k + 8, generator=g)
    U, S, Vh = _ops.rsvd(M.cuda(), Omega.cuda(), k, 2)
    Mf = M.float().numpy()
    err = so.relative_reconstruction_error(Mf, U.cpu().numpy(), S.cpu().numpy(), Vh.cpu().numpy())
    U64, S64, Vh64 = so.batched_randomized_svd(Mf, k, 2, 8, Omega.numpy())
    err64 = so.relative_reconstruction_error(Mf, U64, S64, Vh64)
    assert np.abs(err - err64).max() <= 1e-3, (err, err64)
    np.testing.assert_allclose(S.cpu().numpy(), S64, rtol=2e-3)


@pytest.mark.parametrize("nb,m,dtype", [(700, 512, torch.float16), (650, 128, torch.bfloat16)])
def test_rsvd_many_blocks(nb, m, dtype):
    """Batches of several waves of CTAs (two resident per SM), including single-tile
    blocks (m = 128).  The tensor-core path on 16-bit input must agree with the CUDA-core
    path on the same values as float32 (both products are float32 accurate), and blocks
    around the wave boundaries match the float64 reference algorithm's error within 1e-3."""
    from unsloth_spectral import _ops
    g = torch.Generator().manual_seed(33)
    k = 16
    sig = 0.8 ** torch.arange(32, dtype=torch.float32)
    M16 = ((torch.randn(nb, m, 32, generator=g) * sig) @ torch.randn(nb, 32, 128, generator=g)
           + 0.02 * torch.randn(nb, m, 128, generator=g)).to(dtype)
    Omega = torch.randn(nb, 128, k + 8, generator=g)
    U, S, Vh = _ops.rsvd(M16.cuda(), Omega.cuda(), k, 2)
    U32, S32, Vh32 = _ops.rsvd(M16.float().cuda(), Omega.cuda(), k, 2)
    assert torch.isfinite(S).all() and torch.isfinite(U).all() and torch.isfinite(Vh).all()
    torch.testing.assert_close(S, S32, rtol=1e-4, atol=1e-5 * S32[:, :1].max().item())
    R = (U * S[:, None, :]) @ Vh
    R32 = (U32 * S32[:, None, :]) @ Vh32
    rel = (R - R32).norm(dim=(1, 2)) / R32.norm(dim=(1, 2))
    assert rel.max().item() <= 1e-4, rel.max().item()
    idx = [0, 1, 147, 148, 295, 296, 297, 591, 592, nb - 1]
    Mf = M16[idx].float().numpy()
    err = so.relative_reconstruction_error(Mf, U[idx].cpu().numpy(), S[idx].cpu().numpy(), Vh[idx].cpu().numpy())
    U64, S64, Vh64 = so.batched_randomized_svd(Mf, k, 2, 8, Omega[idx].numpy())
    err64 = so.relative_reconstruction_error(Mf, U64, S64, Vh64)
    assert np.abs(err - err64).max() <= 1e-3, (err, err64)


@pytest.mark.parametrize("m,k,q,dtype", [(512, 32, 2, torch.float16), (512, 16, 2, torch.bfloat16),
                                         (384, 32, 1, torch.float16), (256, 16, 0, torch.float16),
                                         (128, 32, 2, torch.bfloat16), (512, 32, 0, torch.bfloat16)])
def test_rsvd_fused_kernel_matches_chain(monkeypatch, m, k, q, dtype):
    """The fused subspace iteration (one CTA per block, M resident in shared memory, the
    panels in tensor memory) against the multi-kernel chain on the same inputs: the same
    products, pass rules and pivots, so singular values agree to float32 rounding and
    the reconstructions to 1e-4; both match the float64 reference algorithm's error
    within 1e-3.  300 blocks: more than two waves of one CTA per SM."""
    from unsloth_spectral import _ops
    g = torch.Generator().manual_seed(40 + m + k + q)
    nb = 300
    sig = 0.9 ** torch.arange(48, dtype=torch.float32)
    M16 = ((torch.randn(nb, m, 48, generator=g) * sig) @ torch.randn(nb, 48, 128, generator=g)
           + 0.01 * torch.randn(nb, m, 128, generator=g)).to(dtype)
    Omega = torch.randn(nb, 128, k + 8, generator=g)
    monkeypatch.setenv("SPX_RSVD_PATH", "fused")
    U, S, Vh = _ops.rsvd(M16.cuda(), Omega.cuda(), k, q)
    monkeypatch.setenv("SPX_RSVD_PATH", "chain")
    Uc, Sc, Vhc = _ops.rsvd(M16.cuda(), Omega.cuda(), k, q)
    monkeypatch.delenv("SPX_RSVD_PATH")
    assert torch.isfinite(S).all() and torch.isfinite(U).all() and torch.isfinite(Vh).all()
    torch.testing.assert_close(S, Sc, rtol=1e-4, atol=1e-5 * Sc[:, :1].max().item())
    R = (U * S[:, None, :]) @ Vh
    Rc = (Uc * Sc[:, None, :]) @ Vhc
    rel = (R - Rc).norm(dim=(1, 2)) / Rc.norm(dim=(1, 2))
    assert rel.max().item() <= 1e-4, rel.max().item()
    idx = [0, 1, 147, 148, 149, 295, 296, nb - 1]
    Mf = M16[idx].float().numpy()
    err = so.relative_reconstruction_error(Mf, U[idx].cpu().numpy(), S[idx].cpu().numpy(), Vh[idx].cpu().numpy())
    U64, S64, Vh64 = so.batched_randomized_svd(Mf, k, q, 8, Omega[idx].numpy())
    err64 = so.relative_reconstruction_error(Mf, U64, S64, Vh64)
    assert np.abs(err - err64).max() <= 1e-3, (err, err64)


def test_rsvd_zero_block():
    """An all-zero block compresses to zero singular values and zero codes, no NaN."""
    from unsloth_spectral import _ops
    M = torch.zeros(3, 512, 128, dtype=torch.float16, device="cuda")
    Omega = torch.randn(3, 128, 24, device="cuda")
    codes = torch.full((3, 512, 16), 7, dtype=torch.int8, device="cuda")
    qscale = torch.zeros(3, device="cuda")
    U, S, Vh = _ops.rsvd(M, Omega, 16, 2, codes=codes, codes_strides=(512 * 16, 16, 1), qscale=qscale)
    for x in (U, S, Vh, qscale):
        assert torch.isfinite(x).all()
    assert (S == 0).all()
    assert (codes == 0).all()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_public_rsvd_draws_the_reference_sketch(dtype):
    """batched_randomized_svd draws its sketch as rsvd.py:95 does; with the same seed the
    oracle (fed that sketch) gives the same reconstruction error."""
    from unsloth_spectral import batched_randomized_svd
    g = torch.Generator().manual_seed(5)
    M = torch.randn(6, 512, 128, generator=g).to(dtype).cuda()
    torch.manual_seed(123)
    U, S, Vh = batched_randomized_svd(M, 16, n_iter=2, oversampling=8)
    torch.manual_seed(123)
    omega = torch.randn(6, 128, 24, device="cuda")
    Mf = M.float().cpu().numpy()
    ref = so.relative_reconstruction_error(Mf, *so.batched_randomized_svd(Mf, 16, 2, 8, omega.cpu().numpy()))
    got = so.relative_reconstruction_error(Mf, U.float().cpu().numpy(), S.float().cpu().numpy(),
                                           Vh.float().cpu().numpy())
    assert np.abs(got - ref).max() <= 1e-3
    assert U.dtype == dtype


def test_cache_compression_codes_bit_exact_and_error_parity():
    """Appending a full block compresses it on the device; the stored INT8 codes equal
    the oracle quantiser applied to the kernel's own C = U*S, and the block's
    reconstruction error matches the reference algorithm on the same sketch."""
    from unsloth_spectral import SpectralCache, _ops
    from unsloth_spectral import synthetic as syn
    H, D, T = 8, 128, 512
    K, V = syn.kv_per_head(1, 0, 1, H, T + 5, D, 24, 0.85)
    cache = SpectralCache(H, D, block_size=T, k_rank_keys=16, k_rank_values=32, device="cuda",
                          dtype=torch.float16, oversampling=8)
    torch.manual_seed(77)
    cache.append(K.half().cuda(), V.half().cuda())
    assert cache.num_cold_blocks == 1 and cache.hot_len == 5
    torch.manual_seed(77)
    om_k = torch.randn(H, D, 24, device="cuda")
    om_v = torch.randn(H, D, 40, device="cuda")
    Kb = K[0, :, :T].half().cuda()
    U, S, Vh = _ops.rsvd(Kb, om_k, 16, 2)
    C = (U * S[:, None, :]).cpu().numpy()
    _, mm, codes, scale = so.quantize_int8_batched(C)
    t = cache.tiers
    np.testing.assert_array_equal(t.codes_k[0, :, 0, :, :16].cpu().numpy(), codes)
    assert (t.codes_k[0, :, 0, :, 16:] == 0).all()
    np.testing.assert_array_equal(t.scale_k[0, :, 0].cpu().numpy(), scale)
    np.testing.assert_array_equal(t.minmax_k[0, :, 0].cpu().numpy(), mm)
    # value codes are stored in the value-tile layout; untile and compare the same way
    Uv, Sv, _ = _ops.rsvd(V[0, :, :T].half().cuda(), om_v, 32, 2)
    _, mm_v, codes_v, scale_v = so.quantize_int8_batched((Uv * Sv[:, None, :]).cpu().numpy())
    nat = torch.empty_like(t.codes_v[0, :, 0])
    nat[:, _ops.vtile_index(T, t.rank_v_pad, nat.device)] = t.codes_v[0, :, 0]
    nat = nat.view(H, t.rank_v_pad, T).cpu().numpy()
    np.testing.assert_array_equal(nat[:, :32].transpose(0, 2, 1), codes_v)
    assert (nat[:, 32:] == 0).all()
    np.testing.assert_array_equal(t.scale_v[0, :, 0].cpu().numpy(), scale_v)
    # reconstruction error of the stored block vs the oracle on the same sketches
    Kr, Vr = cache.get_kv()
    for X, Xr, om, k in ((K, Kr, om_k, 16), (V, Vr, om_v, 32)):
        Xh = X[0, :, :T].half().float().numpy()
        got = np.linalg.norm((Xr[0, :, :T].float().cpu().numpy() - Xh).reshape(H, -1), axis=1) / \
            np.linalg.norm(Xh.reshape(H, -1), axis=1)
        q, Vh_, mm_, codes_, sc_ = so.compress_tensor(Xh, k, om.cpu().numpy(), 2, 8)
        ref = np.linalg.norm((np.matmul(q, Vh_) - Xh).reshape(H, -1), axis=1) / \
            np.linalg.norm(Xh.reshape(H, -1), axis=1)
        assert np.abs(got - ref).max() <= 1e-3, (got, ref)
    # the hot remainder is the last 5 tokens
    np.testing.assert_array_equal(cache.hot_K.cpu().numpy(), K[:, :, T:].half().numpy())
    assert cache.hot_position_ids.cpu().tolist() == [[512, 513, 514, 515, 516]]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_cache_prompt_compression_batched_equals_blockwise(dtype):
    """A prompt that fills several blocks is compressed with one rSVD launch for the keys
    and one for the values; with the same seed it must give exactly the cold tier (codes,
    scales, min/max, bases, block positions) and hot tier that appending the prompt one
    block at a time gives (the per-block path, two launches per block)."""
    from unsloth_spectral import SpectralCache
    from unsloth_spectral import synthetic as syn
    B, H, D, T, nfull, extra = 2, 4, 128, 512, 4, 100
    K, V = syn.kv_per_head(3, 0, B, H, nfull * T + extra, D, 24, 0.85)
    K, V = K.to(dtype).cuda(), V.to(dtype).cuda()

    def build(chunks):
        cache = SpectralCache(H, D, block_size=T, k_rank_keys=16, k_rank_values=32, device="cuda",
                              dtype=dtype, oversampling=8)
        torch.manual_seed(19)
        for c0, c1 in chunks:
            cache.append(K[:, :, c0:c1], V[:, :, c0:c1])
        return cache

    whole = build([(0, nfull * T + extra)])
    steps = [(c0, min(c0 + T, nfull * T + extra)) for c0 in range(0, nfull * T + extra, T)]
    blockwise = build(steps)
    assert whole.num_cold_blocks == blockwise.num_cold_blocks == nfull
    assert whole.compression_count == blockwise.compression_count == nfull
    a, b = whole.tiers, blockwise.tiers
    for name in ("codes_k", "codes_v", "scale_k", "scale_v", "minmax_k", "minmax_v", "basis_k", "basis_v"):
        x, y = getattr(a, name)[:, :, :nfull], getattr(b, name)[:, :, :nfull]
        assert torch.equal(x, y), name
    assert torch.equal(a.block_pos[:nfull], b.block_pos[:nfull])
    assert a.block_pos[:nfull].tolist() == [i * T for i in range(nfull)]
    assert torch.equal(whole.hot_K, blockwise.hot_K) and torch.equal(whole.hot_V, blockwise.hot_V)
    assert torch.equal(whole.hot_position_ids, blockwise.hot_position_ids)


def test_cache_state_dict_decodes_identically():
    """A compressed cache saved with state_dict (torch.save / torch.load) and loaded into
    a fresh cache decodes to exactly the same output."""
    import io
    from unsloth_spectral import SpectralCache, spectral_attention_forward
    from unsloth_spectral import synthetic as syn
    B, H, nrep, D, T = 2, 4, 4, 128, 512
    K, V = syn.kv_per_head(4, 0, B, H, 2 * T + 70, D, 24, 0.85)
    cache = SpectralCache(H, D, block_size=T, k_rank_keys=16, k_rank_values=32, device="cuda",
                          dtype=torch.float16, oversampling=8)
    torch.manual_seed(23)
    cache.append(K.half().cuda(), V.half().cuda())
    buf = io.BytesIO()
    torch.save(cache.state_dict(), buf)
    buf.seek(0)
    other = SpectralCache(H, D, block_size=T, k_rank_keys=16, k_rank_values=32, device="cuda",
                          dtype=torch.float16, oversampling=8)
    other.load_state_dict(torch.load(buf))
    qpos = 2 * T + 70
    cos, sin = syn.rope_tables(qpos + 8, D, 1e6, device=torch.device("cuda"))
    Q = (torch.randn(B, H * nrep, 1, D, generator=torch.Generator().manual_seed(2)) / math.sqrt(D)).half().cuda()
    a = spectral_attention_forward(Q, cache, cos, sin, qpos)
    b = spectral_attention_forward(Q, other, cos, sin, qpos)
    assert torch.isfinite(a).all()
    assert torch.equal(a, b)


# ------------------------------------------------- fast cold-tier kernel vs generic
FAST_CASES = [
    # seed, B, H, nrep, D, T, nblk, kK, kV, hot, masked   (FP16, D=128, tied, no mask)
    (31, 2, 8, 4, 128, 512, 3, 32, 32, 64, False),
    (32, 3, 2, 8, 128, 128, 5, 32, 16, 7, False),
    (33, 1, 4, 1, 128, 256, 4, 16, 16, 0, False),
    (34, 2, 2, 2, 128, 512, 2, 16, 32, 130, False),
    (35, 5, 8, 4, 128, 512, 9, 32, 32, 1, False),   # several CTAs per block (unit chunks)
]


@pytest.fixture
def generic_path(monkeypatch):
    """use(True): the generic FP32 cold-tier kernel; use(False): the reconstruct kernel."""
    def use(flag):
        monkeypatch.setenv("SPX_DECODE_PATH", "generic" if flag else "fast")
    return use


@pytest.mark.parametrize("case", FAST_CASES)
@pytest.mark.parametrize("mode", ["forward", "decode"])
def test_fast_kernel_matches_oracle_and_generic(case, mode, generic_path):
    r = _random_case(*case)
    generic_path(False)
    fast, ref = _run_random(r, torch.float16, mode)
    _close(fast, ref)
    generic_path(True)
    gen, _ = _run_random(r, torch.float16, mode)
    _close(fast, gen)
    generic_path(False)


@pytest.mark.parametrize("case", [FAST_CASES[0], FAST_CASES[2], FAST_CASES[4]])
@pytest.mark.parametrize("mode", ["forward", "decode"])
def test_fast_kernel_bf16_cache(case, mode, generic_path):
    """A BF16 cache runs the reconstruct kernel (bases and queries converted to FP16 where
    they are staged) and matches the oracle over the same BF16 values, and the generic
    FP32 kernel."""
    r = _random_case(*case)
    generic_path(False)
    assert _path_of(r, torch.bfloat16, mode) == 1
    fast, ref = _run_random(r, torch.bfloat16, mode)
    _close(fast, ref)
    generic_path(True)
    gen, _ = _run_random(r, torch.bfloat16, mode)
    _close(fast, gen)
    generic_path(False)


# (case, plan): plans drive several items and multi-block ranges through one CTA, the
# way large workloads run (units per item, blocks per range, CTAs)
PLAN_CASES = [
    ((51, 3, 4, 4, 128, 512, 6, 32, 32, 9, False), "4,3,2"),     # 3 items per CTA, 3-block ranges
    ((52, 3, 4, 4, 128, 512, 6, 32, 32, 9, False), "5,2,3"),     # ragged last group of units
    ((53, 2, 4, 2, 128, 512, 5, 16, 32, 0, False), "8,5,1"),     # one CTA merges all blocks
    ((54, 2, 4, 8, 128, 256, 7, 32, 16, 3, False), "3,4,2"),     # two M-tiles, ragged last range
]


@pytest.mark.parametrize("case,plan", PLAN_CASES)
def test_fast_kernel_multi_item_plans(case, plan, generic_path, monkeypatch):
    r = _random_case(*case)
    monkeypatch.setenv("SPX_FAST_PLAN", plan)
    generic_path(False)
    fast, ref = _run_random(r, torch.float16, "decode")
    _close(fast, ref)
    generic_path(True)
    gen, _ = _run_random(r, torch.float16, "decode")
    _close(fast, gen)
    generic_path(False)


def test_fast_kernel_long_context_properties(generic_path):
    """A 16-block (8K-token) cache at k=32: fast and generic CUDA paths agree, the
    output is a convex combination of values (softmax weights), and the result is
    invariant to the order in which units are batched."""
    r = _random_case(41, 4, 8, 4, 128, 512, 16, 32, 32, 64, False)
    generic_path(False)
    fast, ref = _run_random(r, torch.float16, "decode")
    generic_path(True)
    gen, _ = _run_random(r, torch.float16, "decode")
    generic_path(False)
    _close(fast, gen)
    _close(fast, ref)
    # one sequence alone gives the same answer as inside the batch
    r1 = {k: (v[1:2] if isinstance(v, np.ndarray) and k in ("codes_K", "codes_V", "scale_K", "scale_V",
                                                               "basis_K", "basis_V", "hot_K", "hot_V", "Q")
              else v) for k, v in r.items()}
    r1["B"] = 1
    one, _ = _run_random(r1, torch.float16, "decode")
    np.testing.assert_allclose(one[0], fast[1], atol=2e-3)


# ------------------------------------------- projection cold-tier kernel vs generic
def _path_of(r, dtype, mode):
    """The cold-tier kernel spx_decode_attn picks for case ``r`` (spx_decode_path)."""
    from unsloth_spectral import _native as N, _ops
    B, H, D, T = r["B"], r["H"], r["D"], r["T"]
    cache = cache_from_arrays(H, D, T, r["kK"], r["kV"], r["codes_K"], r["scale_K"], r["basis_K"], r["codes_V"],
                              r["scale_V"], r["basis_V"], r["start"], r["hot_K"], r["hot_V"], r["hot_pos"], dtype,
                              B=B)
    q = torch.from_numpy(r["Q"]).cuda().to(dtype).reshape(1, B, -1, D).contiguous()
    cos, sin = torch.from_numpy(r["cos"]).cuda(), torch.from_numpy(r["sin"]).cuda()
    rm = N.SPX_ROPE_DISTANCE if mode == "forward" else N.SPX_ROPE_ABSOLUTE
    a, _, keep = _ops.decode_args(q, cache.tiers, cos, sin, r["qpos"], rope_mode=rm)
    return N.load().spx_decode_path(a)


@pytest.fixture
def decode_path(monkeypatch):
    def use(name):
        if name is None:
            monkeypatch.delenv("SPX_DECODE_PATH", raising=False)
        else:
            monkeypatch.setenv("SPX_DECODE_PATH", name)
    return use


PROJ_CASES = [
    # seed, B, H, nrep, D, T, nblk, kK, kV, hot, masked   (FP16, D=128, linear RoPE, no mask)
    (61, 2, 8, 4, 128, 512, 3, 32, 32, 64, False),
    (62, 3, 2, 8, 128, 256, 5, 16, 16, 7, False),      # n_rep 8 x rank 16 = 128 columns
    (63, 1, 4, 1, 128, 256, 4, 16, 16, 0, False),      # MHA, 16 columns, no hot tier
    (64, 2, 2, 2, 128, 512, 2, 16, 32, 130, False),
    (65, 5, 8, 4, 128, 512, 9, 32, 32, 1, False),
    (66, 2, 4, 4, 128, 512, 3, 16, 32, 20, False),     # 64 columns
    (67, 1, 2, 2, 128, 256, 6, 32, 16, 5, False),
]


@pytest.mark.parametrize("case", PROJ_CASES)
@pytest.mark.parametrize("mode", ["forward", "decode"])
def test_proj_kernel_matches_oracle_and_generic(case, mode, decode_path):
    r = _random_case(*case)
    decode_path("proj")
    from unsloth_spectral import _native as N
    assert _path_of(r, torch.float16, mode) == N.SPX_PATH_PROJECTION
    proj, ref = _run_random(r, torch.float16, mode)
    _close(proj, ref)
    decode_path("generic")
    gen, _ = _run_random(r, torch.float16, mode)
    decode_path(None)
    _close(proj, gen)


@pytest.mark.parametrize("case,plan", [
    ((71, 3, 4, 4, 128, 512, 6, 32, 32, 9, False), "4,3,2"),
    ((72, 3, 4, 4, 128, 512, 6, 32, 32, 9, False), "5,2,3"),
    ((73, 2, 4, 2, 128, 512, 5, 16, 32, 0, False), "8,5,1"),
    ((74, 2, 4, 8, 128, 256, 7, 16, 16, 3, False), "3,4,2"),
    ((75, 4, 8, 4, 128, 512, 3, 32, 32, 2, False), "32,1,1"),    # 32 units through one CTA
])
def test_proj_kernel_multi_item_plans(case, plan, decode_path, monkeypatch):
    r = _random_case(*case)
    monkeypatch.setenv("SPX_FAST_PLAN", plan)
    decode_path("proj")
    proj, ref = _run_random(r, torch.float16, "decode")
    _close(proj, ref)


def test_proj_kernel_distance_mode_keys_past_the_query(decode_path):
    """DISTANCE mode with the query placed inside the cold tier: the reference clamps the
    distance of later keys to 0 (spectral_attention.py:198), which the projection kernel
    handles with unrotated projections for those tokens."""
    r = _random_case(76, 2, 4, 4, 128, 512, 3, 32, 32, 10, False)
    r["qpos"] = 700          # inside block 1; block 2 and the hot tier lie after it
    decode_path("proj")
    from unsloth_spectral import _native as N
    assert _path_of(r, torch.float16, "forward") == N.SPX_PATH_PROJECTION
    proj, ref = _run_random(r, torch.float16, "forward")
    _close(proj, ref)


@pytest.mark.parametrize("mode", ["decode", "forward"])
def test_fast_kernel_headline_shape(decode_path, monkeypatch, mode):
    """The reconstruct kernel (the default cold tier) at the timed configuration's
    geometry: 64 blocks of 512 at k=32, n_rep 4, 64 hot tokens, the work plan of the full
    run (32 units per item, 16-block ranges, so every CTA merges 16 blocks per unit in
    its FP16-accumulator arithmetic), on a reduced batch (4 sequences x 8 KV heads);
    against the float32 oracle and the generic FP32 kernel."""
    r = _random_case(76, 4, 8, 4, 128, 512, 64, 32, 32, 64, False)
    monkeypatch.setenv("SPX_FAST_PLAN", "32,16,4")
    decode_path("fast")
    assert _path_of(r, torch.float16, mode) == 1
    fast, ref = _run_random(r, torch.float16, mode)
    _close(fast, ref)
    monkeypatch.delenv("SPX_FAST_PLAN")
    decode_path("generic")
    gen, _ = _run_random(r, torch.float16, mode)
    decode_path(None)
    _close(fast, gen)


def test_proj_kernel_headline_shape(decode_path, monkeypatch):
    """The timed configuration's geometry (64 blocks of 512 at k=32, n_rep 4, 64 hot,
    the work plan of the full run: 32 units per item, 16-block ranges) on a reduced
    batch: projection kernel against the float32 oracle and the generic kernel."""
    r = _random_case(77, 4, 8, 4, 128, 512, 64, 32, 32, 64, False)
    monkeypatch.setenv("SPX_FAST_PLAN", "32,16,4")
    decode_path("proj")
    proj, ref = _run_random(r, torch.float16, "decode")
    _close(proj, ref)
    monkeypatch.delenv("SPX_FAST_PLAN")
    decode_path("generic")
    gen, _ = _run_random(r, torch.float16, "decode")
    decode_path(None)
    _close(proj, gen)


def test_proj_kernel_needs_linear_rope_tables(decode_path):
    """Tables that are not cos/sin(position * theta) keep the reconstruct kernel."""
    from unsloth_spectral import _native as N
    r = _random_case(78, 1, 2, 4, 128, 512, 2, 32, 32, 3, False)
    r["cos"] = r["cos"] * (1.0 + 0.01 * np.arange(r["cos"].shape[0], dtype=np.float32)[:, None] / 1000)
    decode_path("proj")
    assert _path_of(r, torch.float16, "decode") == N.SPX_PATH_RECONSTRUCT
