"""Pin the CPU oracle against outputs recorded from the reference implementation."""
import hashlib

import numpy as np
import pytest

from oracle import spectral_oracle as so
import golden_io as gio


def _cos(a, b):
    a, b = np.ravel(a).astype(np.float64), np.ravel(b).astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def test_quantize_matches_reference_bit_exact():
    z = gio.load("quant")
    q, mm, codes, scale = so.quantize_int8_batched(z["C"])
    assert np.array_equal(q, z["quantized"])          # bit-exact values
    assert np.array_equal(mm, z["scales"])
    # the stored (min, max) recovers the scale the reference divided by
    assert np.array_equal(so.scale_from_minmax(mm), scale)
    # round-half-to-even on the exact ties planted in head 5
    assert list(codes[5, 1, 0:6]) == [2, -4, 0, 0, 2, 126]
    assert np.all(codes[4] == 0)


@pytest.mark.parametrize("i", range(4))
def test_rsvd_matches_reference_error(i):
    z = gio.load("rsvd")
    M16, Omega = gio.rsvd_inputs(z, i)
    digest = hashlib.sha256(np.ascontiguousarray(M16.numpy()).tobytes()).hexdigest()[:16]
    assert digest == str(z[f"c{i}_M_digest"]), "synthetic generator drifted"
    k, q = int(z[f"c{i}_k"]), int(z[f"c{i}_q"])
    M = M16.float().numpy()
    # float64 run of the reference's algorithm with the same sketch: tight match
    U, S, Vh = so.batched_randomized_svd(M, k, q, 8, Omega.numpy())
    err = so.relative_reconstruction_error(M, U, S, Vh)
    np.testing.assert_allclose(err, z[f"c{i}_err64"], atol=1e-6)
    np.testing.assert_allclose(S, z[f"c{i}_S64"], rtol=1e-5)
    # float32 run: matches the reference's float32 result wherever that result is
    # not dominated by rounding (its float32/float64 gap below 1e-4)
    U, S, Vh = so.batched_randomized_svd(M, k, q, 8, Omega.numpy(), dtype=np.float32)
    err32 = so.relative_reconstruction_error(M, U, S, Vh)
    stable = np.abs(z[f"c{i}_err"] - z[f"c{i}_err64"]) < 1e-4
    np.testing.assert_allclose(err32[stable], z[f"c{i}_err"][stable], atol=1e-4)


@pytest.mark.parametrize("name", ["decode_cfg0", "decode_gqa_small", "decode_untied"])
def test_decode_matches_reference(name):
    c = gio.decode_case(name)
    args = (c["Q"], c["blocks"], c["hot_K"], c["hot_V"], c["hot_pos"], c["cos"], c["sin"],
            int(c["qpos"]))
    fwd = so.spectral_attention_forward(*args, scale=float(c["scale"]))
    dec = so.spectral_attention_decode(*args, scale=float(c["scale"]))
    np.testing.assert_allclose(fwd, c["out_forward"], atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(dec, c["out_decode"], atol=2e-5, rtol=1e-4)
    if "mask" in c:
        fm = so.spectral_attention_forward(*args, attention_mask=c["mask"], scale=float(c["scale"]))
        dm = so.spectral_attention_decode(*args, attention_mask=c["mask"], scale=float(c["scale"]))
        np.testing.assert_allclose(fm, c["out_forward_mask"], atol=2e-5, rtol=1e-4)
        np.testing.assert_allclose(dm, c["out_decode_mask"], atol=2e-5, rtol=1e-4)
    b0 = c["blocks"][0]
    sc = so.spectral_score_forward(c["Q"], b0.coeffs_K, b0.basis_K, c["cos"], c["sin"],
                                   b0.start_position)
    np.testing.assert_allclose(sc, c["scores_block0"], atol=1e-4, rtol=1e-4)
    val = so.spectral_value_forward(c["attn_block0"], b0.coeffs_V, b0.basis_V)
    np.testing.assert_allclose(val, c["values_block0"], atol=1e-5, rtol=1e-4)


def test_get_kv_matches_reference_checksum():
    c = gio.decode_case("decode_cfg0")
    K, V = so.get_kv(c["blocks"], c["hot_K"], c["hot_V"])
    assert abs(K.astype(np.float64).sum() - float(c["getkv_K_sum"])) < 1e-2
    assert abs(V.astype(np.float64).sum() - float(c["getkv_V_sum"])) < 1e-2


def test_empty_cache_raises():
    Q = np.zeros((1, 4, 1, 64), np.float32)
    with pytest.raises(ValueError):
        so.spectral_attention_forward(Q, [], None, None, None, np.zeros((4, 64)), np.zeros((4, 64)), 3)
