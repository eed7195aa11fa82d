"""Pin the CPU oracle to the reference's own outputs (tests/golden/golden.npz,
made by tests/golden/make_golden.py from the reference's numpy code)."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from oracle import torque_oracle as O


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("seed", [0, 3, 11])
def test_signs_match_reference(golden, d, seed):
    sl, sr = O.rotation_signs(d, seed)
    np.testing.assert_array_equal(sl, golden[f"signs_l_d{d}_s{seed}"])
    np.testing.assert_array_equal(sr, golden[f"signs_r_d{d}_s{seed}"])


@pytest.mark.parametrize("d", [64, 128, 256])
def test_rotation_bit_exact(golden, d):
    sl, sr = O.rotation_signs(d, 3)
    x = golden[f"rot_in_d{d}"]
    np.testing.assert_array_equal(O.rotate(x, sl, sr), golden[f"rot_out_d{d}"])
    np.testing.assert_array_equal(O.rotate_inverse(x, sl, sr), golden[f"rot_inv_d{d}"])


def test_rotation_matrix(golden):
    sl, sr = O.rotation_signs(64, 3)
    m = O.rotate(np.eye(64, dtype=np.float32), sl, sr).T
    np.testing.assert_array_equal(m, golden["rot_matrix_d64"])


@pytest.mark.parametrize("b", [2, 3, 4])
@pytest.mark.parametrize("seed", [0, 1])
def test_codebook_bit_exact(golden, b, seed):
    np.testing.assert_array_equal(O.gaussian_codebook(b, seed=seed), golden[f"codebook_b{b}_s{seed}"])


def test_codebook_small(golden):
    np.testing.assert_array_equal(O.gaussian_codebook(4, sample_size=20_000, iterations=12, seed=7),
                                  golden["codebook_b4_small_s7"])


def test_quantize_ties(golden):
    cb = np.array([-1.0, -0.25, 0.25, 1.0], np.float32)
    np.testing.assert_array_equal(O.quantize(golden["quant_tie_values"], cb), golden["quant_tie_codes"])


@pytest.mark.parametrize("b", [2, 3, 4])
def test_quantize_midpoints(golden, b):
    cb = golden[f"codebook_b{b}_s0"]
    np.testing.assert_array_equal(O.quantize(golden[f"quant_vals_b{b}"], cb), golden[f"quant_codes_b{b}"])


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("b", [2, 3, 4])
def test_pack_unpack(golden, d, b):
    idx = golden[f"pack_codes_d{d}_b{b}"]
    words = O.pack(idx, b)
    np.testing.assert_array_equal(words, golden[f"pack_words_d{d}_b{b}"])
    np.testing.assert_array_equal(words[0], golden[f"pack_words_row0_d{d}_b{b}"])
    np.testing.assert_array_equal(O.unpack(words, b, d), idx)
    assert words.shape[-1] == O.packed_words(d, b)


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("b", [2, 3, 4])
def test_append_path(golden, d, b):
    sl, sr = O.rotation_signs(d, 0)
    cb = golden[f"codebook_b{b}_s0"]
    got = O.rotate_quantize_pack(golden[f"append_in_d{d}_b{b}"], sl, sr, cb, b)
    np.testing.assert_array_equal(got, golden[f"append_words_d{d}_b{b}"])


def test_streaming_decode(golden):
    got = O.streaming_attention_decode(golden["sad_q"], golden["sad_k"], golden["sad_v"])
    np.testing.assert_array_equal(got, golden["sad_out"])
    f64, _ = O.attention_f64(golden["sad_q"][None], golden["sad_k"], golden["sad_v"])
    np.testing.assert_allclose(f64[0], golden["sad_out"], atol=2e-6, rtol=1e-5)


def test_cache_config1_small(golden):
    c = O.OracleCache(bits=4, head_dim=128, kv_heads=8, rotation_seed=0)
    for t in range(32):
        c.append(golden["c1small_keys"][t], golden["c1small_values"][t])
    kw, vw = c.words()
    np.testing.assert_array_equal(kw[0], golden["c1small_kwords"])
    np.testing.assert_array_equal(vw[0], golden["c1small_vwords"])
    np.testing.assert_array_equal(c.decode(golden["c1small_query"])[0], golden["c1small_decode"])
    c.fused = True
    np.testing.assert_array_equal(c.decode(golden["c1small_query"])[0], golden["c1small_decode_fused"])


def test_cache_config1_full_digest(golden):
    rng = np.random.default_rng(0)
    keys = rng.standard_normal((512, 8, 128)).astype(np.float16)
    vals = rng.standard_normal((512, 8, 128)).astype(np.float16)
    qry = rng.standard_normal((8, 128)).astype(np.float32)
    sl, sr = O.rotation_signs(128, 0)
    ck, cv = golden["codebook_b4_s0"], golden["codebook_b4_s1"]
    kw = O.rotate_quantize_pack(keys, sl, sr, ck, 4).transpose(1, 0, 2)  # [H, seq, W]
    vw = O.rotate_quantize_pack(vals, sl, sr, cv, 4).transpose(1, 0, 2)
    assert hashlib.sha256(np.ascontiguousarray(kw).tobytes()).digest() == golden["c1_kwords_sha"].tobytes()
    assert hashlib.sha256(np.ascontiguousarray(vw).tobytes()).digest() == golden["c1_vwords_sha"].tobytes()
    qr = O.rotate(qry, sl, sr)
    out, _ = O.gqa_decode(qr[None], kw[None], vw[None], ck, cv, 4)
    res = O.rotate_inverse(out[0].astype(np.float32), sl, sr)
    np.testing.assert_allclose(res, golden["c1_decode"], atol=2e-5, rtol=1e-4)


def test_gqa_restatement(golden):
    sl, sr = O.rotation_signs(64, 5)
    # the reference cache draws K/V codebooks with seeds rotation_seed and +1 (cache.py:48-55)
    ck, cv = O.gaussian_codebook(3, seed=5), O.gaussian_codebook(3, seed=6)
    ks, vs = golden["gqa_keys"], golden["gqa_values"]  # [T, L, H, d]
    kw = O.rotate_quantize_pack(ks, sl, sr, ck, 3).transpose(1, 2, 0, 3)  # [L, H, T, W]
    vw = O.rotate_quantize_pack(vs, sl, sr, cv, 3).transpose(1, 2, 0, 3)
    K = O.dequantize(O.unpack(kw, 3, 64), ck)
    np.testing.assert_array_equal(K, golden["gqa_kdeq"])
    qr = O.rotate(golden["gqa_query"], sl, sr)
    out, _ = O.gqa_decode(qr, kw, vw, ck, cv, 3)
    res = O.rotate_inverse(out.astype(np.float32), sl, sr)
    np.testing.assert_allclose(res, golden["gqa_decode"], atol=2e-5, rtol=1e-4)


def test_lse_merge_equals_full():
    rng = np.random.default_rng(3)
    q = rng.standard_normal((4, 64))
    K = rng.standard_normal((100, 64))
    V = rng.standard_normal((100, 64))
    full, lse = O.attention_f64(q, K, V)
    parts = [O.attention_f64(q, K[a:b], V[a:b]) for a, b in ((0, 30), (30, 30), (30, 77), (77, 100))]
    m, l2 = O.lse_merge(np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts]))
    np.testing.assert_allclose(m, full, atol=1e-12)
    np.testing.assert_allclose(l2, lse, atol=1e-12)


@pytest.mark.parametrize("b", [2, 3, 4])
@pytest.mark.parametrize("d", [64, 128, 256])
def test_boundary_quantizer_matches_reference_mlx_rule(golden, d, b):
    """quantize_mlx (run by the golden script over a numpy stand-in for mlx.core)
    against the oracle's restatement: codes and packed words bit-exact."""
    cb = O.gaussian_codebook(b, seed=0)
    np.testing.assert_array_equal(O.boundaries(cb), golden[f"bnd_b{b}"])
    codes = O.quantize_boundaries(golden[f"qmlx_in_d{d}_b{b}"], golden[f"bnd_b{b}"])
    np.testing.assert_array_equal(codes, golden[f"qmlx_codes_d{d}_b{b}"])
    np.testing.assert_array_equal(O.pack(codes, b), golden[f"qmlx_words_d{d}_b{b}"])
