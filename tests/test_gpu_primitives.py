"""Bit-exact parity of the GPU primitives (rotate, quantize, pack, unpack and
the fused rotate+quantize+pack append) with the reference's numpy results
(golden vectors) and with the oracle on fresh seeded inputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import torque_oracle as O

pytestmark = pytest.mark.gpu

import torque_mlx_b200 as T  # noqa: E402


@pytest.mark.parametrize("d", [64, 128, 256])
def test_rotation_bit_exact(golden, d):
    spec = T.RotationSpec.from_seed(head_dim=d, seed=3)
    np.testing.assert_array_equal(spec.signs_left, golden[f"signs_l_d{d}_s3"])
    x = golden[f"rot_in_d{d}"]
    np.testing.assert_array_equal(spec.apply(x), golden[f"rot_out_d{d}"])
    np.testing.assert_array_equal(spec.inverse(x), golden[f"rot_inv_d{d}"])


@pytest.mark.parametrize("dtype", [np.float16, np.float32])
@pytest.mark.parametrize("d", [64, 128, 256])
def test_rotation_random_and_torch(d, dtype):
    rng = np.random.default_rng(d)
    x = (rng.standard_normal((257, 3, d)) * 7).astype(dtype)
    spec = T.RotationSpec.from_seed(head_dim=d, seed=11)
    sl, sr = O.rotation_signs(d, 11)
    np.testing.assert_array_equal(spec.apply(x), O.rotate(x, sl, sr))
    y = spec.apply(torch.from_numpy(x).cuda())
    assert y.is_cuda and y.dtype == torch.float32
    np.testing.assert_array_equal(y.cpu().numpy(), O.rotate(x, sl, sr))
    np.testing.assert_allclose(spec.inverse(spec.apply(x.astype(np.float32))), x.astype(np.float32),
                               rtol=1e-5, atol=1e-4)


def test_rotation_matrix(golden):
    np.testing.assert_array_equal(T.RotationSpec.from_seed(64, 3).matrix(), golden["rot_matrix_d64"])


def test_quantize_ties(golden):
    cb = T.Codebook(bit_width=2, centroids=np.array([-1.0, -0.25, 0.25, 1.0], np.float32))
    np.testing.assert_array_equal(T.quantize(golden["quant_tie_values"], cb), golden["quant_tie_codes"])


@pytest.mark.parametrize("b", [2, 3, 4])
def test_quantize_midpoints_and_random(golden, b):
    cb = T.Codebook(bit_width=b, centroids=golden[f"codebook_b{b}_s0"])
    np.testing.assert_array_equal(T.quantize(golden[f"quant_vals_b{b}"], cb), golden[f"quant_codes_b{b}"])
    rng = np.random.default_rng(b)
    v = (rng.standard_normal(1 << 20) * 2).astype(np.float32)
    np.testing.assert_array_equal(T.quantize(v, cb), O.quantize(v, cb.centroids))


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("b", [2, 3, 4])
def test_pack_unpack(golden, d, b):
    idx = golden[f"pack_codes_d{d}_b{b}"]
    words = T.pack_indices_batched(idx, b)
    assert words.dtype == np.uint32
    np.testing.assert_array_equal(words, golden[f"pack_words_d{d}_b{b}"])
    np.testing.assert_array_equal(T.pack_indices(idx[0], b), golden[f"pack_words_row0_d{d}_b{b}"])
    np.testing.assert_array_equal(T.unpack_indices(golden[f"pack_words_row0_d{d}_b{b}"], b, d),
                                  golden[f"unpack_row0_d{d}_b{b}"])
    np.testing.assert_array_equal(T.unpack_indices(words, b, d), idx)


@pytest.mark.parametrize("b", [2, 3, 4])
@pytest.mark.parametrize("count", [1, 5, 31, 32, 33, 100])
def test_pack_ragged_counts(b, count):
    rng = np.random.default_rng(count)
    idx = rng.integers(0, 1 << b, size=(7, count), dtype=np.uint8)
    w = T.pack_indices_batched(idx, b)
    np.testing.assert_array_equal(w, O.pack(idx, b))
    np.testing.assert_array_equal(T.unpack_indices(w, b, count), idx)


def test_pack_rejects_out_of_range():
    with pytest.raises(ValueError):
        T.pack_indices(np.array([0, 4], np.uint8), 2)


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("b", [2, 3, 4])
def test_fused_append_bit_exact(golden, d, b):
    """pack(quantize(rotate(x))) in one kernel == the reference's three steps."""
    x = golden[f"append_in_d{d}_b{b}"]  # [2, 8, 16, d] fp16 with outlier channels
    cb = T.Codebook(bit_width=b, centroids=golden[f"codebook_b{b}_s0"])
    spec = T.RotationSpec.from_seed(head_dim=d, seed=0)
    words = T.quantize_and_pack_rows(x.reshape(-1, d), cb, bit_width=b, head_dim=d, rotation=spec)
    np.testing.assert_array_equal(words.reshape(golden[f"append_words_d{d}_b{b}"].shape),
                                  golden[f"append_words_d{d}_b{b}"])


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("b", [2, 3, 4])
def test_cache_slab_matches_reference_path(d, b):
    """Device slab == pack(quantize(rotate(x))) per (layer, head, token) —
    tests/test_cache_mlx.py:37-70 of the reference, on N(0,1) fp16 with 1%
    outlier channels x20 (the config-2 input distribution)."""
    rng = np.random.default_rng(100 * d + b)
    L, H, S = 2, 8, 77
    x = rng.standard_normal((L, H, S, d)).astype(np.float32)
    ch = rng.choice(d, size=max(1, d // 100), replace=False)
    x[..., ch] *= 20
    x = x.astype(np.float16)
    y = rng.standard_normal((L, H, S, d)).astype(np.float16)
    cache = T.TorqueKVCache(config=T.TorqueConfig(bit_width=b, head_dim=d, num_layers=L, kv_heads=H),
                            initial_capacity=64)
    cache.append(key=x[:, :, :40], value=y[:, :, :40])
    for t in range(40, S):
        cache.append(key=x[:, :, t], value=y[:, :, t])
    assert cache.sequence_length == S and cache.capacity >= S
    kw, vw = cache.packed_words()
    sl, sr = O.rotation_signs(d, 0)
    np.testing.assert_array_equal(kw, O.rotate_quantize_pack(x, sl, sr, cache.key_codebook.centroids, b))
    np.testing.assert_array_equal(vw, O.rotate_quantize_pack(y, sl, sr, cache.value_codebook.centroids, b))


def test_dual_append_primitive_and_dequantize():
    rng = np.random.default_rng(5)
    a = rng.standard_normal((33, 128)).astype(np.float32)
    bb = rng.standard_normal((33, 128)).astype(np.float32)
    ca, cb = T.build_gaussian_codebook(3, seed=0), T.build_gaussian_codebook(3, seed=1)
    wa, wb = T.quantize_and_pack_rows_dual(a, bb, ca, cb, bit_width=3, head_dim=128)
    np.testing.assert_array_equal(wa, O.pack(O.quantize(a, ca.centroids), 3))
    np.testing.assert_array_equal(wb, O.pack(O.quantize(bb, cb.centroids), 3))
    deq = T.dequantize_packed(wa, ca, bit_width=3, head_dim=128)
    np.testing.assert_array_equal(deq, O.dequantize(O.unpack(wa, 3, 128), ca.centroids))


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("b", [2, 3, 4])
def test_boundary_pack_metal_names_bit_exact(golden, d, b):
    """quantize_and_pack_rows[_dual]_metal keep the reference's names and
    arguments (mlx_ops.py:342-412) and its boundary-count rule: words equal
    the reference's quantize_mlx + pack_indices_batched, midpoints included."""
    x = golden[f"qmlx_in_d{d}_b{b}"]
    bnd = golden[f"bnd_b{b}"]
    want = golden[f"qmlx_words_d{d}_b{b}"]
    wa, wb = T.quantize_and_pack_rows_dual_metal(x, x[::-1].copy(), bnd, bnd, bit_width=b, head_dim=d)
    np.testing.assert_array_equal(wa, want)
    np.testing.assert_array_equal(wb, O.pack(O.quantize_boundaries(x[::-1], bnd), b))
    np.testing.assert_array_equal(T.quantize_and_pack_rows_metal(x, bnd, bit_width=b, head_dim=d), want)
    with pytest.raises(ValueError, match="boundaries_b must have shape"):
        T.quantize_and_pack_rows_dual_metal(x, x, bnd, bnd[:-1], bit_width=b, head_dim=d)
    with pytest.raises(ValueError, match="values_a and values_b must match"):
        T.quantize_and_pack_rows_dual_metal(x, x[:3], bnd, bnd, bit_width=b, head_dim=d)
