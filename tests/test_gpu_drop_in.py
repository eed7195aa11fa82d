"""The reference's own call patterns, replayed against this package.

Each test restates what a reference caller does, with the reference's names,
keywords and shapes, and checks the result the way the reference's tests do:
  * the Qwen adapter's cache construction and decode calls
    (src/torque_mlx/qwen_mlx.py:700, 720-724, 752-761);
  * tests/test_cache_mlx.py:20-35 (append tracks capacity), 37-70
    (append_many_mlx writes the reference's packed words), 74-116 and
    125-160 (grouped decode vs the streaming oracle, with a dense-tail knob),
    165-208 (decode_mlx_with_current vs append then decode), 211-236 (the
    decode-strategy resolution).
The reference skips these without Metal; here they run on the B200 path.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import torque_oracle as O

pytestmark = pytest.mark.gpu

import torque_mlx_b200 as T  # noqa: E402


def _uniform(b):
    return T.Codebook(bit_width=b, centroids=np.linspace(-1.0, 1.0, 1 << b, dtype=np.float32), name="uniform")


def _expected_grouped(cache_cfg, ck, cv, keys_steps, values_steps, grouped_query, seed):
    """tests/test_cache_mlx.py:104-114 restated: export the reference cache's
    dequantized K/V, then streaming decode per query head, rotated back."""
    ref = O.OracleCache(bits=cache_cfg.bit_width, head_dim=cache_cfg.head_dim, num_layers=1,
                        kv_heads=cache_cfg.kv_heads, rotation_seed=seed, cent_k=ck, cent_v=cv)
    for k, v in zip(keys_steps, values_steps):
        ref.append(key=k, value=v)
    kw, vw = ref.words()
    K = O.dequantize(O.unpack(kw, cache_cfg.bit_width, cache_cfg.head_dim), ck)
    V = O.dequantize(O.unpack(vw, cache_cfg.bit_width, cache_cfg.head_dim), cv)
    sl, sr = O.rotation_signs(cache_cfg.head_dim, seed)
    G = grouped_query.shape[0] // cache_cfg.kv_heads
    exp = np.zeros_like(grouped_query)
    for h in range(grouped_query.shape[0]):
        o = O.streaming_attention_decode(O.rotate(grouped_query[h], sl, sr), K[0, h // G], V[0, h // G])
        exp[h] = O.rotate_inverse(o.astype(np.float32), sl, sr)
    return exp


def test_append_tracks_capacity():
    cache = T.TorqueKVCacheMLX(config=T.TorqueConfig(bit_width=4, head_dim=64, num_layers=2, kv_heads=2),
                               key_codebook=_uniform(4), value_codebook=_uniform(4), initial_capacity=2)
    payload = np.zeros((2, 2, 64), dtype=np.float32)
    for _ in range(3):
        cache.append(key=payload, value=payload)
    assert cache.sequence_length == 3
    assert cache.capacity >= 3


def test_append_many_mlx_matches_numpy_reference():
    rng = np.random.default_rng(3)
    cache = T.TorqueKVCacheMLX(config=T.TorqueConfig(bit_width=4, head_dim=64, num_layers=2, kv_heads=2),
                               key_codebook=_uniform(4), value_codebook=_uniform(4), initial_capacity=8)
    keys = rng.uniform(-1.0, 1.0, size=(2, 2, 3, 64)).astype(np.float32)
    values = rng.uniform(-1.0, 1.0, size=(2, 2, 3, 64)).astype(np.float32)
    cache.append_many_mlx(key=torch.from_numpy(keys).cuda(), value=torch.from_numpy(values).cuda())
    sl, sr = O.rotation_signs(64, 0)
    ck = _uniform(4).centroids
    exp_k = O.pack(O.quantize(O.rotate(keys, sl, sr), ck), 4)
    exp_v = O.pack(O.quantize(O.rotate(values, sl, sr), ck), 4)
    np.testing.assert_array_equal(cache._key_codes[:, :, :3, :].cpu().numpy().view(np.uint32), exp_k)
    np.testing.assert_array_equal(cache._value_codes[:, :, :3, :].cpu().numpy().view(np.uint32), exp_v)
    assert cache.sequence_length == 3


@pytest.mark.parametrize("decode_tail_capacity,steps,seed", [(16, 6, 9), (2, 5, 19)])
def test_grouped_decode_matches_reference(decode_tail_capacity, steps, seed):
    rng = np.random.default_rng(seed)
    cfg = T.TorqueConfig(bit_width=4, head_dim=64, num_layers=1, kv_heads=2)
    cache = T.TorqueKVCacheMLX(config=cfg, key_codebook=_uniform(4), value_codebook=_uniform(4),
                               initial_capacity=8, decode_tail_capacity=decode_tail_capacity)
    ks, vs = [], []
    for _ in range(steps):
        ks.append(rng.uniform(-1.0, 1.0, size=(2, 64)).astype(np.float32))
        vs.append(rng.uniform(-1.0, 1.0, size=(2, 64)).astype(np.float32))
        cache.append(key=ks[-1], value=vs[-1])
    grouped_query = rng.uniform(-1.0, 1.0, size=(4, 64)).astype(np.float32)
    actual = cache.decode_mlx(query=grouped_query)
    assert isinstance(actual, np.ndarray) and actual.shape == (4, 64)
    exp = _expected_grouped(cfg, _uniform(4).centroids, _uniform(4).centroids,
                            [k[None] for k in ks], [v[None] for v in vs], grouped_query, 0)
    np.testing.assert_allclose(actual, exp, atol=3e-4, rtol=3e-4)


@pytest.mark.parametrize("decode_tail_capacity", [0, 2])
def test_decode_with_current_matches_append_then_decode(decode_tail_capacity):
    rng = np.random.default_rng(23)
    cfg = T.TorqueConfig(bit_width=4, head_dim=64, num_layers=1, kv_heads=2)
    mk = lambda: T.TorqueKVCacheMLX(config=cfg, key_codebook=_uniform(4), value_codebook=_uniform(4),  # noqa: E731
                                    initial_capacity=8, decode_tail_capacity=decode_tail_capacity)
    first, second = mk(), mk()
    for _ in range(4):
        key = rng.uniform(-1.0, 1.0, size=(2, 64)).astype(np.float32)
        value = rng.uniform(-1.0, 1.0, size=(2, 64)).astype(np.float32)
        first.append(key=key, value=value)
        second.append(key=key, value=value)
    grouped_query = rng.uniform(-1.0, 1.0, size=(4, 64)).astype(np.float32)
    current_key = rng.uniform(-1.0, 1.0, size=(2, 64)).astype(np.float32)
    current_value = rng.uniform(-1.0, 1.0, size=(2, 64)).astype(np.float32)
    actual = first.decode_mlx_with_current(query=grouped_query, key=current_key, value=current_value)
    second.append(key=current_key, value=current_value)
    expected = second.decode_mlx(query=grouped_query)
    np.testing.assert_allclose(actual, expected, atol=3e-4, rtol=3e-4)
    assert first.sequence_length == 4


def test_decode_strategy_resolution_and_validation():
    mk = lambda **kw: T.TorqueKVCacheMLX(  # noqa: E731
        config=T.TorqueConfig(bit_width=4, head_dim=64, num_layers=1, kv_heads=1),
        key_codebook=_uniform(4), value_codebook=_uniform(4), initial_capacity=4, **kw)
    assert mk(decode_strategy="auto").resolve_decode_strategy(sequence_length=128) == "split_batched"
    assert mk(decode_strategy="auto").resolve_decode_strategy(sequence_length=256) == "split_batched"
    assert mk().resolve_decode_strategy(sequence_length=32) == "split_batched"
    assert mk(decode_strategy="fused_per_head").resolve_decode_strategy() == "fused_per_head"
    with pytest.raises(ValueError, match="decode_strategy must be one of"):
        mk(decode_strategy="bogus")
    with pytest.raises(ValueError, match="decode_tail_capacity must be non-negative"):
        mk(decode_tail_capacity=-1)


def test_qwen_adapter_call_pattern():
    """qwen_mlx.py:752-761 builds the cache; :700 and :720-724 decode a
    [1, Hq, 1, d] query step with return_numpy=False and reshape the device
    result; the profiler reads last_decode_profile."""
    Hq, H, d = 8, 2, 128
    cfg = T.TorqueConfig(bit_width=4, head_dim=d, num_layers=1, kv_heads=H, fused_weights=True, rotation_seed=0)
    cache = T.TorqueKVCacheMLX(config=cfg, key_codebook=T.build_gaussian_codebook(4, seed=0),
                               value_codebook=T.build_gaussian_codebook(4, seed=1), decode_tail_capacity=16,
                               profile_decode_components=True, rotate_keys_on_append=True,
                               rotate_values_on_append=False, rotate_queries_on_decode=True)
    gen = torch.Generator(device="cuda").manual_seed(1)
    keys = torch.randn((1, H, 40, d), generator=gen, device="cuda")
    values = torch.randn((1, H, 40, d), generator=gen, device="cuda")
    cache.append_many_mlx(key=keys[0], value=values[0])  # prefill [kv_heads, T, d]
    queries = torch.randn((1, Hq, 1, d), generator=gen, device="cuda")
    out = cache.decode_mlx(query=queries[0, :, 0, :], return_numpy=False)
    assert isinstance(out, torch.Tensor) and out.is_cuda and tuple(out.shape) == (1, Hq, d)
    assert "packed_decode_seconds" in cache.last_decode_profile
    step = out.reshape(1, Hq, 1, d)
    cur_k = torch.randn((1, H, 1, d), generator=gen, device="cuda")
    cur_v = torch.randn((1, H, 1, d), generator=gen, device="cuda")
    with_cur = cache.decode_mlx_with_current(query=queries[0, :, 0, :], key=cur_k[0], value=cur_v[0],
                                             return_numpy=False)
    assert tuple(with_cur.shape) == (1, Hq, d) and cache.sequence_length == 40
    # the oracle: values are stored unrotated-then-not-rotated (rotate_values_on_append=False)
    sl, sr = O.rotation_signs(d, 0)
    k_all = torch.cat([keys[0], cur_k[0]], dim=1).cpu().numpy()
    v_all = torch.cat([values[0], cur_v[0]], dim=1).cpu().numpy()
    kw = O.pack(O.quantize(O.rotate(k_all, sl, sr), cache.key_codebook.centroids), 4)
    vw = O.pack(O.quantize(v_all, cache.value_codebook.centroids), 4)
    qr = O.rotate(queries[0, :, 0, :].cpu().numpy(), sl, sr)
    ref, _ = O.gqa_decode(qr[None], kw[None], vw[None], cache.key_codebook.centroids,
                          cache.value_codebook.centroids, 4)
    np.testing.assert_allclose(with_cur[0].cpu().numpy(), ref[0], atol=4e-3, rtol=2e-2)
    ref40, _ = O.gqa_decode(qr[None], kw[None, :, :40], vw[None, :, :40], cache.key_codebook.centroids,
                            cache.value_codebook.centroids, 4)
    np.testing.assert_allclose(step[0, :, 0].cpu().numpy(), ref40[0], atol=4e-3, rtol=2e-2)
