"""Chunked-prefill attention over packed codes (TorqueKVCache.attend_chunk,
tq_decode_causal) against the float64 oracle.

The chunk's K/V are appended first (bit-exact packing, as everywhere); then
every chunk token t attends the packed prefix and the chunk up to itself.
The oracle decodes each token with its own prefix of the very words the GPU
wrote (the reference's prefill attends dense fresh K/V, qwen_mlx.py:829-845;
here the chunk attends the packed cache, so the packed words are the
reference point).  Tensor-mode tolerance: atol 4e-3 / rtol 2e-2.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import torque_oracle as O

pytestmark = pytest.mark.gpu

import torque_mlx_b200 as T  # noqa: E402


def _oracle_chunk(cache, q, seq: int, prefix_len: int, T_: int):
    """q [layers, T, Hq, d] (unrotated) -> [layers, T, Hq, d]."""
    cfg = cache.config
    kw = cache.key_slab[seq, :, :, : prefix_len + T_].cpu().numpy().view(np.uint32)
    vw = cache.value_slab[seq, :, :, : prefix_len + T_].cpu().numpy().view(np.uint32)
    sl, sr = O.rotation_signs(cfg.head_dim, cfg.rotation_seed)
    out = np.zeros(q.shape)
    for layer in range(cfg.num_layers):
        for t in range(T_):
            qr = O.rotate(q[layer, t], sl, sr)
            o, _ = O.gqa_decode(qr[None], kw[layer][None], vw[layer][None], cache.key_codebook.centroids,
                                cache.value_codebook.centroids, cfg.bit_width,
                                lengths=np.array([prefix_len + t + 1]))
            o = o[0] if cfg.fused_weights else O.rotate_inverse(o[0].astype(np.float32), sl, sr)
            out[layer, t] = o
    return out


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("d,b,H,G,prefix,T_", [(128, 4, 2, 4, 300, 13), (64, 3, 2, 2, 37, 9), (256, 4, 2, 8, 5000, 5),
                                               (128, 2, 1, 1, 0, 21)])
def test_chunk_attention_matches_oracle(fused, d, b, H, G, prefix, T_):
    rng = np.random.default_rng(d + b + prefix)
    cfg = T.TorqueConfig(bit_width=b, head_dim=d, num_layers=1, kv_heads=H, fused_weights=fused)
    cache = T.TorqueKVCache(config=cfg, initial_capacity=128)
    n = prefix + T_
    cache.append(key=rng.standard_normal((H, n, d)).astype(np.float16),
                 value=rng.standard_normal((H, n, d)).astype(np.float16))
    q = rng.standard_normal((1, T_, H * G, d)).astype(np.float32)
    got = cache.attend_chunk(query=q)
    assert got.shape == q.shape
    np.testing.assert_allclose(got, _oracle_chunk(cache, q, 0, prefix, T_), atol=4e-3, rtol=2e-2)


def test_chunk_attention_batch_layers_ragged():
    """Two sequences of different lengths, two layers: every sequence's last
    T tokens are its chunk."""
    rng = np.random.default_rng(5)
    B, L, H, G, d, b, T_ = 2, 2, 2, 4, 128, 3, 6
    cfg = T.TorqueConfig(bit_width=b, head_dim=d, num_layers=L, kv_heads=H)
    cache = T.TorqueKVCache(config=cfg, batch_size=B, initial_capacity=128)
    lens = [700, 40]
    for s, n in enumerate(lens):
        cache.append_sequence(s, key=rng.standard_normal((L, H, n, d)).astype(np.float16),
                              value=rng.standard_normal((L, H, n, d)).astype(np.float16))
    q = rng.standard_normal((B, L, T_, H * G, d)).astype(np.float32)
    got = cache.attend_chunk(query=q)
    for s, n in enumerate(lens):
        np.testing.assert_allclose(got[s], _oracle_chunk(cache, q[s], s, n - T_, T_), atol=4e-3, rtol=2e-2)


def test_chunk_of_one_token_equals_decode():
    rng = np.random.default_rng(9)
    cfg = T.TorqueConfig(bit_width=4, head_dim=128, kv_heads=2)
    cache = T.TorqueKVCache(config=cfg, decode_mode="tensor")
    cache.append(key=rng.standard_normal((2, 500, 128)).astype(np.float16),
                 value=rng.standard_normal((2, 500, 128)).astype(np.float16))
    q = rng.standard_normal((8, 128)).astype(np.float32)
    chunk = cache.attend_chunk(query=q[None, None])[0, 0]
    np.testing.assert_allclose(chunk, cache.decode(query=q), atol=1e-6, rtol=1e-6)
