"""End-to-end decoder on the packed cache (benchmark config 5 geometry, scaled
down): eager and CUDA-graph steps agree, and one decode step's attention equals
dense attention over the cache's own dequantized K/V."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from torque_mlx_b200.decoder import DecoderConfig, PackedKVDecoder  # noqa: E402

TINY = dict(num_layers=2, hidden=256, q_heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000, bits=4)


@pytest.mark.parametrize("fold", ["full", "vo_only"])
def test_graph_and_eager_generation_agree(fold):
    cfg = DecoderConfig(**TINY, fold=fold, seed=3)
    prompt = torch.randint(0, cfg.vocab, (37,), generator=torch.Generator().manual_seed(1)).cuda()
    eager = PackedKVDecoder(cfg, max_tokens=256)
    graph = PackedKVDecoder(cfg, max_tokens=256)
    te = eager.generate(prompt, 6, use_graph=False)
    tg = graph.generate(prompt, 6, use_graph=True)
    assert torch.equal(te, tg)
    assert eager.length == graph.length == 37 + 5
    for ce, cg in zip(eager.caches, graph.caches):
        assert np.array_equal(ce.packed_words()[0], cg.packed_words()[0])


def test_step_attention_matches_dense_over_dequantized_cache():
    cfg = DecoderConfig(**TINY, fold="full", seed=4)
    m = PackedKVDecoder(cfg, max_tokens=256, decode_mode="exact")
    prompt = torch.randint(0, cfg.vocab, (50,), generator=torch.Generator().manual_seed(2)).cuda()
    m.prefill(prompt)
    cache = m.caches[0]
    q = torch.randn(cfg.q_heads, cfg.head_dim, device="cuda")
    got = cache.decode(query=q).cpu().numpy()
    K, V = cache.export_dequantized()  # rotated basis, [1, Hkv, T, d]
    G = cfg.q_heads // cfg.kv_heads
    qn = q.cpu().numpy().astype(np.float64)
    for h in range(cfg.q_heads):
        k, v = K[0, h // G].astype(np.float64), V[0, h // G].astype(np.float64)
        s = k @ qn[h] / np.sqrt(cfg.head_dim)
        p = np.exp(s - s.max())
        np.testing.assert_allclose(got[h], (p @ v) / p.sum(), atol=2e-5, rtol=1e-4)
