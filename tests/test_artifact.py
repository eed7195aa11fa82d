"""Artifact format parity with the reference (tests/golden/artifact_ref was
written by the reference's own TorqueArtifact.save)."""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import ROOT
from oracle import torque_oracle as O
from torque_mlx_b200.artifact import TorqueArtifact, TorqueArtifactManifest, load_torque_artifact

REF_DIR = ROOT / "tests" / "golden" / "artifact_ref"


def test_load_reference_artifact_and_round_trip(tmp_path):
    art = load_torque_artifact(REF_DIR)
    rc = art.runtime_config
    assert (rc.bit_width, rc.head_dim, rc.num_layers, rc.kv_heads, rc.rotation_seed) == (3, 64, 2, 2, 9)
    assert rc.fused_weights and rc.variant_id == "b3-h64-hadamard-fused"
    np.testing.assert_array_equal(art.key_codebook.centroids, O.gaussian_codebook(3, seed=9))
    np.testing.assert_array_equal(art.value_codebook.centroids, O.gaussian_codebook(3, seed=10))
    art.save(tmp_path / "copy")
    ref_manifest = json.loads((REF_DIR / "manifest.json").read_text())
    our_manifest = json.loads((tmp_path / "copy" / "manifest.json").read_text())
    assert our_manifest == ref_manifest
    back = TorqueArtifact.load(tmp_path / "copy")
    for k in ("w_q", "w_k", "w_v", "w_o"):
        np.testing.assert_array_equal(getattr(back.fused_weights, k), getattr(art.fused_weights, k))
    assert back.summary()["weight_shapes"]["w_o"] == [48, 64]


def test_manifest_validation():
    payload = json.loads((REF_DIR / "manifest.json").read_text())
    bad = dict(payload, runtime_config=dict(payload["runtime_config"], fused_weights=False))
    with pytest.raises(ValueError):
        TorqueArtifactManifest.from_dict(bad)
    with pytest.raises(ValueError):
        TorqueArtifactManifest.from_dict({k: v for k, v in payload.items() if k != "key_codebook"})
    with pytest.raises(FileExistsError):
        load_torque_artifact(REF_DIR).save(REF_DIR)


@pytest.mark.gpu
def test_fusion_and_build_cache_match_reference(golden, tmp_path):
    import torque_mlx_b200 as T
    ref = load_torque_artifact(REF_DIR)
    src = {k: golden[f"artifact_src_{k}"] for k in ("w_q", "w_k", "w_v", "w_o")}
    ours = T.build_torque_artifact(model_name="tiny", architecture="toy", source_format="npz",
                                   config=T.TorqueConfig(bit_width=3, head_dim=64, num_layers=2, kv_heads=2,
                                                         rotation_seed=9), **src)
    # the reference multiplies by a dense Pi in fp32 BLAS; the kernel rotates exactly
    for k in ("w_q", "w_k", "w_v", "w_o"):
        np.testing.assert_allclose(getattr(ours.fused_weights, k), getattr(ref.fused_weights, k), atol=2e-6, rtol=1e-5)
    assert ours.manifest.to_dict() == ref.manifest.to_dict()
    cache = ref.build_cache()
    assert isinstance(cache, T.TorqueKVCache) and cache.config.fused_weights
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 2, 5, 64)).astype(np.float32)
    cache.append(key=x, value=x)
    out = cache.decode(query=rng.standard_normal((2, 2, 64)).astype(np.float32))
    assert out.shape == (2, 2, 64) and np.isfinite(out).all()


@pytest.mark.gpu
def test_build_cache_decodes_like_the_reference_cache(golden):
    """A reference-written artifact, loaded here: build_cache() (the GPU cache)
    appends and decodes the same tokens as the reference's numpy cache built
    from the same artifact by the reference (artifact.py:157-162, golden
    vectors from tests/golden/make_golden.py)."""
    cache = load_torque_artifact(REF_DIR).build_cache()
    for t in range(golden["artcache_keys"].shape[0]):
        cache.append(key=golden["artcache_keys"][t], value=golden["artcache_values"][t])
    out = cache.decode(query=golden["artcache_query"])
    np.testing.assert_allclose(out, golden["artcache_decode"], atol=1e-5, rtol=1e-5)
