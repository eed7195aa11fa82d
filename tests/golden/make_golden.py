"""Generate the golden vectors that pin the oracle and the CUDA path.

Run in a container where the reference (cbun/torque-mlx) source tree is
available, naming its root with ``TORQUE_REFERENCE`` or as the first argument:

    TORQUE_REFERENCE=<reference root> python tests/golden/make_golden.py
    python tests/golden/make_golden.py <reference root>

The reference's numpy path imports ``mlx`` eagerly (mlx_ops.py:9 through
__init__.py:23 and cache.py:9) but never calls it, so an empty ``mlx`` stub
package is placed on ``sys.path`` first.  Every vector below is computed by the
reference's own functions; nothing here is computed by this repository's code.
The output ``golden.npz`` is committed; the GPU box never needs the reference.
"""

from __future__ import annotations

import hashlib
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF: Path | None = None


def _reference_root() -> Path:
    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TORQUE_REFERENCE")
    if not arg:
        raise SystemExit("usage: make_golden.py <reference root>  (or set TORQUE_REFERENCE)")
    root = Path(arg)
    if not (root / "src" / "torque_mlx").is_dir():
        raise SystemExit(f"{root} does not hold src/torque_mlx")
    return root


def _import_reference():
    stub = Path(tempfile.mkdtemp(prefix="mlx_stub_"))
    (stub / "mlx").mkdir()
    (stub / "mlx" / "__init__.py").write_text("")
    (stub / "mlx" / "core.py").write_text("")
    sys.path.insert(0, str(stub))
    sys.path.insert(0, str(REF / "src"))
    import torque_mlx.cache as cache
    import torque_mlx.config as config
    import torque_mlx.quantization as quant
    import torque_mlx.reference as reference
    import torque_mlx.rotation as rotation
    return cache, config, quant, reference, rotation


def sha(a: np.ndarray) -> np.ndarray:
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest(), dtype=np.uint8)


class _NumpyMx:
    """Just enough of ``mlx.core`` on numpy to run the reference's own
    ``quantize_mlx`` (quantization.py:139-148) unchanged: array, sum,
    expand_dims and the two dtypes it names."""

    float32 = np.float32
    uint32 = np.uint32

    @staticmethod
    def array(x, dtype=None):
        return np.asarray(x, dtype=dtype)

    sum = staticmethod(np.sum)
    expand_dims = staticmethod(np.expand_dims)


def _quantize_mlx_on_numpy(Q, values, codebook):
    core = sys.modules["mlx.core"]
    names = ("array", "sum", "expand_dims", "float32", "uint32")
    for n in names:
        setattr(core, n, getattr(_NumpyMx, n))
    try:
        return np.asarray(Q.quantize_mlx(values, codebook))
    finally:
        for n in names:
            delattr(core, n)


def main() -> None:
    global REF
    REF = _reference_root()
    cache_mod, config_mod, Q, R, ROT = _import_reference()
    out: dict[str, np.ndarray] = {}

    # --- rotation signs and rotate/inverse (rotation.py:75-102)
    for d in (64, 128, 256):
        for seed in (0, 3, 11):
            spec = ROT.RotationSpec.from_seed(head_dim=d, seed=seed)
            out[f"signs_l_d{d}_s{seed}"] = spec.signs_left
            out[f"signs_r_d{d}_s{seed}"] = spec.signs_right
        rng = np.random.default_rng(100 + d)
        x = rng.standard_normal((40, d)).astype(np.float32)
        x[:, :: max(1, d // 16)] *= 20.0  # outlier channels
        spec = ROT.RotationSpec.from_seed(head_dim=d, seed=3)
        out[f"rot_in_d{d}"] = x
        out[f"rot_out_d{d}"] = spec.apply(x)
        out[f"rot_inv_d{d}"] = spec.inverse(x)
        out[f"rot_matrix_d{d}"] = spec.matrix() if d == 64 else np.zeros(0, np.float32)

    # --- codebooks (quantization.py:89-117), the defaults the caches use
    for b in (2, 3, 4):
        for seed in (0, 1, 2, 3):
            out[f"codebook_b{b}_s{seed}"] = Q.build_gaussian_codebook(b, seed=seed).centroids
    out["codebook_b4_small_s7"] = Q.build_gaussian_codebook(4, sample_size=20_000, iterations=12, seed=7).centroids

    # --- quantize: random values, exact midpoints and the tie-break cases
    tie_cb = Q.Codebook(bit_width=2, centroids=np.array([-1.0, -0.25, 0.25, 1.0], np.float32))
    ties = np.array([-0.625, 0.0, 0.625, -0.9, -0.2, 0.3, 0.8, 5.0, -5.0], np.float32)
    out["quant_tie_values"] = ties
    out["quant_tie_codes"] = Q.quantize(ties, tie_cb)
    for b in (2, 3, 4):
        cb = Q.build_gaussian_codebook(b, seed=0)
        rng = np.random.default_rng(7 + b)
        vals = rng.standard_normal(4096).astype(np.float32) * 1.5
        mids = ((cb.centroids[:-1] + cb.centroids[1:]) / 2.0).astype(np.float32)
        near = np.concatenate([mids, np.nextafter(mids, np.float32(np.inf)), np.nextafter(mids, np.float32(-np.inf))])
        v = np.concatenate([vals, near, cb.centroids, np.array([0.0, -0.0, 1e30, -1e30], np.float32)]).astype(np.float32)
        out[f"quant_vals_b{b}"] = v
        out[f"quant_codes_b{b}"] = Q.quantize(v, cb)

    # --- packing (quantization.py:156-201, 272-290), all (d, b)
    for d in (64, 128, 256):
        for b in (2, 3, 4):
            rng = np.random.default_rng(d * 10 + b)
            idx = rng.integers(0, 1 << b, size=(6, d), dtype=np.uint8)
            out[f"pack_codes_d{d}_b{b}"] = idx
            out[f"pack_words_d{d}_b{b}"] = Q.pack_indices_batched(idx, b)
            out[f"pack_words_row0_d{d}_b{b}"] = Q.pack_indices(idx[0], b)
            out[f"unpack_row0_d{d}_b{b}"] = Q.unpack_indices(Q.pack_indices(idx[0], b), b, d)

    # --- append path: pack(quantize(rotate(x))) with fp16 N(0,1) + 1% outlier channels
    for d in (64, 128, 256):
        for b in (2, 3, 4):
            rng = np.random.default_rng(1000 + d + b)
            x = rng.standard_normal((2, 8, 16, d)).astype(np.float16)
            ch = rng.choice(d, size=max(1, d // 100), replace=False)
            x[..., ch] = (x[..., ch].astype(np.float32) * 20.0).astype(np.float16)
            spec = ROT.RotationSpec.from_seed(head_dim=d, seed=0)
            cb = Q.build_gaussian_codebook(b, seed=0)
            out[f"append_in_d{d}_b{b}"] = x
            out[f"append_words_d{d}_b{b}"] = Q.pack_indices_batched(Q.quantize(spec.apply(x), cb), b)

    # --- numpy cache end to end: config-1 geometry (cache.py:78-140).
    # Small case stored in full; the full 512-token case as digests + output.
    for name, seq in (("c1small", 32), ("c1", 512)):
        rng = np.random.default_rng(0)
        keys = rng.standard_normal((seq, 8, 128)).astype(np.float16)
        vals = rng.standard_normal((seq, 8, 128)).astype(np.float16)
        qry = rng.standard_normal((8, 128)).astype(np.float32)
        cfg = config_mod.TorqueConfig(bit_width=4, head_dim=128, num_layers=1, kv_heads=8, rotation_seed=0)
        c = cache_mod.TorqueKVCache(config=cfg)
        for t in range(seq):
            c.append(key=keys[t], value=vals[t])
        dec = c.decode(query=qry)
        kw = np.stack([np.stack(c._layers[0].key_codes[h]) for h in range(8)])
        vw = np.stack([np.stack(c._layers[0].value_codes[h]) for h in range(8)])
        out[f"{name}_decode"] = dec
        if name == "c1small":
            out[f"{name}_keys"] = keys
            out[f"{name}_values"] = vals
            out[f"{name}_query"] = qry
            out[f"{name}_kwords"] = kw
            out[f"{name}_vwords"] = vw
        else:
            out[f"{name}_kwords_sha"] = sha(kw.astype(np.uint32))
            out[f"{name}_vwords_sha"] = sha(vw.astype(np.uint32))
            out[f"{name}_kwords_head0_tok0_7"] = kw[0, :8]
        fused = cache_mod.TorqueKVCache(config=config_mod.TorqueConfig(
            bit_width=4, head_dim=128, num_layers=1, kv_heads=8, rotation_seed=0, fused_weights=True))
        if name == "c1small":
            for t in range(seq):
                fused.append(key=keys[t], value=vals[t])
            out[f"{name}_decode_fused"] = fused.decode(query=qry)

    # --- GQA decode as tests/test_cache_mlx.py:88-98 (2 layers, Hkv 2, G 4, 3-bit, d 64)
    rng = np.random.default_rng(9)
    cfg = config_mod.TorqueConfig(bit_width=3, head_dim=64, num_layers=2, kv_heads=2, rotation_seed=5)
    c = cache_mod.TorqueKVCache(config=cfg)
    ks = rng.uniform(-1, 1, size=(11, 2, 2, 64)).astype(np.float32)
    vs = rng.uniform(-1, 1, size=(11, 2, 2, 64)).astype(np.float32)
    for t in range(11):
        c.append(key=ks[t], value=vs[t])
    gq = rng.uniform(-1, 1, size=(2, 8, 64)).astype(np.float32)
    K, V = c.export_dequantized()
    exp = np.zeros_like(gq)
    for layer in range(2):
        for qh in range(8):
            o = R.streaming_attention_decode(c.rotation.apply(gq[layer, qh]), K[layer, qh // 4], V[layer, qh // 4])
            exp[layer, qh] = c.rotation.inverse(o)
    out["gqa_keys"] = ks
    out["gqa_values"] = vs
    out["gqa_query"] = gq
    out["gqa_decode"] = exp
    out["gqa_kdeq"] = K
    out["gqa_vdeq"] = V

    # --- streaming_attention_decode on plain data (reference.py:8-42)
    rng = np.random.default_rng(21)
    q = rng.standard_normal(64).astype(np.float32)
    Kp = rng.standard_normal((9, 64)).astype(np.float32)
    Vp = rng.standard_normal((9, 64)).astype(np.float32)
    out["sad_q"], out["sad_k"], out["sad_v"] = q, Kp, Vp
    out["sad_out"] = R.streaming_attention_decode(q, Kp, Vp)

    # --- an artifact written by the reference itself (artifact.py:164-184, 246-296)
    import torque_mlx.artifact as A
    rng = np.random.default_rng(44)
    w = {k: rng.standard_normal(s).astype(np.float32) * 0.05
         for k, s in (("w_q", (64, 32)), ("w_k", (64, 32)), ("w_v", (64, 32)), ("w_o", (48, 64)))}
    art = A.build_torque_artifact(model_name="tiny", architecture="toy", source_format="npz",
                                  config=config_mod.TorqueConfig(bit_width=3, head_dim=64, num_layers=2,
                                                                 kv_heads=2, rotation_seed=9), **w)
    art_dir = HERE / "artifact_ref"
    art.save(art_dir, force=True)
    for k, v in w.items():
        out[f"artifact_src_{k}"] = v

    # --- the MLX path's boundary-count quantizer (quantization.py:128-148), run
    # unchanged over a numpy stand-in for mlx.core, on random rows, exact
    # midpoints and their float neighbours
    for b in (2, 3, 4):
        cb = Q.build_gaussian_codebook(b, seed=0)
        out[f"bnd_b{b}"] = Q.codebook_boundaries(cb)
        rng = np.random.default_rng(70 + b)
        mids = out[f"bnd_b{b}"]
        edge = np.concatenate([mids, np.nextafter(mids, np.float32(np.inf)), np.nextafter(mids, np.float32(-np.inf))])
        for d in (64, 128, 256):
            x = (rng.standard_normal((12, d)) * 1.5).astype(np.float32)
            x.reshape(-1)[: edge.size] = edge
            out[f"qmlx_in_d{d}_b{b}"] = x
            codes = _quantize_mlx_on_numpy(Q, x, cb)
            out[f"qmlx_codes_d{d}_b{b}"] = codes.astype(np.uint8)
            out[f"qmlx_words_d{d}_b{b}"] = Q.pack_indices_batched(codes.astype(np.uint8), b)

    # --- TorqueArtifact.build_cache() (artifact.py:157-162) on the artifact
    # written above, loaded back by the reference, then appended and decoded
    loaded = A.load_torque_artifact(art_dir)
    c = loaded.build_cache()
    rng = np.random.default_rng(45)
    ks = rng.standard_normal((20, 2, 2, 64)).astype(np.float32)
    vs = rng.standard_normal((20, 2, 2, 64)).astype(np.float32)
    for t in range(20):
        c.append(key=ks[t], value=vs[t])
    qa = rng.standard_normal((2, 2, 64)).astype(np.float32)
    out["artcache_keys"], out["artcache_values"], out["artcache_query"] = ks, vs, qa
    out["artcache_decode"] = c.decode(query=qa)

    np.savez_compressed(HERE / "golden.npz", **out)
    total = sum(v.nbytes for v in out.values())
    print(f"wrote {len(out)} arrays, {total / 1e6:.2f} MB raw -> {HERE / 'golden.npz'}")


if __name__ == "__main__":
    main()
