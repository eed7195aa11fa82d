"""Decode parity at the benchmarked shapes (the sizes bench.py reports).

The smaller tests pin codes and attention on short caches.  These run the
CUDA path at the benchmark configurations themselves, where other kernel
variants and plans are taken, and compare with the float64 oracle over the
very packed words the GPU wrote (the append path is bit-exact against the
reference in the primitive tests, so the words are the reference's):

  * 131072 tokens, d 128, 32/8 heads, 4-bit (the north-star shape): the
    16-warp few-unit plan (8 units over every SM, one CTA per SM);
  * benchmark config 3: 131072 tokens, d 256, 16/2 heads, 4-bit: 74 splits a
    unit, merged by the 1024-thread merge kernel (>= 64 parts);
  * benchmark config 4 geometry: batch 64, 3-bit, ragged 16K-32K lengths;
    every unit is decoded on the GPU and 8 whole sequences are checked;
  * benchmark config 2 decode: 4096 tokens, 8/32 heads, every (d, bits),
    fp16 N(0,1) K/V with 1% of the channels scaled x20;
  * 128 fused steps (tq_decode_append) at the config-3 shape against append
    followed by decode: bit-identical outputs and packed words.

Tolerance (tensor mode: fp16 centroids, query and probabilities, fp32
accumulation): atol 4e-3 / rtol 2e-2 elementwise, as in the short tests, and
in addition max |err| <= 1e-2 * max |ref| per output (at 128K tokens the
attention output itself is small, so the scale-relative bound is the one
that bites).  Queries are drawn twice: N(0,1) (a flat softmax) and N(0,1) x 6
(a peaked one that moves the running max often).  The measured errors are
printed (pytest -s) for the record.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import torque_oracle as O

pytestmark = pytest.mark.gpu

import torque_mlx_b200 as T  # noqa: E402

ATOL, RTOL, SCALE_REL = 4e-3, 2e-2, 1e-2


def _fill(cache, lens, seed, *, outliers: float = 0.0):
    """Append fp16 N(0,1) K/V of ``lens[s]`` tokens to every sequence, on the
    device; ``outliers`` > 0 scales a fixed 1% of the channels by that factor."""
    cfg = cache.config
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    L, H, d = cfg.num_layers, cfg.kv_heads, cfg.head_dim
    scale = None
    if outliers:
        ch = np.random.default_rng(seed).choice(d, size=max(1, d // 100), replace=False)
        scale = torch.ones(d, device=dev, dtype=torch.float16)
        scale[torch.as_tensor(ch, device=dev)] = outliers
    for s, n in enumerate(lens):
        done = 0
        while done < n:
            m = int(min(16384, n - done))
            k = torch.randn((L, H, m, d), generator=gen, device=dev, dtype=torch.float16)
            v = torch.randn((L, H, m, d), generator=gen, device=dev, dtype=torch.float16)
            if scale is not None:
                k, v = k * scale, v * scale
            cache.append_sequence(s, key=k, value=v)
            done += m
    torch.cuda.synchronize()


def _words(cache, seq: int):
    """Host copy of sequence ``seq``'s packed K/V words ``[layers, kv_heads, n, W]``."""
    n = int(cache.lengths[seq])
    k = cache.key_slab[seq, :, :, :n].cpu().numpy().view(np.uint32)
    v = cache.value_slab[seq, :, :, :n].cpu().numpy().view(np.uint32)
    return k, v


def _oracle_seq(cache, seq: int, q_rot: np.ndarray) -> np.ndarray:
    """float64 GQA decode of one sequence; q_rot [layers, Hq, d] already rotated."""
    cfg = cache.config
    kw, vw = _words(cache, seq)
    out = np.zeros(q_rot.shape)
    for layer in range(cfg.num_layers):
        o, _ = O.gqa_decode(q_rot[layer][None], kw[layer][None], vw[layer][None], cache.key_codebook.centroids,
                            cache.value_codebook.centroids, cfg.bit_width)
        out[layer] = o[0]
    return out


def _check(got: np.ndarray, ref: np.ndarray, label: str) -> None:
    err = np.abs(got.astype(np.float64) - ref)
    scale = float(np.abs(ref).max())
    print(f"[parity] {label}: max|err| {err.max():.3e}  max|ref| {scale:.3e}  "
          f"rel-to-scale {err.max() / max(scale, 1e-30):.3e}")
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL, err_msg=label)
    assert err.max() <= SCALE_REL * scale, f"{label}: max|err| {err.max():.3e} > {SCALE_REL} x {scale:.3e}"


def _queries(rng, shape, peak: float):
    return (rng.standard_normal(shape) * peak).astype(np.float32)


def _rotated(cache, q: np.ndarray) -> np.ndarray:
    sl, sr = O.rotation_signs(cache.config.head_dim, cache.config.rotation_seed)
    return O.rotate(q, sl, sr).astype(np.float32)


@pytest.mark.parametrize("peak", [1.0, 6.0])
def test_north_star_shape_128k_d128_4bit(peak):
    """131072 tokens, d 128, 32 query / 8 kv heads, 4-bit: the 16-warp plan
    for a few long units (tq_decode.cu make_plan)."""
    cfg = T.TorqueConfig(bit_width=4, head_dim=128, num_layers=1, kv_heads=8, fused_weights=True)
    cache = T.TorqueKVCache(config=cfg, initial_capacity=131072, decode_mode="tensor")
    _fill(cache, [131072], seed=128)
    rng = np.random.default_rng(11)
    q = _queries(rng, (32, 128), peak)
    got = cache.decode(query=q)
    ref = _oracle_seq(cache, 0, _rotated(cache, q)[None])[0]
    _check(got, ref, f"128K d128 4-bit G4 peak {peak}")


@pytest.mark.parametrize("peak", [1.0, 6.0])
def test_config3_shape_128k_d256_wide_merge(peak):
    """Benchmark config 3 geometry: 131072 tokens, d 256, 16/2 heads, 4-bit;
    74 splits a unit go through the 1024-thread merge."""
    cfg = T.TorqueConfig(bit_width=4, head_dim=256, num_layers=1, kv_heads=2, fused_weights=True)
    cache = T.TorqueKVCache(config=cfg, initial_capacity=131072, decode_mode="tensor")
    _fill(cache, [131072], seed=3)
    rng = np.random.default_rng(12)
    q = _queries(rng, (16, 256), peak)
    got, lse = cache.decode(query=q, return_lse=True)
    qr = _rotated(cache, q)
    kw, vw = _words(cache, 0)
    ref, ref_lse = O.gqa_decode(qr[None], kw[0][None], vw[0][None], cache.key_codebook.centroids,
                                cache.value_codebook.centroids, 4)
    _check(got, ref[0], f"config 3 d256 G8 peak {peak}")
    np.testing.assert_allclose(lse, ref_lse[0], atol=2e-2, rtol=1e-3)


def test_config4_geometry_ragged_batch64():
    """Benchmark config 4 geometry: batch 64, 32/8 heads, d 128, 3-bit, lengths
    U{16384..32768}; all 512 units decoded, 8 whole sequences checked."""
    rng = np.random.default_rng(4)
    lens = rng.integers(16384, 32769, size=64)
    cfg = T.TorqueConfig(bit_width=3, head_dim=128, num_layers=1, kv_heads=8, fused_weights=True)
    cache = T.TorqueKVCache(config=cfg, batch_size=64, initial_capacity=int(lens.max()), decode_mode="tensor")
    _fill(cache, lens, seed=44)
    q = _queries(rng, (64, 1, 32, 128), 2.0)
    got = cache.decode(query=q)
    qr = _rotated(cache, q)
    for s in (0, 9, 17, 26, 35, 44, 53, 63):
        _check(got[s], _oracle_seq(cache, s, qr[s]), f"config 4 seq {s} (len {lens[s]})")


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("b", [2, 3, 4])
def test_config2_decode_with_outlier_channels(d, b):
    """Benchmark config 2: 4096 tokens, 8 kv / 32 query heads, fp16 N(0,1)
    K/V with 1% of the channels x20, one decode per (d, bits)."""
    cfg = T.TorqueConfig(bit_width=b, head_dim=d, num_layers=1, kv_heads=8, fused_weights=True)
    cache = T.TorqueKVCache(config=cfg, initial_capacity=4096, decode_mode="tensor")
    _fill(cache, [4096], seed=d * 10 + b, outliers=20.0)
    rng = np.random.default_rng(d + b)
    q = _queries(rng, (32, d), 1.0)
    got = cache.decode(query=q)
    ref = _oracle_seq(cache, 0, _rotated(cache, q)[None])[0]
    _check(got, ref, f"config 2 d{d} b{b}")


def test_config3_128_fused_steps_bit_identical():
    """128 generation steps at the config-3 shape: append_decode (the token is
    packed inside the decode kernel) against append then decode, on two caches
    built from the same tokens.  Outputs and packed words are bit-identical."""
    cfg = T.TorqueConfig(bit_width=4, head_dim=256, num_layers=1, kv_heads=2, fused_weights=True)
    a = T.TorqueKVCache(config=cfg, initial_capacity=131072 + 256, decode_mode="tensor")
    b = T.TorqueKVCache(config=cfg, initial_capacity=131072 + 256, decode_mode="tensor")
    _fill(a, [131072], seed=33)
    _fill(b, [131072], seed=33)
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    for step in range(128):
        k = torch.randn((1, 2, 256), generator=gen, device=dev, dtype=torch.float16)
        v = torch.randn((1, 2, 256), generator=gen, device=dev, dtype=torch.float16)
        q = torch.randn((1, 16, 256), generator=gen, device=dev, dtype=torch.float32)
        fused = a.append_decode(key=k, value=v, query=q)
        b.append(key=k, value=v)
        plain = b.decode(query=q)
        assert torch.equal(fused, plain), f"step {step}"
    assert a.sequence_length == b.sequence_length == 131072 + 128
    assert torch.equal(a.key_slab, b.key_slab) and torch.equal(a.value_slab, b.value_slab)
    # and the last step against the oracle
    qn = q.cpu().numpy()
    ref = _oracle_seq(a, 0, _rotated(a, qn))
    got = fused.cpu().numpy()
    _check(got, ref.reshape(got.shape), "config 3 after 128 fused steps")
