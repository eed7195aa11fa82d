"""CPU oracle for the packed-KV decode path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference (cbun/torque-mlx) algorithms that
the CUDA path must reproduce.  It is the checker, never the thing measured or
shipped: only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline``
/ ``--impl reference`` legs of ``bench.py`` may import it.  The product package
(``torque_mlx_b200``) never imports it and has no CPU fallback.

Pinning: every function here is checked against golden vectors produced by the
reference's own numpy code (``tests/golden/make_golden.py`` imports the
reference with an empty ``mlx`` stub; the vectors live in ``tests/golden/``).

Citations are ``path:line`` inside the reference project.
"""

from __future__ import annotations

from math import ceil, sqrt

import numpy as np

WORD_BITS = 32
SUPPORTED_BITS = (2, 3, 4)
SUPPORTED_HEAD_DIMS = (64, 128, 256)


# --------------------------------------------------------------------------
# rotation  (src/torque_mlx/rotation.py)
# --------------------------------------------------------------------------
def rotation_signs(head_dim: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """(signs_left, signs_right) as drawn by ``RotationSpec.from_seed``
    (rotation.py:75-86): two ``choice([-1, 1])`` draws from ``default_rng(seed)``,
    left first."""
    rng = np.random.default_rng(seed)
    pm = np.array([-1.0, 1.0], dtype=np.float32)
    left = rng.choice(pm, size=head_dim)
    right = rng.choice(pm, size=head_dim)
    return left.astype(np.float32), right.astype(np.float32)


def fwht(x: np.ndarray) -> np.ndarray:
    """Unnormalised Walsh-Hadamard transform on the last axis, fp32, with the
    butterfly stages in the order of rotation.py:19-32 (span 1, 2, 4, ...).
    Each stage maps (a, b) -> (a + b, a - b) for partners ``i`` and ``i + span``."""
    out = np.array(x, dtype=np.float32, copy=True)
    d = out.shape[-1]
    lead = out.shape[:-1]
    span = 1
    while span < d:
        v = out.reshape(*lead, d // (2 * span), 2, span)
        a = v[..., 0, :].copy()
        b = v[..., 1, :].copy()
        v[..., 0, :] = a + b
        v[..., 1, :] = a - b
        out = v.reshape(*lead, d)
        span *= 2
    return out


def rotate(x: np.ndarray, signs_left: np.ndarray, signs_right: np.ndarray) -> np.ndarray:
    """Pi x = D1 H D2 x / sqrt(d)  (rotation.py:88-94).  The division is fp32 by
    ``float32(sqrt(d))`` (numpy's weak-scalar rule), IEEE round-to-nearest."""
    a = np.asarray(x, dtype=np.float32)
    d = a.shape[-1]
    h = fwht(a * signs_right)
    h = h / np.float32(sqrt(d))
    return h * signs_left


def rotate_inverse(x: np.ndarray, signs_left: np.ndarray, signs_right: np.ndarray) -> np.ndarray:
    """Pi^T x  (rotation.py:96-102): the sign vectors swap roles."""
    return rotate(x, signs_right, signs_left)


# --------------------------------------------------------------------------
# codebook + quantizer + packing  (src/torque_mlx/quantization.py)
# --------------------------------------------------------------------------
def packed_words(head_dim: int, bits: int) -> int:
    """quantization.py:76-81."""
    return ceil(head_dim * bits / WORD_BITS)


def gaussian_codebook(bits: int, *, iterations: int = 32, sample_size: int = 200_000,
                      seed: int = 0) -> np.ndarray:
    """Lloyd-Max centroids for N(0,1) as in quantization.py:89-117: quantile
    initialisation, midpoint assignment with ``searchsorted(side='right')``,
    float64 cluster means, early stop on ``allclose``."""
    rng = np.random.default_rng(seed)
    samples = rng.normal(loc=0.0, scale=1.0, size=sample_size).astype(np.float32)
    levels = 1 << bits
    q = np.linspace(0.0, 1.0, levels + 2, dtype=np.float32)[1:-1]
    cent = np.quantile(samples, q).astype(np.float32)
    for _ in range(iterations):
        mids = (cent[:-1] + cent[1:]) / 2.0
        assign = np.searchsorted(mids, samples, side="right")
        new = cent.copy()
        for k in range(levels):
            members = samples[assign == k]
            if members.size:
                new[k] = members.mean(dtype=np.float64)
        done = np.allclose(new, cent)
        cent = new
        if done:
            break
    return np.sort(cent).astype(np.float32)


def quantize(x: np.ndarray, centroids: np.ndarray) -> np.ndarray:
    """argmin_k |x - c_k| in fp32, first index on ties (quantization.py:120-125).
    Processed in blocks so large inputs do not build a giant distance matrix."""
    a = np.asarray(x, dtype=np.float32)
    c = np.asarray(centroids, dtype=np.float32)
    flat = a.reshape(-1)
    out = np.empty(flat.shape, dtype=np.uint8)
    blk = 1 << 20
    for s in range(0, flat.size, blk):
        v = flat[s:s + blk, None]
        out[s:s + blk] = np.argmin(np.abs(v - c[None, :]), axis=1).astype(np.uint8)
    return out.reshape(a.shape)


def boundaries(centroids: np.ndarray) -> np.ndarray:
    """Midpoints of neighbouring centroids in fp32 (codebook_boundaries,
    quantization.py:128-136)."""
    c = np.asarray(centroids, dtype=np.float32)
    return ((c[:-1] + c[1:]) / np.float32(2.0)).astype(np.float32)


def quantize_boundaries(x: np.ndarray, bounds: np.ndarray) -> np.ndarray:
    """The MLX path's quantizer: the number of boundaries each value exceeds
    (quantize_mlx, quantization.py:139-148; the append-pack kernels of
    mlx_ops.py:257-339 use the same count).  A value equal to a boundary
    takes the lower code."""
    a = np.asarray(x, dtype=np.float32)
    b = np.asarray(bounds, dtype=np.float32)
    return (a[..., None] > b).sum(axis=-1).astype(np.uint8)


def pack(codes: np.ndarray, bits: int) -> np.ndarray:
    """LSB-first bitstream per vector (quantization.py:156-201): code i sits at
    bit ``i*bits``; a code that crosses a word edge spills its high bits into the
    low bits of the next word."""
    c = np.asarray(codes, dtype=np.uint64)
    n = c.shape[-1]
    flat = c.reshape(-1, n)
    w = packed_words(n, bits)
    # accumulate into 64-bit lanes per word pair
    out = np.zeros((flat.shape[0], w + 1), dtype=np.uint64)
    for i in range(n):
        off = i * bits
        wi, sh = divmod(off, WORD_BITS)
        v = flat[:, i] << np.uint64(sh)
        out[:, wi] |= v & np.uint64(0xFFFFFFFF)
        out[:, wi + 1] |= v >> np.uint64(32)
    return out[:, :w].astype(np.uint32).reshape(*c.shape[:-1], w)


def unpack(words: np.ndarray, bits: int, count: int) -> np.ndarray:
    """Inverse of :func:`pack` (quantization.py:272-290)."""
    wds = np.asarray(words, dtype=np.uint64)
    w = wds.shape[-1]
    flat = wds.reshape(-1, w)
    padded = np.concatenate([flat, np.zeros((flat.shape[0], 1), np.uint64)], axis=1)
    mask = np.uint64((1 << bits) - 1)
    out = np.empty((flat.shape[0], count), dtype=np.uint8)
    for i in range(count):
        wi, sh = divmod(i * bits, WORD_BITS)
        pair = padded[:, wi] | (padded[:, wi + 1] << np.uint64(32))
        out[:, i] = ((pair >> np.uint64(sh)) & mask).astype(np.uint8)
    return out.reshape(*wds.shape[:-1], count)


def dequantize(codes: np.ndarray, centroids: np.ndarray) -> np.ndarray:
    """quantization.py:151-153."""
    return np.asarray(centroids, dtype=np.float32)[np.asarray(codes)].astype(np.float32)


def rotate_quantize_pack(x: np.ndarray, signs_left, signs_right, centroids, bits: int,
                         *, rotate_input: bool = True) -> np.ndarray:
    """The append path: pack(quantize(rotate(x))) — what
    tests/test_cache_mlx.py:54-70 asserts for the device slab."""
    r = rotate(x, signs_left, signs_right) if rotate_input else np.asarray(x, np.float32)
    return pack(quantize(r, centroids), bits)


# --------------------------------------------------------------------------
# attention  (src/torque_mlx/reference.py, cache.py)
# --------------------------------------------------------------------------
def streaming_attention_decode(query: np.ndarray, keys: np.ndarray, values: np.ndarray) -> np.ndarray:
    """q_len=1 online-softmax decode, token by token, as reference.py:8-42:
    score = fp32 dot * (1/sqrt(d)), running max/denominator in float64,
    output accumulated in fp32.  Pure-Python loop: small cases only."""
    q = np.asarray(query, dtype=np.float32)
    K = np.asarray(keys, dtype=np.float32)
    V = np.asarray(values, dtype=np.float32)
    scale = 1.0 / sqrt(q.shape[0])
    m = -np.inf
    l = 0.0
    out = np.zeros_like(q)
    for k, v in zip(K, V):
        s = float(np.dot(q, k) * scale)
        m_new = max(m, s)
        alpha = 0.0 if np.isneginf(m) else float(np.exp(m - m_new))
        p = float(np.exp(s - m_new))
        out *= alpha
        out += p * v
        l = l * alpha + p
        m = m_new
    if l == 0.0:
        return out
    return out / l


def attention_f64(query: np.ndarray, keys: np.ndarray, values: np.ndarray,
                  scale: float | None = None) -> tuple[np.ndarray, np.ndarray]:
    """Vectorised float64 softmax attention over already-dequantised K/V.

    query [..., G, d], keys/values [..., L, d] -> (out [..., G, d], lse [..., G]).
    Same math as :func:`streaming_attention_decode` without its fp32 rounding;
    used for long contexts where the Python loop is too slow.  An empty
    sequence yields zeros and lse = -inf (reference.py:40-41)."""
    q = np.asarray(query, dtype=np.float64)
    K = np.asarray(keys, dtype=np.float64)
    V = np.asarray(values, dtype=np.float64)
    d = q.shape[-1]
    sc = (1.0 / sqrt(d)) if scale is None else scale
    if K.shape[-2] == 0:
        return np.zeros(q.shape), np.full(q.shape[:-1], -np.inf)
    s = np.einsum("...gd,...ld->...gl", q, K) * sc
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=-1, keepdims=True)
    out = np.einsum("...gl,...ld->...gd", p, V) / l
    lse = (m + np.log(l))[..., 0]
    return out, lse


def gqa_decode(query_rot: np.ndarray, k_words: np.ndarray, v_words: np.ndarray,
               cent_k: np.ndarray, cent_v: np.ndarray, bits: int,
               lengths: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
    """Grouped-query packed decode restated from tests/test_cache_mlx.py:88-98
    and cache_mlx.py:706-722 (kv head = q head // G).

    query_rot [B, Hq, d] (already rotated); k/v words [B, Hkv, L, W];
    lengths [B] (ragged; default full L).  Returns (out_rot [B, Hq, d], lse [B, Hq])."""
    B, Hq, d = query_rot.shape
    _, Hkv, L, _ = k_words.shape
    G = Hq // Hkv
    out = np.zeros((B, Hq, d))
    lse = np.zeros((B, Hq))
    for b in range(B):
        n = L if lengths is None else int(lengths[b])
        for h in range(Hkv):
            K = dequantize(unpack(k_words[b, h, :n], bits, d), cent_k)
            V = dequantize(unpack(v_words[b, h, :n], bits, d), cent_v)
            o, s = attention_f64(query_rot[b, h * G:(h + 1) * G], K, V)
            out[b, h * G:(h + 1) * G] = o
            lse[b, h * G:(h + 1) * G] = s
    return out, lse


def lse_merge(outs: np.ndarray, lses: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Combine normalised partial attentions over disjoint key sets:
    out = sum_r exp(lse_r - LSE) out_r, LSE = logsumexp_r lse_r.
    outs [P, ..., d], lses [P, ...].  Parts with lse = -inf contribute nothing."""
    o = np.asarray(outs, dtype=np.float64)
    s = np.asarray(lses, dtype=np.float64)
    M = s.max(axis=0)
    Ms = np.where(np.isneginf(M), 0.0, M)
    w = np.exp(s - Ms)
    tot = w.sum(axis=0)
    merged = (w[..., None] * o).sum(axis=0) / np.where(tot == 0, 1.0, tot)[..., None]
    return merged, np.where(tot == 0, -np.inf, Ms + np.log(np.where(tot == 0, 1.0, tot)))


class OracleCache:
    """Restatement of the numpy ``TorqueKVCache`` (cache.py:36-227): per-step
    append of ``[layers, kv_heads, d]`` K/V, decode of one query per KV head
    (G = 1), inverse rotation unless ``fused_weights``."""

    def __init__(self, *, bits: int, head_dim: int, num_layers: int = 1, kv_heads: int = 1,
                 rotation_seed: int = 0, fused_weights: bool = False,
                 cent_k: np.ndarray | None = None, cent_v: np.ndarray | None = None):
        self.bits, self.d, self.L, self.H = bits, head_dim, num_layers, kv_heads
        self.fused = fused_weights
        self.cent_k = gaussian_codebook(bits, seed=rotation_seed) if cent_k is None else np.asarray(cent_k, np.float32)
        self.cent_v = gaussian_codebook(bits, seed=rotation_seed + 1) if cent_v is None else np.asarray(cent_v, np.float32)
        self.sl, self.sr = rotation_signs(head_dim, rotation_seed)
        self.k_words: list[np.ndarray] = []
        self.v_words: list[np.ndarray] = []

    @property
    def sequence_length(self) -> int:
        return len(self.k_words)

    def append(self, key: np.ndarray, value: np.ndarray) -> None:
        k = np.asarray(key, np.float32).reshape(self.L, self.H, self.d)
        v = np.asarray(value, np.float32).reshape(self.L, self.H, self.d)
        self.k_words.append(rotate_quantize_pack(k, self.sl, self.sr, self.cent_k, self.bits))
        self.v_words.append(rotate_quantize_pack(v, self.sl, self.sr, self.cent_v, self.bits))

    def words(self) -> tuple[np.ndarray, np.ndarray]:
        """[layers, kv_heads, seq, W] slabs (the layout of layout.py:34-35)."""
        W = packed_words(self.d, self.bits)
        if not self.k_words:
            z = np.zeros((self.L, self.H, 0, W), np.uint32)
            return z, z.copy()
        return np.stack(self.k_words, axis=2), np.stack(self.v_words, axis=2)

    def decode(self, query: np.ndarray, *, streaming: bool = True) -> np.ndarray:
        q = np.asarray(query, np.float32).reshape(self.L, self.H, self.d)
        out = np.zeros_like(q)
        kw, vw = self.words()
        if kw.shape[2] == 0:
            return out
        for l in range(self.L):
            for h in range(self.H):
                qr = rotate(q[l, h], self.sl, self.sr)
                K = dequantize(unpack(kw[l, h], self.bits, self.d), self.cent_k)
                V = dequantize(unpack(vw[l, h], self.bits, self.d), self.cent_v)
                if streaming:
                    o = streaming_attention_decode(qr, K, V)
                else:
                    o = attention_f64(qr[None], K, V)[0][0].astype(np.float32)
                out[l, h] = o if self.fused else rotate_inverse(o, self.sl, self.sr)
        return out
