"""Codebooks, the nearest-centroid quantizer and LSB-first bit packing.

Reference: src/torque_mlx/quantization.py.  ``Codebook``,
``build_gaussian_codebook`` and the size helpers are set-up code (they run
once, on the host, with the reference's exact numpy arithmetic so codebooks
are bit-identical).  ``quantize``, ``dequantize``, ``pack_indices``,
``pack_indices_batched`` and ``unpack_indices`` run in the CUDA library.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from math import ceil
from pathlib import Path

import numpy as np
import torch

from . import _lib, _tensors

SUPPORTED_BIT_WIDTHS = {2, 3, 4}
WORD_BITS = 32


def _validate_bit_width(bit_width: int) -> None:
    if bit_width not in SUPPORTED_BIT_WIDTHS:
        raise ValueError(f"Unsupported bit width: {bit_width}")


@dataclass(frozen=True, slots=True)
class Codebook:
    """Sorted fp32 scalar codebook of 2^bits centroids (quantization.py:21-65)."""

    bit_width: int
    centroids: np.ndarray
    name: str = "gaussian_lloyd_max"

    def __post_init__(self) -> None:
        _validate_bit_width(self.bit_width)
        object.__setattr__(self, "centroids", np.asarray(self.centroids, dtype=np.float32))
        expected = 1 << self.bit_width
        if self.centroids.ndim != 1 or self.centroids.size != expected:
            raise ValueError(
                f"Expected {expected} centroids for {self.bit_width}-bit codebook, got shape {self.centroids.shape}")
        if not np.all(np.diff(self.centroids) >= 0):
            raise ValueError("Centroids must be sorted in ascending order")

    def to_dict(self) -> dict[str, object]:
        return {"bit_width": self.bit_width, "centroids": self.centroids.tolist(), "name": self.name}

    def to_json(self) -> str:
        return json.dumps(self.to_dict(), indent=2, sort_keys=True)

    @classmethod
    def from_dict(cls, payload: dict[str, object]) -> "Codebook":
        return cls(bit_width=int(payload["bit_width"]),
                   centroids=np.asarray(payload["centroids"], dtype=np.float32),
                   name=str(payload.get("name", "gaussian_lloyd_max")))

    @classmethod
    def from_json(cls, payload: str) -> "Codebook":
        return cls.from_dict(json.loads(payload))

    def device_centroids(self) -> torch.Tensor:
        return _tensors.to_cuda(self.centroids, torch.float32)


def save_codebook(codebook: Codebook, path: str | Path) -> None:
    Path(path).write_text(codebook.to_json(), encoding="utf-8")


def load_codebook(path: str | Path) -> Codebook:
    return Codebook.from_json(Path(path).read_text(encoding="utf-8"))


def packed_words_for_head_dim(head_dim: int, bit_width: int) -> int:
    """Words of one packed vector: ceil(d * bits / 32) (quantization.py:76-81)."""
    _validate_bit_width(bit_width)
    if head_dim <= 0:
        raise ValueError("head_dim must be positive")
    return ceil((head_dim * bit_width) / WORD_BITS)


def kv_bytes_per_token(head_dim: int, bit_width: int, kv_heads: int = 1) -> int:
    """quantization.py:84-86."""
    return packed_words_for_head_dim(head_dim=head_dim, bit_width=bit_width) * 4 * kv_heads * 2


def build_gaussian_codebook(bit_width: int, *, iterations: int = 32, sample_size: int = 200_000,
                            seed: int = 0) -> Codebook:
    """Lloyd-Max codebook for N(0, 1) (quantization.py:89-117).

    Set-up code, run once on the host: the sample draw, quantile start,
    midpoint assignment and float64 cluster means follow the reference step
    for step so the centroids are bit-identical to the reference's."""
    _validate_bit_width(bit_width)
    rng = np.random.default_rng(seed)
    samples = rng.normal(loc=0.0, scale=1.0, size=sample_size).astype(np.float32)
    levels = 1 << bit_width
    quantiles = np.linspace(0.0, 1.0, levels + 2, dtype=np.float32)[1:-1]
    centroids = np.quantile(samples, quantiles).astype(np.float32)
    for _ in range(iterations):
        edges = (centroids[:-1] + centroids[1:]) / 2.0
        member = np.searchsorted(edges, samples, side="right")
        updated = centroids.copy()
        for k in range(levels):
            sel = samples[member == k]
            if sel.size:
                updated[k] = sel.mean(dtype=np.float64)
        converged = np.allclose(updated, centroids)
        centroids = updated
        if converged:
            break
    return Codebook(bit_width=bit_width, centroids=np.sort(centroids))


def codebook_boundaries(codebook) -> np.ndarray:
    """Midpoints between neighbouring centroids (quantization.py:128-136)."""
    c = (np.asarray(codebook.centroids, dtype=np.float32) if isinstance(codebook, Codebook)
         else np.asarray(codebook, dtype=np.float32))
    if c.ndim != 1 or c.size < 2:
        raise ValueError("Expected at least two sorted centroids to build quantization boundaries")
    return ((c[:-1] + c[1:]) / 2.0).astype(np.float32)


def _centroids(codebook) -> tuple[np.ndarray, int]:
    if isinstance(codebook, Codebook):
        return codebook.centroids, codebook.bit_width
    c = np.asarray(codebook.centroids if hasattr(codebook, "centroids") else codebook, dtype=np.float32)
    bits = int(np.log2(c.size))
    _validate_bit_width(bits)
    return c, bits


def quantize(values, codebook) -> np.ndarray | torch.Tensor:
    """Nearest-centroid index, ties to the lower index, as uint8
    (quantization.py:120-125).  Runs ``tq_quantize`` on the GPU."""
    lib = _lib.load()
    cent, bits = _centroids(codebook)
    np_out = _tensors.is_numpy(values)
    x = _tensors.to_cuda(values, torch.float32)
    codes = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    c = _tensors.to_cuda(cent, torch.float32)
    _lib.check(lib.tq_quantize(x.data_ptr(), codes.data_ptr(), x.numel(), c.data_ptr(), bits,
                               _lib.stream_ptr()), "quantize")
    return _tensors.out(codes, np_out)


def dequantize(indices, codebook) -> np.ndarray | torch.Tensor:
    """centroids[indices] (quantization.py:151-153) — a gather; for numpy
    inputs this is the reference's own host gather."""
    cent, _ = _centroids(codebook)
    if _tensors.is_numpy(indices):
        return cent[np.asarray(indices)].astype(np.float32)
    c = _tensors.to_cuda(cent, torch.float32)
    return c[indices.to(c.device).long()]


def pack_indices_batched(indices, bit_width: int):
    """Pack the last axis LSB-first into uint32 words (quantization.py:156-201)."""
    lib = _lib.load()
    _validate_bit_width(bit_width)
    np_out = _tensors.is_numpy(indices)
    t = _tensors.to_cuda(indices)
    if t.dtype != torch.uint8:
        if bool((t < 0).any()) or bool((t >= (1 << bit_width)).any()):
            raise ValueError(f"Index out of range for {bit_width}-bit packing")
        t = t.to(torch.uint8)
    elif bool((t >= (1 << bit_width)).any()):
        raise ValueError(f"Index out of range for {bit_width}-bit packing")
    if t.dim() == 0:
        t = t.reshape(1)
    count = t.shape[-1]
    rows = t.numel() // max(count, 1)
    W = packed_words_for_head_dim(count, bit_width) if count else 0
    words = torch.empty((*t.shape[:-1], W), dtype=torch.int32, device=t.device)
    _lib.check(lib.tq_pack(t.data_ptr(), words.data_ptr(), rows, count, bit_width, _lib.stream_ptr()), "pack")
    return _tensors.words_out(words, np_out)


def pack_indices(indices, bit_width: int):
    """Pack a flat index vector (quantization.py:156-173)."""
    if _tensors.is_numpy(indices):
        return pack_indices_batched(np.asarray(indices).reshape(-1), bit_width)
    return pack_indices_batched(indices.reshape(-1), bit_width)


def unpack_indices(words, bit_width: int, count: int):
    """Inverse of packing for one vector, or for every row of a batch
    (quantization.py:272-290)."""
    lib = _lib.load()
    _validate_bit_width(bit_width)
    if count < 0:
        raise ValueError("count must be non-negative")
    np_out = _tensors.is_numpy(words)
    w = _tensors.words_to_cuda(words)
    if w.dim() <= 1:
        w = w.reshape(1, -1)
        lead: tuple[int, ...] = ()
    else:
        lead = tuple(w.shape[:-1])
    if w.shape[-1] < packed_words_for_head_dim(max(count, 1), bit_width) and count:
        raise ValueError("not enough words for count")
    rows = w.numel() // w.shape[-1]
    codes = torch.empty((*lead, count), dtype=torch.uint8, device=w.device)
    if w.shape[-1] != packed_words_for_head_dim(max(count, 1), bit_width):
        w = w[..., : packed_words_for_head_dim(max(count, 1), bit_width)].contiguous()
    _lib.check(lib.tq_unpack(w.data_ptr(), codes.data_ptr(), rows, count, bit_width, _lib.stream_ptr()), "unpack")
    return _tensors.out(codes, np_out)
