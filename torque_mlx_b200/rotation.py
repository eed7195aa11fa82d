"""Structured rotation Pi = D1 H D2 / sqrt(d) (reference: src/torque_mlx/rotation.py).

``RotationSpec.from_seed`` draws the two sign vectors with numpy's
``default_rng(seed)`` exactly as the reference does (rotation.py:75-86), so a
seed gives the same rotation in both projects.  ``apply`` / ``inverse`` run
the warp-shuffle Walsh-Hadamard kernel ``tq_rotate``, which reproduces the
reference's fp32 butterflies and division bit for bit.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib, _tensors
from .config import RotationMode, validate_head_dim

__all__ = ["RotationMode", "RotationSpec", "apply_structured_rotation", "validate_head_dim"]


@dataclass(frozen=True, slots=True)
class RotationSpec:
    """Structured orthogonal rotation Pi = D1 H D2 (rotation.py:51-106)."""

    head_dim: int
    signs_left: np.ndarray
    signs_right: np.ndarray
    seed: int | None = None
    _dev: dict = field(default_factory=dict, init=False, repr=False, compare=False)

    def __post_init__(self) -> None:
        validate_head_dim(self.head_dim)
        object.__setattr__(self, "signs_left", np.asarray(self.signs_left, dtype=np.float32))
        object.__setattr__(self, "signs_right", np.asarray(self.signs_right, dtype=np.float32))
        if self.signs_left.shape != (self.head_dim,) or self.signs_right.shape != (self.head_dim,):
            raise ValueError("Rotation sign vectors must match head_dim")

    @classmethod
    def from_seed(cls, head_dim: int, seed: int = 0) -> "RotationSpec":
        validate_head_dim(head_dim)
        rng = np.random.default_rng(seed)
        pm = np.array([-1.0, 1.0], dtype=np.float32)
        left = rng.choice(pm, size=head_dim)
        right = rng.choice(pm, size=head_dim)
        return cls(head_dim=head_dim, signs_left=left, signs_right=right, seed=seed)

    def device_signs(self) -> tuple[torch.Tensor, torch.Tensor]:
        """(signs_left, signs_right) on the current CUDA device (cached)."""
        dev = _tensors.device()
        key = str(dev)
        if key not in self._dev:
            self._dev[key] = (_tensors.to_cuda(self.signs_left, torch.float32),
                              _tensors.to_cuda(self.signs_right, torch.float32))
        return self._dev[key]

    def _run(self, values, inverse: bool):
        lib = _lib.load()
        np_out = _tensors.is_numpy(values)
        x = _tensors.to_cuda(values, torch.float32, keep_half=True)
        if x.shape[-1] != self.head_dim:
            raise ValueError(f"Expected last dimension {self.head_dim}, got {x.shape[-1]}")
        y = torch.empty(x.shape, dtype=torch.float32, device=x.device)
        sl, sr = self.device_signs()
        first, second = (sl, sr) if inverse else (sr, sl)
        _lib.check(lib.tq_rotate(x.data_ptr(), _lib.dtype_code(x.dtype), y.data_ptr(), x.numel() // self.head_dim,
                                 self.head_dim, first.data_ptr(), second.data_ptr(), _lib.stream_ptr()),
                   "rotate")
        return _tensors.out(y, np_out)

    def apply(self, values):
        """Pi x (rotation.py:88-94)."""
        return self._run(values, inverse=False)

    def inverse(self, values):
        """Pi^T x (rotation.py:96-102)."""
        return self._run(values, inverse=True)

    def matrix(self) -> np.ndarray:
        """Dense Pi (rotation.py:104-106)."""
        return self.apply(np.eye(self.head_dim, dtype=np.float32)).T


def apply_structured_rotation(values, head_dim: int, seed: int = 0):
    """rotation.py:109-110."""
    return RotationSpec.from_seed(head_dim=head_dim, seed=seed).apply(values)
