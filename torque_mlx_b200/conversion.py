"""Offline weight fusion (reference: src/torque_mlx/conversion.py:19-51).

Folds the shared rotation into the attention projections so the model
produces rotated q/k/v and consumes rotated attention outputs:

    W_Q' = Pi W_Q,  W_K' = Pi W_K,  W_V' = Pi W_V,  W_O' = W_O Pi^T

with Q/K/V weights ``[head_dim, input_dim]`` and O ``[output_dim, head_dim]``
(matrix-vector convention).  Pi W for a column block is Pi applied to each
column, and W Pi^T is Pi applied to each row, so both run as the exact
rotation kernel (``tq_rotate``) instead of a dense matmul with Pi.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .rotation import RotationSpec


@dataclass(frozen=True, slots=True)
class FusedAttentionWeights:
    w_q: np.ndarray
    w_k: np.ndarray
    w_v: np.ndarray
    w_o: np.ndarray
    rotation_seed: int


def _rotate_columns(rotation: RotationSpec, w):
    t = torch.as_tensor(np.asarray(w, dtype=np.float32) if not isinstance(w, torch.Tensor) else w)
    out = rotation.apply(t.to(torch.float32).T.contiguous().cuda())
    return out.T.contiguous()


def fuse_attention_weights(*, w_q, w_k, w_v, w_o, rotation: RotationSpec) -> FusedAttentionWeights:
    """Fuse Pi into Q/K/V and Pi^T into O (conversion.py:19-51).  Accepts numpy
    arrays or torch tensors; returns numpy fp32 arrays like the reference."""
    d = rotation.head_dim
    shapes = [tuple(np.shape(w)) for w in (w_q, w_k, w_v)]
    if any(s[0] != d for s in shapes):
        raise ValueError("Q/K/V output dimension must equal rotation head_dim")
    if tuple(np.shape(w_o))[1] != d:
        raise ValueError("O input dimension must equal rotation head_dim")
    q = _rotate_columns(rotation, w_q)
    k = _rotate_columns(rotation, w_k)
    v = _rotate_columns(rotation, w_v)
    o_in = w_o if isinstance(w_o, torch.Tensor) else torch.as_tensor(np.asarray(w_o, dtype=np.float32))
    o = rotation.apply(o_in.to(torch.float32).contiguous().cuda())  # rows of W_O times Pi^T
    return FusedAttentionWeights(w_q=q.cpu().numpy(), w_k=k.cpu().numpy(), w_v=v.cpu().numpy(),
                                 w_o=o.cpu().numpy(), rotation_seed=-1 if rotation.seed is None else rotation.seed)
