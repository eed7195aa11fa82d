"""Packed-code operators on explicit device tensors.

These mirror the reference's kernel wrappers in src/torque_mlx/mlx_ops.py
(same names, argument meaning and errors) but run the sm_100a kernels of
``libtorque_b200.so`` instead of Metal.  Code tensors hold uint32 words in the
reference's LSB-first layout; torch tensors may be ``torch.uint32`` or
``torch.int32`` storage.  Queries given to the ``decode_packed_*`` functions
are already rotated, as in the reference.
"""

from __future__ import annotations

from math import sqrt

import numpy as np
import torch

from . import _lib, _tensors
from .quantization import Codebook, packed_words_for_head_dim

_MODES = {"auto": _lib.DECODE_AUTO, "exact": _lib.DECODE_EXACT, "tensor": _lib.DECODE_TENSOR}


def cuda_available() -> bool:
    """Counterpart of ``metal_available`` (mlx_ops.py:34-45)."""
    try:
        _lib.load()
        return True
    except RuntimeError:
        return False


def decode_mode_code(mode: str | int) -> int:
    if isinstance(mode, int):
        return mode
    try:
        return _MODES[mode]
    except KeyError as exc:
        raise ValueError(f"decode mode must be one of {sorted(_MODES)}") from exc


class Workspace:
    """Grow-only device scratch buffer for the split-K partials."""

    def __init__(self) -> None:
        self.buf: torch.Tensor | None = None

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        return self.buf


_default_ws = Workspace()


def workspace_bytes(units: int, group_size: int, head_dim: int, bits: int, max_len: int,
                    mode: str | int = "auto") -> int:
    lib = _lib.load(require_cuda=False)
    out = _lib.c_size_t(0)
    _lib.check(lib.tq_decode_workspace_size(units, group_size, head_dim, bits, max_len, decode_mode_code(mode),
                                            _lib.ctypes.byref(out)), "decode workspace")
    return int(out.value)


def decode_raw(*, query: torch.Tensor, k_slab: torch.Tensor, v_slab: torch.Tensor, unit_stride: int,
               lengths: torch.Tensor | None, units_per_seq: int, len_offset: int, max_len: int, units: int,
               group_size: int, head_dim: int, bits: int, cent_k: torch.Tensor, cent_v: torch.Tensor,
               out: torch.Tensor, lse: torch.Tensor | None = None, rotate_query: bool = False,
               inverse_rotate: bool = False, signs: tuple[torch.Tensor, torch.Tensor] | None = None,
               scale: float | None = None, mode: str | int = "auto", workspace: Workspace | None = None) -> None:
    """One ``tq_decode`` call on prepared device tensors (see include/torque_b200.h)."""
    lib = _lib.load()
    wsp = workspace or _default_ws
    sl, sr = signs if signs is not None else (None, None)
    args = [query.data_ptr(), int(rotate_query), _lib.ptr(sl), _lib.ptr(sr), k_slab.data_ptr(), v_slab.data_ptr(),
            unit_stride, _lib.ptr(lengths), units_per_seq, len_offset, max_len, units, group_size, head_dim, bits,
            cent_k.data_ptr(), cent_v.data_ptr(), float(1.0 / sqrt(head_dim) if scale is None else scale),
            out.data_ptr(), _lib.ptr(lse), int(inverse_rotate), decode_mode_code(mode), None, 0, _lib.stream_ptr()]
    ws = wsp.buf
    if ws is not None and ws.device == out.device:
        # the usual case: the current buffer is big enough and tq_decode
        # launches straight away; a too-small one is refused before any launch
        args[22], args[23] = ws.data_ptr(), ws.numel()
        status = lib.tq_decode(*args)
        if status != _lib.TQ_E_WORKSPACE:
            _lib.check(status, "decode")
            return
    ws = wsp.get(workspace_bytes(units, group_size, head_dim, bits, max_len, mode), out.device)
    args[22], args[23] = ws.data_ptr(), ws.numel()
    _lib.check(lib.tq_decode(*args), "decode")


def decode_causal_raw(*, query: torch.Tensor, k_slab: torch.Tensor, v_slab: torch.Tensor, unit_stride: int,
                      lengths: torch.Tensor, units_per_seq: int, len_offset: int, max_len: int, units: int,
                      q_tokens: int, group_size: int, head_dim: int, bits: int, cent_k: torch.Tensor,
                      cent_v: torch.Tensor, out: torch.Tensor, lse: torch.Tensor | None = None,
                      rotate_query: bool = False, inverse_rotate: bool = False,
                      signs: tuple[torch.Tensor, torch.Tensor] | None = None, scale: float | None = None,
                      workspace: Workspace | None = None) -> None:
    """One ``tq_decode_causal`` call: the last ``q_tokens`` tokens of every
    unit attend causally (query ``[units, q_tokens, group_size, d]``)."""
    lib = _lib.load()
    wsp = workspace or _default_ws
    sl, sr = signs if signs is not None else (None, None)
    ws = wsp.get(workspace_bytes(units, q_tokens * group_size, head_dim, bits, max_len, "tensor"), out.device)
    _lib.check(lib.tq_decode_causal(
        query.data_ptr(), int(rotate_query), _lib.ptr(sl), _lib.ptr(sr), k_slab.data_ptr(), v_slab.data_ptr(),
        unit_stride, lengths.data_ptr(), units_per_seq, len_offset, max_len, units, q_tokens, group_size, head_dim,
        bits, cent_k.data_ptr(), cent_v.data_ptr(), float(1.0 / sqrt(head_dim) if scale is None else scale),
        out.data_ptr(), _lib.ptr(lse), int(inverse_rotate), ws.data_ptr(), ws.numel(), _lib.stream_ptr()),
        "decode_causal")


def decode_append_raw(*, new_k: torch.Tensor, new_v: torch.Tensor, rotate_k: bool, rotate_v: bool, advance: bool,
                      query: torch.Tensor, k_slab: torch.Tensor, v_slab: torch.Tensor, unit_stride: int,
                      lengths: torch.Tensor, units_per_seq: int, max_len: int, units: int, group_size: int,
                      head_dim: int, bits: int, cent_k: torch.Tensor, cent_v: torch.Tensor, out: torch.Tensor,
                      lse: torch.Tensor | None = None, rotate_query: bool = False, inverse_rotate: bool = False,
                      signs: tuple[torch.Tensor, torch.Tensor] | None = None, scale: float | None = None,
                      mode: str | int = "auto", workspace: Workspace | None = None) -> None:
    """One ``tq_decode_append`` call: pack row u of ``new_k`` / ``new_v``
    ([units, head_dim]) at its sequence's length, attend up to and including
    it, and (``advance``) count it (see include/torque_b200.h)."""
    lib = _lib.load()
    wsp = workspace or _default_ws
    sl, sr = signs if signs is not None else (None, None)
    args = [new_k.data_ptr(), new_v.data_ptr(), _lib.dtype_code(new_k.dtype), int(rotate_k), int(rotate_v),
            int(advance), query.data_ptr(), int(rotate_query), _lib.ptr(sl), _lib.ptr(sr), k_slab.data_ptr(),
            v_slab.data_ptr(), unit_stride, lengths.data_ptr(), units_per_seq, max_len, units, group_size, head_dim,
            bits, cent_k.data_ptr(), cent_v.data_ptr(), float(1.0 / sqrt(head_dim) if scale is None else scale),
            out.data_ptr(), _lib.ptr(lse), int(inverse_rotate), decode_mode_code(mode), None, 0, _lib.stream_ptr()]
    ws = wsp.buf
    if ws is not None and ws.device == out.device:
        args[27], args[28] = ws.data_ptr(), ws.numel()
        status = lib.tq_decode_append(*args)
        if status != _lib.TQ_E_WORKSPACE:
            _lib.check(status, "decode_append")
            return
    ws = wsp.get(workspace_bytes(units, group_size, head_dim, bits, max_len, mode), out.device)
    args[27], args[28] = ws.data_ptr(), ws.numel()
    _lib.check(lib.tq_decode_append(*args), "decode_append")


def decode_exchange_raw(*, exchange, new_k: torch.Tensor | None, new_v: torch.Tensor | None, rotate_k: bool,
                        rotate_v: bool, advance: bool, query: torch.Tensor, k_slab: torch.Tensor,
                        v_slab: torch.Tensor, unit_stride: int, lengths: torch.Tensor, units_per_seq: int,
                        len_offset: int, max_len: int, units: int, group_size: int, head_dim: int, bits: int,
                        cent_k: torch.Tensor, cent_v: torch.Tensor, out: torch.Tensor,
                        lse: torch.Tensor | None = None, rotate_query: bool = False, inverse_rotate: bool = False,
                        signs: tuple[torch.Tensor, torch.Tensor] | None = None, scale: float | None = None,
                        mode: str | int = "auto", workspace: Workspace | None = None) -> None:
    """One ``tq_decode_exchange`` call: this rank's shard decode, the peer
    exchange of the normalised partials and the cross-rank merge (see
    include/torque_b200.h).  ``exchange`` is a ``parallel.PeerExchange``."""
    lib = _lib.load()
    wsp = workspace or _default_ws
    sl, sr = signs if signs is not None else (None, None)
    ws = wsp.get(workspace_bytes(units, group_size, head_dim, bits, max_len, mode), out.device)
    dtype = _lib.dtype_code(new_k.dtype) if new_k is not None else _lib.TQ_F32
    _lib.check(lib.tq_decode_exchange(
        _lib.ptr(new_k), _lib.ptr(new_v), dtype, int(rotate_k), int(rotate_v), int(advance), query.data_ptr(),
        int(rotate_query), _lib.ptr(sl), _lib.ptr(sr), k_slab.data_ptr(), v_slab.data_ptr(), unit_stride,
        lengths.data_ptr(), units_per_seq, len_offset, max_len, units, group_size, head_dim, bits,
        cent_k.data_ptr(), cent_v.data_ptr(), float(1.0 / sqrt(head_dim) if scale is None else scale),
        out.data_ptr(), _lib.ptr(lse), int(inverse_rotate), decode_mode_code(mode), ws.data_ptr(), ws.numel(),
        exchange.bufs.data_ptr(), exchange.rank, exchange.world, exchange.epoch.data_ptr(), exchange.timeout_ns,
        exchange.status.data_ptr(), _lib.stream_ptr()), "decode_exchange")


def _cent(c) -> torch.Tensor:
    if isinstance(c, Codebook):
        c = c.centroids
    return _tensors.to_cuda(c, torch.float32)


def _check_codes(codes: torch.Tensor, bit_width: int, head_dim: int, name: str) -> int:
    W = packed_words_for_head_dim(head_dim, bit_width)
    if codes.shape[-1] != W:
        raise ValueError(f"packed width mismatch for {name}: expected {W}, got {codes.shape[-1]}")
    return W


def decode_packed_attention_split_batched(query, k_codes, v_codes, centroids_k, centroids_v, *,
                                          bit_width: int, head_dim: int, mode: str = "auto",
                                          return_lse: bool = False):
    """softmax(q.K^T / sqrt(d)) V per batch row over packed codes
    (mlx_ops.py:571-595).  query [BH, d]; k/v codes [BH, L, W] -> [BH, d]."""
    np_out = _tensors.is_numpy(query)
    q = _tensors.to_cuda(query, torch.float32)
    kc = _tensors.words_to_cuda(k_codes)
    vc = _tensors.words_to_cuda(v_codes)
    if q.dim() != 2 or q.shape[1] != head_dim:
        raise ValueError(f"batched query must have shape (batch, {head_dim}), got {tuple(q.shape)}")
    W = _check_codes(kc, bit_width, head_dim, "k_codes")
    _check_codes(vc, bit_width, head_dim, "v_codes")
    if kc.dim() != 3 or kc.shape != vc.shape or kc.shape[0] != q.shape[0]:
        raise ValueError("batched packed codes must have shape (batch, seq, packed_words) matching the query")
    B, L = int(kc.shape[0]), int(kc.shape[1])
    out = torch.empty((B, head_dim), dtype=torch.float32, device=q.device)
    lse = torch.empty((B,), dtype=torch.float32, device=q.device)
    decode_raw(query=q, k_slab=kc, v_slab=vc, unit_stride=L * W, lengths=None, units_per_seq=1, len_offset=L,
               max_len=L, units=B, group_size=1, head_dim=head_dim, bits=bit_width, cent_k=_cent(centroids_k),
               cent_v=_cent(centroids_v), out=out, lse=lse, mode=mode)
    if return_lse:
        return _tensors.out(out, np_out), _tensors.out(lse, np_out)
    return _tensors.out(out, np_out)


def decode_packed_attention(query, k_codes, v_codes, centroids_k, centroids_v, *, bit_width: int,
                            head_dim: int, mode: str = "auto"):
    """Single-head fused decode (mlx_ops.py:663-692): query [d]; codes [L, W] -> [d]."""
    np_out = _tensors.is_numpy(query)
    q = _tensors.to_cuda(query, torch.float32).reshape(1, -1)
    kc = _tensors.words_to_cuda(k_codes)
    vc = _tensors.words_to_cuda(v_codes)
    W = packed_words_for_head_dim(head_dim, bit_width)
    if kc.shape[-1] != W or vc.shape[-1] != W:
        raise ValueError("packed width mismatch for fused decode kernel")
    res = decode_packed_attention_split_batched(q, kc.reshape(1, -1, W), vc.reshape(1, -1, W), centroids_k,
                                                centroids_v, bit_width=bit_width, head_dim=head_dim, mode=mode)
    return _tensors.out(res[0], np_out)


decode_packed_attention_split = decode_packed_attention


def decode_packed_attention_split_batched_with_current(query, k_codes, v_codes, centroids_k, centroids_v,
                                                       current_keys, current_values, *, bit_width: int,
                                                       head_dim: int, mode: str = "auto"):
    """Attend packed codes plus one dense current token per row
    (mlx_ops.py:598-660).  The packed part is one ``tq_decode`` (which also
    yields its log-sum-exp); the current token is a second softmax part with
    lse = its scaled score, and ``tq_lse_merge`` combines the two exactly."""
    lib = _lib.load()
    np_out = _tensors.is_numpy(query)
    q = _tensors.to_cuda(query, torch.float32)
    ck = _tensors.to_cuda(current_keys, torch.float32)
    cv = _tensors.to_cuda(current_values, torch.float32)
    if q.dim() != 2 or q.shape[1] != head_dim:
        raise ValueError(f"batched query must have shape (batch, {head_dim}), got {tuple(q.shape)}")
    if ck.shape != q.shape:
        raise ValueError(f"current_keys must have shape {tuple(q.shape)}, got {tuple(ck.shape)}")
    if cv.shape != q.shape:
        raise ValueError(f"current_values must have shape {tuple(q.shape)}, got {tuple(cv.shape)}")
    kc = _tensors.words_to_cuda(k_codes)
    vc = _tensors.words_to_cuda(v_codes)
    if kc.dim() != 3 or vc.dim() != 3:
        raise ValueError("packed codes must have shape (batch, seq, packed_words)")
    if kc.shape != vc.shape:
        raise ValueError(f"k_codes and v_codes must match, got {tuple(kc.shape)} and {tuple(vc.shape)}")
    if kc.shape[0] != q.shape[0]:
        raise ValueError("packed codes and query must agree on batch dimension")
    B = q.shape[0]
    if kc.shape[1] == 0:
        return _tensors.out(cv.clone(), np_out)
    outs = torch.empty((2, B, head_dim), dtype=torch.float32, device=q.device)
    lses = torch.empty((2, B), dtype=torch.float32, device=q.device)
    o, s = decode_packed_attention_split_batched(q, kc, vc, centroids_k, centroids_v, bit_width=bit_width,
                                                 head_dim=head_dim, mode=mode, return_lse=True)
    outs[0].copy_(o)
    lses[0].copy_(s)
    outs[1].copy_(cv)
    lses[1].copy_((q * ck).sum(dim=1) * (1.0 / sqrt(head_dim)))
    res = torch.empty((B, head_dim), dtype=torch.float32, device=q.device)
    _lib.check(lib.tq_lse_merge(outs.data_ptr(), lses.data_ptr(), 2, B, head_dim, res.data_ptr(), None, 0, None,
                                None, _lib.stream_ptr()), "lse merge")
    return _tensors.out(res, np_out)


def lse_merge(outs: torch.Tensor, lses: torch.Tensor, *, out: torch.Tensor | None = None,
              lse_out: torch.Tensor | None = None, inverse_rotation=None) -> torch.Tensor:
    """Merge P normalised partial attentions ``outs [P, rows, d]`` with their
    natural-log ``lses [P, rows]`` (``tq_lse_merge``); optionally rotate the
    merged rows back with ``inverse_rotation`` (a RotationSpec)."""
    lib = _lib.load()
    P, rows, d = outs.shape
    res = out if out is not None else torch.empty((rows, d), dtype=torch.float32, device=outs.device)
    sl = sr = None
    if inverse_rotation is not None:
        sl, sr = inverse_rotation.device_signs()
    _lib.check(lib.tq_lse_merge(outs.contiguous().data_ptr(), lses.contiguous().data_ptr(), P, rows, d,
                                res.data_ptr(), _lib.ptr(lse_out), int(inverse_rotation is not None),
                                _lib.ptr(sl), _lib.ptr(sr), _lib.stream_ptr()), "lse merge")
    return res


def quantize_and_pack_rows(values, codebook, *, bit_width: int, head_dim: int, rotation=None):
    """Quantize + pack rows ``[R, d]`` into words ``[R, W]`` in one launch
    (mlx_ops.py:342-371).  Unlike the Metal kernel, which counts boundaries,
    this uses the reference numpy quantizer's nearest-centroid rule
    (quantization.py:120-125), so it needs the codebook itself.  ``rotation``
    (a RotationSpec) rotates the rows first, fused in the same kernel."""
    return quantize_and_pack_rows_dual(values, None, codebook, None, bit_width=bit_width, head_dim=head_dim,
                                       rotation=rotation)[0]


def quantize_and_pack_rows_dual(values_a, values_b, codebook_a, codebook_b, *, bit_width: int, head_dim: int,
                                rotation=None):
    """K and V rows in one launch (mlx_ops.py:374-412)."""
    lib = _lib.load()
    np_out = _tensors.is_numpy(values_a)
    a = _tensors.to_cuda(values_a, torch.float32, keep_half=True)
    if a.dim() != 2 or a.shape[1] != head_dim:
        raise ValueError(f"values_a must have shape (rows, {head_dim}), got {tuple(a.shape)}")
    b = None
    if values_b is not None:
        b = _tensors.to_cuda(values_b, torch.float32, keep_half=True).to(a.dtype)
        if b.shape != a.shape:
            raise ValueError(f"values_a and values_b must match, got {tuple(a.shape)} and {tuple(b.shape)}")
    W = packed_words_for_head_dim(head_dim, bit_width)
    R = int(a.shape[0])
    wa = torch.empty((R, W), dtype=torch.int32, device=a.device)
    wb = torch.empty((R, W), dtype=torch.int32, device=a.device) if b is not None else None
    ca = _cent(codebook_a)
    cb = _cent(codebook_b) if b is not None else None
    sl = sr = None
    if rotation is not None:
        sl, sr = rotation.device_signs()
    _lib.check(lib.tq_append_kv(a.data_ptr(), _lib.ptr(b), _lib.dtype_code(a.dtype), R, 1, head_dim, bit_width,
                                _lib.ptr(sl), _lib.ptr(sr), int(rotation is not None), ca.data_ptr(), _lib.ptr(cb),
                                wa.data_ptr(), _lib.ptr(wb), W, 1, None, 1, 0, _lib.stream_ptr()), "append")
    ra = _tensors.words_out(wa, np_out)
    rb = _tensors.words_out(wb, np_out) if wb is not None else None
    return ra, rb


def _boundaries(b, bit_width: int, label: str) -> torch.Tensor:
    t = _tensors.to_cuda(b, torch.float32)
    expected = (1 << bit_width) - 1
    if t.dim() != 1 or t.shape[0] != expected:
        raise ValueError(f"{label} must have shape ({expected},), got {tuple(t.shape)}")
    return t


def quantize_and_pack_rows_dual_metal(values_a, values_b, boundaries_a, boundaries_b, *, bit_width: int,
                                      head_dim: int):
    """Drop-in for ``quantize_and_pack_rows_dual_metal`` (mlx_ops.py:374-412):
    already-rotated rows ``[R, d]`` of two sets, each quantized by counting
    the boundaries it exceeds (the MLX rule, quantization.py:139-148) and
    packed, in one launch (tq_quantize_pack_boundaries).  Same argument
    checks and messages as the reference."""
    lib = _lib.load()
    np_out = _tensors.is_numpy(values_a)
    a = _tensors.to_cuda(values_a, torch.float32)
    if a.dim() != 2 or a.shape[1] != head_dim:
        raise ValueError(f"values_a must have shape (rows, {head_dim}), got {tuple(a.shape)}")
    b = _tensors.to_cuda(values_b, torch.float32)
    if tuple(b.shape) != tuple(a.shape):
        raise ValueError(f"values_a and values_b must match, got {tuple(a.shape)} and {tuple(b.shape)}")
    ba = _boundaries(boundaries_a, bit_width, "boundaries_a")
    bb = _boundaries(boundaries_b, bit_width, "boundaries_b")
    W = packed_words_for_head_dim(head_dim, bit_width)
    R = int(a.shape[0])
    wa = torch.empty((R, W), dtype=torch.int32, device=a.device)
    wb = torch.empty((R, W), dtype=torch.int32, device=a.device)
    _lib.check(lib.tq_quantize_pack_boundaries(a.data_ptr(), b.data_ptr(), R, head_dim, bit_width, ba.data_ptr(),
                                               bb.data_ptr(), wa.data_ptr(), wb.data_ptr(), _lib.stream_ptr()),
               "quantize and pack")
    return _tensors.words_out(wa, np_out), _tensors.words_out(wb, np_out)


def quantize_and_pack_rows_metal(values, boundaries, *, bit_width: int, head_dim: int):
    """Drop-in for ``quantize_and_pack_rows_metal`` (mlx_ops.py:342-371): one
    set of already-rotated rows, boundary-count quantizer, packed words."""
    lib = _lib.load()
    np_out = _tensors.is_numpy(values)
    a = _tensors.to_cuda(values, torch.float32)
    if a.dim() != 2 or a.shape[1] != head_dim:
        raise ValueError(f"values must have shape (rows, {head_dim}), got {tuple(a.shape)}")
    bd = _boundaries(boundaries, bit_width, "boundaries")
    W = packed_words_for_head_dim(head_dim, bit_width)
    R = int(a.shape[0])
    wa = torch.empty((R, W), dtype=torch.int32, device=a.device)
    _lib.check(lib.tq_quantize_pack_boundaries(a.data_ptr(), None, R, head_dim, bit_width, bd.data_ptr(), None,
                                               wa.data_ptr(), None, _lib.stream_ptr()), "quantize and pack")
    return _tensors.words_out(wa, np_out)


def dequantize_packed(words, codebook, *, bit_width: int, head_dim: int):
    """centroids[unpack(words)] for rows of packed words -> fp32 ``[..., d]``."""
    lib = _lib.load()
    np_out = _tensors.is_numpy(words)
    w = _tensors.words_to_cuda(words)
    _check_codes(w, bit_width, head_dim, "words")
    rows = w.numel() // w.shape[-1]
    out = torch.empty((*w.shape[:-1], head_dim), dtype=torch.float32, device=w.device)
    _lib.check(lib.tq_dequantize_packed(w.data_ptr(), out.data_ptr(), rows, head_dim, bit_width,
                                        _cent(codebook).data_ptr(), _lib.stream_ptr()), "dequantize")
    return _tensors.out(out, np_out)


def as_numpy_words(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int32).cpu().numpy().view(np.uint32)


# ---------------------------------------------------------------------------
# decoder glue (tq_rmsnorm / tq_rope_qk / tq_silu_mul): bf16 in and out
# ---------------------------------------------------------------------------
def _bf16_rows(x: torch.Tensor, name: str) -> torch.Tensor:
    if x.dtype != torch.bfloat16 or not x.is_cuda or not x.is_contiguous():
        raise ValueError(f"{name} must be a contiguous bf16 CUDA tensor")
    return x


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """Row-wise RMSNorm over the last axis: bf16(bf16(x * rsqrt(mean(x^2) + eps)) * weight)."""
    lib = _lib.load()
    _bf16_rows(x, "x")
    _bf16_rows(weight, "weight")
    n = x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    _lib.check(lib.tq_rmsnorm(x.data_ptr(), weight.data_ptr(), float(eps), x.numel() // n, n, out.data_ptr(),
                              _lib.stream_ptr()), "rmsnorm")
    return out


def rope_qk(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, position: torch.Tensor, q_heads: int,
            kv_heads: int, head_dim: int, q_out: torch.Tensor, k_out: torch.Tensor) -> None:
    """RoPE on the q and k heads of one fused qkv row at the device position
    ``position`` (int64 scalar tensor): q_out [q_heads, d] fp32 (bf16 values),
    k_out [kv_heads, d] bf16."""
    lib = _lib.load()
    _bf16_rows(qkv, "qkv")
    if position.dtype != torch.int64 or q_out.dtype != torch.float32 or k_out.dtype != torch.bfloat16:
        raise ValueError("rope_qk: position int64, q_out fp32 and k_out bf16 expected")
    _lib.check(lib.tq_rope_qk(qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), position.data_ptr(), q_heads, kv_heads,
                              head_dim, q_out.data_ptr(), k_out.data_ptr(), _lib.stream_ptr()), "rope_qk")


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """SwiGLU activation of rows [gate | up]: bf16(bf16(silu(gate)) * up)."""
    lib = _lib.load()
    _bf16_rows(gate_up, "gate_up")
    f = gate_up.shape[-1] // 2
    rows = gate_up.numel() // (2 * f)
    out = torch.empty(gate_up.shape[:-1] + (f,), dtype=torch.bfloat16, device=gate_up.device) if out is None else out
    _lib.check(lib.tq_silu_mul(gate_up.data_ptr(), rows, f, out.data_ptr(), _lib.stream_ptr()), "silu_mul")
    return out


_GEMV_MODES = {"bf16": 0, "f32": 1, "rms": 2, "silu": 3}


def gemv(weight: torch.Tensor, x: torch.Tensor, *, mode: str = "bf16", norm_weight: torch.Tensor | None = None,
         eps: float = 0.0, residual: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """One-token linear layer ``y = W x' (+ residual)`` (tq_gemv): ``weight``
    [n, k] bf16; ``x'`` is ``x`` (mode "bf16"), bf16 of an fp32 ``x`` ("f32"),
    its RMSNorm ("rms", with ``norm_weight`` / ``eps``) or the SwiGLU
    activation of a [gate | up] row ("silu").  Returns bf16 [n]."""
    lib = _lib.load()
    _bf16_rows(weight, "weight")
    n, k = weight.shape
    want = 2 * k if mode == "silu" else k
    if x.numel() != want or not x.is_contiguous() or x.dtype != (torch.float32 if mode == "f32" else torch.bfloat16):
        raise ValueError(f"gemv: x must be a contiguous {'fp32' if mode == 'f32' else 'bf16'} vector of {want}")
    if residual is not None and (residual.numel() != n or residual.dtype != torch.bfloat16):
        raise ValueError("gemv: residual must be bf16 with n elements")
    out = torch.empty(n, dtype=torch.bfloat16, device=weight.device) if out is None else out
    _lib.check(lib.tq_gemv(weight.data_ptr(), x.data_ptr(), _GEMV_MODES[mode], _lib.ptr(norm_weight), float(eps),
                           _lib.ptr(residual), out.data_ptr(), n, k, _lib.stream_ptr()), "gemv")
    return out
