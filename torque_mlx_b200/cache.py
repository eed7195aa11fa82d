"""Device-resident packed KV cache for B200 — the drop-in for the reference's
``TorqueKVCache`` (src/torque_mlx/cache.py:36-227) that also covers the
grouped-query / multi-token / append-then-attend surface of
``TorqueKVCacheMLX`` (src/torque_mlx/cache_mlx.py:41-799) and adds a batch of
independent sequences.

Storage: two int32 slabs ``[batch, layers, kv_heads, capacity, W]`` holding
the reference's packed uint32 words (``PackedKVLayout.tensor_shape`` with a
leading batch axis), plus device-resident per-sequence lengths.  A unit
``(seq, layer, kv_head)`` is one contiguous ``[capacity, W]`` run of words, so
decode streams it front to back.  Every step runs in libtorque_b200.so:

  append  -> tq_append_kv   (rotate + quantize + pack into the slab)
             tq_lengths_add (advance the device lengths)
  decode  -> tq_decode      (split-K packed attention + merge + Pi^T)

Inputs may be numpy arrays (copied to the device; numpy comes back, like the
reference) or torch tensors (CUDA tensors come back).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from math import sqrt

import numpy as np
import torch

from . import _lib, _tensors, ops
from .config import TorqueConfig
from .layout import CacheMetadata, PackedKVLayout
from .quantization import Codebook, build_gaussian_codebook, packed_words_for_head_dim
from .rotation import RotationSpec

_CAP_ALIGN = 128  # capacity granule (tokens); keeps every unit 16-byte aligned


def _round_cap(n: int) -> int:
    return max(_CAP_ALIGN, (n + _CAP_ALIGN - 1) // _CAP_ALIGN * _CAP_ALIGN)


@dataclass(eq=False)
class TorqueKVCache:
    """Rotation-native packed KV cache on the GPU.

    Same constructor fields and methods as the reference's numpy cache
    (``config``, ``key_codebook``, ``value_codebook``; ``append``, ``decode``,
    ``reset``, ``export_dequantized``, ``metadata``, ``sequence_length``) and
    the MLX cache's knobs (``initial_capacity``, ``growth_factor``,
    ``rotate_{keys,values}_on_append``, ``rotate_queries_on_decode``).

    Extensions: ``batch_size`` independent sequences with their own lengths,
    grouped-query decode (query heads = G x kv heads), multi-token appends,
    ``decode_with_current`` and a ``decode_mode`` of ``"auto"`` (tensor cores
    when G >= 2), ``"exact"`` (fp32 CUDA cores) or ``"tensor"``.
    """

    config: TorqueConfig = field(default_factory=TorqueConfig)
    key_codebook: Codebook | None = None
    value_codebook: Codebook | None = None
    initial_capacity: int = 256
    growth_factor: int = 2
    batch_size: int = 1
    decode_mode: str = "auto"
    rotate_keys_on_append: bool = True
    rotate_values_on_append: bool = True
    rotate_queries_on_decode: bool = True

    def __post_init__(self) -> None:
        self.config.validate()
        if self.initial_capacity <= 0:
            raise ValueError("initial_capacity must be positive")
        if self.growth_factor < 2:
            raise ValueError("growth_factor must be at least 2")
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive")
        ops.decode_mode_code(self.decode_mode)
        cfg = self.config
        # codebook seeds follow cache.py:48-55 (K: rotation_seed, V: rotation_seed + 1)
        self.key_codebook = self.key_codebook or build_gaussian_codebook(cfg.bit_width, seed=cfg.rotation_seed)
        self.value_codebook = self.value_codebook or build_gaussian_codebook(cfg.bit_width, seed=cfg.rotation_seed + 1)
        if self.key_codebook.bit_width != cfg.bit_width or self.value_codebook.bit_width != cfg.bit_width:
            raise ValueError("codebook bit width does not match the config")
        self.rotation = RotationSpec.from_seed(head_dim=cfg.head_dim, seed=cfg.rotation_seed)
        self._layout: PackedKVLayout = cfg.layout
        self._W = packed_words_for_head_dim(cfg.head_dim, cfg.bit_width)
        self._dev = _tensors.device()
        self._ck = _tensors.to_cuda(self.key_codebook.centroids, torch.float32)
        self._cv = _tensors.to_cuda(self.value_codebook.centroids, torch.float32)
        self._signs = self.rotation.device_signs()
        self._cap = _round_cap(self.initial_capacity)
        shape = (self.batch_size, cfg.num_layers, cfg.kv_heads, self._cap, self._W)
        self._k = torch.zeros(shape, dtype=torch.int32, device=self._dev)
        self._v = torch.zeros(shape, dtype=torch.int32, device=self._dev)
        self._len_dev = torch.zeros((self.batch_size,), dtype=torch.int32, device=self._dev)
        self._len_host = np.zeros((self.batch_size,), dtype=np.int64)
        self._ws = ops.Workspace()

    # ------------------------------------------------------------------ info
    @property
    def sequence_length(self) -> int:
        """Tokens held (the longest sequence when ``batch_size`` > 1)."""
        return int(self._len_host.max())

    @property
    def lengths(self) -> np.ndarray:
        return self._len_host.copy()

    @property
    def offset(self) -> int:
        return self.sequence_length

    @property
    def capacity(self) -> int:
        return self._cap

    @property
    def metadata(self) -> CacheMetadata:
        cfg = self.config
        return CacheMetadata(variant_id=cfg.variant_id, bit_width=cfg.bit_width, head_dim=cfg.head_dim,
                             num_layers=cfg.num_layers, kv_heads=cfg.kv_heads,
                             rotation_mode=cfg.rotation_mode.value, fused_weights=cfg.fused_weights,
                             codebook_name=self.key_codebook.name)

    @property
    def key_slab(self) -> torch.Tensor:
        """``[batch, layers, kv_heads, capacity, W]`` words (int32 storage)."""
        return self._k

    @property
    def value_slab(self) -> torch.Tensor:
        return self._v

    @property
    def device_lengths(self) -> torch.Tensor:
        return self._len_dev

    def packed_words(self) -> tuple[np.ndarray, np.ndarray]:
        """Host copy of the packed words, reference layout ``[layers, kv_heads,
        seq, W]`` (batch 1) or ``[batch, layers, kv_heads, seq, W]``."""
        n = self.sequence_length
        k = ops.as_numpy_words(self._k[..., :n, :])
        v = ops.as_numpy_words(self._v[..., :n, :])
        return (k[0], v[0]) if self.batch_size == 1 else (k, v)

    # --------------------------------------------------------------- storage
    def _ensure_capacity(self, needed: int) -> None:
        if needed <= self._cap:
            return
        cap = self._cap
        while cap < needed:
            cap *= self.growth_factor
        cap = _round_cap(cap)
        shape = (self.batch_size, self.config.num_layers, self.config.kv_heads, cap, self._W)
        nk = torch.zeros(shape, dtype=torch.int32, device=self._dev)
        nv = torch.zeros(shape, dtype=torch.int32, device=self._dev)
        n = self.sequence_length
        nk[..., :n, :].copy_(self._k[..., :n, :])
        nv[..., :n, :].copy_(self._v[..., :n, :])
        self._k, self._v, self._cap = nk, nv, cap

    def reset(self) -> None:
        self._len_dev.zero_()
        self._len_host[:] = 0

    # ---------------------------------------------------------------- shapes
    def _norm_kv(self, x, label: str) -> torch.Tensor:
        """-> contiguous ``[batch, layers, kv_heads, T, d]`` on the device
        (shape rules of cache.py:216-227 and cache_mlx.py:474-498)."""
        cfg = self.config
        L, H, d, B = cfg.num_layers, cfg.kv_heads, cfg.head_dim, self.batch_size
        t = _tensors.to_cuda(x, torch.float32, keep_half=True)
        s = tuple(t.shape)
        if B == 1:
            if s == (d,):
                if (L, H) != (1, 1):
                    raise ValueError(f"{label} shape {s} only valid for 1 layer / 1 head")
                return t.reshape(1, 1, 1, 1, d)
            if s == (H, d):
                if L != 1:
                    raise ValueError(f"{label} shape {s} only valid for 1 layer")
                return t.reshape(1, 1, H, 1, d)
            if s == (L, H, d):
                return t.reshape(1, L, H, 1, d)
            if len(s) == 3 and L == 1 and s[0] == H and s[2] == d:
                return t.reshape(1, 1, H, s[1], d)
            if len(s) == 4 and s[0] == L and s[1] == H and s[3] == d:
                return t.reshape(1, L, H, s[2], d)
            raise ValueError(f"{label} must have shape ({L}, {H}, seq_len, {d}) or a compatible single-token "
                             f"form, got {s}")
        if s == (B, L, H, d):
            return t.reshape(B, L, H, 1, d)
        if len(s) == 5 and s[:3] == (B, L, H) and s[4] == d:
            return t
        if L == 1 and len(s) == 3 and s == (B, H, d):
            return t.reshape(B, 1, H, 1, d)
        raise ValueError(f"{label} must have shape ({B}, {L}, {H}, seq_len, {d}) or ({B}, {L}, {H}, {d}), got {s}")

    def _norm_query(self, x) -> tuple[torch.Tensor, int, tuple[int, ...]]:
        """-> ([batch*layers*Hq, d] fp32, Hq, output shape)."""
        cfg = self.config
        L, H, d, B = cfg.num_layers, cfg.kv_heads, cfg.head_dim, self.batch_size
        t = _tensors.to_cuda(x, torch.float32)
        s = tuple(t.shape)
        if B == 1:
            if s == (d,):
                if (L, H) != (1, 1):
                    raise ValueError(f"query shape {s} only valid for 1 layer / 1 head")
                hq, out_shape = 1, (d,)
            elif len(s) == 2 and s[1] == d and L == 1:
                hq, out_shape = s[0], s
            elif len(s) == 3 and s[0] == L and s[2] == d:
                hq = s[1]
                out_shape = (hq, d) if L == 1 and hq != 1 else s
                if L == 1 and hq == 1:
                    out_shape = (d,)
            else:
                raise ValueError(f"query must have shape ({L}, query_heads, {d}) or a compatible 1-layer form, "
                                 f"got {s}")
        else:
            if len(s) == 4 and s[0] == B and s[1] == L and s[3] == d:
                hq, out_shape = s[2], s
            elif L == 1 and len(s) == 3 and s[0] == B and s[2] == d:
                hq, out_shape = s[1], s
            else:
                raise ValueError(f"query must have shape ({B}, {L}, query_heads, {d}), got {s}")
        if hq % H != 0:
            raise ValueError(f"query head count {hq} must be divisible by kv_heads {H}")
        if hq // H > 16:
            raise ValueError(f"query group size {hq // H} exceeds 16")
        return t.reshape(B * L * hq, d).contiguous(), hq, out_shape

    # ----------------------------------------------------------------- append
    def _launch_append(self, k: torch.Tensor | None, v: torch.Tensor | None, *, groups: int, tokens: int,
                       k_slab: torch.Tensor, v_slab: torch.Tensor, start: torch.Tensor, groups_per_seq: int,
                       rotate: bool) -> None:
        lib = _lib.load()
        cfg = self.config
        sl, sr = self._signs
        first = k if k is not None else v
        _lib.check(lib.tq_append_kv(
            first.data_ptr(), v.data_ptr() if (k is not None and v is not None) else None,
            _lib.dtype_code(first.dtype), groups, tokens, cfg.head_dim, cfg.bit_width, sl.data_ptr(), sr.data_ptr(),
            int(rotate), (self._ck if k is not None else self._cv).data_ptr(), self._cv.data_ptr(),
            (k_slab if k is not None else v_slab).data_ptr(), v_slab.data_ptr(), self._cap * self._W, self._cap,
            start.data_ptr(), groups_per_seq, 0, _lib.stream_ptr()), "append")

    def _write(self, keys: torch.Tensor, values: torch.Tensor, *, seq: int | None = None) -> int:
        """Pack ``[B', L, H, T, d]`` rows at each sequence's current length
        without advancing it; returns T."""
        cfg = self.config
        if keys.shape != values.shape:
            raise ValueError(f"key/value shapes must match, got {tuple(keys.shape)} and {tuple(values.shape)}")
        if values.dtype != keys.dtype:
            values = values.to(keys.dtype)
        T = int(keys.shape[3])
        if T == 0:
            return 0
        if seq is None:
            need = int(self._len_host.max()) + T
        else:
            need = int(self._len_host[seq]) + T
        self._ensure_capacity(need)
        groups = int(keys.shape[0]) * cfg.num_layers * cfg.kv_heads
        gps = cfg.num_layers * cfg.kv_heads
        if seq is None:
            ks, vs, start = self._k, self._v, self._len_dev
        else:
            ks, vs, start = self._k[seq], self._v[seq], self._len_dev[seq:seq + 1]
        k = keys.reshape(groups, T, cfg.head_dim).contiguous()
        v = values.reshape(groups, T, cfg.head_dim).contiguous()
        if self.rotate_keys_on_append == self.rotate_values_on_append:
            self._launch_append(k, v, groups=groups, tokens=T, k_slab=ks, v_slab=vs, start=start,
                                groups_per_seq=gps, rotate=self.rotate_keys_on_append)
        else:
            self._launch_append(k, None, groups=groups, tokens=T, k_slab=ks, v_slab=vs, start=start,
                                groups_per_seq=gps, rotate=self.rotate_keys_on_append)
            self._launch_append(None, v, groups=groups, tokens=T, k_slab=ks, v_slab=vs, start=start,
                                groups_per_seq=gps, rotate=self.rotate_values_on_append)
        return T

    def _advance(self, T: int, seq: int | None = None) -> None:
        lib = _lib.load()
        if seq is None:
            _lib.check(lib.tq_lengths_add(self._len_dev.data_ptr(), self.batch_size, T, _lib.stream_ptr()),
                       "lengths")
            self._len_host += T
        else:
            _lib.check(lib.tq_lengths_add(self._len_dev[seq:seq + 1].data_ptr(), 1, T, _lib.stream_ptr()),
                       "lengths")
            self._len_host[seq] += T

    def _advance_device(self, T: int) -> None:
        lib = _lib.load()
        _lib.check(lib.tq_lengths_add(self._len_dev.data_ptr(), self.batch_size, T, _lib.stream_ptr()), "lengths")

    def append(self, *, key, value) -> None:
        """Append one step (``[layers, kv_heads, d]`` and the reference's short
        forms) or T tokens (``[layers, kv_heads, T, d]``) to every sequence
        (cache.py:78-96, cache_mlx.py:151-171)."""
        k = self._norm_kv(key, "key")
        v = self._norm_kv(value, "value")
        if k.shape[:4] != v.shape[:4]:
            raise ValueError(f"key/value sequence dimensions must match, got {tuple(k.shape)} and {tuple(v.shape)}")
        T = self._write(k, v)
        if T:
            self._advance(T)

    append_many = append
    append_many_mlx = append

    def append_sequence(self, seq: int, *, key, value) -> None:
        """Append ``[layers, kv_heads, T, d]`` tokens to sequence ``seq`` only
        (ragged prefill of a batch)."""
        if not 0 <= seq < self.batch_size:
            raise ValueError(f"sequence index {seq} out of range")
        cfg = self.config
        t = _tensors.to_cuda(key, torch.float32, keep_half=True)
        u = _tensors.to_cuda(value, torch.float32, keep_half=True)
        want = (cfg.num_layers, cfg.kv_heads)
        if t.dim() != 4 or tuple(t.shape[:2]) != want or t.shape[3] != cfg.head_dim or t.shape != u.shape:
            raise ValueError(f"key/value must have shape ({want[0]}, {want[1]}, T, {cfg.head_dim})")
        T = self._write(t.unsqueeze(0), u.unsqueeze(0), seq=seq)
        if T:
            self._advance(T, seq)

    # ----------------------------------------------------------------- decode
    def _decode(self, q: torch.Tensor, hq: int, *, extra: int, return_lse: bool, full_capacity: bool = False,
                out: torch.Tensor | None = None):
        cfg = self.config
        G = hq // cfg.kv_heads
        units = self.batch_size * cfg.num_layers * cfg.kv_heads
        if out is None:
            out = torch.empty_like(q)
        lse = torch.empty((q.shape[0],), dtype=torch.float32, device=q.device) if return_lse else None
        # The split plan follows max_len; a captured step plans for the whole
        # capacity so the graph stays valid while the device lengths grow.
        max_len = self._cap if full_capacity else min(self._cap, self.sequence_length + extra)
        ops.decode_raw(query=q, k_slab=self._k, v_slab=self._v, unit_stride=self._cap * self._W,
                       lengths=self._len_dev, units_per_seq=cfg.num_layers * cfg.kv_heads, len_offset=extra,
                       max_len=max_len, units=units, group_size=G,
                       head_dim=cfg.head_dim, bits=cfg.bit_width, cent_k=self._ck, cent_v=self._cv, out=out, lse=lse,
                       rotate_query=self.rotate_queries_on_decode, inverse_rotate=not cfg.fused_weights,
                       signs=self._signs, scale=1.0 / sqrt(cfg.head_dim), mode=self.decode_mode, workspace=self._ws)
        return out, lse

    def decode(self, *, query, return_lse: bool = False):
        """Decode attention for one query step (cache.py:98-140,
        cache_mlx.py:173-234).  ``query`` is ``[layers, Hq, d]`` (or the
        reference's 1-layer short forms; ``[batch, layers, Hq, d]`` for a
        batch); Hq = G x kv_heads.  Returns the same shape; with
        ``return_lse`` also the natural-log sum-exp per query row."""
        np_out = _tensors.is_numpy(query)
        q, hq, out_shape = self._norm_query(query)
        out, lse = self._decode(q, hq, extra=0, return_lse=return_lse)
        res = _tensors.out(out.reshape(out_shape), np_out)
        if return_lse:
            lse_shape = out_shape[:-1] if len(out_shape) > 1 else ()
            return res, _tensors.out(lse.reshape(lse_shape), np_out)
        return res

    decode_mlx = decode

    def _step(self, k: torch.Tensor, v: torch.Tensor, q: torch.Tensor, hq: int, *, advance: bool, return_lse: bool,
              full_capacity: bool = False, out: torch.Tensor | None = None):
        """Fused append + decode of one token per sequence (tq_decode_append):
        ``k``/``v`` are ``[B, L, H, 1, d]``; the token is packed at each
        sequence's length and attended; ``advance`` counts it on the device
        (the host copy of the lengths is the caller's to update)."""
        cfg = self.config
        self._ensure_capacity(int(self._len_host.max()) + 1)
        if v.dtype != k.dtype:
            v = v.to(k.dtype)
        G = hq // cfg.kv_heads
        units = self.batch_size * cfg.num_layers * cfg.kv_heads
        if out is None:
            out = torch.empty_like(q)
        lse = torch.empty((q.shape[0],), dtype=torch.float32, device=q.device) if return_lse else None
        max_len = self._cap if full_capacity else min(self._cap, int(self._len_host.max()) + 1)
        ops.decode_append_raw(
            new_k=k.reshape(units, cfg.head_dim), new_v=v.reshape(units, cfg.head_dim),
            rotate_k=self.rotate_keys_on_append, rotate_v=self.rotate_values_on_append, advance=advance, query=q,
            k_slab=self._k, v_slab=self._v, unit_stride=self._cap * self._W, lengths=self._len_dev,
            units_per_seq=cfg.num_layers * cfg.kv_heads, max_len=max_len, units=units, group_size=G,
            head_dim=cfg.head_dim, bits=cfg.bit_width, cent_k=self._ck, cent_v=self._cv, out=out, lse=lse,
            rotate_query=self.rotate_queries_on_decode, inverse_rotate=not cfg.fused_weights, signs=self._signs,
            scale=1.0 / sqrt(cfg.head_dim), mode=self.decode_mode, workspace=self._ws)
        return out, lse

    def append_decode(self, *, key, value, query, return_lse: bool = False):
        """One generation step in one fused call: append one token to every
        sequence (``key``/``value`` in ``append``'s single-token shapes) and
        attend ``query`` over the cache including it.  Same result as
        ``append`` followed by ``decode``, with the token packed inside the
        decode kernel (tq_decode_append)."""
        np_out = _tensors.is_numpy(query)
        q, hq, out_shape = self._norm_query(query)
        k = self._norm_kv(key, "key")
        v = self._norm_kv(value, "value")
        if k.shape[3] != 1 or v.shape[3] != 1:
            raise ValueError("append_decode expects a single token per sequence for key/value")
        out, lse = self._step(k, v, q, hq, advance=True, return_lse=return_lse)
        self._len_host += 1
        res = _tensors.out(out.reshape(out_shape), np_out)
        if return_lse:
            lse_shape = out_shape[:-1] if len(out_shape) > 1 else ()
            return res, _tensors.out(lse.reshape(lse_shape), np_out)
        return res

    def decode_with_current(self, *, query, key, value):
        """Attend the cache plus one current token that is not yet appended
        (cache_mlx.py:236-302): the token is packed at each sequence's next
        position and attended, but the lengths do not advance, so a later
        ``append`` of the same token gives the same cache."""
        np_out = _tensors.is_numpy(query)
        q, hq, out_shape = self._norm_query(query)
        k = self._norm_kv(key, "key")
        v = self._norm_kv(value, "value")
        if k.shape[3] != 1 or v.shape[3] != 1:
            raise ValueError("decode_with_current expects a single current token for key/value")
        out, _ = self._step(k, v, q, hq, advance=False, return_lse=False)
        return _tensors.out(out.reshape(out_shape), np_out)

    decode_mlx_with_current = decode_with_current

    def attend_chunk(self, *, query):
        """Chunked-prefill attention on the packed cache: the last T tokens of
        every sequence (appended already, e.g. by ``append``) attend causally,
        each over the packed prefix and the chunk up to itself — the prefill
        step of the reference's chunked loop (qwen_mlx.py:829-845), here over
        packed codes.  ``query`` is ``[layers, T, Hq, d]`` (batch 1) or
        ``[batch, layers, T, Hq, d]``; the result has its shape.  Runs as
        ``tq_decode_causal`` launches of up to 16 query rows per kv head."""
        cfg = self.config
        np_out = _tensors.is_numpy(query)
        t = _tensors.to_cuda(query, torch.float32)
        shape = tuple(t.shape)
        B, L, H, d = self.batch_size, cfg.num_layers, cfg.kv_heads, cfg.head_dim
        if t.dim() == 4 and B == 1:
            t = t.unsqueeze(0)
        if t.dim() != 5 or t.shape[0] != B or t.shape[1] != L or t.shape[4] != d:
            raise ValueError(f"query must have shape ({L}, T, query_heads, {d}) or ({B}, {L}, T, query_heads, {d}), "
                             f"got {shape}")
        T, hq = int(t.shape[2]), int(t.shape[3])
        if hq % H != 0:
            raise ValueError(f"query head count {hq} must be divisible by kv_heads {H}")
        G = hq // H
        if G > 16:
            raise ValueError(f"query group size {G} exceeds 16")
        if T < 1 or T > int(self._len_host.min()):
            raise ValueError("attend_chunk needs 1 <= T <= every sequence's length (append the chunk first)")
        q = t.reshape(B, L, T, H, G, d).permute(0, 1, 3, 2, 4, 5)  # [B, L, H, T, G, d]: unit-major rows
        out = torch.empty_like(q)
        units = B * L * H
        step = max(1, 16 // G)
        max_len = min(self._cap, self.sequence_length)
        for j0 in range(0, T, step):
            j1 = min(T, j0 + step)
            qs = q[:, :, :, j0:j1].contiguous()
            os_ = torch.empty_like(qs)
            ops.decode_causal_raw(query=qs, k_slab=self._k, v_slab=self._v, unit_stride=self._cap * self._W,
                                  lengths=self._len_dev, units_per_seq=L * H, len_offset=-(T - j1), max_len=max_len,
                                  units=units, q_tokens=j1 - j0, group_size=G, head_dim=d, bits=cfg.bit_width,
                                  cent_k=self._ck, cent_v=self._cv, out=os_, rotate_query=self.rotate_queries_on_decode,
                                  inverse_rotate=not cfg.fused_weights, signs=self._signs,
                                  scale=1.0 / sqrt(d), workspace=self._ws)
            out[:, :, :, j0:j1] = os_
        res = out.permute(0, 1, 3, 2, 4, 5).reshape(B, L, T, hq, d).reshape(shape)
        return _tensors.out(res, np_out)

    # ------------------------------------------------------------ CUDA graph
    def capture_step(self, *, key, value, query, steps_per_replay: int = 1) -> "CapturedDecodeStep":
        """Capture one decode step (append one token to every sequence, then
        attend) into CUDA graphs for launch-free replay.  ``key``/``value``/
        ``query`` are example CUDA tensors in the shapes ``append``/``decode``
        take; their contents are copied into static input buffers.
        ``steps_per_replay`` > 1 puts that many consecutive fused steps in the
        ``step`` graph, so short steps are not bound by the host's replay rate."""
        return CapturedDecodeStep(self, key=key, value=value, query=query, steps_per_replay=steps_per_replay)

    # ------------------------------------------------------------------ misc
    def export_dequantized(self) -> tuple[np.ndarray, np.ndarray]:
        """Dequantized rotated contents ``[layers, kv_heads, seq, d]`` (or with
        a leading batch axis) for tests and benchmarks (cache.py:189-214).
        Positions past a shorter sequence's length are zero."""
        cfg = self.config
        n = self.sequence_length
        keys = ops.dequantize_packed(self._k[..., :n, :].contiguous(), self._ck, bit_width=cfg.bit_width,
                                     head_dim=cfg.head_dim)
        values = ops.dequantize_packed(self._v[..., :n, :].contiguous(), self._cv, bit_width=cfg.bit_width,
                                       head_dim=cfg.head_dim)
        pos = torch.arange(n, device=self._dev)
        valid = (pos[None, :] < self._len_dev[:, None].to(torch.int64)).reshape(self.batch_size, 1, 1, n, 1)
        keys = (keys * valid).cpu().numpy()
        values = (values * valid).cpu().numpy()
        return (keys[0], values[0]) if self.batch_size == 1 else (keys, values)

    def make_mask(self, N: int, *, window_size: int | None = None, return_array: bool = False):
        """Attention mask helper of the MLX-LM cache protocol (cache_mlx.py:317-334)."""
        if N == 1:
            return None
        if not return_array and (window_size is None or N <= window_size):
            return "causal"
        offset = self.offset
        rinds = torch.arange(offset + N, device=self._dev)
        linds = torch.arange(offset, offset + N, device=self._dev) if offset else rinds
        mask = linds[:, None] >= rinds[None]
        if window_size is not None:
            mask = mask & (linds[:, None] < rinds[None] + window_size)
        return mask


TorqueKVCacheB200 = TorqueKVCache

DecodeStrategy = str
SUPPORTED_DECODE_STRATEGIES: tuple[str, ...] = ("auto", "split_batched", "fused_per_head")


@dataclass(eq=False)
class TorqueKVCacheMLX(TorqueKVCache):
    """Drop-in for the reference's device cache ``TorqueKVCacheMLX``
    (cache_mlx.py:40-125): same constructor knobs and the ``decode_mlx`` /
    ``decode_mlx_with_current`` calls with ``return_numpy``.

    * ``decode_tail_capacity`` (cache_mlx.py:50): the reference keeps up to that
      many single-token appends as dequantized fp16 rows before packing them.
      Here every append is packed at once by the append kernel, which the
      decode reads directly, so no tail is needed; the value is validated and
      kept.  Results equal those of the reference's packed path (the tail
      rows hold the same centroids, rounded to fp16).
    * ``decode_strategy`` (cache_mlx.py:51): validated against the reference's
      choices and reported by ``resolve_decode_strategy``; the B200 decode is
      one fused kernel for every strategy.
    * ``profile_decode_components`` (cache_mlx.py:52): when set,
      ``last_decode_profile`` gets the wall time of each decode call
      (``packed_decode_seconds``, synchronised).
    """

    decode_tail_capacity: int = 16
    decode_strategy: DecodeStrategy = "split_batched"
    profile_decode_components: bool = False

    def __post_init__(self) -> None:
        if self.decode_tail_capacity < 0:
            raise ValueError("decode_tail_capacity must be non-negative")
        if self.decode_strategy not in SUPPORTED_DECODE_STRATEGIES:
            raise ValueError("decode_strategy must be one of " + ", ".join(SUPPORTED_DECODE_STRATEGIES))
        super().__post_init__()
        self.last_decode_profile: dict[str, float] = {}

    def resolve_decode_strategy(self, *, sequence_length: int | None = None) -> str:
        """cache_mlx.py:742-745: ``auto`` resolves to ``split_batched``."""
        return self.decode_strategy if self.decode_strategy != "auto" else "split_batched"

    @property
    def _key_codes(self) -> torch.Tensor:
        """Packed K words ``[layers, kv_heads, capacity, W]`` (int32 storage of
        the uint32 words), as the reference's attribute of that name."""
        return self._k[0] if self.batch_size == 1 else self._k

    @property
    def _value_codes(self) -> torch.Tensor:
        return self._v[0] if self.batch_size == 1 else self._v

    def _finalize(self, out: torch.Tensor, query_heads: int, return_numpy: bool):
        """cache_mlx.py:340-351: numpy with the 1-layer / 1-head squeezes, or
        the device array ``[layers, Hq, d]``."""
        L, d = self.config.num_layers, self.config.head_dim
        out = out.reshape(L, query_heads, d) if self.batch_size == 1 else out.reshape(-1, L, query_heads, d)
        if not return_numpy:
            return out
        arr = out.cpu().numpy()
        if self.batch_size == 1 and L == 1 and query_heads == 1:
            return arr[0, 0]
        if self.batch_size == 1 and L == 1:
            return arr[0]
        return arr

    def _timed(self, fn):
        if not self.profile_decode_components:
            return fn()
        import time
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        res = fn()
        torch.cuda.synchronize()
        self.last_decode_profile["packed_decode_seconds"] = time.perf_counter() - t0
        return res

    def decode_mlx(self, *, query, return_numpy: bool = True):
        """cache_mlx.py:173-234."""
        self.last_decode_profile = {}
        q, hq, _ = self._norm_query(query)
        out, _ = self._timed(lambda: self._decode(q, hq, extra=0, return_lse=False))
        return self._finalize(out, hq, return_numpy)

    def decode_mlx_with_current(self, *, query, key, value, return_numpy: bool = True):
        """cache_mlx.py:236-302: attend the cache plus one current token that is
        not appended."""
        self.last_decode_profile = {}
        q, hq, _ = self._norm_query(query)
        k = self._norm_kv(key, "key")
        v = self._norm_kv(value, "value")
        if k.shape[3] != 1 or v.shape[3] != 1:
            raise ValueError("decode_mlx_with_current expects a single current token for key/value")
        out, _ = self._timed(lambda: self._step(k, v, q, hq, advance=False, return_lse=False))
        return self._finalize(out, hq, return_numpy)


class CapturedDecodeStep:
    """One decode step of a TorqueKVCache replayed from CUDA graphs.

    Three graphs over the static key / value / query buffers and the static
    output: ``append`` (tq_append_kv + tq_lengths_add), ``decode`` (tq_decode)
    and ``step`` (tq_decode_append: both in one decode launch plus the merge).  The decode plan covers the cache's whole capacity, so the
    captured launch stays valid as the device lengths grow; call ``step`` (or
    the two replays) until ``remaining`` reaches zero, then capture again.
    """

    def __init__(self, cache: TorqueKVCache, *, key, value, query, steps_per_replay: int = 1):
        if steps_per_replay < 1:
            raise ValueError("steps_per_replay must be positive")
        self.steps_per_replay = int(steps_per_replay)
        if not (isinstance(key, torch.Tensor) and key.is_cuda and isinstance(query, torch.Tensor) and query.is_cuda):
            raise ValueError("capture_step needs CUDA tensors")
        self.cache = cache
        k = cache._norm_kv(key, "key")
        if k.shape[3] != 1:
            raise ValueError("a captured step appends exactly one token per sequence")
        self.key = k.clone()
        self.value = cache._norm_kv(value, "value").to(k.dtype).clone()
        q, hq, self._out_shape = cache._norm_query(query)
        self.query = q.clone()
        self.out = torch.empty_like(self.query)
        self._hq = hq
        cache._ensure_capacity(cache.sequence_length + self.steps_per_replay)
        stream = torch.cuda.Stream(device=cache._dev)
        stream.wait_stream(torch.cuda.current_stream(cache._dev))
        with torch.cuda.stream(stream):
            # size the workspace for the capacity plan before capturing
            cache._decode(self.query, hq, extra=0, return_lse=False, full_capacity=True, out=self.out)
            stream.synchronize()
            self.g_append = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.g_append, stream=stream):
                cache._write(self.key, self.value)
                cache._advance_device(1)
            self.g_decode = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.g_decode, stream=stream):
                cache._decode(self.query, hq, extra=0, return_lse=False, full_capacity=True, out=self.out)
            self.g_step = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.g_step, stream=stream):
                for _ in range(self.steps_per_replay):  # lengths advance on the device between steps
                    cache._step(self.key, self.value, self.query, hq, advance=True, return_lse=False,
                                full_capacity=True, out=self.out)
        torch.cuda.current_stream(cache._dev).wait_stream(stream)

    @property
    def remaining(self) -> int:
        """Steps left before the captured plan would run past the capacity."""
        return self.cache.capacity - int(self.cache._len_host.max())

    def append(self) -> None:
        if self.remaining < 1:
            raise RuntimeError("cache capacity reached: capture the step again")
        self.g_append.replay()
        self.cache._len_host += 1

    def decode(self) -> torch.Tensor:
        self.g_decode.replay()
        return self.out.reshape(self._out_shape)

    def run(self, *, key, value, query) -> torch.Tensor:
        """Serving form of a captured step: copy this step's new key/value and
        query (same shapes as at capture; host tensors - pinned for an
        asynchronous copy - or device tensors) into the static input buffers on
        the current stream, then replay one fused step.  Returns the static
        output buffer (overwritten by the next step; copy it out before)."""
        if self.steps_per_replay != 1:
            raise ValueError("run() needs a step captured with steps_per_replay=1")
        for dst, src, name in ((self.key, key, "key"), (self.value, value, "value"), (self.query, query, "query")):
            if not isinstance(src, torch.Tensor) or src.numel() != dst.numel():
                raise ValueError(f"{name} must be a tensor with {dst.numel()} elements, as at capture")
            dst.view(-1).copy_(src.reshape(-1), non_blocking=True)
        return self.step()

    def step(self) -> torch.Tensor:
        """Append the static token and attend, as one fused replay
        (tq_decode_append: the decode kernel packs the token); with
        ``steps_per_replay`` = k, k such steps (the output is the last one's)."""
        if self.remaining < self.steps_per_replay:
            raise RuntimeError("cache capacity reached: capture the step again")
        self.g_step.replay()
        self.cache._len_host += self.steps_per_replay
        return self.out.reshape(self._out_shape)
