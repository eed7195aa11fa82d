"""tq_decode_static — the decode entry point that allocates nothing.

Some callers cannot hand the library a workspace: a caller running inside a
memory pool it does not own, a foreign-language binding without access to the
CUDA allocator, or a server whose device memory is fixed at start-up.  For
them tq_decode_static keeps the split-K partials in a scratch array built into
the library.  These tests call it through the C ABI and compare it with
tq_decode (caller-provided workspace) on the same packed cache, twice in a
row, because every call reuses the same scratch.  This file sorts last so a
stop-at-first-failure run has already run every other test.
"""

from __future__ import annotations

import ctypes
from math import sqrt

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

import torque_mlx_b200 as T  # noqa: E402
from torque_mlx_b200 import _lib, ops  # noqa: E402


def _call(lib, fn, cache, q, out, lse, mode, ws=None):
    cfg = cache.config
    units = cache.batch_size * cfg.num_layers * cfg.kv_heads
    G = q.shape[0] // units
    sl, sr = cache.rotation.device_signs()
    args = [q.data_ptr(), 1, sl.data_ptr(), sr.data_ptr(), cache.key_slab.data_ptr(), cache.value_slab.data_ptr(),
            cache.capacity * T.packed_words_for_head_dim(cfg.head_dim, cfg.bit_width),
            cache.device_lengths.data_ptr(), cfg.num_layers * cfg.kv_heads, 0, cache.sequence_length, units, G,
            cfg.head_dim, cfg.bit_width, cache._ck.data_ptr(), cache._cv.data_ptr(), ctypes.c_float(1 / sqrt(cfg.head_dim)),
            out.data_ptr(), lse.data_ptr(), 1, ops.decode_mode_code(mode)]
    if ws is not None:
        args += [ws.data_ptr(), ws.numel()]
    args.append(_lib.stream_ptr())
    return fn(*args)


@pytest.mark.parametrize("mode,atol,rtol", [("tensor", 4e-3, 2e-2), ("exact", 2e-5, 1e-4)])
def test_static_scratch_decode_matches_workspace_decode(mode, atol, rtol):
    lib = _lib.load()
    rng = np.random.default_rng(31)
    cfg = T.TorqueConfig(bit_width=3, head_dim=128, num_layers=2, kv_heads=4)
    cache = T.TorqueKVCache(config=cfg, batch_size=3, decode_mode=mode)
    for s, n in enumerate((2000, 37, 5000)):
        cache.append_sequence(s, key=rng.standard_normal((2, 4, n, 128)).astype(np.float16),
                              value=rng.standard_normal((2, 4, n, 128)).astype(np.float16))
    dev = torch.device("cuda")
    rows = 3 * 2 * 4 * 4  # batch x layers x kv heads x G=4
    ws = torch.empty(ops.workspace_bytes(3 * 2 * 4, 4, 128, 3, cache.sequence_length, mode), dtype=torch.uint8,
                     device=dev)
    for call in range(2):  # the scratch keeps the previous call's contents
        q = torch.from_numpy(rng.standard_normal((rows, 128)).astype(np.float32)).to(dev)
        ref, ref_lse = torch.empty_like(q), torch.empty(rows, device=dev)
        got, got_lse = torch.full_like(q, float("nan")), torch.full((rows,), float("nan"), device=dev)
        _lib.check(_call(lib, lib.tq_decode, cache, q, ref, ref_lse, mode, ws=ws), "tq_decode")
        _lib.check(_call(lib, lib.tq_decode_static, cache, q, got, got_lse, mode), "tq_decode_static")
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(), atol=atol, rtol=rtol,
                                   err_msg=f"call {call}")
        np.testing.assert_allclose(got_lse.cpu().numpy(), ref_lse.cpu().numpy(), atol=atol, rtol=rtol)


def test_static_scratch_rejects_oversized_plans():
    """A plan whose partials exceed the built-in scratch is refused before any launch."""
    lib = _lib.load()
    need = ctypes.c_size_t()
    _lib.check(lib.tq_decode_workspace_size(60000, 16, 256, 4, 1 << 20, 1, ctypes.byref(need)), "size")
    assert need.value > 16 << 20
    dummy = torch.zeros(16, device="cuda")
    status = lib.tq_decode_static(dummy.data_ptr(), 0, None, None, dummy.data_ptr(), dummy.data_ptr(), 1 << 24, None, 1,
                                  1 << 20, 1 << 20, 60000, 16, 256, 4, dummy.data_ptr(), dummy.data_ptr(),
                                  ctypes.c_float(1.0), dummy.data_ptr(), None, 0, 1, _lib.stream_ptr())
    assert status == _lib.TQ_E_SCRATCH_LIMIT
    with pytest.raises(ValueError, match="scratch"):
        _lib.check(status, "tq_decode_static")


def test_static_scratch_unaligned_auto_takes_exact_plan():
    """Slabs that are not 16-byte aligned make AUTO run the exact kernel.  The
    scratch check sizes that plan, so an oversized one is refused with
    TQ_E_SCRATCH_LIMIT (not a workspace error), and the workspace size that AUTO
    reports covers it."""
    lib = _lib.load()
    units, G, d, b, n = 64, 16, 256, 4, 1 << 20
    sizes = {}
    for mode in (0, 1, 2):  # auto, exact, tensor
        need = ctypes.c_size_t()
        _lib.check(lib.tq_decode_workspace_size(units, G, d, b, n, mode, ctypes.byref(need)), "size")
        sizes[mode] = need.value
    assert sizes[2] <= 16 << 20 < sizes[1]
    assert sizes[0] >= max(sizes[1], sizes[2])
    dummy = torch.zeros(64, device="cuda")
    odd = dummy.data_ptr() + 4  # 4-byte aligned, not 16
    status = lib.tq_decode_static(dummy.data_ptr(), 0, None, None, odd, odd, n * (d * b // 32), None, 1, n, n,
                                  units, G, d, b, dummy.data_ptr(), dummy.data_ptr(), ctypes.c_float(1.0),
                                  dummy.data_ptr(), None, 0, 0, _lib.stream_ptr())
    assert status == _lib.TQ_E_SCRATCH_LIMIT


def test_static_scratch_unaligned_slabs_match_workspace_decode():
    """An AUTO decode over slabs shifted off 16-byte alignment (exact kernel)
    gives the same result through the scratch as through a workspace."""
    lib = _lib.load()
    rng = np.random.default_rng(8)
    cfg = T.TorqueConfig(bit_width=4, head_dim=64, num_layers=1, kv_heads=2)
    cache = T.TorqueKVCache(config=cfg, decode_mode="auto")
    cache.append(key=rng.standard_normal((1, 2, 700, 64)).astype(np.float16),
                 value=rng.standard_normal((1, 2, 700, 64)).astype(np.float16))
    dev = torch.device("cuda")
    kbuf = torch.zeros(cache.key_slab.numel() + 1, dtype=torch.int32, device=dev)
    vbuf = torch.zeros_like(kbuf)
    kbuf[1:].copy_(cache.key_slab.reshape(-1))
    vbuf[1:].copy_(cache.value_slab.reshape(-1))
    W = T.packed_words_for_head_dim(64, 4)
    sl, sr = cache.rotation.device_signs()
    ws = torch.empty(ops.workspace_bytes(2, 4, 64, 4, cache.sequence_length, "auto"), dtype=torch.uint8, device=dev)
    for call in range(2):
        q = torch.from_numpy(rng.standard_normal((8, 64)).astype(np.float32)).to(dev)
        outs = []
        for fn, extra in ((lib.tq_decode, [ws.data_ptr(), ws.numel()]), (lib.tq_decode_static, [])):
            out = torch.full_like(q, float("nan"))
            args = [q.data_ptr(), 1, sl.data_ptr(), sr.data_ptr(), kbuf[1:].data_ptr(), vbuf[1:].data_ptr(),
                    cache.capacity * W, cache.device_lengths.data_ptr(), 2, 0, cache.sequence_length, 2, 4, 64, 4,
                    cache._ck.data_ptr(), cache._cv.data_ptr(), ctypes.c_float(1 / 8), out.data_ptr(), None, 1, 0,
                    *extra, _lib.stream_ptr()]
            _lib.check(fn(*args), "decode")
            outs.append(out)
        torch.cuda.synchronize()
        np.testing.assert_allclose(outs[1].cpu().numpy(), outs[0].cpu().numpy(), atol=2e-5, rtol=1e-4,
                                   err_msg=f"call {call}")
        cache.decode_mode = "exact"  # the kernel AUTO took for the shifted slabs
        ref = cache.decode(query=q)
        cache.decode_mode = "auto"
        np.testing.assert_allclose(outs[0].cpu().numpy(), ref.cpu().numpy(), atol=2e-5, rtol=1e-4)
