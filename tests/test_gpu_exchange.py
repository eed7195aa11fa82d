"""tq_decode_exchange on one GPU: the fused exchange + cross-rank merge.

Several ranks cannot be run as separate kernels on one GPU (they would wait
on one another), so these tests drive one rank's kernel with the other
ranks' side prepared by the host:
  * world 1: the exchange path equals the plain decode;
  * world 2, rank 0: the other rank's normalised partial and its flag are
    written into this rank's buffer before the launch (what the peer's kernel
    would have stored), and the peer's buffer is a second local allocation.
    The merged output must equal the float64 oracle over both shards' tokens,
    and this rank's partial must have landed in the peer's buffer with its
    flag;
  * a peer that never arrives: the flag stays unset, the bounded wait gives
    up after the timeout, status reads TQ_E_TIMEOUT, the rows are NaN, and
    the GPU context stays usable.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import torque_oracle as O

pytestmark = pytest.mark.gpu

import torque_mlx_b200 as T  # noqa: E402
from torque_mlx_b200 import _lib, ops  # noqa: E402
from torque_mlx_b200.parallel import PeerExchange  # noqa: E402

H, G, d, b = 2, 8, 256, 4
ROWS = H * G


class _LocalExchange:
    """The attributes tq_decode_exchange reads, over buffers of this process:
    ``bufs[rank]`` is this rank's buffer, the others stand in for peers."""

    def __init__(self, world: int, rank: int, timeout_s: float):
        nbytes = _lib.c_size_t(0)
        _lib.check(_lib.load().tq_exchange_buffer_bytes(d, world, ROWS, _lib.ctypes.byref(nbytes)), "size")
        self.mem = [torch.zeros(int(nbytes.value) // 4, dtype=torch.float32, device="cuda") for _ in range(world)]
        self.bufs = torch.tensor([m.data_ptr() for m in self.mem], dtype=torch.int64, device="cuda")
        self.rank, self.world, self.rows = rank, world, ROWS
        self.epoch = torch.zeros(ROWS, dtype=torch.int32, device="cuda")
        self.status = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.timeout_ns = int(timeout_s * 1e9)

    def slot(self, buf: int, parity: int, src: int) -> torch.Tensor:
        data = self.mem[buf][: 2 * self.world * ROWS * (d + 4)].view(2, self.world, ROWS, d + 4)
        return data[parity, src]

    def flags(self, buf: int) -> torch.Tensor:
        return self.mem[buf][2 * self.world * ROWS * (d + 4):].view(torch.int32)[: self.world * ROWS].view(
            self.world, ROWS)


def _shard(seed: int, n: int):
    rng = np.random.default_rng(seed)
    cfg = T.TorqueConfig(bit_width=b, head_dim=d, kv_heads=H, fused_weights=True)
    cache = T.TorqueKVCache(config=cfg, decode_mode="tensor")
    cache.append(key=rng.standard_normal((H, n, d)).astype(np.float16),
                 value=rng.standard_normal((H, n, d)).astype(np.float16))
    return cache


def _run(cache, x, q, out):
    cfg = cache.config
    ops.decode_exchange_raw(exchange=x, new_k=None, new_v=None, rotate_k=True, rotate_v=True, advance=False,
                            query=q, k_slab=cache.key_slab, v_slab=cache.value_slab,
                            unit_stride=cache.capacity * cache._W, lengths=cache.device_lengths, units_per_seq=H,
                            len_offset=0, max_len=cache.sequence_length, units=H, group_size=G, head_dim=d,
                            bits=b, cent_k=cache._ck, cent_v=cache._cv, out=out, rotate_query=True,
                            inverse_rotate=False, signs=cache._signs, mode="tensor", workspace=cache._ws)


def _oracle_partial(cache, q):
    kw, vw = cache.packed_words()  # [layers=1, H, n, W]
    sl, sr = O.rotation_signs(d, 0)
    return O.gqa_decode(O.rotate(q, sl, sr)[None], kw[0][None], vw[0][None], cache.key_codebook.centroids,
                        cache.value_codebook.centroids, b)


def test_world1_exchange_equals_plain_decode():
    cache = _shard(1, 5000)
    x = PeerExchange(d, ROWS)  # no process group: world 1
    q = torch.randn((ROWS, d), device="cuda")
    out = torch.empty_like(q)
    for step in range(3):  # epochs 1..3 reuse both parities
        _run(cache, x, q, out)
        ref = cache.decode(query=q)
        torch.testing.assert_close(out, ref, atol=1e-6, rtol=1e-6, msg=f"step {step}")
    x.check()
    assert int(x.epoch[0]) == 3
    x.close()


def test_world2_fake_peer_merges_to_the_oracle():
    c0, c1 = _shard(2, 3000), _shard(3, 1234)
    x = _LocalExchange(world=2, rank=0, timeout_s=1.0)
    qn = np.random.default_rng(4).standard_normal((ROWS, d)).astype(np.float32)
    q = torch.from_numpy(qn).cuda()
    # the peer's side of step 1 (parity 1): its normalised partial, then its flag
    o1, l1 = _oracle_partial(c1, qn)
    slot = x.slot(0, 1, 1)
    slot[:, :d].copy_(torch.from_numpy(o1[0].astype(np.float32)))
    slot[:, d].copy_(torch.from_numpy(l1[0].astype(np.float32)))
    x.flags(0)[1].fill_(1)
    out = torch.empty_like(q)
    _run(c0, x, q, out)
    torch.cuda.synchronize()
    assert int(x.status.item()) == 0
    # oracle over the union of both shards' words
    k0, v0 = c0.packed_words()
    k1, v1 = c1.packed_words()
    sl, sr = O.rotation_signs(d, 0)
    ref, _ = O.gqa_decode(O.rotate(qn, sl, sr)[None], np.concatenate([k0[0], k1[0]], 1)[None],
                          np.concatenate([v0[0], v1[0]], 1)[None], c0.key_codebook.centroids,
                          c0.value_codebook.centroids, b)
    np.testing.assert_allclose(out.cpu().numpy(), ref[0], atol=4e-3, rtol=2e-2)
    # this rank's partial reached the peer's buffer, flagged with epoch 1
    o0, l0 = _oracle_partial(c0, qn)
    got = x.slot(1, 1, 0)
    np.testing.assert_allclose(got[:, :d].cpu().numpy(), o0[0], atol=4e-3, rtol=2e-2)
    np.testing.assert_allclose(got[:, d].cpu().numpy(), l0[0], atol=2e-2, rtol=1e-3)
    assert torch.all(x.flags(1)[0] == 1) and torch.all(x.flags(0)[0] == 1)
    assert torch.all(x.epoch == 1)


def test_peer_that_never_arrives_times_out():
    cache = _shard(5, 700)
    x = _LocalExchange(world=2, rank=0, timeout_s=0.02)  # nothing ever sets rank 1's flag
    q = torch.randn((ROWS, d), device="cuda")
    out = torch.zeros_like(q)
    _run(cache, x, q, out)
    torch.cuda.synchronize()
    assert int(x.status.item()) == _lib.TQ_E_TIMEOUT
    assert torch.isnan(out).all()
    # the context is still usable: a plain decode right after works
    ref = cache.decode(query=q)
    assert torch.isfinite(ref).all()
