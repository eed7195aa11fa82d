"""Sequence-sharded decode on the GPU path, one rank per visible GPU (up to 4),
each rank a child process with an NCCL process group (used for set-up and,
with exchange="nccl", for the all-gather).  With one GPU the group has one
rank and the test still runs the exchange kernels.

Checked against the float64 oracle over the packed words of a single cache
that holds every token (the shards' words are the same words: the append is
bit-exact), after eager round-robin steps and after captured steps that append
on the last rank.  NVLS is off, as for every multi-rank test here."""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle(full, qry):
    from oracle import torque_oracle as O
    cfg = full.config
    kw, vw = full.packed_words()
    sl, sr = O.rotation_signs(cfg.head_dim, cfg.rotation_seed)
    o, _ = O.gqa_decode(O.rotate(qry, sl, sr)[None], kw[0][None], vw[0][None], full.key_codebook.centroids,
                        full.value_codebook.centroids, cfg.bit_width)
    return O.rotate_inverse(o[0].astype(np.float32), sl, sr)


def _worker(rank, world, port, exchange, q):
    import torch.distributed as dist

    import torque_mlx_b200 as T
    from torque_mlx_b200.parallel import SequencePlan, SequenceShardedDecoder

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=timedelta(seconds=60))
    try:
        rng = np.random.default_rng(5)
        H, G, d, n, extra = 2, 8, 256, 3000, 5
        keys = rng.standard_normal((H, n + extra, d)).astype(np.float16)
        vals = rng.standard_normal((H, n + extra, d)).astype(np.float16)
        qry = rng.standard_normal((H * G, d)).astype(np.float32)
        plan = SequencePlan(world=world, prefill=n)
        a, b = plan.prefill_range(rank)
        cfg = T.TorqueConfig(bit_width=4, head_dim=d, kv_heads=H, fused_weights=True)
        dec = SequenceShardedDecoder(T.TorqueKVCache(config=cfg), plan, exchange=exchange)
        dec.prefill(keys[:, a:b], vals[:, a:b])
        errs = []
        full = T.TorqueKVCache(config=T.TorqueConfig(bit_width=4, head_dim=d, kv_heads=H))
        full.append(key=keys[:, :n], value=vals[:, :n])
        for t in range(n, n + extra):  # eager steps, new tokens round robin
            got = dec.step(keys[:, t], vals[:, t], torch.from_numpy(qry).cuda()).cpu().numpy()
            full.append(key=keys[:, t], value=vals[:, t])
            errs.append(float(np.max(np.abs(got - _oracle(full, qry)))))
        got = dec.decode(torch.from_numpy(qry).cuda()).cpu().numpy()
        errs.append(float(np.max(np.abs(got - _oracle(full, qry)))))
        if exchange == "peer":
            dec._x.check()
        dec.close()
        # graph-captured steps with new tokens on the last rank
        plan2 = SequencePlan(world=world, prefill=n, append_to_last=True)
        dec2 = SequenceShardedDecoder(T.TorqueKVCache(config=cfg), plan2, exchange=exchange)
        dec2.prefill(keys[:, a:b], vals[:, a:b])
        kt = torch.from_numpy(keys[:, n]).cuda()
        vt = torch.from_numpy(vals[:, n]).cuda()
        dec2.capture_step(kt, vt, torch.from_numpy(qry).cuda())
        full2 = T.TorqueKVCache(config=T.TorqueConfig(bit_width=4, head_dim=d, kv_heads=H))
        full2.append(key=keys[:, :n], value=vals[:, :n])
        for _ in range(3):  # the captured token is appended again each step
            got2 = dec2.step_graph().cpu().numpy()
            full2.append(key=keys[:, n], value=vals[:, n])
            errs.append(float(np.max(np.abs(got2 - _oracle(full2, qry)))))
        if exchange == "peer":
            dec2._x.check()
        dec2.close()
        torch.cuda.synchronize()
        q.put((rank, max(errs)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["peer", "nccl"])
def test_sequence_sharded_decode_matches_oracle(exchange):
    import torch.multiprocessing as mp

    world = min(4, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, exchange, qu)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        for p in procs:
            p.join(timeout=240)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    errs = dict(qu.get(timeout=5) for _ in range(world))
    # tensor-mode decode (fp16 operands) against the float64 oracle
    assert max(errs.values()) < 4e-3, errs


def test_one_process_two_devices():
    """One process decoding on two GPUs in turn: the kernels' shared-memory
    opt-in and occupancy are per device, so the second device's launches are
    as valid as the first's (needs two visible GPUs)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torque_mlx_b200 as T
    from oracle import torque_oracle as O

    rng = np.random.default_rng(2)
    keys = rng.standard_normal((2, 3000, 128)).astype(np.float16)
    vals = rng.standard_normal((2, 3000, 128)).astype(np.float16)
    qry = rng.standard_normal((8, 128)).astype(np.float32)
    outs = []
    for dev in (0, 1, 0):
        with torch.cuda.device(dev):
            cache = T.TorqueKVCache(config=T.TorqueConfig(bit_width=4, head_dim=128, kv_heads=2),
                                    decode_mode="tensor")
            cache.append(key=keys, value=vals)
            outs.append(cache.decode(query=qry))
            if dev == 1:
                kw, vw = cache.packed_words()
                sl, sr = O.rotation_signs(128, 0)
                o, _ = O.gqa_decode(O.rotate(qry, sl, sr)[None], kw[0][None], vw[0][None],
                                    cache.key_codebook.centroids, cache.value_codebook.centroids, 4)
                np.testing.assert_allclose(outs[-1], O.rotate_inverse(o[0].astype(np.float32), sl, sr),
                                           atol=4e-3, rtol=2e-2)
    np.testing.assert_array_equal(outs[0], outs[1])
    np.testing.assert_array_equal(outs[0], outs[2])
