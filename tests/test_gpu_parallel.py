"""Sequence-sharded decode on the GPU path (NCCL process group; one rank per
visible GPU up to 2, each rank a child process).  With one GPU the group has
one rank and the test still runs the exchange and tq_lse_merge."""

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


def _worker(rank, world, port, q):
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
        dec = SequenceShardedDecoder(T.TorqueKVCache(config=cfg), plan)
        dec.prefill(keys[:, a:b], vals[:, a:b])
        for t in range(n, n + extra):
            dec.append(keys[:, t], vals[:, t])
        got = dec.decode(torch.from_numpy(qry).cuda()).cpu().numpy()
        full = T.TorqueKVCache(config=T.TorqueConfig(bit_width=4, head_dim=d, kv_heads=H))
        full.append(key=keys, value=vals)
        ref = full.decode(query=qry)
        err = float(np.max(np.abs(got - ref)))
        # graph-captured steps with new tokens on the last rank
        plan2 = SequencePlan(world=world, prefill=n, append_to_last=True)
        dec2 = SequenceShardedDecoder(T.TorqueKVCache(config=cfg), plan2)
        dec2.prefill(keys[:, a:b], vals[:, a:b])
        kt = torch.from_numpy(keys[:, n]).cuda()
        vt = torch.from_numpy(vals[:, n]).cuda()
        dec2.capture_step(kt, vt, torch.from_numpy(qry).cuda())
        got2 = dec2.step_graph().cpu().numpy()
        full2 = T.TorqueKVCache(config=T.TorqueConfig(bit_width=4, head_dim=d, kv_heads=H))
        full2.append(key=keys[:, :n + 1], value=vals[:, :n + 1])
        err = max(err, float(np.max(np.abs(got2 - full2.decode(query=qry)))))
        dec2.release()
        torch.cuda.synchronize()
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


def test_sequence_sharded_decode_matches_single_rank():
    import torch.multiprocessing as mp

    world = min(2, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, qu)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        for p in procs:
            p.join(timeout=180)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    errs = dict(qu.get(timeout=5) for _ in range(world))
    assert max(errs.values()) < 2e-4, errs
