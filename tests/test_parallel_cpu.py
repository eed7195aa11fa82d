"""Host-side logic of the multi-GPU partitions, run as world-size-2 gloo ranks
on CPU: the token plan, the partial exchange and the LSE merge reproduce a
single-rank decode.  (The per-rank decode here is the oracle; on GPUs it is
tq_decode and the merge is tq_lse_merge.)"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import torque_oracle as O
from torque_mlx_b200.parallel import SequencePlan, gather_partials, shard_batch


def test_shard_batch_covers_everything():
    for batch in (1, 7, 64):
        for world in (1, 2, 3, 8):
            ranges = [shard_batch(batch, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))


@pytest.mark.parametrize("last", [False, True])
@pytest.mark.parametrize("world,prefill", [(2, 10), (3, 100), (8, 131072), (4, 2)])
def test_sequence_plan_is_consistent(world, prefill, last):
    plan = SequencePlan(world=world, prefill=prefill, append_to_last=last)
    length = prefill + 23
    owners = [plan.owner(p) for p in range(length)]
    for r in range(world):
        a, b = plan.prefill_range(r)
        assert all(owners[p] == r for p in range(a, b))
        assert plan.local_count(r, length) == owners.count(r)
    if last:  # graph-captured steps: every new token lands on the last rank
        assert all(o == world - 1 for o in owners[prefill:])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        d, b, n, G = 64, 4, 301, 4
        ck, cv = O.gaussian_codebook(b, seed=0), O.gaussian_codebook(b, seed=1)
        kw = O.pack(rng.integers(0, 16, size=(n, d)), b)
        vw = O.pack(rng.integers(0, 16, size=(n, d)), b)
        qr = rng.standard_normal((G, d))
        plan = SequencePlan(world=world, prefill=250)
        mine = [p for p in range(n) if plan.owner(p) == rank]
        K = O.dequantize(O.unpack(kw[mine], b, d), ck)
        V = O.dequantize(O.unpack(vw[mine], b, d), cv)
        o, lse = O.attention_f64(qr, K, V)
        outs, lses = gather_partials(torch.from_numpy(o).float(), torch.from_numpy(lse).float())
        merged, _ = O.lse_merge(outs.numpy(), lses.numpy())
        full, _ = O.attention_f64(qr, O.dequantize(O.unpack(kw, b, d), ck), O.dequantize(O.unpack(vw, b, d), cv))
        q.put((rank, float(np.max(np.abs(merged - full)))))
    finally:
        dist.destroy_process_group()


def test_sequence_split_exchange_and_merge_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    errs = dict(q.get(timeout=5) for _ in range(world))
    assert max(errs.values()) < 1e-5, errs
