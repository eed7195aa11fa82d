"""Multi-GPU partitions of the packed-KV decode path (one process per GPU).

The reference runs on one device only; these partitions are new.

* Batch sharding (benchmark config 4): each rank owns whole sequences and runs
  the unchanged single-GPU step; there is no collective on the data path.
  ``shard_batch`` gives the rank's slice.

* Sequence sharding (benchmark config 3, long batch-1 contexts): each rank
  owns a contiguous share of the prefill tokens plus the new tokens it is
  assigned (round robin, or all on the last rank for graph-captured steps).
  With ``exchange="peer"`` (the default) a step is one ``tq_decode_exchange``
  call per rank: the rank's shard decode, then a merge kernel that stores the
  rank's normalised partial (o_r, lse_r) into every rank's exchange buffer
  over NVLink (CUDA IPC mappings, ``PeerExchange``), publishes it with a
  system-scope flag, waits (bounded) for the other ranks' flags and merges
      o = sum_r exp(lse_r - LSE) o_r  (then Pi^T)
  which equals attention over the union of the shards.  No host round trip
  and no library collective in the step; one CUDA graph per step per rank.
  ``exchange="nccl"`` keeps the all-gather variant: local decode, NCCL
  all-gather of [o_r | lse_r], ``tq_lse_merge``.

The token plan and the all-gather exchange are plain torch.distributed and are
tested on CPU with gloo ranks; the peer exchange is tested on GPUs.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def shard_batch(batch: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of the sequences rank ``rank`` owns (contiguous, sizes differ by <= 1)."""
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclass
class SequencePlan:
    """Which rank holds which token positions of one sequence: contiguous
    prefill shards, then new tokens round robin (``append_to_last=False``) or
    all on the last rank (``True``, which keeps every rank's decode step the
    same each time, so it can be captured in a CUDA graph)."""

    world: int
    prefill: int
    append_to_last: bool = False

    def prefill_range(self, rank: int) -> tuple[int, int]:
        """Contiguous share of the prefill tokens."""
        return shard_batch(self.prefill, rank, self.world)

    def owner(self, position: int) -> int:
        """Rank that stores token ``position``: the prefill shards, then round robin."""
        if position < self.prefill:
            base, extra = divmod(self.prefill, self.world)
            big = extra * (base + 1)
            return position // (base + 1) if position < big else extra + (position - big) // max(base, 1)
        if self.append_to_last:
            return self.world - 1
        return (position - self.prefill) % self.world

    def local_count(self, rank: int, length: int) -> int:
        """Tokens rank holds when the sequence is ``length`` long."""
        a, b = self.prefill_range(rank)
        n = b - a
        extra = max(0, length - self.prefill)
        if self.append_to_last:
            return n + (extra if rank == self.world - 1 else 0)
        n += extra // self.world + (1 if rank < extra % self.world else 0)
        return n


def gather_partials(out: torch.Tensor, lse: torch.Tensor, group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """All-gather every rank's normalised partial ``out [rows, d]`` and its
    ``lse [rows]``; returns ``([P, rows, d], [P, rows])``.  One collective:
    the two tensors travel as one ``[rows, d + 1]`` buffer."""
    world = dist.get_world_size(group)
    rows, d = out.shape
    buf = torch.empty((rows, d + 1), dtype=torch.float32, device=out.device)
    buf[:, :d].copy_(out)
    buf[:, d].copy_(lse)
    recv = torch.empty((world, rows, d + 1), dtype=torch.float32, device=out.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(recv, buf, group=group)
    else:
        dist.all_gather(list(recv.unbind(0)), buf, group=group)
    return recv[..., :d], recv[..., d].contiguous()


class PeerExchange:
    """The exchange buffers of a sequence-shard group (tq_exchange_* in
    include/torque_b200.h): this rank's zero-filled buffer plus CUDA IPC
    mappings of every other rank's, whose handles travel over the process
    group.  ``rows`` query rows of ``head_dim`` per step.  Set-up only: the
    step itself (``ops.decode_exchange_raw``) needs no host involvement.

    ``timeout_s`` bounds every device-side wait for a peer; a wait that gives
    up sets ``status`` (checked by :meth:`check`)."""

    def __init__(self, head_dim: int, rows: int, group=None, timeout_s: float = 1.0):
        from . import _lib
        self._lib = lib = _lib.load()
        dev = torch.device("cuda", torch.cuda.current_device())
        on = dist.is_initialized()
        self.rank = dist.get_rank(group) if on else 0
        self.world = dist.get_world_size(group) if on else 1
        self.head_dim, self.rows = head_dim, rows
        nbytes = _lib.c_size_t(0)
        _lib.check(lib.tq_exchange_buffer_bytes(head_dim, self.world, rows, _lib.ctypes.byref(nbytes)), "exchange")
        self.nbytes = int(nbytes.value)
        own = _lib.ctypes.c_void_p()
        handle = (_lib.ctypes.c_char * 64)()
        _lib.check(lib.tq_exchange_alloc(self.nbytes, _lib.ctypes.byref(own), handle), "exchange alloc")
        self._own = own.value
        got: list = [bytes(handle)]
        if self.world > 1:
            got = [None] * self.world
            dist.all_gather_object(got, bytes(handle), group=group)
        self.handle = bytes(handle)
        self._opened: list[int] = []
        ptrs = []
        for r in range(self.world):
            if r == self.rank:
                ptrs.append(self._own)
                continue
            p = _lib.ctypes.c_void_p()
            hb = (_lib.ctypes.c_char * 64).from_buffer_copy(got[r])
            _lib.check(lib.tq_exchange_open(hb, _lib.ctypes.byref(p)), "exchange open")
            self._opened.append(p.value)
            ptrs.append(p.value)
        self.bufs = torch.tensor(ptrs, dtype=torch.int64, device=dev)
        self.epoch = torch.zeros(rows, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.timeout_ns = int(timeout_s * 1e9)
        self.group = group
        if self.world > 1:
            dist.barrier(group)  # every buffer is zeroed and mapped before anyone writes

    def check(self) -> None:
        """Raise if a device wait for a peer gave up since the last check."""
        s = int(self.status.item())
        if s != 0:
            self.status.zero_()
            raise RuntimeError(f"sequence-shard exchange: a peer did not arrive within "
                               f"{self.timeout_ns / 1e9:.3g} s (status {s})")

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after a barrier, so no
        peer still writes into it)."""
        if self._own is None:
            return
        torch.cuda.synchronize()
        for p in self._opened:
            self._lib.tq_exchange_close(p)
        self._opened = []
        if self.world > 1 and dist.is_initialized():
            dist.barrier(self.group)
        self._lib.tq_exchange_free(self._own)
        self._own = None


class SequenceShardedDecoder:
    """Decode one long sequence whose packed tokens are spread over the ranks
    of ``group``.  ``cache`` is this rank's TorqueKVCache (batch 1) holding its
    share; it must be built with ``fused_weights=True`` so the local decode
    returns rotated partials — the inverse rotation runs once, after the merge,
    when ``rotate_back`` is set."""

    def __init__(self, cache, plan: SequencePlan, group=None, rotate_back: bool = True, exchange: str = "peer",
                 timeout_s: float = 1.0):
        if exchange not in ("peer", "nccl"):
            raise ValueError("exchange must be 'peer' or 'nccl'")
        if not cache.config.fused_weights:
            raise ValueError("the local shard cache must use fused_weights=True (rotated partials)")
        if cache.batch_size != 1:
            raise ValueError("sequence sharding holds one sequence per cache")
        self.cache = cache
        self.plan = plan
        self.group = group
        on = dist.is_initialized()
        self.rank = dist.get_rank(group) if on else 0
        self.world = dist.get_world_size(group) if on else 1
        self.rotate_back = rotate_back
        self.length = 0  # global sequence length
        self.exchange = exchange
        self.timeout_s = timeout_s
        self._x: PeerExchange | None = None

    # ------------------------------------------------------------ peer path
    def _peer(self, rows: int) -> PeerExchange:
        if self._x is None or self._x.rows != rows:
            if self._x is not None:
                self._x.close()
            self._x = PeerExchange(self.cache.config.head_dim, rows, self.group, self.timeout_s)
        return self._x

    def _peer_step(self, q: torch.Tensor, hq: int, k=None, v=None, *, full_capacity: bool, out: torch.Tensor):
        """tq_decode_exchange: local shard decode (+ the fused append of the new
        token when this rank owns it), peer exchange, cross-rank merge."""
        from . import ops
        c = self.cache
        cfg = c.config
        units = cfg.num_layers * cfg.kv_heads
        x = self._peer(q.shape[0])
        if k is not None:
            c._ensure_capacity(c.sequence_length + 1)
        max_len = c._cap if full_capacity else min(c._cap, c.sequence_length + (1 if k is not None else 0))
        ops.decode_exchange_raw(
            exchange=x, new_k=None if k is None else k.reshape(units, cfg.head_dim),
            new_v=None if v is None else v.to(k.dtype).reshape(units, cfg.head_dim),
            rotate_k=c.rotate_keys_on_append, rotate_v=c.rotate_values_on_append, advance=k is not None, query=q,
            k_slab=c._k, v_slab=c._v, unit_stride=c._cap * c._W, lengths=c._len_dev, units_per_seq=units,
            len_offset=1 if k is not None else 0, max_len=max_len, units=units, group_size=hq // cfg.kv_heads,
            head_dim=cfg.head_dim, bits=cfg.bit_width, cent_k=c._ck, cent_v=c._cv, out=out,
            rotate_query=c.rotate_queries_on_decode, inverse_rotate=self.rotate_back, signs=c._signs,
            mode=c.decode_mode, workspace=c._ws)

    def step(self, key, value, query):
        """One eager generation step: the owner of the next position packs the
        token inside its decode kernel, every rank decodes its shard, and the
        partials meet over the peer exchange.  Returns the merged output."""
        if self.exchange != "peer":
            self.append(key, value)
            return self.decode(query)
        c = self.cache
        q, hq, shape = c._norm_query(query)
        own = self.plan.owner(self.length) == self.rank
        k = c._norm_kv(key, "key") if own else None
        v = c._norm_kv(value, "value") if own else None
        out = torch.empty_like(q)
        self._peer_step(q, hq, k, v, full_capacity=False, out=out)
        if own:
            c._len_host += 1
        self.length += 1
        return out.reshape(shape)

    def close(self) -> None:
        """Release the exchange buffers (collective: every rank calls it)."""
        self.release()
        if self._x is not None:
            self._x.close()
            self._x = None

    def prefill(self, key, value) -> None:
        """Append this rank's share ``[layers, kv_heads, T_r, d]`` of the prefill."""
        self.cache.append(key=key, value=value)
        self.length = self.plan.prefill

    def append(self, key, value) -> None:
        """Append the next token; only its owner stores it."""
        if self.plan.owner(self.length) == self.rank:
            self.cache.append(key=key, value=value)
        self.length += 1

    def capture_step(self, key, value, query, steps_per_replay: int = 1) -> None:
        """Capture one decode step for replay; needs ``plan.append_to_last``.
        With the peer exchange, ``steps_per_replay`` > 1 captures that many
        consecutive steps in one graph (every rank must use the same count).

        Two CUDA graphs around one eager collective: ``local`` (append on the
        owning rank, local decode, partials staged into the static
        ``[rows, d + 1]`` send buffer), the NCCL all-gather issued eagerly on
        the same stream, and ``merge`` (tq_lse_merge + inverse rotation).  The
        collective stays outside the graphs so no graph holds communicator
        resources.  Inputs are copied from the example tensors."""
        if not self.plan.append_to_last:
            raise ValueError("graph capture needs SequencePlan(append_to_last=True)")
        self.steps_per_replay = 1
        if self.exchange == "peer":
            return self._capture_peer(key, value, query, steps_per_replay)
        from . import ops
        c = self.cache
        self.owner = self.rank == self.world - 1
        self._k = c._norm_kv(key, "key").clone()
        self._v = c._norm_kv(value, "value").to(self._k.dtype).clone()
        q, hq, self._qshape = c._norm_query(query)
        self._q = q.clone()
        c._ensure_capacity(c.sequence_length + 1)
        d = c.config.head_dim
        rows = self._q.shape[0]
        self._send = torch.empty((rows, d + 1), dtype=torch.float32, device=self._q.device)
        self._recv = torch.empty((self.world, rows, d + 1), dtype=torch.float32, device=self._q.device)
        inv = c.rotation if self.rotate_back else None

        def local():
            if self.owner:
                c._write(self._k, self._v)
                c._advance_device(1)
            o, s = c._decode(self._q, hq, extra=0, return_lse=True, full_capacity=True)
            self._send[:, :d].copy_(o)
            self._send[:, d].copy_(s)

        def merge():
            return ops.lse_merge(self._recv[..., :d], self._recv[..., d].contiguous(), inverse_rotation=inv)

        # size the decode workspace and warm the collective outside capture
        c._decode(self._q, hq, extra=0, return_lse=True, full_capacity=True)
        self._gather()
        torch.cuda.synchronize()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self.g_local = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.g_local, stream=side, capture_error_mode="thread_local"):
                local()
            self.g_merge = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.g_merge, stream=side, capture_error_mode="thread_local"):
                self._out = merge()
        torch.cuda.current_stream().wait_stream(side)
        assert self._out.shape == (rows, d)

    def _capture_peer(self, key, value, query, steps_per_replay: int) -> None:
        """One CUDA graph per rank holds the whole step: tq_decode_exchange
        (the last rank also packs the new token) — two kernel launches, with
        the exchange and the cross-rank merge on the device."""
        c = self.cache
        self.owner = self.rank == self.world - 1
        self._k = c._norm_kv(key, "key").clone()
        self._v = c._norm_kv(value, "value").to(self._k.dtype).clone()
        q, hq, self._qshape = c._norm_query(query)
        self._q = q.clone()
        self._out = torch.empty_like(self._q)
        c._ensure_capacity(c.sequence_length + steps_per_replay)
        k = self._k if self.owner else None
        v = self._v if self.owner else None
        self._peer(self._q.shape[0])
        # the workspace is sized outside capture; the capture itself launches nothing
        from . import ops
        cfg = c.config
        units = cfg.num_layers * cfg.kv_heads
        c._ws.get(ops.workspace_bytes(units, hq // cfg.kv_heads, cfg.head_dim, cfg.bit_width, c._cap,
                                      c.decode_mode), self._q.device)
        torch.cuda.synchronize()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self.g_step = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.g_step, stream=side, capture_error_mode="thread_local"):
                for _ in range(steps_per_replay):
                    self._peer_step(self._q, hq, k, v, full_capacity=True, out=self._out)
        torch.cuda.current_stream().wait_stream(side)
        self.g_local = self.g_merge = None
        self.steps_per_replay = steps_per_replay

    def _gather(self) -> None:
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(self._recv, self._send, group=self.group)
        else:
            dist.all_gather(list(self._recv.unbind(0)), self._send, group=self.group)

    def step_graph(self):
        """One captured step: local graph, all-gather, merge graph.  Returns
        the merged output (a static buffer, overwritten by the next step)."""
        n = self.steps_per_replay
        if self.owner and self.cache.capacity - self.cache.sequence_length < n:
            raise RuntimeError("cache capacity reached: capture again")
        if self.exchange == "peer":
            self.g_step.replay()
            if self.owner:
                self.cache._len_host += n
            self.length += n
            return self._out.reshape(self._qshape)
        self.g_local.replay()
        self._gather()
        self.g_merge.replay()
        if self.owner:
            self.cache._len_host += 1
        self.length += 1
        return self._out.reshape(self._qshape)

    def release(self) -> None:
        """Drop the captured graphs (call before destroying the process group)."""
        self.g_local = self.g_merge = self.g_step = None

    def decode(self, query):
        """Full-sequence decode: local partial -> all-gather -> LSE merge."""
        from . import ops
        if self.exchange == "peer":
            np_out = not isinstance(query, torch.Tensor)
            q, hq, shape = self.cache._norm_query(query)
            res = torch.empty_like(q)
            self._peer_step(q, hq, full_capacity=False, out=res)
            res = res.reshape(shape)
            return res.cpu().numpy() if np_out else res
        q = query if isinstance(query, torch.Tensor) else torch.as_tensor(query)
        out, lse = self.cache.decode(query=q, return_lse=True)
        shape = out.shape
        d = shape[-1]
        outs, lses = gather_partials(out.reshape(-1, d), lse.reshape(-1), self.group)
        merged = ops.lse_merge(outs, lses, inverse_rotation=self.cache.rotation if self.rotate_back else None)
        return merged.reshape(shape)


def run_sequence_split_bench(args, wl, rank: int, world: int) -> None:
    """bench.py's sequence-split mode (config 3 at N > 1): a fixed 131072-token
    context split over the ranks (strong scaling); each step appends one token
    on its owner rank and decodes across all ranks."""
    import json

    import torque_mlx_b200 as T

    dev = torch.device("cuda", torch.cuda.current_device())
    H, Hq, d, bits = wl["kv_heads"], wl["q_heads"], wl["head_dim"], wl["bits"]
    L = wl["len_lo"]
    plan = SequencePlan(world=world, prefill=L, append_to_last=True)
    a, b = plan.prefill_range(rank)
    cfg = T.TorqueConfig(bit_width=bits, head_dim=d, num_layers=1, kv_heads=H, rotation_seed=0, fused_weights=True)
    cache = T.TorqueKVCache(config=cfg, initial_capacity=(b - a) + (args.warmup + args.steps + 512
                                                                    if rank == world - 1 else 128))
    gen = torch.Generator(device=dev)
    gen.manual_seed(wl["seed"] * 7919 + rank)
    for s in range(a, b, 16384):
        n = min(16384, b - s)
        cache.append(key=torch.randn((1, H, n, d), generator=gen, device=dev, dtype=torch.float16),
                     value=torch.randn((1, H, n, d), generator=gen, device=dev, dtype=torch.float16))
    dec = SequenceShardedDecoder(cache, plan)
    dec.length = L
    ring = 8
    gen.manual_seed(17)  # identical new tokens / queries on every rank
    new_k = torch.randn((ring, 1, H, d), generator=gen, device=dev, dtype=torch.float16)
    new_v = torch.randn((ring, 1, H, d), generator=gen, device=dev, dtype=torch.float16)
    qs = torch.randn((ring, 1, Hq, d), generator=gen, device=dev, dtype=torch.float32)
    dec.capture_step(new_k[0], new_v[0], qs[0])  # per rank: local graph, all-gather, merge graph
    for _ in range(args.warmup):
        dec.step_graph()
    torch.cuda.synchronize()
    dist.barrier()
    stream = torch.cuda.current_stream()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(args.steps):
        dec.step_graph()
    s1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([s0.elapsed_time(s1)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.steps
    W = T.packed_words_for_head_dim(d, bits)
    total_bytes = (L + args.warmup + args.steps // 2) * H * 2 * W * 4
    if rank == 0:
        from pathlib import Path
        peaks = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
        peak, kind = ((float(json.loads(peaks.read_text())["hbm_gbs"]), "measured") if peaks.exists()
                      else (6650.0, "fallback"))
        achieved = total_bytes / world / (ms / 1e3) / 1e9
        print(json.dumps({
            "metric": "decode tokens/s", "value": 1.0 / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": f"u32 packed {bits}-bit codes; fp16 mma",
            "data": "synthetic (seeded fp16 N(0,1) K/V)",
            "config": {"workload": args.workload, "desc": wl["desc"], "global_batch": 1,
                       "parallelism": f"sequence-split x{world} + NCCL all-gather + LSE merge",
                       "timing": "per rank per step: CUDA graph (append on the last rank + decode), NCCL all-gather, CUDA graph (merge)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None, "peak_kind": kind,
                         "note": "per-GPU packed bytes / whole step time (decode + all-gather + merge)"},
            "gpu_launches": 5 * args.steps,
        }), flush=True)
    dec.release()
    torch.cuda.synchronize()
    dist.destroy_process_group()
