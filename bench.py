"""Benchmark of the B200 packed-KV decode path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

One step = one decode step of the workload: every sequence appends one new
token (rotate + quantize + pack of K and V for all kv heads) and attends all
query heads over its packed cache.  Default workload = benchmark config 4:
batch 64 per GPU, 32 query / 8 kv heads, head_dim 128, 3-bit codes, lengths
U{16384..32768} (seeded), fp16 N(0,1) K/V.  Multi-GPU runs shard the batch
(each rank owns 64 sequences; weak scaling, no collective on the data path).

The same JSON line also carries
  * ``seq_split``: benchmark config 3 (batch 1, 131072 tokens, 16/2 heads,
    d 256, 4-bit) with the sequence split over all N ranks: per rank one CUDA
    graph per step (tq_decode_exchange: shard decode, NVLink peer exchange of
    the partials and the cross-rank merge; the last rank packs the new
    token).  Strong scaling; at N = 1 it is the single-GPU config-3 step;
  * at N = 1, ``workloads``: the north-star shape (131072 tokens, d 128,
    32/8 heads, 4-bit), benchmark config 1 (end to end through the public
    API) and the benchmark config-2 sweep (append rows/s and GB/s of
    rotate+quantize+pack over 4096 x 8 rows x (K, V), and one decode per
    (d, bits)).

Prints ONE JSON line on rank 0.  ``--impl reference`` times the reference's
CPU algorithm (the oracle restatement of TorqueKVCache.decode) on the host
cores instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from contextlib import nullcontext
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_BYTES = 126 * 1000 * 1000  # B200 L2

WORKLOADS = {
    "config4": dict(batch=64, q_heads=32, kv_heads=8, head_dim=128, bits=3, len_lo=16384, len_hi=32768,
                    seed=4, steps=2000,
                    desc="BASELINE config 4: batched decode, batch 64/GPU x 16K-32K tokens, 32q/8kv heads, d128, "
                         "3-bit"),
    "config4_4bit": dict(batch=64, q_heads=32, kv_heads=8, head_dim=128, bits=4, len_lo=16384, len_hi=32768,
                         seed=4, steps=2000,
                         desc="config-4 geometry at 4 bits (the north-star bit width): batch 64/GPU x 16K-32K "
                              "tokens, 32q/8kv heads, d128"),
    "config3": dict(batch=1, q_heads=16, kv_heads=2, head_dim=256, bits=4, len_lo=131072, len_hi=131072, seed=3,
                    steps=3000,
                    desc="BASELINE config 3: long-context batch-1 decode, 131072 tokens, 16q/2kv heads, d256, 4-bit"),
    "config5": dict(batch=1, q_heads=16, kv_heads=8, head_dim=128, bits=4, len_lo=972, len_hi=972, seed=5,
                    steps=64, layers=28, hidden=2048, ffn=6144, vocab=151936,
                    desc="BASELINE config 5: random-init 28-layer GQA decoder (hidden 2048, 16q/8kv, d128, FFN 6144, "
                         "vocab 151936, bf16 N(0,0.02)), 4-bit packed KV with Pi folded into Wq/Wk/Wv/Wo; prefill 972 "
                         "random tokens, then generate"),
    "longctx128": dict(batch=1, q_heads=32, kv_heads=8, head_dim=128, bits=4, len_lo=131072, len_hi=131072, seed=5,
                       steps=3000,
                       desc="north-star case: batch-1 decode, 131072 tokens, 32q/8kv heads, d128, 4-bit"),
}


def _peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _traffic_ratio(workload: str):
    """DRAM bytes / algorithmic bytes of the decode kernel, from one ncu capture
    (profiles/ncu_traffic.json)."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if p.exists():
        return json.loads(p.read_text()).get(workload, {}).get("traffic_over_algorithmic")
    return None


def workload_lengths(wl: dict, rank: int) -> np.ndarray:
    rng = np.random.default_rng(wl["seed"] * 1000 + rank)
    return rng.integers(wl["len_lo"], wl["len_hi"] + 1, size=wl["batch"])


def config_dict(name: str, wl: dict, world: int) -> dict:
    """The workload description both arms print (identical for one workload and N)."""
    return {"workload": name, "desc": wl["desc"], "global_batch": wl["batch"] * world, "per_gpu_batch": wl["batch"],
            "q_heads": wl["q_heads"], "kv_heads": wl["kv_heads"], "head_dim": wl["head_dim"], "bits": wl["bits"],
            "mean_len": float(np.mean(workload_lengths(wl, 0))),
            "parallelism": f"batch-shard x{world}" if wl["batch"] > 1 else "single sequence",
            "l2": "no flush; every step reads more than 2x L2 of packed codes (caches under 2x L2 are replicated "
                  "and cycled step by step)"}


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed
    region, for the GPU named by its UUID (nvidia-smi ignores
    CUDA_VISIBLE_DEVICES, so the CUDA ordinal could name another GPU)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, cuda_index: int):
        try:
            import torch
            self.gpu = f"GPU-{torch.cuda.get_device_properties(cuda_index).uuid}"
        except Exception:  # noqa: BLE001 - fall back to the ordinal
            self.gpu = str(cuda_index)
        self.proc = None
        self.path = Path(tempfile.mkstemp(prefix="clocks_", suffix=".csv")[1])

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
            t0 = time.time()  # start timing only once the sampler is producing rows
            while time.time() - t0 < 5 and self.path.stat().st_size == 0:
                time.sleep(0.05)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self) -> dict:
        rows = []
        if self.path.exists():
            for line in self.path.read_text().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU reference arm: the reference's numpy decode algorithm (oracle restatement)
# ---------------------------------------------------------------------------
def _cpu_unit(args):
    """One (sequence, kv head) unit: unpack + dequantize every token, then the
    token-by-token streaming softmax per query head (cache.py:98-140 and
    reference.py:8-42; GQA as tests/test_cache_mlx.py:88-98)."""
    from oracle import torque_oracle as O
    kw, vw, q, ck, cv, bits, d = args
    K = O.dequantize(O.unpack(kw, bits, d), ck)
    V = O.dequantize(O.unpack(vw, bits, d), cv)
    return [O.streaming_attention_decode(qg, K, V) for qg in q]


def cpu_reference_rate(wl: dict, *, tokens: int, seqs: int, cores: int, seed: int = 0) -> tuple[float, str]:
    """Decode ``seqs`` sequences of ``tokens`` packed tokens of the workload's
    geometry on ``cores`` processes; returns (decode tokens/s scaled to the
    workload's mean length, sample description)."""
    from multiprocessing import get_context

    from oracle import torque_oracle as O
    rng = np.random.default_rng(seed)
    d, b, H, Hq = wl["head_dim"], wl["bits"], wl["kv_heads"], wl["q_heads"]
    G = Hq // H
    W = O.packed_words(d, b)
    ck, cv = O.gaussian_codebook(b, seed=0), O.gaussian_codebook(b, seed=1)
    tasks = []
    for _ in range(seqs):
        for _h in range(H):
            kw = rng.integers(0, 2**32, size=(tokens, W), dtype=np.uint64).astype(np.uint32)
            vw = rng.integers(0, 2**32, size=(tokens, W), dtype=np.uint64).astype(np.uint32)
            tasks.append((kw, vw, rng.standard_normal((G, d)).astype(np.float32), ck, cv, b, d))
    t0 = time.perf_counter()
    if cores > 1:
        with get_context("fork").Pool(cores) as pool:
            pool.map(_cpu_unit, tasks, chunksize=1)
    else:
        for t in tasks:
            _cpu_unit(t)
    dt = time.perf_counter() - t0
    mean_len = (wl["len_lo"] + wl["len_hi"]) / 2
    sample = (f"{seqs} sequence(s) x {H} kv heads x {G} q heads over {tokens} packed tokens, {cores} processes; "
              f"tokens/s scaled to the workload mean length {mean_len:.0f} (cost is linear in length)")
    return seqs / dt * (tokens / mean_len), sample


def run_reference(args, wl) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    use = max(1, min(os.cpu_count() or 1, 64))
    seqs = max(1, use // wl["kv_heads"])
    rates, sample = [], ""
    for i in range(args.warmup + args.steps):
        r, sample = cpu_reference_rate(wl, tokens=2048, seqs=seqs, cores=use, seed=i)
        if i >= args.warmup:
            rates.append(r)
    value = statistics.median(rates)
    line = {"impl": "reference", "metric": "decode tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * wl["batch"] * args.gpus / value, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32/f64", "data": "synthetic",
            "config": config_dict(args.workload, wl, args.gpus),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": use, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def build_cache(wl: dict, rank: int, torch, T, extra: int = 256, fused_weights: bool = False):
    dev = torch.device("cuda", torch.cuda.current_device())
    lens = workload_lengths(wl, rank)
    B = wl["batch"]
    cfg = T.TorqueConfig(bit_width=wl["bits"], head_dim=wl["head_dim"], num_layers=1, kv_heads=wl["kv_heads"],
                         rotation_seed=0, fused_weights=fused_weights)
    cache = T.TorqueKVCache(config=cfg, batch_size=B, initial_capacity=int(lens.max()) + extra,
                            decode_mode=wl.get("decode_mode", "auto"))
    gen = torch.Generator(device=dev)
    gen.manual_seed(wl["seed"] * 7919 + rank)
    H, d = wl["kv_heads"], wl["head_dim"]
    chunk = 16384
    for s in range(B):
        done = 0
        while done < lens[s]:
            n = int(min(chunk, lens[s] - done))
            k = torch.randn((1, H, n, d), generator=gen, device=dev, dtype=torch.float16)
            v = torch.randn((1, H, n, d), generator=gen, device=dev, dtype=torch.float16)
            cache.append_sequence(s, key=k, value=v)
            done += n
    torch.cuda.synchronize()
    return cache, lens


def _replicas(nbytes: int, cap: int = 32) -> int:
    """Copies of a cache needed so consecutive steps read more than 2x L2."""
    return 1 if nbytes >= 2 * L2_BYTES else min(cap, -(-2 * L2_BYTES // nbytes))


def time_graph_steps(torch, stream, steps_g, n_steps: int, world: int, dist=None, sampler=None):
    """Replay ``steps_g[j % R]`` n_steps times; returns (elapsed ms over the
    timed region, per-replay event ms).  Barrier + synchronize on both sides;
    ``sampler`` (a ClockSampler) records the clocks during the timed region."""
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with sampler if sampler is not None else nullcontext():
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for j in range(n_steps):
            ev[j][0].record(stream)
            steps_g[j % len(steps_g)]()
            ev[j][1].record(stream)
        end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    return start.elapsed_time(end), [a.elapsed_time(b) for a, b in ev]


def max_over_ranks(torch, dist, world: int, x: float) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def measure_batch(torch, T, wl: dict, steps: int, warmup: int, rank: int, world: int, dist=None,
                  sampler=None, unroll: int = 0) -> dict:
    """The fused step graph (tq_decode_append + split merge) over a batch cache."""
    cache, lens = build_cache(wl, rank, torch, T, extra=warmup + steps + 640)
    B, Hq, H, d, bits = wl["batch"], wl["q_heads"], wl["kv_heads"], wl["head_dim"], wl["bits"]
    W = T.packed_words_for_head_dim(d, bits)
    cache_bytes = int(np.sum(lens)) * H * 2 * W * 4
    reps = _replicas(cache_bytes)
    caches = [cache] + [build_cache(wl, rank, torch, T, extra=warmup + steps + 640)[0] for _ in range(reps - 1)]
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev)
    gen.manual_seed(rank + 17)
    ring = 8  # distinct new-token / query sets, reused round robin
    new_k = torch.randn((ring, B, 1, H, d), generator=gen, device=dev, dtype=torch.float16)
    new_v = torch.randn((ring, B, 1, H, d), generator=gen, device=dev, dtype=torch.float16)
    qs = torch.randn((ring, B, 1, Hq, d), generator=gen, device=dev, dtype=torch.float32)

    def kv(t):  # batch 1 uses the reference's [layers, kv_heads, d] step form
        return t if B > 1 else t[0]

    # Short steps (batch 1) are captured U to a graph, so the host's replay rate
    # does not bound them; every replay still runs U complete fused steps.
    U = unroll if unroll else (8 if B == 1 else 1)
    graphs = [c.capture_step(key=kv(new_k[0]), value=kv(new_v[0]), query=kv(qs[0]), steps_per_replay=U)
              for c in caches]
    for i in range(max(1, warmup // U)):
        graphs[i % reps].step()
    torch.cuda.synchronize()
    start_lens = [int(c.lengths.sum()) for c in caches]
    stream = torch.cuda.current_stream()
    n_rep = max(1, steps // U)
    elapsed, rep_ms = time_graph_steps(torch, stream, [g.step for g in graphs], n_rep, world, dist, sampler)
    elapsed = max_over_ranks(torch, dist, world, elapsed)  # covers n_rep * U steps
    dec_ms = [t / U for t in rep_ms]
    # attended bytes per step (including the appended token)
    alg = [(start_lens[j % reps] + B * ((j // reps) * U + k + 1)) * H * 2 * W * 4 for j in range(n_rep)
           for k in range(U)]
    return dict(cache=caches, graphs=graphs, lens=lens, reps=reps, cache_bytes=cache_bytes, elapsed_ms=elapsed,
                dec_ms=dec_ms, alg_bytes=alg, new_k=new_k, new_v=new_v, qs=qs, kv=kv, unroll=U, n_steps=n_rep * U)


def e2e_public_api(torch, dist, world: int, m: dict, steps: int) -> tuple[float, int, int]:
    """Serving-style loop through the public API: each step's new K/V and
    queries start in pinned host memory and are copied to the device, one
    fused ``append_decode`` call appends and attends, and the output is
    copied back to pinned memory and waited for.  Returns (ms per step, H2D
    bytes, D2H bytes)."""
    new_k, new_v, qs, kv, caches = m["new_k"], m["new_v"], m["qs"], m["kv"], m["cache"]
    hk, hv, hq = new_k.cpu().pin_memory(), new_v.cpu().pin_memory(), qs.cpu().pin_memory()
    dk, dv, dq = torch.empty_like(new_k[0]), torch.empty_like(new_v[0]), torch.empty_like(qs[0])
    host_out = torch.empty(qs[0].shape, dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for j in range(steps):
        r = j % hk.shape[0]
        dk.copy_(hk[r], non_blocking=True)  # host -> device
        dv.copy_(hv[r], non_blocking=True)
        dq.copy_(hq[r], non_blocking=True)
        res = caches[j % len(caches)].append_decode(key=kv(dk), value=kv(dv), query=kv(dq))
        host_out.copy_(res.reshape(host_out.shape), non_blocking=True)  # device -> host
        stream.synchronize()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(torch, dist, world, e0.elapsed_time(e1)) / steps
    h2d = int(hk[0].numel() * 2 + hv[0].numel() * 2 + hq[0].numel() * 4)
    return ms, h2d, int(host_out.numel() * 4)


def e2e_captured_step(torch, dist, world: int, m: dict, steps: int) -> float:
    """Serving loop through the captured-step API (CapturedDecodeStep.run):
    each step's new K/V and queries are copied from pinned host memory into
    the step's input buffers, one graph replay appends and attends, and the
    output is copied back to pinned memory and waited for.  Returns ms/step."""
    new_k, new_v, qs = m["new_k"], m["new_v"], m["qs"]
    graphs = m["graphs"] if m["unroll"] == 1 else None
    if graphs is None:
        return float("nan")
    hk, hv, hq = new_k.cpu().pin_memory(), new_v.cpu().pin_memory(), qs.cpu().pin_memory()
    host_out = torch.empty(qs[0].shape, dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for j in range(steps):
        r = j % hk.shape[0]
        out = graphs[j % len(graphs)].run(key=hk[r], value=hv[r], query=hq[r])  # host -> device, replay
        host_out.copy_(out.reshape(host_out.shape), non_blocking=True)        # device -> host
        stream.synchronize()
    e1.record(stream)
    torch.cuda.synchronize()
    return max_over_ranks(torch, dist, world, e0.elapsed_time(e1)) / steps


def measure_seq_split(torch, T, dist, steps: int, warmup: int, rank: int, world: int) -> dict:
    """Benchmark config 3 with the 131072-token sequence split over the ranks
    (strong scaling).  Each rank's shard is replicated until consecutive steps
    read more than 2x L2 per GPU; the replicas are separate decoders whose
    graphs are cycled step by step."""
    from torque_mlx_b200.parallel import SequencePlan, SequenceShardedDecoder

    wl = WORKLOADS["config3"]
    dev = torch.device("cuda", torch.cuda.current_device())
    H, Hq, d, bits, L = wl["kv_heads"], wl["q_heads"], wl["head_dim"], wl["bits"], wl["len_lo"]
    W = T.packed_words_for_head_dim(d, bits)
    plan = SequencePlan(world=world, prefill=L, append_to_last=True)
    a, b = plan.prefill_range(rank)
    shard_bytes = (b - a) * H * 2 * W * 4
    # every rank must use the same replica count (they step together)
    smallest = min(plan.prefill_range(r)[1] - plan.prefill_range(r)[0] for r in range(world))
    reps = _replicas(smallest * H * 2 * W * 4)
    cfg = T.TorqueConfig(bit_width=bits, head_dim=d, num_layers=1, kv_heads=H, rotation_seed=0, fused_weights=True)
    gen = torch.Generator(device=dev)
    decs = []
    per_rep_steps = (warmup + steps) // reps + 2
    for rep in range(reps):
        cache = T.TorqueKVCache(config=cfg, initial_capacity=(b - a) + (per_rep_steps + 256
                                                                        if rank == world - 1 else 128))
        gen.manual_seed(wl["seed"] * 7919 + rank * 101 + rep)
        for s in range(a, b, 16384):
            n = min(16384, b - s)
            cache.append(key=torch.randn((1, H, n, d), generator=gen, device=dev, dtype=torch.float16),
                         value=torch.randn((1, H, n, d), generator=gen, device=dev, dtype=torch.float16))
        dec = SequenceShardedDecoder(cache, plan, exchange="peer", timeout_s=5.0)
        dec.length = L
        decs.append(dec)
    gen.manual_seed(17)  # identical new token / query on every rank
    new_k = torch.randn((1, H, d), generator=gen, device=dev, dtype=torch.float16)
    new_v = torch.randn((1, H, d), generator=gen, device=dev, dtype=torch.float16)
    q = torch.randn((1, Hq, d), generator=gen, device=dev, dtype=torch.float32)
    U = 8  # steps per graph replay (same on every rank)
    for dec in decs:
        dec.capture_step(new_k, new_v, q, steps_per_replay=U)
    if world > 1:
        dist.barrier()
    for i in range(max(1, warmup // U)):
        decs[i % reps].step_graph()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    n_rep = max(1, steps // U)
    elapsed, _ = time_graph_steps(torch, stream, [dec.step_graph for dec in decs], n_rep, world, dist)
    for dec in decs:
        dec._x.check()
    elapsed = max_over_ranks(torch, dist, world, elapsed)
    ms = elapsed / (n_rep * U)
    peak, kind = _peaks()
    per_gpu = shard_bytes / (ms / 1e3) / 1e9
    res = {"workload": "config3", "desc": wl["desc"] + f"; sequence split over {world} GPU(s)",
           "n_gpus": world, "ms_per_step": ms, "tokens_per_s": 1e3 / ms, "scaling": "strong",
           "parallelism": f"sequence-split x{world}: tq_decode_exchange (shard decode + NVLink peer exchange + "
                          "cross-rank LSE merge, one CUDA graph per step per rank)",
           "per_gpu_packed_bytes": shard_bytes, "per_gpu_gbs": per_gpu, "hbm_frac": per_gpu / peak,
           "peak": peak, "peak_kind": kind,
           "l2": (f"{reps} replica(s) of the {shard_bytes / 1e6:.1f} MB shard per GPU cycled step by step"
                  if reps > 1 else "shard larger than 2x L2"),
           "gpu_launches": 2 * n_rep * U, "steps_per_graph_replay": U}
    for dec in decs:
        dec.close()
    return res


def measure_config2(torch, T, steps: int = 20) -> dict:
    """Benchmark config 2: append (rotate + quantize + pack) throughput over
    4096 x 8 rows of K and of V, and one packed decode (32 query heads) per
    (d, bits); fp16 N(0,1) K/V with 1% of the channels x20."""
    from torque_mlx_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    peak, _ = _peaks()
    out = {}
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)

    def timed(fn):
        times = []
        for i in range(steps + 3):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            if i >= 3:
                times.append(e0.elapsed_time(e1))
        return statistics.median(times)

    for d in (64, 128, 256):
        for bits in (2, 3, 4):
            H, L, Hq = 8, 4096, 32
            W = T.packed_words_for_head_dim(d, bits)
            gen = torch.Generator(device=dev).manual_seed(d * 10 + bits)
            scale = torch.ones(d, device=dev, dtype=torch.float16)
            ch = np.random.default_rng(d + bits).choice(d, size=max(1, d // 100), replace=False)
            scale[torch.as_tensor(ch, device=dev)] = 20.0
            k = torch.randn((1, H, L, d), generator=gen, device=dev, dtype=torch.float16) * scale
            v = torch.randn((1, H, L, d), generator=gen, device=dev, dtype=torch.float16) * scale
            cfg = T.TorqueConfig(bit_width=bits, head_dim=d, num_layers=1, kv_heads=H, fused_weights=True)
            cache = T.TorqueKVCache(config=cfg, initial_capacity=L)
            cache.append(key=k, value=v)
            sl, sr = cache._signs
            st = _lib.stream_ptr()

            def append():
                _lib.check(lib.tq_append_kv(k.data_ptr(), v.data_ptr(), _lib.TQ_F16, H, L, d, bits, sl.data_ptr(),
                                            sr.data_ptr(), 1, cache._ck.data_ptr(), cache._cv.data_ptr(),
                                            cache._k.data_ptr(), cache._v.data_ptr(), cache._cap * W, cache._cap,
                                            None, 1, 0, st), "append")

            ms = timed(append)
            rows = 2 * H * L
            abytes = rows * (2 * d + 4 * W)
            q = torch.randn((Hq, d), generator=gen, device=dev)
            dms = timed(lambda: cache.decode(query=q))
            dbytes = L * H * 2 * W * 4
            out[f"d{d}_b{bits}"] = {
                "append_rows_per_s": rows / (ms / 1e3), "append_gbs": abytes / (ms / 1e3) / 1e9,
                "append_hbm_frac": abytes / (ms / 1e3) / 1e9 / peak, "append_us": ms * 1e3,
                "decode_us": dms * 1e3, "decode_packed_gbs": dbytes / (dms / 1e3) / 1e9}
    return {"desc": "BASELINE config 2: 4096 tokens x 8 kv heads, K and V rotate+quantize+pack (bytes = rows x "
                    "(2d fp16 in + 4W out)), then one decode with 32 query heads (eager public API, L2 flushed "
                    "before each timed launch)", "shapes": out}


def measure_config1(torch, T) -> dict:
    """Benchmark config 1 end to end through the public API: numpy K/V of 512
    tokens appended step by step, then one decode, host result."""
    rng = np.random.default_rng(0)
    keys = rng.standard_normal((512, 8, 128)).astype(np.float16)
    vals = rng.standard_normal((512, 8, 128)).astype(np.float16)
    qry = rng.standard_normal((8, 128)).astype(np.float32)
    cfg = T.TorqueConfig(bit_width=4, head_dim=128, kv_heads=8)
    times = []
    out = None
    for _ in range(3):
        cache = T.TorqueKVCache(config=cfg, initial_capacity=512)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for t in range(512):
            cache.append(key=keys[t], value=vals[t])
        t1 = time.perf_counter()
        out = cache.decode(query=qry)  # numpy in -> numpy out (synchronises)
        t2 = time.perf_counter()
        times.append((t1 - t0, t2 - t1))
    return {"desc": "BASELINE config 1: batch 1, 512 tokens, 8/8 heads, d128, 4-bit; numpy K/V appended token by "
                    "token through TorqueKVCache.append, then one .decode (host in, host out)",
            "append_ms_per_token": min(t[0] for t in times) / 512 * 1e3,
            "decode_ms": min(t[1] for t in times) * 1e3, "checksum": float(out.sum())}


def _step_summary(m: dict, wl: dict, peak: float) -> dict:
    ms = statistics.mean(m["dec_ms"])
    byts = statistics.mean(m["alg_bytes"])
    step_ms = m["elapsed_ms"] / m["n_steps"]
    return {"desc": wl["desc"], "ms_per_step": step_ms, "tokens_per_s": wl["batch"] / (step_ms / 1e3),
            "packed_kv_gbs": byts / (ms / 1e3) / 1e9, "hbm_frac": byts / (ms / 1e3) / 1e9 / peak,
            "l2": f"{m['reps']} replica(s) cycled" if m["reps"] > 1 else "cache larger than 2x L2"}


def run_decoder(args, wl) -> None:
    """Config 5: greedy generation with the whole token step in one CUDA graph."""
    import torch

    from torque_mlx_b200.decoder import DecoderConfig, PackedKVDecoder

    torch.cuda.set_device(0)
    cfg = DecoderConfig(num_layers=wl["layers"], hidden=wl["hidden"], q_heads=wl["q_heads"], kv_heads=wl["kv_heads"],
                        head_dim=wl["head_dim"], ffn=wl["ffn"], vocab=wl["vocab"], bits=wl["bits"], fold="full")
    model = PackedKVDecoder(cfg, max_tokens=wl["len_lo"] + args.warmup + 2 * args.steps + 64)
    prompt = torch.randint(0, cfg.vocab, (wl["len_lo"],), generator=torch.Generator().manual_seed(wl["seed"]))
    tok = model.prefill(prompt.cuda()).argmax(-1).reshape(())
    model.capture()
    for _ in range(args.warmup):
        tok = model.step_graph(tok).clone()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    with ClockSampler(0) as clocks:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            tok = model.step_graph(tok)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    # end to end: eager public API, generated token read back to the host every step
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ids = []
    for _ in range(min(args.steps, 16)):
        tok = model.step(tok).argmax(-1).reshape(())
        ids.append(int(tok.item()))
    e2e_ms = (time.perf_counter() - t0) * 1e3 / len(ids)
    weight_bytes = sum(t.numel() * t.element_size() for lay in model.layers for t in lay.values()) + \
        model.lm_head.numel() * 2
    peak, kind = _peaks()
    print(json.dumps({
        "metric": "decode tokens/s", "value": 1e3 / ms, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 weights; u32 packed 4-bit KV", "data": "synthetic (random-init weights, random prompt tokens)",
        "config": {"workload": "config5", "desc": wl["desc"], "global_batch": 1, "prompt": wl["len_lo"],
                   "parallelism": "single GPU", "timing": "one CUDA graph per generated token"},
        "roofline": {"bound": "hbm", "achieved": weight_bytes / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": weight_bytes / (ms / 1e3) / 1e9 / peak, "traffic": None, "peak_kind": kind,
                     "note": "bf16 weight stream per token (packed KV is ~29 MB of it)"},
        "e2e": {"value": 1e3 / e2e_ms, "unit": "tokens/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8},
        "gpu_launches": None, "clocks": clocks.summary()}), flush=True)


def run_ours(args, wl) -> None:
    import torch
    import torch.distributed as dist

    import torque_mlx_b200 as T

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        # a stuck peer ends the run with an error instead of the 10-minute default wait
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=180))

    B, H, bits = wl["batch"], wl["kv_heads"], wl["bits"]
    clocks = ClockSampler(local)
    m = measure_batch(torch, T, wl, args.steps, args.warmup, rank, world, dist, sampler=clocks)
    value = B * world / (m["elapsed_ms"] / 1e3 / m["n_steps"])
    e2e_steps = max(3, min(args.steps, 200))
    cap_ms = e2e_captured_step(torch, dist, world, m, e2e_steps)
    e2e_ms, h2d, d2h = e2e_public_api(torch, dist, world, m, e2e_steps)
    eager_value = B * world / (e2e_ms / 1e3)
    e2e_value = B * world / (cap_ms / 1e3) if cap_ms == cap_ms else eager_value
    seq = None
    if not args.no_seq_split:
        try:
            seq = measure_seq_split(torch, T, dist, args.seq_steps, args.warmup, rank, world)
        except Exception as exc:  # noqa: BLE001 - the batch-shard line stands on its own
            seq = {"workload": "config3", "n_gpus": world, "error": f"{type(exc).__name__}: {exc}"[:300]}
            torch.cuda.synchronize()
    extra = {}
    if world == 1 and not args.no_extra:
        peak, _ = _peaks()
        w2 = WORKLOADS["longctx128"]
        extra["longctx128"] = _step_summary(measure_batch(torch, T, w2, 1000, args.warmup, 0, 1), w2, peak)
        extra["config2"] = measure_config2(torch, T)
        extra["config1"] = measure_config1(torch, T)

    if rank == 0:
        peak, peak_kind = _peaks()
        mean_dec_ms = statistics.mean(m["dec_ms"])
        mean_bytes = statistics.mean(m["alg_bytes"])
        achieved = mean_bytes / (mean_dec_ms / 1e3) / 1e9
        ratio = _traffic_ratio(args.workload)
        line = {
            "metric": "decode tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": m["elapsed_ms"] / m["n_steps"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": f"u32 packed {bits}-bit codes; fp16 mma, fp32 softmax/accumulate",
            "data": "synthetic (seeded fp16 N(0,1) K/V and fp32 queries generated on device)",
            "config": config_dict(args.workload, wl, world),
            "l2_detail": ("no flush; inputs larger than L2 (packed cache %.2f GB per GPU)" % (mean_bytes / 1e9))
            if m["reps"] == 1 else
            ("no flush; %d replicas of the %.0f MB cache cycled step by step" % (m["reps"], m["cache_bytes"] / 1e6)),
            "packed_kv_gbs": achieved,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": (ratio * mean_bytes) if ratio else None,
                         "traffic_note": "ncu DRAM bytes / algorithmic bytes of decode_mma_kernel (one capture, "
                                         "profiles/ncu_traffic.json) x this launch's algorithmic bytes",
                         "kernel": "tq_decode_append (decode_mma_kernel packing the new token + "
                                   "merge_partials_kernel)", "peak_kind": peak_kind,
                         "bytes_per_launch": mean_bytes, "launch_ms": mean_dec_ms},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "call": "CapturedDecodeStep.run (the serving form of the captured fused step): each step's "
                            "new K/V and queries copied in from pinned host memory, one graph replay, the output "
                            "copied back to pinned memory and waited for",
                    "eager_append_decode": {"value": eager_value, "unit": "tokens/s",
                                            "call": "TorqueKVCache.append_decode with the same host copies"}},
            "gpu_launches": 2 * m["n_steps"],
            "timing": "device loop = CUDA-graph replay of the fused step (tq_decode_append: append packed inside "
                      "the decode kernel, then the split merge), CUDA events, max over ranks",
            "clocks": clocks.summary(),
        }
        if seq is not None:
            line["seq_split"] = seq
        if extra:
            line["workloads"] = extra
        if world == 1 and not args.no_cpu_baseline:
            cores = max(1, min(os.cpu_count() or 1, 64))
            rate, sample = cpu_reference_rate(wl, tokens=2048, seqs=max(1, cores // H), cores=cores)
            line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port",
                                    "sample": sample}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_single(args, wl) -> None:
    """A batch-1 workload on one GPU through the cached step graph
    (longctx128, config 3 without the split)."""
    import torch

    import torque_mlx_b200 as T
    torch.cuda.set_device(0)
    peak, kind = _peaks()
    clocks = ClockSampler(0)
    m = measure_batch(torch, T, wl, args.steps, args.warmup, 0, 1, sampler=clocks)
    s = _step_summary(m, wl, peak)
    print(json.dumps({"metric": "decode tokens/s", "value": s["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1,
                      "steps": m["n_steps"], "steps_per_graph_replay": m["unroll"], "warmup": args.warmup, "ms_per_step": s["ms_per_step"],
                      "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                      "config": config_dict(args.workload, wl, 1),
                      "roofline": {"bound": "hbm", "achieved": s["packed_kv_gbs"], "peak": peak, "unit": "GB/s",
                                   "frac": s["hbm_frac"], "peak_kind": kind,
                                   "launch_ms": statistics.mean(m["dec_ms"])},
                      "l2_detail": s["l2"], "gpu_launches": 2 * m["n_steps"], "clocks": clocks.summary()}),
          flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: about a second of timed work for the workload)")
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default="config4", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-seq-split", action="store_true", help="skip the config-3 sequence-split keys")
    ap.add_argument("--no-extra", action="store_true", help="skip the extra N=1 workloads")
    ap.add_argument("--seq-steps", type=int, default=3000)
    ap.add_argument("--batch", type=int, default=None, help="override the per-GPU batch (small profiling cases)")
    ap.add_argument("--decode-mode", default="auto", choices=["auto", "tensor", "exact"],
                    help="decode kernel (exact: the fp32 CUDA-core kernel, for the tensor-core comparison)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    wl = dict(WORKLOADS[args.workload])
    if args.batch:
        wl["batch"] = args.batch
    wl["decode_mode"] = args.decode_mode
    if args.steps is None:
        args.steps = wl["steps"] if args.impl == "ours" else 5
    if args.impl == "reference":
        run_reference(args, wl)
    elif args.workload == "config5":
        run_decoder(args, wl)
    elif wl["batch"] == 1:
        run_single(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
