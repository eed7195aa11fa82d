"""Benchmark of the B200 packed-KV decode path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

One step = one decode step of the workload: every sequence appends one new
token (rotate + quantize + pack of K and V for all kv heads) and attends all
query heads over its packed cache.  Default workload = benchmark config 4:
batch 64 per GPU, 32 query / 8 kv heads, head_dim 128, 3-bit codes, lengths
U{16384..32768} (seeded), fp16 N(0,1) K/V.  Multi-GPU runs shard the batch
(each rank owns 64 sequences; weak scaling, no collective on the data path).
``--workload config3`` runs benchmark config 3 (batch 1, 16/2 heads, d 256,
4-bit, 131072-token context; N>1 splits the sequence across ranks and merges
with an NCCL all-gather + LSE merge).

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
                    steps=5000,
                    desc="BASELINE config 3: long-context batch-1 decode, 131072 tokens, 16q/2kv heads, d256, 4-bit"),
    "config5": dict(batch=1, q_heads=16, kv_heads=8, head_dim=128, bits=4, len_lo=972, len_hi=972, seed=5,
                    steps=64, layers=28, hidden=2048, ffn=6144, vocab=151936,
                    desc="BASELINE config 5: random-init 28-layer GQA decoder (hidden 2048, 16q/8kv, d128, FFN 6144, "
                         "vocab 151936, bf16 N(0,0.02)), 4-bit packed KV with Pi folded into Wq/Wk/Wv/Wo; prefill 972 "
                         "random tokens, then generate"),
    "longctx128": dict(batch=1, q_heads=32, kv_heads=8, head_dim=128, bits=4, len_lo=131072, len_hi=131072, seed=5,
                       steps=5000,
                       desc="north-star case: batch-1 decode, 131072 tokens, 32q/8kv heads, d128, 4-bit"),
}


def _peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _traffic(workload: str):
    p = ROOT / "profiles" / "ncu_traffic.json"
    if p.exists():
        return json.loads(p.read_text()).get(workload)
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
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
            "config": {"workload": args.workload, "desc": wl["desc"], "global_batch": wl["batch"] * args.gpus},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": use, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def build_cache(wl: dict, rank: int, torch, T, extra: int = 256):
    dev = torch.device("cuda", torch.cuda.current_device())
    rng = np.random.default_rng(wl["seed"] * 1000 + rank)
    B = wl["batch"]
    lens = rng.integers(wl["len_lo"], wl["len_hi"] + 1, size=B)
    cfg = T.TorqueConfig(bit_width=wl["bits"], head_dim=wl["head_dim"], num_layers=1, kv_heads=wl["kv_heads"],
                         rotation_seed=0)
    cache = T.TorqueKVCache(config=cfg, batch_size=B, initial_capacity=int(lens.max()) + extra)
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
    if wl["batch"] == 1 and world > 1:
        from torque_mlx_b200.parallel import run_sequence_split_bench
        run_sequence_split_bench(args, wl, rank, world)
        return

    cache, lens = build_cache(wl, rank, torch, T, extra=args.warmup + args.steps + 512)
    B, Hq, H, d, bits = wl["batch"], wl["q_heads"], wl["kv_heads"], wl["head_dim"], wl["bits"]
    W = T.packed_words_for_head_dim(d, bits)
    # A cache smaller than 2x L2 is replicated and the replicas are cycled,
    # so every step reads codes that the previous steps evicted from L2.
    cache_bytes = int(np.sum(lens)) * H * 2 * W * 4
    reps = 1 if cache_bytes >= 2 * L2_BYTES else -(-2 * L2_BYTES // cache_bytes)
    caches = [cache] + [build_cache(wl, rank, torch, T, extra=args.warmup + args.steps + 512)[0]
                        for _ in range(reps - 1)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(rank + 17)
    ring = 8  # distinct new-token / query sets, reused round robin
    new_k = torch.randn((ring, B, 1, H, d), generator=gen, device=dev, dtype=torch.float16)
    new_v = torch.randn((ring, B, 1, H, d), generator=gen, device=dev, dtype=torch.float16)
    qs = torch.randn((ring, B, 1, Hq, d), generator=gen, device=dev, dtype=torch.float32)

    def kv(t):  # batch 1 uses the reference's [layers, kv_heads, d] step form
        return t if B > 1 else t[0]

    # device-timed loop: the step replayed from CUDA graphs (no host launch gaps)
    steps_g = [c.capture_step(key=kv(new_k[0]), value=kv(new_v[0]), query=kv(qs[0])) for c in caches]
    for i in range(args.warmup):
        steps_g[i % reps].step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    alg_bytes = []
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for j in range(args.steps):
            r = (args.warmup + j) % reps
            alg_bytes.append((int(caches[r].lengths.sum()) + B) * H * 2 * W * 4)  # attended incl. the new token
            ev[j][0].record(stream)
            steps_g[r].step()  # one graph: tq_decode_append (packs the token, attends) + split merge
            ev[j][1].record(stream)
        end.record(stream)
        torch.cuda.synchronize()
    elapsed_ms = start.elapsed_time(end)
    dec_ms = [a.elapsed_time(b) for a, b in ev]
    if world > 1:
        t = torch.tensor([elapsed_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
        dist.barrier()
    ms_per_step = elapsed_ms / args.steps
    value = B * world / (elapsed_ms / 1e3 / args.steps)

    # ---- end to end through the public API with host buffers ----
    e2e_steps = max(3, min(args.steps, 200))
    # Serving-style loop: each step's new K/V and queries start in pinned host
    # memory and are copied to the device on the compute stream, the eager
    # public API appends and decodes, and the step's output is read back into
    # pinned host memory and waited for before the next step.
    hk, hv, hq = new_k.cpu().pin_memory(), new_v.cpu().pin_memory(), qs.cpu().pin_memory()
    dk, dv, dq = torch.empty_like(new_k[0]), torch.empty_like(new_v[0]), torch.empty_like(qs[0])
    host_out = torch.empty(qs[0].shape, dtype=torch.float32).pin_memory()
    checksum = 0.0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for j in range(e2e_steps):
        r = j % ring
        dk.copy_(hk[r], non_blocking=True)                 # host -> device
        dv.copy_(hv[r], non_blocking=True)
        dq.copy_(hq[r], non_blocking=True)
        c = caches[j % reps]
        c.append(key=kv(dk), value=kv(dv))
        res = c.decode(query=kv(dq))
        host_out.copy_(res.reshape(host_out.shape), non_blocking=True)  # device -> host
        stream.synchronize()
        checksum += float(host_out[0, 0, 0, 0])
    e1.record(stream)
    torch.cuda.synchronize()
    outs = [host_out]
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = B * world / (e2e_ms / 1e3 / e2e_steps)
    h2d = int(hk[0].numel() * 2 + hv[0].numel() * 2 + hq[0].numel() * 4)
    d2h = int(outs[0].numel() * 4)

    if rank == 0:
        peak, peak_kind = _peaks()
        mean_dec_ms = statistics.mean(dec_ms)
        mean_bytes = statistics.mean(alg_bytes)
        achieved = mean_bytes / (mean_dec_ms / 1e3) / 1e9
        line = {
            "metric": "decode tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": f"u32 packed {bits}-bit codes; fp16 mma, fp32 softmax/accumulate",
            "data": "synthetic (seeded fp16 N(0,1) K/V and fp32 queries generated on device)",
            "config": {"workload": args.workload, "desc": wl["desc"], "global_batch": B * world, "per_gpu_batch": B,
                       "q_heads": Hq, "kv_heads": H, "head_dim": d, "bits": bits,
                       "mean_len": float(np.mean(lens)), "parallelism": f"batch-shard x{world}",
                       "l2": ("no flush; inputs larger than L2 (packed cache %.2f GB per GPU)" % (mean_bytes / 1e9))
                       if reps == 1 else
                       ("no flush; %d replicas of the %.0f MB cache (%.0f MB) cycled step by step, so each step "
                        "reads codes evicted from the 126 MB L2" % (reps, cache_bytes / 1e6, reps * cache_bytes / 1e6))},
            "packed_kv_gbs": achieved,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": _traffic(args.workload),
                         "kernel": "tq_decode_append (decode_mma_kernel packing the new token + merge_partials_kernel)", "peak_kind": peak_kind,
                         "bytes_per_launch": mean_bytes, "launch_ms": mean_dec_ms},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": 2 * args.steps,
            "timing": "device loop = CUDA-graph replay of the fused step (tq_decode_append: append packed inside the decode kernel, then the split merge); e2e = eager public API (append/decode) with pinned-host inputs copied in and the output copied back and waited for every step",
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            cores = max(1, min(os.cpu_count() or 1, 64))
            rate, sample = cpu_reference_rate(wl, tokens=2048, seqs=max(1, cores // H), cores=cores)
            line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port",
                                    "sample": sample}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: about a second of timed work for the workload)")
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default="config4", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None, help="override the per-GPU batch (small profiling cases)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    wl = dict(WORKLOADS[args.workload])
    if args.batch:
        wl["batch"] = args.batch
    if args.steps is None:
        args.steps = wl["steps"] if args.impl == "ours" else 5
    if args.impl == "reference":
        run_reference(args, wl)
    elif args.workload == "config5":
        run_decoder(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
