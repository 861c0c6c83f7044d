#!/usr/bin/env python
"""decisions/s of the Laya mmBERT decision forward on B200.

Workload (one step = one forward over one batch): batched Snake-style
decisions, 64 sequences of 175-180 tokens (uniform), 8 option markers each,
act/escalate head on [CLS]; seeded synthetic weights (N(0, 0.02), bf16/f16
exact) and token ids. The reference publishes no GPU or batched number, so
vs_baseline is null.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N > 1 runs under torchrun, one process per GPU; every rank runs its own
batch of 64 decisions per step (weak scaling, model replicated, no
collective on the data path); the time is the max over ranks of the summed
per-step CUDA-event durations. `--impl reference` times the CPU path (the
oracle's restatement of laya-zig's forward) on the host cores instead.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decisions/s (180-tok, bs=64)"
UNIT = "decisions/s"
BATCH = 64
D_MODEL = 768
GEMM_PARAMS = 124_452_864          # projection weights per token (encoder 110,297,088 + head 14,155,776)
FALLBACK = {"bf16_tflops_sustained": 1400.0, "bf16_tflops": 1590.0, "hbm_gbs": 6650.0}


def l2_bytes() -> int:
    """The current device's L2 size (126 MB on a B200; 0 without a GPU)."""
    import torch
    if not torch.cuda.is_available():
        return 0
    return int(torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size)


def flush_bytes() -> int:
    """Bytes written between timed steps to flush L2: 1.25x its size, in MiB."""
    return ((l2_bytes() * 5 // 4) + (1 << 20) - 1) >> 20 << 20


def config(world: int):
    return {"workload": "batched Snake-style decisions: 64 seqs x 175-180 tokens (uniform), 8 option markers, "
                        "act head on [CLS]; mmBERT-base 22 layers + 2 head layers",
            "global_batch": BATCH * world, "seq_len": 180, "parallelism": "replicas dp%d (no collective)" % world,
            "l2": "flushed between timed steps (%d MB write, 1.25x the %d MB L2)" % (flush_bytes() // 10**6,
                                                                                l2_bytes() // 10**6)}


def attn_flops(L: int) -> float:
    s = sum(min(L, i + 65) - max(0, i - 64) for i in range(L))
    return 4.0 * 768 * (10 * L * L + 14 * s)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return FALLBACK, "fallback"


def traffic_per_launch():
    """dram read+write bytes per projection-GEMM launch, from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "gemm_tc_snake64.txt")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            if line.startswith("traffic_bytes_per_launch:"):
                try:
                    return float(line.split(":", 1)[1].split()[0])
                except ValueError:
                    return None
    return None


class Clocks:
    """nvidia-smi clocks + throttle reasons sampled during the timed region."""
    Q = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids):
        self.uuids = set(u.lower() for u in uuids if u)
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.Q, "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait(timeout=10)
        self.f.seek(0)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            c = [x.strip() for x in line.split(",")]
            if len(c) < 10:
                continue
            if self.uuids and c[1].lower() not in self.uuids:
                continue
            try:
                sm.append(float(c[2]))
                mx.append(float(c[3]))
            except ValueError:
                continue
            for n, v in zip(names, c[6:10]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(weights, batch, budget_s=15.0, max_n=32, threads=None):
    """The oracle (a C restatement of laya-zig's CPU forward) on the host cores."""
    from oracle import oracle
    threads = threads or min(os.cpu_count() or 1, 8)  # the reference's default thread count
    m = oracle.model_from_bf16(weights)
    m.forward(batch[0].ids, batch[0].markers, batch[0].qtype, threads=threads)  # warm pages
    t0 = time.perf_counter()
    n = 0
    while n < max_n and (n == 0 or time.perf_counter() - t0 < budget_s):
        d = batch[n % len(batch)]
        m.forward(d.ids, d.markers, d.qtype, threads=threads)
        n += 1
    dt = time.perf_counter() - t0
    m.close()
    return {"value": n / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": "%d decisions of the batch (175-180 tokens, 8 markers), one forward at a time, %.1f s" % (n, dt)}


def run_reference(args, world):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from laya_zig_b200 import synth
    from oracle import oracle
    weights = synth.make_weights(0)
    batch = synth.snake_batch(BATCH, seed=2)
    threads = os.cpu_count() or 1
    m = oracle.model_from_bf16(weights)
    per_step = 2
    i = 0

    def step():
        nonlocal i
        for _ in range(per_step):
            d = batch[i % len(batch)]
            m.forward(d.ids, d.markers, d.qtype, threads=threads)
            i += 1

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    v = per_step * args.steps / dt
    sample = "%d decisions per step from the 64-decision batch, one forward at a time on %d threads" % (per_step, threads)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded weights and token ids)",
        "config": config(world),
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "laya-zig's Zig build cannot be compiled here (no Zig toolchain); this is the oracle's C "
                "restatement of its forward (src/main.zig:2641-2817), packed 16-column GEMM included",
    }), flush=True)


def run_sweep(args, world: int):
    """--workload sweep: the throughput sweep (65,536 decisions, lengths
    uniform in [128, 512]) packed into length-sorted buckets of <= 32,768
    tokens and spread over the ranks longest-processing-time first. Every
    bucket of this rank is staged in HBM first; a step is one pass over all
    of them, timed with CUDA events on the launching stream, max over ranks.
    Total work is fixed, so the scaling is strong."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from laya_zig_b200 import gpu, shard, synth

    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    weights = synth.make_weights(0)
    model = gpu.LayaGPU.from_bf16(weights, device=local, precision=args.precision)
    n = args.sweep_n
    sw = synth.sweep_decisions(n, seed=4)
    mine, _ = shard.shard(sw, world, rank)
    staged, tokens, flops = [], 0, 0.0
    for idx in mine:
        dec = [sw[i] for i in idx]
        p = gpu.pack(dec)
        dev = {k: torch.from_numpy(v.view(np.int32)).cuda() for k, v in p.items() if k != "max_len"}
        S, M, G = len(dec), len(p["ids"]), int(p["cu_markers"][-1])
        db = gpu.DeviceBatch(dev["ids"].data_ptr(), dev["cu_seqlens"].data_ptr(), dev["markers"].data_ptr(),
                             dev["cu_markers"].data_ptr(), dev["qtypes"].data_ptr(), S, M, G, p["max_len"])
        staged.append((db, torch.zeros(max(G, 1), device="cuda"), torch.zeros((S, 2), device="cuda"), dev))
        tokens += M
        flops += shard.bucket_cost([len(d.ids) for d in dec])
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream
    for _ in range(args.warmup):  # every bucket shape once: workspace growth, graphs for the small ones
        for db, lg, ac, _ in staged:
            model.forward_device(db, lg.data_ptr(), ac.data_ptr(), stream=sp)
    model.sync()
    barrier()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    clocks = Clocks([uuid] if uuid else [])
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(args.steps):
        for db, lg, ac, _ in staged:
            model.forward_device(db, lg.data_ptr(), ac.data_ptr(), stream=sp)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    model.sync()
    for _, _, ac, _ in staged:
        a = ac.cpu().numpy()
        assert np.isfinite(a).all() and np.allclose(a.sum(1), 1, atol=1e-4), "bad act output"
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
        dist.destroy_process_group()
    t_max = float(t.item())
    model.close()
    if rank != 0:
        return
    print(json.dumps({
        "metric": "decisions/s (sweep: %d decisions, L 128-512)" % n, "value": n * args.steps / (t_max / 1e3),
        "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t_max / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": args.precision, "data": "synthetic (seeded weights and token ids)",
        "config": {"workload": "throughput sweep: %d decisions, lengths uniform in [128, 512], length-sorted "
                               "buckets of <= 32,768 tokens, LPT over ranks" % n,
                   "global_batch": n, "seq_len": "128-512", "parallelism": "replicas dp%d (no collective)" % world,
                   "rank0_buckets": len(mine), "rank0_tokens": tokens,
                   "l2": "every bucket's activations exceed L2"},
        "rank0_tokens_per_s": tokens * args.steps / (t_max / 1e3),
        "rank0_tflops": flops * args.steps / (t_max / 1e3) / 1e12,
        "gpu_launches": len(mine) * 171 * args.steps,
        "clocks": clk,
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default="bf16", choices=["bf16", "f16"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="snake", choices=["snake", "sweep"],
                    help="snake: the 64 x 180 headline batch (default); sweep: the bucketed throughput sweep")
    ap.add_argument("--sweep-n", type=int, default=65536)
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        run_reference(args, world)
        return
    if args.workload == "sweep":
        run_sweep(args, world)
        return

    import numpy as np
    import torch
    import torch.distributed as dist
    from laya_zig_b200 import gpu, synth

    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    weights = synth.make_weights(0)
    model = gpu.LayaGPU.from_bf16(weights, device=local, precision=args.precision)
    batch = synth.snake_batch(BATCH, seed=2 + 1000 * rank)   # each rank its own shard of decisions
    p = gpu.pack(batch)
    M, S, G = len(p["ids"]), len(batch), int(p["cu_markers"][-1])
    dev = {k: torch.from_numpy(v.view(np.int32)).cuda() for k, v in p.items() if k != "max_len"}
    db = gpu.DeviceBatch(dev["ids"].data_ptr(), dev["cu_seqlens"].data_ptr(), dev["markers"].data_ptr(),
                         dev["cu_markers"].data_ptr(), dev["qtypes"].data_ptr(), S, M, G, p["max_len"])
    logits = torch.zeros(G, dtype=torch.float32, device="cuda")
    act = torch.zeros((S, 2), dtype=torch.float32, device="cuda")
    flush = torch.empty(flush_bytes(), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()          # every launch, flush and event of the timed loop goes here
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream

    for _ in range(max(3, args.warmup)):
        model.forward_device(db, logits.data_ptr(), act.data_ptr(), stream=sp)
    model.sync()
    barrier()

    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    clocks = Clocks([uuid] if uuid else [])
    clocks.start()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    for i in range(args.steps):
        flush.zero_()
        starts[i].record(stream)
        model.forward_device(db, logits.data_ptr(), act.data_ptr(), stream=sp)
        ends[i].record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    model.sync()
    t_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    t = torch.tensor([t_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t_max = float(t.item())
    value = world * S * args.steps / (t_max / 1e3)
    a = act.cpu().numpy()
    assert np.isfinite(a).all() and np.allclose(a.sum(1), 1, atol=1e-4), "bad act output"

    # e2e: the public host-buffer call (laya_gpu_forward_batch) every step: the
    # step's ids/markers copied from the caller's host arrays through pinned
    # staging to the device, the forward, logits + act back into host arrays.
    pb = gpu.PreparedBatch(batch)
    model.forward_prepared(pb)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model.forward_prepared(pb)
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e = world * S * args.steps / float(te.item())
    h2d = 4 * M + 4 * (S + 1) + 4 * S + 4 * G + 4 * (S + 1)
    d2h = 4 * G + 8 * S + 4

    # dominant kernel (projection GEMMs): CUDA events around every launch, same stream
    stage_ms, launches = model.profile(db, logits.data_ptr(), act.data_ptr(), iters=5, stream=sp)
    gemm_stages = ["gemm_qkv", "gemm_out", "gemm_up", "gemm_down"]
    gemm_ms = sum(stage_ms[s] for s in gemm_stages) / 5
    gemm_launches = sum(launches[s] for s in gemm_stages)
    gemm_flops = 2.0 * M * GEMM_PARAMS
    pk, src = peaks()
    peak = float(pk.get("bf16_tflops_sustained", FALLBACK["bf16_tflops_sustained"]))
    achieved = gemm_flops / (gemm_ms / 1e3) / 1e12
    tr = traffic_per_launch()
    attn_step = sum(attn_flops(len(d.ids)) for d in batch)
    flops_step = gemm_flops + attn_step
    # the other kernel families against their own bounds, same profiled pass
    hbm = float(pk.get("hbm_gbs", FALLBACK["hbm_gbs"]))
    hbm_src = "%s hbm_gbs (%s)" % ("MEASURED_PEAKS.json" if src == "measured" else "fallback", src)

    def per_launch_ms(stage):
        return stage_ms[stage] / 5 / max(1, launches[stage])

    secondary = []
    if launches.get("norm"):
        ln_bytes = M * (D_MODEL * 4 + D_MODEL * 2)  # f32 row in, 16-bit row out
        a = ln_bytes / (per_launch_ms("norm") / 1e3) / 1e9
        secondary.append({"kernel": "ln_kernel (%d launches per step)" % launches["norm"], "bound": "hbm",
                          "algorithmic_bytes_per_launch": ln_bytes, "achieved": a, "peak": hbm, "unit": "GB/s",
                          "frac": a / hbm, "peak_source": hbm_src})
    if launches.get("attention"):
        a = attn_step / (stage_ms["attention"] / 5 / 1e3) / 1e12
        secondary.append({"kernel": "attention_kernel (%d launches per step)" % launches["attention"],
                          "bound": "tensor", "algorithmic_flops_per_step": attn_step, "achieved": a, "peak": peak,
                          "unit": "TFLOP/s", "frac": a / peak,
                          "peak_source": "%s bf16_tflops_sustained (%s)" % (
                              "MEASURED_PEAKS.json" if src == "measured" else "fallback", src)})
    for st, name, nbytes in (("embed", "embed_kernel", M * (D_MODEL * 2 + D_MODEL * 4 + D_MODEL * 2)),
                             ("final", "final_kernel", M * (D_MODEL * 4 + D_MODEL * 4 + D_MODEL * 2))):
        if launches.get(st):
            a = nbytes / (per_launch_ms(st) / 1e3) / 1e9
            secondary.append({"kernel": name, "bound": "hbm", "algorithmic_bytes_per_launch": nbytes, "achieved": a,
                              "peak": hbm, "unit": "GB/s", "frac": a / hbm, "peak_source": hbm_src})
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        model.close()
        return

    base = None
    if world == 1 and not args.no_cpu_baseline:
        base = cpu_baseline(weights, batch)
    out = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": args.precision, "data": "synthetic (seeded weights and token ids)",
        "config": config(world),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": tr,
                     "kernel": "gemm_pair_kernel (tcgen05 cta_group::2 projection GEMMs, %d launches per step)" % gemm_launches,
                     "peak_source": "%s bf16_tflops_sustained (%s)" % ("MEASURED_PEAKS.json" if src == "measured"
                                                                        else "fallback", src),
                     "algorithmic_flops_per_step": gemm_flops},
        "cpu_baseline": base,
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": sum(launches.values()) * args.steps,
        "clocks": clk,
        "stage_ms_per_step": {k: v / 5 for k, v in stage_ms.items()},
        "whole_step_tflops": flops_step / (t_max / args.steps / 1e3) / 1e12,
        "secondary_rooflines": secondary,
    }
    print(json.dumps(out), flush=True)
    model.close()


if __name__ == "__main__":
    main()
