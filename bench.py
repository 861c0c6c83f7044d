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

Other workloads (not the headline line):
  --workload sweep   65,536 decisions of 128-512 tokens in length buckets (strong scaling)
  --workload gemm    the four projection shapes at M = 180 and M = 11,520, each
                     launch timed alone (the reference's --benchgemm)
  --workload long    one 8,192-token decision (latency, attention roofline)
  --workload single  one decision per call (the --serve / --snake latency)

Kernel times in the rooflines: a CUDA graph of one forward with an event pair
around every launch gives each launch's time; the event nodes stop
programmatic dependent launch from overlapping neighbours, so those times
over-count. The roofline time of a kernel family is its share of the
profiled total applied to the real (PDL-overlapped) step time measured in
the timed region; the raw event-pair figure is reported beside it. Peaks:
MEASURED_PEAKS.json, burst bf16 for a run whose clocks saw no power cap,
sustained bf16 when `sw_power_cap` was active.
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


def tensor_peak(clk):
    """(bf16 TFLOP/s peak, label): the burst figure unless the timed region
    ran under the power cap, which only seconds-long loads reach."""
    pk, src = peaks()
    name = "MEASURED_PEAKS.json" if src == "measured" else "fallback"
    capped = "sw_power_cap" in (clk or {}).get("reasons", [])
    key = "bf16_tflops_sustained" if capped else "bf16_tflops"
    why = "sw_power_cap active in the timed region" if capped else "no power cap in the timed region"
    return float(pk.get(key, FALLBACK[key])), "%s %s (%s, %s)" % (name, key, src, why)


def hbm_peak():
    pk, src = peaks()
    name = "MEASURED_PEAKS.json" if src == "measured" else "fallback"
    return float(pk.get("hbm_gbs", FALLBACK["hbm_gbs"])), "%s hbm_gbs (%s)" % (name, src)


def attn_flops_split(L: int):
    """(global, sliding) attention FLOPs of one sequence: 4*768*L^2 per global
    layer (8 encoder + 2 head), 4*768*S(L) per sliding layer (14)."""
    s = sum(min(L, i + 65) - max(0, i - 64) for i in range(L))
    return 4.0 * 768 * 10 * L * L, 4.0 * 768 * 14 * s


def launch_profile(model, db, lg_ptr, act_ptr, stream, iters=5):
    """Per-launch event-pair times of one forward, grouped: returns
    (total_ms, {family: [ms per launch, ...]}) with the encoder attention
    launches split into global (layer % 3 == 0, and the two head layers) and
    sliding ones."""
    prof = model.profile_launches(db, lg_ptr, act_ptr, iters=iters, stream=stream)
    fam = {}
    attn_i = 0
    for stage, ms in prof:
        key = stage
        if stage == "attention":
            key = "attention_global" if (attn_i >= 22 or attn_i % 3 == 0) else "attention_sliding"
            attn_i += 1
        fam.setdefault(key, []).append(ms / iters)
    return sum(ms for _, ms in prof) / iters, fam


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
    ranks = per_rank(world, float(t.item()), clk, float(tokens))
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
        "per_rank": [{"rank": r["rank"], "ms": r["ms"], "sm_mhz": r["sm_mhz"], "tokens": int(r["extra"])}
                     for r in ranks],
        "rank0_tokens_per_s": tokens * args.steps / (t_max / 1e3),
        "rank0_tflops": flops * args.steps / (t_max / 1e3) / 1e12,
        "gpu_launches": len(mine) * 171 * args.steps,
        "clocks": clk,
    }), flush=True)


def per_rank(world, t_ms, clk, extra=0.0):
    """[{rank, ms, sm_mhz, extra}] gathered from every rank (one small NCCL
    all-gather; the same call on every rank)."""
    import torch
    import torch.distributed as dist
    v = torch.tensor([t_ms, clk.get("sm_mhz") or -1.0, extra], dtype=torch.float64, device="cuda")
    if world <= 1:
        rows = [v]
    else:
        rows = [torch.zeros_like(v) for _ in range(world)]
        dist.all_gather(rows, v)
    return [{"rank": r, "ms": float(x[0]), "sm_mhz": float(x[1]) if x[1] >= 0 else None, "extra": float(x[2])}
            for r, x in enumerate(rows)]


def _clock_region(local):
    import torch
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    return Clocks([uuid] if uuid else [])


GEMM_SHAPES = [("QKV", 2304, 768), ("attn-out", 768, 768), ("GLU Wi", 2304, 768), ("FFN-out", 768, 1152)]


def run_gemm(args):
    """--workload gemm: the projection shapes at M = 180 and 11,520 through
    laya_gpu_linear (the drop-in for linear16: bf16 operands, f32 out,
    tcgen05 cta_group::2 kernel), each launch timed alone with CUDA events on
    its stream after an L2 flush that leaves no dirty lines (a write of a
    buffer larger than L2, then a read of another one); A ~ N(0, 1), W ~
    N(0, 0.02), rounded to bf16. Beside it, cuBLAS through torch.mm on the
    same operands (f32 out where torch offers it). Every output is checked
    against an f64 product."""
    import torch
    from laya_zig_b200 import gpu
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream
    # L2 flush before every timed launch: a write of a buffer larger than L2
    # evicts the operands, then a read of a second one evicts the first's
    # dirty lines, so their write-back (as large as a launch's own traffic
    # here) happens before the launch's start event, not inside it
    flush = torch.empty(flush_bytes(), dtype=torch.uint8, device="cuda")
    flush_rd = torch.zeros(flush_bytes() // 4, dtype=torch.int32, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(7)
    steps, warm = max(args.steps, 1), max(args.warmup, 3)

    def timed(fn):
        for _ in range(warm):
            fn()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for a, b in ev:
            flush.zero_()
            flush_rd.sum()
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize()
        return statistics.median(a.elapsed_time(b) for a, b in ev)

    clocks = _clock_region(0)
    clocks.start()
    rows = []
    for M in (180, 11520):
        for name, N, K in GEMM_SHAPES:
            a = torch.randn(M, K, device="cuda", generator=gen).to(torch.bfloat16)
            w = (torch.randn(N, K, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
            out = torch.empty(M, N, dtype=torch.float32, device="cuda")
            run = lambda: gpu.linear(a.data_ptr(), w.data_ptr(), 0, out.data_ptr(), M, N, K, "BF16", sp)
            ms = timed(run)
            ref = a.double() @ w.double().t()
            err = float(((out.double() - ref).abs().amax(1) / ref.abs().amax(1)).max())
            try:
                cub = lambda: torch.mm(a, w.t(), out_dtype=torch.float32)
                cub()
                cub_kind = "torch.mm bf16 -> f32"
            except Exception:
                cub = lambda: torch.mm(a, w.t())
                cub_kind = "torch.mm bf16 -> bf16"
            cms = timed(cub)
            fl = 2.0 * M * N * K
            rows.append({"shape": name, "M": M, "N": N, "K": K, "us": ms * 1e3, "tflops": fl / (ms / 1e3) / 1e12,
                         "cublas_us": cms * 1e3, "cublas_tflops": fl / (cms / 1e3) / 1e12, "cublas": cub_kind,
                         "max_row_rel_err_vs_f64": err})
            assert err < 1e-4, (name, M, err)
    clk = clocks.stop()
    peak, peak_src = tensor_peak(clk)
    big = [r for r in rows if r["M"] == 11520]
    fl = sum(2.0 * r["M"] * r["N"] * r["K"] for r in big)
    t = sum(r["us"] for r in big) / 1e6
    for r in rows:
        r["frac"] = r["tflops"] / peak
    print(json.dumps({
        "metric": "projection GEMM TFLOP/s at M=11520 (QKV, attn-out, GLU Wi, FFN-out), each launch alone",
        "value": fl / t / 1e12, "unit": "TFLOP/s", "n_gpus": 1, "steps": steps, "warmup": warm,
        "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (A ~ N(0,1), W ~ N(0,0.02), bf16)",
        "config": {"workload": "isolated projection GEMMs through laya_gpu_linear (f32 out), M in {180, 11520}",
                   "l2": "flushed before every timed launch (%d MB write, then a %d MB read of another "
                         "buffer: cold and clean)" % (flush_bytes() // 10**6, flush_bytes() // 10**6),
                   "time": "median of %d launches" % steps},
        "roofline": {"bound": "tensor", "achieved": fl / t / 1e12, "peak": peak, "unit": "TFLOP/s",
                     "frac": fl / t / 1e12 / peak, "traffic": None, "peak_source": peak_src,
                     "kernel": "gemm_pair_kernel<EPI_F32> (laya_gpu_linear)"},
        "shapes": rows, "clocks": clk, "gpu_launches": len(rows) * (steps + warm),
    }), flush=True)


def run_long(args):
    """--workload long: one 8,192-token decision with 16 markers (global
    attention every third layer), resident in HBM; a step is one forward,
    timed with CUDA events on its stream after an L2 flush. e2e: the host
    call laya_gpu_forward with host ids. Attention and GEMM rooflines from the
    per-launch profile (launches of milliseconds, so the event pairs cost
    little)."""
    import numpy as np
    import torch
    from laya_zig_b200 import gpu, synth
    torch.cuda.set_device(0)
    weights = synth.make_weights(0)
    model = gpu.LayaGPU.from_bf16(weights, device=0, precision=args.precision)
    d = synth.long_decision(args.long_len, 16, seed=3)
    p = gpu.pack([d])
    dev = {k: torch.from_numpy(v.view(np.int32)).cuda() for k, v in p.items() if k != "max_len"}
    M, G = len(p["ids"]), int(p["cu_markers"][-1])
    db = gpu.DeviceBatch(dev["ids"].data_ptr(), dev["cu_seqlens"].data_ptr(), dev["markers"].data_ptr(),
                         dev["cu_markers"].data_ptr(), dev["qtypes"].data_ptr(), 1, M, G, p["max_len"])
    logits = torch.zeros(G, dtype=torch.float32, device="cuda")
    act = torch.zeros((1, 2), dtype=torch.float32, device="cuda")
    flush = torch.empty(flush_bytes(), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream
    steps = max(args.steps, 1)
    for _ in range(max(3, args.warmup)):
        model.forward_device(db, logits.data_ptr(), act.data_ptr(), stream=sp)
    model.sync()
    clocks = _clock_region(0)
    clocks.start()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in ev:
        flush.zero_()
        a.record(stream)
        model.forward_device(db, logits.data_ptr(), act.data_ptr(), stream=sp)
        b.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    model.sync()
    ms = sum(a.elapsed_time(b) for a, b in ev) / steps
    t0 = time.perf_counter()
    for _ in range(steps):
        model.forward(d.ids, d.qtype, d.markers)
    e2e_ms = (time.perf_counter() - t0) * 1e3 / steps
    prof_total, fam = launch_profile(model, db, logits.data_ptr(), act.data_ptr(), sp, iters=3)
    attr = ms / prof_total
    peak, peak_src = tensor_peak(clk)
    g_fl, s_fl = attn_flops_split(M)
    gemm_fl = 2.0 * M * GEMM_PARAMS
    fams = {"attention_global": g_fl, "attention_sliding": s_fl,
            "projection GEMMs": gemm_fl}
    gemm_ms = sum(sum(fam.get(f, [])) for f in ["gemm_qkv", "gemm_out", "gemm_up", "gemm_down"])
    times = {"attention_global": sum(fam.get("attention_global", [])),
             "attention_sliding": sum(fam.get("attention_sliding", [])), "projection GEMMs": gemm_ms}
    rl = [{"kernel": k, "bound": "tensor", "algorithmic_flops": fl, "event_pair_ms": times[k],
           "achieved": fl / (times[k] * attr / 1e3) / 1e12, "achieved_event_pairs": fl / (times[k] / 1e3) / 1e12,
           "peak": peak, "unit": "TFLOP/s", "frac": fl / (times[k] * attr / 1e3) / 1e12 / peak,
           "peak_source": peak_src} for k, fl in fams.items() if times[k] > 0]
    a = act.cpu().numpy()
    assert np.isfinite(a).all() and abs(a.sum() - 1) < 1e-4
    h2d = 4 * M + 4 * 2 + 4 + 4 * G + 4 * 2
    print(json.dumps({
        "metric": "long-context decision latency (1 x %d tokens, 16 markers)" % M, "value": 1e3 / ms,
        "unit": "decisions/s", "n_gpus": 1, "steps": steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
        "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": args.precision,
        "data": "synthetic (seeded weights and token ids)",
        "config": {"workload": "one decision of %d tokens, 16 markers at random positions, global attention "
                               "every third layer, sliding window 128 elsewhere" % M,
                   "l2": "flushed between timed steps"},
        "latency_ms": ms, "roofline": rl[0] if rl else None, "rooflines": rl,
        "whole_step_tflops": (g_fl + s_fl + gemm_fl) / (ms / 1e3) / 1e12,
        "e2e": {"value": 1e3 / e2e_ms, "unit": "decisions/s", "latency_ms": e2e_ms, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": 4 * G + 8 + 4 + 768 * 4},
        "timing": "family share of the per-launch event-pair profile x the timed step (profiled %.3f ms vs %.3f ms)"
                  % (prof_total, ms),
        "clocks": clk, "gpu_launches": (sum(len(v) for v in fam.values()) + 2) * steps,
    }), flush=True)
    model.close()


def run_single(args):
    """--workload single: the latency of one decision, the --serve / --snake
    case of the reference (one forward per request): the C1 decision (64
    tokens, 4 markers) and one Snake-style decision of 180 tokens (8
    markers), each through the host call laya_gpu_forward (ids copied in,
    logits/act/pooled copied out, one cached CUDA graph replayed) and as a
    device-resident forward timed with CUDA events."""
    import numpy as np
    import torch
    from laya_zig_b200 import gpu, synth
    torch.cuda.set_device(0)
    model = gpu.LayaGPU.from_bf16(synth.make_weights(0), device=0, precision=args.precision)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    steps = max(args.steps, 1)
    rows = []
    clocks = _clock_region(0)
    clocks.start()
    for name, d in (("C1 1x64, 4 markers", synth.parity_decision(1)), ("1x180, 8 markers", synth.snake_batch(1)[0])):
        for _ in range(max(3, args.warmup)):
            model.forward(d.ids, d.qtype, d.markers)
        t0 = time.perf_counter()
        for _ in range(steps):
            model.forward(d.ids, d.qtype, d.markers)
        host_ms = (time.perf_counter() - t0) * 1e3 / steps
        p = gpu.pack([d])
        dev = {k: torch.from_numpy(v.view(np.int32)).cuda() for k, v in p.items() if k != "max_len"}
        G = int(p["cu_markers"][-1])
        db = gpu.DeviceBatch(dev["ids"].data_ptr(), dev["cu_seqlens"].data_ptr(), dev["markers"].data_ptr(),
                             dev["cu_markers"].data_ptr(), dev["qtypes"].data_ptr(), 1, len(p["ids"]), G, p["max_len"])
        lg = torch.zeros(G, device="cuda")
        ac = torch.zeros((1, 2), device="cuda")
        for _ in range(3):
            model.forward_device(db, lg.data_ptr(), ac.data_ptr(), stream=stream.cuda_stream)
        model.sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            model.forward_device(db, lg.data_ptr(), ac.data_ptr(), stream=stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        model.sync()
        rows.append({"decision": name, "host_call_ms": host_ms, "device_ms": e0.elapsed_time(e1) / steps})
    clk = clocks.stop()
    model.close()
    print(json.dumps({
        "metric": "single-decision latency (host call laya_gpu_forward)", "value": rows[1]["host_call_ms"],
        "unit": "ms", "n_gpus": 1, "steps": steps, "warmup": max(3, args.warmup),
        "ms_per_step": rows[1]["host_call_ms"], "higher_is_better": False, "scaling": "none", "vs_baseline": None,
        "dtype": args.precision, "data": "synthetic (seeded weights and token ids)",
        "config": {"workload": "one decision per call: C1 (64 tokens) and a 180-token Snake-style decision; "
                               "consecutive calls, L2 not flushed (each call is a separate request)"},
        "decisions": rows, "clocks": clk, "gpu_launches": 171 * steps * 4,
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default="bf16", choices=["bf16", "f16"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="snake", choices=["snake", "sweep", "gemm", "long", "single"],
                    help="snake: the 64 x 180 headline batch (default); sweep: the bucketed throughput sweep; "
                         "gemm: isolated projection GEMMs; long: one 8192-token decision; "
                         "single: one-decision latency")
    ap.add_argument("--sweep-n", type=int, default=65536)
    ap.add_argument("--long-len", type=int, default=8192, help="--workload long: the sequence length")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        run_reference(args, world)
        return
    if args.workload == "sweep":
        run_sweep(args, world)
        return
    if args.workload == "gemm":
        run_gemm(args)
        return
    if args.workload == "long":
        run_long(args)
        return
    if args.workload == "single":
        run_single(args)
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
    ranks = per_rank(world, t_ms, clk)
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

    # Kernel families: per-launch event-pair times of one forward (5 passes),
    # attributed to the real step by their share of the profiled total.
    step_ms = t_max / args.steps
    prof_total, fam = launch_profile(model, db, logits.data_ptr(), act.data_ptr(), sp, iters=5)
    attr = step_ms / prof_total
    gemm_fams = ["gemm_qkv", "gemm_out", "gemm_up", "gemm_down"]
    gemm_prof_ms = sum(sum(fam.get(f, [])) for f in gemm_fams)
    gemm_launches = sum(len(fam.get(f, [])) for f in gemm_fams)
    gemm_flops = 2.0 * M * GEMM_PARAMS
    peak, peak_src = tensor_peak(clk)
    achieved = gemm_flops / (gemm_prof_ms * attr / 1e3) / 1e12
    achieved_pairs = gemm_flops / (gemm_prof_ms / 1e3) / 1e12
    tr = traffic_per_launch()
    attn_g = sum(attn_flops_split(len(d.ids))[0] for d in batch)
    attn_s = sum(attn_flops_split(len(d.ids))[1] for d in batch)
    flops_step = gemm_flops + attn_g + attn_s
    hbm, hbm_src = hbm_peak()
    timing = ("family share of a per-launch event-pair profile (5 passes) x the timed step time; "
              "profiled total %.3f ms vs step %.3f ms" % (prof_total, step_ms))

    secondary = []
    for f, name, nbytes in (("norm", "ln_kernel", M * (D_MODEL * 4 + D_MODEL * 2)),
                            ("embed", "embed_kernel", M * (D_MODEL * 2 + D_MODEL * 4 + D_MODEL * 2 + 256)),
                            ("final", "final_kernel", M * (D_MODEL * 4 + D_MODEL * 4 + D_MODEL * 2))):
        if fam.get(f):
            per = sum(fam[f]) / len(fam[f])
            a = nbytes / (per * attr / 1e3) / 1e9
            secondary.append({"kernel": "%s (%d launches per step)" % (name, len(fam[f])), "bound": "hbm",
                              "algorithmic_bytes_per_launch": nbytes, "achieved": a, "peak": hbm, "unit": "GB/s",
                              "frac": a / hbm, "achieved_event_pairs": nbytes / (per / 1e3) / 1e9,
                              "peak_source": hbm_src})
    for f, fl in (("attention_sliding", attn_s), ("attention_global", attn_g)):
        if fam.get(f):
            t = sum(fam[f])
            a = fl / (t * attr / 1e3) / 1e12
            secondary.append({"kernel": "attention_kernel, %s layers (%d launches per step)" % (f[10:], len(fam[f])),
                              "bound": "tensor", "algorithmic_flops_per_step": fl, "achieved": a, "peak": peak,
                              "unit": "TFLOP/s", "frac": a / peak, "achieved_event_pairs": fl / (t / 1e3) / 1e12,
                              "peak_source": peak_src})
    for f in gemm_fams:
        if fam.get(f):
            per_tok = {"gemm_qkv": (22 * 3 * 768 * 768 + 2 * 3 * 768 * 768),
                       "gemm_out": 24 * 768 * 768,
                       "gemm_up": 22 * 2 * 1152 * 768 + 2 * 3072 * 768,
                       "gemm_down": 22 * 1152 * 768 + 2 * 3072 * 768}[f]
            fl = 2.0 * M * per_tok
            t = sum(fam[f])
            a = fl / (t * attr / 1e3) / 1e12
            secondary.append({"kernel": "gemm_pair_kernel %s (%d launches per step)" % (f, len(fam[f])),
                              "bound": "tensor", "algorithmic_flops_per_step": fl, "achieved": a, "peak": peak,
                              "unit": "TFLOP/s", "frac": a / peak, "achieved_event_pairs": fl / (t / 1e3) / 1e12,
                              "peak_source": peak_src})
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
                     "peak_source": peak_src, "timing": timing, "achieved_event_pairs": achieved_pairs,
                     "algorithmic_flops_per_step": gemm_flops},
        "cpu_baseline": base,
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": (sum(len(v) for v in fam.values()) + (2 if G else 0)) * args.steps,
        "clocks": clk,
        "family_ms_per_step": {k: sum(v) * attr for k, v in fam.items()},
        "per_rank": [{"rank": r["rank"], "ms_per_step": r["ms"] / args.steps, "sm_mhz": r["sm_mhz"]} for r in ranks],
        "whole_step_tflops": flops_step / (step_ms / 1e3) / 1e12,
        "secondary_rooflines": secondary,
    }
    print(json.dumps(out), flush=True)
    model.close()


if __name__ == "__main__":
    main()
