"""Benchmark of the B200 K-quant hot path (one JSON line on rank 0).

Workload "q4k_ffn": the Llama-3-8B FFN matvec set in Q4_K at batch 1
(gate and up 4096->14336 sharing one input, down 14336->4096) -- one step is
one pass over the three weights.  Four seeded weight sets (396 MB) rotate
between steps so every step streams its weights from HBM, not L2 (126 MB).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's CPU path (the oracle restatement of
SharpInfer's TensorOps.MatVecMul over weights dequantised to f32 at load
time, Quantization.cs:415-469 + TensorOps.cs:63-72) on the host cores.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, FFN = 4096, 14336
Q4K_BYTES = lambda rows, cols: rows * (cols // 256) * 144  # noqa: E731
STEP_BYTES = 2 * Q4K_BYTES(FFN, HIDDEN) + Q4K_BYTES(HIDDEN, FFN)  # weight bytes per step
ACT_BYTES = 4 * (HIDDEN + 2 * FFN) + 4 * (FFN + HIDDEN)            # x in, y out (f32)
NSETS = 4
METRIC = "Q4_K decode matvec HBM GB/s (Llama-3-8B FFN gate/up/down, batch 1)"


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clock and throttle reasons during the timed region."""

    Q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q, "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 6:
                self.rows.append(parts)

    def stop(self):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[2 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_reference(steps, warmup, sample_s=None):
    """Time the reference CPU path: f32 MatVecMul over load-time-dequantised Q4_K weights."""
    import oracle
    from sharpinfer_b200 import native as N
    from sharpinfer_b200.backend import synth_blocks_host, synth_f32_host
    threads = os.cpu_count() or 1
    shapes = [(FFN, HIDDEN), (FFN, HIDDEN), (HIDDEN, FFN)]
    W = []
    for i, (r, c) in enumerate(shapes):
        blocks = synth_blocks_host(N.SI_Q4_K, r, c, 1234, 100 + i, N.SYNTH_PLAIN, 0.01)
        W.append(oracle.dequant(N.SI_Q4_K, blocks, r * c).reshape(r, c))
    x = synth_f32_host(HIDDEN, 1234, 7)
    h = synth_f32_host(FFN, 1234, 8)

    def step():
        oracle.matvec_f32(W[0], x, threads)
        oracle.matvec_f32(W[1], x, threads)
        oracle.matvec_f32(W[2], h, threads)

    for _ in range(warmup):
        step()
    n = steps
    t0 = time.perf_counter()
    if sample_s is not None:  # bounded sample: as many steps as fit in sample_s
        n = 0
        while time.perf_counter() - t0 < sample_s or n == 0:
            step()
            n += 1
    else:
        for _ in range(n):
            step()
    dt = (time.perf_counter() - t0) / n
    return {"value": STEP_BYTES / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "ms_per_step": dt * 1e3, "steps": n,
            "sample": "%d steps of the f32 gate/up/down matvecs (weights dequantised at load, 4 B/weight "
                      "streamed as the reference does), %d threads; GB/s counts the Q4_K bytes of the same work"
                      % (n, threads)}


def run_reference(args, world, rank):
    if rank != 0:
        return
    r = cpu_reference(args.steps, args.warmup)
    line = {"metric": METRIC, "value": round(r["value"], 3), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": r["steps"], "warmup": args.warmup, "ms_per_step": round(r["ms_per_step"], 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Q4_K blocks, x ~ N(0,1))", "impl": "reference",
            "config": {"workload": "q4k_ffn: Llama-3-8B FFN gate/up (4096->14336) + down (14336->4096) Q4_K matvec, batch 1",
                       "parallelism": "replicas"},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": round(r["value"], 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local):
    import torch
    import torch.distributed as dist
    from sharpinfer_b200 import B200Context, native as N
    from sharpinfer_b200.backend import synth_f32_host

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))
    ctx = B200Context(local)
    dev = torch.device("cuda", local)
    sets = []
    for s in range(NSETS):
        sets.append([ctx.synth_weight(N.SI_Q4_K, FFN, HIDDEN, 1234 + s, 100, N.SYNTH_PLAIN, 0.01),
                     ctx.synth_weight(N.SI_Q4_K, FFN, HIDDEN, 1234 + s, 101, N.SYNTH_PLAIN, 0.01),
                     ctx.synth_weight(N.SI_Q4_K, HIDDEN, FFN, 1234 + s, 102, N.SYNTH_PLAIN, 0.01)])
    x = torch.from_numpy(synth_f32_host(HIDDEN, 1234, 7)).to(dev).reshape(1, -1)
    h = torch.from_numpy(synth_f32_host(FFN, 1234, 8)).to(dev).reshape(1, -1)
    with torch.cuda.stream(ctx.torch_stream):
        yg = torch.empty((1, FFN), device=dev)
        yu = torch.empty((1, FFN), device=dev)
        yd = torch.empty((1, HIDDEN), device=dev)
    torch.cuda.synchronize()
    stream = ctx.torch_stream
    torch.cuda.set_stream(stream)  # all torch work on the context stream: no cross-stream waits
    nk = 3 * (args.steps)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * nk)]

    def step(i, timed_kernels=False):
        g, u, d = sets[i % NSETS]
        ctx.act_prepare(x)
        k = 3 * i
        if timed_kernels:
            ev[2 * k].record(stream)
        ctx.qmatvec_prepared(g, 1, out=yg)
        if timed_kernels:
            ev[2 * k + 1].record(stream)
            ev[2 * k + 2].record(stream)
        ctx.qmatvec_prepared(u, 1, out=yu)
        if timed_kernels:
            ev[2 * k + 3].record(stream)
        ctx.act_prepare(h)
        if timed_kernels:
            ev[2 * k + 4].record(stream)
        ctx.qmatvec_prepared(d, 1, out=yd)
        if timed_kernels:
            ev[2 * k + 5].record(stream)

    for i in range(args.warmup):
        step(i)
    ctx.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        step(i)
    t1.record(stream)
    ctx.synchronize()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    clk = clocks.stop()
    # kernel durations (separate pass with events around every matvec kernel)
    for i in range(args.steps):
        step(i, timed_kernels=True)
    ctx.synchronize()
    kms = [ev[2 * k].elapsed_time(ev[2 * k + 1]) for k in range(nk)]
    # per-launch bytes: gate/up 33,030,144 B and down 33,030,144 B; all three equal
    kern_ms = statistics.mean(kms)
    # e2e through the host-buffer entry point (H2D x, kernels, D2H y, every step)
    xh = synth_f32_host(HIDDEN, 1234, 7)
    hh = synth_f32_host(FFN, 1234, 8)

    def e2e_step(i):
        g, u, d = sets[i % NSETS]
        ctx.qmatvec_host(g, xh)
        ctx.qmatvec_host(u, xh)
        ctx.qmatvec_host(d, hh)

    for i in range(args.warmup):
        e2e_step(i)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    w0 = time.perf_counter()
    for i in range(args.steps):
        e2e_step(i)
    e1.record(stream)
    ctx.synchronize()
    wall_ms = (time.perf_counter() - w0) * 1e3 / args.steps
    e2e_ms = max(e0.elapsed_time(e1) / args.steps, wall_ms)

    t = torch.tensor([ms, e2e_ms, kern_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, kern_ms = t.tolist()
    if rank == 0:
        peak, peak_kind = measured_peaks()
        per_launch = Q4K_BYTES(FFN, HIDDEN) + 4 * (HIDDEN + FFN)
        achieved = per_launch / (kern_ms * 1e-3) / 1e9
        traffic = None
        tp = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tp):
            traffic = json.load(open(tp)).get("q4k_qmv_bytes_per_launch")
        line = {
            "metric": METRIC, "value": round(world * STEP_BYTES / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q4_k x f32 (f16x2 hi/lo MMA, f32 accumulate)",
            "data": "synthetic (seeded Q4_K blocks, x ~ N(0,1))",
            "config": {"workload": "q4k_ffn: Llama-3-8B FFN gate/up (4096->14336) + down (14336->4096) Q4_K matvec, batch 1",
                       "parallelism": "replicas" if world > 1 else "single",
                       "l2": "inputs larger than L2: %d rotating weight sets, %.0f MB" % (NSETS, NSETS * STEP_BYTES / 1e6),
                       "bytes_per_step": STEP_BYTES},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": "k_qmv_q4k (gate 14336x4096)", "peak_source": peak_kind},
            "e2e": {"value": round(world * STEP_BYTES / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": 4 * (2 * HIDDEN + FFN), "d2h_bytes_per_step": 4 * (2 * FFN + HIDDEN)},
            "gpu_launches": 5 * args.steps,
            "clocks": clk,
        }
        if not args.no_cpu_baseline:
            cb = cpu_reference(0, 1, sample_s=args.cpu_seconds)
            line["cpu_baseline"] = {k: (round(v, 3) if isinstance(v, float) else v) for k, v in cb.items()
                                    if k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)
    for s in sets:
        for w in s:
            w.free()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
