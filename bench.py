"""Benchmark of the B200 K-quant decode path (one JSON line on rank 0).

Workload: greedy decode of a Llama-3-8B-architecture model in Q4_K_M form
(Q4_K projections and token embedding, Q6_K lm_head, f32 norms; seeded
synthetic weights -- no checkpoint is available offline), f16 KV cache
prefilled to 4096 positions, batch 1.  One step = one token through all 32
layers + lm_head + argmax (Transformer.Forward, src/SharpInfer.Core/Layers/
Transformer.cs:67-162).  Weights (4.36 GB) and KV (0.54 GB) far exceed the
126 MB L2, so every step streams them from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

value: tokens/s of the device-resident greedy loop (si_decode_generate),
timed with CUDA events.  e2e: tokens/s through the host-facing per-token call
(si_decode_step: token id copied in, argmax copied out, every step).
roofline: the dominant kernel, the fused gate/up Q4_K matvec (28672 x 4096,
66 MB), timed alone with CUDA events over 40 graph-captured launches on
rotating weight copies; the whole step's bytes per token against the same
peak are reported beside it.  On one GPU the line also carries the other
workloads the metric is quoted on: `matvec` (4096 x 4096 Q4_K and the 8B
layer matvec set at batch 1/4/16), `prefill` (the Q4_K GEMM at 512 and 2048
tokens and the 2048-token causal attention) and `tp1_70b` (the 70B model
decoded on one GPU, with its first 16 greedy tokens).
--impl reference times the reference's CPU path -- the oracle restatement of
SharpInfer's managed forward pass over the same weights -- on the host cores,
loading only the oracle's library.
Under torchrun (N > 1) the workload is the Llama-3-70B architecture in the
same Q4_K_M form, f16 KV prefilled to 8192 positions: the N ranks decode the
one sequence tensor-parallel (TP = N, partial sums exchanged in peer memory)
and value is that sequence's tokens/s.  The line carries `parity`: the 70B
architecture cut to 2 layers, decoded 4 steps at TP = N, against the oracle.
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

SEED = 20261201
KV_LEN = 4096
START_TOKEN = 128000
KV_LEN_70B = 8192
NCHECK = 16  # greedy tokens decoded first from START_TOKEN and reported (tokens_check)
BATCH16 = 16  # sequences of the 70B batch decode
METRIC = "decode tok/s + Q4_K matvec HBM GB/s (8B Q4_K_M 1 GPU; 70B TP at 2/4/8)"
# dram__bytes_read.sum + dram__bytes_write.sum of one gate/up k_qmv1 launch
# (28672 x 4096 Q4_K, batch 1) from an ncu --set full capture of
# `bench.py --layers 2` (summary under profiles/): the algorithmic bytes,
# no re-reads.
GATEUP_TRAFFIC = 66131712


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def q4k_bytes(rows, cols):
    return rows * (cols // 256) * 144


def q6k_bytes(rows, cols):
    return rows * (cols // 256) * 210


def q8_bytes(rows, cols):
    return rows * (cols // 32) * 34


class Cfg:
    """The fields of si_model_config (Transformer.cs:43-56), usable by the
    oracle without loading the library; native() gives the C struct."""

    def __init__(self, n_layers, hidden, intermediate, n_heads, n_kv_heads, vocab, max_seq, max_batch=1):
        self.n_layers, self.hidden, self.intermediate = n_layers, hidden, intermediate
        self.n_heads, self.n_kv_heads, self.vocab = n_heads, n_kv_heads, vocab
        self.max_seq, self.max_batch, self.head_dim = max_seq, max_batch, 128
        self.rms_eps, self.rope_theta = 1e-5, 500000.0
        self.weight_qtype, self.lm_head_qtype, self.emb_qtype = 12, 14, 12  # Q4_K, Q6_K, Q4_K

    def cut(self, n_layers):
        return Cfg(n_layers, self.hidden, self.intermediate, self.n_heads, self.n_kv_heads, self.vocab,
                   self.max_seq, self.max_batch)

    def native(self):
        from sharpinfer_b200.model import config
        return config(self.n_layers, self.hidden, self.intermediate, self.n_heads, self.n_kv_heads, self.vocab,
                      self.max_seq, self.max_batch)


def token_bytes(cfg, ctx_len, batch=1):
    """Algorithmic bytes one decode step reads: every weight once, the KV
    cache of each of the batch's sequences up to ctx_len, the embedding rows,
    norms and activations ignored."""
    h, i, L = cfg.hidden, cfg.intermediate, cfg.n_layers
    qkv = (cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim
    per_layer = q4k_bytes(qkv, h) + q4k_bytes(h, cfg.n_heads * cfg.head_dim) + q4k_bytes(2 * i, h) + q4k_bytes(h, i)
    kv = 2 * ctx_len * cfg.n_kv_heads * cfg.head_dim * 2
    return L * (per_layer + batch * kv) + q6k_bytes(cfg.vocab, h)


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
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def positions_needed(args):
    """Cache positions a run appends after the prefix: the checked tokens,
    warm-up, timed steps and the per-token e2e steps."""
    return NCHECK + args.warmup + 2 * args.steps + 8


def llama8b(max_seq):
    return Cfg(32, 4096, 14336, 32, 8, 128256, max_seq)


def llama70b(max_seq, max_batch=1):
    return Cfg(80, 8192, 28672, 64, 8, 128256, max_seq, max_batch)


def model_cfg(args):
    # The capacity is a whole number of 1024-position blocks independent of the
    # step counts in the usual range, so every run of one model (any N, any
    # K/W up to a few hundred) builds the same cache and attention split plan.
    cap = args.ctx + 1024 * max(1, -(-positions_needed(args) // 1024))
    # the 70B model holds BATCH16 sequences: batch 1 and batch 16 run on one copy of the weights
    c = llama70b(cap, BATCH16) if args.model == "70b" else llama8b(cap)
    if args.layers and args.layers != c.n_layers:
        c = c.cut(args.layers)
    return c


def workload_name(args, world=1):
    if args.model == "70b":
        name = "decode70b: Llama-3-70B arch (80 layers, hidden 8192, 64/8 heads, FFN 28672, vocab 128256) " \
               "Q4_K_M, f16 KV prefilled to %d, batch 1, greedy, tensor parallel over %d GPU(s)" % (args.ctx, world)
        full = 80
    else:
        name = "decode8b: Llama-3-8B arch (32 layers, hidden 4096, 32/8 heads, FFN 14336, vocab 128256) Q4_K_M, " \
               "f16 KV prefilled to %d, batch 1, greedy" % args.ctx
        full = 32
        if world > 1:
            name += ", tensor parallel over %d GPUs" % world
    if args.layers and args.layers != full:
        name = name.replace("%d layers" % full, "%d of its %d layers" % (args.layers, full))
    return name


def config_dict(args, world, cfg):
    """The `config` of both arms' lines (identical by construction)."""
    tb = token_bytes(cfg, args.ctx + NCHECK + args.warmup + args.steps // 2)
    return {"workload": workload_name(args, world), "global_batch": 1, "seq_len": args.ctx,
            "parallelism": "tp%d" % world if world > 1 else "single",
            "l2": "inputs larger than L2 (%.2f GB streamed per step)" % (tb / 1e9)}


# ---------------------------------------------------------------- CPU baseline

def host_ram_available():
    try:
        import psutil
        return psutil.virtual_memory().available
    except Exception:
        return 0


def oracle_model_bytes(cfg, ctx_len):
    """Host bytes of the oracle holding cfg: quant blocks plus the f32 KV cache."""
    qkv = (cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim
    layer = q4k_bytes(qkv, cfg.hidden) + q4k_bytes(cfg.hidden, cfg.n_heads * 128) + \
        q4k_bytes(2 * cfg.intermediate, cfg.hidden) + q4k_bytes(cfg.hidden, cfg.intermediate)
    kv = 2 * cfg.max_seq * cfg.n_kv_heads * cfg.head_dim * 4
    return cfg.n_layers * (layer + kv) + q6k_bytes(cfg.vocab, cfg.hidden) + q4k_bytes(cfg.vocab, cfg.hidden)


def cpu_decode(cfg, ctx_len, ntokens, warmup, max_seconds=None):
    """The reference CPU path (oracle restatement of Transformer.Forward) on
    the host cores: greedy tokens/s over the same synthetic model.  Stops
    after ntokens, or once max_seconds have passed (at least one token)."""
    import oracle
    t0 = time.time()
    om = oracle.synthetic_model(cfg, SEED, n_seq=1, kv_len=ctx_len)
    build_s = time.time() - t0
    tok = START_TOKEN
    pos = ctx_len
    for _ in range(warmup):
        tok = oracle.argmax(om.forward(0, tok, pos))
        pos += 1
    n = 0
    t1 = time.perf_counter()
    while n < ntokens and (max_seconds is None or n == 0 or time.perf_counter() - t1 < max_seconds):
        tok = oracle.argmax(om.forward(0, tok, pos))
        pos += 1
        n += 1
    dt = time.perf_counter() - t1
    del om
    threads = oracle.nthreads()
    return {"value": n / dt, "unit": "tok/s", "cores": threads, "kind": "port", "tokens": n, "warmup": warmup,
            "ms_per_step": dt / n * 1e3, "timed_s": dt, "build_s": build_s,
            "sample": "%d greedy decode steps (after %d warm-up) of the same %d-layer Q4_K_M model at ctx %d "
                      "(weights dequantised row by row, f32 arithmetic of TensorOps, KV values rounded through "
                      "f16), %d threads" % (n, warmup, cfg.n_layers, ctx_len, threads)}


def cpu_decode_cuts(cfg, ctx_len, steps, max_seconds):
    """A model whose oracle does not fit host memory: the oracle decodes the
    model cut to 2 and to 10 layers (at least `steps` tokens each, timed
    alone), and a token of the whole model is t2 + (L - 2) (t10 - t2) / 8."""
    r2 = cpu_decode(cfg.cut(2), ctx_len, steps, 2, max_seconds=max_seconds / 3)
    r10 = cpu_decode(cfg.cut(10), ctx_len, steps, 2, max_seconds=2 * max_seconds / 3)
    t2, t10 = r2["ms_per_step"], r10["ms_per_step"]
    t = t2 + (cfg.n_layers - 2) * max(t10 - t2, 0.0) / 8
    return {"value": 1e3 / t, "unit": "tok/s", "cores": r2["cores"], "kind": "port",
            "tokens": r2["tokens"] + r10["tokens"], "warmup": 4, "ms_per_step": t,
            "timed_s": r2["timed_s"] + r10["timed_s"], "build_s": r2["build_s"] + r10["build_s"],
            "sample": "host memory too small for the whole model: the oracle decoded it cut to 2 layers (%d steps, "
                      "%.1f ms/token) and to 10 layers (%d steps, %.1f ms/token) at ctx %d, %d threads; a %d-layer "
                      "token is t2 + %d (t10 - t2) / 8 = %.1f ms"
                      % (r2["tokens"], t2, r10["tokens"], t10, ctx_len, r2["cores"], cfg.n_layers,
                         cfg.n_layers - 2, t)}


def cpu_sample(cfg, ctx_len, steps, warmup, seconds):
    """The oracle decoding the whole model when the host holds it (with room
    to spare), else the layer-cut estimate."""
    if host_ram_available() > 1.5 * oracle_model_bytes(cfg, ctx_len) + (8 << 30):
        return cpu_decode(cfg, ctx_len, steps, warmup, max_seconds=seconds)
    return cpu_decode_cuts(cfg, ctx_len, max(steps, 20), seconds)


def run_reference(args, world, rank):
    """The reference arm: rank 0 alone times the oracle port of the
    reference's CPU path; the other ranks exit at once."""
    if rank != 0:
        return
    cfg = model_cfg(args)
    warm = args.warmup if cfg.n_layers <= 32 else 1
    r = cpu_sample(cfg, args.ctx, args.steps, warm, args.ref_seconds)
    line = {"metric": METRIC, "value": round(r["value"], 4), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": r["tokens"], "warmup": r["warmup"], "ms_per_step": round(r["ms_per_step"], 2),
            "timed_s": round(r["timed_s"], 2), "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Q4_K_M weights and f16 KV prefix; no checkpoint offline)", "impl": "reference",
            "config": config_dict(args, world, cfg),
            "cpu_baseline": {k: (round(v, 4) if isinstance(v, float) else v) for k, v in r.items()
                             if k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": round(r["value"], 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------- GPU measurements

def graph_ms(ctx, torch, fn, reps):
    """Average ms of fn(i) over `reps` launches captured in one CUDA graph on
    the context stream (host launch overhead outside the timing)."""
    s = ctx.torch_stream
    for i in range(3):
        fn(i)
    ctx.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(reps):
            fn(i)
    g.replay()
    ctx.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    g.replay()
    e1.record(s)
    ctx.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del g
    return ms


def matvec_roofline(ctx, torch, dev, rows=2 * 14336, cols=4096, reps=40):
    """Average duration of the fused gate/up Q4_K matvec (rows x cols; 28672 x
    4096 for the 8B model) over `reps` launches on rotating weight copies
    (together > 250 MB, twice the L2), captured in one CUDA graph."""
    from sharpinfer_b200 import native as N
    from sharpinfer_b200.backend import synth_f32_host
    ncopy = max(4, -(-250_000_000 // q4k_bytes(rows, cols)))
    ws = [ctx.synth_weight(N.SI_Q4_K, rows, cols, SEED + i, 77, N.SYNTH_MODEL, 1.0 / (23.3 * 64.0))
          for i in range(ncopy)]
    x = torch.from_numpy(synth_f32_host(cols, SEED, 78)).to(dev).reshape(1, -1)
    y = torch.empty((1, rows), device=dev)
    ctx.act_prepare(x)
    ms = graph_ms(ctx, torch, lambda i: ctx.qmatvec_prepared(ws[i % ncopy], 1, out=y), reps)
    for w in ws:
        w.free()
    return ms, q4k_bytes(rows, cols) + 4 * (cols + rows)


# (name, qtype, rows, cols): the single 4096 x 4096 Q4_K matvec and the 8B
# layer set -- fused gate/up and down Q4_K, Q6_K lm_head, Q8_0 4096 x 4096
MATVEC_SHAPES = (("q4k_4096x4096", 12, 4096, 4096), ("q4k_gateup_28672x4096", 12, 28672, 4096),
                 ("q4k_down_4096x14336", 12, 4096, 14336), ("q6k_lmhead_128256x4096", 14, 128256, 4096),
                 ("q8_0_4096x4096", 8, 4096, 4096))


def matvec_set(ctx, torch, dev, batches=(1, 4, 16)):
    """The matvec set at each batch: microseconds per call of si_qmatvec
    (activation preparation + matvec) and of the matvec alone on prepared
    activations, each averaged over 40 graph-captured launches on rotating
    weight copies (together > 250 MB, twice the L2); GB/s of the algorithmic
    bytes (weights + f32 x and y) against the measured HBM peak."""
    from sharpinfer_b200 import native as N
    from sharpinfer_b200.backend import synth_f32_host
    peak, _ = measured_peaks()
    wbytes = {12: q4k_bytes, 14: q6k_bytes, 8: q8_bytes}
    rows_out = []
    for name, qt, rows, cols in MATVEC_SHAPES:
        wb = wbytes[qt](rows, cols)
        ncopy = max(2, -(-250_000_000 // wb))
        ws = [ctx.synth_weight(qt, rows, cols, SEED + i, 90 + qt, N.SYNTH_PLAIN, 0.01) for i in range(ncopy)]
        for B in batches:
            x = torch.from_numpy(synth_f32_host(B * cols, SEED, 91)).to(dev).reshape(B, cols)
            y = torch.empty((B, rows), device=dev)
            nbytes = wb + 4 * B * (rows + cols)
            us_op = 1e3 * graph_ms(ctx, torch, lambda i: ctx.qmatvec(ws[i % ncopy], x, out=y), 40)
            ctx.act_prepare(x)
            us_k = 1e3 * graph_ms(ctx, torch, lambda i: ctx.qmatvec_prepared(ws[i % ncopy], B, out=y), 40)
            rows_out.append({"shape": name, "batch": B, "bytes": nbytes, "us_call": round(us_op, 2),
                             "us_kernel": round(us_k, 2), "gbs_call": round(nbytes / us_op / 1e3, 1),
                             "gbs_kernel": round(nbytes / us_k / 1e3, 1),
                             "frac_kernel": round(nbytes / us_k / 1e3 / peak, 4)})
            del x, y
        for w in ws:
            w.free()
    return rows_out


PREFILL_SHAPES = ((4096, 4096), (14336, 4096), (4096, 14336))  # (N rows, K cols): q/o, gate/up, down


def prefill_set(ctx, torch, dev, M, reps):
    """Prefill GEMM (si_qgemm, tcgen05) on the 8B projection shapes at M
    tokens, y = x W^T with W Q4_K in HBM and x bf16 resident: whole-call ms
    per shape (dequantisation, conversion and GEMM); the gate/up shape again
    with its f16 weight cached (conversion + tensor-core GEMM only); and
    flash prefill attention at seq = M, causal, 32 q / 8 kv heads, d = 128."""
    from sharpinfer_b200 import native as N
    flops = tot_ms = 0.0
    rows = []
    cached = None
    last = None
    for n, k in PREFILL_SHAPES:
        w = ctx.synth_weight(N.SI_Q4_K, n, k, SEED, 91, N.SYNTH_MODEL, 1.0 / (23.3 * 64.0))
        x = torch.randn(M, k, device=dev).to(torch.bfloat16)
        y = torch.empty(M, n, device=dev)
        ms = graph_ms(ctx, torch, lambda i: ctx.qgemm(w, x, out=y), reps)
        fl = 2.0 * M * n * k
        flops += fl
        tot_ms += ms
        rows.append({"N": n, "K": k, "us": round(ms * 1e3, 1), "tflops": round(fl / ms / 1e9, 1)})
        if n == 14336:
            ctx.qgemm_cache_weight(w)
            cached = (fl, graph_ms(ctx, torch, lambda i: ctx.qgemm(w, x, out=y), reps))
        last = (x, y, w)
        w.free()
    H, Hkv = 32, 8
    q = torch.randn(1, H, M, 128, device=dev).to(torch.bfloat16)
    kk = torch.randn(1, Hkv, M, 128, device=dev).to(torch.bfloat16)
    vv = torch.randn(1, Hkv, M, 128, device=dev).to(torch.bfloat16)
    ao = torch.empty(1, H, M, 128, device=dev)
    att_ms = graph_ms(ctx, torch, lambda i: ctx.attn_prefill(q, kk, vv, 1.0 / 128 ** 0.5, True, out=ao), reps)
    att_flops = 4.0 * M * M * 128 * H / 2
    del q, kk, vv, ao, last
    return {"M": M, "tflops": round(flops / tot_ms / 1e9, 1), "ms": round(tot_ms, 4), "shapes": rows,
            "gateup_cached_tflops": round(cached[0] / cached[1] / 1e9, 1),
            "attention": {"seq": M, "heads": "32/8", "us": round(att_ms * 1e3, 1),
                          "tflops": round(att_flops / att_ms / 1e9, 1)}}


def decode_batch16(ctx, torch, m, cfg, pos0, steps=16):
    """BATCH16 sequences (prefilled KV, distinct start tokens) decoded
    together from pos0: the first 4 greedy tokens of every sequence, then
    ms per step of a graph-replayed greedy loop timed with CUDA events."""
    toks = [(START_TOKEN + 7919 * b) % cfg.vocab for b in range(BATCH16)]
    chk = m.generate(toks, pos0, 4)
    w = m.generate([int(v) for v in chk[-1]], pos0 + 4, 3)
    s = ctx.torch_stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx.synchronize()
    e0.record(s)
    m.generate([int(v) for v in w[-1]], pos0 + 7, steps)
    e1.record(s)
    ctx.synchronize()
    return e0.elapsed_time(e1) / steps, [[int(v) for v in row] for row in chk.T]


def batch16_entry(cfg, ctx_len, ms, steps, world, tokens):
    peak, _ = measured_peaks()
    tb = token_bytes(cfg, ctx_len + 7 + steps // 2, BATCH16)
    return {"batch": BATCH16, "tok_s": round(BATCH16 * 1e3 / ms, 2), "ms_per_step": round(ms, 3), "steps": steps,
            "bytes_per_step": tb, "decode_roofline_frac": round(tb / (ms * 1e-3) / 1e9 / (peak * world), 4),
            "tokens_check": tokens}


def tp1_70b(ctx, torch, args):
    """The 70B model decoded on this one GPU: its first NCHECK greedy tokens
    (the tensor-parallel runs must produce the same ones) and tok/s of a
    graph-replayed greedy loop timed with CUDA events."""
    from sharpinfer_b200.model import DecodeModel
    a70 = argparse.Namespace(**vars(args))
    a70.model, a70.ctx, a70.layers = "70b", KV_LEN_70B, 0
    cfg = model_cfg(a70)
    m = DecodeModel(ctx, cfg.native())
    m.synth(SEED)
    m.kv_synth(a70.ctx, SEED)
    chk = m.generate([START_TOKEN], a70.ctx, NCHECK)
    pos = a70.ctx + NCHECK
    tok = int(chk[-1, 0])
    w = m.generate([tok], pos, 3)
    pos += 3
    n = 32
    s = ctx.torch_stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx.synchronize()
    e0.record(s)
    m.generate([int(w[-1, 0])], pos, n)
    e1.record(s)
    ctx.synchronize()
    ms = e0.elapsed_time(e1) / n
    ms16, chk16 = decode_batch16(ctx, torch, m, cfg, a70.ctx)
    m.free()
    peak, _ = measured_peaks()
    tb = token_bytes(cfg, a70.ctx + NCHECK + 3 + n // 2)
    return {"workload": workload_name(a70, 1), "tok_s": round(1e3 / ms, 2), "ms_per_token": round(ms, 3),
            "steps": n, "decode_roofline_frac": round(tb / (ms * 1e-3) / 1e9 / peak, 4),
            "tokens_check": [int(v) for v in chk[:, 0]],
            "batch16": batch16_entry(cfg, a70.ctx, ms16, 16, 1, chk16)}


def tp_parity_gpu(ctx, args, world, rank):
    """TP = world decode of the 70B architecture cut to 2 layers (full hidden
    size, heads, FFN and vocabulary; ctx 8192): 4 greedy steps with logits.
    Returns (tokens, this rank's logit slices)."""
    from sharpinfer_b200.model import DecodeModel, exchange_handles
    cfg = llama70b(KV_LEN_70B + 1024, BATCH16).cut(2)
    m = DecodeModel(ctx, cfg.native(), tp=world, rank=rank)
    m.synth(SEED)
    m.kv_synth(KV_LEN_70B, SEED)
    m.tp_connect(exchange_handles(m.tp_handle()))
    toks, logits = [START_TOKEN], []
    for s in range(4):
        out, lg = m.step([toks[-1]], KV_LEN_70B + s, logits=True)
        toks.append(int(out[0]))
        logits.append(lg[0].copy())
    # one batch-16 step: every sequence from its own prefilled KV
    t16 = [(START_TOKEN + 7919 * b) % cfg.vocab for b in range(BATCH16)]
    out16, lg16 = m.step(t16, KV_LEN_70B, logits=True)
    logits.append(lg16.copy())
    toks.append([t16, [int(v) for v in out16]])
    ctx.synchronize()
    return m, toks, logits


def tp_parity_check(toks, slices):
    """Rank 0, after the GPUs are done: the oracle's forward pass over the
    same 2-layer 70B cut, fed the same tokens, against the gathered logits."""
    import oracle

    def rel_l2(a, b):
        a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
        return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))

    cfg = llama70b(KV_LEN_70B + 1024, BATCH16).cut(2)
    om = oracle.synthetic_model(cfg, SEED, n_seq=BATCH16, kv_len=KV_LEN_70B)
    worst, equal = 0.0, True
    for s in range(4):
        lg = np.concatenate([sl[s] for sl in slices])
        ref = om.forward(0, toks[s], KV_LEN_70B + s)
        worst = max(worst, rel_l2(lg, ref))
        equal = equal and (toks[s + 1] == oracle.argmax(ref))
    t16, out16 = toks[5]
    lg16 = np.concatenate([sl[4] for sl in slices], axis=1)
    worst16, equal16 = 0.0, True
    for b in range(BATCH16):
        ref = om.forward(b, t16[b], KV_LEN_70B)
        worst16 = max(worst16, rel_l2(lg16[b], ref))
        equal16 = equal16 and (out16[b] == oracle.argmax(ref))
    return {"workload": "Llama-3-70B arch cut to 2 layers, TP over all GPUs, ctx %d: 4 greedy steps at batch 1, "
                        "then one step at batch %d" % (KV_LEN_70B, BATCH16),
            "max_rel_l2": float("%.3g" % worst), "tokens_equal": bool(equal), "tokens": toks[1:5],
            "batch16_max_rel_l2": float("%.3g" % worst16), "batch16_tokens_equal": bool(equal16),
            "batch16_tokens": out16, "bar": 1e-3}


def run_ours(args, world, rank, local):
    import torch
    import torch.distributed as dist
    from sharpinfer_b200 import B200Context
    from sharpinfer_b200.model import DecodeModel

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=600))
    dev = torch.device("cuda", local)
    ctx = B200Context(local)
    torch.cuda.set_stream(ctx.torch_stream)
    cfg = model_cfg(args)
    m = DecodeModel(ctx, cfg.native(), tp=world, rank=rank)
    m.synth(SEED)
    m.kv_synth(args.ctx, SEED)
    if world > 1:  # tensor parallelism: map every rank's partial-sum buffer
        from sharpinfer_b200.model import exchange_handles
        m.tp_connect(exchange_handles(m.tp_handle()))
    stream = ctx.torch_stream
    # the first NCHECK greedy tokens (captures the decode graph), then warm-up
    chk = m.generate([START_TOKEN], args.ctx, NCHECK)
    wtok = m.generate([int(chk[-1, 0])], args.ctx + NCHECK, args.warmup)
    pos = args.ctx + NCHECK + args.warmup
    tok = int(wtok[-1, 0])
    ctx.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    gen = m.generate([tok], pos, args.steps)
    e1.record(stream)
    ctx.synchronize()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    pos += args.steps
    tok = int(gen[-1, 0])
    # e2e: the per-token host call (token id in, argmax out, synchronous)
    for _ in range(3):
        tok = int(m.step([tok], pos)[0])
        pos += 1
    if world > 1:
        dist.barrier()
    w0 = time.perf_counter()
    for _ in range(args.steps):
        tok = int(m.step([tok], pos)[0])
        pos += 1
    e2e_ms = (time.perf_counter() - w0) * 1e3 / args.steps
    kernels_per_step = m.step_kernels(1)
    ms16, chk16 = 0.0, None
    if args.model == "70b" and not args.no_extras:  # the same model at batch 16 (from the prefilled KV again)
        if world > 1:
            dist.barrier()
        ms16, chk16 = decode_batch16(ctx, torch, m, cfg, args.ctx)
    ctx.synchronize()
    if world > 1:
        dist.barrier()  # every rank is done with the peers' buffers before any is freed
    m.free()
    # the dominant kernel: this rank's fused gate/up matvec
    gu_rows, gu_cols = 2 * cfg.intermediate // world, cfg.hidden
    kern_ms, kern_bytes = matvec_roofline(ctx, torch, dev, gu_rows, gu_cols)
    t = torch.tensor([ms, e2e_ms, kern_ms, ms16], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, kern_ms, ms16 = t.tolist()

    extra = {}
    par = None
    if world > 1 and not args.no_parity:
        pm, ptoks, plg = tp_parity_gpu(ctx, args, world, rank)
        got = [None] * world
        dist.all_gather_object(got, plg)
        dist.barrier()
        pm.free()
        par = (ptoks, got)
    if world == 1 and args.model == "8b" and not args.no_extras:
        clk2 = ClockSampler(local)
        clk2.start()
        mv = matvec_set(ctx, torch, dev)
        pf = [prefill_set(ctx, torch, dev, M, max(args.warmup, 5)) for M in (512, 2048)]
        clk_x = clk2.stop()
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
            os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
        c1 = next(r for r in mv if r["shape"] == "q4k_4096x4096" and r["batch"] == 1)
        extra["matvec"] = {"c1_q4k_4096x4096_b1": {k: c1[k] for k in ("gbs_call", "gbs_kernel", "frac_kernel",
                                                                      "us_call", "us_kernel")},
                           "shapes": mv, "l2": "rotating weight copies, > 250 MB per shape",
                           "peak_gbs": measured_peaks()[0], "clocks": clk_x}
        extra["prefill"] = {"runs": pf, "peak_tflops": peaks.get("bf16_tflops", 1590.0),
                            "dtype": "f16 x f16 -> f32 (tcgen05 kind::f16)"}
        extra["tp1_70b"] = tp1_70b(ctx, torch, args)
    ctx.synchronize()
    torch.cuda.set_stream(torch.cuda.default_stream(dev))
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return  # the CPU work below runs with the other ranks gone
    peak, peak_kind = measured_peaks()
    achieved = kern_bytes / (kern_ms * 1e-3) / 1e9
    tb = token_bytes(cfg, args.ctx + NCHECK + args.warmup + args.steps // 2)
    # ncu measured the 8B shape (no re-reads); other shapes: the same bytes per unit
    traffic = GATEUP_TRAFFIC if (gu_rows, gu_cols) == (28672, 4096) else int(kern_bytes)
    line = {
        "metric": METRIC, "value": round(1e3 / ms, 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "q4_k/q6_k weights x f32 activations (f16 hi/lo MMA, f32 accumulate), f16 KV",
        "data": "synthetic (seeded Q4_K_M weights and f16 KV prefix; no checkpoint offline)",
        "config": config_dict(args, world, cfg),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": "k_qmv1 (batch-1 Q4_K), fused gate/up %dx%d (%.1f MB)" % (gu_rows, gu_cols,
                                                                                      kern_bytes / 1e6),
                     "peak_source": peak_kind + " (burst copy)"},
        "decode_roofline": {"bytes_per_token": tb, "achieved_gbs": round(tb / (ms * 1e-3) / 1e9, 1),
                            "frac": round(tb / (ms * 1e-3) / 1e9 / (peak * world), 4)},
        "e2e": {"value": round(1e3 / e2e_ms, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 * world,
                "d2h_bytes_per_step": 4 * world},
        "gpu_launches": kernels_per_step * args.steps * world,
        "clocks": clk,
        "tokens_check": [int(v) for v in chk[:, 0]],
    }
    if chk16 is not None:
        line["batch16"] = batch16_entry(cfg, args.ctx, ms16, 16, world, chk16)
        line["batch16"]["workload"] = workload_name(args, world).replace("batch 1,", "batch %d," % BATCH16)
    line.update(extra)
    if par is not None:
        line["parity"] = tp_parity_check(par[0], par[1])
    if not args.no_cpu_baseline:
        cb = cpu_sample(cfg, args.ctx, 10 ** 6, 1, args.cpu_seconds)
        line["cpu_baseline"] = {k: (round(v, 4) if isinstance(v, float) else v) for k, v in cb.items()
                                if k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps(line), flush=True)


def run_matvec(args):
    """--workload matvec: the matvec set alone (value: the 4096 x 4096 Q4_K
    batch-1 call in GB/s)."""
    import torch
    from sharpinfer_b200 import B200Context
    dev = torch.device("cuda", 0)
    ctx = B200Context(0)
    torch.cuda.set_stream(ctx.torch_stream)
    peak, peak_kind = measured_peaks()
    clocks = ClockSampler(0)
    clocks.start()
    rows_out = matvec_set(ctx, torch, dev)
    clk = clocks.stop()
    from sharpinfer_b200 import native as N
    w = ctx.synth_weight(12, 4096, 4096, SEED, 92, N.SYNTH_PLAIN, 0.01)
    from sharpinfer_b200.backend import synth_f32_host
    xh = synth_f32_host(4096, SEED, 93).reshape(1, 4096)
    for _ in range(5):
        ctx.qmatvec_host(w, xh)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ctx.qmatvec_host(w, xh)
    e2e_us = (time.perf_counter() - t0) * 1e6 / args.steps
    w.free()
    c1 = next(r for r in rows_out if r["shape"] == "q4k_4096x4096" and r["batch"] == 1)
    gu = next(r for r in rows_out if r["shape"] == "q4k_gateup_28672x4096" and r["batch"] == 1)
    line = {"metric": METRIC, "value": c1["gbs_call"], "unit": "GB/s", "n_gpus": 1, "steps": 40,
            "warmup": 3, "ms_per_step": round(c1["us_call"] / 1e3, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q4_k/q6_k/q8_0 weights x f32 activations (f16 hi/lo MMA, f32 accumulate)",
            "data": "synthetic (seeded quant blocks, x ~ N(0, 1))",
            "config": {"workload": "matvec: 4096x4096 Q4_K and the 8B layer set at batch 1/4/16",
                       "l2": "rotating weight copies, > 250 MB per shape"},
            "shapes": rows_out,
            "roofline": {"bound": "hbm", "achieved": gu["gbs_kernel"], "peak": peak, "unit": "GB/s",
                         "frac": gu["frac_kernel"], "traffic": GATEUP_TRAFFIC,
                         "kernel": "k_qmv1, fused gate/up 28672x4096, batch 1", "peak_source": peak_kind},
            "e2e": {"value": round((4096 * 16 * 144 + 8 * 4096) / e2e_us / 1e3, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": 4 * 4096, "d2h_bytes_per_step": 4 * 4096},
            "gpu_launches": 3 * 40 * len(rows_out), "clocks": clk}
    print(json.dumps(line), flush=True)
    ctx.synchronize()
    torch.cuda.set_stream(torch.cuda.default_stream(dev))
    ctx.close()


def run_prefill(args, local):
    """--workload prefill: the prefill GEMM at --prefill-m tokens (value:
    whole-call TFLOP/s over the three 8B projection shapes)."""
    import torch
    from sharpinfer_b200 import B200Context
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = B200Context(local)
    torch.cuda.set_stream(ctx.torch_stream)
    M = args.prefill_m
    clocks = ClockSampler(local)
    clocks.start()
    r = prefill_set(ctx, torch, dev, M, args.steps)
    clk = clocks.stop()
    # e2e: x from pinned host memory, y back to host, every call (gate/up shape)
    from sharpinfer_b200 import native as N
    n, k = 14336, 4096
    w = ctx.synth_weight(N.SI_Q4_K, n, k, SEED, 91, N.SYNTH_MODEL, 1.0 / (23.3 * 64.0))
    x = torch.randn(M, k, device=dev).to(torch.bfloat16)
    y = torch.empty(M, n, device=dev)
    xh = x.cpu().pin_memory()
    yh = torch.empty(M, n, pin_memory=True)
    for _ in range(2):
        x.copy_(xh, non_blocking=True)
        ctx.qgemm(w, x, out=y)
        yh.copy_(y, non_blocking=True)
    ctx.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        x.copy_(xh, non_blocking=True)
        ctx.qgemm(w, x, out=y)
        yh.copy_(y, non_blocking=True)
    ctx.synchronize()
    host_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    w.free()
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    peak = peaks.get("bf16_tflops", 1590.0)
    line = {"metric": "prefill GEMM TFLOP/s (Llama-3-8B Q4_K projections, bf16 activations)",
            "value": r["tflops"], "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
            "warmup": 3, "ms_per_step": r["ms"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 x f16 -> f32 (tcgen05 kind::f16)", "data": "synthetic",
            "config": {"workload": "prefill%d: M=%d x (N,K) in %s, Q4_K weights" % (M, M, list(PREFILL_SHAPES)),
                       "l2": "weights and activations per shape > L2 (HBM-resident)"},
            "shapes": r["shapes"], "attention": r["attention"],
            "roofline": {"bound": "tensor", "achieved": r["gateup_cached_tflops"], "peak": peak, "unit": "TFLOP/s",
                         "frac": round(r["gateup_cached_tflops"] / peak, 4), "traffic": None,
                         "kernel": "k_gemm_tc (+ bf16->f16 conversion), N=14336 K=4096, f16 weight cached",
                         "peak_source": "measured" if peaks else "fallback"},
            "e2e": {"value": round(2.0 * M * n * k / host_ms / 1e9, 1), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": M * k * 2, "d2h_bytes_per_step": M * n * 4},
            "gpu_launches": 3 * 3 * args.steps, "clocks": clk}
    print(json.dumps(line), flush=True)
    del x, y, xh, yh
    ctx.synchronize()
    torch.cuda.set_stream(torch.cuda.default_stream(dev))
    torch.cuda.synchronize()
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--ref-seconds", type=float, default=60.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the matvec / prefill / 70B keys of the N=1 line")
    ap.add_argument("--no-parity", action="store_true", help="skip the tensor-parallel parity check (N > 1)")
    ap.add_argument("--model", default=None, choices=["8b", "70b"],
                    help="decode model (default: 8b on one GPU, 70b tensor parallel on several)")
    ap.add_argument("--layers", type=int, default=0, help="transformer layers (0: the whole model)")
    ap.add_argument("--ctx", type=int, default=0, help="prefilled KV positions (0: 4096 for 8b, 8192 for 70b)")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "matvec"])
    ap.add_argument("--prefill-m", type=int, default=2048, help="tokens of the prefill GEMM workload")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup()
    if args.model is None:
        args.model = "70b" if world > 1 else "8b"
    if not args.ctx:
        args.ctx = KV_LEN_70B if args.model == "70b" else KV_LEN
    if args.impl == "reference":
        run_reference(args, world, rank)
    elif args.workload == "prefill":
        if rank == 0:
            run_prefill(args, local)
    elif args.workload == "matvec":
        if rank == 0:
            run_matvec(args)
    else:
        run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
