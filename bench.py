#!/usr/bin/env python3
"""Benchmark of the B200 layer-stack forward (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C3] [--impl tk|reference]

A "step" is one forward of the layer stack over one synthetic batch of the
chosen configuration (default C3: batch 256, seq 256, d_model 1024, 16
heads, ffn 4096, 4 layers, bidirectional -- the large-batch GEMM regime that
BASELINE.json runs at 1/2/4/8 GPUs). Weights are the harness's default
initialisation under torch.manual_seed(0); x ~ N(0, 1) fp32, seeded on the
CPU. Batch rows are independent, so under torchrun every rank runs its own
full batch on its own GPU with no data-path collective (weak scaling); the
value is all ranks' tokens over the max-over-ranks device time.

Metric: tokens/s (= B*S*1000 / ms per forward, the harness's throughput,
src/torch_transformer_benchmark.py:565-567). ``value`` is device-timed with
inputs resident in HBM (inputs are > L2, so no flush is needed); ``e2e``
times the same forward through the public API with the input copied from
pinned host memory and the fp32 output copied back every step.

``--impl reference`` times the fp32 CPU forward of the reference model (the
oracle's restatement of BaselineTransformer; the reference is pure Python
and does not travel to the GPU box) on the host cores, one bounded
batch-slice per step. For C5 and A14 (S = 100,000) the CPU forward of even
one sequence is ~10^14 FLOP per layer, so the CPU figure is extrapolated from
the exact query-chunked oracle: two one-layer runs over all keys with 8 and R
query rows give the per-row cost and the all-row (LayerNorm / K / V) cost,
scaled to S rows and L layers. A14 is the reference's case 14
(configs/shapes.json: batch 32, seq 100000, d 1024, 16 heads, ffn 1024, 2
layers).

C1 and C2 fit in L2: their steps are timed one by one with an L2 flush
(a 512 MB write) between them, outside the events. Larger configurations
exceed L2 and are timed back to back.
"""

from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parent
PKG = ROOT / "transformer-kernel_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402

# name: (B, S, d, H, ffn, L, causal)
CONFIGS = {
    "C1": (64, 128, 128, 4, 128, 4, True),
    "C2": (1, 512, 512, 8, 2048, 4, True),
    "C3": (256, 256, 1024, 16, 4096, 4, False),
    "C4": (8, 8192, 1024, 16, 4096, 2, True),
    "C5": (32, 100000, 1024, 16, 4096, 1, True),
    # configs/shapes.json case 14: the reference's out-of-core case (2 layers, ffn 1024)
    "A14": (32, 100000, 1024, 16, 1024, 2, True),
}
# The reference's published numbers for the same metric and shape (one T4):
# C1 is appendix case 1 (pass-2 default, 1.405 ms = 5.83 M tokens/s,
# results/pass2-default.json); A14 is appendix case 14 (155.4 s per forward,
# 20,597 tokens/s, results/case14-full.json). No other config was published.
PUBLISHED_TOKENS_PER_S = {"C1": 5.83e6, "A14": 20597.0}
# The reference's appendix shapes (configs/shapes.json; every case causal):
# case: (B, S, d, H, ffn, L), with its best published T4 time in ms
# (README.md:298-312 pass two; case 14: README.md:401-405).
APPENDIX = {
    1: ((64, 128, 128, 4, 128, 4), 1.42), 2: ((1, 128, 128, 4, 128, 4), 0.30),
    3: ((4, 128, 128, 4, 128, 4), 0.31), 4: ((16, 128, 128, 4, 128, 4), 0.43),
    5: ((128, 128, 128, 4, 128, 4), 2.66), 6: ((10000, 128, 128, 4, 128, 4), 198.57),
    7: ((64, 128, 32, 4, 32, 4), 1.60), 8: ((64, 128, 1024, 4, 1024, 4), 25.23),
    9: ((64, 128, 128, 1, 128, 4), 1.43), 10: ((64, 128, 128, 2, 128, 4), 1.50),
    11: ((64, 128, 128, 16, 128, 4), 2.18), 12: ((64, 32, 128, 4, 128, 4), 0.42),
    13: ((64, 1024, 128, 4, 128, 4), 18.75), 14: ((32, 100000, 1024, 16, 1024, 2), 155400.0),
}
# timed steps when --steps is not given (C5: ~1 s per forward on one GPU)
DEFAULT_STEPS = {"C5": 3, "A14": 3}
# configurations whose working set fits in the 126 MB L2: flush it between steps
L2_RESIDENT = ("C1", "C2")
METRIC = "layer-stack forward tokens/s"


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        m = json.loads(path.read_text())
        return m["hbm_gbs"], m["bf16_tflops"], m["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def gemm_flops(T, d, ffn):
    return {"gemm_qkv": 2 * T * d * 3 * d, "gemm_o": 2 * T * d * d, "gemm_o_ln": 2 * T * d * d,
            "gemm_ffn_in": 2 * T * d * ffn, "gemm_ffn_out": 2 * T * ffn * d, "gemm_ffn_out_ln": 2 * T * ffn * d}


def attn_flops(B, S, H, hd, causal):
    pairs = S * (S + 1) / 2 if causal else S * S
    return 4 * B * H * pairs * hd


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi while timing."""

    FIELDS = "timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        import tempfile

        self.path = tempfile.mktemp(prefix="tk_clocks_", suffix=".csv")
        try:
            # -f writes each sample straight to the file (a pipe would be
            # block-buffered and lost when the sampler is stopped).
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.index), "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.5)  # first sample lands before the timed region
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.3)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            try:
                self.lines = [ln for ln in pathlib.Path(self.path).read_text().splitlines() if ln.strip()]
                os.unlink(self.path)
            except OSError:
                self.lines = []

    def mark(self, which: str) -> None:
        """Record the host time at the start / end of the timed region."""
        setattr(self, which, time.time())

    def summary(self):
        """Median SM clock and throttle reasons over the samples taken inside
        the timed region (marked with mark('t_start') / mark('t_end'))."""
        import datetime

        lo = getattr(self, "t_start", 0.0) - 0.05
        hi = getattr(self, "t_end", float("inf")) + 0.05
        sms, maxes, reasons, outside = [], [], set(), 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                sm, smax = float(f[2]), float(f[3])
            except ValueError:
                continue
            if not (lo <= ts <= hi):
                outside += 1
                continue
            sms.append(sm)
            maxes.append(smax)
            for name, flag in zip(names, f[6:10]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms), "period_ms": 50}


def cpu_forward_rate(cfg_tuple, seconds, sample_batch, steps=None):
    """Oracle (fp32 CPU BaselineTransformer restatement) tokens/s on a
    batch slice. Returns (tokens_per_s, threads, description)."""
    from oracle import StackConfig, generate_random_case, init_params, stack_forward

    B, S, d, H, ffn, L, causal = cfg_tuple
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    nb = min(B, sample_batch)
    cfg = StackConfig(nb, S, d, H, ffn, L, causal)
    params = init_params(cfg, seed=0)
    x, mask = generate_random_case(cfg, seed=1234 + 100000)
    stack_forward(params, cfg, x[:1], mask[:1])  # warm
    times = []
    t_end = time.perf_counter() + seconds
    n = 0
    while True:
        t0 = time.perf_counter()
        stack_forward(params, cfg, x, mask)
        times.append(time.perf_counter() - t0)
        n += 1
        if (steps is not None and n >= steps) or (steps is None and time.perf_counter() >= t_end):
            break
    med = statistics.median(times)
    return nb * S / med, threads, f"{nb} of {B} sequences x {n} forwards, median {med * 1e3:.1f} ms", times


def cpu_long_seq_rate(cfg_tuple, rows=1024, reps=2):
    """fp32 CPU tokens/s for one long sequence, extrapolated: the exact
    query-chunked oracle is run for one layer over all S keys with 8 and with
    `rows` evenly spread query rows (best of `reps` each); t(R) = t0 + R *
    t_row gives the per-row cost t_row and the all-row part t0 (LayerNorm, K
    and V projections); one layer of one sequence costs t0 + S * t_row, and
    the L layers of the stack L times that (every layer does the same work).
    Returns (tokens_per_s, threads, description, [seconds per sequence])."""
    from oracle import StackConfig, generate_random_case, init_params, stack_forward_rows

    B, S, d, H, ffn, L, causal = cfg_tuple
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = StackConfig(1, S, d, H, ffn, 1, causal)
    params = init_params(cfg, seed=0)
    x, _ = generate_random_case(cfg, seed=1234 + 100000)

    def timed(n):
        idx = torch.linspace(0, S - 1, n).round().long()
        t0 = time.perf_counter()
        stack_forward_rows(params, cfg, x, idx, None, q_chunk=64)
        return time.perf_counter() - t0

    timed(8)  # warm
    t_lo = min(timed(8) for _ in range(reps))
    t_hi = min(timed(rows) for _ in range(reps))
    t_row = max(t_hi - t_lo, 1e-9) / (rows - 8)
    t_seq = L * (max(t_lo - 8 * t_row, 0.0) + S * t_row)
    desc = (f"1 of {B} sequences, extrapolated: query-chunked oracle, one layer over all {S} keys with 8 and "
            f"{rows} spread query rows (best of {reps}: {t_lo:.2f} s, {t_hi:.2f} s), x {L} layers -> "
            f"{t_seq:.1f} s per sequence")
    return S / t_seq, threads, desc, [t_seq]


def run_reference(args, cfg_tuple, rank):
    """--impl reference: the CPU fp32 reference forward on the host cores."""
    if rank != 0:
        return
    B, S, d, H, ffn, L, causal = cfg_tuple
    if args.config in ("C5", "A14"):
        value, threads, desc, times = cpu_long_seq_rate(cfg_tuple)
        med, sample = times[0], 1
    else:
        sample = 8 if args.config in ("C3",) else (1 if args.config == "C4" else B)
        rate, threads, desc, times = cpu_forward_rate(cfg_tuple, 0, sample, steps=args.warmup + args.steps)
        times = times[args.warmup:] or times
        med = statistics.median(times)
        value = min(B, sample) * S / med
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": med * 1e3 * (B / min(B, sample)), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": f"{args.config} b{B} s{S} d{d} h{H} ffn{ffn} L{L} {'causal' if causal else 'bidir'}",
                   "global_batch": B, "seq_len": S, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": desc if args.config in ("C5", "A14") else f"{min(B, sample)} of {B} sequences per step"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_sweep(args):
    """Appendix-shape sweep on one GPU (the reference's src/sweep.py runs the
    same 14 shapes through its harness): per case, the public drop-in
    (graph-replayed when a forward is short), warm-up, then the median of
    per-forward CUDA-event samples with an L2 flush between samples; one JSON
    line per case with the reference's best published T4 time beside it."""
    import dataclasses

    import _tklib as tk
    import cuda_graphs
    import optimized

    overrides = {}
    for item in args.set:
        key, _, value = item.partition("=")
        overrides[key] = value == "True" if value in ("True", "False") else value
    if overrides:
        optimized.configure(**overrides)
    cases = sorted(APPENDIX) if args.sweep == "all" else [int(c) for c in args.sweep.split(",")]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    scratch = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    for case in cases:
        (B, S, d, H, ffn, L), t4_ms = APPENDIX[case]
        cfg = optimized.TransformerConfig(B, S, d, H, ffn, L, True)
        torch.manual_seed(0)
        big = B * S >= 1_000_000
        model = (optimized.OptimizedTransformer(cfg) if big else cuda_graphs.GraphedTransformer(cfg)).to(dev).eval()
        gen = torch.Generator().manual_seed(1234 + 100000)
        x = torch.randn(B, S, d, generator=gen).to(dev)
        mask = torch.ones(B, S, dtype=torch.bool, device=dev)
        samples = []
        with torch.inference_mode():
            for _ in range((0 if big else cuda_graphs.WARMUP_BEFORE_CAPTURE + 1) + 3):
                model(x, mask)
            torch.cuda.synchronize(dev)
            n = 3 if big else (args.steps if args.steps else 30)
            for _ in range(n):
                scratch.fill_(1)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                model(x, mask)
                b.record(stream)
                samples.append((a, b))
            torch.cuda.synchronize(dev)
        ms = statistics.median(a.elapsed_time(b) for a, b in samples)
        line = {"case": case, "shape": {"batch": B, "seq": S, "d_model": d, "heads": H, "ffn": ffn, "layers": L,
                                        "causal": True},
                "ms": ms, "tokens_per_s": B * S * 1000.0 / ms, "samples": n,
                "reference_t4_ms": t4_ms, "speedup_vs_reference_t4": t4_ms / ms,
                "path": ("one-launch stack kernel" if model.settings.fused_small_stack
                         and tk.lib().tk_stack_small_supported(d, H, ffn, S) else "per-layer kernels"),
                "settings": dataclasses.asdict(model.settings)}
        print(json.dumps(line), flush=True)
        del model, x
        torch.cuda.empty_cache()
    return 0


def run_strong(args, cfg_tuple):
    """Strong scaling in one process: the public ShardedTransformer splits
    the batch over --gpus local GPUs (input handed over on cuda:0, shards
    copied over NVLink, per-device graph replicas, outputs gathered back on
    cuda:0). cuda:0's current stream waits on every device, so CUDA events
    on it time the whole sharded forward (the max over devices)."""
    import _tklib as tk
    import optimized
    import sharded

    B, S, d, H, ffn, L, causal = cfg_tuple
    n = args.gpus
    if torch.cuda.device_count() < n:
        raise SystemExit(f"--strong --gpus {n}: only {torch.cuda.device_count()} GPUs visible")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    torch.manual_seed(0)
    model = optimized.OptimizedTransformer(optimized.TransformerConfig(B, S, d, H, ffn, L, causal)).to(dev).eval()
    shard = sharded.ShardedTransformer(model, [f"cuda:{i}" for i in range(n)])
    gen = torch.Generator().manual_seed(1234 + 100000)
    x_host = torch.randn(B, S, d, generator=gen).pin_memory()
    mask = torch.ones(B, S, dtype=torch.bool, device=dev)
    x = x_host.to(dev)
    out_host = torch.empty(B, S, d, dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(dev)
    with torch.inference_mode():
        import cuda_graphs
        for _ in range(cuda_graphs.WARMUP_BEFORE_CAPTURE + 1 + args.warmup):
            shard(x, mask)
        for i in range(n):
            tk.check_device_errors(torch.device("cuda", i))
        torch.cuda.synchronize(dev)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(0) as clk:
            clk.mark("t_start")
            t0.record(stream)
            for _ in range(args.steps):
                shard(x, mask)
            t1.record(stream)
            torch.cuda.synchronize(dev)
            clk.mark("t_end")
        ms = t0.elapsed_time(t1) / args.steps
        # end to end: pinned host input -> cuda:0 -> sharded forward -> pinned host output
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            x.copy_(x_host, non_blocking=True)
            out_host.copy_(shard(x, mask), non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = e0.elapsed_time(e1) / args.steps
        for i in range(n):
            tk.check_device_errors(torch.device("cuda", i))
    tokens = B * S
    line = {
        "metric": METRIC, "value": tokens * 1000.0 / ms, "unit": "tokens/s", "n_gpus": n, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16 operands / f32 accumulate+residual", "data": "synthetic",
        "config": {"workload": f"{args.config} b{B} s{S} d{d} h{H} ffn{ffn} L{L} {'causal' if causal else 'bidir'}",
                   "global_batch": B, "seq_len": S,
                   "parallelism": f"dp{n} in one process (batch split over {n} GPUs, NVLink scatter/gather)",
                   "l2": "inputs and activations > 126 MB L2; no flush"},
        "e2e": {"value": tokens * 1000.0 / e2e_ms, "unit": "tokens/s", "ms_per_step": e2e_ms,
                "path": "pinned host -> cuda:0 -> ShardedTransformer -> pinned host",
                "h2d_bytes_per_step": x_host.numel() * 4, "d2h_bytes_per_step": out_host.numel() * 4},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


def measured_traffic(config, kernel, batch):
    """DRAM bytes (read + write) per launch of `kernel` from the committed ncu
    summary profiles/dram_traffic.json, captured on a smaller batch of the
    same configuration and scaled by rows (the kernels' traffic is
    proportional to the batch); None when no capture covers it."""
    path = ROOT / "profiles" / "dram_traffic.json"
    try:
        table = json.loads(path.read_text())
        entry = table[config][kernel]
    except (OSError, KeyError, ValueError):
        return None
    return entry["bytes_per_launch"] * batch / entry["batch"]


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default 60; C5: 3)")
    ap.add_argument("--warmup", type=int, default=None, help="untimed warm-up steps (default 5; C5: 3)")
    ap.add_argument("--config", default="C3", choices=sorted(CONFIGS))
    ap.add_argument("--batch", type=int, default=0, help="override the config's batch (small profiling cases)")
    ap.add_argument("--impl", default="tk", choices=["tk", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="bounded CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-chunks", type=int, default=4, help="batch slices of the streamed end-to-end forward")
    ap.add_argument("--sweep", default="", help="comma-separated appendix cases (or 'all'): one JSON line each, "
                                                "timed like the harness (median of CUDA-event samples)")
    ap.add_argument("--set", action="append", default=[], metavar="FIELD=VALUE",
                    help="--sweep: override an OptimizerSettings field (e.g. fused_small_stack=False)")
    ap.add_argument("--strong", action="store_true",
                    help="one process drives --gpus local GPUs: the config's batch is split across them "
                         "(ShardedTransformer, NVLink scatter/gather) -- strong scaling")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = DEFAULT_STEPS.get(args.config, 60)
    if args.warmup is None:
        args.warmup = 3 if args.config in ("C5", "A14") else 5
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg_tuple = CONFIGS[args.config]
    if args.batch > 0:
        cfg_tuple = (args.batch,) + cfg_tuple[1:]
    B, S, d, H, ffn, L, causal = cfg_tuple

    if args.impl == "reference":
        run_reference(args, cfg_tuple, rank)
        return 0
    if args.sweep:
        return run_sweep(args)
    if args.strong:
        if world > 1:
            ap.error("--strong runs in one process; do not launch it under torchrun")
        return run_strong(args, cfg_tuple)

    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    import _tklib as tk
    import cuda_graphs
    import optimized

    ocfg = optimized.TransformerConfig(B, S, d, H, ffn, L, causal)
    torch.manual_seed(0)
    # The public graph-replaying drop-in (the reference's --cuda-graphs
    # path); its eager superclass forward is used for the per-kernel trace.
    # C5 (one ~1 s forward per step) runs the eager drop-in: a graph saves
    # nothing there and its static input/output copies would cost 26 GB.
    graphed = args.config not in ("C5", "A14")
    model = (cuda_graphs.GraphedTransformer(ocfg) if graphed else optimized.OptimizedTransformer(ocfg)).to(dev).eval()
    eager_forward = optimized.OptimizedTransformer.forward
    gen = torch.Generator().manual_seed(1234 + 100000)
    x_host = torch.randn(B, S, d, generator=gen).pin_memory()
    mask_host = torch.ones(B, S, dtype=torch.bool).pin_memory()
    x = x_host.to(dev)
    mask = mask_host.to(dev)
    out_host = torch.empty(B, S, d, dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    flush = args.config in L2_RESIDENT
    scratch = torch.empty(512 << 20, dtype=torch.uint8, device=dev) if flush else None

    with torch.inference_mode():
        # ---- graph capture (untimed), then device-resident timing ----
        if graphed:
            for _ in range(cuda_graphs.WARMUP_BEFORE_CAPTURE + 1):
                model(x, mask)
        for _ in range(args.warmup):
            model(x, mask)
        tk.check_device_errors(dev)
        barrier()
        torch.cuda.synchronize(dev)
        with Clocks(local) as clk:
            clk.mark("t_start")
            if flush:
                # one event pair per step; the L2 flush between steps is outside them
                pairs = []
                for _ in range(args.steps):
                    scratch.fill_(1)
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record(stream)
                    model(x, mask)
                    b.record(stream)
                    pairs.append((a, b))
                torch.cuda.synchronize(dev)
                local_ms = sum(a.elapsed_time(b) for a, b in pairs) / args.steps
            else:
                t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                t0.record(stream)
                for _ in range(args.steps):
                    model(x, mask)
                t1.record(stream)
                torch.cuda.synchronize(dev)
                local_ms = t0.elapsed_time(t1) / args.steps
            clk.mark("t_end")
        barrier()
        ms = max_over_ranks(local_ms)
        clocks = clk.summary()
        tk.check_device_errors(dev)

        # ---- per-kernel event timing (separate pass, same stream) ----
        trace = []
        model.launch_trace = trace
        for _ in range(args.steps):
            eager_forward(model, x, mask)
        torch.cuda.synchronize(dev)
        model.launch_trace = None
        per = {}
        for name, a, b in trace:
            per.setdefault(name, []).append(a.elapsed_time(b))
        launches_per_step = len(trace) // args.steps

        # ---- end to end: pinned host input -> forward -> host output ----
        # Large batches go through the public streamed API (H2D, forward
        # and D2H of batch slices overlap); small ones copy in, replay the
        # graph and copy out.
        streamed = x_host.numel() * 4 >= (64 << 20)
        chunks = args.e2e_chunks

        def e2e_step():
            if streamed:
                model.forward_from_host(x_host, mask_host, out_host=out_host, chunks=chunks)
            else:
                x.copy_(x_host, non_blocking=True)
                out_host.copy_(model(x, mask), non_blocking=True)

        for _ in range(3):
            e2e_step()
        barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)

    tokens = B * S
    value = world * tokens * 1000.0 / ms
    hbm, tf_burst, tf_sus, peak_kind = peaks()
    # dominant kernel by total time
    totals = {k: sum(v) for k, v in per.items()}
    dom = max(totals, key=totals.get)
    avg_ms = statistics.fmean(per[dom])
    T = tokens
    fl = gemm_flops(T, d, ffn)
    if dom in fl:
        achieved = fl[dom] / (avg_ms * 1e-3) / 1e12
        roof = {"kernel": dom, "bound": "tensor", "achieved": achieved, "peak": tf_sus, "unit": "TFLOP/s",
                "frac": achieved / tf_sus, "peak_kind": f"{peak_kind} bf16 sustained"}
    elif dom == "stack_small":
        # the whole forward is one kernel: all GEMM and attention FLOP of the stack
        g = gemm_flops(T, d, ffn)
        total = L * (g["gemm_qkv"] + g["gemm_o"] + g["gemm_ffn_in"] + g["gemm_ffn_out"]
                     + attn_flops(B, S, H, d // H, causal))
        achieved = total / (avg_ms * 1e-3) / 1e12
        roof = {"kernel": dom, "bound": "tensor", "achieved": achieved, "peak": tf_sus, "unit": "TFLOP/s",
                "frac": achieved / tf_sus, "peak_kind": f"{peak_kind} bf16 sustained",
                "note": "one-launch whole-stack kernel; latency-bound at this size"}
    elif dom == "attn":
        achieved = attn_flops(B, S, H, d // H, causal) / (avg_ms * 1e-3) / 1e12
        roof = {"kernel": dom, "bound": "tensor", "achieved": achieved, "peak": tf_sus, "unit": "TFLOP/s",
                "frac": achieved / tf_sus, "peak_kind": f"{peak_kind} bf16 sustained"}
    else:
        achieved = T * d * (4 + 2) / (avg_ms * 1e-3) / 1e9
        roof = {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "peak_kind": f"{peak_kind} copy"}
    roof["traffic"] = measured_traffic(args.config, dom, B)
    share = {k: round(v / sum(totals.values()), 4) for k, v in sorted(totals.items(), key=lambda kv: -kv[1])}
    kernels_ms = {k: round(statistics.fmean(v), 5) for k, v in per.items()}

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return 0

    cpu = None
    if not args.no_cpu_baseline:
        if args.config in ("C5", "A14"):
            rate, threads, desc, _ = cpu_long_seq_rate(cfg_tuple)
        else:
            sample = 8 if args.config == "C3" else (1 if args.config == "C4" else B)
            rate, threads, desc, _ = cpu_forward_rate(cfg_tuple, args.cpu_seconds, sample)
        cpu = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": desc}

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (value / PUBLISHED_TOKENS_PER_S[args.config]
                        if args.config in PUBLISHED_TOKENS_PER_S and args.batch == 0 else None),
        "dtype": "f16 operands / f32 accumulate+residual", "data": "synthetic",
        "config": {"workload": f"{args.config} b{B} s{S} d{d} h{H} ffn{ffn} L{L} {'causal' if causal else 'bidir'}",
                   "global_batch": B * world, "seq_len": S, "parallelism": f"dp{world} (batch-sharded, no collective)",
                   "l2": ("L2 flushed between steps (512 MB write outside the events)" if flush
                          else "inputs and activations > 126 MB L2; no flush")},
        "e2e": {"value": world * tokens * 1000.0 / e2e_ms, "unit": "tokens/s", "ms_per_step": e2e_ms,
                "path": f"forward_from_host, {chunks} streamed slices" if streamed else "copy in, graph replay, copy out",
                "h2d_bytes_per_step": x_host.numel() * 4, "d2h_bytes_per_step": out_host.numel() * 4},
        "roofline": roof,
        "kernel_ms": kernels_ms,
        "kernel_share": share,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
