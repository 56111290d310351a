#!/usr/bin/env python3
"""Benchmark of the B200 layer-stack forward (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C3] [--impl tk|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      # the batch split over N GPUs

A "step" is one forward of the layer stack over one synthetic batch of the
chosen configuration (default C3: batch 256, seq 256, d_model 1024, 16
heads, ffn 4096, 4 layers, bidirectional -- the large-batch GEMM regime that
BASELINE.json runs at 1/2/4/8 GPUs). Weights are the harness's default
initialisation under torch.manual_seed(0); x ~ N(0, 1) fp32, seeded on the
CPU (the harness's generator and init; no dataset is involved).

One GPU: the public graph-replaying drop-in (GraphedTransformer) on the
whole batch. N GPUs (torchrun, one process per GPU): the north-star split
(distributed.BatchSplitForward) -- the batch lives in rank 0's HBM, every
rank computes its shard of sequences, and the fp32 output is gathered back
into rank 0's HBM over NVLink inside the timed step (strong scaling: the
global batch is the config's at every N). ``--replicas`` instead runs the
whole batch on every rank (weak scaling, no exchange).

Metric: tokens/s (= B*S*1000 / ms per forward, the harness's throughput,
src/torch_transformer_benchmark.py:565-567). ``value`` is device-timed with
inputs resident in HBM (inputs are > L2, so no flush is needed), the max
over ranks; ``e2e`` times the same forward through the public API from
pinned host memory, the fp32 output copied back every step
(``forward_from_host``; under torchrun each rank streams its own shard).
``roofline`` is the dominant kernel's achieved rate over the measured burst
peak (per-launch CUDA-event times of a separate traced pass), and
``roofline_per_kernel`` lists every kernel the same way. ``extra_configs``
carries the other BASELINE.json configurations measured the same way
(C1, C2, C4, C5 on one GPU; C4 and C5 split over the N GPUs under torchrun).

``--impl reference`` times the fp32 CPU forward of the reference model (the
oracle's restatement of BaselineTransformer; the reference is pure Python
and does not travel to the GPU box) on the host cores, one bounded
batch-slice per step; ``ms_per_step`` is the measured slice time and the
full-batch extrapolation has its own key. For C5 and A14 (S = 100,000) the
CPU forward of even one sequence is ~10^14 FLOP per layer, so the CPU figure
is extrapolated from the exact query-chunked oracle: two one-layer runs over
all keys with 8 and R query rows give the per-row cost and the all-row
(LayerNorm / K / V) cost, scaled to S rows and L layers. A14 is the
reference's case 14 (configs/shapes.json: batch 32, seq 100000, d 1024, 16
heads, ffn 1024, 2 layers).

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
    """(HBM GB/s, bf16 burst TFLOP/s, bf16 sustained TFLOP/s, source)."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        m = json.loads(path.read_text())
        return m["hbm_gbs"], m["bf16_tflops"], m["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def attn_flops(B, S, H, hd, causal):
    """Useful attention FLOP: 4 * B * H * hd per unmasked (query, key) pair."""
    pairs = S * (S + 1) / 2 if causal else S * S
    return 4 * B * H * pairs * hd


def kernel_work(name, cfg_tuple, batch):
    """Algorithmic work of one launch of kernel `name` in a forward over
    `batch` sequences: ("tensor", FLOP) for GEMMs and attention (2*M*N*K;
    4*B*H*hd*pairs) or ("hbm", bytes) for LayerNorm (rows*d*bytes per
    element: ln_in reads fp32 x and writes fp16 h plus the fp32 residual
    copy, 10 B; ln reads fp32 and writes fp16, 6 B; ln_out writes fp32, 8 B)."""
    _, S, d, H, ffn, L, causal = cfg_tuple
    T = batch * S
    gemm = {"gemm_qkv": (d, 3 * d), "gemm_o": (d, d), "gemm_o_ln": (d, d), "gemm_ffn_in": (d, ffn),
            "gemm_ffn_out": (ffn, d), "gemm_ffn_out_ln": (ffn, d)}
    if name in gemm:
        k, n = gemm[name]
        return "tensor", 2.0 * T * n * k
    if name == "attn":
        return "tensor", attn_flops(batch, S, H, d // H, causal)
    if name == "stack_small":
        per_layer = 2.0 * T * (4 * d * d + 2 * d * ffn) + attn_flops(batch, S, H, d // H, causal)
        return "tensor", L * per_layer
    per_elt = {"ln_in": 10, "ln": 6, "ln_out": 8}.get(name, 6)
    return "hbm", float(T * d * per_elt)


def roofline_table(per, cfg_tuple, batch, config_name=None):
    """Per-kernel rooflines from per-launch CUDA-event times (ms lists), each
    against the measured burst peak (the kernels are timed launch by launch,
    not inside a seconds-long loop); returns (table, dominant kernel's entry)."""
    hbm, tf_burst, tf_sus, kind = peaks()
    totals = {k: sum(v) for k, v in per.items()}
    grand = sum(totals.values()) or 1.0
    table = {}
    for name, times in per.items():
        bound, work = kernel_work(name, cfg_tuple, batch)
        avg = statistics.fmean(times)
        if bound == "tensor":
            achieved, peak, unit = work / (avg * 1e-3) / 1e12, tf_burst, "TFLOP/s"
        else:
            achieved, peak, unit = work / (avg * 1e-3) / 1e9, hbm, "GB/s"
        table[name] = {"bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
                       "frac": round(achieved / peak, 4), "avg_ms": round(avg, 5),
                       "launches_per_step": None, "share": round(totals[name] / grand, 4)}
    dom = max(totals, key=totals.get)
    e = table[dom]
    roof = {"kernel": dom, "bound": e["bound"], "achieved": e["achieved"], "peak": e["peak"], "unit": e["unit"],
            "frac": e["frac"],
            "peak_kind": f"{kind} {'bf16 burst' if e['bound'] == 'tensor' else 'copy'}",
            "frac_of_sustained": (round(e["achieved"] / tf_sus, 4) if e["bound"] == "tensor" else None),
            "traffic": measured_traffic(config_name, dom, batch) if config_name else None}
    return table, roof


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


def workload(name, cfg_tuple):
    B, S, d, H, ffn, L, causal = cfg_tuple
    return f"{name} b{B} s{S} d{d} h{H} ffn{ffn} L{L} {'causal' if causal else 'bidir'}"


def run_reference(args, cfg_tuple, rank):
    """--impl reference: the CPU fp32 reference forward on the host cores,
    one bounded batch slice per step; under torchrun rank 0 alone runs."""
    if rank != 0:
        return
    B, S, d, H, ffn, L, causal = cfg_tuple
    if args.config in ("C5", "A14"):
        value, threads, desc, times = cpu_long_seq_rate(cfg_tuple)
        slice_ms, sample = times[0] * 1e3, 1
        sample_desc = desc
    else:
        sample = min(B, 8 if args.config in ("C3",) else (1 if args.config == "C4" else B))
        rate, threads, desc, times = cpu_forward_rate(cfg_tuple, 0, sample, steps=args.warmup + args.steps)
        times = times[args.warmup:] or times
        slice_ms = statistics.median(times) * 1e3
        value = sample * S * 1000.0 / slice_ms
        sample_desc = f"{sample} of {B} sequences per step (median of {len(times)} timed steps)"
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": slice_ms, "higher_is_better": True,
        "scaling": "strong" if args.gpus > 1 and not args.replicas else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": workload(args.config, cfg_tuple), "global_batch": B, "seq_len": S},
        "parallelism": "cpu (host cores of rank 0)",
        "step_sample": sample_desc,
        "full_batch_ms_extrapolated": slice_ms * B / sample,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample_desc},
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


def trace_kernels(model, x, mask, steps):
    """Per-launch CUDA-event times of every kernel over `steps` eager forwards
    (separate pass, same stream): {name: [ms, ...]}, launches per forward."""
    import optimized

    trace = []
    model.launch_trace = trace
    for _ in range(steps):
        optimized.OptimizedTransformer.forward(model, x, mask)
    torch.cuda.synchronize(x.device)
    model.launch_trace = None
    per = {}
    for name, a, b in trace:
        per.setdefault(name, []).append(a.elapsed_time(b))
    return per, len(trace) // steps


def attach_launch_counts(table, per, steps):
    for name, times in per.items():
        table[name]["launches_per_step"] = len(times) // steps
    return table


def timed_steps(fn, steps, stream, dev, flush_buf=None):
    """Mean ms per step of `fn` on `stream`: back to back between one event
    pair, or (with `flush_buf`) one event pair per step with an L2 flush
    (a write larger than L2) between steps, outside the events."""
    if flush_buf is None:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            fn()
        t1.record(stream)
        torch.cuda.synchronize(dev)
        return t0.elapsed_time(t1) / steps
    pairs = []
    for _ in range(steps):
        flush_buf.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        pairs.append((a, b))
    torch.cuda.synchronize(dev)
    return sum(a.elapsed_time(b) for a, b in pairs) / steps


def device_input(cfg_tuple, dev, seed=1234 + 100000):
    """x ~ N(0, 1) fp32 drawn on the device (seeded) for the extra
    configurations, whose inputs reach 13 GB."""
    B, S, d = cfg_tuple[:3]
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return torch.randn(B, S, d, device=dev, generator=g)


def measure_one_gpu(name, dev, steps=None, warmup=3):
    """One GPU, device-resident: ms per forward, tokens/s, the dominant
    kernel's roofline and the per-kernel table, clocks (extra configurations
    of the default run)."""
    import _tklib as tk
    import cuda_graphs
    import optimized

    cfg_tuple = CONFIGS[name]
    B, S, d, H, ffn, L, causal = cfg_tuple
    steps = steps or (2 if name in ("C5", "A14") else 20)
    torch.manual_seed(0)
    ocfg = optimized.TransformerConfig(B, S, d, H, ffn, L, causal)
    graphed = name not in ("C5", "A14")
    model = (cuda_graphs.GraphedTransformer(ocfg) if graphed else optimized.OptimizedTransformer(ocfg)).to(dev).eval()
    x = device_input(cfg_tuple, dev)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev) if name in L2_RESIDENT else None
    with torch.inference_mode():
        for _ in range((cuda_graphs.WARMUP_BEFORE_CAPTURE + 1 if graphed else 0) + warmup):
            model(x)
        tk.check_device_errors(dev)
        with Clocks(dev.index) as clk:
            clk.mark("t_start")
            ms = timed_steps(lambda: model(x), steps, stream, dev, flush)
            clk.mark("t_end")
        per, launches = trace_kernels(model, x, None, max(1, min(steps, 5)))
        tk.check_device_errors(dev)
    table, roof = roofline_table(per, cfg_tuple, B, name)
    attach_launch_counts(table, per, max(1, min(steps, 5)))
    del model, x
    torch.cuda.empty_cache()
    return {"workload": workload(name, cfg_tuple), "ms_per_step": ms, "value": B * S * 1000.0 / ms,
            "unit": "tokens/s", "steps": steps, "warmup": warmup,
            "vs_baseline": (B * S * 1000.0 / ms / PUBLISHED_TOKENS_PER_S[name]
                            if name in PUBLISHED_TOKENS_PER_S else None),
            "l2": "flushed between steps" if flush is not None else "working set > L2",
            "data": "synthetic, x drawn on the device", "roofline": roof, "roofline_per_kernel": table,
            "gpu_launches_per_step": launches, "clocks": clk.summary()}


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
    ap.add_argument("--e2e-chunks", type=int, default=0,
                    help="batch slices of the streamed end-to-end forward (default: ~16+ sequences a slice, <= 2)")
    ap.add_argument("--extras", default="auto",
                    help="comma-separated extra configurations measured after the main one (default: C1,C2,C4,C5 "
                         "on one GPU, C4,C5 split under torchrun); 'none' to skip")
    ap.add_argument("--micro-batches", type=int, default=2,
                    help="torchrun split: micro-batches per rank (copy-in / forward / copy-out overlap)")
    ap.add_argument("--replicas", action="store_true",
                    help="torchrun: every rank runs the whole batch (weak scaling, no exchange)")
    ap.add_argument("--split", action="store_true",
                    help="run the batch-split path (the torchrun default) even on one GPU")
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

    if args.impl == "reference":
        run_reference(args, cfg_tuple, rank)
        return 0
    if args.sweep:
        return run_sweep(args)
    if args.strong:
        if world > 1:
            ap.error("--strong runs in one process; do not launch it under torchrun")
        return run_strong(args, cfg_tuple)
    if (world > 1 and not args.replicas) or args.split:
        if world == 1:
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", "29561")
            os.environ.setdefault("RANK", "0")
            os.environ.setdefault("WORLD_SIZE", "1")
        return run_split(args, cfg_tuple, world, rank, local)
    return run_single(args, cfg_tuple, world, rank, local)


def cpu_baseline(args, cfg_tuple):
    if args.no_cpu_baseline:
        return None
    B = cfg_tuple[0]
    if args.config in ("C5", "A14"):
        rate, threads, desc, _ = cpu_long_seq_rate(cfg_tuple)
    else:
        sample = 8 if args.config == "C3" else (1 if args.config == "C4" else B)
        rate, threads, desc, _ = cpu_forward_rate(cfg_tuple, args.cpu_seconds, sample)
    return {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": desc}


def e2e_chunks(args, batch):
    if args.e2e_chunks > 0:
        return args.e2e_chunks
    return max(1, min(2, batch // 16))


def extras_list(args, world):
    if args.extras == "none" or args.batch > 0:
        return []
    if args.extras != "auto":
        return [c for c in args.extras.split(",") if c and c != args.config]
    if world > 1:
        return [c for c in ("C4", "C5") if c != args.config]
    return [c for c in ("C1", "C2", "C4", "C5") if c != args.config]


def run_single(args, cfg_tuple, world, rank, local):
    """One GPU (or --replicas: every rank its own whole batch)."""
    import torch.distributed as dist
    from datetime import timedelta

    B, S, d, H, ffn, L, causal = cfg_tuple
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
    # path). C5 (one ~1 s forward per step) runs the eager drop-in: a graph
    # saves nothing there.
    graphed = args.config not in ("C5", "A14")
    model = (cuda_graphs.GraphedTransformer(ocfg) if graphed else optimized.OptimizedTransformer(ocfg)).to(dev).eval()
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

    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev) if args.config in L2_RESIDENT else None
    with torch.inference_mode():
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
            local_ms = timed_steps(lambda: model(x, mask), args.steps, stream, dev, flush)
            clk.mark("t_end")
        barrier()
        ms = max_over_ranks(local_ms)
        clocks = clk.summary()
        tk.check_device_errors(dev)

        trace_steps = max(1, min(args.steps, 10))
        per, launches_per_step = trace_kernels(model, x, mask, trace_steps)

        # end to end: pinned host input -> forward -> pinned host output,
        # through the public streamed API (copies overlap the forward, also
        # across consecutive calls); small batches copy in, replay, copy out
        streamed = x_host.numel() * 4 >= (64 << 20)
        chunks = e2e_chunks(args, B)

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
        e2e_ms = max_over_ranks(timed_steps(e2e_step, args.steps, stream, dev))
        barrier()

    tokens = B * S
    value = world * tokens * 1000.0 / ms
    table, roof = roofline_table(per, cfg_tuple, B, args.config if args.batch == 0 else None)
    attach_launch_counts(table, per, trace_steps)

    extras = {}
    if rank == 0 and world == 1:
        del model, x
        torch.cuda.empty_cache()
        for name in extras_list(args, world):
            extras[name] = measure_one_gpu(name, dev)
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return 0
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (value / PUBLISHED_TOKENS_PER_S[args.config]
                        if args.config in PUBLISHED_TOKENS_PER_S and args.batch == 0 else None),
        "dtype": "f16 operands / f32 accumulate+residual", "data": "synthetic",
        "config": {"workload": workload(args.config, cfg_tuple), "global_batch": B * world, "seq_len": S},
        "parallelism": ("1 GPU" if world == 1 else f"{world} replicas (each rank the whole batch, no exchange)"),
        "l2": ("L2 flushed between steps (512 MB write outside the events)" if flush is not None
               else "inputs and activations > 126 MB L2; no flush"),
        "e2e": {"value": world * tokens * 1000.0 / e2e_ms, "unit": "tokens/s", "ms_per_step": e2e_ms,
                "path": (f"forward_from_host, {chunks} streamed slices per call, consecutive calls pipelined"
                         if streamed else "copy in, graph replay, copy out"),
                "h2d_bytes_per_step": x_host.numel() * 4, "d2h_bytes_per_step": out_host.numel() * 4},
        "roofline": roof,
        "roofline_per_kernel": table,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu_baseline(args, cfg_tuple),
        "extra_configs": extras,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_split(args, cfg_tuple, world, rank, local):
    """torchrun, one process per GPU: the north-star split of one batch."""
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    try:
        main_line = split_config(args, args.config, cfg_tuple, world, rank, local, dev, host_input=True)
        extras = {}
        for name in extras_list(args, world):
            extras[name] = split_config(args, name, CONFIGS[name], world, rank, local, dev, host_input=False)
        if rank == 0:
            main_line["extra_configs"] = extras
            print(json.dumps(main_line), flush=True)
        dist.barrier(device_ids=[local])
    finally:
        dist.destroy_process_group()
    return 0


def split_config(args, name, cfg_tuple, world, rank, local, dev, host_input):
    """One configuration through distributed.BatchSplitForward; returns the
    JSON line (meaningful on rank 0)."""
    import torch.distributed as dist

    import _tklib as tk
    import distributed
    import optimized
    from sharded import shard_bounds

    B, S, d, H, ffn, L, causal = cfg_tuple
    main = host_input
    steps = args.steps if main else (2 if name in ("C5", "A14") else 20)
    warmup = args.warmup if main else 3
    torch.manual_seed(0)  # identical weights on every rank
    model = optimized.OptimizedTransformer(optimized.TransformerConfig(B, S, d, H, ffn, L, causal)).to(dev).eval()
    split = distributed.BatchSplitForward(model, (B, S, d), micro_batches=args.micro_batches)
    b0, b1 = split.bounds
    x_host = None
    if main:
        gen = torch.Generator().manual_seed(1234 + 100000)
        x_host = torch.randn(B, S, d, generator=gen).pin_memory()
        if rank == 0:
            split.input.copy_(x_host)
    elif rank == 0:
        split.input.copy_(device_input(cfg_tuple, dev))
    stream = torch.cuda.current_stream(dev)

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.inference_mode():
        for _ in range(2 + warmup):  # slot graphs are captured on a slot's second use
            split.step()
        tk.check_device_errors(dev)
        dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)
        with Clocks(local) as clk:
            clk.mark("t_start")
            local_ms = timed_steps(split.step, steps, stream, dev)
            clk.mark("t_end")
        dist.barrier(device_ids=[local])
        ms = max_over_ranks(local_ms)
        tk.check_device_errors(dev)
        clocks = [None] * world
        dist.all_gather_object(clocks, clk.summary())

        # parity: the gathered rows of the first and last sequence of every
        # rank's shard against a one-GPU forward of those sequences on rank 0
        parity = None
        if rank == 0:
            picks = sorted({v for r in range(world) for v in
                            (shard_bounds(B, world, r)[0], shard_bounds(B, world, r)[1] - 1)
                            if shard_bounds(B, world, r)[1] > shard_bounds(B, world, r)[0]})
            worst, exact = 0.0, True
            per_chunk = 4 if S * d <= (1 << 22) else 1
            for i in range(0, len(picks), per_chunk):
                idx = torch.tensor(picks[i:i + per_chunk], device=dev)
                want = model(split.input.index_select(0, idx))
                got = split.output.index_select(0, idx)
                diff = (want - got).abs().max().item()
                worst = max(worst, diff)
                exact = exact and bool(torch.equal(want, got))
            parity = {"sequences_checked": len(picks), "against": "one-GPU forward of the same sequences",
                      "bit_exact": exact, "max_abs_diff": worst}

        # per-kernel times on this rank's micro-batch shape (rank 0)
        per, launches = {}, 0
        mb = split.micro[0][1] - split.micro[0][0] if split.micro else 0
        if rank == 0 and mb:
            xs = split.slots[0]["x"][:mb]
            per, launches = trace_kernels(model, xs, None, 3 if main else 1)

        # end to end: every rank streams its own shard from pinned host memory
        e2e_ms = None
        if main:
            xs_host = x_host[b0:b1]
            os_host = torch.empty_like(xs_host).pin_memory()
            chunks = e2e_chunks(args, b1 - b0)
            if b1 > b0:
                for _ in range(3):
                    model.forward_from_host(xs_host, None, out_host=os_host, chunks=chunks)
            dist.barrier(device_ids=[local])
            torch.cuda.synchronize(dev)
            e2e_local = timed_steps(lambda: model.forward_from_host(xs_host, None, out_host=os_host, chunks=chunks)
                                    if b1 > b0 else None, steps, stream, dev)
            e2e_ms = max_over_ranks(e2e_local)
        split.close()
    line = None
    if rank == 0:
        table, roof = roofline_table(per, cfg_tuple, mb, name if main and args.batch == 0 else None) if per \
            else ({}, None)
        attach_launch_counts(table, per, 3 if main else 1)
        tokens = B * S
        line = {
            "metric": METRIC, "value": tokens * 1000.0 / ms, "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 operands / f32 accumulate+residual", "data": "synthetic",
            "config": {"workload": workload(name, cfg_tuple), "global_batch": B, "seq_len": S},
            "parallelism": (f"batch split over {world} GPUs: input in rank 0's HBM, shards copied over NVLink "
                            f"(copy engines, CUDA IPC), {len(split.micro)} micro-batches per rank overlapping "
                            f"copy-in / forward / copy-out, fp32 output gathered into rank 0's HBM in the step"),
            "l2": "inputs and activations > 126 MB L2; no flush",
            "parity": parity,
            "roofline": roof,
            "roofline_per_kernel": table,
            "roofline_note": f"per-kernel times on one micro-batch ({mb} sequences) of rank 0",
            "gpu_launches": launches * len(split.micro) * steps,
            "gpu_launches_scope": "rank 0's kernels in the timed steps",
            "clocks": clocks[0],
            "clocks_all_ranks": clocks,
        }
        if main:
            line["e2e"] = {"value": tokens * 1000.0 / e2e_ms, "unit": "tokens/s", "ms_per_step": e2e_ms,
                           "path": "every rank: forward_from_host over its shard (pinned host -> its GPU -> pinned host)",
                           "h2d_bytes_per_step": x_host.numel() * 4, "d2h_bytes_per_step": x_host.numel() * 4}
            line["cpu_baseline"] = None  # timed on one GPU's runs only (the N = 1 line)
    del split, model
    torch.cuda.empty_cache()
    return line


if __name__ == "__main__":
    raise SystemExit(main())
