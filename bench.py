#!/usr/bin/env python
"""Benchmark of the hot path (one JSON line on rank 0).

Headline (benchmark configuration 2, workloads.FA_F16_CAUSAL): FlashAttention forward, fp16, causal,
q/k/v [B=4, H=16, S=2048, D=128] ~ N(0,1)*0.5, TFLOP/s with causal FLOPs =
2*B*H*S^2*D. The same run also measures, under "extra":
  * the other benchmark configurations per rank (attention D=64/32, bf16, fp32;
    GEMM 8192^3 fp16 + bias + ReLU and fp32 2048^3; the row family on
    X[65536, 4096] fp32), each with its roofline and, at N=1, its CPU baseline;
  * benchmark configuration 5 as fixed total problems split across the ranks
    ("scale_fa", "scale_gemm", "scale_rows_*": strong scaling, per-rank times,
    efficiency against rank 0 timing the whole problem alone, and a sampled
    oracle check per rank).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b2|reference]
  python bench.py --only fa_d64        # one configuration alone (ncu captures)

Multi-GPU (torchrun, one process per GPU): the headline runs the same per-rank
workload on every rank ("weak" scaling, no data-path collective); value = all
ranks' FLOPs / max-over-ranks device time.
Timing: CUDA events around each launch on the launching stream; L2 (126 MB) is
flushed by writing a 256 MB buffer between timed launches, outside the events.
"""
from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def load_traffic():
    """Per-launch DRAM bytes of each bench configuration (config name -> bytes), from
    the committed ncu summaries (dram__bytes_read.sum + dram__bytes_write.sum)."""
    p = ROOT / "profiles" / "traffic.txt"
    out = {}
    if p.exists():
        for line in p.read_text().splitlines():
            parts = line.split()
            if len(parts) >= 2 and not line.startswith("#"):
                try:
                    out[parts[0]] = float(parts[1])
                except ValueError:
                    pass
    return out


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        # One long-running `nvidia-smi -lms 200`: the driver query is set up once,
        # not once per sample (a fresh nvidia-smi per sample perturbed the timed
        # launches).
        try:
            self._p = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",  # one index or "0,1,.."
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self._first.set()
            return
        for line in self._p.stdout:
            if line.strip():
                self.samples.append([f.strip() for f in line.strip().split(",")])
                self._first.set()
            if self._stop.is_set():
                break
        self._first.set()

    def wait_first(self, timeout: float) -> None:
        """Block until the first sample arrived (or timeout): the query process is up."""
        self._first.wait(timeout)

    def __enter__(self):
        self._p = None
        self._first = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._p is not None:
            self._p.terminate()
            try:
                self._p.wait(timeout=5)
            except Exception:
                self._p.kill()
        if self._t:
            self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        mhz = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in self.samples:
            for i, n in enumerate(names):
                if len(s) > 5 + i and s[5 + i].lower().startswith("active"):
                    reasons.add(n)
        per_gpu = {}
        for s in self.samples:
            if s[1].replace(".", "").isdigit():
                per_gpu.setdefault(s[0], []).append(float(s[1]))
        out = {"sm_mhz": statistics.median(mhz) if mhz else None,
               "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
               "samples": len(self.samples)}
        if len(per_gpu) > 1:
            out["sm_mhz_per_gpu"] = {g: statistics.median(v) for g, v in sorted(per_gpu.items())}
        return out


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        dist.init_process_group(backend)
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_launches(fn, steps, warmup, flush_buf, world):
    """Device time per launch (ms): events around each launch, L2 flushed between.

    The warm-up steps (flush + launch, like the timed ones) are queued after the
    opening synchronize + barrier and run straight into the timed steps, outside
    every event pair, which also puts the host ahead of the device, so no step's
    events include host launch latency.
    """
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    for _ in range(warmup):  # the same sequence as a timed step
        flush_buf.zero_()
        fn()
    evs = []
    st = torch.cuda.current_stream()
    for _ in range(steps):
        flush_buf.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(st)
        fn()
        b.record(st)
        evs.append((a, b))
    torch.cuda.synchronize()
    barrier(world)
    return [a.elapsed_time(b) for a, b in evs]


# ------------------------------------------------------------------ CPU side
def cpu_info(threads=None):
    """(threads used, CPU model name) of this host."""
    model = "unknown"
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return threads or os.cpu_count() or 1, model


def cpu_rate(fn, units, seconds):
    """Run fn (one warm-up, then repeatedly for >= `seconds`, at least twice);
    returns (units per second, runs, elapsed s)."""
    fn()
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds or n < 2:
        fn()
        n += 1
    dt = time.perf_counter() - t0
    return units * n / dt, n, dt


def cpu_baseline(value, unit, sample, threads, model, extrapolated=False):
    d = {"value": value, "unit": unit, "cores": threads, "cpu_model": model, "kind": "port",
         "sample": sample}
    if extrapolated:
        d["extrapolated"] = True
    return d


def cpu_fa(cfg, seconds, threads, model):
    """Oracle attention on one (b, h) head of cfg (all of cfg when it is small)."""
    from oracle import oracle as O
    from triton_msl_b200 import workloads as W
    heads = cfg.B * cfg.H if cfg.S * cfg.S * cfg.B * cfg.H <= (1 << 22) else 1
    one = W.FAConfig("sample", 1, heads, cfg.S, cfg.D, cfg.causal, cfg.dtype, cfg.std)
    q, k, v = W.fa_inputs(one, seed=1)
    sm = 1.0 / 8 if cfg.dtype == torch.float32 else None
    rate, n, dt = cpu_rate(lambda: O.ref_attention(q, k, v, cfg.causal, sm), one.flops(), seconds)
    whole = heads == cfg.B * cfg.H
    sample = (f"{n} x {'all' if whole else 'one (b,h) head of'} [{cfg.B},{cfg.H},{cfg.S},{cfg.D}] "
              f"causal={cfg.causal}, fp32 torch-CPU oracle, {dt:.1f}s")
    return cpu_baseline(round(rate / 1e12, 5), "TFLOP/s", sample, threads, model)


def cpu_gemm(cfg, seconds, threads, model, rows=None):
    """Oracle GEMM on the first `rows` rows of A (all when None), extrapolated per FLOP."""
    from oracle import oracle as O
    from triton_msl_b200 import workloads as W
    import dataclasses
    sub = cfg if rows is None or rows >= cfg.M else dataclasses.replace(cfg, M=rows)
    a, bm, bias = W.gemm_inputs(sub, seed=1)
    rate, n, dt = cpu_rate(lambda: O.ref_gemm(a, bm, bias, cfg.activation, cfg.out_dtype),
                           sub.flops(), seconds)
    sample = f"{n} x A[{sub.M},{sub.K}] @ B[{sub.K},{sub.N}] ({cfg.activation}), fp32 torch-CPU oracle, {dt:.1f}s"
    return cpu_baseline(round(rate / 1e12, 5), "TFLOP/s", sample, threads, model,
                        extrapolated=sub is not cfg)


def cpu_gemm_chain(cfg, chain, seconds, threads, model, rows=256):
    """Oracle GEMM + epilogue chain on the first `rows` rows of A, extrapolated per FLOP."""
    from oracle import oracle as O
    from triton_msl_b200 import workloads as W
    import dataclasses
    sub = dataclasses.replace(cfg, M=min(rows, cfg.M))
    a, bm, bias = W.gemm_inputs(sub, seed=1)
    rate, n, dt = cpu_rate(lambda: O.ref_gemm_epilogue(a, bm, chain, bias, torch.float16),
                           sub.flops(), seconds)
    sample = (f"{n} x A[{sub.M},{sub.K}] @ B[{sub.K},{sub.N}] with the chain "
              f"{[c[0] for c in chain]}, fp32 torch-CPU oracle, {dt:.1f}s")
    return cpu_baseline(round(rate / 1e12, 5), "TFLOP/s", sample, threads, model,
                        extrapolated=sub.M != cfg.M)


def cpu_reduce_axis(cfg, seconds, threads, model, rows=4096):
    """Oracle sum over dim 0 of the first `rows` rows of X, per byte read."""
    from oracle import oracle as O
    from triton_msl_b200 import workloads as W
    import dataclasses
    sub = dataclasses.replace(cfg, rows=min(rows, cfg.rows))
    x, _, _ = W.row_inputs(sub, seed=1)
    byt = sub.rows * sub.cols * 4 + sub.cols * 4
    rate, n, dt = cpu_rate(lambda: O.ref_reduce_axis(x, "sum", 0), byt, seconds)
    sample = f"{n} x sum over dim 0 of X[{sub.rows},{sub.cols}] fp32, torch-CPU oracle, {dt:.1f}s"
    return cpu_baseline(round(rate / 1e9, 3), "GB/s", sample, threads, model,
                        extrapolated=sub.rows != cfg.rows)


def cpu_rows(cfg, op, seconds, threads, model, rows=4096):
    from oracle import oracle as O
    from triton_msl_b200 import workloads as W
    import dataclasses
    sub = dataclasses.replace(cfg, rows=min(rows, cfg.rows))
    x, w, b = W.row_inputs(sub, seed=1)
    fn = {"softmax": lambda: O.ref_softmax(x), "layernorm": lambda: O.ref_layernorm(x, w, b, 1e-5),
          "rmsnorm": lambda: O.ref_rmsnorm(x, w, 1e-6), "sum": lambda: O.ref_sum(x),
          "max": lambda: O.ref_max(x), "argmax": lambda: O.ref_argmax(x)}[op]
    rate, n, dt = cpu_rate(fn, sub.bytes(op), seconds)
    sample = f"{n} x {op} over X[{sub.rows},{sub.cols}] fp32, torch-CPU oracle, {dt:.1f}s"
    return cpu_baseline(round(rate / 1e9, 3), "GB/s", sample, threads, model,
                        extrapolated=sub.rows != cfg.rows)


def run_reference(args, world, rank):
    """Reference arm: the reference's CPU oracle path for FA (the reference's
    Metal kernels cannot run here), timed on this host's cores, same metric."""
    if rank != 0:
        return
    from triton_msl_b200 import workloads as W
    cfg = W.FA_F16_CAUSAL
    from oracle import oracle as O
    threads, model = cpu_info()
    torch.set_num_threads(threads)
    heads = 2
    samp = W.FAConfig("sample", 1, heads, cfg.S, cfg.D, cfg.causal, cfg.dtype, cfg.std)
    q, k, v = W.fa_inputs(samp, seed=1)
    for _ in range(args.warmup):
        O.ref_attention(q, k, v, cfg.causal)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.ref_attention(q, k, v, cfg.causal)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.mean(times)
    val = samp.flops() / (ms / 1e3) / 1e12
    sample = f"{heads} (b,h) heads of [4,16,2048,128] causal per step, fp32 torch-CPU oracle"
    print(json.dumps({
        "impl": "reference", "metric": "fa_fwd_fp16_causal_d128_tflops", "value": round(val, 5),
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": cfg.name, "B": cfg.B, "H": cfg.H, "S": cfg.S, "D": cfg.D,
                   "causal": True, "sample": sample},
        "cpu_baseline": {"value": round(val, 5), "unit": "TFLOP/s", "cores": threads,
                         "cpu_model": model, "kind": "port", "sample": sample},
        "e2e": {"value": round(val, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------- rooflines
def fp32_ffma_peak_tflops(peaks):
    """Nominal fp32 CUDA-core peak: 148 SMs x 128 FFMA lanes x 2 FLOP x max SM clock."""
    return 148 * 128 * 2 * float(peaks.get("sm_max_mhz", 1965.0)) * 1e6 / 1e12


def mufu_ex2_peak(peaks):
    """Nominal MUFU exponential rate: 16 ex2 / clk / SM x 148 SMs x max SM clock (per s)."""
    return 16 * 148 * float(peaks.get("sm_max_mhz", 1965.0)) * 1e6


def roofline(name, achieved, peak, unit, bound, traffic_bytes, peak_kind):
    return {"kernel": name, "bound": bound, "achieved": round(achieved, 2), "peak": round(peak, 1),
            "unit": unit, "frac": round(achieved / peak, 4), "peak_source": peak_kind,
            "traffic": traffic_bytes}


def fa_roofline(kname, cfg, ms, peaks, peak_kind, traffic):
    ach = cfg.flops() / (ms / 1e3) / 1e12
    tb = traffic.get(cfg.name)
    if kname == "fa_simt":
        rl = roofline(kname, ach, fp32_ffma_peak_tflops(peaks), "TFLOP/s", "fp32-ffma", tb,
                      "nominal fp32 FFMA (148 SM x 128 x 2 x sm_max_mhz)")
    else:
        rl = roofline(kname, ach, float(peaks["bf16_tflops"]), "TFLOP/s", "tensor", tb,
                      peak_kind + " bf16 burst")
        # second ceiling for the small head dims: one exponential per score
        scores = cfg.B * cfg.H * (cfg.S * (cfg.S + 1) / 2 if cfg.causal else cfg.S * cfg.S)
        rate = scores / (ms / 1e3)
        rl["exp"] = {"scores_per_s": float(f"{rate:.4g}"), "mufu_ex2_per_s": float(f"{mufu_ex2_peak(peaks):.4g}"),
                     "frac": round(rate / mufu_ex2_peak(peaks), 4),
                     "note": "one exp per score; the kernel also computes part of them on the FMA pipe"}
    return rl


# ------------------------------------------------------------------- GPU arm
def all_gather_floats(x: float, world: int):
    if world == 1:
        return [x]
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


def time_one(fn, steps, warmup, flush, world):
    """(max-over-ranks mean ms, per-rank mean ms)."""
    ms = statistics.mean(time_launches(fn, steps, warmup, flush, world))
    per = all_gather_floats(ms, world)
    return max(per), per


def measure_link(h2d_bytes, d2h_bytes, dev, world, steps=5):
    """Plain pinned host<->device copies of one e2e step's byte counts: alone and
    both directions at once on two streams (what the e2e pipeline overlaps),
    timed on the device, max over ranks (all ranks copy at the same time)."""
    hin = torch.empty(h2d_bytes, dtype=torch.uint8).pin_memory()
    hout = torch.empty(d2h_bytes, dtype=torch.uint8).pin_memory()
    din = torch.empty(h2d_bytes, dtype=torch.uint8, device=dev)
    dout = torch.empty(d2h_bytes, dtype=torch.uint8, device=dev)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()

    def run(mode):
        torch.cuda.synchronize()
        barrier(world)
        cur = torch.cuda.current_stream()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(cur)
        s1.wait_stream(cur)
        s2.wait_stream(cur)
        for _ in range(steps):
            if mode in ("h2d", "both"):
                with torch.cuda.stream(s1):
                    din.copy_(hin, non_blocking=True)
            if mode in ("d2h", "both"):
                with torch.cuda.stream(s2):
                    hout.copy_(dout, non_blocking=True)
        cur.wait_stream(s1)
        cur.wait_stream(s2)
        b.record(cur)
        torch.cuda.synchronize()
        return max(all_gather_floats(a.elapsed_time(b) / steps, world))

    run("both")  # warm-up
    h2d_ms, d2h_ms, both_ms = run("h2d"), run("d2h"), run("both")
    del hin, hout, din, dout
    return {"h2d_gbs_per_gpu": round(h2d_bytes / (h2d_ms / 1e3) / 1e9, 1),
            "d2h_gbs_per_gpu": round(d2h_bytes / (d2h_ms / 1e3) / 1e9, 1),
            "both_ms": round(both_ms, 4)}


def run_b2(args, world, rank, local):
    import triton_msl_b200 as b2
    from triton_msl_b200 import workloads as W
    dev = torch.device("cuda", torch.cuda.current_device())
    peaks, peak_kind = load_peaks()
    traffic = load_traffic()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    threads, model = cpu_info()
    do_cpu = rank == 0 and world == 1 and not args.no_cpu
    torch.set_num_threads(max(1, threads // max(1, int(os.environ.get("LOCAL_WORLD_SIZE", world)))))

    # ---------------- headline: FA fp16 causal D=128 ----------------
    cfg = W.FA_F16_CAUSAL
    q, k, v = W.fa_inputs(cfg, device=dev, seed=rank)
    fa = lambda: b2.flash_attn_fwd(q, k, v, causal=True)
    fa()
    kern = b2.last_kernel()
    if kern != "fa_sm100":
        raise RuntimeError(f"headline FA ran on {kern}, not the tensor-core kernel")
    # Each rank samples its own GPU's clocks from before the first timed step to
    # the end of the GPU work (the headline's own timed region is a few
    # milliseconds, shorter than one 200 ms sample); rank 0 gathers the
    # summaries. No extended pre-warm: the idle SM clock is already the maximum,
    # and a sub-second loop of back-to-back launches before the timed steps
    # tripped the power cap.
    sampler = ClockSampler(local)
    sampler.__enter__()
    sampler.wait_first(5.0)
    try:
        times = time_launches(fa, args.steps, args.warmup, flush, world)
        ms_rank = statistics.mean(times)
        per_rank = all_gather_floats(ms_rank, world)
        ms = max(per_rank)
        flops = cfg.flops()
        value = world * flops / (ms / 1e3) / 1e12
        rl = fa_roofline("fa_sm100", cfg, ms, peaks, peak_kind, traffic)

        # e2e through the public host-tensor entry point: every step copies q, k, v
        # from pinned host memory, runs the kernel and reads o back, chunk-pipelined
        # over (batch, head) on three streams (copies both ways overlap the kernel;
        # the inputs are CPU-prepared, so a step's uploads overlap the previous
        # step's read-back)
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        ho = torch.empty_like(hq).pin_memory()

        def e2e_step():
            b2.flash_attn_fwd_host(hq, hk, hv, causal=True, out=ho, host_inputs_ready=True)

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        st = torch.cuda.current_stream()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        gc.collect()
        gc.disable()  # no collector pause inside the host-paced e2e steps
        h0 = time.perf_counter()
        evs[0].record(st)
        for i in range(args.steps):
            e2e_step()
            evs[i + 1].record(st)
        host_ms = (time.perf_counter() - h0) * 1e3 / args.steps
        torch.cuda.synchronize()
        gc.enable()
        barrier(world)
        step_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
        e2e_per_rank = all_gather_floats(sum(step_ms) / args.steps, world)
        e2e_host_ms = max(all_gather_floats(host_ms, world))
        e2e_step_max = max(all_gather_floats(max(step_ms), world))
        e2e_step_min = max(all_gather_floats(min(step_ms), world))
        e2e_ms = max(e2e_per_rank)
        e2e_val = world * flops / (e2e_ms / 1e3) / 1e12
        h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))
        d2h = ho.numel() * ho.element_size()
        del hq, hk, hv, ho, q, k, v
        link = measure_link(h2d, d2h, dev, world)
        link["e2e_ms"] = round(e2e_ms, 4)
        link["e2e_step_ms_min_max"] = [round(e2e_step_min, 4), round(e2e_step_max, 4)]
        link["e2e_host_enqueue_ms_per_step"] = round(e2e_host_ms, 4)
        link["e2e_frac_of_link"] = round(link["both_ms"] / e2e_ms, 4)
        link["note"] = ("e2e is bounded by the host link: both_ms = the step's host->device and "
                        "device->host bytes as plain pinned copies, both directions at once, "
                        "all ranks at once")

        extra = {}
        if not args.headline_only:
            extra = run_extras(args, world, rank, dev, flush, peaks, peak_kind, traffic, do_cpu,
                               threads, model)
            extra.update(run_scale(args, world, rank, dev, flush, peaks, peak_kind, traffic, do_cpu,
                                   threads, model))
    finally:
        sampler.__exit__()

    summaries = [sampler.summary()]
    if world > 1:
        import torch.distributed as dist
        summaries = [None] * world
        dist.all_gather_object(summaries, sampler.summary())
    if rank != 0:
        return
    clocks = summaries[0]
    if world > 1:
        mhz = [c["sm_mhz"] for c in summaries if c.get("sm_mhz")]
        clocks = {"sm_mhz": statistics.median(mhz) if mhz else None,
                  "sm_max_mhz": max((c["sm_max_mhz"] or 0) for c in summaries) or None,
                  "reasons": sorted({r for c in summaries for r in c["reasons"]}),
                  "samples": sum(c.get("samples", 0) for c in summaries),
                  "sm_mhz_per_rank": [c["sm_mhz"] for c in summaries]}
    threads_all, _ = cpu_info()
    torch.set_num_threads(threads_all)
    cb = cpu_fa(cfg, args.cpu_seconds if world == 1 else 3.0, threads_all, model)
    line = {
        "metric": "fa_fwd_fp16_causal_d128_tflops", "value": round(value, 2), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": cfg.name, "B": cfg.B, "H": cfg.H, "S": cfg.S, "D": cfg.D,
                   "causal": True, "flops_per_step_per_gpu": flops,
                   "l2": "flushed between timed launches (256 MB write)",
                   "parallelism": f"(batch,head) shards x{world}, no collective"},
        "per_rank_ms": [round(x, 4) for x in per_rank],
        "roofline": rl,
        "cpu_baseline": cb,
        "e2e": {"value": round(e2e_val, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "per_rank_ms": [round(x, 4) for x in e2e_per_rank],
                "link": link},
        "gpu_launches": args.steps,  # headline timed region: one fa_sm100 launch per step
        "clocks": clocks,
        "extra": extra,
    }
    print(json.dumps(line), flush=True)


def run_extras(args, world, rank, dev, flush, peaks, peak_kind, traffic, do_cpu, threads, model):
    """The other benchmark configurations (attention D=64/32, bf16, fp32; GEMM 8192^3 +
    bias + ReLU and fp32 2048^3; the row family at 65536x4096), per-rank
    weak-scaling copies, same timing rules, each with its roofline, its own
    ncu traffic and (N=1, rank 0) its CPU baseline."""
    import triton_msl_b200 as b2
    from triton_msl_b200 import workloads as W
    out = {}
    steps = max(3, min(args.steps, 10))
    cs = args.cpu_seconds_extra
    fa_cfgs = ((W.FA_F16_CAUSAL_D64, {}), (W.FA_F16_CAUSAL_D32, {}), (W.FA_BF16_CAUSAL, {}),
               (W.FA_F32, {"sm_scale": 1 / 8}))
    for cfg, kw in fa_cfgs:
        q, k, v = W.fa_inputs(cfg, device=dev, seed=rank)
        fn = lambda: b2.flash_attn_fwd(q, k, v, causal=cfg.causal, **kw)
        fn()
        kname = b2.last_kernel()
        ms, per = time_one(fn, steps, 3, flush, world)
        ach = cfg.flops() / (ms / 1e3) / 1e12
        e = {"value": round(world * ach, 2), "unit": "TFLOP/s", "ms": round(ms, 4),
             "per_rank_ms": [round(x, 4) for x in per], "kernel": kname,
             "roofline": fa_roofline(kname, cfg, ms, peaks, peak_kind, traffic)}
        if do_cpu:
            e["cpu_baseline"] = cpu_fa(cfg, cs, threads, model)
        out[cfg.name] = e
        del q, k, v
    g32 = W.GEMM_F32
    a32, b32, _ = W.gemm_inputs(g32, device=dev, seed=rank)
    fn = lambda: b2.gemm(a32, b32)
    fn()
    kname = b2.last_kernel()
    ms, per = time_one(fn, steps, 3, flush, world)
    ach32 = g32.flops() / (ms / 1e3) / 1e12
    e = {"value": round(world * ach32, 2), "unit": "TFLOP/s", "ms": round(ms, 4),
         "per_rank_ms": [round(x, 4) for x in per], "kernel": kname}
    if kname == "gemm_sm100_tf32x3":
        # fp32 product as 3xTF32 (split pass + one tensor-core GEMM over 3K): the
        # tensor pipe does 3x the listed FLOPs at the tf32 rate, taken as half the
        # measured bf16 rate (the nominal dense ratio, 1.1 vs 2.25 PFLOP/s)
        e["roofline"] = roofline(kname, 3 * ach32, float(peaks["bf16_tflops"]) / 2, "TFLOP/s",
                                 "tensor", traffic.get(g32.name), peak_kind + " bf16 burst / 2")
        e["note"] = ("3xTF32 on tensor cores (max-abs 1e-4 met); achieved counts the 3 tf32 "
                     "products, against tf32 peak = measured bf16 / 2; split launches included")
    else:
        e["roofline"] = roofline(kname, ach32, fp32_ffma_peak_tflops(peaks), "TFLOP/s", "fp32-ffma",
                                 traffic.get(g32.name), "nominal fp32 FFMA")
    if do_cpu:
        e["cpu_baseline"] = cpu_gemm(g32, cs, threads, model)
    out[g32.name] = e
    del a32, b32
    g = W.GEMM_F16
    a, bm, bias = W.gemm_inputs(g, device=dev, seed=rank)
    fn = lambda: b2.gemm(a, bm, bias, "relu", torch.float16)
    fn()
    kname = b2.last_kernel()
    ms, per = time_one(fn, steps, 3, flush, world)
    ach = g.flops() / (ms / 1e3) / 1e12
    e = {"value": round(world * ach, 2), "unit": "TFLOP/s", "ms": round(ms, 4),
         "per_rank_ms": [round(x, 4) for x in per], "kernel": kname,
         "roofline": roofline(kname, ach, float(peaks["bf16_tflops"]), "TFLOP/s", "tensor",
                              traffic.get(g.name), peak_kind + " bf16 burst")}
    if do_cpu:
        e["cpu_baseline"] = cpu_gemm(g, cs, threads, model, rows=256)
    out[g.name] = e
    del a, bm, bias
    r = W.ROWS_F32
    x, w, bb = W.row_inputs(r, device=dev, seed=rank)
    ops = {"softmax": lambda: b2.row_softmax(x),
           "layernorm": lambda: b2.row_layernorm(x, w, bb, 1e-5),
           "rmsnorm": lambda: b2.row_rmsnorm(x, w, 1e-6),
           "sum": lambda: b2.row_sum(x), "max": lambda: b2.row_max(x),
           "argmax": lambda: b2.row_argmax(x)}
    for op, fn in ops.items():
        fn()
        kname = b2.last_kernel()
        ms, per = time_one(fn, steps, 3, flush, world)
        gbs = r.bytes(op) / (ms / 1e3) / 1e9
        e = {"value": round(world * gbs, 1), "unit": "GB/s", "ms": round(ms, 4),
             "per_rank_ms": [round(x_, 4) for x_ in per], "kernel": kname,
             "roofline": roofline(f"{kname}_{op}", gbs, float(peaks["hbm_gbs"]), "GB/s", "hbm",
                                  traffic.get(f"{r.name}_{op}"), peak_kind + " copy")}
        if do_cpu:
            e["cpu_baseline"] = cpu_rows(r, op, cs, threads, model)
        out[f"{r.name}_{op}"] = e
    # the same X reduced over its other axis (sum over rows: 4096 outputs)
    fn = lambda: b2.reduce(x, "sum", 0)
    fn()
    kname = b2.last_kernel()
    ms, per = time_one(fn, steps, 3, flush, world)
    byt = r.rows * r.cols * 4 + r.cols * 4
    gbs = byt / (ms / 1e3) / 1e9
    out[f"{r.name}_sum_dim0"] = {
        "value": round(world * gbs, 1), "unit": "GB/s", "ms": round(ms, 4),
        "per_rank_ms": [round(x_, 4) for x_ in per], "kernel": kname,
        "roofline": roofline(kname, gbs, float(peaks["hbm_gbs"]), "GB/s", "hbm",
                             traffic.get(f"{r.name}_sum_dim0"), peak_kind + " copy")}
    if do_cpu:
        out[f"{r.name}_sum_dim0"]["cpu_baseline"] = cpu_reduce_axis(r, cs, threads, model)
    del x, w, bb
    # GEMM 8192^3 fp16 with a general epilogue chain (bias, scale, GELU, clamp)
    a, bm, bias = W.gemm_inputs(g, device=dev, seed=rank)
    chain = [("add_bias",), ("mul", 0.5), ("gelu",), ("clamp", -1.0, 4.0)]
    fn = lambda: b2.gemm_epilogue(a, bm, chain, bias, torch.float16)
    fn()
    kname = b2.last_kernel()
    ms, per = time_one(fn, steps, 3, flush, world)
    ach = g.flops() / (ms / 1e3) / 1e12
    out["gemm_f16_8192_epilogue_chain"] = {
        "value": round(world * ach, 2), "unit": "TFLOP/s", "ms": round(ms, 4),
        "per_rank_ms": [round(x_, 4) for x_ in per], "kernel": kname, "chain": [c[0] for c in chain],
        "roofline": roofline(kname, ach, float(peaks["bf16_tflops"]), "TFLOP/s", "tensor",
                             traffic.get("gemm_f16_8192_epilogue_chain"),
                             peak_kind + " bf16 burst")}
    if do_cpu:
        out["gemm_f16_8192_epilogue_chain"]["cpu_baseline"] = cpu_gemm_chain(g, chain, cs, threads, model)
    del a, bm, bias
    return out


def run_scale(args, world, rank, dev, flush, peaks, peak_kind, traffic, do_cpu, threads, model):
    """benchmark configuration 5 and the row family as fixed total problems split across
    the ranks with no collective (strong scaling): FA bf16 causal [64,32,8192,128]
    by (batch, head), GEMM bf16 65536x16384x16384 by 128-row M-tiles (B built on
    every rank from one seed: a replicated local copy), rows 65536x4096 fp32
    (softmax, argmax) by rows. Each rank builds only its own shard, on its own
    GPU. value = total work / max-over-ranks time; efficiency = T(1) / (N T(N)),
    T(1) timed by rank 0 alone on the whole problem in the same run (at N=1 the
    shard is the whole problem). A sampled (b,h) head, row block of C and row
    block of X per rank is checked against the CPU oracle."""
    import math
    import triton_msl_b200 as b2
    from oracle import oracle as O
    from triton_msl_b200 import shard, workloads as W
    out = {}
    sus = float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]))
    steps = max(3, min(args.steps, 10))

    pending = []  # (extra key, build whole problem, launch fn) for the T(1) timings

    def finish(name, metric_unit, total, shard_work, ms, per, full_ms, kname, err, tol, extra):
        eff = full_ms / (world * ms) if full_ms else None
        if metric_unit == "TFLOP/s":
            per_gpu = shard_work / (ms / 1e3) / 1e12
            rl = roofline(kname, per_gpu, sus, "TFLOP/s", "tensor", traffic.get(name),
                          peak_kind + " bf16 sustained (a step of tens of ms runs under the power cap)")
            val = total / (ms / 1e3) / 1e12
        else:
            per_gpu = shard_work / (ms / 1e3) / 1e9
            rl = roofline(kname, per_gpu, float(peaks["hbm_gbs"]), "GB/s", "hbm", traffic.get(name),
                          peak_kind + " copy")
            val = total / (ms / 1e3) / 1e9
        e = {"value": round(val, 2), "unit": metric_unit, "n_gpus": world, "scaling": "strong",
             "ms": round(ms, 4), "per_rank_ms": [round(x, 4) for x in per],
             "full_problem_ms_1gpu": round(full_ms, 4) if full_ms else None,
             "efficiency": round(eff, 4) if eff else None, "kernel": kname,
             "roofline_per_gpu": rl,
             "oracle_check": {"max_err_over_ranks": float(f"{err:.3e}"), "tol": tol, "ok": err <= tol},
             "parallelism": f"shards x{world}, no collective"}
        e.update(extra)
        return e

    def full_time(build, fn_of):
        """Rank 0 alone times the whole problem (others wait at the barrier)."""
        if world == 1:
            return None
        res = None
        if rank == 0:
            objs = build()
            fn = fn_of(objs)
            fn()
            res = statistics.mean(time_launches(fn, steps, 3, flush, 1))
            del objs, fn
            torch.cuda.empty_cache()
        barrier(world)
        return max(all_gather_floats(res or 0.0, world))

    # ---------------------------------------------------------------- FA
    cfg = W.FA_BF16_SCALE
    lo, hi = shard.unit_range(cfg.B * cfg.H, world, rank)
    n = hi - lo

    def fa_build(units, seed):
        g = torch.Generator(device=dev).manual_seed(seed)
        return [(torch.randn((1, units, cfg.S, cfg.D), generator=g, device=dev) * cfg.std).to(cfg.dtype)
                for _ in range(3)]

    q, k, v = fa_build(n, 1000 + rank)
    fn = lambda: b2.flash_attn_fwd(q, k, v, causal=True)
    fn()
    kname = b2.last_kernel()
    ms, per = time_one(fn, steps, args.warmup, flush, world)
    o = fn()
    i = n // 2
    ref = O.ref_attention(q[:, i:i + 1].cpu(), k[:, i:i + 1].cpu(), v[:, i:i + 1].cpu(), True)
    err = max(all_gather_floats(O.normwise_err(o[:, i:i + 1], ref), world))
    del q, k, v, o
    pending.append(("scale_fa", lambda: fa_build(cfg.B * cfg.H, 999),
                    lambda t: (lambda: b2.flash_attn_fwd(t[0], t[1], t[2], causal=True))))
    full = None
    e = finish(cfg.name, "TFLOP/s", cfg.flops(), cfg.flops() * n / (cfg.B * cfg.H), ms, per, full,
               kname, err, O.TOL_LOWP_REL + 2.0 ** -8, {"units_rank0": n})
    if do_cpu:
        e["cpu_baseline"] = cpu_fa(cfg, args.cpu_seconds_extra, threads, model)
    out["scale_fa"] = e

    # -------------------------------------------------------------- GEMM
    gc = W.GEMM_BF16_SCALE
    lo, hi = shard.unit_range(gc.M, world, rank, align=128)
    s_ = 1.0 / math.sqrt(gc.K)

    def gemm_build(rows, seed):
        g = torch.Generator(device=dev).manual_seed(seed)
        a = (torch.randn((rows, gc.K), generator=g, device=dev) * s_).to(gc.dtype)
        g2 = torch.Generator(device=dev).manual_seed(4242)   # B: the same on every rank
        bm = (torch.randn((gc.K, gc.N), generator=g2, device=dev) * s_).to(gc.dtype)
        return a, bm

    a, bm = gemm_build(hi - lo, 2000 + rank)
    fn = lambda: b2.gemm(a, bm)
    fn()
    kname = b2.last_kernel()
    ms, per = time_one(fn, steps, args.warmup, flush, world)
    c = fn()
    r0 = (hi - lo) // 2
    ref = O.ref_gemm(a[r0:r0 + 32].cpu(), bm.cpu(), None, "none", torch.bfloat16)
    err = max(all_gather_floats(O.normwise_err(c[r0:r0 + 32], ref), world))
    del a, bm, c
    torch.cuda.empty_cache()
    pending.append(("scale_gemm", lambda: gemm_build(gc.M, 1999), lambda t: (lambda: b2.gemm(t[0], t[1]))))
    full = None
    e = finish(gc.name, "TFLOP/s", gc.flops(), 2.0 * (hi - lo) * gc.N * gc.K, ms, per, full, kname,
               err, O.TOL_LOWP_REL + 2.0 ** -8, {"rows_rank0": hi - lo})
    if do_cpu:
        e["cpu_baseline"] = cpu_gemm(gc, args.cpu_seconds_extra, threads, model, rows=64)
    out["scale_gemm"] = e

    # -------------------------------------------------------------- rows
    rc = W.ROWS_F32
    lo, hi = shard.unit_range(rc.rows, world, rank)
    import dataclasses
    for op in ("softmax", "argmax"):
        def rows_build(nrows, seed):
            return (torch.randn((nrows, rc.cols), generator=torch.Generator(device=dev).manual_seed(seed),
                                device=dev),)
        (x,) = rows_build(hi - lo, 3000 + rank)
        f = b2.row_softmax if op == "softmax" else b2.row_argmax
        fn = lambda: f(x)
        fn()
        kname = b2.last_kernel()
        ms, per = time_one(fn, steps, args.warmup, flush, world)
        y = fn()
        xs = x[:256].cpu()
        if op == "softmax":
            err = O.max_abs_err(y[:256], O.ref_softmax(xs))
            tol = O.TOL_F32_ABS
        else:
            err = 0.0 if torch.equal(y[:256].cpu(), O.ref_argmax(xs)) else 1.0
            tol = 0.0
        err = max(all_gather_floats(err, world))
        del x, y
        pending.append((f"scale_rows_{op}", (lambda rb=rows_build: rb(rc.rows, 2999)),
                        (lambda t, f=f: (lambda: f(t[0])))))
        full = None
        sub = dataclasses.replace(rc, rows=hi - lo)
        e = finish(f"{rc.name}_{op}", "GB/s", rc.bytes(op), sub.bytes(op), ms, per, full, kname,
                   err, tol, {"rows_rank0": hi - lo})
        if do_cpu:
            e["cpu_baseline"] = cpu_rows(rc, op, args.cpu_seconds_extra, threads, model)
        out[f"scale_rows_{op}"] = e
    # T(1): rank 0 alone on each whole problem, after every sharded measurement
    # (so the long single-GPU runs do not heat rank 0 ahead of its shard timings)
    # lightest first (the rows), each after a 1 s idle pause so a whole-problem
    # run does not start on a GPU still held down by the previous one's power draw
    for key, build, fn_of in sorted(pending, key=lambda p: not p[0].startswith("scale_rows")):
        barrier(world)
        time.sleep(1.0)
        full = full_time(build, fn_of)
        e = out[key]
        e["full_problem_ms_1gpu"] = round(full, 4) if full else None
        e["efficiency"] = round(full / (world * e["ms"]), 4) if full else None
    return out


ONLY = ("headline", "fa_d64", "fa_d32", "fa_bf16", "fa_f32", "gemm_f16", "gemm_f32",
        "rows_softmax", "rows_layernorm", "rows_rmsnorm", "rows_sum", "rows_max", "rows_argmax",
        "gemm_bf16_scale_shard", "rows_sum_dim0", "gemm_f16_chain", "rows_argmax_dim0",
        "rows_long_softmax", "rows_long_argmax", "rows_f16_argmax")


def run_only(args):
    """One configuration in a process that allocates only its inputs (for ncu
    captures: one kernel family, a few launches, a few GB on the device)."""
    import triton_msl_b200 as b2
    from triton_msl_b200 import workloads as W
    dev = torch.device("cuda", 0)
    name = args.only
    if name.startswith("fa_") or name == "headline":
        cfg = {"headline": W.FA_F16_CAUSAL, "fa_d64": W.FA_F16_CAUSAL_D64, "fa_d32": W.FA_F16_CAUSAL_D32,
               "fa_bf16": W.FA_BF16_CAUSAL, "fa_f32": W.FA_F32}[name]
        q, k, v = W.fa_inputs(cfg, device=dev)
        kw = {"sm_scale": 1 / 8} if cfg.dtype == torch.float32 else {}
        fn = lambda: b2.flash_attn_fwd(q, k, v, causal=cfg.causal, **kw)
        work, unit = cfg.flops(), "TFLOP/s"
    elif name in ("gemm_f16", "gemm_f32"):
        cfg = W.GEMM_F16 if name == "gemm_f16" else W.GEMM_F32
        a, bm, bias = W.gemm_inputs(cfg, device=dev)
        fn = (lambda: b2.gemm(a, bm, bias, "relu", torch.float16)) if name == "gemm_f16" \
            else (lambda: b2.gemm(a, bm))
        work, unit = cfg.flops(), "TFLOP/s"
    elif name == "gemm_f16_chain":
        cfg = W.GEMM_F16
        a, bm, bias = W.gemm_inputs(cfg, device=dev)
        chain = [("add_bias",), ("mul", 0.5), ("gelu",), ("clamp", -1.0, 4.0)]
        fn = lambda: b2.gemm_epilogue(a, bm, chain, bias, torch.float16)
        work, unit = cfg.flops(), "TFLOP/s"
    elif name == "rows_sum_dim0":
        r = W.ROWS_F32
        x, _, _ = W.row_inputs(r, device=dev)
        fn = lambda: b2.reduce(x, "sum", 0)
        work, unit = r.rows * r.cols * 4 + r.cols * 4, "GB/s"
    elif name == "rows_argmax_dim0":
        r = W.ROWS_F32
        x, _, _ = W.row_inputs(r, device=dev)
        fn = lambda: b2.reduce(x, "argmax", 0)
        work, unit = r.rows * r.cols * 4 + r.cols * 8, "GB/s"
    elif name in ("rows_long_softmax", "rows_long_argmax", "rows_f16_argmax"):
        # rows past the register-resident limit (fp32 [4096, 65536]) and 16-bit
        # argmax (fp16 [65536, 4096]): same seeded N(0, 1) values
        shape, dt = ((4096, 65536), torch.float32) if "long" in name else ((65536, 4096), torch.float16)
        g = torch.Generator(device=dev).manual_seed(0)
        x = torch.randn(*shape, device=dev, generator=g).to(dt)
        rd = x.numel() * x.element_size()
        if name == "rows_long_softmax":
            fn, work = (lambda: b2.row_softmax(x)), 2 * rd
        else:
            fn, work = (lambda: b2.row_argmax(x)), rd + 8 * shape[0]
        unit = "GB/s"
    elif name == "gemm_bf16_scale_shard":
        cfg = W.GEMM_BF16_SCALE
        a = torch.randn(8192, cfg.K, device=dev).to(cfg.dtype)
        bm = torch.randn(cfg.K, cfg.N, device=dev).to(cfg.dtype)
        fn = lambda: b2.gemm(a, bm)
        work, unit = 2.0 * 8192 * cfg.N * cfg.K, "TFLOP/s"
    else:
        op = name.split("_", 1)[1]
        r = W.ROWS_F32
        x, w, bb = W.row_inputs(r, device=dev)
        fn = {"softmax": lambda: b2.row_softmax(x), "layernorm": lambda: b2.row_layernorm(x, w, bb, 1e-5),
              "rmsnorm": lambda: b2.row_rmsnorm(x, w, 1e-6), "sum": lambda: b2.row_sum(x),
              "max": lambda: b2.row_max(x), "argmax": lambda: b2.row_argmax(x)}[op]
        work, unit = r.bytes(op), "GB/s"
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    fn()
    ms = statistics.median(time_launches(fn, args.steps, args.warmup, flush, 1))
    rate = work / (ms / 1e3) / (1e12 if unit == "TFLOP/s" else 1e9)
    print(json.dumps({"only": name, "kernel": b2.last_kernel(), "ms_median": round(ms, 4),
                      "value": round(rate, 2), "unit": unit, "steps": args.steps}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b2", choices=["b2", "reference"])
    ap.add_argument("--headline-only", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines of the extras")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU-baseline sample length of the headline")
    ap.add_argument("--cpu-seconds-extra", type=float, default=1.5,
                    help="CPU-baseline sample length of each extra configuration")
    ap.add_argument("--only", choices=ONLY, default=None,
                    help="time one configuration alone (1 GPU; small process for ncu captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.only:
        run_only(args)
        return
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_b2(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
