#!/usr/bin/env python
"""bench.py -- device-timed throughput of the B200 attention (and MLP) hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        bench.py --gpus N ...
    python bench.py --impl reference ...     # the CPU implementation of the path

A "step" is one pass of the hot path over one batch: one attention forward
over this rank's (batch, head) shard (or one MLP block for cfg3).  Inputs are
generated on each GPU from the seed before timing, per (batch, head) pair, so
any sharding reproduces the same tensors.  Timing follows the reference's
method (CUDA events around the kernel loop after warm-up, ``bench.py:49-74``
of the reference) with a barrier + synchronize on both sides and the maximum
over ranks.  Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import statistics
import sys
import threading
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from cs348k_fast_attention_grammar_b200.inputs import (ATTN_CONFIGS, MLP_CONFIGS,  # noqa: E402
                                                       make_mlp, make_qkv, pair_tensor)
from cs348k_fast_attention_grammar_b200.parallel import (reduce_error_stats,  # noqa: E402
                                                         shard_range, verify_pairs)

METRIC = "attn fwd TFLOP/s per GPU, % of bf16 tensor peak; box TFLOP/s at 1/2/4/8 GPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
L2_BYTES = 126 * 1024 * 1024


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=sorted(list(ATTN_CONFIGS) + list(MLP_CONFIGS)
                                               + ["ref512", "ln"]),
                    default="cfg2")
    ap.add_argument("--pairs", type=int, default=0,
                    help="attention: only the first N (batch, head) pairs (a small case "
                         "of the same kernel, e.g. for a profiler)")
    ap.add_argument("--rows", type=int, default=0,
                    help="cfg3 / ln: only the first N rows of X (a small case)")
    ap.add_argument("--kernel-only", action="store_true",
                    help="warm-up and timed launches only: no verification, e2e, CPU "
                         "baseline, comparators or secondary lines (profiler runs)")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the cfg1 / cfg3 lines of the default single-GPU run")
    ap.add_argument("--no-sdpa", action="store_true",
                    help="skip the same-GPU torch SDPA (cuDNN) comparator")
    ap.add_argument("--sdpa-only", action="store_true",
                    help="attention configs: time only the torch SDPA (cuDNN) comparator on "
                         "the same seeded tensors (a profiler run of the library kernel)")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--e2e-chunks", type=int, default=8,
                    help="(batch, head) chunks pipelined over the copy/kernel streams")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--verify-pairs", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    return ap.parse_args(argv)


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------
def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", 0.0)),
                "source": "measured"}
    except Exception:
        return dict(FALLBACK_PEAKS, source="fallback")


def load_traffic(config: str):
    """Per-launch DRAM bytes (read + write) of the dominant kernel, from the
    committed ncu summary profiles/ncu_traffic.txt (``<config> <bytes>`` lines)."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 2 and parts[0] == config:
                    return float(parts[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML (the library
    nvidia-smi reads) every 20 ms while the timed region runs."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting", 0x10: "sync_boost"}

    def __init__(self, device_index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            if not uuid.startswith("GPU-"):
                uuid = "GPU-" + uuid
            self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._nvml = pynvml
        except Exception as e:  # noqa: BLE001
            self.error = f"nvml unavailable: {e}"

    def _reasons_now(self):
        n = self._nvml
        fn = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            getattr(n, "nvmlDeviceGetCurrentClocksThrottleReasons")
        return fn(self._h)

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM))
                mask = self._reasons_now()
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.02)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if self._nvml is None:
            return {"error": getattr(self, "error", "nvml unavailable")}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def timed_loop(fn, steps: int, world: int, device) -> float:
    """Mean ms per step over ``steps`` calls, CUDA events on the current
    stream, barrier + synchronize on both sides, max over ranks."""
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        fn()
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / steps
    slowest, fastest = rank_ms_spread(ms, world, device)
    LAST_RANK_MS.update(min=fastest, max=slowest)
    if world > 1:
        dist.barrier()
    return slowest


def rank_ms_spread(ms: float, world: int, device) -> tuple:
    """(slowest, fastest) of every rank's ``ms`` (one all-reduce)."""
    if world == 1:
        return ms, ms
    t = torch.tensor([ms, -ms], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t[0].item(), -t[1].item()


# Fastest and slowest rank of the last timed_loop (the reported time is the
# slowest); the spread shows whether one GPU or all of them set the time.
LAST_RANK_MS = {"min": 0.0, "max": 0.0}


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def timed_reps(fn, reps: int, world: int, device) -> dict:
    """The reference search's convention (grammar/optimization.py:284-300):
    ``reps`` calls, each timed alone with CUDA events and synchronised; the
    minimum is the least noise-contaminated sample.  Max over ranks of each
    rank's min and median."""
    stream = torch.cuda.current_stream(device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    times = []
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for _ in range(reps):
        e0.record(stream)
        fn()
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    return {"min_ms": max_over_ranks(min(times), world, device),
            "median_ms": max_over_ranks(statistics.median(times), world, device),
            "reps": reps}


@contextlib.contextmanager
def stdout_to_stderr():
    """Point file descriptor 1 at stderr for the block: NCCL prints its
    version banner on stdout when a communicator is created, and stdout
    carries the one JSON line."""
    sys.stdout.flush()
    saved = os.dup(1)
    try:
        os.dup2(2, 1)
        yield
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def attn_flops(cfg, pairs=None) -> float:
    import oracle  # only for the FLOP convention of the reference (old/benchmark.py:131)
    n = cfg["B"] * cfg["H"] if pairs is None else pairs
    return float(oracle.attention_flops(1, n, cfg["S"], cfg["D"], cfg["causal"]))


def cpu_attention_sample(cfg, seconds: float, max_pairs: int = 10_000):
    """Time the CPU restatement of the naive path (oracle.naive_torch_pair) on
    seeded pairs until ``seconds`` elapse; returns (TFLOP/s, pairs, seconds)."""
    import oracle
    torch.set_num_threads(host_cores())
    done, t_total = 0, 0.0
    p = 0
    while done < max_pairs and (t_total < seconds or done == 0):
        q, k, v = (pair_tensor(cfg["seed"], n, p, cfg["S"], cfg["D"], cfg["amp"], "cpu",
                               torch.float32) for n in ("q", "k", "v"))
        t0 = time.perf_counter()
        oracle.naive_torch_pair(q, k, v, causal=cfg["causal"])
        t_total += time.perf_counter() - t0
        done += 1
        p += 1
    return attn_flops(cfg, done) / t_total / 1e12, done, t_total


# ---------------------------------------------------------------------------
# reference arm: the CPU implementation of the path on this host
# ---------------------------------------------------------------------------
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if args.config in MLP_CONFIGS:
        return run_reference_mlp(args)
    if args.config == "ref512":
        return run_reference_ref512(args)
    import oracle
    cfg = ATTN_CONFIGS[args.config]
    torch.set_num_threads(host_cores())
    q, k, v = (pair_tensor(cfg["seed"], n, 0, cfg["S"], cfg["D"], cfg["amp"], "cpu",
                           torch.float32) for n in ("q", "k", "v"))
    for _ in range(args.warmup):
        oracle.naive_torch_pair(q, k, v, causal=cfg["causal"])
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.naive_torch_pair(q, k, v, causal=cfg["causal"])
        times.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.mean(times)
    value = attn_flops(cfg, 1) / (ms * 1e-3) / 1e12
    sample = (f"one (batch, head) pair per step (S={cfg['S']}, D={cfg['D']}, "
              f"causal={cfg['causal']}) of the {args.config} workload; pairs are independent")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,1) per pair", "config": workload_config(args, cfg),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample, "cpu": cpu_model(),
                         "what": "oracle.naive_torch_pair: correct restatement of "
                                 "pytorch-naive.py:41-63 in fp32 torch"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference_mlp(args):
    import oracle
    cfg = MLP_CONFIGS[args.config]
    torch.set_num_threads(host_cores())
    rows = 256
    x, w1, w2 = (t.float() for t in make_mlp(dict(cfg, M=rows), "cpu"))
    fn = lambda: torch.nn.functional.gelu(x @ w1, approximate="tanh") @ w2  # noqa: E731
    for _ in range(args.warmup):
        fn()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.mean(times)
    value = oracle.mlp_flops(rows, cfg["K"], cfg["N"]) / (ms * 1e-3) / 1e12
    line = {"impl": "reference", "metric": "MLP block TFLOP/s", "value": value,
            "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": f"{args.config} MLP, {rows} rows"},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                             "kind": "port", "sample": f"{rows} rows of X per step"},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def workload_config(args, cfg, num_pairs=None):
    S, D = cfg["S"], cfg["D"]
    n = cfg["B"] * cfg["H"] if num_pairs is None else num_pairs
    qkv_bytes = 3 * n * S * D * 2
    sub = "" if n == cfg["B"] * cfg["H"] else f" (first {n} (batch, head) pairs)"
    return {"workload": (f"{args.config}: attention forward {'causal' if cfg['causal'] else 'non-causal'}"
                         f" bf16 B={cfg['B']} H={cfg['H']} S={S} D={D}{sub}"),
            "B": cfg["B"], "H": cfg["H"], "S": S, "D": D, "causal": cfg["causal"],
            "seed": cfg["seed"], "parallelism": f"dp over batch*head x {args.gpus}",
            "l2": (f"inputs larger than L2 ({qkv_bytes / 2**20:.0f} MiB of Q/K/V per step "
                   f"> 126 MiB), no flush") if qkv_bytes > L2_BYTES else
                  "L2 not flushed (inputs smaller than L2)"}


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        with stdout_to_stderr():
            dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
            dist.barrier()

    import cs348k_fast_attention_grammar_b200 as fab
    fab.load()
    if args.config in MLP_CONFIGS:
        line = bench_mlp(args, fab, device, world, rank)
    elif args.config == "ref512":
        line = bench_ref512(args, fab, device, world, rank)
    elif args.config == "ln":
        line = bench_ln(args, fab, device, world, rank)
    else:
        line = bench_attention(args, fab, device, world, rank)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def roofline(achieved_tflops, peaks, traffic):
    """Fraction of the measured burst bf16 peak (the conservative figure);
    the sustained-peak fraction (power-capped clocks, long loops) rides along."""
    peak = peaks["bf16_tflops"]
    out = {"bound": "tensor", "achieved": achieved_tflops, "peak": peak, "unit": "TFLOP/s",
           "frac": achieved_tflops / peak, "traffic": traffic,
           "peak_source": f"{peaks['source']} (bf16 dense burst, cuBLAS)"}
    if peaks.get("bf16_tflops_sustained"):
        out["frac_of_sustained_peak"] = achieved_tflops / peaks["bf16_tflops_sustained"]
    return out


def attention_timing(args, fab, cfg, pairs, device, world, steps, warmup):
    """Seeded Q/K/V for ``pairs`` on this GPU, ``warmup`` untimed launches,
    then ``steps`` timed ones (window mean, clocks sampled meanwhile) and five
    individually timed reps (min / median)."""
    q, k, v = make_qkv(cfg, pairs, device)
    o = torch.empty_like(q)
    step = lambda: fab.attention(q, k, v, causal=cfg["causal"], out=o)  # noqa: E731
    for _ in range(max(warmup, 0)):
        step()
    torch.cuda.synchronize()
    with ClockSampler(local_index(device)) as clk:
        ms = timed_loop(step, steps, world, device)
    rank_ms = dict(LAST_RANK_MS)
    reps = timed_reps(step, 5, world, device)
    return {"q": q, "k": k, "v": v, "o": o, "ms": ms, "reps": reps, "clocks": clk.summary(),
            "rank_ms": rank_ms}


def sdpa_same_gpu(q, k, v, o, causal, flops_local, steps, warmup, world, device):
    """torch scaled_dot_product_attention with the cuDNN backend on the same
    tensors, timed the same way (a library comparator, not this repo's path),
    plus the largest difference between its output and ours."""
    try:
        from torch.nn.attention import SDPBackend, sdpa_kernel
        with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
            f = lambda: torch.nn.functional.scaled_dot_product_attention(  # noqa: E731
                q, k, v, is_causal=causal)
            for _ in range(max(warmup, 1)):
                ref = f()
            torch.cuda.synchronize()
            ms = timed_loop(f, steps, world, device)
        n = min(4, q.shape[1])
        diff = (ref[:, :n].float() - o[:, :n].float()).abs().max().item()
        del ref
        tf = flops_local / (ms * 1e-3) / 1e12
        return {"value": tf, "unit": "TFLOP/s per GPU", "ms_per_step": ms,
                "max_abs_diff_vs_ours": diff,
                "what": "torch SDPA, cuDNN backend, same tensors, same event window"}
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}


def bench_attention(args, fab, device, world, rank):
    cfg = ATTN_CONFIGS[args.config]
    num_pairs = cfg["B"] * cfg["H"] if args.pairs <= 0 else min(args.pairs, cfg["B"] * cfg["H"])
    pairs = shard_range(num_pairs, world, rank)
    if args.sdpa_only:
        q, k, v = make_qkv(cfg, pairs, device)
        o = torch.empty_like(q)
        flops_local = attn_flops(cfg, len(pairs))
        r = sdpa_same_gpu(q, k, v, o, cfg["causal"], flops_local, args.steps, args.warmup,
                          world, device)
        return {"metric": METRIC, "impl": "torch SDPA (cuDNN) comparator", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup,
                "config": workload_config(args, cfg, num_pairs), "sdpa_same_gpu": r}
    t = attention_timing(args, fab, cfg, pairs, device, world, args.steps, args.warmup)
    q, k, v, o, ms = t["q"], t["k"], t["v"], t["o"], t["ms"]
    flops_total = attn_flops(cfg, num_pairs)
    value = flops_total / (ms * 1e-3) / 1e12
    flops_local = attn_flops(cfg, len(pairs))
    achieved = flops_local / (ms * 1e-3) / 1e12
    peaks = load_peaks()
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "ms_per_step_min": t["reps"]["min_ms"], "reps": t["reps"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": f"synthetic: seeded N(0,1)*{cfg['amp']} per (batch, head) pair (Philox), bf16",
        "config": workload_config(args, cfg, num_pairs),
        "per_gpu_tflops": value / world,
        "pct_of_peak": 100.0 * achieved / peaks["bf16_tflops"],
        "roofline": roofline(achieved, peaks,
                             load_traffic(args.config) if args.pairs <= 0 else None),
        "gpu_launches": args.steps,
        "clocks": t["clocks"],
        "rank_ms_per_step": {"fastest": t["rank_ms"]["min"], "slowest": t["rank_ms"]["max"]},
        "flops_per_step": flops_total,
        "flop_convention": "4*B*H*S^2*D, halved when causal (old/benchmark.py:131)",
    }
    if args.kernel_only:
        return line

    # verification: seeded subset of pairs vs a torch fp32 reference, per owner
    vp = verify_pairs(num_pairs, args.verify_pairs)
    max_abs, sum_abs, count = 0.0, 0.0, 0
    for p in vp:
        if p in pairs:
            i = p - pairs.start
            ref = torch_ref_pair(q[0, i], k[0, i], v[0, i], cfg["causal"])
            d = (o[0, i].float() - ref).abs()
            max_abs = max(max_abs, d.max().item())
            sum_abs += d.sum().item()
            count += d.numel()
    verify = reduce_error_stats(max_abs, sum_abs, count, device)
    verify.update({"pairs": len(vp), "ok": verify["max_abs"] <= 2e-2 and verify["mean_abs"] <= 2e-3,
                   "reference": "torch fp32 on GPU, per pair"})
    line["verify"] = verify

    if not args.no_sdpa:
        line["sdpa_same_gpu"] = sdpa_same_gpu(q, k, v, o, cfg["causal"], flops_local,
                                              args.steps, args.warmup, world, device)
    if world > 1:
        line["gather"] = timed_gather(o, world, rank, device)
        line["gather_ms"] = line["gather"]["ms"]

    if not args.no_e2e:
        line["e2e"] = attention_e2e(args, fab, cfg, q, k, v, world, device, flops_total)
        line["host_link"] = host_link_probe(world, device)

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tf, npairs_cpu, secs = cpu_attention_sample(cfg, args.cpu_seconds)
        line["cpu_baseline"] = {
            "value": tf, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{npairs_cpu} (batch, head) pairs of {args.config} in {secs:.1f} s "
                      "(pairs are independent; throughput scales linearly)",
            "cpu": cpu_model(),
            "what": "oracle.naive_torch_pair: correct restatement of pytorch-naive.py:41-63"}
    else:
        line["cpu_baseline"] = None

    del q, k, v, o, t
    if world == 1 and args.config == "cfg2" and args.pairs <= 0 and not args.no_secondary:
        line["secondary"] = secondary_lines(args, fab, device, peaks)
    return line


def secondary_lines(args, fab, device, peaks):
    """The other single-GPU BASELINE configurations, device-timed on the same
    box as the headline: cfg1 (D = 64, non-causal) with its cuDNN comparator,
    and the cfg3 MLP block."""
    out = {}
    cfg = ATTN_CONFIGS["cfg1"]
    n = cfg["B"] * cfg["H"]
    t = attention_timing(args, fab, cfg, range(n), device, 1, args.steps, args.warmup)
    flops = attn_flops(cfg, n)
    tf = flops / (t["ms"] * 1e-3) / 1e12
    ref = torch_ref_pair(t["q"][0, 0], t["k"][0, 0], t["v"][0, 0], cfg["causal"])
    err = (t["o"][0, 0].float() - ref).abs()
    out["cfg1"] = {"workload": "attention forward non-causal bf16 B=8 H=16 S=4096 D=64",
                   "value": tf, "unit": "TFLOP/s", "ms_per_step": t["ms"],
                   "ms_per_step_min": t["reps"]["min_ms"],
                   "roofline": roofline(tf, peaks, load_traffic("cfg1")),
                   "clocks": t["clocks"], "gpu_launches": args.steps,
                   "verify": {"pairs": 1, "max_abs": err.max().item(),
                              "mean_abs": err.mean().item()}}
    if not args.no_sdpa:
        out["cfg1"]["sdpa_same_gpu"] = sdpa_same_gpu(t["q"], t["k"], t["v"], t["o"],
                                                     cfg["causal"], flops, args.steps,
                                                     args.warmup, 1, device)
    del t, ref, err
    out["legacy_fp16"] = legacy_fp16_line(args, fab, device, peaks)
    m = mlp_timing(args, fab, MLP_CONFIGS["cfg3"], MLP_CONFIGS["cfg3"]["M"], device, 1)
    out["cfg3"] = {"workload": "MLP block Y = gelu_tanh(X W1) W2, M=8192 K=4096 N=16384 bf16",
                   "value": m["value"], "unit": "TFLOP/s", "ms_per_step": m["ms"],
                   "ms_per_step_min": m["reps"]["min_ms"],
                   "roofline": roofline(m["dominant_tflops"], peaks, load_traffic("cfg3")),
                   "gemm_ms": m["gemm_ms"], "torch_same_gpu": m["torch_same_gpu"],
                   "clocks": m["clocks"], "gpu_launches": 2 * args.steps,
                   "verify": m["verify"]}
    return out


def legacy_fp16_line(args, fab, device, peaks):
    """The reference's legacy harness problem (old/benchmark.py:90-96): B8
    S2048 H16 D64, fp16, non-causal, (B, S, H, D) tensors passed as strides;
    device-timed like the headline, with torch SDPA (cuDNN) on the same
    permuted tensors."""
    B, S, H, D = 8, 2048, 16, 64
    g = torch.Generator(device=device).manual_seed(7)
    q, k, v = (torch.randn((B, S, H, D), generator=g, device=device).to(torch.float16)
               for _ in range(3))
    o = torch.empty_like(q)
    ov = o.permute(0, 2, 1, 3)
    qv, kv, vv = (t.permute(0, 2, 1, 3) for t in (q, k, v))
    step = lambda: fab.attention(qv, kv, vv, out=ov)  # noqa: E731
    for _ in range(max(args.warmup, 1)):
        step()
    torch.cuda.synchronize()
    with ClockSampler(local_index(device)) as clk:
        ms = timed_loop(step, args.steps, 1, device)
    flops = 4.0 * B * H * S * S * D
    tf = flops / (ms * 1e-3) / 1e12
    ref = torch_ref_pair(qv[0, 0], kv[0, 0], vv[0, 0], False)
    err = (ov[0, 0].float() - ref).abs()
    line = {"workload": "legacy harness: attention (B, S, H, D) = (8, 2048, 16, 64) fp16, "
                        "non-causal, strided layout",
            "value": tf, "unit": "TFLOP/s", "ms_per_step": ms, "dtype": "f16",
            "roofline": roofline(tf, peaks, None), "clocks": clk.summary(),
            "gpu_launches": args.steps,
            "verify": {"pairs": 1, "max_abs": err.max().item(), "mean_abs": err.mean().item()}}
    if not args.no_sdpa:
        line["sdpa_same_gpu"] = sdpa_same_gpu(qv, kv, vv, ov, False, flops, args.steps,
                                              args.warmup, 1, device)
    return line


def timed_gather(o, world, rank, device, reps=3):
    """NCCL gather of the O shards on rank 0: one untimed gather (communicator
    and channel set-up), then ``reps`` gathers timed with CUDA events, max over
    ranks.  GB/s counts the bytes that land on rank 0 from the other ranks."""
    bufs = [torch.empty_like(o) for _ in range(world)] if rank == 0 else None

    def once():
        dist.gather(o, gather_list=bufs, dst=0)
    once()
    torch.cuda.synchronize()
    ms = timed_loop(once, reps, world, device)
    moved = (world - 1) * o.numel() * o.element_size()
    return {"ms": ms, "gbs_into_rank0": moved / (ms * 1e-3) / 1e9, "bytes_into_rank0": moved,
            "reps": reps, "what": "warm dist.gather of the O shards (NCCL), CUDA events"}


def host_link_probe(world, device, nbytes=512 << 20, reps=3):
    """Plain pinned-host <-> device copies (one cudaMemcpyAsync each), every
    rank at once, timed with CUDA events: the host-link bound that the e2e
    figure runs against.  Max over ranks; the aggregate is world x bytes over
    that time."""
    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(nbytes, dtype=torch.uint8, device=device)
    out = {"bytes_per_gpu": nbytes, "reps": reps}
    for name, fn in (("h2d", lambda: d.copy_(h, non_blocking=True)),
                     ("d2h", lambda: h.copy_(d, non_blocking=True))):
        fn()
        torch.cuda.synchronize()
        ms = timed_loop(fn, reps, world, device)
        out[f"{name}_gbs_per_gpu"] = nbytes / (ms * 1e-3) / 1e9
        out[f"{name}_gbs_aggregate"] = world * nbytes / (ms * 1e-3) / 1e9
    return out


def local_index(device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def torch_ref_pair(q, k, v, causal, row_chunk=2048):
    qf, kf, vf = q.float(), k.float(), v.float()
    S, D = qf.shape
    out = torch.empty_like(qf)
    for r0 in range(0, S, row_chunk):
        s = (qf[r0:r0 + row_chunk] @ kf.t()) / math.sqrt(D)
        if causal:
            rows = torch.arange(r0, min(S, r0 + row_chunk), device=q.device)[:, None]
            s = s.masked_fill(torch.arange(S, device=q.device)[None, :] > rows, float("-inf"))
        out[r0:r0 + row_chunk] = torch.softmax(s, dim=-1) @ vf
    return out


def attention_e2e(args, fab, cfg, q, k, v, world, device, flops_total):
    """Same metric through the public API fed from pinned host buffers:
    H2D of this rank's Q/K/V, the kernel, D2H of O, every step."""
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    oh = torch.empty(q.shape, dtype=torch.bfloat16, pin_memory=True)
    ws = {}
    step = lambda: fab.attention_from_host(qh, kh, vh, causal=cfg["causal"], out=oh,  # noqa
                                           device=device, workspace=ws,
                                           chunks=args.e2e_chunks)
    step()
    torch.cuda.synchronize()
    steps = max(1, args.e2e_steps)
    ms = timed_loop(step, steps, world, device)
    return {"value": flops_total / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "steps": steps, "h2d_bytes_per_step": 3 * q.numel() * 2 * world,
            "d2h_bytes_per_step": q.numel() * 2 * world,
            "path": "attention_from_host: pinned host -> device -> host, (batch, head) pairs "
                    f"in {args.e2e_chunks} chunks pipelined over copy-in / kernel / copy-out "
                    "streams"}


# The reference's own problem and its published numbers (NVIDIA L4, fp32,
# results/attn-full.json:38-41 -- the grammar search's best kernel -- and
# results/flash2-sota.json:46-49 -- torch SDPA).
REF512_FLOPS = 4 * 512 * 512 * 64 + 6 * 512 * 512      # program_flops, kernel_ast.py:1110-1147
REF512_PUBLISHED_TFLOPS = 0.646


def bench_ref512(args, fab, device, world, rank):
    """The reference's kernel-module call fn(KT, Q, V) at N=512, d=64 with fp32
    device arrays, exactly as its bench.py:45-74 times it (inputs and the
    callee-allocated output, casts included), through kernel_module.fn."""
    from cs348k_fast_attention_grammar_b200 import kernel_module
    g = torch.Generator(device=device).manual_seed(0)
    ins = [torch.randn(*dims, generator=g, device=device, dtype=torch.float32)
           for _name, dims in kernel_module.KERNEL_META["inputs"]]
    step = lambda: kernel_module.fn(*ins)  # noqa: E731
    # One call is ~20 us of host and GPU work: time at least 1000 of them so
    # the loop's fixed cost does not weigh on the per-call figure.
    warmup, steps = max(args.warmup, 200), max(args.steps, 1000)
    for _ in range(warmup):
        step()
    with ClockSampler(local_index(device)) as clk:
        ms = timed_loop(step, steps, world, device)
    value = REF512_FLOPS * world / (ms * 1e-3) / 1e12
    # Like-for-like on the same GPU: the reference's flash-attn2-sota.py call,
    # torch SDPA on [1, 1, 512, 64] fp32 (its fn(K, Q, V)), timed the same way.
    KT, Q, V = ins
    k4, q4, v4 = (t.reshape(1, 1, 512, 64) for t in (KT.t().contiguous(), Q, V))
    sdpa = lambda: torch.nn.functional.scaled_dot_product_attention(q4, k4, v4)  # noqa: E731
    for _ in range(warmup):
        sdpa()
    ms_sdpa = timed_loop(sdpa, steps, world, device)
    peaks = load_peaks()
    return {"metric": "reference kernel-module attention TFLOP/s (program_flops, N=512 d=64)",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": value / REF512_PUBLISHED_TFLOPS,
            "vs_baseline_note": "published 0.646 TFLOP/s is the reference's best searched "
                                "kernel on an NVIDIA L4 (results/attn-full.json)",
            "dtype": "bf16 compute, fp32 in/out", "data": "synthetic: randn fp32 (bench.py:45-46)",
            "config": {"workload": "ref512: fn(KT[64,512], Q[512,64], V[512,64]) fp32, "
                                   "non-causal, kernel-module protocol",
                       "l2": "not flushed (1 MB of inputs)"},
            "roofline": roofline(4 * 512 * 512 * 64 / (ms * 1e-3) / 1e12, peaks, None),
            "sdpa_same_gpu": {"value": REF512_FLOPS * world / (ms_sdpa * 1e-3) / 1e12,
                              "unit": "TFLOP/s", "ms_per_call": ms_sdpa,
                              "what": "torch scaled_dot_product_attention fp32 [1,1,512,64] "
                                      "(flash-attn2-sota.py's call) on this GPU"},
            "gpu_launches": 2 * steps, "clocks": clk.summary(), "cpu_baseline": None,
            "e2e": None}


def run_reference_ref512(args):
    """The reference's numerically correct naive path at its own problem on
    the host's cores (oracle.naive_fn restates pytorch-naive.py's intent)."""
    import numpy as np
    import oracle
    rng = np.random.default_rng(0)
    KT, Q, V = (rng.standard_normal(s).astype(np.float32) for s in ((64, 512), (512, 64), (512, 64)))
    for _ in range(args.warmup):
        oracle.naive_fn(KT, Q, V)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.naive_fn(KT, Q, V)
    ms = 1e3 * (time.perf_counter() - t0) / args.steps
    value = REF512_FLOPS / (ms * 1e-3) / 1e12
    line = {"impl": "reference", "metric": "reference kernel-module attention TFLOP/s "
            "(program_flops, N=512 d=64)", "value": value, "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "ref512"},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": host_cores(),
                             "kind": "port", "sample": "the whole N=512 d=64 problem per step"},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def mlp_timing(args, fab, cfg, rows_total, device, world, rank=0):
    """This rank's row block of the first ``rows_total`` rows of X with the
    full weights: warm-up, timed MLP blocks (window mean, clocks), five
    individually timed reps, per-GEMM durations, and a 32-row spot check
    against a torch fp32 reference."""
    x_full, w1, w2 = make_mlp(dict(cfg, M=rows_total), device)
    K, N = cfg["K"], cfg["N"]
    rows = shard_range(rows_total, world, rank)
    x = x_full[rows.start:rows.stop].contiguous()
    del x_full
    Mr = x.shape[0]
    hidden = torch.empty((Mr, N), dtype=torch.bfloat16, device=device)
    y = torch.empty((Mr, K), dtype=torch.bfloat16, device=device)
    step = lambda: fab.mlp(x, w1, w2, act="gelu_tanh", hidden=hidden, out=y)  # noqa: E731
    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()
    with ClockSampler(local_index(device)) as clk:
        ms = timed_loop(step, args.steps, world, device)
    reps = timed_reps(step, 5, world, device)
    # per-GEMM durations for the roofline of the dominant kernel: each GEMM
    # alone over its own event window of the same number of launches
    t1 = timed_loop(lambda: fab.gemm_act(x, w1, act="gelu_tanh", out=hidden), args.steps,
                    world, device)
    t2 = timed_loop(lambda: fab.gemm_act(hidden, w2, act="none", out=y), args.steps,
                    world, device)
    # library comparator on the same tensors: cuBLAS GEMMs + torch's tanh-GELU
    ref_fn = lambda: torch.nn.functional.gelu(x @ w1, approximate="tanh") @ w2  # noqa: E731
    for _ in range(max(args.warmup, 1)):
        ref_fn()
    ms_lib = timed_loop(ref_fn, args.steps, world, device)
    gemm_flops = 2.0 * Mr * K * N
    sel = torch.from_numpy(__import__("numpy").random.default_rng(rank).choice(
        Mr, min(32, Mr), replace=False)).to(device)
    h = torch.nn.functional.gelu(x[sel].float() @ w1.float(), approximate="tanh")
    ref = h.to(torch.bfloat16).float() @ w2.float()
    d = (y[sel].float() - ref).abs()
    verify = reduce_error_stats(d.max().item(), d.sum().item(), d.numel(), device)
    verify.update({"ok": verify["max_abs"] <= 2e-2 and verify["mean_abs"] <= 2e-3,
                   "reference": "torch fp32 on GPU, 32 rows per rank"})
    flops = 4.0 * rows_total * K * N
    return {"x": x, "w1": w1, "w2": w2, "y": y, "ms": ms, "reps": reps,
            "clocks": clk.summary(), "value": flops / (ms * 1e-3) / 1e12, "flops": flops,
            "gemm_ms": {"gemm1_gelu": t1, "gemm2": t2},
            "torch_same_gpu": {"value": flops / (ms_lib * 1e-3) / 1e12,
                               "unit": "TFLOP/s", "ms_per_step": ms_lib,
                               "what": "torch: gelu(x @ w1, tanh) @ w2 (cuBLAS GEMMs + "
                                       "elementwise GELU), same tensors, same event window"},
            "dominant_tflops": gemm_flops / (max(t1, t2) * 1e-3) / 1e12, "verify": verify}


def bench_mlp(args, fab, device, world, rank):
    """MLP block, rows of X sharded over the ranks (weights replicated; every
    rank regenerates the same seeded tensors and keeps its row block), Y
    gathered on rank 0 after timing (warm, event-timed) and spot-checked
    against a torch fp32 reference."""
    import oracle
    cfg = MLP_CONFIGS[args.config]
    K, N = cfg["K"], cfg["N"]
    M = cfg["M"] if args.rows <= 0 else min(args.rows, cfg["M"])
    m = mlp_timing(args, fab, cfg, M, device, world, rank)
    x, w1, w2, y, ms = m["x"], m["w1"], m["w2"], m["y"], m["ms"]
    Mr = x.shape[0]
    peaks = load_peaks()
    line = {"metric": "MLP block TFLOP/s", "value": m["value"], "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "ms_per_step_min": m["reps"]["min_ms"], "reps": m["reps"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic: X~N(0,1), W~N(0,1/fan_in), bf16",
            "config": {"workload": f"{args.config}: Y=gelu_tanh(X W1) W2, M={M} K={K} N={N}",
                       "parallelism": f"rows of X over {world} ranks, weights replicated",
                       "l2": "inputs larger than L2 (X 64 MiB + W1 128 MiB + W2 128 MiB)"},
            "pct_of_peak": 100.0 * m["value"] / world / peaks["bf16_tflops"],
            "roofline": roofline(m["dominant_tflops"], peaks,
                                 load_traffic(args.config) if args.rows <= 0 else None),
            "gemm_ms": m["gemm_ms"], "torch_same_gpu": m["torch_same_gpu"],
            "gpu_launches": 2 * args.steps, "clocks": m["clocks"], "verify": m["verify"]}
    if args.kernel_only:
        return line
    e2e = None
    if not args.no_e2e:
        # Same metric through the public API with X streamed from pinned host
        # memory and Y returned to it every step (weights stay resident).
        xh = x.cpu().pin_memory()
        yh = torch.empty((Mr, K), dtype=torch.bfloat16, pin_memory=True)
        ws = {}
        e2e_step = lambda: fab.mlp_from_host(xh, w1, w2, act="gelu_tanh", out=yh,  # noqa: E731
                                             workspace=ws)
        e2e_step()
        torch.cuda.synchronize()
        steps = max(1, args.e2e_steps)
        ms_e2e = timed_loop(e2e_step, steps, world, device)
        e2e = {"value": m["flops"] / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
               "ms_per_step": ms_e2e, "steps": steps, "h2d_bytes_per_step": M * K * 2,
               "d2h_bytes_per_step": M * K * 2,
               "path": "mlp_from_host: pinned host X -> device -> host Y, rows in 4 chunks "
                       "pipelined over copy-in / GEMMs / copy-out streams; weights resident"}
    line["e2e"] = e2e
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(host_cores())
        rows_cpu = 128
        xc, w1c, w2c = (t.float() for t in make_mlp(dict(cfg, M=rows_cpu), "cpu"))
        t_total, n_done = 0.0, 0
        while t_total < args.cpu_seconds or n_done == 0:
            t0 = time.perf_counter()
            torch.nn.functional.gelu(xc @ w1c, approximate="tanh") @ w2c
            t_total += time.perf_counter() - t0
            n_done += 1
        cpu = {"value": n_done * oracle.mlp_flops(rows_cpu, K, N) / t_total / 1e12,
               "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{n_done} x {rows_cpu} rows of X (full weights) in {t_total:.1f} s; "
                         "rows are independent",
               "cpu": cpu_model(),
               "what": "fp32 torch gelu_tanh(X W1) W2, the oracle's MLP formula"}
    line["cpu_baseline"] = cpu
    if world > 1 and M % world == 0:
        line["gather"] = timed_gather(y.view(1, Mr, K), world, rank, device)
        line["gather_ms"] = line["gather"]["ms"]
    return line


def bench_ln(args, fab, device, world, rank):
    """Row LayerNorm alone (the last stage of the reference's MLP block) on
    ``--rows`` rows of cfg3's feature width: an HBM-bound kernel."""
    K = MLP_CONFIGS["cfg3"]["K"]
    rows = args.rows if args.rows > 0 else 16384
    g = torch.Generator(device=device).manual_seed(0)
    x = torch.randn((rows, K), generator=g, device=device).to(torch.bfloat16)
    y = torch.empty_like(x)
    step = lambda: fab.layer_norm_rows(x, out=y)  # noqa: E731
    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()
    with ClockSampler(local_index(device)) as clk:
        ms = timed_loop(step, args.steps, world, device)
    nbytes = 4.0 * rows * K
    gbs = nbytes / (ms * 1e-3) / 1e9
    peaks = load_peaks()
    return {"metric": "row LayerNorm GB/s", "value": gbs * world, "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: N(0,1) bf16",
            "config": {"workload": f"ln: row LayerNorm {rows} x {K} bf16 (no affine)"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"], "traffic": None},
            "gpu_launches": args.steps, "clocks": clk.summary()}


if __name__ == "__main__":
    sys.exit(main())
