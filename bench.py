"""Benchmark of the B200 causal-attention / warp-softmax path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl pmkl_b200|reference]

Default workload: BASELINE config 3, causal self-attention bf16 B16 H32 S4096
D128, inputs N(0,1) (synthetic, seeded), one step = one forward of the whole
configuration (the rank's (batch, head) shard of it when N > 1).  Inputs are
1.5 GB (> 126 MB L2), so no L2 flush is needed between steps.

One JSON line on rank 0:
  value     whole-job TFLOP/s (4*D*S(S+1)/2 per (b,h) slice: the two
            contractions over the unmasked pairs) from the device-timed region
            (CUDA events, max over ranks), inputs resident in HBM;
  e2e       the same metric through the public API
            (pmkl_function.fused_self_attention) with the step's inputs copied
            host->device from pinned memory and O, m, l copied back inside the
            timed region; the step's slices go in --e2e-chunks chunks whose
            copies overlap the attention of the neighbouring chunks;
  roofline  the attention kernel's achieved TFLOP/s per launch vs the measured
            bf16 peak (MEASURED_PEAKS.json), with the exp unit's (MUFU)
            fraction beside it;
  clocks    SM clock and clock-event reasons sampled through NVML every few
            milliseconds during the timed region;
  cpu_baseline  the reference's own CPU implementation (its torch extension
            compiled from its sources into oracle/_ref) on a bounded sample;
  sub       the default run also measures BASELINE configs 2 and 4 (attention)
            and 5 (softmax) the same way, each with its own value, roofline
            (config 2 against the exp unit, which binds at head size 64;
            softmax against the measured copy bandwidth), end-to-end leg, CPU
            baseline and clocks (--no-sub skips them).

--impl reference runs that reference CPU implementation instead, with one
worker process per host core, each step a bounded sample of the workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

ATTN_METRIC = "causal attention TFLOP/s/GPU & % dense peak; whole-box TFLOP/s at 1/2/4/8"

WORKLOADS = {
    # name: (B, H, S, D, dtype, std, causal, description)
    "attention": (16, 32, 4096, 128, "bfloat16", 1.0, True, "BASELINE config 3: causal self-attention bf16 B16 H32 S4096 D128"),
    "attention-cfg2": (8, 16, 1024, 64, "float16", 1.0, True, "BASELINE config 2: causal self-attention fp16 B8 H16 S1024 D64"),
    "attention-cfg4": (1, 32, 32768, 128, "bfloat16", 0.5, True, "BASELINE config 4: causal self-attention bf16 B1 H32 S32768 D128"),
    "attention-cfg1": (2, 4, 128, 64, "float32", 1.0, True, "BASELINE config 1: causal self-attention fp32 B2 H4 S128 D64"),
    "softmax": (65536, 1024, None, None, "float32", 2.0, None, "BASELINE config 5: warp softmax fp32 65536 x 1024"),
    "softmax-bf16": (65536, 1024, None, None, "bfloat16", 2.0, None,
                     "warp softmax bf16 in / bf16 out 65536 x 1024 (the general kernel's path)"),
    "attention-bwd": (16, 32, 4096, 128, "bfloat16", 1.0, True,
                      "backward of BASELINE config 3: fused_self_attention_bw bf16 B16 H32 S4096 D128 causal"),
    "softmax-gen": (65536, 1023, None, None, "float32", 2.0, None,
                    "warp softmax fp32 65536 x 1023 (odd row length: the general kernel's path)"),
    "attention-bwd-fp32": (8, 32, 2048, 64, "float32", 1.0, True,
                           "backward fp32 B8 H32 S2048 D64 causal (the CUDA-core backward's path)"),
}
BWD_METRIC = "causal attention backward TFLOP/s (whole box)"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="attention", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="pmkl_b200", choices=["pmkl_b200", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--e2e-chunks", type=int, default=8,
                    help="slice chunks per end-to-end step (copies of one chunk overlap the attention of another)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--no-sub", action="store_true",
                    help="default workload only: skip the configs 2, 4 and 5 sub-records")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--kernel", type=int, default=0,
                    help="pmkl_attention_kernel value for the device-timed leg (0 = automatic choice)")
    ap.add_argument("--shape", default=None,
                    help="override the workload size for profiler captures: B,H,S,D for attention, "
                         "ROWS,COLS for softmax (the bench line then describes that size)")
    return ap.parse_args()


def attn_flops_per_slice(S: int, D: int, causal: bool) -> float:
    pairs = S * (S + 1) / 2 if causal else S * S
    return 4.0 * D * pairs


def attn_bwd_flops_per_slice(S: int, D: int, causal: bool) -> float:
    """The five contractions of the backward (S, dP, dV, dK, dQ) over the
    unmasked pairs: 2.5 x the forward's."""
    return 2.5 * attn_flops_per_slice(S, D, causal)


def shard(n_units: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous split of n_units over world ranks (sizes differ by <= 1)."""
    lo = rank * n_units // world
    hi = (rank + 1) * n_units // world
    return lo, hi


def measured_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return {"bf16_tflops": d["bf16_tflops"], "bf16_tflops_sustained": d.get("bf16_tflops_sustained"),
                "hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def profile_traffic(workload: str):
    """DRAM bytes per unit from the committed ncu summary, if any."""
    p = REPO / "profiles" / "traffic.json"
    if not p.is_file():
        return None
    d = json.loads(p.read_text())
    return d.get(workload)


# ----------------------------------------------------------------------------- clocks
REASON_BITS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}


class ClockSampler:
    """Samples SM clock, power and clock-event reasons of this rank's GPU
    every few milliseconds through NVML (read-only queries) on a background
    thread, so that even a timed region of a few tens of milliseconds holds
    several samples.  window(t0, t1) summarises the samples taken inside a
    host-time window.  Falls back to nothing when NVML is unavailable."""

    def __init__(self, local: int, enabled: bool, period_s: float = 0.004):
        import threading

        self.samples = []
        self.thread = None
        self.max_mhz = None
        if not enabled:
            return
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self.nvml = pynvml
            try:
                uuid = str(torch.cuda.get_device_properties(local).uuid)
                self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[local]) if vis else local
                self.h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            return
        self.stop_flag = threading.Event()
        self.period = period_s
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def _run(self):
        nv = self.nvml
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop_flag.is_set():
            try:
                self.samples.append((time.perf_counter(), nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM),
                                     int(get_reasons(self.h)), nv.nvmlDeviceGetPowerUsage(self.h) / 1e3))
            except Exception:
                pass
            time.sleep(self.period)

    def window(self, t0: float, t1: float) -> dict | None:
        sel = [x for x in list(self.samples) if t0 <= x[0] <= t1]
        if not sel:
            # the region was shorter than one sampling period: the nearest sample
            later = [x for x in list(self.samples) if x[0] >= t0]
            sel = later[:1]
        if not sel:
            return None
        reasons = sorted({n for n, bit in REASON_BITS.items() for x in sel if x[2] & bit})
        return {"sm_mhz": statistics.median(x[1] for x in sel), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(sel), "power_w_max": max(x[3] for x in sel), "source": "NVML, every ~4 ms"}

    def stop(self):
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join(timeout=2)


# ----------------------------------------------------------------------------- dist
def dist_init(n_gpus: int):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus and world > 1:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    import torch
    import torch.distributed as dist

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x: float, world: int) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def timed_loop(step, steps: int, warmup: int, world: int, sampler: "ClockSampler | None" = None):
    """W untimed steps, then K steps between barrier + synchronize; returns
    (total ms of the K steps, list of per-step ms, clock summary of the timed
    region or None) on this rank."""
    import torch

    for _ in range(warmup):
        step()
    barrier(world)
    t_host0 = time.perf_counter()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    start.record()
    for i in range(steps):
        ev[i][0].record()
        step()
        ev[i][1].record()
    end.record()
    torch.cuda.synchronize()
    t_host1 = time.perf_counter()
    barrier(world)
    clocks = sampler.window(t_host0, t_host1) if sampler is not None else None
    return start.elapsed_time(end), [a.elapsed_time(b) for a, b in ev], clocks


# ----------------------------------------------------------------------------- reference CPU code
def _ref_attention_worker(args):
    """Runs the reference's CPU forward (its torch extension, built from its
    sources into oracle/_ref) on one seeded causal prefix problem."""
    r, D, dtype_name, std, causal, seed = args
    import torch

    torch.set_num_threads(1)
    from oracle import build_ref

    ext = build_ref.load_ref_ext()
    dt = getattr(torch, dtype_name)
    g = torch.Generator().manual_seed(seed)
    q, k, v = [(torch.randn(1, 1, r, D, generator=g) * std).to(dt) for _ in range(3)]
    t0 = time.perf_counter()
    ext.fused_self_attention_fw(q, k, v, causal)
    return time.perf_counter() - t0


def _ref_attention_bwd_worker(args):
    """Runs the reference's CPU backward (fused_self_attention_bw of its torch
    extension, O(S^3 D)) on one seeded r-row problem; returns seconds."""
    r, D, dtype_name, std, causal, seed = args
    import torch

    torch.set_num_threads(1)
    from oracle import build_ref

    ext = build_ref.load_ref_ext()
    dt = getattr(torch, dtype_name)
    g = torch.Generator().manual_seed(seed)
    q, k, v, do = [(torch.randn(1, 1, r, D, generator=g) * std).to(dt) for _ in range(4)]
    _, m, l = ext.fused_self_attention_fw(q, k, v, causal)
    t0 = time.perf_counter()
    ext.fused_self_attention_bw(do, q, k, v, m, l, causal)
    return time.perf_counter() - t0


def pick_bwd_rows(D: int, dtype_name: str, causal: bool, budget_s: float) -> int:
    """Largest r whose single-core reference backward (time ~ r^3) fits budget_s."""
    t = _ref_attention_bwd_worker((32, D, dtype_name, 1.0, causal, 0))
    r = int(32 * (budget_s / max(t, 1e-6)) ** (1.0 / 3.0))
    return max(16, min(512, r))


def _ref_softmax_worker(args):
    """The reference's host_softmax_forward (compiled from its sources into
    oracle/_ref) on `rows` seeded rows, `reps` times over the same input;
    returns the seconds of the calls."""
    rows, el, seed = args[:3]
    reps = args[3] if len(args) > 3 else 1
    import numpy as np

    from oracle import build_ref

    fn = build_ref.load_ref_softmax()
    x = (np.random.default_rng(seed).standard_normal(rows * el) * 2).astype(np.float32)
    y = np.empty_like(x)
    t0 = time.perf_counter()
    for _ in range(reps):
        fn(y.ctypes.data, x.ctypes.data, el, el, rows)
    return time.perf_counter() - t0


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def pick_prefix_rows(S: int, D: int, dtype_name: str, causal: bool, budget_s: float) -> int:
    """Largest causal prefix length r <= S whose single-core reference time
    fits budget_s, from one calibration run at r = 256."""
    t = _ref_attention_worker((256, D, dtype_name, 1.0, causal, 0))
    per_flop = t / attn_flops_per_slice(256, D, causal)
    r = int(math.sqrt(2.0 * budget_s / per_flop / (4.0 * D)))
    return max(128, min(S, r))


def cpu_baseline_attention(S, D, dtype_name, std, causal, budget_s=20.0) -> dict:
    """Single core, one bounded sample: the reference on a causal prefix of
    one (b, h) slice (rows [0, r) of a slice are exactly the prefix problem)."""
    r = pick_prefix_rows(S, D, dtype_name, causal, budget_s)
    t = _ref_attention_worker((r, D, dtype_name, std, causal, 7))
    return {"value": attn_flops_per_slice(r, D, causal) / t / 1e12, "unit": "TFLOP/s", "cores": 1,
            "kind": "reference",
            "sample": f"reference fused_self_attention_fw (CPU, {dtype_name}) on one (b,h) slice, causal prefix "
                      f"of {r} of {S} rows, D={D}, {t:.1f} s on 1 core"}


def reference_record(name: str, wl, steps: int, warmup: int, budget_total_s: float) -> dict:
    """The reference's own CPU implementation of workload `name` on all host
    cores (one spawn-started process per core), each step a bounded sample."""
    import multiprocessing as mp

    B, H, S, D, dtype_name, std, causal, desc = wl
    cores = host_cores()
    ctx = mp.get_context("spawn")
    total_steps = steps + warmup
    budget = max(0.5, min(20.0, budget_total_s / max(1, total_steps)))
    if name.startswith("softmax"):
        rows_total, el = B, H
        probe = _ref_softmax_worker((256, el, 0))
        rows = max(1, min(rows_total // cores if rows_total >= cores else rows_total, int(budget / (probe / 256))))
        work = [(rows, el, 100 + i) for i in range(cores)]
        unit_per_step = cores * rows * el * 8.0 / 1e9  # GB moved per step (read + write fp32)
        unit, metric = "GB/s", SOFTMAX_METRIC
        sample = f"reference host_softmax_forward (CPU fp32), {rows} rows x {el} per core per step"
    elif name.startswith("attention-bwd"):
        r = pick_bwd_rows(D, dtype_name, causal, budget)
        work = [(r, D, dtype_name, std, causal, 100 + i) for i in range(cores)]
        unit_per_step = cores * attn_bwd_flops_per_slice(r, D, causal) / 1e12
        unit, metric = "TFLOP/s", BWD_METRIC
        sample = (f"reference fused_self_attention_bw (CPU, {dtype_name}, O(S^3 D)): per step each of {cores} "
                  f"worker processes runs the backward of one {r}-row causal (b,h) problem, D={D}")
    else:
        r = pick_prefix_rows(S, D, dtype_name, causal, budget)
        work = [(r, D, dtype_name, std, causal, 100 + i) for i in range(cores)]
        unit_per_step = cores * attn_flops_per_slice(r, D, causal) / 1e12
        unit, metric = "TFLOP/s", ATTN_METRIC
        sample = (f"reference fused_self_attention_fw (CPU, {dtype_name}): per step each of {cores} worker "
                  f"processes runs a causal prefix of {r} of {S} rows of one (b,h) slice, D={D}")
    fn = (_ref_softmax_worker if name.startswith("softmax") else
          _ref_attention_bwd_worker if name.startswith("attention-bwd") else _ref_attention_worker)
    times = []
    with ctx.Pool(cores) as pool:
        for i in range(total_steps):
            t0 = time.perf_counter()
            pool.map(fn, work, chunksize=1)
            dt = time.perf_counter() - t0
            if i >= warmup:
                times.append(dt)
    tot = sum(times)
    value = unit_per_step * len(times) / tot
    return {
        "impl": "reference", "metric": metric, "value": value, "unit": unit,
        "steps": steps, "warmup": warmup, "ms_per_step": 1e3 * tot / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype_name,
        "data": "synthetic (seeded N(0, std^2))",
        "config": {"workload": desc, "sample": sample},
        "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_reference_arm(args, wl, rank, world):
    """--impl reference: the main workload, then (default run) the same
    sub-workloads as the B200 arm with a few steps each."""
    if rank != 0:
        return None
    line = reference_record(args.workload, wl, args.steps, args.warmup, 150.0)
    line["n_gpus"] = args.gpus
    if sub_records_enabled(args):
        line["sub"] = {}
        for key, name, _, _, _ in SUB_RECORDS:
            rec = reference_record(name, WORKLOADS[name], min(args.steps, 4), 1, 20.0)
            line["sub"][key] = rec
    return line


# ----------------------------------------------------------------------------- B200 arm
# Sub-records the default run adds to its line: (key, workload, minimum timed
# steps, end-to-end steps, single-core CPU baseline budget in seconds).
SUB_RECORDS = [
    ("attention_cfg2", "attention-cfg2", 200, 5, 10.0),
    ("attention_cfg4", "attention-cfg4", 20, 3, 10.0),
    ("softmax_cfg5", "softmax", 100, 5, None),
]
SOFTMAX_METRIC = "warp softmax GB/s (whole box)"
MUFU_EX2_PER_CLK_PER_SM = 16  # nominal sm_100 exp2 (MUFU) throughput


def sub_records_enabled(args) -> bool:
    return args.workload == "attention" and not args.shape and not args.no_sub


def sm_count(local: int) -> int:
    import torch

    return torch.cuda.get_device_properties(local).multi_processor_count


def mufu_roofline(exps_per_launch: float, launch_ms: float, clocks: dict | None, n_sm: int) -> dict:
    """Exp-unit roofline: algorithmic exps (one per unmasked score) per launch
    over the launch time, against 16 ex2 per clock per SM at the median SM
    clock sampled during the timed region."""
    mhz = (clocks or {}).get("sm_mhz") or 1965.0
    peak = MUFU_EX2_PER_CLK_PER_SM * n_sm * mhz * 1e6 / 1e9
    achieved = exps_per_launch / (launch_ms / 1e3) / 1e9
    return {"achieved": achieved, "peak": peak, "unit": "Gexp/s", "frac": achieved / peak,
            "peak_source": f"nominal {MUFU_EX2_PER_CLK_PER_SM} ex2/clk/SM x {n_sm} SMs at {mhz:.0f} MHz (sampled)"}


def run_attention(args, name, wl, rank, world, local, sampler, steps, e2e_steps, cpu_budget):
    import torch

    import pmkl_b200
    from pmkl_function import fused_self_attention

    B, H, S, D, dtype_name, std, causal, desc = wl
    dt = getattr(torch, dtype_name)
    n_slices = B * H
    lo, hi = shard(n_slices, world, rank)
    ns = hi - lo
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(args.seed + rank)
    q, k, v = [(torch.randn(ns, 1, S, D, generator=g, device=dev) * std).to(dt) for _ in range(3)]
    o = torch.empty_like(q)
    m = torch.empty(ns, 1, S, dtype=dt, device=dev)
    l = torch.empty_like(m)
    stream = torch.cuda.current_stream()

    def step():
        pmkl_b200.attention_fwd(q, k, v, o, m, l, causal, kernel=args.kernel, stream=stream)

    kernel_name = pmkl_b200.attention_kernel_name(q, k, v, o, args.kernel)

    total_ms, per_ms, clocks = timed_loop(step, steps, args.warmup, world, sampler)
    flops_rank = ns * attn_flops_per_slice(S, D, causal)
    flops_all = n_slices * attn_flops_per_slice(S, D, causal)
    t_max = max_over_ranks(total_ms, world)
    value = flops_all * steps / (t_max / 1e3) / 1e12
    launch_avg = statistics.mean(per_ms)
    achieved = flops_rank / (launch_avg / 1e3) / 1e12
    achieved_min = max_over_ranks(-achieved, world)  # slowest rank
    peaks = measured_peaks()
    pairs = S * (S + 1) / 2 if causal else S * S

    # End to end through the public API: every step copies q, k, v in from
    # pinned host memory, calls fused_self_attention and copies O, m, l back.
    # The step's slices go in chunks on three streams, so that the H2D copy of
    # chunk c+1, the attention of chunk c and the D2H copy of chunk c-1 overlap
    # (PCIe carries both directions at once).
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    oh = torch.empty(q.shape, dtype=dt).pin_memory()
    mh = torch.empty(m.shape, dtype=dt).pin_memory()
    lh = torch.empty(m.shape, dtype=dt).pin_memory()
    qd, kd, vd = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    n_chunks = max(1, min(args.e2e_chunks, ns))
    bounds = [shard(ns, n_chunks, c) for c in range(n_chunks)]
    s_in, s_run, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(n_chunks)]
    ev_run = [torch.cuda.Event() for _ in range(n_chunks)]

    def e2e_step():
        main = torch.cuda.current_stream()
        s_in.wait_stream(main)
        for c, (a, b) in enumerate(bounds):
            with torch.cuda.stream(s_in):
                qd[a:b].copy_(qh[a:b], non_blocking=True)
                kd[a:b].copy_(kh[a:b], non_blocking=True)
                vd[a:b].copy_(vh[a:b], non_blocking=True)
                ev_in[c].record(s_in)
            with torch.cuda.stream(s_run):
                s_run.wait_event(ev_in[c])
                out, om, ol = fused_self_attention(qd[a:b], kd[a:b], vd[a:b], causal)
                ev_run[c].record(s_run)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_run[c])
                for src in (out, om, ol):
                    src.record_stream(s_out)
                oh[a:b].copy_(out, non_blocking=True)
                mh[a:b].copy_(om, non_blocking=True)
                lh[a:b].copy_(ol, non_blocking=True)
        main.wait_stream(s_out)

    e2e_steps = max(1, min(e2e_steps, steps))
    e2e_ms, _, _ = timed_loop(e2e_step, e2e_steps, min(args.warmup, 3), world)
    e2e_t = max_over_ranks(e2e_ms, world)
    e2e_value = flops_all * e2e_steps / (e2e_t / 1e3) / 1e12
    h2d = 3 * q.numel() * q.element_size()
    d2h = o.numel() * o.element_size() + 2 * m.numel() * m.element_size()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and cpu_budget:
        try:
            cpu = cpu_baseline_attention(S, D, dtype_name, std, causal, cpu_budget)
        except FileNotFoundError as e:
            cpu = {"value": None, "unit": "TFLOP/s", "cores": 1, "kind": "reference",
                   "sample": f"unavailable: {e}"}

    traffic = profile_traffic(name)
    tensor = {"bound": "tensor", "achieved": -achieved_min, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
              "frac": -achieved_min / peaks["bf16_tflops"],
              "peak_source": f"{peaks['source']} bf16 burst (sustained {peaks['bf16_tflops_sustained']})",
              "traffic": (traffic * ns if traffic is not None else None),
              "algorithmic_bytes": 4 * q.numel() * q.element_size() + 2 * m.numel() * m.element_size(),
              "kernel": kernel_name, "launch_ms_avg": launch_avg}
    mufu = mufu_roofline(ns * pairs, launch_avg, clocks, sm_count(local))
    if D == 64:
        # Head size 64: a key tile of a 128-row query tile costs 16384 exps
        # (1024 MUFU cycles) against 4.2 MFLOP of contractions (512 tensor
        # cycles), so the exp unit is the binding roofline.
        roofline = dict(mufu, bound="mufu", kernel=kernel_name, launch_ms_avg=launch_avg,
                        traffic=tensor["traffic"], algorithmic_bytes=tensor["algorithmic_bytes"],
                        tensor={k: tensor[k] for k in ("achieved", "peak", "unit", "frac", "peak_source")})
    else:
        roofline = dict(tensor, mufu=mufu)
    line = {
        "metric": ATTN_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": t_max / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": dtype_name, "data": f"synthetic, seeded N(0, {std}^2) generated on device",
        "config": {"workload": desc, "B": B, "H": H, "S": S, "D": D, "causal": causal,
                   "parallelism": f"(batch, head) shards over {world} GPU(s), no inter-GPU traffic",
                   "slices_per_gpu": ns, "flop_convention": "4*D*S(S+1)/2 per (b,h) slice",
                   "l2": ("inputs (3 x %.0f MiB per GPU) exceed the 126 MB L2; no flush"
                          % (q.numel() * q.element_size() / 2**20)) if 3 * q.numel() * q.element_size() > 126e6
                   else "inputs fit in L2: every timed launch reads them from L2 after the first"},
        "per_gpu_tflops": value / world,
        "frac_of_peak": value / world / peaks["bf16_tflops"],
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "pmkl_function.fused_self_attention", "steps": e2e_steps,
                "chunks": n_chunks, "overlap": "H2D / attention / D2H of consecutive chunks on three streams"},
        "gpu_launches": steps,
        "roofline": roofline,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    return line


def run_attention_bwd(args, name, wl, rank, world, local, sampler, steps, e2e_steps, cpu_budget):
    """One step = pmkl_causal_attention_bwd over the rank's (b, h) shard: the
    persistent forward in its backward instantiation (per-row b and delta from
    its epilogue), the dQ kernel and the dK/dV kernel.  m, l come from one
    forward before the timed region, in the input dtype as the reference
    returns them."""
    import torch

    import pmkl_b200
    import pmkl_pytorch_ext

    B, H, S, D, dtype_name, std, causal, desc = wl
    dt = getattr(torch, dtype_name)
    simt = dtype_name == "float32" or D not in (64, 128)  # the CUDA-core backward
    n_slices = B * H
    lo, hi = shard(n_slices, world, rank)
    ns = hi - lo
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(args.seed + rank)
    q, k, v, do = [(torch.randn(ns, 1, S, D, generator=g, device=dev) * std).to(dt) for _ in range(4)]
    o = torch.empty_like(q)
    m = torch.empty(ns, 1, S, dtype=dt, device=dev)
    l = torch.empty_like(m)
    pmkl_b200.attention_fwd(q, k, v, o, m, l, causal)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ws = torch.empty(pmkl_b200.attention_bwd_workspace_size(ns, 1, S, D, dt, args.kernel), dtype=torch.uint8,
                     device=dev)
    stream = torch.cuda.current_stream()

    def step():
        pmkl_b200.attention_bwd(do, q, k, v, m, l, dq, dk, dv, causal, kernel=args.kernel, workspace=ws,
                                stream=stream)

    total_ms, per_ms, clocks = timed_loop(step, steps, args.warmup, world, sampler)
    flops_rank = ns * attn_bwd_flops_per_slice(S, D, causal)
    flops_all = n_slices * attn_bwd_flops_per_slice(S, D, causal)
    t_max = max_over_ranks(total_ms, world)
    value = flops_all * steps / (t_max / 1e3) / 1e12
    launch_avg = statistics.mean(per_ms)
    achieved = -max_over_ranks(-(flops_rank / (launch_avg / 1e3) / 1e12), world)
    peaks = measured_peaks()

    # End to end through the reference-facing binding: H2D of dout, q, k, v, m,
    # l from pinned memory, fused_self_attention_bw, D2H of dq, dk, dv.
    hosts = [t.cpu().pin_memory() for t in (do, q, k, v, m, l)]
    devs = [torch.empty_like(t) for t in (do, q, k, v, m, l)]
    outs_h = [torch.empty(q.shape, dtype=dt).pin_memory() for _ in range(3)]
    n_chunks = max(1, min(args.e2e_chunks, ns))
    bounds = [shard(ns, n_chunks, c) for c in range(n_chunks)]
    s_in, s_run, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(n_chunks)]
    ev_run = [torch.cuda.Event() for _ in range(n_chunks)]

    def e2e_step():
        # Slice chunks on three streams: H2D of chunk c+1, backward of chunk c
        # and D2H of chunk c-1 overlap.
        main = torch.cuda.current_stream()
        s_in.wait_stream(main)
        for c, (a, b) in enumerate(bounds):
            with torch.cuda.stream(s_in):
                for d_, h_ in zip(devs, hosts):
                    d_[a:b].copy_(h_[a:b], non_blocking=True)
                ev_in[c].record(s_in)
            with torch.cuda.stream(s_run):
                s_run.wait_event(ev_in[c])
                grads = pmkl_pytorch_ext.fused_self_attention_bw(*(d_[a:b] for d_ in devs), causal)
                ev_run[c].record(s_run)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_run[c])
                for h_, g_ in zip(outs_h, grads):
                    g_.record_stream(s_out)
                    h_[a:b].copy_(g_, non_blocking=True)
        main.wait_stream(s_out)

    e2e_steps = max(1, min(e2e_steps, steps))
    e2e_ms, _, _ = timed_loop(e2e_step, e2e_steps, min(args.warmup, 3), world)
    e2e_value = flops_all * e2e_steps / (max_over_ranks(e2e_ms, world) / 1e3) / 1e12
    h2d = sum(t.numel() * t.element_size() for t in hosts)
    d2h = sum(t.numel() * t.element_size() for t in outs_h)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and cpu_budget:
        try:
            r = pick_bwd_rows(D, dtype_name, causal, cpu_budget)
            tt = _ref_attention_bwd_worker((r, D, dtype_name, std, causal, 7))
            cpu = {"value": attn_bwd_flops_per_slice(r, D, causal) / tt / 1e12, "unit": "TFLOP/s", "cores": 1,
                   "kind": "reference",
                   "sample": f"reference fused_self_attention_bw (CPU, {dtype_name}, O(S^3 D) as written) on one "
                             f"{r}-row causal (b,h) problem, D={D}, {tt:.1f} s on 1 core"}
        except FileNotFoundError as e:
            cpu = {"value": None, "unit": "TFLOP/s", "cores": 1, "kind": "reference", "sample": f"unavailable: {e}"}

    return {
        "metric": BWD_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": t_max / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": dtype_name, "data": f"synthetic, seeded N(0, {std}^2) generated on device",
        "config": {"workload": desc, "B": B, "H": H, "S": S, "D": D, "causal": causal,
                   "parallelism": f"(batch, head) shards over {world} GPU(s), no inter-GPU traffic",
                   "slices_per_gpu": ns, "flop_convention": "10*D*S(S+1)/2 per (b,h) slice (5 contractions)",
                   "l2": "inputs (4 x %.0f MiB per GPU) exceed the 126 MB L2; no flush" % (q.numel() * q.element_size() / 2**20)},
        "per_gpu_tflops": value / world,
        "frac_of_peak": value / world / peaks["bf16_tflops"],
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "pmkl_pytorch_ext.fused_self_attention_bw", "steps": e2e_steps,
                "chunks": n_chunks, "overlap": "H2D / backward / D2H of consecutive chunks on three streams"},
        "gpu_launches": (2 if simt else 4 if args.kernel == 3 else 3) * steps,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops"],
                     "peak_source": f"{peaks['source']} bf16 burst (sustained {peaks['bf16_tflops_sustained']})",
                     "traffic": None,
                     "kernel": ("one backward call: attn_bwd_simt_q_kernel + attn_bwd_simt_kv_kernel (CUDA cores)"
                                if simt else "one backward call: attn_fwd_pp_kernel (delta epilogue) + "
                                "attn_bwd_dq_kernel + attn_bwd_dkv_kernel"),
                     "note": ("fp32 on CUDA cores: the bf16 tensor peak is context, not this path's bound"
                              if simt else None),
                     "launch_ms_avg": launch_avg},
        "clocks": clocks,
        "cpu_baseline": cpu,
    }


def softmax_kernel_name(esz: int, el: int) -> str:
    """The kernel pmkl_warp_softmax_fwd picks for contiguous, aligned rows of
    `el` elements with input and output of one dtype of `esz` bytes."""
    if esz == 4 and el % 4 == 0:
        return "softmax_vec_kernel"
    if el % 8 == 0:
        return "softmax_vec8_kernel"
    return "softmax_gen_kernel"


def run_softmax(args, name, wl, rank, world, local, sampler, steps, e2e_steps, cpu_budget):
    import torch

    import pmkl_b200

    rows_all, el = wl[0], wl[1]
    dt = getattr(torch, wl[4])
    esz = torch.tensor([], dtype=dt).element_size()
    lo, hi = shard(rows_all, world, rank)
    rows = hi - lo
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(args.seed + rank)
    x = (torch.randn(rows, el, generator=g, device=dev) * wl[5]).to(dt)
    y = torch.empty_like(x)
    stream = torch.cuda.current_stream()

    def step():
        pmkl_b200.warp_softmax_fwd(y, x, el, el, rows, stream=stream)

    total_ms, per_ms, clocks = timed_loop(step, steps, args.warmup, world, sampler)
    bytes_rank = 2.0 * rows * el * esz
    bytes_all = 2.0 * rows_all * el * esz
    t_max = max_over_ranks(total_ms, world)
    value = bytes_all * steps / (t_max / 1e3) / 1e9
    launch_avg = statistics.mean(per_ms)
    achieved = -max_over_ranks(-(bytes_rank / (launch_avg / 1e3) / 1e9), world)
    peaks = measured_peaks()

    xh = x.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    xd, yd = torch.empty_like(x), torch.empty_like(y)
    n_chunks = max(1, min(args.e2e_chunks, rows))
    bounds = [shard(rows, n_chunks, c) for c in range(n_chunks)]
    s_in, s_run, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(n_chunks)]
    ev_run = [torch.cuda.Event() for _ in range(n_chunks)]

    def e2e_step():
        # Row chunks on three streams: H2D of chunk c+1, softmax of chunk c and
        # D2H of chunk c-1 overlap.
        main = torch.cuda.current_stream()
        s_in.wait_stream(main)
        for c, (a, b) in enumerate(bounds):
            with torch.cuda.stream(s_in):
                xd[a:b].copy_(xh[a:b], non_blocking=True)
                ev_in[c].record(s_in)
            s_run.wait_event(ev_in[c])
            pmkl_b200.warp_softmax_fwd(yd[a:b], xd[a:b], el, el, b - a, stream=s_run)
            ev_run[c].record(s_run)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_run[c])
                yh[a:b].copy_(yd[a:b], non_blocking=True)
        main.wait_stream(s_out)

    e2e_steps = max(1, min(e2e_steps, steps))
    e2e_ms, _, _ = timed_loop(e2e_step, e2e_steps, min(args.warmup, 3), world)
    e2e_value = bytes_all * e2e_steps / (max_over_ranks(e2e_ms, world) / 1e3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and dt == torch.float32:
        try:
            # the whole problem (all rows_all rows), repeated for ~5 s of CPU work
            n = rows_all
            t1 = _ref_softmax_worker((n, el, 9, 1))
            reps = max(1, min(100, int(5.0 / max(t1, 1e-3))))
            t = _ref_softmax_worker((n, el, 9, reps))
            cpu = {"value": reps * n * el * 8.0 / t / 1e9, "unit": "GB/s", "cores": 1, "kind": "reference",
                   "sample": f"reference host_softmax_forward (CPU fp32) on all {n} rows x {el}, {reps} "
                             f"repetitions, {t:.1f} s on 1 core"}
        except FileNotFoundError as e:
            cpu = {"value": None, "unit": "GB/s", "cores": 1, "kind": "reference", "sample": f"unavailable: {e}"}
    traffic = profile_traffic(name)
    return {
        "metric": SOFTMAX_METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": t_max / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32" if esz == 4 else wl[4],
        "data": "synthetic, seeded N(0, 4) generated on device",
        "config": {"workload": wl[7], "rows": rows_all, "elements": el, "parallelism": f"row shards over {world} GPU(s)",
                   "l2": "%.0f MiB in + out per GPU exceed the 126 MB L2; no flush" % (2 * rows * el * esz / 2**20)},
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": rows * el * esz,
                "d2h_bytes_per_step": rows * el * esz, "api": "pmkl_warp_softmax_fwd (C ABI)", "steps": e2e_steps,
                "chunks": n_chunks, "overlap": "H2D / softmax / D2H of consecutive row chunks on three streams"},
        "gpu_launches": steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_source": f"{peaks['source']} copy bandwidth",
                     "traffic": (traffic * rows if traffic is not None else None),
                     "algorithmic_bytes": bytes_rank,
                     "kernel": softmax_kernel_name(esz, el), "launch_ms_avg": launch_avg},
        "clocks": clocks,
        "cpu_baseline": cpu,
    }


RUNNERS = {"softmax": run_softmax, "softmax-bf16": run_softmax, "softmax-gen": run_softmax,
           "attention-bwd": run_attention_bwd, "attention-bwd-fp32": run_attention_bwd}


def run_workload(args, name, wl, rank, world, local, sampler, steps, e2e_steps, cpu_budget):
    fn = RUNNERS.get(name, run_attention)
    return fn(args, name, wl, rank, world, local, sampler, steps, e2e_steps, cpu_budget)


def main():
    args = parse_args()
    wl = WORKLOADS[args.workload]
    if args.shape:
        dims = [int(x) for x in args.shape.split(",")]
        if args.workload.startswith("softmax"):
            wl = (dims[0], dims[1]) + wl[2:7] + (f"warp softmax {wl[4]} {dims[0]} x {dims[1]} (profiling size)",)
        else:
            wl = tuple(dims[:4]) + wl[4:7] + (f"causal self-attention {wl[4]} B{dims[0]} H{dims[1]} S{dims[2]} "
                                              f"D{dims[3]} (profiling size)",)
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        line = run_reference_arm(args, wl, rank, int(os.environ.get("WORLD_SIZE", "1")))
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    rank, world, local = dist_init(args.gpus)
    sampler = ClockSampler(local, not args.no_clocks)
    try:
        line = run_workload(args, args.workload, wl, rank, world, local, sampler, args.steps, args.e2e_steps,
                            20.0 if args.workload != "attention-bwd" else 15.0)
        if sub_records_enabled(args):
            # The other BASELINE workloads, measured the same way in the same
            # run (device-timed value, roofline, end-to-end leg, CPU baseline,
            # clocks), with their own step counts.
            line["sub"] = {}
            for key, name, min_steps, e2e_steps, budget in SUB_RECORDS:
                rec = run_workload(args, name, WORKLOADS[name], rank, world, local, sampler,
                                   max(args.steps, min_steps), e2e_steps, budget)
                line["sub"][key] = rec
                line["gpu_launches_all"] = line.get("gpu_launches_all", line["gpu_launches"]) + rec["gpu_launches"]
        if world > 1:
            # every rank's clocks; a throttled rank throttles the whole job
            line["clocks_per_rank"] = gather_clocks(line.get("clocks"), world)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        sampler.stop()
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


def gather_clocks(clocks, world):
    import torch.distributed as dist

    out = [None] * world
    dist.all_gather_object(out, clocks)
    return out


if __name__ == "__main__":
    main()
