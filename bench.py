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
            bf16 peak (MEASURED_PEAKS.json);
  cpu_baseline  the reference's own CPU implementation (its torch extension
            compiled from its sources into oracle/_ref) on a bounded sample.

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
    "softmax": (65536, 1024, None, None, "float32", 2.0, None, "BASELINE config 5: warp softmax fp32 65536 x 1024"),
    "attention-bwd": (16, 32, 4096, 128, "bfloat16", 1.0, True,
                      "backward of BASELINE config 3: fused_self_attention_bw bf16 B16 H32 S4096 D128 causal"),
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
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, n_gpus: int, enabled: bool):
        self.proc = None
        self.path = None
        if not enabled:
            return
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        idx = vis if vis else ",".join(str(i) for i in range(n_gpus))
        out_dir = REPO / "gpurun_out"
        out_dir.mkdir(exist_ok=True)
        self.path = out_dir / f"clocks_{os.getpid()}.csv"
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", idx, "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


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
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
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


def timed_loop(step, steps: int, warmup: int, world: int):
    """W untimed steps, then K steps between barrier + synchronize; returns
    (total ms of the K steps, list of per-step ms) on this rank."""
    import torch

    for _ in range(warmup):
        step()
    barrier(world)
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
    barrier(world)
    return start.elapsed_time(end), [a.elapsed_time(b) for a, b in ev]


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
    rows, el, seed = args
    import numpy as np

    from oracle import build_ref

    fn = build_ref.load_ref_softmax()
    x = (np.random.default_rng(seed).standard_normal(rows * el) * 2).astype(np.float32)
    y = np.empty_like(x)
    t0 = time.perf_counter()
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


def run_reference_arm(args, wl, rank, world):
    """--impl reference: the reference's own CPU implementation on all host
    cores (one process per core), each step a bounded sample."""
    import multiprocessing as mp

    if rank != 0:
        return None
    B, H, S, D, dtype_name, std, causal, desc = wl
    cores = host_cores()
    ctx = mp.get_context("spawn")
    total_steps = args.steps + args.warmup
    budget = max(0.5, min(20.0, 150.0 / max(1, total_steps)))
    if args.workload == "softmax":
        rows_total, el = B, H
        probe = _ref_softmax_worker((256, el, 0))
        rows = max(1, min(rows_total // cores if rows_total >= cores else rows_total, int(budget / (probe / 256))))
        work = [(rows, el, 100 + i) for i in range(cores)]
        unit_per_step = cores * rows * el * 8.0 / 1e9  # GB moved per step (read + write fp32)
        unit, metric = "GB/s", "warp softmax GB/s (whole box)"
        sample = f"reference host_softmax_forward (CPU fp32), {rows} rows x {el} per core per step"
    elif args.workload != "attention-bwd":
        r = pick_prefix_rows(S, D, dtype_name, causal, budget)
        work = [(r, D, dtype_name, std, causal, 100 + i) for i in range(cores)]
        unit_per_step = cores * attn_flops_per_slice(r, D, causal) / 1e12
        unit, metric = "TFLOP/s", ATTN_METRIC
        sample = (f"reference fused_self_attention_fw (CPU, {dtype_name}): per step each of {cores} worker "
                  f"processes runs a causal prefix of {r} of {S} rows of one (b,h) slice, D={D}")
    elif args.workload == "attention-bwd":
        r = pick_bwd_rows(D, dtype_name, causal, budget)
        work = [(r, D, dtype_name, std, causal, 100 + i) for i in range(cores)]
        unit_per_step = cores * attn_bwd_flops_per_slice(r, D, causal) / 1e12
        unit, metric = "TFLOP/s", BWD_METRIC
        sample = (f"reference fused_self_attention_bw (CPU, {dtype_name}, O(S^3 D)): per step each of {cores} "
                  f"worker processes runs the backward of one {r}-row causal (b,h) problem, D={D}")
    fn = {"softmax": _ref_softmax_worker, "attention-bwd": _ref_attention_bwd_worker}.get(args.workload,
                                                                                          _ref_attention_worker)
    times = []
    with ctx.Pool(cores) as pool:
        for i in range(total_steps):
            t0 = time.perf_counter()
            pool.map(fn, work, chunksize=1)
            dt = time.perf_counter() - t0
            if i >= args.warmup:
                times.append(dt)
    tot = sum(times)
    value = unit_per_step * len(times) / tot
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype_name,
        "data": "synthetic (seeded N(0, std^2))",
        "config": {"workload": desc, "sample": sample},
        "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


# ----------------------------------------------------------------------------- B200 arm
def run_attention(args, wl, rank, world, local):
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

    sampler = ClockSampler(world, (not args.no_clocks) and rank == 0)
    total_ms, per_ms = timed_loop(step, args.steps, args.warmup, world)
    clocks = sampler.stop()
    flops_rank = ns * attn_flops_per_slice(S, D, causal)
    flops_all = n_slices * attn_flops_per_slice(S, D, causal)
    t_max = max_over_ranks(total_ms, world)
    value = flops_all * args.steps / (t_max / 1e3) / 1e12
    launch_avg = statistics.mean(per_ms)
    achieved = flops_rank / (launch_avg / 1e3) / 1e12
    achieved_min = max_over_ranks(-achieved, world)  # slowest rank
    peaks = measured_peaks()

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

    e2e_steps = max(1, min(args.e2e_steps, args.steps))
    e2e_ms, _ = timed_loop(e2e_step, e2e_steps, min(args.warmup, 3), world)
    e2e_t = max_over_ranks(e2e_ms, world)
    e2e_value = flops_all * e2e_steps / (e2e_t / 1e3) / 1e12
    h2d = 3 * q.numel() * q.element_size()
    d2h = o.numel() * o.element_size() + 2 * m.numel() * m.element_size()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline_attention(S, D, dtype_name, std, causal)
        except FileNotFoundError as e:
            cpu = {"value": None, "unit": "TFLOP/s", "cores": 1, "kind": "reference",
                   "sample": f"unavailable: {e}"}

    traffic = profile_traffic(args.workload)
    line = {
        "metric": ATTN_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": dtype_name, "data": f"synthetic, seeded N(0, {std}^2) generated on device",
        "config": {"workload": desc, "B": B, "H": H, "S": S, "D": D, "causal": causal,
                   "parallelism": f"(batch, head) shards over {world} GPU(s), no inter-GPU traffic",
                   "slices_per_gpu": ns, "flop_convention": "4*D*S(S+1)/2 per (b,h) slice",
                   "l2": "inputs (3 x %.0f MiB per GPU) exceed the 126 MB L2; no flush" % (q.numel() * q.element_size() / 2**20)},
        "per_gpu_tflops": value / world,
        "frac_of_peak": value / world / peaks["bf16_tflops"],
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "pmkl_function.fused_self_attention", "steps": e2e_steps,
                "chunks": n_chunks, "overlap": "H2D / attention / D2H of consecutive chunks on three streams"},
        "gpu_launches": args.steps,
        "roofline": {"bound": "tensor", "achieved": -achieved_min, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": -achieved_min / peaks["bf16_tflops"],
                     "peak_source": f"{peaks['source']} bf16 burst (sustained {peaks['bf16_tflops_sustained']})",
                     "traffic": (traffic * ns if traffic is not None else None),
                     "algorithmic_bytes": 4 * q.numel() * q.element_size() + 2 * m.numel() * m.element_size(),
                     "kernel": kernel_name, "launch_ms_avg": launch_avg},
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    return line


def run_attention_bwd(args, wl, rank, world, local):
    """One step = pmkl_causal_attention_bwd over the rank's (b, h) shard: the
    forward with fp32 outputs (delta needs O, which the reference's backward
    does not take), the row-statistics kernel, the dQ kernel and the dK/dV
    kernel.  m, l come from one forward before the timed region, in the input
    dtype as the reference returns them."""
    import torch

    import pmkl_b200
    import pmkl_pytorch_ext

    B, H, S, D, dtype_name, std, causal, desc = wl
    dt = getattr(torch, dtype_name)
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
    ws = torch.empty(pmkl_b200.attention_bwd_workspace_size(ns, 1, S, D, dt), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def step():
        pmkl_b200.attention_bwd(do, q, k, v, m, l, dq, dk, dv, causal, kernel=args.kernel, workspace=ws,
                                stream=stream)

    sampler = ClockSampler(world, (not args.no_clocks) and rank == 0)
    total_ms, per_ms = timed_loop(step, args.steps, args.warmup, world)
    clocks = sampler.stop()
    flops_rank = ns * attn_bwd_flops_per_slice(S, D, causal)
    flops_all = n_slices * attn_bwd_flops_per_slice(S, D, causal)
    t_max = max_over_ranks(total_ms, world)
    value = flops_all * args.steps / (t_max / 1e3) / 1e12
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

    e2e_steps = max(1, min(args.e2e_steps, args.steps))
    e2e_ms, _ = timed_loop(e2e_step, e2e_steps, min(args.warmup, 3), world)
    e2e_value = flops_all * e2e_steps / (max_over_ranks(e2e_ms, world) / 1e3) / 1e12
    h2d = sum(t.numel() * t.element_size() for t in hosts)
    d2h = sum(t.numel() * t.element_size() for t in outs_h)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            r = pick_bwd_rows(D, dtype_name, causal, 15.0)
            tt = _ref_attention_bwd_worker((r, D, dtype_name, std, causal, 7))
            cpu = {"value": attn_bwd_flops_per_slice(r, D, causal) / tt / 1e12, "unit": "TFLOP/s", "cores": 1,
                   "kind": "reference",
                   "sample": f"reference fused_self_attention_bw (CPU, {dtype_name}, O(S^3 D) as written) on one "
                             f"{r}-row causal (b,h) problem, D={D}, {tt:.1f} s on 1 core"}
        except FileNotFoundError as e:
            cpu = {"value": None, "unit": "TFLOP/s", "cores": 1, "kind": "reference", "sample": f"unavailable: {e}"}

    return {
        "metric": BWD_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_max / args.steps, "higher_is_better": True, "scaling": "weak",
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
        "gpu_launches": 4 * args.steps,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops"],
                     "peak_source": f"{peaks['source']} bf16 burst (sustained {peaks['bf16_tflops_sustained']})",
                     "traffic": None,
                     "kernel": "one backward call: attn_fwd_pp_kernel (fp32 out) + bwd_rowstat_kernel + "
                               "attn_bwd_dq_kernel + attn_bwd_dkv_kernel",
                     "launch_ms_avg": launch_avg},
        "clocks": clocks,
        "cpu_baseline": cpu,
    }


def run_softmax(args, wl, rank, world, local):
    import torch

    import pmkl_b200

    rows_all, el = wl[0], wl[1]
    lo, hi = shard(rows_all, world, rank)
    rows = hi - lo
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(args.seed + rank)
    x = torch.randn(rows, el, generator=g, device=dev) * wl[5]
    y = torch.empty_like(x)
    stream = torch.cuda.current_stream()

    def step():
        pmkl_b200.warp_softmax_fwd(y, x, el, el, rows, stream=stream)

    sampler = ClockSampler(world, (not args.no_clocks) and rank == 0)
    total_ms, per_ms = timed_loop(step, args.steps, args.warmup, world)
    clocks = sampler.stop()
    bytes_rank = 2.0 * rows * el * 4
    bytes_all = 2.0 * rows_all * el * 4
    t_max = max_over_ranks(total_ms, world)
    value = bytes_all * args.steps / (t_max / 1e3) / 1e9
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

    e2e_steps = max(1, min(args.e2e_steps, args.steps))
    e2e_ms, _ = timed_loop(e2e_step, e2e_steps, min(args.warmup, 3), world)
    e2e_value = bytes_all * e2e_steps / (max_over_ranks(e2e_ms, world) / 1e3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            n = 8192
            t = _ref_softmax_worker((n, el, 9))
            cpu = {"value": n * el * 8.0 / t / 1e9, "unit": "GB/s", "cores": 1, "kind": "reference",
                   "sample": f"reference host_softmax_forward (CPU fp32) on {n} rows x {el}, {t:.2f} s on 1 core"}
        except FileNotFoundError as e:
            cpu = {"value": None, "unit": "GB/s", "cores": 1, "kind": "reference", "sample": f"unavailable: {e}"}
    traffic = profile_traffic(args.workload)
    return {
        "metric": "warp softmax GB/s (whole box)", "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_max / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic, seeded N(0, 4) generated on device",
        "config": {"workload": wl[7], "rows": rows_all, "elements": el, "parallelism": f"row shards over {world} GPU(s)",
                   "l2": "256 MiB in + 256 MiB out per GPU at N=1 exceed the 126 MB L2; no flush"},
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": rows * el * 4,
                "d2h_bytes_per_step": rows * el * 4, "api": "pmkl_warp_softmax_fwd (C ABI)", "steps": e2e_steps,
                "chunks": n_chunks, "overlap": "H2D / softmax / D2H of consecutive row chunks on three streams"},
        "gpu_launches": args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_source": f"{peaks['source']} copy bandwidth",
                     "traffic": (traffic * rows if traffic is not None else None),
                     "algorithmic_bytes": bytes_rank, "kernel": "softmax_vec_kernel", "launch_ms_avg": launch_avg},
        "clocks": clocks,
        "cpu_baseline": cpu,
    }


def main():
    args = parse_args()
    wl = WORKLOADS[args.workload]
    if args.shape:
        dims = [int(x) for x in args.shape.split(",")]
        if args.workload == "softmax":
            wl = (dims[0], dims[1]) + wl[2:7] + (f"warp softmax fp32 {dims[0]} x {dims[1]} (profiling size)",)
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
    try:
        if args.workload == "softmax":
            line = run_softmax(args, wl, rank, world, local)
        elif args.workload == "attention-bwd":
            line = run_attention_bwd(args, wl, rank, world, local)
        else:
            line = run_attention(args, wl, rank, world, local)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
