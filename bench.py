#!/usr/bin/env python
"""Headline benchmark: fused attention forward TFLOP/s on B200 (sm_100a), 1..8 GPUs.

    python bench.py                                   # 1 GPU, config 4, defaults
    python bench.py --gpus 1 --steps 200 --warmup 10
    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        --master-port 29511 bench.py --gpus 8
    python bench.py --impl reference                  # the reference's CPU implementation, same metric

One step = one attention forward over one batch of the workload (BASELINE config 4 by default:
B=1, H=32, N=16384, d=128, bf16, Q,V ~ N(0,0.5), K with 1% of rows per head scaled x8) on every rank.
Work is partitioned over heads: each rank owns its own B*H heads (weak scaling: rank r processes global
heads [r*BH, (r+1)*BH) of a batch of B*world), with no collective on the data path; the only collectives
are the barrier and the max-over-ranks of the measured times.

Printed on rank 0, one JSON line:
  value     aggregate TFLOP/s = 4*B*H*N^2*d FLOPs of all ranks / max-over-ranks device time of K steps,
            inputs resident in HBM (C-ABI call per step, CUDA events on the launching stream).
  e2e       the same metric through the public API with host buffers: every step calls
            cuda_attn.fused_tc_host on pinned host Q, K, V, which copies them in, runs the kernel and copies O
            back (head chunks pipelined over three streams), all inside the timed region.
  roofline  the tensor-core attention kernel alone (CUDA-event brackets around each of its launches in
            the timed region): algorithmic FLOPs per launch / average launch time, against the measured
            sustained bf16 peak; traffic = DRAM bytes per launch from the committed ncu summary of
            config 4 (null for the other workloads, which that summary does not cover).
  cpu_baseline  the oracle port of the reference's CPU path (fp32 SDPA math on CPU) on a bounded sample.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "phantom-a100_b200"), ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "attention fwd TFLOP/s per GPU & % of B200 tensor peak at 1/2/4/8 GPUs"
PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "attn_fwd_tc_config4_traffic.txt")
TRAFFIC_WORKLOAD = "config4"  # the workload that summary was captured on; other workloads report null
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="config4", help="config2 | config3 | config4 | config5_n<N>_d<d>")
    ap.add_argument("--e2e-steps", type=int, default=None, help="steps of the end-to-end loop (default: steps/4)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="target length of the CPU baseline sample")
    return ap.parse_args()


def get_config(name):
    from cuda_attn.workloads import CONFIGS, sweep_config
    if name in CONFIGS:
        return CONFIGS[name]
    m = re.fullmatch(r"config5_n(\d+)_d(\d+)", name)
    if m:
        return sweep_config(int(m.group(1)), int(m.group(2)))
    raise SystemExit(f"unknown config {name}")


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def load_peaks():
    try:
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return FALLBACK_PEAKS, "fallback"


def load_traffic():
    """DRAM bytes per launch of the tensor-core kernel from the committed ncu summary, or None."""
    try:
        with open(TRAFFIC_FILE) as f:
            for line in f:
                m = re.match(r"\s*dram_bytes_per_launch:\s*([0-9.eE+]+)", line)
                if m:
                    return float(m.group(1))
    except OSError:
        pass
    return None


# ------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples of one GPU while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_uuid: str | None):
        self.uuid = gpu_uuid
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"]
        if self.uuid:
            cmd[1:1] = ["-i", self.uuid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        pw = [num(r[3]) for r in rows if num(r[3]) is not None]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows), "power_w_max": max(pw) if pw else None}


# ------------------------------------------------------------------------------------------ CPU side
def cpu_sample_rows(cfg, seconds_target):
    """Rows of head 0 that the CPU baseline processes, sized for about `seconds_target` of work at the
    ~65 GFLOP/s the fp32 SDPA math path reaches on 8 host cores."""
    flops_per_row = 4.0 * cfg.N * cfg.d
    rows = int(seconds_target * 65e9 / flops_per_row)
    return max(64, min(cfg.N, rows - rows % 64))


def time_cpu_reference(cfg, rows, threads):
    """The reference's CPU ground truth (fp32 SDPA math on CPU, oracle.reference_sdpa) on the first
    `rows` query rows of head 0 against all N keys (non-causal rows are independent, so this is an exact
    sample of the workload). Returns (seconds, flops)."""
    import torch
    from cuda_attn.workloads import make_inputs
    from oracle import reference_sdpa
    torch.set_num_threads(threads)
    q, k, v = make_inputs(cfg, heads=(0, 1), device="cpu")
    q, k, v = (x.float() for x in (q, k, v))
    chunk = 2048
    t0 = time.perf_counter()
    for r0 in range(0, rows, chunk):
        reference_sdpa(q[:, :, r0:min(rows, r0 + chunk)], k, v, False)
    dt = time.perf_counter() - t0
    return dt, 4.0 * rows * cfg.N * cfg.d


def run_reference_arm(args, rank, world):
    """--impl reference: the reference's CPU implementation of the path, timed on this host."""
    if rank != 0:
        return 0
    import torch
    cfg = get_config(args.config)
    if cfg.causal:
        raise SystemExit("reference arm samples query rows; causal configs are not supported here")
    threads = os.cpu_count() or 1
    rows = min(cfg.N, 1024)  # one bounded sample per step (~0.1-0.5 s on 8 cores)
    for _ in range(max(args.warmup, 0)):
        time_cpu_reference(cfg, rows, threads)
    times = []
    flops = 0.0
    for _ in range(args.steps):
        dt, flops = time_cpu_reference(cfg, rows, threads)
        times.append(dt)
    total = sum(times)
    value = flops * args.steps / total / 1e12
    sample = f"head 0, query rows [0,{rows}) x all {cfg.N} keys of {cfg.name} per step (fp32 SDPA math on CPU)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": cfg.describe(),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "torch_threads": torch.get_num_threads(),
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------ GPU side
def main():
    args = parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    import cuda_attn
    from cuda_attn.capi import CAPI
    from cuda_attn.workloads import Config, make_inputs

    base = get_config(args.config)
    # weak scaling: each rank owns a full config-sized batch of heads; global batch = B * world
    cfg = Config(base.name, base.B * world, base.H, base.N, base.d, base.dtype, base.causal, base.std,
                 base.k_outlier_frac, base.k_outlier_scale, base.seed, base.notes)
    my_heads = (rank * base.BH, (rank + 1) * base.BH)
    q, k, v = make_inputs(cfg, heads=my_heads, device=dev)
    o = torch.empty_like(q)
    capi = CAPI()
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # correctness gate (as the reference benchmark does, benchmark.py:165-171): sampled rows of two heads
    # against the package's fp32 SDPA ground truth; a wrong result is reported, never timed as valid
    capi.fused_tc(q, k, v, o, causal=cfg.causal)
    torch.cuda.synchronize()
    gate = {}
    rows = torch.arange(0, cfg.N, max(1, cfg.N // 128), device=dev)
    for h in (0, base.BH - 1):
        ref = cuda_attn.reference(q[:, h:h + 1, rows], k[:, h:h + 1], v[:, h:h + 1], False) if not cfg.causal \
            else cuda_attn.reference(q[:, h:h + 1], k[:, h:h + 1], v[:, h:h + 1], True)[:, :, rows]
        out = o[:, h:h + 1, rows].float()
        err = (out - ref).abs().max().item()
        rel = ((out - ref).norm() / ref.norm()).item()
        gate = {"max_abs": max(gate.get("max_abs", 0.0), err), "rel_l2": max(gate.get("rel_l2", 0.0), rel)}
    status = capi.device_status()
    gate_ok = status == 0 and gate["rel_l2"] < 5e-3 and gate["max_abs"] < 2e-2

    def step():
        capi.fused_tc(q, k, v, o, causal=cfg.causal, stream=stream)

    # ---- device-resident loop: value + roofline
    for _ in range(args.warmup):
        step()
    barrier()
    torch.cuda.synchronize()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    sampler.start()
    time.sleep(0.2)
    capi.launch_count(reset=True)
    capi.kernel_timing(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    barrier()
    ms_total = e0.elapsed_time(e1)
    kernel_ms, kernel_launches = capi.kernel_timing_read()
    capi.kernel_timing(False)
    launches = capi.launch_count()
    status |= capi.device_status()
    ms_total_max = max_over_ranks(ms_total)
    ms_per_step = ms_total_max / args.steps
    total_flops = cfg.flops()  # all ranks' heads (B*world*H)
    value = total_flops / (ms_per_step * 1e-3) / 1e12

    # ---- end-to-end loop through the public API with host buffers
    e2e_steps = args.e2e_steps or max(3, args.steps // 4)
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    ho = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)

    def e2e_step():
        # public API for host-resident tensors: head chunks stream through the GPU, host->device copy of
        # chunk i+1, attention of chunk i and device->host copy of chunk i-1 overlapping
        cuda_attn.fused_tc_host(hq, hk, hv, cfg.causal, out=ho, synchronize=False)

    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    f1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1)) / e2e_steps
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv))
    d2h = ho.numel() * ho.element_size()
    e2e_ok = torch.equal(ho.to(dev), o)

    peaks, peak_kind = load_peaks()
    peak_sus = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    peak_burst = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    flops_per_launch = base.flops()
    avg_kernel_ms = kernel_ms / kernel_launches if kernel_launches else None
    achieved = flops_per_launch / (avg_kernel_ms * 1e-3) / 1e12 if avg_kernel_ms else None
    kernel_ms_max = max_over_ranks(avg_kernel_ms or 0.0)

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0

    cpu = None
    if not args.no_cpu_baseline and world == 1 and not cfg.causal:
        threads = os.cpu_count() or 1
        rows_cpu = cpu_sample_rows(base, args.cpu_seconds)
        dt, fl = time_cpu_reference(base, rows_cpu, threads)
        cpu = {"value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"head 0, query rows [0,{rows_cpu}) x all {base.N} keys of {base.name}, fp32 SDPA "
                         f"math on CPU (oracle.reference_sdpa), {dt:.1f} s"}

    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": {"torch.bfloat16": "bf16", "torch.float16": "f16",
                                        "torch.float32": "f32"}[str(base.dtype)],
        "data": "synthetic: " + (base.notes or f"N(0,{base.std})") + ", seeded per global head",
        "config": dict(cfg.describe(), global_batch=cfg.B, heads_per_gpu=base.BH,
                       parallelism=f"heads sharded over {world} GPU(s), no collective",
                       l2="no flush: Q/K/V per GPU %.0f MiB > 126 MB L2" % (3 * q.numel() * q.element_size() / 2**20)),
        "per_gpu_tflops": value / world,
        "pct_of_peak": {"sustained": 100.0 * value / world / peak_sus, "burst": 100.0 * value / world / peak_burst,
                        "peaks": peak_kind},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_sus, "unit": "TFLOP/s",
                     "frac": (achieved / peak_sus) if achieved else None, "traffic": load_traffic() if base.name == TRAFFIC_WORKLOAD else None,
                     "kernel": "phantom::tc::attn_fwd_tc", "kernel_ms_avg": avg_kernel_ms,
                     "kernel_ms_avg_max_rank": kernel_ms_max, "flops_per_launch": flops_per_launch,
                     "peak_kind": f"{peak_kind} bf16 sustained (MEASURED_PEAKS.json bf16_tflops_sustained)",
                     "frac_of_burst": (achieved / peak_burst) if achieved else None},
        "e2e": {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "steps": e2e_steps,
                "path": "pinned host -> cuda_attn.fused_tc_host (public API; copies overlapped with the kernel over head chunks: 8 full, the last cut in halves) -> pinned host", "matches_value_run": e2e_ok},
        "gpu_launches": launches,
        "kernel_launches_timed": kernel_launches,
        "clocks": clocks,
        "correctness": dict(gate, status=status, ok=gate_ok),
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0 if gate_ok else 1


if __name__ == "__main__":
    sys.exit(main())
