#!/usr/bin/env python
"""Headline benchmark: fused attention forward TFLOP/s on B200 (sm_100a), 1..8 GPUs.

    python bench.py                                   # 1 GPU, config 4, defaults
    python bench.py --gpus 1 --steps 200 --warmup 10
    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        --master-port 29511 bench.py --gpus 8
    python bench.py --impl reference                  # the reference's CPU implementation, same metric

One step = one attention forward over one batch of the workload (BASELINE config 4 by default:
B=1, H=32, N=16384, d=128, bf16, Q,V ~ N(0,0.5), K with 1% of rows per head scaled x8). Work is
partitioned over heads with no collective on the data path:
  --scaling strong (default)  the config's B*H heads are split over the ranks (config 4 on 8 GPUs: 4 heads
                              per GPU), as BASELINE configs 3 and 4 are quoted;
  --scaling weak              every rank owns a config-sized batch (rank r: global heads [r*BH, (r+1)*BH)).
The collectives are the barrier, the max-over-ranks of the measured times, and, outside the timed region,
the gather of sampled output rows of every head to rank 0, which checks them.

Correctness gate (before timing; reference bench/benchmark.py:165-171), the tests' criterion: sampled
query rows of every head against a float64 reference rounded to the output dtype, relative L2 of that
sampled output <= 1e-3 and max |error| <= 2e-3 beyond one output ulp (the largest single head's relative
L2 is reported beside it). A failure prints ok=false and exits 1.

Printed on rank 0, one JSON line:
  value     aggregate TFLOP/s = 4*B*H*N^2*d FLOPs of all ranks / max-over-ranks device time of K steps,
            inputs resident in HBM (C-ABI call per step, CUDA events on the launching stream).
  e2e       the same metric through the public API with host buffers: every step calls
            cuda_attn.fused_tc_host on pinned host Q, K, V, which copies them in, runs the kernel and copies O
            back (head chunks pipelined over three streams), all inside the timed region.
  roofline  the tensor-core attention kernel alone (CUDA-event brackets around each of its launches in
            the timed region): algorithmic FLOPs per launch / average launch time, against the measured
            bf16 peak for a region of that length (burst below 1 s, sustained above); traffic = DRAM bytes
            per launch from the committed ncu summary of config 4 (null for the other workloads).
  cpu_baseline  the oracle port of the reference's CPU path (fp32 SDPA math on CPU) on a bounded sample.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
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
SPEC_DENSE_BF16_TFLOPS = 2250.0  # B200 nominal dense bf16, for context beside the measured peak
SUSTAINED_AFTER_MS = 1000.0      # a timed region longer than this is compared with the sustained peak
TOL_RELL2, TOL_MAXABS = 1e-3, 2e-3  # north star: relative L2 and max abs (beyond one output ulp)
MANTISSA_BITS = {"torch.float16": 10, "torch.bfloat16": 7}
GATE_ROWS = 64                   # sampled query rows per head in the correctness gate
L2_BYTES = 126 << 20             # B200 L2; inputs below twice this are flushed out between timed steps


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="config4", help="config2 | config3 | config4 | config5_n<N>_d<d>")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="strong: the config's heads split over the ranks; weak: a config-sized batch per rank")
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
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "20"]
        if self.uuid:
            cmd[1:1] = ["-i", self.uuid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        # nvidia-smi takes a while to start (longer with several ranks starting it at once); a timed region of
        # a few milliseconds (8 GPUs sharing config 4) would otherwise end before its first sample
        t0 = time.time()
        while time.time() - t0 < 5.0 and self._lines() < 1 and self.proc.poll() is None:
            time.sleep(0.01)

    def _lines(self) -> int:
        try:
            with open(self.path) as f:
                return sum(1 for line in f if line.count(",") >= 8)
        except OSError:
            return 0

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        # at least one sample after the timed region (samples every 20 ms)
        n, t0 = self._lines(), time.time()
        while time.time() - t0 < 0.5 and self._lines() <= n and self.proc.poll() is None:
            time.sleep(0.005)
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
        # samples under load: power at least half of the highest seen (idle samples before the first launch
        # and after the last one would otherwise pull the median towards the idle clock)
        loaded = [num(r[1]) for r in rows if num(r[1]) is not None and num(r[3]) is not None and pw
                  and num(r[3]) >= 0.5 * max(pw)]
        return {"sm_mhz": statistics.median(loaded) if loaded else (statistics.median(sm) if sm else None),
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons), "samples": len(rows),
                "samples_under_load": len(loaded), "sm_mhz_all_samples": statistics.median(sm) if sm else None,
                "power_w_max": max(pw) if pw else None}


# ------------------------------------------------------------------------------------------ CPU side
def time_cpu_reference(cfg, heads, rows, threads):
    """The reference's CPU ground truth (fp32 SDPA math on CPU, oracle.reference_sdpa) on the first `rows`
    query rows of each of the global heads [0, heads) against all N keys (non-causal rows are independent,
    so this is an exact sample of the workload). Returns (seconds, flops)."""
    import torch
    from cuda_attn.workloads import make_inputs
    from oracle import reference_sdpa
    torch.set_num_threads(threads)
    dt, flops = 0.0, 0.0
    for h in range(heads):
        q, k, v = make_inputs(cfg, heads=(h, h + 1), device="cpu")
        q, k, v = (x.float() for x in (q, k, v))
        chunk = 2048
        t0 = time.perf_counter()
        for r0 in range(0, rows, chunk):
            reference_sdpa(q[:, :, r0:min(rows, r0 + chunk)], k, v, False)
        dt += time.perf_counter() - t0
        flops += 4.0 * rows * cfg.N * cfg.d
    return dt, flops


def cpu_baseline(cfg, seconds_target, threads):
    """The CPU baseline on a sample of about `seconds_target` seconds: whole heads (all query rows) from
    head 0 on, as many as the rate of a first, untimed head (which also warms the thread pool) allows, at
    most all of the config's heads."""
    head_s, _ = time_cpu_reference(cfg, 1, cfg.N, threads)
    heads = int(max(1, min(cfg.BH, round(seconds_target / max(head_s, 1e-6)))))
    dt, fl = time_cpu_reference(cfg, heads, cfg.N, threads)
    return {"value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"heads [0,{heads}) of {cfg.name}, all {cfg.N} query rows x all keys each, fp32 SDPA math on "
                      f"CPU (oracle.reference_sdpa), {dt:.1f} s"}


def run_reference_arm(args, rank, world):
    """--impl reference: the reference's CPU implementation of the path, timed on this host."""
    if rank != 0:
        return 0
    import torch
    cfg = get_config(args.config)
    if cfg.causal:
        raise SystemExit("reference arm samples query rows; causal configs are not supported here")
    threads = os.cpu_count() or 1
    rows = min(cfg.N, 4096)  # one bounded sample per step (~0.05-0.3 s on 8-16 cores)
    for _ in range(max(args.warmup, 0)):
        time_cpu_reference(cfg, 1, rows, threads)
    times = []
    flops = 0.0
    for _ in range(args.steps):
        dt, flops = time_cpu_reference(cfg, 1, rows, threads)
        times.append(dt)
    total = sum(times)
    value = flops * args.steps / total / 1e12
    sample = f"head 0, query rows [0,{rows}) x all {cfg.N} keys of {cfg.name} per step (fp32 SDPA math on CPU)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": cfg.describe(),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "torch_threads": torch.get_num_threads(),
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------ GPU side
def reference_rows(q, k, v, rows, causal):
    """float64 softmax(q[rows] k^T / sqrt(d)) v of one head ((N, d) tensors) on the device: the gate's truth."""
    import torch
    d = q.shape[-1]
    s = (q[rows].double() @ k.double().T) * (1.0 / math.sqrt(d))
    if causal:
        s.masked_fill_(torch.arange(k.shape[0], device=s.device)[None, :] > rows[:, None], float("-inf"))
    return torch.softmax(s, dim=-1) @ v.double()


def gate_errors(out, ref64, dtype):
    """The tests' parity figures of 16-bit output rows against the float64 truth: relative L2 against the
    truth rounded to the output dtype, the largest error beyond one output ulp, and the raw max abs."""
    import torch
    out = out.double()
    ref_r = ref64.to(dtype).double()
    bits = MANTISSA_BITS[str(dtype)]
    ulp = torch.exp2(torch.floor(torch.log2(ref_r.abs().clamp_min(2.0 ** -14))) - bits)
    diff = (out - ref_r).abs()
    den = ref_r.norm().item()
    return {"rel_l2": (out - ref_r).norm().item() / den if den > 0 else out.norm().item(),
            "max_excess": (diff - ulp).max().item(), "max_abs_raw": (out - ref64).abs().max().item()}


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
    from cuda_attn.dist import gather_heads
    from cuda_attn.workloads import Config, head_range, make_inputs

    base = get_config(args.config)
    if args.scaling == "weak":
        # every rank owns a config-sized batch; the job is B*world batches
        job = Config(base.name, base.B * world, base.H, base.N, base.d, base.dtype, base.causal, base.std,
                     base.k_outlier_frac, base.k_outlier_scale, base.seed, base.notes)
        my_heads = (rank * base.BH, (rank + 1) * base.BH)
    else:
        if base.BH < world:
            raise SystemExit(f"strong scaling needs at least one head per rank ({base.BH} heads, {world} ranks)")
        job = base
        my_heads = head_range(base.BH, world, rank)
    n_mine = my_heads[1] - my_heads[0]
    q, k, v = make_inputs(job, heads=my_heads, device=dev)  # (1, n_mine, N, d)
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

    # ---- correctness gate (reference bench/benchmark.py:165-171), before any timing: sampled query rows of
    # every head are gathered to rank 0, which regenerates each head's seeded inputs and checks the rows
    # against the float64 truth with the tests' criterion
    capi.fused_tc(q, k, v, o, causal=job.causal)
    torch.cuda.synchronize()
    rows = torch.linspace(0, job.N - 1, min(job.N, GATE_ROWS), device=dev).round().long().unique()
    samples = o[0][:, rows].contiguous().unsqueeze(0)  # (1, n_mine, rows, d)
    gathered = gather_heads(samples, job.BH, world, rank) if world > 1 else samples
    status = capi.device_status()
    gate = {"heads_checked": 0, "rows_per_head": int(rows.numel()), "rel_l2": 0.0, "rel_l2_max_head": 0.0,
            "max_excess": 0.0, "max_abs_raw": 0.0}
    if rank == 0:
        num = den = 0.0
        for h in range(job.BH):
            hq, hk, hv = (x[0, 0] for x in make_inputs(job, heads=(h, h + 1), device=dev))
            ref = reference_rows(hq, hk, hv, rows, job.causal)
            err = gate_errors(gathered[0, h], ref, job.dtype)
            ref_r = ref.to(job.dtype).double()
            num += (gathered[0, h].double() - ref_r).norm().item() ** 2
            den += ref_r.norm().item() ** 2
            gate["rel_l2_max_head"] = max(gate["rel_l2_max_head"], err["rel_l2"])
            for key in ("max_excess", "max_abs_raw"):
                gate[key] = max(gate[key], err[key])
            gate["heads_checked"] += 1
        gate["rel_l2"] = math.sqrt(num / den) if den > 0 else math.sqrt(num)
    status = int(max_over_ranks(float(status)))
    gate_ok = status == 0 and gate["rel_l2"] <= TOL_RELL2 and gate["max_excess"] <= TOL_MAXABS
    if world > 1:
        t = torch.tensor([1.0 if gate_ok else 0.0], device=dev)
        dist.broadcast(t, src=0)
        gate_ok = bool(t.item() > 0.5)

    # peak device memory of one call through the torch API (reference bench/benchmark.py:96-102 records
    # peak_memory_mb): torch's allocation (O) plus the library's per-launch scratch high-water mark
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats(dev)
    mem_base = torch.cuda.memory_allocated(dev)
    capi.scratch_bytes(reset=True)
    o_api = cuda_attn.fused_tc(q, k, v, job.causal)
    torch.cuda.synchronize()
    scratch_hw, scratch_reserved = capi.scratch_bytes()
    peak_mem = {"torch_mb": (torch.cuda.max_memory_allocated(dev) - mem_base) / 2**20,
                "library_scratch_mb": scratch_hw / 2**20, "library_pool_reserved_mb": scratch_reserved / 2**20}
    peak_mem["peak_memory_mb"] = peak_mem["torch_mb"] + peak_mem["library_scratch_mb"]
    del o_api

    def step():
        capi.fused_tc(q, k, v, o, causal=job.causal, stream=stream)

    qkv_bytes = 3 * q.numel() * q.element_size()
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev) if qkv_bytes < 2 * L2_BYTES else None

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
    barrier()
    torch.cuda.synchronize()
    if flush is None:
        # inputs larger than L2: K steps back to back between one event pair
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        ms_total = e0.elapsed_time(e1)
    else:
        # inputs within L2: L2 flushed (a write larger than L2) before every step, outside its event pair
        pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                 for _ in range(args.steps)]
        for a, b in pairs:
            flush.zero_()
            a.record(stream)
            step()
            b.record(stream)
        torch.cuda.synchronize()
        ms_total = sum(a.elapsed_time(b) for a, b in pairs)
    clocks = sampler.stop()
    barrier()
    kernel_ms, kernel_launches = capi.kernel_timing_read()
    capi.kernel_timing(False)
    launches = capi.launch_count()
    status = int(max_over_ranks(float(capi.device_status())))
    gate_ok = gate_ok and status == 0
    ms_total_max = max_over_ranks(ms_total)
    ms_per_step = ms_total_max / args.steps
    total_flops = job.flops()  # every rank's heads
    value = total_flops / (ms_per_step * 1e-3) / 1e12

    # ---- end-to-end loop through the public API with host buffers
    e2e_steps = args.e2e_steps or max(3, args.steps // 4)
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    ho = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)

    def e2e_step():
        # public API for host-resident tensors: head chunks stream through the GPU, host->device copy of
        # chunk i+1, attention of chunk i and device->host copy of chunk i-1 overlapping
        cuda_attn.fused_tc_host(hq, hk, hv, job.causal, out=ho, synchronize=False)

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
    # the host pipeline runs every query block over its whole K/V range; the device-resident run may have
    # cut its last wave into K/V parts (few-wave launches), which agrees within tolerance, not bit for bit
    ho_dev = ho.to(dev)
    e2e_same = {"bitwise": bool(torch.equal(ho_dev, o))}
    if not e2e_same["bitwise"]:
        e2e_same["rel_l2"] = ((ho_dev.double() - o.double()).norm() / o.double().norm()).item()

    peaks, peak_kind = load_peaks()
    peak_sus = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    peak_burst = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    sustained = ms_total_max >= SUSTAINED_AFTER_MS
    peak = peak_sus if sustained else peak_burst
    flops_per_launch = job.flops(heads=n_mine)
    avg_kernel_ms = kernel_ms / kernel_launches if kernel_launches else None
    achieved = flops_per_launch / (avg_kernel_ms * 1e-3) / 1e12 if avg_kernel_ms else None
    kernel_ms_max = max_over_ranks(avg_kernel_ms or 0.0)
    sm_mhz = (clocks or {}).get("sm_mhz")

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0 if gate_ok else 1

    cpu = None
    if not args.no_cpu_baseline and world == 1 and not job.causal:
        cpu = cpu_baseline(base, args.cpu_seconds, os.cpu_count() or 1)

    per_gpu = value / world
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": {"torch.bfloat16": "bf16", "torch.float16": "f16",
                                        "torch.float32": "f32"}[str(base.dtype)],
        "data": "synthetic: " + (base.notes or f"N(0,{base.std})") + ", seeded per global head",
        "config": dict(job.describe(), global_batch=job.B, heads_per_gpu=n_mine,
                       parallelism=f"heads sharded over {world} GPU(s) ({args.scaling} scaling), no collective",
                       l2=("no flush: Q/K/V per GPU %.0f MiB, more than twice the 126 MB L2" % (qkv_bytes / 2**20))
                       if flush is None else ("L2 flushed before every step (%d MiB write, outside the step's event "
                                              "pair): Q/K/V per GPU %.0f MiB" % (2 * L2_BYTES >> 20, qkv_bytes / 2**20))),
        "per_gpu_tflops": per_gpu,
        "pct_of_peak": {"measured_burst": 100.0 * per_gpu / peak_burst, "measured_sustained": 100.0 * per_gpu / peak_sus,
                        "spec_dense": 100.0 * per_gpu / SPEC_DENSE_BF16_TFLOPS, "peaks": peak_kind},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": (achieved / peak) if achieved else None,
                     "traffic": load_traffic() if base.name == TRAFFIC_WORKLOAD and args.scaling == "strong"
                     and world == 1 else None,
                     "peak_kind": (f"{peak_kind} bf16 " + ("sustained (MEASURED_PEAKS.json bf16_tflops_sustained)"
                                   if sustained else "burst (MEASURED_PEAKS.json bf16_tflops)") +
                                   f": timed region {ms_total_max:.0f} ms " +
                                   (">=" if sustained else "<") + f" {SUSTAINED_AFTER_MS:.0f} ms"),
                     "frac_of_burst": (achieved / peak_burst) if achieved else None,
                     "frac_of_sustained": (achieved / peak_sus) if achieved else None,
                     "frac_of_spec_dense": (achieved / SPEC_DENSE_BF16_TFLOPS) if achieved else None,
                     "kernel": "phantom::tc::attn_fwd_tc", "kernel_ms_avg": avg_kernel_ms,
                     "kernel_ms_avg_max_rank": kernel_ms_max, "flops_per_launch": flops_per_launch,
                     "kernel_mcycles_at_median_sm_clock": avg_kernel_ms * sm_mhz * 1e-3 if avg_kernel_ms and sm_mhz else None},
        "e2e": {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "steps": e2e_steps,
                "path": "pinned host -> cuda_attn.fused_tc_host (public API; copies overlapped with the kernel over head chunks: at most 8 full ones of at least 32 MiB per input tensor, the last cut in halves down to 8 MiB) -> pinned host", "matches_value_run": e2e_same},
        "memory": dict(peak_mem, inputs_mb=3 * q.numel() * q.element_size() / 2**20,
                       note="one cuda_attn.fused_tc call on this rank's heads: O from torch plus the library's "
                            "scratch (bf16: fp16 copy of V; multi-wave: work counter; K/V parts: partials)"),
        "gpu_launches": launches,
        "kernel_launches_timed": kernel_launches,
        "clocks": clocks,
        "correctness": dict(gate, criterion=f"relative L2 of the sampled output (all checked heads) <= {TOL_RELL2} "
                                              f"vs the float64 truth rounded to the output dtype; max abs <= "
                                              f"{TOL_MAXABS} beyond one output ulp; rel_l2_max_head: the largest "
                                              f"single head's figure, reported",
                            status=status, ok=gate_ok),
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0 if gate_ok else 1


if __name__ == "__main__":
    sys.exit(main())
