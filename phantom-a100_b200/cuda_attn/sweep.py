"""Sequence-length sweep of the attention kernels (the reference's bench/benchmark.py, on B200).

    python -m cuda_attn.sweep                                   # B*H=64, fp16, d 64 and 128
    python -m cuda_attn.sweep --ns 1024 4096 --impls fused_tc sdpa_default --dtype bf16 --out sweep.csv

For every (causal, d, N) and implementation: a correctness gate against the fp32 math-backend SDPA
(reference bench/benchmark.py:165-171; fp16/bf16 relative L2 <= 1e-3 against the rounded reference, fp32
max abs <= 1e-4) - a wrong result is recorded as wrong_result and never timed - then warm-ups and timed
runs with CUDA events and the L2 flushed before each run (benchmark.py:78-93; the flush buffer is twice
the L2 size), median / p10 / p90. Reported: TFLOP/s (4*B*H*N^2*d, halved when causal), algorithmic HBM
GB/s (Q, K, V read and O written once), their fractions of the measured peaks, and the roofline regime
(HBM-bound below the ridge intensity peak_flops / peak_bandwidth, tensor-bound above).
"""
from __future__ import annotations

import argparse
import csv
import os
import sys
from datetime import datetime, timezone

import numpy as np
import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

from . import KERNELS, fused_tuned, reference
from .hw_counters import load_peaks


def sdpa_math_backend(q, k, v, causal):
    """torch SDPA restricted to the math backend (materialises the N x N scores; calibration only)."""
    with sdpa_kernel(SDPBackend.MATH):
        return F.scaled_dot_product_attention(q, k, v, is_causal=causal)


def sdpa_library(q, k, v, causal):
    """torch SDPA with its default backend choice (a library kernel; calibration only)."""
    return F.scaled_dot_product_attention(q, k, v, is_causal=causal)


IMPLS = dict(KERNELS, fused_tuned_128x64=lambda q, k, v, c: fused_tuned(q, k, v, c, True, 128, 64),
             sdpa_math=sdpa_math_backend, sdpa_default=sdpa_library)
TENSOR_CORE = {"fused_vec", "fused_db", "fused_tc", "fused_tuned_128x64"}


def attention_flops(b, h, n, d, causal):
    """Two N x N x d matmuls per (batch, head): 2 * 2 * N^2 * d FLOPs; causal keeps half of them."""
    return (0.5 if causal else 1.0) * 4.0 * b * h * n * n * d


def time_cuda(fn, warmup, iters, flush_buf):
    """Per-run device time of fn() in ms as (median, p10, p90). Every run is bracketed by its own event
    pair on the current stream, with the L2 cache overwritten (flush_buf, larger than L2) just before the
    pair; the runs are queued back to back and read after one synchronize, so host launch gaps between
    runs do not enter the figures."""
    for _ in range(warmup):
        fn()
    stream = torch.cuda.current_stream()
    marks = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for start, stop in marks:
        flush_buf.fill_(1)
        start.record(stream)
        fn()
        stop.record(stream)
    stop.synchronize()
    ms = np.array([a.elapsed_time(b) for a, b in marks])
    return float(np.median(ms)), float(np.percentile(ms, 10)), float(np.percentile(ms, 90))


def peak_memory_mb(fn, lib=None):
    """Device memory one call takes beyond what was allocated before it (reference bench/benchmark.py:96-102):
    torch's peak allocation delta plus, for this library's kernels, its per-launch scratch high-water mark
    (the scratch comes from the library's own memory pool, which torch does not see)."""
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    if lib is not None:
        lib.scratch_bytes(reset=True)
    fn()
    torch.cuda.synchronize()
    mb = (torch.cuda.max_memory_allocated() - base) / 2**20
    if lib is not None:
        mb += lib.scratch_bytes()[0] / 2**20
    return mb


def check(out, ref, dtype):
    out, ref = out.double(), ref.double()
    if dtype == torch.float32:
        err = (out - ref).abs().max().item()
        return err, err <= 1e-4
    ref_r = ref.to(dtype).double()
    rel = ((out - ref_r).norm() / ref_r.norm()).item()
    return rel, rel <= 1e-3


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--impls", nargs="+", default=["fused_tc", "sdpa_default"])
    p.add_argument("--ns", nargs="+", type=int, default=[128, 256, 512, 1024, 2048, 4096, 8192])
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--heads", type=int, default=64)
    p.add_argument("--dims", nargs="+", type=int, default=[64, 128])
    p.add_argument("--dtype", choices=["fp16", "bf16", "fp32"], default="fp16")
    p.add_argument("--causal", choices=["off", "on", "both"], default="off")
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--iters", type=int, default=50)
    p.add_argument("--out", default="sweep.csv")
    a = p.parse_args(argv)

    assert torch.cuda.is_available(), "the sweep needs a CUDA GPU"
    dtype = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[a.dtype]
    peaks = load_peaks()
    ridge = peaks["bf16_tflops_sustained"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    flush = torch.empty(max(2 * l2, 64 * 2**20), dtype=torch.uint8, device="cuda")
    meta = dict(gpu=torch.cuda.get_device_name(), cc="sm_%d%d" % torch.cuda.get_device_capability(),
                torch=torch.__version__, timestamp=datetime.now(timezone.utc).isoformat(timespec="seconds"))
    fields = ["gpu", "cc", "torch", "timestamp", "impl", "dtype", "causal", "B", "H", "N", "d", "median_ms", "p10_ms",
              "p90_ms", "tflops", "hbm_gbs", "frac_bf16_sustained", "frac_hbm", "regime", "peak_memory_mb", "err",
              "status"]
    from .capi import CAPI
    lib = CAPI()
    causal_modes = {"off": [False], "on": [True], "both": [False, True]}[a.causal]
    with open(a.out, "w", newline="") as fh:
        w = csv.DictWriter(fh, fieldnames=fields)
        w.writeheader()
        for causal in causal_modes:
            for d in a.dims:
                for n in a.ns:
                    b, h = a.batch, a.heads
                    g = torch.Generator(device="cuda").manual_seed(n * 1000 + d)
                    q, k, v = (torch.randn(b, h, n, d, device="cuda", generator=g).to(dtype) for _ in range(3))
                    ref = reference(q, k, v, causal) if n <= 8192 else None
                    flops = attention_flops(b, h, n, d, causal)
                    nbytes = 4.0 * b * h * n * d * q.element_size()
                    regime = "hbm" if flops / nbytes < ridge else "tensor"
                    for name in a.impls:
                        row = dict(meta, impl=name, dtype=a.dtype, causal=causal, B=b, H=h, N=n, d=d, regime=regime)
                        if name in TENSOR_CORE and (dtype == torch.float32 or d not in (64, 128)):
                            w.writerow(dict(row, status="unsupported"))
                            continue
                        fn = lambda: IMPLS[name](q, k, v, causal)  # noqa: E731
                        try:
                            if ref is not None:
                                err, ok = check(fn(), ref, dtype)
                                if not ok:
                                    w.writerow(dict(row, err=f"{err:.2e}", status="wrong_result"))
                                    continue
                            else:
                                err = float("nan")
                            med, p10, p90 = time_cuda(fn, a.warmup, a.iters, flush)
                            mem = peak_memory_mb(fn, lib if name in TENSOR_CORE else None)
                        except torch.cuda.OutOfMemoryError:
                            torch.cuda.empty_cache()
                            w.writerow(dict(row, status="oom"))
                            continue
                        tf = flops / (med * 1e-3) / 1e12
                        gbs = nbytes / (med * 1e-3) / 1e9
                        w.writerow(dict(row, median_ms=f"{med:.4f}", p10_ms=f"{p10:.4f}", p90_ms=f"{p90:.4f}",
                                        tflops=f"{tf:.2f}", hbm_gbs=f"{gbs:.1f}",
                                        frac_bf16_sustained=f"{tf / peaks['bf16_tflops_sustained']:.3f}",
                                        frac_hbm=f"{gbs / peaks['hbm_gbs']:.3f}", peak_memory_mb=f"{mem:.3f}",
                                        err=f"{err:.2e}", status="ok"))
                        fh.flush()
                        print(f"causal={causal!s:5} d={d:3} N={n:5} {name:20} {med:8.4f} ms {tf:8.1f} TFLOP/s "
                              f"{gbs:8.1f} GB/s [{regime}] err={err:.1e}", flush=True)
                    del q, k, v, ref
    print(f"wrote {a.out}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
