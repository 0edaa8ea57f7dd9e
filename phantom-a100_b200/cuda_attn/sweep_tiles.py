"""Launch-shape sweep of the tensor-core kernel: the reference's tile sweep (bench/sweep_tiles.py), on B200.

    python -m cuda_attn.sweep_tiles                          # N = 1024, 4096, 8192; B=4, H=16, d=64, fp16
    python -m cuda_attn.sweep_tiles --ns 16384 --batch 1 --heads 32 --dim 128 --dtype bf16 --out tiles.csv

The reference timed each compiled (BR, BC) tile x {single, double buffer} of its tuned WMMA kernel and
printed the winner per sequence length (bench/sweep_tiles.py:22-63). On sm_100a the tile is fixed by the
tcgen05 instruction shape (128-row Q tiles, 128-key K/V tiles, a TMA ring of fixed depth), so the
reference's eight tile configs all run the same kernel: they are swept first, as the reference does, and
should time alike. The knobs that do change this kernel's schedule are its launch shape
(phantom_attn_set_launch_shape):

  l2_group_kib  K/V bytes per scheduling group of heads. The persistent CTAs take every query block of a
                group before the next group; a group whose K/V fits L2 streams it from DRAM once.
  max_ctas      size of the persistent grid (default: one CTA per SM).

Every configuration passes a correctness gate first, as in the reference (sweep_tiles.py:47-49, max abs
difference <= 2e-3 against the reference result; here the result of the default launch shape, itself
checked against the fp32 math-backend SDPA at relative L2 <= 1e-3 where that fits in memory); a wrong
result is recorded as wrong_result and never timed. Timing: CUDA events, L2 flushed before every run;
the configurations are timed interleaved, one run each per round for --iters rounds, and each reports the
median of its runs. (Timed one after the other, the first configuration ran 5-12% faster than the same
kernel timed later: the GPU starts cool and settles under its power cap.) One CSV row per configuration,
the reference's columns first.
"""
from __future__ import annotations

import argparse
import csv
import statistics
import sys

import torch

from . import fused_tc, fused_tuned, reference
from .capi import CAPI
from .sweep import attention_flops, check

# The reference's compiled tiles of fused_tuned (reference csrc/kernels/fused_tuned.cuh:206-207).
TILES = [(64, 32), (64, 64), (128, 32), (128, 64)]
# L2 head-group sizes (KiB): 2 MiB .. 128 MiB, and 0 = automatic (16 MiB).
GROUPS_KIB = [0, 2048, 4096, 8192, 16384, 32768, 65536, 131072]


def time_interleaved(fns, warmup, rounds, flush_buf):
    """Per function: (median, p10, p90) ms of `rounds` runs, timed one run of each function per round
    with CUDA events and the L2 flushed before every run, so that clock drift falls on all alike."""
    for fn in fns:
        for _ in range(warmup):
            fn()
    torch.cuda.synchronize()
    times = [[] for _ in fns]
    for _ in range(rounds):
        for i, fn in enumerate(fns):
            flush_buf.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            times[i].append(s.elapsed_time(e))
    out = []
    for t in times:
        qs = statistics.quantiles(t, n=10) if len(t) >= 2 else [t[0]] * 9
        out.append((statistics.median(t), qs[0], qs[-1]))
    return out


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--ns", nargs="+", type=int, default=[1024, 4096, 8192])
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--heads", type=int, default=16)
    p.add_argument("--dim", type=int, default=64, choices=[64, 128])
    p.add_argument("--dtype", choices=["fp16", "bf16"], default="fp16")
    p.add_argument("--causal", action="store_true")
    p.add_argument("--groups-kib", nargs="+", type=int, default=GROUPS_KIB)
    p.add_argument("--max-ctas", nargs="+", type=int, default=[0],
                   help="persistent grid caps to sweep (0 = one CTA per SM)")
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--iters", type=int, default=50)
    p.add_argument("--out", default=None)
    a = p.parse_args(argv)

    assert torch.cuda.is_available(), "the tile sweep needs a CUDA GPU"
    dtype = {"fp16": torch.float16, "bf16": torch.bfloat16}[a.dtype]
    gpu = torch.cuda.get_device_name()
    out = a.out or f"tiles_{gpu.replace(' ', '_')}{'_causal' if a.causal else ''}.csv"
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    flush = torch.empty(max(2 * l2, 64 * 2**20), dtype=torch.uint8, device="cuda")
    lib = CAPI()
    fields = ["gpu", "N", "br", "bc", "double_buffer", "l2_group_kib", "max_ctas", "median_ms", "p10_ms",
              "p90_ms", "tflops", "err", "status"]
    b, h, d = a.batch, a.heads, a.dim
    try:
        with open(out, "w", newline="") as fh:
            w = csv.DictWriter(fh, fieldnames=fields)
            w.writeheader()
            for n in a.ns:
                g = torch.Generator(device="cuda").manual_seed(n * 1000 + d)
                q, k, v = (torch.randn(b, h, n, d, device="cuda", generator=g).to(dtype) for _ in range(3))
                flops = attention_flops(b, h, n, d, a.causal)
                lib.set_launch_shape(0, 0)
                base = fused_tc(q, k, v, a.causal)
                if n <= 8192:
                    err, ok = check(base, reference(q, k, v, a.causal), dtype)
                    if not ok:
                        raise RuntimeError(f"N={n}: default launch shape fails the SDPA gate (rel L2 {err:.2e})")
                configs = [dict(br=br, bc=bc, double_buffer=db, l2_group_kib=0, max_ctas=0)
                           for br, bc in TILES for db in (False, True)]
                configs += [dict(br="", bc="", double_buffer="", l2_group_kib=kib, max_ctas=ctas)
                            for kib in a.groups_kib for ctas in a.max_ctas]

                def run(c):
                    lib.set_launch_shape(c["l2_group_kib"], c["max_ctas"])
                    if c["br"] != "":
                        return fused_tuned(q, k, v, a.causal, c["double_buffer"], c["br"], c["bc"])
                    return fused_tc(q, k, v, a.causal)

                timed = []
                for c in configs:
                    diff = (run(c).float() - base.float()).abs().max().item()
                    if diff > 2e-3:
                        w.writerow(dict(gpu=gpu, N=n, **c, err=f"{diff:.2e}", status="wrong_result"))
                    else:
                        timed.append((c, diff))
                stats = time_interleaved([lambda c=c: run(c) for c, _ in timed], a.warmup, a.iters, flush)
                best = None
                for (c, diff), (med, p10, p90) in zip(timed, stats):
                    row = dict(gpu=gpu, N=n, **c)
                    tf = flops / (med * 1e-3) / 1e12
                    w.writerow(dict(row, median_ms=f"{med:.4f}", p10_ms=f"{p10:.4f}", p90_ms=f"{p90:.4f}",
                                    tflops=f"{tf:.1f}", err=f"{diff:.2e}", status="ok"))
                    fh.flush()
                    label = (f"BR={c['br']:3} BC={c['bc']:3} double_buffer={c['double_buffer']!s:5}" if c["br"] != ""
                             else f"l2_group={c['l2_group_kib'] >> 10 or 'auto':>4} MiB max_ctas={c['max_ctas'] or 'auto'}")
                    print(f"N={n:5} {label:40} {med:8.4f} ms {tf:7.1f} TFLOP/s", flush=True)
                    if best is None or med < best[0]:
                        best = (med, label)
                if best:
                    print(f"--> best at N={n}: {best[1]} ({best[0]:.4f} ms)\n", flush=True)
                del q, k, v, base
    finally:
        lib.set_launch_shape(0, 0)
    print(f"wrote {out}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
