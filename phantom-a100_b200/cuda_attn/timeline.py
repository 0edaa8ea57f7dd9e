"""Copy / compute timeline of the host pipeline (cuda_attn.fused_tc_host), from CUDA events.

The reference's bench/profile.sh took an Nsight Systems timeline of its benchmark. Here the question that
view answers for this path - how the host->device copies, the attention launches and the device->host
copies of fused_tc_host overlap, and what bounds a call - is measured with CUDA events recorded around
every stage of every chunk (the `trace` argument of fused_tc_host), for back-to-back calls:

    python -m cuda_attn.timeline                       # BASELINE config 4, 8 chunks, 3 timed calls
    python -m cuda_attn.timeline --config config3 --chunks 16 --out timeline.md

Printed: per chunk the start / end of each stage (ms from the first timed call's start), per stage the
busy time and the achieved link bandwidth, and the time per call.
"""
from __future__ import annotations

import argparse
import sys

import torch

from . import fused_tc_host
from .workloads import CONFIGS, make_inputs


def run(cfg_name: str = "config4", chunks: int = 8, calls: int = 3, warmup: int = 2):
    cfg = CONFIGS[cfg_name]
    q, k, v = make_inputs(cfg, device="cuda")
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    ho = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    for _ in range(warmup):
        fused_tc_host(hq, hk, hv, cfg.causal, out=ho, chunks=chunks, synchronize=False)
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    traces = []
    t_start.record(cur)
    for _ in range(calls):
        tr = []
        fused_tc_host(hq, hk, hv, cfg.causal, out=ho, chunks=chunks, synchronize=False, trace=tr)
        traces.append(tr)
    t_end.record(cur)
    torch.cuda.synchronize()
    rel = t_start.elapsed_time
    rows = []
    for c, tr in enumerate(traces):
        for i, rec in enumerate(tr):
            rows.append({"call": c, "chunk": i, "heads": rec["heads"],
                         **{st: (rel(rec[st][0]), rel(rec[st][1])) for st in ("h2d", "attend", "d2h")}})
    per_head_in = 3 * cfg.N * cfg.d * q.element_size()
    per_head_out = cfg.N * cfg.d * q.element_size()
    total = t_start.elapsed_time(t_end)
    busy = {st: sum(r[st][1] - r[st][0] for r in rows) for st in ("h2d", "attend", "d2h")}
    summary = {"config": cfg_name, "chunks": chunks, "ms_per_call": total / calls,
               "h2d_busy_ms_per_call": busy["h2d"] / calls, "attend_busy_ms_per_call": busy["attend"] / calls,
               "d2h_busy_ms_per_call": busy["d2h"] / calls,
               "h2d_gbs_while_busy": per_head_in * cfg.BH * calls / (busy["h2d"] * 1e-3) / 1e9,
               "d2h_gbs_while_busy": per_head_out * cfg.BH * calls / (busy["d2h"] * 1e-3) / 1e9}
    return summary, rows


def to_markdown(summary: dict, rows: list, argv: list[str]) -> str:
    out = ["# fused_tc_host timeline (CUDA events)", "", "```", "python -m cuda_attn.timeline " + " ".join(argv), "```",
           "", "| figure | value |", "|---|---|"]
    out += [f"| {k} | {v:.3f} |" if isinstance(v, float) else f"| {k} | {v} |" for k, v in summary.items()]
    out += ["", "| call | chunk | heads | h2d ms | attend ms | d2h ms |", "|---|---|---|---|---|---|"]
    for r in rows:
        out.append(f"| {r['call']} | {r['chunk']} | {r['heads']} | {r['h2d'][0]:.3f}-{r['h2d'][1]:.3f} | "
                   f"{r['attend'][0]:.3f}-{r['attend'][1]:.3f} | {r['d2h'][0]:.3f}-{r['d2h'][1]:.3f} |")
    return "\n".join(out) + "\n"


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", default="config4", choices=[c for c in CONFIGS if c != "config1"])
    ap.add_argument("--chunks", type=int, default=8)
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--out", default=None, help="write a markdown summary here")
    a = ap.parse_args(argv)
    summary, rows = run(a.config, a.chunks, a.calls)
    for k, v in summary.items():
        print(f"{k:26s} {v:.3f}" if isinstance(v, float) else f"{k:26s} {v}")
    for r in rows:
        print(f"call {r['call']} chunk {r['chunk']:2d} heads {r['heads']:2d}  h2d {r['h2d'][0]:8.3f}-{r['h2d'][1]:8.3f}"
              f"  attend {r['attend'][0]:8.3f}-{r['attend'][1]:8.3f}  d2h {r['d2h'][0]:8.3f}-{r['d2h'][1]:8.3f}")
    if a.out:
        with open(a.out, "w") as f:
            f.write(to_markdown(summary, rows, argv))
    return 0


if __name__ == "__main__":
    sys.exit(main())
