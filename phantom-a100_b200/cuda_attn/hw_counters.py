"""Nsight Compute counters of the attention kernels on B200, and the roofline figures derived from them.

The reference's autotune/hw_counters.py collected ncu metrics to compare GPGPU-Sim with an A100. Here the
same capability - kernel counters from ncu, a metric that cannot be collected reported as UNOBSERVABLE
rather than failing the run, and several launches of one forward call combined into one record - serves
the B200 roofline of this path:

  key           ncu metric (gb100)                                               one call (several launches)
  time_s        gpu__time_duration.sum                                           sum
  tensor_pct    sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active   time-weighted mean
  mufu_pct      sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active       time-weighted mean
  fma_pct       sm__pipe_fma_cycles_active.avg.pct_of_peak_sustained_active      time-weighted mean
  issue_pct     smsp__issue_active.avg.pct_of_peak_sustained_active              time-weighted mean
  warps_pct     sm__warps_active.avg.pct_of_peak_sustained_active                time-weighted mean
  dram_read     dram__bytes_read.sum                                             sum
  dram_write    dram__bytes_write.sum                                            sum
  registers     launch__registers_per_thread                                     of the longest launch

How it works, in three steps that can run on different machines:

  1. check    the requested metrics against the chip's own list (`ncu --query-metrics --chip gb100`, which
              needs no GPU); unknown ones are left out of the capture and reported UNOBSERVABLE.
  2. capture  one ncu run (`--clock-control none`, so ncu never locks the GPU clocks) of the command,
              filtered to the kernels of interest (-k / -s / -c), written to an .ncu-rep file.
  3. read     the report with Nsight Compute's own Python reader (ncu_report, shipped with ncu under
              extras/python), in ncu's base units: time in ns, bytes, percent.

A call of the bf16 path is three launches (stage_v_f16, the main attn_fwd_tc, and an attn_fwd_tc for heads
whose V overflows fp16, which returns at once when there are none), and a call whose last wave runs as K/V
parts adds merge_kv_parts: `calls()` groups the launches of each call, and `aggregate()` combines them.

    python -m cuda_attn.hw_counters --flops 4.398e12 --bytes 536870912 --out profiles/x.md -- \
        python bench.py --config config4 --steps 1 --warmup 1 --no-cpu-baseline
"""
from __future__ import annotations

import argparse
import glob
import json
import os
import re
import shlex
import shutil
import subprocess
import sys
import tempfile
from dataclasses import dataclass

UNOBSERVABLE = "UNOBSERVABLE"


@dataclass(frozen=True)
class Counter:
    key: str
    metric: str
    combine: str       # "sum" | "time_mean" | "longest"
    scale: float = 1.0  # factor from ncu's base unit to the key's unit


COUNTERS = [
    Counter("time_s", "gpu__time_duration.sum", "sum", 1e-9),
    Counter("tensor_pct", "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active", "time_mean"),
    Counter("mufu_pct", "sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active", "time_mean"),
    Counter("fma_pct", "sm__pipe_fma_cycles_active.avg.pct_of_peak_sustained_active", "time_mean"),
    Counter("issue_pct", "smsp__issue_active.avg.pct_of_peak_sustained_active", "time_mean"),
    Counter("warps_pct", "sm__warps_active.avg.pct_of_peak_sustained_active", "time_mean"),
    Counter("dram_read", "dram__bytes_read.sum", "sum"),
    Counter("dram_write", "dram__bytes_write.sum", "sum"),
    Counter("registers", "launch__registers_per_thread", "longest"),
]
ATTENTION_KERNEL = "attn_fwd_tc"
PERMISSION_TEXT = ("ERR_NVGPUCTRPERM", "permission to access NVIDIA GPU Performance Counters")  # ncu's messages


def base_name(metric: str) -> str:
    """The counter a metric is read from: `sm__x.avg.pct_of_peak_sustained_active` -> `sm__x`."""
    return metric.split(".", 1)[0]


def chip_metrics(chip: str = "gb100", ncu: str | None = None) -> set[str] | None:
    """Base names of every metric ncu knows for `chip` (no GPU needed), or None if ncu cannot say."""
    ncu = ncu or shutil.which("ncu")
    if not ncu:
        return None
    try:
        out = subprocess.run([ncu, "--query-metrics", "--chip", chip, "--csv"], capture_output=True, text=True,
                             timeout=120).stdout
    except (OSError, subprocess.TimeoutExpired):
        return None
    names = {line.split(",", 1)[0].strip('"').rsplit(".", 1)[-1] for line in out.splitlines()[1:] if line.startswith('"')}
    return names or None


def split_metrics(metrics: list[str], known: set[str] | None) -> tuple[list[str], list[str]]:
    """(metrics to capture, metrics the chip does not have). launch__ figures are launch statistics,
    always present; with no chip list every metric is attempted."""
    if known is None:
        return list(metrics), []
    keep = [m for m in metrics if m.startswith("launch__") or base_name(m) in known]
    return keep, [m for m in metrics if m not in keep]


def ncu_command(cmd: list[str], report: str, metrics: list[str], kernel_regex: str, skip: int, count: int,
                ncu: str = "ncu") -> list[str]:
    return [ncu, "--clock-control", "none", "--metrics", ",".join(metrics), "-k", f"regex:{kernel_regex}",
            "-s", str(skip), "-c", str(count), "-f", "-o", report, *cmd]


def report_reader():
    """Nsight Compute's ncu_report module (extras/python next to the ncu installation), or None."""
    try:
        import ncu_report  # noqa: F401
        return ncu_report
    except ImportError:
        pass
    ncu = shutil.which("ncu")
    roots = []
    if ncu:
        real = os.path.realpath(ncu)
        roots += [os.path.join(os.path.dirname(os.path.dirname(real)), "extras", "python"),
                  os.path.join(os.path.dirname(real), "extras", "python")]
    roots += sorted(glob.glob("/opt/nvidia/nsight-compute/*/extras/python"), reverse=True)
    for r in roots:
        if os.path.exists(os.path.join(r, "ncu_report.py")):
            sys.path.insert(0, r)
            try:
                import ncu_report
                return ncu_report
            except ImportError:
                sys.path.remove(r)
    return None


def read_report(path: str, metrics: list[str], reader=None) -> list[dict]:
    """One record per profiled launch: {'kernel': demangled name, <metric>: value in ncu base units or None}."""
    reader = reader or report_reader()
    if reader is None:
        raise RuntimeError("Nsight Compute's ncu_report module was not found")
    ctx = reader.load_report(path)
    out = []
    for r in range(ctx.num_ranges()):
        rng = ctx.range_by_idx(r)
        for a in range(rng.num_actions()):
            act = rng.action_by_idx(a)
            rec = {"kernel": act.name()}
            for m in metrics:
                v = act.metric_by_name(m)
                rec[m] = None if v is None else float(v.as_double())
            out.append(rec)
    return out


MERGE_KERNEL = "merge_kv_parts"


def is_overflow_launch(name: str) -> bool:
    """Whether a launch is the second attention launch of a bf16 call, the one for heads whose V overflows
    fp16: `attn_fwd_tc<D, BF16, KV_PARTS, OVF_HEADS>` with OVF_HEADS set."""
    m = re.search(ATTENTION_KERNEL + r"<([^>]*)>", name)
    if not m:
        return False
    args = [a.strip() for a in m.group(1).split(",")]
    return len(args) >= 4 and args[3] in ("1", "true")


def calls(launches: list[dict], last: str = ATTENTION_KERNEL) -> list[list[dict]]:
    """Group launches into forward calls: each group ends with the main launch of the attention kernel (a
    bf16 call is stage_v_f16 then attn_fwd_tc; an fp16 call with more units than CTAs is zero_counter then
    attn_fwd_tc, when the capture's filter takes zero_counter in), followed by the merge_kv_parts launch
    when the call cut its last wave into K/V parts and, for bf16, the attention launch for fp16-overflow
    heads. Launches after the last main attention launch form no call."""
    groups, cur = [], []
    for rec in launches:
        if (MERGE_KERNEL in rec["kernel"] or is_overflow_launch(rec["kernel"])) and groups and not cur:
            groups[-1].append(rec)
            continue
        cur.append(rec)
        if last in rec["kernel"]:
            groups.append(cur)
            cur = []
    return groups


def aggregate(group: list[dict]) -> dict:
    """One record for a group of launches, in the counters' units; a counter missing from any launch it
    needs is UNOBSERVABLE."""
    t = [rec.get("gpu__time_duration.sum") for rec in group]
    longest = max(range(len(group)), key=lambda i: t[i] or 0.0) if group else None
    out = {"kernels": [rec["kernel"] for rec in group]}
    for c in COUNTERS:
        vals = [rec.get(c.metric) for rec in group]
        if not group or (c.combine != "longest" and any(v is None for v in vals)):
            out[c.key] = UNOBSERVABLE
        elif c.combine == "sum":
            out[c.key] = sum(vals) * c.scale
        elif c.combine == "time_mean":
            if any(x is None for x in t) or sum(t) <= 0:
                out[c.key] = UNOBSERVABLE
            else:
                out[c.key] = sum(v * x for v, x in zip(vals, t)) / sum(t) * c.scale
        else:
            v = vals[longest]
            out[c.key] = UNOBSERVABLE if v is None else v * c.scale
    return out


def load_peaks(path: str | None = None) -> dict:
    """Measured peaks (MEASURED_PEAKS.json at the repository root) or the pool's fallback figures."""
    path = path or os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                                "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"bf16_tflops": p["bf16_tflops"], "bf16_tflops_sustained": p["bf16_tflops_sustained"],
                "hbm_gbs": p["hbm_gbs"], "kind": "measured"}
    except (OSError, ValueError, KeyError):
        return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "kind": "fallback"}


def roofline(rec: dict, flops: float | None = None, algorithmic_bytes: float | None = None,
             peaks: dict | None = None) -> dict:
    """Roofline figures of one aggregated record: achieved TFLOP/s and its fraction of the measured bf16
    peaks, DRAM GB/s and its fraction of the measured copy bandwidth, and DRAM bytes over the algorithmic
    bytes (well above 1 means re-reads)."""
    peaks = peaks or load_peaks()
    out = {"peaks": peaks["kind"]}
    t = rec.get("time_s")
    timed = isinstance(t, float) and t > 0
    if timed and flops:
        out["tflops"] = flops / t / 1e12
        out["frac_bf16_burst"] = out["tflops"] / peaks["bf16_tflops"]
        out["frac_bf16_sustained"] = out["tflops"] / peaks["bf16_tflops_sustained"]
    rd, wr = rec.get("dram_read"), rec.get("dram_write")
    if timed and isinstance(rd, float) and isinstance(wr, float):
        out["dram_gbs"] = (rd + wr) / t / 1e9
        out["frac_hbm"] = out["dram_gbs"] / peaks["hbm_gbs"]
        if algorithmic_bytes:
            out["traffic_over_algorithmic"] = (rd + wr) / algorithmic_bytes
    return out


def profile(cmd: list[str], kernel_regex: str = "attn_fwd_tc|stage_v_f16|merge_kv_parts", skip: int = 0, count: int = 2,
            report: str | None = None, chip: str = "gb100", timeout: int = 900) -> dict:
    """check -> capture -> read for `cmd`. Returns {'status', 'launches', 'unobservable', 'report', 'log'};
    status ok | no_ncu | no_permission | no_reader | error."""
    ncu = shutil.which("ncu")
    if not ncu:
        return {"status": "no_ncu", "launches": [], "unobservable": [], "report": None, "log": ""}
    wanted = [c.metric for c in COUNTERS]
    metrics, missing = split_metrics(wanted, chip_metrics(chip, ncu))
    report = report or os.path.join(tempfile.mkdtemp(prefix="hwc_"), "capture")
    p = subprocess.run(ncu_command(cmd, report, metrics, kernel_regex, skip, count, ncu), stdout=subprocess.PIPE,
                       stderr=subprocess.STDOUT, text=True, timeout=timeout)
    res = {"launches": [], "unobservable": missing, "report": report + ".ncu-rep", "log": p.stdout[-3000:],
           "command": shlex.join(ncu_command(cmd, report, metrics, kernel_regex, skip, count, "ncu"))}
    if any(s in p.stdout for s in PERMISSION_TEXT):
        return dict(res, status="no_permission")
    if p.returncode != 0 or not os.path.exists(res["report"]):
        return dict(res, status="error")
    reader = report_reader()
    if reader is None:
        return dict(res, status="no_reader")
    res["launches"] = read_report(res["report"], metrics, reader)
    return dict(res, status="ok" if res["launches"] else "error")


def summary_markdown(res: dict, cmd: list[str], flops, nbytes, peaks: dict) -> str:
    lines = [f"# ncu counters via `cuda_attn.hw_counters`", "",
             f"Produced by (run in `{os.path.basename(os.getcwd())}/`, after the same command exited 0 without "
             "ncu):", "",
             "```", "python -m cuda_attn.hw_counters " + " ".join(sys.argv[1:]), "```", "",
             "which ran:", "", "```", res.get("command", ""), "```", ""]
    groups = calls(res["launches"])
    for i, g in enumerate(groups):
        agg = aggregate(g)
        rf = roofline(agg, flops, nbytes, peaks)
        lines += [f"## call {i + 1}: " + " + ".join(k.split("(")[0] for k in agg["kernels"]), "",
                  "| figure | value |", "|---|---|"]
        for k, v in list(agg.items())[1:] + list(rf.items()):
            lines.append(f"| {k} | {v:.4g} |" if isinstance(v, float) else f"| {k} | {v} |")
        lines.append("")
    if res["unobservable"]:
        lines.append("Not available on this chip / ncu: " + ", ".join(res["unobservable"]))
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--kernel", default="attn_fwd_tc|stage_v_f16|merge_kv_parts", help="ncu -k regex")
    ap.add_argument("--skip", type=int, default=0, help="matching launches to skip (ncu -s)")
    ap.add_argument("--count", type=int, default=2, help="matching launches to profile (ncu -c)")
    ap.add_argument("--flops", type=float, default=None, help="algorithmic FLOPs of one call")
    ap.add_argument("--bytes", type=float, default=None, help="algorithmic HBM bytes of one call")
    ap.add_argument("--report", default=None, help="keep the .ncu-rep at this path (without the suffix)")
    ap.add_argument("--out", default=None, help="write a markdown summary here")
    ap.add_argument("cmd", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    cmd = a.cmd[1:] if a.cmd and a.cmd[0] == "--" else a.cmd
    res = profile(cmd, a.kernel, a.skip, a.count, a.report)
    if res["status"] != "ok":
        print(json.dumps({k: res[k] for k in ("status", "unobservable", "log")}))
        return 1
    peaks = load_peaks()
    for g in calls(res["launches"]):
        agg = aggregate(g)
        print(json.dumps(dict(agg, **roofline(agg, a.flops, a.bytes, peaks), unobservable=res["unobservable"])))
    if a.out:
        with open(a.out, "w") as f:
            f.write(summary_markdown(res, cmd, a.flops, a.bytes, peaks))
    return 0


if __name__ == "__main__":
    sys.exit(main())
