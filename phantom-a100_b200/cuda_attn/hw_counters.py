"""Hardware counters of the attention kernels from Nsight Compute, on B200.

The reference's autotune/hw_counters.py (MAPPING 33-76, parse_ncu_csv 105-122, profile 125-156,
aggregate 159-193) mapped GPGPU-Sim counters onto A100 ncu metrics. On B200 the quantities that explain
this path are read directly:

  time          gpu__time_duration.sum                                   kernel duration
  tensor_pipe   sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active   tcgen05 MMA pipe busy %
  mufu_pipe     sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active       ex2 (softmax) pipe %
  fma_pipe      sm__pipe_fma_cycles_active.avg.pct_of_peak_sustained_active
  issue         sm__issue_active.avg.pct_of_peak_sustained_elapsed
  occupancy     sm__warps_active.avg.pct_of_peak_sustained_active
  dram_read / dram_write   dram__bytes_read.sum / dram__bytes_write.sum
  registers     launch__registers_per_thread

and, with the algorithmic counts of the workload, derived figures: achieved TFLOP/s = 4*B*H*N^2*d / time
against the measured bf16 peak at large N, and HBM GB/s = (dram read + write) / time against the measured
copy bandwidth at short N (peaks from MEASURED_PEAKS.json when present).

As in the reference, a metric this ncu does not know is dropped and reported as UNOBSERVABLE instead of
failing the run, and a missing counter permission is reported as status "no_permission". Every ncu run
passes --clock-control none (ncu must not lock the GPU clocks).

    python -m cuda_attn.hw_counters --flops 4.398e12 -- python bench.py --config config4 --steps 2 ...
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import re
import shutil
import subprocess
import sys

UNOBSERVABLE = "UNOBSERVABLE"

MAPPING = {
    "time": "gpu__time_duration.sum",
    "tensor_pipe": "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
    "mufu_pipe": "sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active",
    "fma_pipe": "sm__pipe_fma_cycles_active.avg.pct_of_peak_sustained_active",
    "issue": "sm__issue_active.avg.pct_of_peak_sustained_elapsed",
    "occupancy": "sm__warps_active.avg.pct_of_peak_sustained_active",
    "dram_read": "dram__bytes_read.sum",
    "dram_write": "dram__bytes_write.sum",
    "registers": "launch__registers_per_thread",
}
PERM_ERRORS = ("ERR_NVGPUCTRPERM", "does not have permission", "permission to access NVIDIA GPU Performance Counters")
_BAD_METRIC = re.compile(r"Failed to find metric (\S+)")
_UNIT_SCALE = {"ns": 1e-9, "us": 1e-6, "usecond": 1e-6, "ms": 1e-3, "msecond": 1e-3, "s": 1.0, "nsecond": 1e-9,
               "byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "%": 1.0}


def _num(v: str):
    v = (v or "").replace(",", "").strip()
    if v in ("", "n/a", "N/A"):
        return None
    try:
        return float(v)
    except ValueError:
        return None


def parse_ncu_csv(text: str) -> list[dict]:
    """Parse `ncu --csv --page raw` output (one row per launch, a units row after the header) into one dict
    per launch: {'kernel': name, <metric>: value in base units (seconds, bytes, %)}."""
    lines = text.splitlines()
    start = next((i for i, l in enumerate(lines) if l.startswith('"ID"')), None)
    if start is None:
        return []
    rows = list(csv.reader(io.StringIO("\n".join(lines[start:]))))
    header, units = rows[0], None
    out = []
    for r in rows[1:]:
        if len(r) != len(header):
            continue
        if not r[0].strip().isdigit():
            units = dict(zip(header, r))  # the units row
            continue
        d = dict(zip(header, r))
        k = {"kernel": d.get("Kernel Name", "")}
        for m in MAPPING.values():
            if m in d:
                v = _num(d[m])
                if v is not None and units:
                    v *= _UNIT_SCALE.get(units.get(m, "").strip(), 1.0)
                k[m] = v
        out.append(k)
    return out


def profile(cmd: list[str], kernel_regex: str = "attn_fwd_tc", launch_skip: int = 0, launch_count: int = 1,
            metrics: list[str] | None = None, timeout: int = 900) -> dict:
    """Run `cmd` under ncu for the matching kernel launches. Returns {'status', 'kernels', 'dropped_metrics',
    'log'}; status ok | no_ncu | no_permission | error."""
    ncu = shutil.which("ncu")
    if not ncu:
        return {"status": "no_ncu", "kernels": [], "dropped_metrics": [], "log": ""}
    metrics = list(metrics or MAPPING.values())
    dropped = []
    for _ in range(len(metrics) + 1):
        full = [ncu, "--csv", "--page", "raw", "--print-units", "base", "--clock-control", "none",
                "-k", f"regex:{kernel_regex}",
                "-s", str(launch_skip), "-c", str(launch_count), "--metrics", ",".join(metrics), *cmd]
        p = subprocess.run(full, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, timeout=timeout)
        log = p.stdout
        if any(e in log for e in PERM_ERRORS):
            return {"status": "no_permission", "kernels": [], "dropped_metrics": dropped, "log": log[-2000:]}
        bad = [b.strip(".'\"") for b in _BAD_METRIC.findall(log)]
        bad = [b for b in bad if b in metrics]
        if bad:
            for b in bad:
                metrics.remove(b)
                dropped.append(b)
            if metrics:
                continue
        kernels = parse_ncu_csv(log)
        return {"status": "ok" if kernels else "error", "kernels": kernels, "dropped_metrics": dropped,
                "log": "" if kernels else log[-2000:]}
    return {"status": "error", "kernels": [], "dropped_metrics": dropped, "log": ""}


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


def derive(kernel: dict, flops: float | None = None, algorithmic_bytes: float | None = None,
           peaks: dict | None = None) -> dict:
    """One launch's counters in the mapping's names plus the roofline figures: achieved TFLOP/s and its
    fraction of the bf16 peaks, DRAM GB/s and its fraction of the measured copy bandwidth, and DRAM bytes
    over the algorithmic bytes (above 1 means re-reads)."""
    peaks = peaks or load_peaks()
    out = {}
    for key, metric in MAPPING.items():
        out[key] = kernel.get(metric, None)
        if out[key] is None:
            out[key] = UNOBSERVABLE
    t = kernel.get(MAPPING["time"])
    rd, wr = kernel.get(MAPPING["dram_read"]), kernel.get(MAPPING["dram_write"])
    if t and flops:
        out["tflops"] = flops / t / 1e12
        out["frac_bf16_burst"] = out["tflops"] / peaks["bf16_tflops"]
        out["frac_bf16_sustained"] = out["tflops"] / peaks["bf16_tflops_sustained"]
    if t and rd is not None and wr is not None:
        out["dram_gbs"] = (rd + wr) / t / 1e9
        out["frac_hbm"] = out["dram_gbs"] / peaks["hbm_gbs"]
        if algorithmic_bytes:
            out["traffic_over_algorithmic"] = (rd + wr) / algorithmic_bytes
    out["peaks"] = peaks["kind"]
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--kernel", default="attn_fwd_tc")
    ap.add_argument("--skip", type=int, default=0)
    ap.add_argument("--count", type=int, default=1)
    ap.add_argument("--flops", type=float, default=None, help="algorithmic FLOPs of one launch")
    ap.add_argument("--bytes", type=float, default=None, help="algorithmic HBM bytes of one launch")
    ap.add_argument("cmd", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    cmd = a.cmd[1:] if a.cmd and a.cmd[0] == "--" else a.cmd
    res = profile(cmd, a.kernel, a.skip, a.count)
    if res["status"] != "ok":
        print(json.dumps({k: res[k] for k in ("status", "dropped_metrics", "log")}))
        return 1
    for k in res["kernels"]:
        print(json.dumps(dict(kernel=k["kernel"][:80], **derive(k, a.flops, a.bytes), dropped=res["dropped_metrics"])))
    return 0


if __name__ == "__main__":
    sys.exit(main())
