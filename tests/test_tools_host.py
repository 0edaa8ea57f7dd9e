"""CPU: the measurement tooling - ncu counter parsing and roofline derivation (cuda_attn.hw_counters, the
B200 counterpart of the reference's autotune/hw_counters.py) - on synthetic ncu output and fakes."""
import subprocess

import pytest

from cuda_attn import hw_counters as hc

CSV = '''==PROF== Connected to process 1
"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","gpu__time_duration.sum","sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active","dram__bytes_read.sum","dram__bytes_write.sum","launch__registers_per_thread"
"","","","","","","","nsecond","%","byte","byte","register/thread"
"0","7","python","box","void phantom::tc::attn_fwd_tc<128, true>(...)","1","7","3508512","63.47","403596544","114652416","168"
'''


def test_parse_ncu_csv_scales_units():
    ks = hc.parse_ncu_csv(CSV)
    assert len(ks) == 1
    k = ks[0]
    assert "attn_fwd_tc" in k["kernel"]
    assert k["gpu__time_duration.sum"] == pytest.approx(3.508512e-3)
    assert k["dram__bytes_read.sum"] == pytest.approx(403596544)
    assert k["sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active"] == pytest.approx(63.47)


def test_parse_other_units():
    text = CSV.replace('"nsecond"', '"msecond"').replace('"3508512"', '"3.508512"').replace('"byte","byte"', '"Mbyte","Mbyte"')
    text = text.replace('"403596544","114652416"', '"403.596544","114.652416"')
    k = hc.parse_ncu_csv(text)[0]
    assert k["gpu__time_duration.sum"] == pytest.approx(3.508512e-3)
    assert k["dram__bytes_write.sum"] == pytest.approx(114652416)


def test_derive_roofline_figures():
    k = hc.parse_ncu_csv(CSV)[0]
    peaks = {"bf16_tflops": 1652.7, "bf16_tflops_sustained": 1411.6, "hbm_gbs": 6550.4, "kind": "measured"}
    d = hc.derive(k, flops=4.398046511104e12, algorithmic_bytes=536870912.0, peaks=peaks)
    assert d["tflops"] == pytest.approx(4.398046511104e12 / 3.508512e-3 / 1e12)
    assert d["frac_bf16_sustained"] == pytest.approx(d["tflops"] / 1411.6)
    assert d["traffic_over_algorithmic"] == pytest.approx((403596544 + 114652416) / 536870912.0)
    assert d["mufu_pipe"] == hc.UNOBSERVABLE  # not in this capture


def test_profile_without_ncu(monkeypatch):
    monkeypatch.setattr(hc.shutil, "which", lambda name: None)
    assert hc.profile(["true"])["status"] == "no_ncu"


class _Run:
    def __init__(self, outs):
        self.outs, self.calls = list(outs), []

    def __call__(self, cmd, **kw):
        self.calls.append(cmd)
        return subprocess.CompletedProcess(cmd, 0, stdout=self.outs.pop(0))


def test_profile_reports_missing_permission(monkeypatch):
    monkeypatch.setattr(hc.shutil, "which", lambda name: "/usr/bin/ncu")
    monkeypatch.setattr(hc.subprocess, "run", _Run(["==ERROR== ERR_NVGPUCTRPERM - no access"]))
    assert hc.profile(["true"])["status"] == "no_permission"


def test_profile_drops_unknown_metric_and_retries(monkeypatch):
    monkeypatch.setattr(hc.shutil, "which", lambda name: "/usr/bin/ncu")
    bad = "sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active"
    run = _Run([f"==ERROR== Failed to find metric {bad}", CSV])
    monkeypatch.setattr(hc.subprocess, "run", run)
    res = hc.profile(["true"])
    assert res["status"] == "ok" and res["dropped_metrics"] == [bad]
    assert bad not in run.calls[1][run.calls[1].index("--metrics") + 1]
    assert "--clock-control" in run.calls[0] and run.calls[0][run.calls[0].index("--clock-control") + 1] == "none"
