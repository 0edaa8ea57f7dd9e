"""CPU: the measurement tooling (cuda_attn.hw_counters, the B200 counterpart of the reference's
autotune/hw_counters.py): metric pre-flight against the chip list, the ncu command line, reading a report
through a reader object, grouping launches into calls, aggregation and roofline figures - on fakes, and
on Nsight Compute's own sample report where the image has one."""
import glob
import os
import subprocess

import pytest

from cuda_attn import hw_counters as hc

T, TENSOR, DR, DW, REGS = ("gpu__time_duration.sum", "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
                           "dram__bytes_read.sum", "dram__bytes_write.sum", "launch__registers_per_thread")
PEAKS = {"bf16_tflops": 1662.3, "bf16_tflops_sustained": 1395.6, "hbm_gbs": 6556.5, "kind": "measured"}


def launch(kernel, t_ns, tensor=None, rd=None, wr=None, regs=None):
    rec = {"kernel": kernel}
    rec.update({T: t_ns, TENSOR: tensor, DR: rd, DW: wr, REGS: regs})
    return rec


def test_split_metrics_keeps_known_and_launch_stats():
    known = {"gpu__time_duration", "dram__bytes_read"}
    keep, missing = hc.split_metrics([T, DR, TENSOR, REGS], known)
    assert keep == [T, DR, REGS] and missing == [TENSOR]
    assert hc.split_metrics([T, TENSOR], None) == ([T, TENSOR], [])


def test_ncu_command_never_locks_clocks_and_writes_a_report():
    cmd = hc.ncu_command(["python", "bench.py"], "/tmp/r", [T, DR], "attn_fwd_tc", 3, 2)
    assert cmd[cmd.index("--clock-control") + 1] == "none"
    assert cmd[cmd.index("-o") + 1] == "/tmp/r"
    assert cmd[cmd.index("-s") + 1] == "3" and cmd[cmd.index("-c") + 1] == "2"
    assert cmd[-2:] == ["python", "bench.py"]


class _Metric:
    def __init__(self, v):
        self.v = v

    def as_double(self):
        return self.v


class _Action:
    def __init__(self, name, values):
        self._name, self._values = name, values

    def name(self):
        return self._name

    def metric_by_name(self, m):
        return _Metric(self._values[m]) if m in self._values else None


class _Range:
    def __init__(self, actions):
        self.actions = actions

    def num_actions(self):
        return len(self.actions)

    def action_by_idx(self, i):
        return self.actions[i]


class _Reader:
    def __init__(self, actions):
        self.actions = actions

    def load_report(self, path):
        rng = _Range(self.actions)

        class Ctx:
            def num_ranges(self):
                return 1

            def range_by_idx(self, i):
                return rng
        return Ctx()


def test_read_report_through_a_reader_object():
    reader = _Reader([_Action("tc::stage_v_f16(...)", {T: 66000.0, DR: 1.34e8}),
                      _Action("tc::attn_fwd_tc<128, true>(...)", {T: 3.2e6, DR: 4.0e8, TENSOR: 73.2})])
    recs = hc.read_report("x.ncu-rep", [T, DR, TENSOR], reader)
    assert [r["kernel"][:6] for r in recs] == ["tc::st", "tc::at"]
    assert recs[0][TENSOR] is None and recs[1][TENSOR] == 73.2


def test_calls_group_staging_with_the_attention_kernel():
    ls = [launch("tc::stage_v_f16", 1), launch("tc::attn_fwd_tc<128, true>", 2), launch("tc::attn_fwd_tc<64, false>", 3),
          launch("tc::stage_v_f16", 4)]
    groups = hc.calls(ls)
    assert [[r[T] for r in g] for g in groups] == [[1, 2], [3]]


def test_calls_attach_the_overflow_heads_launch():
    # a bf16 call: staging, main launch, K/V-part merge, the launch for fp16-overflow heads; then an fp16 call
    ls = [launch("stage_v_f16", 1), launch("void attn_fwd_tc<128, 1, 1, 0>(...)", 2),
          launch("void merge_kv_parts<128, 1>(...)", 3), launch("void attn_fwd_tc<128, 1, 0, 1>(...)", 4),
          launch("void attn_fwd_tc<64, 0, 0, 0>(...)", 5)]
    assert [[r[T] for r in g] for g in hc.calls(ls)] == [[1, 2, 3, 4], [5]]
    assert hc.is_overflow_launch("attn_fwd_tc<128, true, false, true>")
    assert not hc.is_overflow_launch("attn_fwd_tc<128, true, false, false>") and not hc.is_overflow_launch("stage_v_f16")


def test_calls_start_an_fp16_call_at_its_counter_zeroing():
    ls = [launch("tc::zero_counter(int*)", 1), launch("void attn_fwd_tc<64, 0, 0, 0>(...)", 2),
          launch("void attn_fwd_tc<64, 0, 0, 0>(...)", 3)]
    assert [[r[T] for r in g] for g in hc.calls(ls)] == [[1, 2], [3]]


def test_calls_attach_the_merge_of_k_v_parts():
    ls = [launch("tc::stage_v_f16", 1), launch("tc::attn_fwd_tc<128, true, true>", 2),
          launch("tc::merge_kv_parts<128, true>", 3), launch("tc::attn_fwd_tc<128, false, false>", 4)]
    assert [[r[T] for r in g] for g in hc.calls(ls)] == [[1, 2, 3], [4]]


def test_aggregate_sums_weights_and_takes_the_longest():
    g = [launch("tc::stage_v_f16", 1.0e5, tensor=0.0, rd=1.0e8, wr=1.0e8, regs=38),
         launch("tc::attn_fwd_tc", 3.0e6, tensor=70.0, rd=4.0e8, wr=1.2e8, regs=168)]
    a = hc.aggregate(g)
    assert a["time_s"] == pytest.approx(3.1e-3)
    assert a["dram_read"] == pytest.approx(5.0e8) and a["dram_write"] == pytest.approx(2.2e8)
    assert a["tensor_pct"] == pytest.approx(70.0 * 3.0e6 / 3.1e6)
    assert a["registers"] == 168
    assert a["mufu_pct"] == hc.UNOBSERVABLE  # not captured


def test_aggregate_marks_a_partly_missing_sum_unobservable():
    a = hc.aggregate([launch("a", 1.0e5, rd=1.0), launch("tc::attn_fwd_tc", 2.0e5, rd=None)])
    assert a["dram_read"] == hc.UNOBSERVABLE


def test_roofline_figures():
    a = hc.aggregate([launch("tc::attn_fwd_tc", 3.2e6, rd=4.0e8, wr=1.2e8)])
    r = hc.roofline(a, flops=4.398046511104e12, algorithmic_bytes=536870912.0, peaks=PEAKS)
    assert r["tflops"] == pytest.approx(4.398046511104e12 / 3.2e-3 / 1e12)
    assert r["frac_bf16_burst"] == pytest.approx(r["tflops"] / 1662.3)
    assert r["traffic_over_algorithmic"] == pytest.approx(5.2e8 / 536870912.0)
    assert r["dram_gbs"] == pytest.approx(5.2e8 / 3.2e-3 / 1e9)


def test_profile_without_ncu(monkeypatch):
    monkeypatch.setattr(hc.shutil, "which", lambda name: None)
    assert hc.profile(["true"])["status"] == "no_ncu"


def test_profile_reports_missing_permission(monkeypatch, tmp_path):
    monkeypatch.setattr(hc.shutil, "which", lambda name: "/usr/bin/ncu")
    monkeypatch.setattr(hc, "chip_metrics", lambda chip, ncu=None: None)
    runs = []

    def fake_run(cmd, **kw):
        runs.append(cmd)
        return subprocess.CompletedProcess(cmd, 1, stdout="==ERROR== ERR_NVGPUCTRPERM - no access")
    monkeypatch.setattr(hc.subprocess, "run", fake_run)
    res = hc.profile(["true"], report=str(tmp_path / "r"))
    assert res["status"] == "no_permission"
    assert len(runs) == 1 and "--clock-control" in runs[0]


def test_profile_leaves_unknown_metrics_out_of_the_capture(monkeypatch, tmp_path):
    monkeypatch.setattr(hc.shutil, "which", lambda name: "/usr/bin/ncu")
    monkeypatch.setattr(hc, "chip_metrics", lambda chip, ncu=None: {"gpu__time_duration", "dram__bytes_read",
                                                                     "dram__bytes_write"})
    seen = {}

    def fake_run(cmd, **kw):
        seen["metrics"] = cmd[cmd.index("--metrics") + 1].split(",")
        open(cmd[cmd.index("-o") + 1] + ".ncu-rep", "w").close()
        return subprocess.CompletedProcess(cmd, 0, stdout="")
    monkeypatch.setattr(hc.subprocess, "run", fake_run)
    monkeypatch.setattr(hc, "report_reader", lambda: _Reader([_Action("tc::attn_fwd_tc", {T: 1.0e6})]))
    res = hc.profile(["true"], report=str(tmp_path / "r"))
    assert res["status"] == "ok"
    assert TENSOR in res["unobservable"] and TENSOR not in seen["metrics"] and T in seen["metrics"]
    assert hc.aggregate(hc.calls(res["launches"])[0])["time_s"] == pytest.approx(1.0e-3)


def test_chip_list_of_the_installed_ncu():
    names = hc.chip_metrics("gb100")
    if names is None:
        pytest.skip("ncu cannot list gb100 metrics here")
    for c in hc.COUNTERS:
        assert c.metric.startswith("launch__") or hc.base_name(c.metric) in names, c.metric


def test_read_nsight_compute_sample_report():
    reader = hc.report_reader()
    extras = os.path.dirname(os.path.dirname(os.path.abspath(reader.__file__))) if reader else ""
    samples = sorted(glob.glob(os.path.join(extras, "samples", "*", "*.ncu-rep")))
    if reader is None or not samples:
        pytest.skip("no ncu_report module or sample report in this image")
    recs = hc.read_report(samples[0], [T, DR], reader)
    assert recs and recs[0][T] > 0 and recs[0][DR] > 0


def test_tools_at_the_reference_paths():
    """The reference runs its tools as `python bench/benchmark.py`, `bench/sweep_tiles.py`, `bench/run_one.py`
    from its root and imports `autotune.hw_counters`; the same paths under phantom-a100_b200/ reach this
    library's implementations."""
    import sys
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "phantom-a100_b200")
    for script, word in (("bench/benchmark.py", "--impls"), ("bench/sweep_tiles.py", "--dim"),
                         ("bench/run_one.py", "--impl")):
        r = subprocess.run([sys.executable, script, "--help"], cwd=pkg, capture_output=True, text=True, timeout=600)
        assert r.returncode == 0 and word in r.stdout, (script, r.stderr[-500:])
    from autotune import hw_counters as at
    assert at is hc
