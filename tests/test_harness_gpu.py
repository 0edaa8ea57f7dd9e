"""GPU: the torch-free C harness (tests/harness/attn_harness) drives the C ABI directly - seeded inputs,
cudaMalloc'd buffers, one call, a float64 CPU check (oracle/ref64.c) - as the reference's sim/harness.cu
drove its launchers. Each case must print a PASS RESULT line."""
import os
import re
import subprocess

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [
    "fused_tc 4 300 64 f16 0",
    "fused_tc 2 513 128 bf16 1",
    "fused_tc 1 1 128 f16 0",
    "fused_tc_noalloc 3 700 128 bf16 0",
    "fused_tuned:128:64:1 2 257 64 f16 1",
    "fused 2 100 80 f32 0",
    "naive 1 65 32 f32 1",
    "tiled 2 129 256 bf16 0",
]


@pytest.fixture(scope="module")
def harness(cuda_ok):
    import importlib.util
    spec = importlib.util.spec_from_file_location("harness_build", os.path.join(HERE, "harness", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build()


@pytest.mark.parametrize("case", CASES)
def test_harness_case_passes(harness, case):
    p = subprocess.run([harness, *case.split()], capture_output=True, text=True, timeout=300)
    line = next((l for l in p.stdout.splitlines() if l.startswith("RESULT")), "")
    assert "status=PASS" in line, (p.returncode, p.stdout, p.stderr)
    assert p.returncode == 0


def test_harness_timing_line(harness):
    env = dict(os.environ, HARNESS_ITERS="5")
    p = subprocess.run([harness, "fused_tc", "16", "2048", "128", "bf16", "0"], capture_output=True, text=True,
                       timeout=300, env=env)
    m = re.search(r"TIME .*median_ms=([0-9.]+).*tflops=([0-9.]+)", p.stdout)
    assert m and float(m.group(1)) > 0, p.stdout
