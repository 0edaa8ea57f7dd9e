"""Shared test setup: import paths, the `gpu` marker, seeded input generation and parity checks.

Parity criteria (the reference's tolerances, tests/test_correctness.py:12 and BASELINE north star):
  * fp32 outputs:  max |out - ref| <= 1e-4 against the float64 oracle.
  * fp16 / bf16 outputs (fp32 accumulation): relative-L2 <= 1e-3 and max |out - ref| <= 2e-3 + ulp,
    where ref is the float64 oracle rounded to the output dtype and ulp is that dtype's spacing at
    |ref| (a correctly computed value may round to the neighbouring 16-bit number). With ulp = 0 this
    is the reference's 2e-3 max-abs bound; the allowance matters for bf16 (8 bits of mantissa), whose
    rounding alone exceeds 2e-3 once |O| > 0.5.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "phantom-a100_b200")
for p in (PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

TOL_FP32 = 1e-4
TOL_MAXABS_16 = 2e-3
TOL_RELL2_16 = 1e-3
MANTISSA_BITS = {"float16": 10, "bfloat16": 7}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA GPUs")


def torch_dtype_name(dtype) -> str:
    return str(dtype).replace("torch.", "")


def make_qkv(b, h, n, d, dtype, scale=1.0, seed=0, device="cuda"):
    """Seeded inputs as in the reference tests (test_correctness.py:17-20): fp32 randn * scale, then cast."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    return [(torch.randn(b, h, n, d, device=device, dtype=torch.float32, generator=g) * scale).to(dtype)
            for _ in range(3)]


def ulp(x: np.ndarray, dtype_name: str) -> np.ndarray:
    """Spacing of a 16-bit float format at |x| (normal range)."""
    bits = MANTISSA_BITS[dtype_name]
    ax = np.maximum(np.abs(x), np.float32(2.0 ** -14))
    return np.exp2(np.floor(np.log2(ax)) - bits)


def parity_errors(out: np.ndarray, ref64: np.ndarray, dtype_name: str) -> dict:
    """Error figures of a kernel output against the float64 oracle."""
    from oracle import round_to
    out = np.asarray(out, dtype=np.float64)
    res = {"max_abs_raw": float(np.abs(out - ref64).max()) if out.size else 0.0}
    if dtype_name == "float32":
        res["max_abs"] = res["max_abs_raw"]
        return res
    ref_r = round_to(ref64.astype(np.float32), dtype_name).astype(np.float64)
    diff = np.abs(out - ref_r)
    res["max_abs"] = float(diff.max())
    res["max_excess"] = float((diff - ulp(ref_r, dtype_name)).max())
    den = float(np.linalg.norm(ref_r))
    res["rel_l2"] = float(np.linalg.norm(out - ref_r) / den) if den > 0 else float(np.linalg.norm(out))
    return res


def assert_parity(out: np.ndarray, ref64: np.ndarray, dtype_name: str, what: str = "") -> dict:
    e = parity_errors(out, ref64, dtype_name)
    assert np.isfinite(np.asarray(out, dtype=np.float64)).all(), f"{what}: non-finite output"
    if dtype_name == "float32":
        assert e["max_abs"] <= TOL_FP32, f"{what}: max abs error {e['max_abs']:.2e} > {TOL_FP32:.0e}"
    else:
        assert e["rel_l2"] <= TOL_RELL2_16, f"{what}: relative L2 {e['rel_l2']:.2e} > {TOL_RELL2_16:.0e} ({e})"
        assert e["max_excess"] <= TOL_MAXABS_16, f"{what}: max abs error beyond one ulp {e['max_excess']:.2e} ({e})"
    return e


@pytest.fixture(scope="session")
def cuda_ok():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return True


@pytest.fixture(scope="session")
def capi():
    from cuda_attn.capi import CAPI
    return CAPI()
