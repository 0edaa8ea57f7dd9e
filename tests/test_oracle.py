"""CPU: the oracle against the reference's own outputs (golden vectors) and the reference's algorithm tests.

The golden .npz files were produced by tests/golden/make_golden.py from b4batunde/Phantom-A100's
cuda_attn/online_softmax_ref.py and cuda_attn.reference; passing here pins oracle/ to the reference.
"""
import glob
import os

import numpy as np
import pytest

from oracle import attention_naive, attention_online, reference_sdpa, round_to, sampled_rows_naive

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
PIN = 2e-6  # float32 storage of the golden outputs


def load(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    d = {k: z[k] for k in z.files}
    for t in ("q", "k", "v"):
        if f"{t}_bf16bits" in d:
            d[t] = (d.pop(f"{t}_bf16bits").astype(np.uint32) << 16).view(np.float32)
        elif d[t].dtype == np.float16:
            d[t] = d[t].astype(np.float32)
    return d


def test_golden_files_present():
    names = {os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz"))}
    assert {"config1", "tiles", "scale10", "fp16p", "bf16_d128", "outlier"} <= names
    assert {f"n{n}_c{c}" for n in (1, 31, 65, 257) for c in (0, 1)} <= names


@pytest.mark.parametrize("name", [f"n{n}_c{c}" for n in (1, 31, 65, 257) for c in (0, 1)] + ["config1"])
def test_oracle_matches_reference_outputs(name):
    g = load(name)
    c = bool(g["causal"])
    np.testing.assert_allclose(attention_naive(g["q"], g["k"], g["v"], c), g["naive"], atol=PIN, rtol=0)
    np.testing.assert_allclose(attention_online(g["q"], g["k"], g["v"], c), g["online"], atol=PIN, rtol=0)
    np.testing.assert_allclose(reference_sdpa(g["q"], g["k"], g["v"], c), g["sdpa"], atol=PIN, rtol=0)


def test_config1_checksum_over_all_heads():
    """BASELINE config 1 in full (B=1, H=42, N=128, d=64): per-head output sums of all 42 heads."""
    g = load("config1")
    rng = np.random.default_rng(20240101)
    q, k, v = (rng.standard_normal((1, 42, 128, 64)).astype(np.float32) for _ in range(3))
    np.testing.assert_array_equal(q[:, :2], g["q"])  # generator stream unchanged
    o = attention_naive(q, k, v, False)
    np.testing.assert_allclose(o.sum(axis=(-1, -2)), g["head_sums_naive"], atol=1e-4, rtol=1e-6)
    np.testing.assert_allclose((o ** 2).sum(axis=(-1, -2)), g["head_sumsq_naive"], rtol=1e-6)


@pytest.mark.parametrize("br,bc", [(16, 16), (64, 32), (128, 64)])
def test_oracle_tile_shapes_match_reference(br, bc):
    g = load("tiles")
    out = attention_online(g["q"], g["k"], g["v"], True, br, bc)
    np.testing.assert_allclose(out, g[f"online_{br}_{bc}"], atol=PIN, rtol=0)
    np.testing.assert_allclose(out, g["naive"], atol=1e-5, rtol=1e-4)


def test_oracle_large_scores_match_reference():
    g = load("scale10")
    np.testing.assert_allclose(attention_online(g["q"], g["k"], g["v"]), g["online"], atol=PIN, rtol=0)
    np.testing.assert_allclose(attention_naive(g["q"], g["k"], g["v"]), g["naive"], atol=PIN, rtol=0)


def test_oracle_fp16_p_model_matches_reference():
    g = load("fp16p")
    out = attention_online(g["q"], g["k"], g["v"], False, br=64, bc=64, p_dtype="float16")
    np.testing.assert_allclose(out, g["online_p16"], atol=PIN, rtol=0)


@pytest.mark.parametrize("name", ["bf16_d128", "outlier"])
def test_oracle_bf16_cases_match_reference(name):
    g = load(name)
    np.testing.assert_allclose(attention_naive(g["q"], g["k"], g["v"]), g["naive"], atol=PIN, rtol=0)
    if "naive_causal" in g:
        np.testing.assert_allclose(attention_naive(g["q"], g["k"], g["v"], True), g["naive_causal"], atol=PIN)
    if "online" in g:
        np.testing.assert_allclose(attention_online(g["q"], g["k"], g["v"]), g["online"], atol=PIN, rtol=0)


# ---- the reference's algorithm tests (tests/test_algorithm.py), restated against this oracle
@pytest.mark.parametrize("n", [1, 31, 32, 63, 64, 65, 100, 257])
@pytest.mark.parametrize("causal", [False, True])
def test_online_matches_naive(n, causal):
    rng = np.random.default_rng(n)
    q, k, v = (rng.standard_normal((2, 3, n, 64)).astype(np.float32) for _ in range(3))
    np.testing.assert_allclose(attention_online(q, k, v, causal), attention_naive(q, k, v, causal),
                               atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("scale", [10.0, 100.0])
def test_online_is_stable_for_large_scores(scale):
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 1, 200, 64)).astype(np.float32) for _ in range(3))
    out = attention_online(q * scale, k * scale, v)
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out, attention_naive(q * scale, k * scale, v), atol=1e-4, rtol=1e-3)


@pytest.mark.parametrize("n", [1, 64, 65, 1000])
@pytest.mark.parametrize("causal", [False, True])
def test_fp16_p_stays_within_test_tolerance(n, causal):
    rng = np.random.default_rng(7)
    q, k, v = (rng.standard_normal((1, 2, n, 64)).astype(np.float16).astype(np.float32) for _ in range(3))
    out = round_to(attention_online(q, k, v, causal, br=64, bc=64, p_dtype="float16"), "float16")
    assert np.abs(out - attention_naive(q, k, v, causal)).max() <= 2e-3


def test_bf16_inputs_need_fp16_p():
    """Budget of the tensor-core kernel's P.V precision for bf16 inputs (d=128, BN=128 tiles): rounding P
    to bf16 alone exceeds the 1e-3 relative-L2 bound, rounding it to fp16 fits. This is why the kernel
    stages V as fp16 for bf16 inputs."""
    from conftest import parity_errors
    rng = np.random.default_rng(3)
    q, k, v = (round_to(rng.standard_normal((1, 2, 1024, 128)).astype(np.float32), "bf16") for _ in range(3))
    ref = attention_naive(q, k, v)
    e_bf = parity_errors(round_to(attention_online(q, k, v, br=128, bc=128, p_dtype="bfloat16"), "bf16"),
                         ref, "bfloat16")
    e_fp = parity_errors(round_to(attention_online(q, k, v, br=128, bc=128, p_dtype="float16"), "bf16"),
                         ref, "bfloat16")
    assert e_bf["rel_l2"] > 1.5e-3
    assert e_fp["rel_l2"] < 1e-3


def test_round_to_matches_torch():
    import torch
    x = np.random.default_rng(5).standard_normal(10000).astype(np.float32) * 100
    for name, td in (("bfloat16", torch.bfloat16), ("float16", torch.float16)):
        np.testing.assert_array_equal(round_to(x, name), torch.from_numpy(x).to(td).float().numpy())


@pytest.mark.parametrize("causal", [False, True])
def test_sampled_rows_equal_full(causal):
    rng = np.random.default_rng(9)
    q, k, v = (rng.standard_normal((1, 2, 150, 32)).astype(np.float32) for _ in range(3))
    rows = np.array([0, 7, 64, 149])
    np.testing.assert_allclose(sampled_rows_naive(q, k, v, rows, causal),
                               attention_naive(q, k, v, causal)[..., rows, :], atol=1e-12)
