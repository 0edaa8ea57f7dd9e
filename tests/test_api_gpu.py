"""GPU: the reference's correctness suite (tests/test_correctness.py), run against this package's cuda_attn
API (the PyTorch extension over the C ABI). Same shapes, seeds and tolerances; deliberate differences:
bf16 is accepted by every kernel, the tensor-core kernels also take d = 128, and the CUDA-core kernels
take any d <= 256, so the rejection tests use head dims that remain unsupported."""
import pytest
import torch

from conftest import assert_parity, make_qkv, torch_dtype_name

pytestmark = pytest.mark.gpu

import cuda_attn  # noqa: E402

TOL = {torch.float32: 1e-4, torch.float16: 2e-3}
SHAPES_N = [1, 15, 16, 63, 64, 65, 128, 512, 1000, 1024, 2048]
ALL = list(cuda_attn.KERNELS)


@pytest.fixture(autouse=True)
def _gpu(cuda_ok):
    yield
    assert cuda_attn.device_status() == 0


def check(out, ref, dtype):
    if dtype == torch.bfloat16:
        assert_parity(out.double().cpu().numpy(), ref.double().cpu().numpy(), "bfloat16")
    else:
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= TOL[dtype], f"max abs error {err:.2e} > {TOL[dtype]:.0e}"


def skip_unsupported(name, dtype):
    if dtype == torch.float32 and name in cuda_attn.FP16_ONLY:
        pytest.skip(f"{name} takes 16-bit inputs only")


@pytest.mark.parametrize("name", ALL)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("n", SHAPES_N)
@pytest.mark.parametrize("causal", [False, True])
def test_matches_reference(name, dtype, n, causal):
    skip_unsupported(name, dtype)
    q, k, v = make_qkv(2, 4, n, 64, dtype)
    out = cuda_attn.KERNELS[name](q, k, v, causal)
    torch.cuda.synchronize()
    assert out.shape == q.shape and out.dtype == dtype
    check(out, cuda_attn.reference(q, k, v, causal), dtype)


@pytest.mark.parametrize("br,bc", [(64, 32), (64, 64), (128, 32), (128, 64)])
@pytest.mark.parametrize("double_buffer", [False, True])
@pytest.mark.parametrize("causal", [False, True])
def test_tuned_tile_configs(br, bc, double_buffer, causal):
    q, k, v = make_qkv(2, 3, 333, 64, torch.float16)
    out = cuda_attn.fused_tuned(q, k, v, causal, double_buffer, br, bc)
    check(out, cuda_attn.reference(q, k, v, causal), torch.float16)


@pytest.mark.parametrize("name", ALL)
@pytest.mark.parametrize("scale", [10.0, 30.0])
def test_large_scores_do_not_overflow(name, scale):
    dtype = torch.float16 if name in cuda_attn.FP16_ONLY else torch.float32
    q, k, v = make_qkv(1, 2, 256, 64, dtype)
    q, k = (q.float() * scale).to(dtype), (k.float() * scale).to(dtype)
    out = cuda_attn.KERNELS[name](q, k, v)
    assert torch.isfinite(out).all()
    assert (out.float() - cuda_attn.reference(q, k, v)).abs().max().item() < 1e-2


@pytest.mark.parametrize("d", [64, 128])
def test_long_sequence_fused_versions_agree(d):
    q, k, v = make_qkv(1, 2, 8192, d, torch.float16)
    base = cuda_attn.fused(q, k, v).float()
    for name in ("fused_vec", "fused_db", "fused_tc"):
        assert (cuda_attn.KERNELS[name](q, k, v).float() - base).abs().max().item() < 2e-3, name


@pytest.mark.parametrize("name", ["naive", "tiled", "fused"])
@pytest.mark.parametrize("d", [32, 80, 128])
def test_other_head_dims_for_cuda_core_kernels(name, d):
    q, k, v = make_qkv(1, 2, 200, d, torch.float32)
    check(cuda_attn.KERNELS[name](q, k, v), cuda_attn.reference(q, k, v), torch.float32)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_tensor_core_head_dims(d, dtype):
    q, k, v = make_qkv(2, 2, 300, d, dtype)
    out = cuda_attn.fused_tc(q, k, v)
    assert_parity(out.double().cpu().numpy(), cuda_attn.reference(q, k, v).double().cpu().numpy(),
                  torch_dtype_name(dtype))


@pytest.mark.parametrize("name", ["fused_vec", "fused_tc"])
@pytest.mark.parametrize("d", [32, 96, 256])
def test_tensor_core_kernels_reject_unsupported_head_dim(name, d):
    q, k, v = make_qkv(1, 1, 64, d, torch.float16)
    with pytest.raises(RuntimeError, match="head dimension"):
        cuda_attn.KERNELS[name](q, k, v)


def test_cuda_core_kernels_reject_unsupported_head_dim():
    q, k, v = make_qkv(1, 1, 16, 512, torch.float32)
    with pytest.raises(RuntimeError, match="head dimension"):
        cuda_attn.fused(q, k, v)


def test_fp16_only_kernels_reject_fp32():
    q, k, v = make_qkv(1, 1, 64, 64, torch.float32)
    for name in cuda_attn.FP16_ONLY:
        with pytest.raises(RuntimeError, match="float16"):
            cuda_attn.KERNELS[name](q, k, v)


def test_input_validation():
    q, k, v = make_qkv(1, 1, 64, 64, torch.float16)
    with pytest.raises(RuntimeError, match="contiguous"):
        cuda_attn.fused(q.transpose(2, 3), k, v)
    with pytest.raises(RuntimeError, match="dtype"):
        cuda_attn.fused(q, k.float(), v)
    with pytest.raises(RuntimeError, match="not compiled"):
        cuda_attn.fused_tuned(q, k, v, br=32, bc=32)
    with pytest.raises(RuntimeError, match="same shape"):
        cuda_attn.fused_tc(q, k[:, :, :32].contiguous(), v)


def test_misaligned_pointer_rejected():
    base = torch.zeros(1 * 1 * 64 * 64 + 4, device="cuda", dtype=torch.float16)
    q = base[4:].view(1, 1, 64, 64)  # 8-byte offset
    with pytest.raises(RuntimeError, match="16-byte aligned"):
        cuda_attn.fused_tc(q, q, q)


def test_sweep_tool_writes_gated_rows(tmp_path):
    """cuda_attn.sweep (the reference's bench/benchmark.py on B200): every row passes the correctness gate."""
    import csv
    from cuda_attn import sweep
    out = tmp_path / "s.csv"
    assert sweep.main(["--ns", "128", "640", "--dims", "64", "128", "--heads", "4", "--iters", "3", "--warmup", "1",
                       "--impls", "fused_tc", "fused", "--out", str(out)]) == 0
    rows = list(csv.DictReader(open(out)))
    assert len(rows) == 8 and all(r["status"] == "ok" for r in rows), rows
    # peak memory of one call: at least O (B*H*N*d fp16 elements; the sweep's default dtype)
    for r in rows:
        o_mb = 4 * int(r["N"]) * int(r["d"]) * 2 / 2**20
        assert float(r["peak_memory_mb"]) >= o_mb - 1e-3, r


def test_scratch_bytes_report_the_pool_high_water_mark():
    """phantom_attn_scratch_bytes: a bf16 call takes the fp16 copy of V (2*B*H*N*d bytes) plus flags and, when
    its launch has several waves, the work counter from the library pool; the high-water mark covers that
    and restarts on reset; a one-wave fp16 call takes no scratch."""
    from cuda_attn.capi import CAPI
    lib = CAPI()
    q = torch.randn(1, 8, 2048, 128, device="cuda").to(torch.bfloat16)
    o = torch.empty_like(q)
    lib.fused_tc(q, q, q, o)
    torch.cuda.synchronize()
    lib.scratch_bytes(reset=True)
    lib.fused_tc(q, q, q, o)
    torch.cuda.synchronize()
    hw, reserved = lib.scratch_bytes(reset=True)
    assert hw >= 2 * q.numel() and reserved >= hw, (hw, reserved)
    h = torch.randn(1, 2, 256, 64, device="cuda").half()
    lib.fused_tc(h, h, h, torch.empty_like(h))
    torch.cuda.synchronize()
    assert lib.scratch_bytes()[0] == 0


def test_run_one_and_timeline_tools():
    """cuda_attn.run_one (a fixed profiling target) runs; cuda_attn.timeline orders every chunk's stages
    (input copy, attention, output copy) and accounts for every head of every call."""
    from cuda_attn import run_one, timeline
    assert run_one.main(["--impl", "fused_tc", "--n", "512", "--dim", "128", "--dtype", "bf16", "--reps", "2"]) == 0
    summary, rows = timeline.run("config2", chunks=4, calls=2, warmup=1)
    assert summary["ms_per_call"] > 0 and summary["h2d_gbs_while_busy"] > 1
    from cuda_attn.workloads import CONFIGS
    assert sum(r["heads"] for r in rows) == 2 * CONFIGS["config2"].BH
    for r in rows:
        assert r["h2d"][0] <= r["h2d"][1] <= r["attend"][0] + 1e-3
        assert r["attend"][0] <= r["attend"][1] <= r["d2h"][0] + 1e-3 and r["d2h"][0] <= r["d2h"][1]
