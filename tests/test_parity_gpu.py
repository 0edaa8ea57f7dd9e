"""GPU parity: the sm_100a kernels, called through the C ABI (libphantom_attn.so via ctypes), against the
CPU oracle on identical seeded inputs.

Criteria (conftest.py): fp32 max-abs 1e-4; fp16/bf16 relative-L2 1e-3 and max-abs 2e-3 beyond one
output ulp, against the float64 oracle rounded to the output dtype. Full-size BASELINE configs are
checked on sampled query rows (rows are independent, so the sampled oracle is exact) plus properties
that hold at any size: every row written and finite, each output inside the convex hull of V's
columns, bit-identical reruns.
"""
import numpy as np
import pytest
import torch

from conftest import assert_parity, make_qkv, torch_dtype_name
from oracle import attention_naive, sampled_rows_naive

pytestmark = pytest.mark.gpu

SMALL_N = [1, 15, 64, 65, 127, 128, 129, 255, 256, 257, 511, 1000]


def np64(t):
    return t.float().cpu().numpy().astype(np.float64)


def run_capi(capi, fn_name, q, k, v, causal=False, **kw):
    o = torch.full_like(q, float("nan"))  # canary: every element must be written
    getattr(capi, fn_name)(q, k, v, o, causal=causal, **kw)
    torch.cuda.synchronize()
    return o


@pytest.fixture(autouse=True)
def _status_clean(cuda_ok, capi):
    yield
    assert capi.device_status() == 0, "a bounded device wait expired"


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("n", SMALL_N)
@pytest.mark.parametrize("causal", [False, True])
def test_fused_tc_matches_oracle(capi, dtype, d, n, causal):
    q, k, v = make_qkv(1, 2, n, d, dtype, seed=n)
    o = run_capi(capi, "fused_tc", q, k, v, causal)
    ref = attention_naive(np64(q), np64(k), np64(v), causal)
    assert_parity(np64(o), ref, torch_dtype_name(dtype), f"fused_tc {dtype} d={d} n={n} causal={causal}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d", [32, 64, 80, 128, 256])
@pytest.mark.parametrize("n", [1, 63, 65, 200])
@pytest.mark.parametrize("fn", ["fused", "naive", "tiled"])
def test_cuda_core_kernel_matches_oracle(capi, dtype, d, n, fn):
    causal = n == 63
    q, k, v = make_qkv(1, 2, n, d, dtype, seed=d + n)
    o = run_capi(capi, fn, q, k, v, causal)
    ref = attention_naive(np64(q), np64(k), np64(v), causal)
    assert_parity(np64(o), ref, torch_dtype_name(dtype), f"{fn} {dtype} d={d} n={n}")


@pytest.mark.parametrize("br,bc", [(64, 32), (64, 64), (128, 32), (128, 64)])
@pytest.mark.parametrize("double_buffer", [False, True])
def test_fused_tuned_tiles_run_the_tensor_core_kernel(capi, br, bc, double_buffer):
    q, k, v = make_qkv(2, 3, 333, 64, torch.float16)
    o = run_capi(capi, "fused_tuned", q, k, v, True, double_buffer=double_buffer, br=br, bc=bc)
    o_tc = run_capi(capi, "fused_tc", q, k, v, True)
    assert torch.equal(o, o_tc)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("scale", [10.0, 30.0])
def test_large_scores_do_not_overflow(capi, dtype, scale):
    q, k, v = make_qkv(1, 2, 256, 64, dtype)
    q, k = (q.float() * scale).to(dtype), (k.float() * scale).to(dtype)
    o = run_capi(capi, "fused_tc", q, k, v)
    assert torch.isfinite(o).all()
    ref = attention_naive(np64(q), np64(k), np64(v))
    assert np.abs(np64(o) - ref).max() < 1e-2 + 2.0 ** -7  # reference tolerance at this scale (+ bf16 ulp)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("growth", [3.0, 10.0])
def test_row_max_growing_mid_sequence(capi, dtype, d, causal, growth):
    """Keys of the second half are `growth` times larger, so every row's running max jumps after the
    first K/V tiles: the kernel must rescale O (accumulated by earlier P.V products) and l before the
    next product, in whichever Q tile and TMEM region holds them."""
    q, k, v = make_qkv(1, 2, 1500, d, dtype, seed=int(growth) * 7 + d)
    k = k.clone()
    k[:, :, 750:] = (k[:, :, 750:].float() * growth).to(dtype)
    o = run_capi(capi, "fused_tc", q, k, v, causal)
    ref = attention_naive(np64(q), np64(k), np64(v), causal)
    assert_parity(np64(o), ref, torch_dtype_name(dtype), f"growth {growth} {dtype} d={d} causal={causal}")


def test_bf16_head_beyond_fp16_range_falls_back_to_bf16_p(capi):
    """A bf16 V value outside the fp16 range makes that head compute P.V in bf16 (finite, looser bound);
    the other heads keep fp16 P and the tight bound."""
    q, k, v = make_qkv(1, 2, 300, 128, torch.bfloat16, seed=5)
    v[0, 1, 17, 3] = 1.0e6
    o = run_capi(capi, "fused_tc", q, k, v)
    ref = attention_naive(np64(q), np64(k), np64(v))
    assert torch.isfinite(o).all()
    assert_parity(np64(o)[:, :1], ref[:, :1], "bfloat16", "head 0 (fp16 P)")
    rel = np.linalg.norm(np64(o)[:, 1] - ref[:, 1]) / np.linalg.norm(ref[:, 1])
    assert rel < 5e-3, rel


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_persistent_ctas_mixed_units(capi, d, causal):
    """160 heads at N = 300: 320 work units (a two-tile and a one-tile query block per head) on at most
    one persistent CTA per SM, so every CTA runs several units of both shapes back to back and its
    barrier phases, K/V ring and TMEM regions carry across unit boundaries."""
    q, k, v = make_qkv(2, 80, 300, d, torch.float16, seed=11 + d)
    o = run_capi(capi, "fused_tc", q, k, v, causal)
    ref = attention_naive(np64(q), np64(k), np64(v), causal)
    assert_parity(np64(o), ref, "float16", f"160 heads d={d} causal={causal}")


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("n", [129, 256])
def test_causal_two_tile_units_back_to_back(capi, d, n):
    """Causal, 400 heads of two Q tiles: every unit has two K/V tiles and tile A runs only the first (the
    second lies after all of A's rows), so B and the issuers can finish a unit while A still writes the
    previous one; several units per persistent CTA. Checks the results and that no bounded wait expired."""
    q, k, v = make_qkv(4, 100, n, d, torch.bfloat16, seed=31 + n + d)
    o = run_capi(capi, "fused_tc", q, k, v, True)
    assert capi.device_status() == 0, "a bounded device wait expired"
    ref = attention_naive(np64(q), np64(k), np64(v), True)
    assert_parity(np64(o), ref, "bfloat16", f"400 heads N={n} d={d} causal")


def test_bf16_fallback_heads_among_fp16_p_heads(capi):
    """Every seventh of 160 bf16 heads holds a V value beyond the fp16 range: the call's main launch
    (fp16 P, fp16-staged V) skips those heads and its second launch computes them with bf16 P and the
    original V; every head must come out right."""
    q, k, v = make_qkv(1, 160, 300, 128, torch.bfloat16, seed=21)
    bad = list(range(0, 160, 7))
    for h in bad:
        v[0, h, (h * 13) % 300, h % 128] = 1.0e6
    o = run_capi(capi, "fused_tc", q, k, v)
    assert torch.isfinite(o).all()
    ref = attention_naive(np64(q), np64(k), np64(v))
    good = [h for h in range(160) if h not in bad]
    assert_parity(np64(o)[:, good], ref[:, good], "bfloat16", "fp16-P heads")
    for h in bad:
        rel = np.linalg.norm(np64(o)[:, h] - ref[:, h]) / np.linalg.norm(ref[:, h])
        assert rel < 5e-3, (h, rel)


@pytest.mark.parametrize("causal", [False, True])
def test_overflow_heads_across_consecutive_calls(capi, causal):
    """bf16 calls that alternate between V with and without fp16-overflowing heads (300 heads at N = 300,
    several units per persistent CTA). A call's second launch must compute exactly its own overflowing
    heads: one without any, made after one with them (its scratch may be the same memory), must leave every
    head to the main launch, and one with them after one without must compute them."""
    q, k, v = make_qkv(1, 300, 300, 128, torch.bfloat16, seed=23)
    bad = list(range(3, 300, 37))
    v_bad = v.clone()
    for h in bad:
        v_bad[0, h, (h * 7) % 300, h % 128] = 2.0e5  # beyond fp16's 65504, exact in bf16
    ref_clean = attention_naive(np64(q), np64(k), np64(v), causal)
    ref_bad = attention_naive(np64(q), np64(k), np64(v_bad), causal)
    good = [h for h in range(300) if h not in bad]
    for call, with_bad in enumerate([True, False, True, False]):
        o = run_capi(capi, "fused_tc", q, k, v_bad if with_bad else v, causal)
        ref = ref_bad if with_bad else ref_clean
        assert_parity(np64(o)[:, good], ref[:, good], "bfloat16", f"call {call}: heads without overflow")
        if with_bad:
            for h in bad:
                rel = np.linalg.norm(np64(o)[:, h] - ref[:, h]) / np.linalg.norm(ref[:, h])
                assert rel < 5e-3, (call, h, rel)
        else:
            assert_parity(np64(o)[:, bad], ref[:, bad], "bfloat16", f"call {call}: formerly overflowing heads")


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("heads,n", [(24, 1000), (20, 300)])
def test_launch_shapes_give_identical_results(capi, d, causal, heads, n):
    """Every launch shape computes each Q tile the same way, so the output is bit-identical to the
    default shape's: one CTA running every unit from the work counter, 7, 11 or 13 CTAs, one head per L2
    group, and all heads in one group (bf16, so the staged-V path runs too). Non-causal shapes whose last
    partial wave is at most half the grid split its query blocks into one-tile units: at N = 1000 on the
    148 CTAs of a B200 and on 5, 7 or 11 CTAs; at N = 300 (an odd tile count) on 7, 11 or 13 CTAs with
    all heads in one group. The others do not. The default result matches the oracle."""
    q, k, v = make_qkv(2, heads, n, d, torch.bfloat16, seed=31 + d + n)
    try:
        capi.set_launch_shape(0, 0)
        capi.set_kv_parts(False)  # every block over its whole K/V range: identical for every shape
        base = run_capi(capi, "fused_tc", q, k, v, causal)
        for kib, ctas in [(0, 1), (0, 7), (0, 11), (0, 13), (1, 0), (1 << 30, 0), (1, 5), (1, 11)]:
            capi.set_launch_shape(kib, ctas)
            assert capi.get_launch_shape() == (kib, ctas)
            o = run_capi(capi, "fused_tc", q, k, v, causal)
            assert torch.equal(o, base), (kib, ctas)
    finally:
        capi.set_launch_shape(0, 0)
        capi.set_kv_parts(True)
    ref = attention_naive(np64(q), np64(k), np64(v), causal)
    assert_parity(np64(base), ref, "bfloat16", f"default launch shape d={d} causal={causal}")


# (B*H, N, d, dtype, persistent-grid cap): launches of few waves whose last partial wave (more than half the
# grid) the library cuts into K/V parts on a B200 (148 SMs): config 4's 8-GPU shard (4 heads: 256 blocks on
# 148 CTAs, 4 parts), the same on a 100-CTA grid (7 parts), 8 heads at N = 8192 (4 parts) and d = 64 on a
# 120-CTA grid (3 parts).
KV_PART_CASES = [(4, 16384, 128, torch.bfloat16, 0), (4, 16384, 128, torch.bfloat16, 100),
                 (8, 8192, 128, torch.float16, 0), (10, 8192, 64, torch.float16, 120)]


@pytest.mark.parametrize("bh,n,d,dtype,cap", KV_PART_CASES)
def test_tail_kv_parts_match_the_oracle(capi, bh, n, d, dtype, cap):
    """The tail's query blocks run as K/V parts whose partial results the last-finishing part merges: the
    output matches the oracle (every row of the first query blocks, where the tail lies, and sampled rows
    elsewhere), differs from the whole-range computation only within tolerance, and is the same on a
    rerun."""
    q, k, v = make_qkv(1, bh, n, d, dtype, scale=0.5 if dtype == torch.bfloat16 else 1.0, seed=90 + n + d)
    try:
        capi.set_launch_shape(0, cap)
        parts = run_capi(capi, "fused_tc", q, k, v)
        again = run_capi(capi, "fused_tc", q, k, v)
        capi.set_kv_parts(False)
        whole = run_capi(capi, "fused_tc", q, k, v)
    finally:
        capi.set_launch_shape(0, 0)
        capi.set_kv_parts(True)
    assert torch.equal(parts, again), "rerun differs"
    assert not torch.equal(parts, whole), "no K/V parts ran (plan did not cut the tail)"
    rng = np.random.default_rng(bh + n)
    rows = np.unique(np.concatenate([np.arange(0, 256), rng.choice(n, 48, replace=False)]))
    for h in sorted({0, bh // 2, bh - 1}):
        ref = sampled_rows_naive(np64(q[0, h]), np64(k[0, h]), np64(v[0, h]), rows)
        assert_parity(np64(parts[0, h])[rows], ref, torch_dtype_name(dtype), f"K/V parts head {h}")
        assert_parity(np64(whole[0, h])[rows], ref, torch_dtype_name(dtype), f"whole range head {h}")


def test_tail_kv_parts_with_a_bf16_fallback_head(capi):
    """A head whose V exceeds the fp16 range (bf16 P) inside a K/V-parted tail: its parts use bf16 P
    throughout and merge to a finite result close to the truth."""
    q, k, v = make_qkv(1, 8, 8192, 128, torch.bfloat16, scale=0.5, seed=95)
    v[0, 7, 77, 5] = 2.0e6
    o = run_capi(capi, "fused_tc", q, k, v)
    assert torch.isfinite(o).all()
    rows = np.arange(0, 256)
    ref = sampled_rows_naive(np64(q[0, 7]), np64(k[0, 7]), np64(v[0, 7]), rows)
    rel = np.linalg.norm(np64(o[0, 7])[rows] - ref) / np.linalg.norm(ref)
    assert rel < 5e-3, rel
    ref6 = sampled_rows_naive(np64(q[0, 6]), np64(k[0, 6]), np64(v[0, 6]), rows)
    assert_parity(np64(o[0, 6])[rows], ref6, "bfloat16", "fp16-P head beside it")


def test_kv_parts_switch_rejects_other_values(capi):
    from cuda_attn.capi import ERR_INVALID
    assert capi.get_kv_parts() is True
    rc = capi.lib.phantom_attn_set_kv_parts(2)
    assert rc == ERR_INVALID and "0 or 1" in capi.last_error()
    assert capi.get_kv_parts() is True


@pytest.mark.parametrize("d", [64, 128])
def test_output_16_byte_but_not_32_byte_aligned(capi, d):
    """The C ABI accepts any 16-byte-aligned O; the epilogue's 32-byte stores are used only when O is
    32-byte aligned, so an output that starts 16 bytes into an allocation is written correctly too (with
    K/V parts as well: 4 heads at N = 16384 cut the tail on a B200)."""
    for bh, n in ((3, 1000), (4, 16384 if d == 128 else 4096)):
        q, k, v = make_qkv(1, bh, n, d, torch.bfloat16, scale=0.5, seed=bh + d)
        base = torch.full((q.numel() + 16,), float("nan"), dtype=q.dtype, device=q.device)
        o = base[8:8 + q.numel()].view(q.shape)  # 8 bf16 = 16 bytes past a 256-byte-aligned start
        assert o.data_ptr() % 32 == 16
        capi.fused_tc(q, k, v, o)
        o_ref = torch.empty_like(q)
        capi.fused_tc(q, k, v, o_ref)
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref), (bh, n)


def test_non_default_stream(capi):
    q, k, v = make_qkv(1, 4, 777, 128, torch.bfloat16, seed=3)
    s = torch.cuda.Stream()
    o = torch.empty_like(q)
    with torch.cuda.stream(s):
        capi.fused_tc(q, k, v, o, stream=s)
    s.synchronize()
    ref = attention_naive(np64(q), np64(k), np64(v))
    assert_parity(np64(o), ref, "bfloat16", "non-default stream")


# (BH, N, d, dtype) of the concurrent launches: each has more work units (query blocks of two 128-row
# tiles) than a B200 has SMs, so its persistent CTAs take units from a work counter while the others run.
CONCURRENT = [(64, 4096, 128, torch.bfloat16), (48, 4096, 128, torch.float16), (96, 2048, 64, torch.float16),
              (80, 2048, 64, torch.bfloat16)]


def test_overlapping_launches_on_four_streams(capi):
    """Multi-wave launches queued on four streams at once overlap on the GPU. Each launch has its own
    work counter (and bf16 staging buffer), so every launch computes all of its query blocks: each output
    equals the same call made alone, bit for bit, and matches the oracle on sampled rows."""
    inputs = [make_qkv(1, bh, n, d, dt, seed=60 + i) for i, (bh, n, d, dt) in enumerate(CONCURRENT)]
    serial = [run_capi(capi, "fused_tc", q, k, v) for q, k, v in inputs]
    streams = [torch.cuda.Stream() for _ in CONCURRENT]
    for rep in range(3):
        outs = [torch.full_like(q, float("nan")) for q, _, _ in inputs]
        torch.cuda.synchronize()
        for s, (q, k, v), o in zip(streams, inputs, outs):
            capi.fused_tc(q, k, v, o, stream=s)  # queued back to back: the four kernels overlap
        torch.cuda.synchronize()
        for i, (o, ref) in enumerate(zip(outs, serial)):
            assert torch.equal(o, ref), f"launch {i} (round {rep}) differs from the serial call"
    rng = np.random.default_rng(5)
    for (q, k, v), o, (bh, n, d, dt) in zip(inputs, serial, CONCURRENT):
        rows = np.unique(np.concatenate([[0, n - 1], rng.choice(n, 24, replace=False)]))
        for h in (0, bh - 1):
            ref = sampled_rows_naive(np64(q[0, h]), np64(k[0, h]), np64(v[0, h]), rows)
            assert_parity(np64(o[0, h])[rows], ref, torch_dtype_name(dt), f"BH={bh} N={n} d={d} head {h}")


def test_two_threads_through_the_host_pipeline(capi):
    """Two host threads run fused_tc_host at once (each on its own three streams): its full chunks (4 heads
    at N = 16384, 6 heads at N = 8192) are 256 and 192 work units, so both threads' kernels use work
    counters concurrently. Each result equals the device-resident call bit for bit."""
    import threading
    import cuda_attn
    jobs = [make_qkv(1, 12, 16384, 128, torch.bfloat16, scale=0.5, seed=70),
            make_qkv(1, 16, 8192, 128, torch.float16, seed=71)]
    expect = [run_capi(capi, "fused_tc", q, k, v).cpu() for q, k, v in jobs]
    host = [[x.cpu().pin_memory() for x in job] for job in jobs]
    results, errors = [None, None], []

    def work(i):
        try:
            for _ in range(2):
                results[i] = cuda_attn.fused_tc_host(*host[i], chunks=3, min_chunk_bytes=0, min_tail_bytes=0)
        except Exception as e:  # reported by the main thread
            errors.append(e)

    threads = [threading.Thread(target=work, args=(i,)) for i in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    for i in range(2):
        assert torch.equal(results[i], expect[i]), f"thread {i} differs from the device-resident call"


def test_host_pipeline_chained_calls_without_synchronising(capi):
    """Back-to-back host calls overlap (the next call's input copies start at once); a call whose input is
    an earlier call's output still being copied back waits for that copy: chaining two layers (O of the
    first as Q of the second) with synchronize=False equals the device-resident chain bit for bit."""
    import cuda_attn
    q, k, v = make_qkv(1, 12, 2048, 128, torch.bfloat16, seed=41)
    o1 = torch.empty_like(q)
    capi.fused_tc(q, k, v, o1)
    o2 = torch.empty_like(q)
    capi.fused_tc(o1, k, v, o2)
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    h1 = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    h2 = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    for _ in range(2):
        cuda_attn.fused_tc_host(hq, hk, hv, out=h1, chunks=4, synchronize=False, min_chunk_bytes=0, min_tail_bytes=0)
        cuda_attn.fused_tc_host(h1, hk, hv, out=h2, chunks=4, synchronize=False, min_chunk_bytes=0, min_tail_bytes=0)
    torch.cuda.synchronize()
    assert torch.equal(h1, o1.cpu()) and torch.equal(h2, o2.cpu())


def test_reruns_are_bit_identical(capi):
    q, k, v = make_qkv(2, 4, 1500, 128, torch.bfloat16, seed=8)
    a = run_capi(capi, "fused_tc", q, k, v, True)
    b = run_capi(capi, "fused_tc", q, k, v, True)
    assert torch.equal(a, b)


# ---------------------------------------------------------------- BASELINE configs at full size
def check_full_size(capi, q, k, v, causal, dtype_name, heads, n_rows=96, seed=0):
    o = run_capi(capi, "fused_tc", q, k, v, causal)
    B, H, N, d = q.shape
    qf, kf, vf, of = (x.reshape(B * H, N, d) for x in (q, k, v, o))
    assert torch.isfinite(of).all(), "unwritten or non-finite output"
    # convex hull: every output element lies within [min_j V[j, c], max_j V[j, c]] of its head
    vmin = vf.float().amin(dim=1, keepdim=True)
    vmax = vf.float().amax(dim=1, keepdim=True)
    slack = 2e-2 * (vmax - vmin).abs() + 1e-3
    assert bool(((of.float() >= vmin - slack) & (of.float() <= vmax + slack)).all()), "output outside hull of V"
    rng = np.random.default_rng(seed)
    for h in heads:
        rows = np.unique(np.concatenate([[0, N - 1], rng.choice(N, size=min(N, n_rows), replace=False)]))
        ref = sampled_rows_naive(np64(qf[h]), np64(kf[h]), np64(vf[h]), rows, causal)
        assert_parity(np64(of[h])[rows], ref, dtype_name, f"head {h} sampled rows")
    return o


def test_config2_full_size(capi):
    from cuda_attn.workloads import CONFIGS, make_inputs
    cfg = CONFIGS["config2"]
    q, k, v = make_inputs(cfg)
    check_full_size(capi, q, k, v, cfg.causal, "float16", heads=[0, 77, 127])


def test_config3_full_size(capi):
    from cuda_attn.workloads import CONFIGS, make_inputs
    cfg = CONFIGS["config3"]
    q, k, v = make_inputs(cfg)
    check_full_size(capi, q, k, v, cfg.causal, "bfloat16", heads=[0, 64, 127])


def test_config4_full_size_with_outliers(capi):
    from cuda_attn.workloads import CONFIGS, make_inputs
    cfg = CONFIGS["config4"]
    q, k, v = make_inputs(cfg)
    check_full_size(capi, q, k, v, cfg.causal, "bfloat16", heads=[0, 31], n_rows=64)


@pytest.mark.parametrize("n", [128, 256, 512, 1024, 2048, 4096, 8192])
@pytest.mark.parametrize("d", [64, 128])
def test_config5_sweep(capi, n, d):
    from cuda_attn.workloads import make_inputs, sweep_config
    cfg = sweep_config(n, d)
    q, k, v = make_inputs(cfg)
    check_full_size(capi, q, k, v, cfg.causal, "float16", heads=[0, 63], n_rows=48)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_causal_full_size(capi, dtype):
    q, k, v = make_qkv(1, 4, 4096, 128, dtype, seed=21)
    check_full_size(capi, q, k, v, True, torch_dtype_name(dtype), heads=[0, 3], n_rows=64)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("chunks", [1, 3, 8])
def test_host_pipeline_equals_device_call(capi, dtype, chunks):
    """fused_tc_host streams head chunks through the GPU; heads are independent, so the result must equal
    the device-resident call bit for bit, for any chunking (including a ragged last chunk; the byte floors
    are turned off so that these small heads are chunked by count)."""
    import cuda_attn
    q, k, v = make_qkv(2, 5, 700, 128, dtype, seed=31)
    o_dev = torch.empty_like(q)
    capi.fused_tc(q, k, v, o_dev, causal=True)
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    o_host = cuda_attn.fused_tc_host(hq, hk, hv, causal=True, chunks=chunks, min_chunk_bytes=0, min_tail_bytes=0)
    assert not o_host.is_cuda and o_host.dtype == dtype
    assert torch.equal(o_host, o_dev.cpu())


def test_host_pipeline_byte_floors_equal_device_call(capi):
    """With the default byte floors, 12 heads of 2 MiB per tensor (N = 8192, d = 128) run as two 6-head
    chunks (a full chunk would need 16 heads for 32 MiB; the halving stops at 4 heads = 8 MiB): the trace
    shows the plan, and the result equals the device-resident call without K/V parts bit for bit (the
    pipeline turns them off; this shape's device call would cut its last wave into parts)."""
    import cuda_attn
    q, k, v = make_qkv(1, 12, 8192, 128, torch.float16, seed=32)
    o_dev = torch.empty_like(q)
    was = capi.get_kv_parts()
    capi.set_kv_parts(False)
    try:
        capi.fused_tc(q, k, v, o_dev)
    finally:
        capi.set_kv_parts(was)
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    trace = []
    o_host = cuda_attn.fused_tc_host(hq, hk, hv, trace=trace)
    assert [r["heads"] for r in trace] == [6, 6]
    assert torch.equal(o_host, o_dev.cpu())
