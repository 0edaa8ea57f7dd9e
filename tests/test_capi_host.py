"""CPU: the C-ABI library loads, exports every symbol include/phantom_attn.h declares, and rejects bad
arguments with the reference's error texts before touching a GPU. The Python API mirrors the
reference's names."""
import ctypes
import os

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "phantom_attn.h")


@pytest.fixture(scope="module")
def lib():
    from cuda_attn.capi import CAPI
    return CAPI()


def test_exports_every_declared_symbol(lib):
    from cuda_attn.capi import SIGNATURES, header_symbols
    declared = header_symbols(HEADER)
    assert len(declared) >= 9
    for name in declared:
        assert hasattr(lib.lib, name), f"{name} declared in phantom_attn.h but not exported"
    assert set(declared) == set(SIGNATURES), "ctypes signature table out of sync with the header"


def test_version(lib):
    assert lib.lib.phantom_attn_version() >= 10000


def _call(lib, fn, BH=1, N=16, d=64, dtype=1, causal=0, extra=()):
    p = ctypes.c_void_p(16)
    return fn(p, p, p, p, BH, N, d, dtype, causal, *extra, None)


@pytest.mark.parametrize("name", ["phantom_attn_fused_tc", "phantom_attn_fused", "phantom_attn_naive",
                                  "phantom_attn_tiled"])
def test_rejects_empty_and_bad_dtype(lib, name):
    from cuda_attn.capi import ERR_INVALID
    fn = getattr(lib.lib, name)
    assert _call(lib, fn, N=0) == ERR_INVALID and "non-empty" in lib.last_error()
    assert _call(lib, fn, BH=0) == ERR_INVALID and "non-empty" in lib.last_error()
    assert _call(lib, fn, dtype=7) == ERR_INVALID and "dtype" in lib.last_error()


def test_rejects_oversized_grid(lib):
    from cuda_attn.capi import ERR_UNSUPPORTED
    assert _call(lib, lib.lib.phantom_attn_fused_tc, BH=70000) == ERR_UNSUPPORTED
    assert "65535" in lib.last_error()


def test_fused_tuned_rejects_uncompiled_tiles(lib):
    from cuda_attn.capi import ERR_UNSUPPORTED
    rc = _call(lib, lib.lib.phantom_attn_fused_tuned, extra=(1, 32, 32))
    assert rc == ERR_UNSUPPORTED and "not compiled" in lib.last_error()


def test_launch_count_resets(lib):
    lib.launch_count(reset=True)
    assert lib.launch_count() == 0


def test_launch_shape_is_per_thread_and_validated(lib):
    """The launch-shape override (host state only, no GPU) reads back, is per calling thread, and
    rejects negative values and oversized groups with PHANTOM_ATTN_ERR_INVALID."""
    import threading

    from cuda_attn.capi import ERR_INVALID, CapiError
    try:
        assert lib.get_launch_shape() == (0, 0)
        lib.set_launch_shape(4096, 17)
        assert lib.get_launch_shape() == (4096, 17)
        seen = []
        t = threading.Thread(target=lambda: seen.append(lib.get_launch_shape()))
        t.start()
        t.join()
        assert seen == [(0, 0)]
        for kib, ctas in [(-1, 0), (0, -1), ((1 << 40) + 1, 0)]:
            with pytest.raises(CapiError) as e:
                lib.set_launch_shape(kib, ctas)
            assert e.value.code == ERR_INVALID and "set_launch_shape" in str(e.value)
        assert lib.get_launch_shape() == (4096, 17)
    finally:
        lib.set_launch_shape(0, 0)


def test_python_api_mirrors_reference_names():
    import cuda_attn
    for name in ("naive", "tiled", "fused", "fused_tuned", "fused_vec", "fused_db", "fused_tc", "reference",
                 "KERNELS", "FP16_ONLY"):
        assert hasattr(cuda_attn, name)
    assert list(cuda_attn.KERNELS) == ["naive", "tiled", "fused", "fused_vec", "fused_db", "fused_tc"]
    assert cuda_attn.FP16_ONLY == {"fused_vec", "fused_db", "fused_tc"}


def test_torch_binding_rejects_cpu_tensors():
    import torch
    import cuda_attn
    q = torch.zeros(1, 1, 8, 64)
    for name, fn in cuda_attn.KERNELS.items():
        with pytest.raises(RuntimeError, match="CUDA tensors"):
            fn(q, q, q)


def test_torch_binding_signatures():
    import cuda_attn
    ext = cuda_attn._ext()
    doc = ext.fused_tuned.__doc__
    for arg in ("causal: bool = False", "double_buffer: bool = True", "br: ", "= 64", "bc: ", "= 32"):
        assert arg in doc
    assert "causal: bool = False" in ext.fused_tc.__doc__


@pytest.mark.parametrize("bh,chunks", [(32, 8), (128, 8), (10, 3), (10, 1), (1, 8), (7, 8), (5, 3), (2, 8), (1000, 7)])
def test_host_pipeline_chunk_plan(bh, chunks):
    """fused_tc_host's chunk plan covers every head once: full chunks, then the last one cut into halves
    down to chunks of two heads (a short tail after the last input copy); one chunk when chunks <= 1."""
    from cuda_attn.pipeline import chunk_plan
    sizes = chunk_plan(bh, chunks)
    assert sum(sizes) == bh and min(sizes) >= 1
    if chunks <= 1:
        assert sizes == [bh]
        return
    per = sizes[0]
    assert per == -(-bh // chunks)
    assert all(s <= per for s in sizes)
    assert sizes == sorted(sizes, reverse=True)
    assert sizes[-1] <= 3  # halving stops once fewer than four heads are left


@pytest.mark.parametrize("bh,head_bytes,expect", [
    (128, 128 << 10, [64, 64]),                   # config 2: 16 MiB per tensor in all, no full 32 MiB chunk
    (128, 1 << 20, [32, 32, 32, 16, 8, 8]),       # config 3
    (32, 4 << 20, [8, 8, 8, 4, 2, 2]),            # config 4
    (4, 4 << 20, [2, 2]),                         # config 4's 8-GPU shard
    (16, 1 << 20, [8, 8]),                        # config 3's 8-GPU shard
    (3, 64 << 20, [1, 1, 1]),                     # heads above the floor: chunk by count
    (1, 1 << 10, [1]),
])
def test_host_pipeline_chunk_plan_byte_floors(bh, head_bytes, expect):
    """With a head's bytes given, full chunks hold at least MIN_CHUNK_BYTES of each input tensor and the
    tail halving stops at MIN_TAIL_BYTES (small copies run far below the host link's rate)."""
    from cuda_attn.pipeline import MIN_CHUNK_BYTES, MIN_TAIL_BYTES, chunk_plan
    sizes = chunk_plan(bh, 8, head_bytes, MIN_CHUNK_BYTES, MIN_TAIL_BYTES)
    assert sizes == expect
    assert sum(sizes) == bh and sizes == sorted(sizes, reverse=True)
