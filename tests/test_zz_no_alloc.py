"""GPU: phantom_attn_fused_tc_noalloc, the entry point for callers that cannot allocate device memory
while they run (a plugin host that owns all device memory and hands over only inputs and outputs, a
real-time loop that forbids allocator calls after start-up). It must give the results of the allocating
phantom_attn_fused_tc, on consecutive calls that share its static scratch, refuse bf16 inputs that do
not fit that scratch, allocate nothing, and report an expired device wait through device_status.

Kept in a file that pytest collects last, so a failure here never hides the rest of the suite.
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import assert_parity, make_qkv, torch_dtype_name

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d", [64, 128])
def test_noalloc_matches_allocating_entry_point_twice(cuda_ok, capi, dtype, d):
    # two calls in a row with different inputs and sizes: the second must not see the first's scratch
    for seed, (bh, n) in enumerate([(6, 1000), (3, 257)]):
        q, k, v = make_qkv(1, bh, n, d, dtype, seed=seed + 40)
        o_ref = torch.empty_like(q)
        capi.fused_tc(q, k, v, o_ref, causal=bool(seed))
        o = torch.full_like(q, float("nan"))
        capi.fused_tc_noalloc(q, k, v, o, causal=bool(seed))
        torch.cuda.synchronize()
        assert torch.isfinite(o).all()
        assert_parity(o.double().cpu().numpy(), o_ref.double().cpu().numpy(), torch_dtype_name(dtype),
                      f"noalloc call {seed + 1} vs fused_tc")


def test_noalloc_rejects_bf16_inputs_beyond_its_scratch(cuda_ok, capi):
    from cuda_attn.capi import ERR_UNSUPPORTED, CapiError
    # B*H*N*d = 1 * 8 * 32768 * 128 = 33.6M elements: the fp16 copy of V alone is 64 MiB
    t = torch.empty(1, 8, 32768, 128, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(CapiError) as e:
        capi.fused_tc_noalloc(t, t, t, t)
    assert e.value.code == ERR_UNSUPPORTED and "scratch" in str(e.value)


def test_noalloc_overflow_heads_across_consecutive_calls(cuda_ok, capi):
    """bf16 calls through the allocation-free entry point share one static array, counters and overflow
    word included: a call with fp16-overflowing V heads, one without, and one with again must each equal
    the allocating entry point's result."""
    q, k, v = make_qkv(1, 64, 600, 128, torch.bfloat16, seed=61)
    v_bad = v.clone()
    for h in range(5, 64, 11):
        v_bad[0, h, (h * 13) % 600, h % 128] = 3.0e5  # beyond fp16's 65504
    for call, vv in enumerate([v_bad, v, v_bad]):
        o_ref = torch.empty_like(q)
        capi.fused_tc(q, k, vv, o_ref)
        o = torch.full_like(q, float("nan"))
        capi.fused_tc_noalloc(q, k, vv, o)
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref), f"noalloc call {call + 1} differs from fused_tc"
    assert capi.device_status() == 0


STATUS_PROBE, STATUS_NOALLOC = 16, 256  # include/phantom_attn.h


def test_noalloc_wait_expiry_is_reported_by_device_status(cuda_ok, capi):
    """An expired bounded wait on the allocation-free path lands in the status word inside its static
    array; device_status reads and clears that word too and flags it with STATUS_NOALLOC. The probe runs
    the kernels' bounded wait on a barrier nothing arrives on and, once the entry point is set up on the
    device, records its bit in that word as well."""
    q, k, v = make_qkv(1, 2, 200, 64, torch.float16, seed=9)
    o = torch.empty_like(q)
    capi.fused_tc_noalloc(q, k, v, o)  # sets the entry point up on this device
    assert capi.device_status() == 0
    capi.wait_expiry_probe()
    assert capi.device_status() == STATUS_PROBE | STATUS_NOALLOC
    assert capi.device_status() == 0, "reading must clear both words"
    capi.fused_tc_noalloc(q, k, v, o)
    torch.cuda.synchronize()
    o_ref = torch.empty_like(q)
    capi.fused_tc(q, k, v, o_ref)
    assert torch.equal(o, o_ref), "the entry point must still work after an expiry was reported"
    assert capi.device_status() == 0


_NO_ALLOC_PROBE = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from cuda_attn.capi import CAPI
lib = CAPI()
g = torch.Generator(device="cuda").manual_seed(0)
shapes = [(64, 2048, 128, torch.bfloat16), (32, 1000, 64, torch.bfloat16), (96, 2048, 64, torch.float16),
          (8, 300, 128, torch.float16)]
bufs = [[torch.randn(1, bh, n, d, device="cuda", generator=g).to(dt) for _ in range(4)] for bh, n, d, dt in shapes]
for q, k, v, o in bufs:      # first launches load each kernel (lazy module loading allocates code memory)
    lib.fused_tc_noalloc(q, k, v, o)
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
for rep in range(3):
    for q, k, v, o in bufs:  # multi-wave launches (work counter) and bf16 staging, in the static array only
        lib.fused_tc_noalloc(q, k, v, o, causal=bool(rep % 2))
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
print("FREE_DELTA", free0 - free1)
"""


def test_noalloc_allocates_no_device_memory(cuda_ok):
    """In a fresh process (no library memory pool exists yet), repeated allocation-free calls of every
    dtype and head dimension, multi-wave and bf16 included, leave the device's free memory unchanged: a
    call that went through the pool would create it and reserve memory."""
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "phantom-a100_b200")
    p = subprocess.run([sys.executable, "-c", _NO_ALLOC_PROBE, pkg], capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    delta = [int(l.split()[1]) for l in p.stdout.splitlines() if l.startswith("FREE_DELTA")]
    assert delta == [0], (p.stdout[-500:], p.stderr[-500:])
