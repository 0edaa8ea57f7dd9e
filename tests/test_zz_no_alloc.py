"""GPU: phantom_attn_fused_tc_noalloc, the entry point for callers that cannot allocate device memory
while they run (a plugin host that owns all device memory and hands over only inputs and outputs, a
real-time loop that forbids allocator calls after start-up). It must give the results of the allocating
phantom_attn_fused_tc, on consecutive calls that share its static scratch, and refuse bf16 inputs that
do not fit that scratch.

Kept in a file that pytest collects last, so a failure here never hides the rest of the suite.
"""
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
