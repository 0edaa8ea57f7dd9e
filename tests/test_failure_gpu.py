"""GPU: the failure path of the bounded device waits, made to happen without any fault.

The tensor-core kernel waits on mbarriers (TMA copies landing, MMAs completing, softmax hand-offs).
Each wait gives up after a limit (about a second), raises the CTA's abort flag, records a bit in the
device status word and lets the kernel drain and exit, so a lost signal is reported, not a hang.
`phantom_attn_wait_expiry_probe` runs that same wait on a barrier nothing arrives on; the test checks
that the expiry is reported through `phantom_attn_device_status`, that the word is cleared by the read,
and that the context is still usable: the attention kernel runs and matches the oracle afterwards."""
import time

import numpy as np
import pytest
import torch

from conftest import assert_parity, make_qkv, torch_dtype_name
from oracle import attention_naive

pytestmark = pytest.mark.gpu

STATUS_PROBE = 16  # PHANTOM_ATTN_STATUS_PROBE in include/phantom_attn.h
STATUS_NOALLOC = 256  # PHANTOM_ATTN_STATUS_NOALLOC: the bit came (also) from fused_tc_noalloc's word


def test_expired_wait_is_reported_and_context_stays_usable(cuda_ok, capi):
    assert capi.device_status() == 0
    t0 = time.perf_counter()
    capi.wait_expiry_probe()
    status = capi.device_status()  # synchronises: returns once the probe kernel has given up and exited
    elapsed = time.perf_counter() - t0
    # once fused_tc_noalloc has run on this device, its word gets the probe's bit too
    assert status & ~STATUS_NOALLOC == STATUS_PROBE, f"status 0x{status:x}: the wait did not expire as a bounded wait"
    assert 0.2 < elapsed < 30.0, f"probe took {elapsed:.2f} s (limit is about a second of GPU clock)"
    assert capi.device_status() == 0, "reading the status word must clear it"

    q, k, v = make_qkv(1, 2, 300, 128, torch.bfloat16, seed=3)
    o = torch.full_like(q, float("nan"))
    capi.fused_tc(q, k, v, o, causal=True)
    torch.cuda.synchronize()
    ref = attention_naive(*(x.float().cpu().numpy().astype(np.float64) for x in (q, k, v)), True)
    assert_parity(o.float().cpu().numpy().astype(np.float64), ref, torch_dtype_name(torch.bfloat16), "after probe")
    assert capi.device_status() == 0
