"""A fixed profiling target: one kernel, one shape, a few calls (the role of the reference's
bench/run_one.py, here with the head dimension and dtype of the B200 kernels selectable).

    python -m cuda_attn.run_one --impl fused_tc --n 4096 --dim 128 --dtype bf16
    ncu --clock-control none -k regex:attn_fwd_tc -s 2 -c 1 python -m cuda_attn.run_one --impl fused_tc --reps 3
"""
from __future__ import annotations

import argparse
import sys

import torch

from . import KERNELS, FP16_ONLY


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--impl", choices=sorted(KERNELS), default="fused_tc")
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--dim", type=int, default=64)
    ap.add_argument("--dtype", choices=["fp16", "bf16", "fp32"], default="fp16")
    ap.add_argument("--causal", action="store_true")
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    dtype = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[a.dtype]
    if a.impl in FP16_ONLY and dtype == torch.float32:
        raise SystemExit(f"{a.impl} takes fp16 or bf16 inputs")
    g = torch.Generator(device="cuda").manual_seed(a.seed)
    q, k, v = (torch.randn(a.batch, a.heads, a.n, a.dim, device="cuda", generator=g).to(dtype) for _ in range(3))
    fn = KERNELS[a.impl]
    for _ in range(a.reps):
        o = fn(q, k, v, a.causal)
    torch.cuda.synchronize()
    print(f"ran {a.impl} B={a.batch} H={a.heads} N={a.n} d={a.dim} {a.dtype} causal={a.causal} x{a.reps}; "
          f"out {tuple(o.shape)} finite={bool(torch.isfinite(o).all())}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
