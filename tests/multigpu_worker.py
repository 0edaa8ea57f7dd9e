"""One rank of the 2-GPU test (tests/test_multigpu.py), run under torchrun with the NCCL backend.

Each rank generates and attends its contiguous share of the B*H heads (no collective on the compute path),
then the outputs are gathered to rank 0 (cuda_attn.dist.gather_heads over NCCL), which runs every head on
its own GPU and requires the gathered result to be equal bit for bit. Prints MULTIGPU_OK on rank 0.
"""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "phantom-a100_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from cuda_attn.capi import CAPI  # noqa: E402
from cuda_attn.dist import gather_heads  # noqa: E402
from cuda_attn.workloads import Config, head_range, make_inputs  # noqa: E402


def main() -> int:
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    lib = CAPI()
    ok = True
    # (config, causal): bf16 d=128 with K outliers (multi-wave per rank), fp16 d=64 with an odd head count
    jobs = [Config("mg_bf16", 2, 9, 4096, 128, torch.bfloat16, std=0.5, k_outlier_frac=0.01, seed=3),
            Config("mg_fp16", 1, 13, 1500, 64, torch.float16, causal=True, seed=4)]
    # every query block over its whole K/V range, so that a rank's result does not depend on how many heads
    # it holds (with K/V parts, a tail's blocks merge partial results and match only within tolerance)
    lib.set_kv_parts(False)
    for cfg in jobs:
        mine = head_range(cfg.BH, world, rank)
        q, k, v = make_inputs(cfg, heads=mine, device=dev)
        o = torch.empty_like(q)
        lib.fused_tc(q, k, v, o, causal=cfg.causal)
        torch.cuda.synchronize()
        full = gather_heads(o, cfg.BH, world, rank)
        if rank == 0:
            qa, ka, va = (x.reshape(1, cfg.BH, cfg.N, cfg.d) for x in make_inputs(cfg, device=dev))
            oa = torch.empty_like(qa)
            lib.fused_tc(qa, ka, va, oa, causal=cfg.causal)
            torch.cuda.synchronize()
            same = torch.equal(full, oa)
            print(f"{cfg.name}: heads {cfg.BH} over {world} ranks, gathered == single GPU: {same}", flush=True)
            ok = ok and same
    status = torch.tensor([float(lib.device_status())], device=dev)
    dist.all_reduce(status, op=dist.ReduceOp.MAX)
    flag = torch.tensor([1.0 if ok else 0.0], device=dev)
    dist.broadcast(flag, src=0)
    dist.destroy_process_group()
    if rank == 0 and flag.item() > 0.5 and status.item() == 0:
        print("MULTIGPU_OK", flush=True)
    return 0 if flag.item() > 0.5 and status.item() == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
