"""Multi-GPU partitioning of the attention forward: one process per GPU, heads sharded, no collective on
the compute path (every (batch, head) is independent; reference grid axis blockIdx.y = bh,
csrc/kernels/fused_tc.cuh:57). Outputs are gathered to rank 0 only to verify them.

    rank, world = dist.get_rank(), dist.get_world_size()
    start, stop = head_range(B * H, world, rank)          # this rank's heads
    o_local = cuda_attn.fused_tc(q_local, k_local, v_local)
    o_full = gather_heads(o_local, B * H, world, rank)     # rank 0 only; None elsewhere

Works with the NCCL backend (GPU tensors) and gloo (CPU tensors, used by the host tests).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .workloads import head_range

__all__ = ["head_range", "gather_heads", "shard_heads"]


def shard_heads(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's contiguous slice of the flattened B*H heads of a (B, H, N, d) tensor, shaped (1, h, N, d)."""
    B, H, N, d = x.shape
    start, stop = head_range(B * H, world, rank)
    return x.reshape(B * H, N, d)[start:stop].unsqueeze(0)


def gather_heads(local: torch.Tensor, total_heads: int, world: int, rank: int, dst: int = 0):
    """Gather every rank's (1, h_r, N, d) output to rank `dst` as one (1, total_heads, N, d) tensor.

    Shards may differ in size by one head; they are padded to the largest shard for the collective and
    trimmed afterwards. Returns the full tensor on `dst` and None on the other ranks."""
    _, h, N, d = local.shape
    start, stop = head_range(total_heads, world, rank)
    if stop - start != h:
        raise ValueError(f"rank {rank} holds {h} heads, expected {stop - start}")
    hmax = max(b - a for a, b in (head_range(total_heads, world, r) for r in range(world)))
    buf = local.new_zeros((hmax, N, d))
    buf[:h] = local[0]
    parts = [torch.empty_like(buf) for _ in range(world)] if rank == dst else None
    dist.gather(buf, gather_list=parts, dst=dst)
    if rank != dst:
        return None
    out = [parts[r][: head_range(total_heads, world, r)[1] - head_range(total_heads, world, r)[0]]
           for r in range(world)]
    return torch.cat(out, dim=0).unsqueeze(0)
