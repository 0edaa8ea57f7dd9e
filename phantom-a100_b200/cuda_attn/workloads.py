"""Benchmark / parity workloads: the configurations the reference's headline metric is quoted on, with
seeded synthetic inputs and the algorithmic FLOP and byte counts used for the roofline.

Inputs are generated per global (batch*head) index with its own seed, so a run sharded over heads across
ranks reproduces exactly the tensors of a single-GPU run (rank r generates only its heads).

FLOPs per forward = 4 * B * H * N^2 * d (two matmuls of 2 N^2 d each; reference bench/benchmark.py:63-66),
halved when causal. Algorithmic HBM bytes = 4 * B * H * N * d * elem (Q, K, V read once, O written once).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class Config:
    name: str
    B: int
    H: int
    N: int
    d: int
    dtype: torch.dtype
    causal: bool = False
    std: float = 1.0               # Q/K/V ~ N(0, std)
    k_outlier_frac: float = 0.0    # fraction of K rows per head scaled by k_outlier_scale
    k_outlier_scale: float = 8.0
    seed: int = 0
    notes: str = field(default="", compare=False)

    @property
    def BH(self) -> int:
        return self.B * self.H

    @property
    def elem(self) -> int:
        return torch.tensor([], dtype=self.dtype).element_size()

    def flops(self, heads: int | None = None) -> float:
        bh = self.BH if heads is None else heads
        f = 4.0 * bh * self.N * self.N * self.d
        return f / 2 if self.causal else f

    def hbm_bytes(self, heads: int | None = None) -> float:
        bh = self.BH if heads is None else heads
        return 4.0 * bh * self.N * self.d * self.elem

    def describe(self) -> dict:
        return {"workload": self.name, "B": self.B, "H": self.H, "N": self.N, "d": self.d,
                "dtype": str(self.dtype).replace("torch.", ""), "causal": self.causal,
                "distribution": self.notes or f"N(0,{self.std})"}


# BASELINE configs (BASELINE.json "configs"); config 1 is the reference's CPU-only case.
CONFIGS = {
    "config1": Config("config1", 1, 42, 128, 64, torch.float32, notes="N(0,1) fp32, CPU oracle case"),
    "config2": Config("config2", 8, 16, 1024, 64, torch.float16),
    "config3": Config("config3", 4, 32, 4096, 128, torch.bfloat16),
    "config4": Config("config4", 1, 32, 16384, 128, torch.bfloat16, std=0.5, k_outlier_frac=0.01,
                      notes="Q,V ~ N(0,0.5) (std 0.5); K ~ N(0,0.5) with 1% of rows per head scaled x8"),
}
SWEEP_N = (128, 256, 512, 1024, 2048, 4096, 8192)


def sweep_config(n: int, d: int) -> Config:
    """sequence-length sweep, B*H = 64, fp16 N(0,1)."""
    return Config(f"config5_n{n}_d{d}", 1, 64, n, d, torch.float16)


def head_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) share of `total` heads for `rank` of `world` (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def make_inputs(cfg: Config, heads: tuple[int, int] | None = None, device: str | torch.device = "cuda"):
    """Seeded (q, k, v) of shape (1, stop - start, N, d) for global heads [start, stop) of cfg (all heads
    by default, shaped (B, H, N, d)). Head h uses seed (cfg.seed * 1_000_003 + h) for q, k, v in turn."""
    start, stop = heads if heads is not None else (0, cfg.BH)
    nh = stop - start
    dev = torch.device(device)
    q = torch.empty(nh, cfg.N, cfg.d, device=dev, dtype=cfg.dtype)
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    for i, h in enumerate(range(start, stop)):
        g = torch.Generator(device=dev).manual_seed(cfg.seed * 1_000_003 + h)
        for t in (q, k, v):
            x = torch.randn(cfg.N, cfg.d, device=dev, dtype=torch.float32, generator=g) * cfg.std
            if t is k and cfg.k_outlier_frac > 0:
                n_out = max(1, int(round(cfg.k_outlier_frac * cfg.N)))
                rows = torch.randperm(cfg.N, device=dev, generator=g)[:n_out]
                x[rows] *= cfg.k_outlier_scale
            t[i].copy_(x.to(cfg.dtype))
    if heads is None:
        shape = (cfg.B, cfg.H, cfg.N, cfg.d)
    else:
        shape = (1, nh, cfg.N, cfg.d)
    return q.view(shape), k.view(shape), v.view(shape)
