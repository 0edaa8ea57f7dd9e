"""Generate the golden vectors that pin the oracle to the reference's own implementation.

    python tests/golden/make_golden.py --reference /path/to/Phantom-A100

Imports b4batunde/Phantom-A100's CPU code (cuda_attn/online_softmax_ref.py: attention_naive,
attention_online; cuda_attn/__init__.py: reference = fp32 SDPA math) from the given checkout and runs it
on seeded inputs. The outputs are written to tests/golden/*.npz together with the inputs, so the pin
does not depend on the random generator. This script needs the reference checkout and is run once by
hand; the tests only read the .npz files.

Cases (all small; the full-size configs are checked on the GPU with row sampling instead):
  config1   BASELINE config 1 (B=1, H=42, N=128, d=64, fp32 N(0,1)): first 2 heads stored in full,
            plus per-head sums of the outputs of all 42 heads (a checksum of the whole config).
  n{N}_c{C} the reference test_algorithm.py sizes N in {1, 31, 65, 257}, causal 0/1, d=64.
  tiles     tile-size invariance inputs (test_algorithm.py:30-35) with causal and 3 tile shapes.
  scale10   large scores (test_algorithm.py:21-27), x10.
  fp16p     fp16-rounded inputs with the reference's fp16-P model (test_algorithm.py:38-46), N=512.
  bf16_d128 bf16-rounded inputs, d=128, N=200 (the tensor-core dtype/head dim the reference lacks):
            naive float64 output only.
  outlier   config-4 distribution at small size: N(0,0.5) with 1% of K rows scaled x8, bf16-rounded,
            d=128, N=384.

Outputs are stored as float32 (enough to pin the oracle at 1e-6); 16-bit inputs are stored in their
16-bit form (bf16 as uint16 bit patterns, key suffix "_bf16bits").
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def bf16_round(x: np.ndarray) -> np.ndarray:
    """bfloat16 round-to-nearest-even of float32 values, returned as float32 (torch is the reference)."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def bits(x: np.ndarray) -> np.ndarray:
    """uint16 bit patterns of bf16-representable float32 values."""
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of a b4batunde/Phantom-A100 checkout")
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    import torch
    from cuda_attn import reference as ref_sdpa  # the reference's fp32 SDPA math ground truth
    from cuda_attn.online_softmax_ref import attention_naive, attention_online

    def sdpa(q, k, v, causal):
        return ref_sdpa(*(torch.from_numpy(x) for x in (q, k, v)), causal).numpy()

    out = {}

    # config 1, full: inputs from a seeded generator, outputs of all three reference functions
    rng = np.random.default_rng(20240101)
    q, k, v = (rng.standard_normal((1, 42, 128, 64)).astype(np.float32) for _ in range(3))
    naive = attention_naive(q, k, v, False)
    online = attention_online(q, k, v, False)
    sd = sdpa(q, k, v, False)
    out["config1"] = dict(q=q[:, :2], k=k[:, :2], v=v[:, :2], naive=naive[:, :2], online=online[:, :2],
                          sdpa=sd[:, :2], head_sums_naive=naive.sum(axis=(-1, -2)),
                          head_sumsq_naive=(naive ** 2).sum(axis=(-1, -2)), causal=np.array(False))

    for n in (1, 31, 65, 257):
        for c in (False, True):
            rng = np.random.default_rng(n)
            q, k, v = (rng.standard_normal((1, 2 if n < 257 else 1, n, 64)).astype(np.float32) for _ in range(3))
            out[f"n{n}_c{int(c)}"] = dict(q=q, k=k, v=v, naive=attention_naive(q, k, v, c),
                                          online=attention_online(q, k, v, c), sdpa=sdpa(q, k, v, c),
                                          causal=np.array(c))

    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((1, 1, 300, 64)).astype(np.float32) for _ in range(3))
    tiles = {"q": q, "k": k, "v": v, "naive": attention_naive(q, k, v, True), "causal": np.array(True)}
    for br, bc in ((16, 16), (64, 32), (128, 64)):
        tiles[f"online_{br}_{bc}"] = attention_online(q, k, v, True, br, bc)
    out["tiles"] = tiles

    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 1, 200, 64)).astype(np.float32) for _ in range(3))
    q, k = q * 10, k * 10
    out["scale10"] = dict(q=q, k=k, v=v, naive=attention_naive(q, k, v), online=attention_online(q, k, v),
                          causal=np.array(False))

    rng = np.random.default_rng(7)
    q, k, v = (rng.standard_normal((1, 1, 512, 64)).astype(np.float16).astype(np.float32) for _ in range(3))
    out["fp16p"] = dict(q=q.astype(np.float16), k=k.astype(np.float16), v=v.astype(np.float16),
                        naive=attention_naive(q, k, v, False),
                        online_p16=attention_online(q, k, v, False, br=64, bc=64, p_fp16=True),
                        causal=np.array(False))

    rng = np.random.default_rng(11)
    q, k, v = (bf16_round(rng.standard_normal((1, 1, 200, 128)).astype(np.float32)) for _ in range(3))
    out["bf16_d128"] = dict(q_bf16bits=bits(q), k_bf16bits=bits(k), v_bf16bits=bits(v),
                            naive=attention_naive(q, k, v, False), naive_causal=attention_naive(q, k, v, True), causal=np.array(False))

    rng = np.random.default_rng(4)
    q, k, v = ((rng.standard_normal((1, 1, 384, 128)) * 0.5).astype(np.float32) for _ in range(3))
    for h in range(1):
        rows = rng.choice(384, size=max(1, 384 // 100), replace=False)
        k[0, h, rows] *= 8.0
    q, k, v = (bf16_round(x) for x in (q, k, v))
    out["outlier"] = dict(q_bf16bits=bits(q), k_bf16bits=bits(k), v_bf16bits=bits(v),
                          naive=attention_naive(q, k, v, False), online=attention_online(q, k, v), causal=np.array(False))

    for name, arrays in out.items():
        arrays = {key: (x.astype(np.float32) if x.dtype == np.float64 else x) for key, x in arrays.items()}
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **arrays)
        print(f"wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
