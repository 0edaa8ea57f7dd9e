"""NumPy restatement of the reference's CPU model of the fused attention forward.
TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the checker and the CPU baseline, never the product.

Source being restated: b4batunde/Phantom-A100 cuda_attn/online_softmax_ref.py (NumPy model of the
fused kernels) and cuda_attn/__init__.py:78-84 (the fp32 SDPA ground truth of its GPU tests).
"""
from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634  # log2(e); online_softmax_ref.py:11, device_common.cuh:22


def round_to(x: np.ndarray, dtype: str | None) -> np.ndarray:
    """Round float32 values to float16 or bfloat16 (round to nearest even) and return them as float32.

    dtype None returns x unchanged. bfloat16 keeps the upper 16 bits of the float32 pattern after adding
    half an ulp (with ties to even), which is what __float2bfloat16_rn / cvt.rn.bf16 compute for finite
    inputs."""
    x = np.asarray(x, dtype=np.float32)
    if dtype is None:
        return x
    if dtype in ("float16", "f16", "fp16"):
        return x.astype(np.float16).astype(np.float32)
    if dtype in ("bfloat16", "bf16"):
        bits = x.view(np.uint32).astype(np.uint64)
        bits = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
        return bits.astype(np.uint32).view(np.float32)
    raise ValueError(f"unknown dtype {dtype!r}")


def attention_naive(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool = False) -> np.ndarray:
    """softmax(Q K^T / sqrt(d)) V in float64 on (..., N, d) arrays (online_softmax_ref.py:14-24)."""
    q64, k64, v64 = (np.asarray(x, dtype=np.float64) for x in (q, k, v))
    n, d = q64.shape[-2:]
    scores = np.matmul(q64, np.swapaxes(k64, -1, -2)) * (1.0 / np.sqrt(d))
    if causal:
        above = np.triu(np.ones((n, n), dtype=bool), k=1)  # key index > query index
        scores = np.where(above, -np.inf, scores)
    scores -= scores.max(axis=-1, keepdims=True)
    w = np.exp(scores)
    w /= w.sum(axis=-1, keepdims=True)
    return np.matmul(w, v64)


def sampled_rows_naive(q: np.ndarray, k: np.ndarray, v: np.ndarray, rows: np.ndarray,
                       causal: bool = False) -> np.ndarray:
    """attention_naive restricted to the query rows `rows` (1-D index array) of every head.

    Rows of softmax attention are independent, so this equals attention_naive(q, k, v)[..., rows, :]
    while costing O(len(rows) * N * d) instead of O(N^2 * d); it checks full-size outputs by sampling."""
    rows = np.asarray(rows)
    q64 = np.asarray(q[..., rows, :], dtype=np.float64)
    k64, v64 = np.asarray(k, dtype=np.float64), np.asarray(v, dtype=np.float64)
    n, d = k64.shape[-2:]
    scores = np.matmul(q64, np.swapaxes(k64, -1, -2)) * (1.0 / np.sqrt(d))
    if causal:
        above = np.arange(n)[None, :] > rows[:, None]
        scores = np.where(above, -np.inf, scores)
    scores -= scores.max(axis=-1, keepdims=True)
    w = np.exp(scores)
    w /= w.sum(axis=-1, keepdims=True)
    return np.matmul(w, v64)


def attention_online(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool = False, br: int = 64,
                     bc: int = 32, p_dtype: str | None = None, p_fp16: bool = False,
                     row_offset: int = 0) -> np.ndarray:
    """Tile-by-tile online softmax in float32, the way the fused kernels compute it
    (online_softmax_ref.py:27-63).

    Each block of `br` query rows is pre-scaled by log2(e)/sqrt(d); K/V stream in tiles of `bc` keys;
    per row a running max m and running sum l; alpha = exp2(m_old - m_new) rescales l and O; the output
    is O / l. p_dtype ("float16" / "bfloat16") rounds P before the P @ V product while l sums the
    unrounded values - the model of a tensor-core P.V (p_fp16=True is the reference's name for
    p_dtype="float16").

    Extension for row-sampled checks and baselines: q may hold fewer rows than k / v (a contiguous slice
    of the queries starting at global row `row_offset`); with equal lengths and row_offset = 0 this is
    exactly the reference function."""
    if p_fp16:
        p_dtype = "float16"
    q32, k32, v32 = (np.asarray(x, dtype=np.float32) for x in (q, k, v))
    *lead, n_q, d = q32.shape
    n_k = k32.shape[-2]
    out = np.empty_like(q32)
    scale_log2 = np.float32(LOG2E / np.sqrt(d))
    neg_inf = np.float32(-np.inf)

    for r0 in range(0, n_q, br):
        r1 = min(r0 + br, n_q)
        qs = q32[..., r0:r1, :] * scale_log2
        rows = np.arange(r0, r1) + row_offset
        m = np.full((*lead, r1 - r0), neg_inf, dtype=np.float32)
        l = np.zeros((*lead, r1 - r0), dtype=np.float32)
        acc = np.zeros((*lead, r1 - r0, d), dtype=np.float32)
        stop = min(n_k, row_offset + r1) if causal else n_k
        for c0 in range(0, stop, bc):
            c1 = min(c0 + bc, n_k)
            s = np.matmul(qs, np.swapaxes(k32[..., c0:c1, :], -1, -2))
            if causal:
                s = np.where(np.arange(c0, c1)[None, :] > rows[:, None], neg_inf, s)
            m_new = np.maximum(m, s.max(axis=-1))
            dead = np.isneginf(m_new)  # row with every key so far masked
            with np.errstate(invalid="ignore"):
                alpha = np.where(dead, 0.0, np.exp2(m - m_new)).astype(np.float32)
                p = np.where(dead[..., None], 0.0, np.exp2(s - m_new[..., None])).astype(np.float32)
            l = l * alpha + p.sum(axis=-1)
            acc = acc * alpha[..., None] + np.matmul(round_to(p, p_dtype), v32[..., c0:c1, :])
            m = m_new
        out[..., r0:r1, :] = acc / l[..., None]
    return out


def reference_sdpa(q, k, v, causal: bool = False):
    """fp32 math-backend scaled_dot_product_attention on CPU (cuda_attn/__init__.py:78-84): the ground
    truth the reference's GPU tests compare every kernel with. Accepts NumPy arrays or torch tensors and
    returns a float32 NumPy array."""
    import torch
    from torch.nn.attention import SDPBackend, sdpa_kernel

    def t(x):
        return (x if isinstance(x, torch.Tensor) else torch.from_numpy(np.asarray(x))).float().cpu()

    with sdpa_kernel(SDPBackend.MATH):
        o = torch.nn.functional.scaled_dot_product_attention(t(q), t(k), t(v), is_causal=causal)
    return o.numpy()
