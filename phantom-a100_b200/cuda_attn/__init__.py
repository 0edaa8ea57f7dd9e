"""B200 (sm_100a) attention kernels behind the API of b4batunde/Phantom-A100's `cuda_attn` package.

    import cuda_attn
    o = cuda_attn.fused_tc(q, k, v, causal=False)   # q, k, v: (B, H, N, d) CUDA tensors

Same names, signatures and error behaviour as the reference API (cuda_attn/__init__.py:40-94):

  fused_tc, fused_tuned, fused_vec, fused_db   tcgen05 tensor-core kernel (TMEM accumulators, TMA K/V
                                               ring); fp16 or bf16, head dim 64 or 128.
  fused, naive, tiled                          fp32-arithmetic CUDA-core kernel; fp32/fp16/bf16, d <= 256.
  reference                                    fp32 math-backend SDPA, the ground truth of the tests.
  fused_tc_host                                fused_tc for host (pinned) tensors: head chunks streamed
                                               through the GPU with copies overlapping the kernel.

The kernels live in libphantom_attn.so (C ABI: include/phantom_attn.h); `_C` is the PyTorch
extension over it. There is no CPU fallback: if the extension is missing, every kernel call raises.
Build it with `python phantom-a100_b200/build.py`.
"""
from __future__ import annotations

import torch

_EXT = None  # cached extension module


def _ext():
    """Load the compiled extension on first use (no JIT, no fallback)."""
    global _EXT
    if _EXT is None:
        try:
            from . import _C as ext
        except ImportError as e:  # pragma: no cover - depends on the build
            raise ImportError(
                "cuda_attn._C is not built; run `python phantom-a100_b200/build.py` (needs nvcc 12.8+)") from e
        _EXT = ext
    return _EXT


def naive(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> torch.Tensor:
    """v1 entry point. On sm_100a: the fused fp32 CUDA-core kernel (no N x N workspace)."""
    return _ext().naive(q, k, v, causal)


def tiled(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> torch.Tensor:
    """v2 entry point. On sm_100a: the fused fp32 CUDA-core kernel (no N x N workspace)."""
    return _ext().tiled(q, k, v, causal)


def fused(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> torch.Tensor:
    """v3: fused online softmax, fp32 arithmetic on CUDA cores. fp32/fp16/bf16, head dim <= 256."""
    return _ext().fused(q, k, v, causal)


def fused_tuned(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                double_buffer: bool = True, br: int = 64, bc: int = 32) -> torch.Tensor:
    """v3.1/v3.2 entry point. (br, bc) must be one of (64, 32), (64, 64), (128, 32), (128, 64), as in the
    reference; the work runs on the tcgen05 tensor-core kernel. fp16/bf16, head dim 64 or 128."""
    return _ext().fused_tuned(q, k, v, causal, double_buffer, br, bc)


def fused_vec(q, k, v, causal=False):
    """v3.1 entry point with default tiles."""
    return fused_tuned(q, k, v, causal, double_buffer=False)


def fused_db(q, k, v, causal=False):
    """v3.2 entry point with default tiles."""
    return fused_tuned(q, k, v, causal, double_buffer=True)


def fused_tc(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> torch.Tensor:
    """v4: both matmuls on 5th-gen tensor cores (tcgen05.mma, fp32 accumulators in TMEM), online softmax
    between them, K/V streamed by TMA. fp16 or bf16, head dim 64 or 128, sm_100a."""
    return _ext().fused_tc(q, k, v, causal)


def reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> torch.Tensor:
    """FP32 math-backend SDPA: the ground truth every kernel is tested against (reference
    cuda_attn/__init__.py:78-84)."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    with sdpa_kernel(SDPBackend.MATH):
        return torch.nn.functional.scaled_dot_product_attention(
            q.float(), k.float(), v.float(), is_causal=causal)


def device_status() -> int:
    """Read and clear the device status word of the current device (0 = every bounded wait in the
    tensor-core kernel completed). Synchronises the device."""
    return _ext().device_status()


from .pipeline import fused_tc_host  # noqa: E402  (host-resident inputs, copies overlapped with compute)

# Every version, in the order the reference builds them.
KERNELS = {"naive": naive, "tiled": tiled, "fused": fused,
           "fused_vec": fused_vec, "fused_db": fused_db, "fused_tc": fused_tc}
# Versions that only take 16-bit inputs (the reference's float16-only set; bf16 is accepted too).
FP16_ONLY = {"fused_vec", "fused_db", "fused_tc"}

__all__ = ["naive", "tiled", "fused", "fused_tuned", "fused_vec", "fused_db", "fused_tc",
           "reference", "KERNELS", "FP16_ONLY", "device_status", "fused_tc_host"]
