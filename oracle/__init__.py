"""CPU oracle for the fused attention forward. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg (and its `--impl reference` arm)
may import this package, and only as the checker or the timed CPU baseline - never as the product
path. The product (phantom-a100_b200/cuda_attn, libphantom_attn.so) never imports it and has no CPU
fallback.

Contents (restating b4batunde/Phantom-A100, path:line within that project):

  attention_naive    cuda_attn/online_softmax_ref.py:14-24   float64 textbook softmax(QK^T/sqrt(d))V
  attention_online   cuda_attn/online_softmax_ref.py:27-63   float32 tile-by-tile online softmax in the
                                                             log2 domain; optional 16-bit rounding of P
                                                             (the reference's p_fp16 model of v4)
  reference_sdpa     cuda_attn/__init__.py:78-84             fp32 math-backend SDPA (torch, CPU)
  round_to           -                                       fp16 / bf16 round-to-nearest-even in NumPy

Parity is pinned: tests/golden/*.npz hold outputs of the reference's own oracle functions, produced by
tests/golden/make_golden.py importing the reference, and tests/test_oracle.py checks this restatement
against them.
"""
from .online_softmax import (LOG2E, attention_naive, attention_online, reference_sdpa, round_to,
                             sampled_rows_naive)

__all__ = ["LOG2E", "attention_naive", "attention_online", "reference_sdpa", "round_to", "sampled_rows_naive"]
