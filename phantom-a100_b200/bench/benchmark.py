"""Entry point at the reference's path for the sequence-length sweep against torch's SDPA (reference bench/benchmark.py).

    python bench/benchmark.py [options]        # run from phantom-a100_b200/, as the reference runs it from its root

The implementation is cuda_attn.sweep (same options as `python -m cuda_attn.sweep`).
"""
import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))

from cuda_attn.sweep import main  # noqa: E402

if __name__ == "__main__":
    sys.exit(main())
