"""Entry point at the reference's path for one fixed call to profile with ncu (reference bench/run_one.py).

    python bench/run_one.py [options]        # run from phantom-a100_b200/, as the reference runs it from its root

The implementation is cuda_attn.run_one (same options as `python -m cuda_attn.run_one`).
"""
import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))

from cuda_attn.run_one import main  # noqa: E402

if __name__ == "__main__":
    sys.exit(main())
