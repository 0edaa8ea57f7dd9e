"""Nsight Compute counters of the attention kernels, at the reference's module path (autotune/hw_counters.py).

    python -m autotune.hw_counters [options] -- <command>      # from phantom-a100_b200/
    from autotune import hw_counters                           # the same module as cuda_attn.hw_counters
"""
import sys

from cuda_attn import hw_counters as _impl

sys.modules[__name__] = _impl

if __name__ == "__main__":
    sys.exit(_impl.main())
