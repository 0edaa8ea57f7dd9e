"""Build recipe for oracle/_ref/ - the reference's own harness, compiled from its sources in place.
TEST INFRASTRUCTURE ONLY (a checker / comparison baseline, never the product).

    python oracle/build_ref.py --reference /path/to/Phantom-A100
    PHANTOM_REFERENCE=/path/to/Phantom-A100 python oracle/build_ref.py

Compiles b4batunde/Phantom-A100's sim/harness.cu (its torch-free driver: seeded fp16 inputs, every
kernel v1..v4 from csrc/kernels/*.cuh, a float64 CPU check and a CUDA-event TIME line; harness.cu:1-167)
with nvcc for sm_100a, straight from the reference checkout (no source is copied into this repository).
Output: oracle/_ref/harness (git-ignored; it travels with the tree to the GPU box). The result lets the
reference's recompiled WMMA kernel (fused_tc) be timed on a B200 beside the tcgen05 kernel:

    HARNESS_ITERS=100 oracle/_ref/harness fused_tc 128 1024      # BASELINE config 2 (B*H=128, N=1024)

Without a reference checkout (no --reference, no PHANTOM_REFERENCE) this is a no-op.
"""
from __future__ import annotations

import argparse
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def reference_dir(reference: str | None = None) -> str | None:
    """The reference checkout: the argument, else $PHANTOM_REFERENCE, else None."""
    return reference or os.environ.get("PHANTOM_REFERENCE") or None


def build(reference: str | None = None, force: bool = False) -> str | None:
    reference = reference_dir(reference)
    if reference is None:
        return None
    src = os.path.join(reference, "sim", "harness.cu")
    if not os.path.exists(src):
        return None
    os.makedirs(OUT, exist_ok=True)
    exe = os.path.join(OUT, "harness")
    deps = [src] + [os.path.join(reference, "csrc", "kernels", f) for f in os.listdir(os.path.join(reference, "csrc", "kernels"))]
    if not force and os.path.exists(exe) and all(os.path.getmtime(d) <= os.path.getmtime(exe) for d in deps):
        return exe
    # the reference's own flags (setup.py:25-29) with the B200 target in place of its 75..90 list
    cmd = [os.path.join(CUDA_HOME, "bin", "nvcc"), "-O3", "-lineinfo", "--use_fast_math", "-std=c++17",
           "-gencode", "arch=compute_100a,code=sm_100a", f"-I{os.path.join(reference, 'csrc')}", src, "-o", exe]
    subprocess.run(cmd, check=True)
    return exe


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="reference checkout (default: $PHANTOM_REFERENCE)")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.reference, a.force) or "reference checkout not found; nothing built")
