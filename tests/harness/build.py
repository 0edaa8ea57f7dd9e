"""Build recipe of the torch-free harness (tests/harness/attn_harness): g++ over attn_harness.cpp and the
float64 oracle oracle/ref64.c, linked against the library's C ABI (libphantom_attn.so). Test
infrastructure; the binary is git-ignored and travels with the tree."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
EXE = os.path.join(HERE, "attn_harness")


def build(force: bool = False) -> str:
    srcs = [os.path.join(HERE, "attn_harness.cpp"), os.path.join(ROOT, "oracle", "ref64.c"),
            os.path.join(ROOT, "oracle", "ref64.h"), os.path.join(ROOT, "include", "phantom_attn.h")]
    if not force and os.path.exists(EXE) and all(os.path.getmtime(s) <= os.path.getmtime(EXE) for s in srcs):
        return EXE
    lib_dir = os.path.join(ROOT, "phantom-a100_b200", "cuda_attn")
    obj = os.path.join(HERE, "ref64.o")
    subprocess.run(["gcc", "-O2", "-c", srcs[1], "-o", obj], check=True)
    subprocess.run(["g++", "-O2", "-std=c++17", f"-I{ROOT}/include", f"-I{ROOT}/oracle", f"-I{CUDA}/include", srcs[0], obj,
                    f"-L{lib_dir}", "-lphantom_attn", f"-L{CUDA}/lib64", "-lcudart",
                    "-Wl,-rpath,$ORIGIN/../../phantom-a100_b200/cuda_attn", f"-Wl,-rpath,{CUDA}/lib64", "-o", EXE],
                   check=True)
    os.remove(obj)
    return EXE


if __name__ == "__main__":
    print(build(force=True))
