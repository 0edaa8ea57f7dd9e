"""In-tree build of the attention library.

    python phantom-a100_b200/build.py            # incremental
    python phantom-a100_b200/build.py --force    # rebuild everything

Produces, next to the Python package (so the files travel with the source tree):

  cuda_attn/libphantom_attn.so   the C-ABI library (include/phantom_attn.h): tcgen05 tensor-core kernel,
                                 fp32 CUDA-core kernel, argument checks. nvcc, sm_100a only.
  cuda_attn/_C<ext-suffix>       the PyTorch extension with the reference's pybind entry points, linked
                                 against libphantom_attn.so (rpath $ORIGIN).

No JIT cache under ~/.cache is used. Object files go to phantom-a100_b200/_build/.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig

PKG_ROOT = os.path.dirname(os.path.abspath(__file__))
REPO_ROOT = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
OUT_DIR = os.path.join(PKG_ROOT, "cuda_attn")
BUILD_DIR = os.path.join(PKG_ROOT, "_build")
INCLUDE = os.path.join(REPO_ROOT, "include")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall"] + ARCH

KERNEL_SOURCES = ["attn_tc_sm100.cu", "attn_simt.cu", "capi.cu"]
HEADERS = ["sm100_ptx.cuh", "launchers.h"]
LIB_NAME = "libphantom_attn.so"


def _newer(target: str, deps: list[str]) -> bool:
    """True if target exists and is newer than every dependency."""
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_library(force: bool = False, verbose: bool = False) -> str:
    """Compile the kernels and the C ABI into cuda_attn/libphantom_attn.so."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "phantom_attn.h")]
    objs = []
    for src in KERNEL_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD_DIR, src.replace(".cu", ".o"))
        if force or not _newer(o, [s] + headers):
            _run([NVCC, *NVCC_FLAGS, "-I", INCLUDE, "-c", s, "-o", o], verbose)
        objs.append(o)
    lib = os.path.join(OUT_DIR, LIB_NAME)
    if force or not _newer(lib, objs):
        _run([NVCC, "-shared", "--cudart", "shared", *ARCH, *objs, "-o", lib,
              "-Xlinker", f"-rpath,{CUDA_HOME}/lib64"], verbose)
    return lib


def build_torch_extension(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/bindings.cpp into the cuda_attn._C extension module."""
    import torch
    import torch.utils.cpp_extension as ce

    src = os.path.join(CSRC, "bindings.cpp")
    lib = os.path.join(OUT_DIR, LIB_NAME)
    out = os.path.join(OUT_DIR, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))
    # Depends on the C ABI (header), not on the library's contents: kernel edits need no relink.
    if not force and os.path.exists(lib) and _newer(out, [src, os.path.join(INCLUDE, "phantom_attn.h")]):
        return out
    inc = ce.include_paths("cuda") + [sysconfig.get_paths()["include"], INCLUDE]
    libdirs = ce.library_paths("cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H", "-w"]
    cmd += [f"-I{p}" for p in inc]
    cmd += [src, "-o", out]
    cmd += [f"-L{p}" for p in libdirs] + [f"-L{OUT_DIR}"]
    cmd += ["-lphantom_attn", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
            "-lcudart", "-Wl,-rpath,$ORIGIN"]
    _run(cmd, verbose)
    return out


def build(force: bool = False, verbose: bool = False, torch_ext: bool = True) -> None:
    if shutil.which(NVCC) is None and not os.path.exists(NVCC):
        raise RuntimeError(f"nvcc not found at {NVCC}")
    build_library(force, verbose)
    if torch_ext:
        build_torch_extension(force, verbose)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--no-torch", action="store_true", help="build only the C-ABI library")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    build(a.force, a.verbose, not a.no_torch)
    print("built:", ", ".join(sorted(f for f in os.listdir(OUT_DIR) if f.endswith(".so"))))
    sys.exit(0)
