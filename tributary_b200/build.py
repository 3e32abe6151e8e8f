"""Build libtributary_b200.so in-tree with nvcc for sm_100a.

    python -m tributary_b200.build          # or tributary_b200.build.build()

The library is one translation unit (csrc/rt_library.cu). It links only the
CUDA runtime (static) and reaches the driver API through
cudaGetDriverEntryPoint, so it loads on any box with the NVIDIA driver.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_NAME = "libtributary_b200.so"
LIB_PATH = os.path.join(PKG, LIB_NAME)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "--use_fast_math",
    "-Xcompiler", "-fPIC,-O2",
    "-Xptxas", "-v",
]


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC)
                  if f.endswith((".cu", ".cuh", ".h"))) + [os.path.join(INCLUDE, "rt_attention.h")]


def is_stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(s) > t for s in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not is_stale():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-shared",
           "-o", tmp, os.path.join(CSRC, "rt_library.cu"), "-cudart", "static"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    log = proc.stdout + proc.stderr
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{log}")
    # registers, spills and shared memory per kernel (build output, kept out of
    # the package and of version control); compile times are left out
    os.makedirs(os.path.join(REPO, "_build"), exist_ok=True)
    with open(os.path.join(REPO, "_build", "ptxas.log"), "w") as f:
        f.write("".join(l for l in log.splitlines(keepends=True) if "Compile time" not in l))
    if verbose:
        print(log)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
