"""Build the XLA FFI handlers (rt_xla_ffi.cc) for a JAX caller.

    python -m tributary_b200.ffi.build_ffi

Compiles against the XLA FFI headers that jax ships (jax.ffi.include_dir())
and links libtributary_b200.so. Where jax is not importable the handlers
cannot be built: build() returns None and says why.
"""
from __future__ import annotations

import os
import subprocess
import sys

from ..build import INCLUDE, LIB_NAME, PKG, build as build_library

HERE = os.path.dirname(os.path.abspath(__file__))
FFI_LIB = os.path.join(HERE, "librt_xla_ffi.so")


def build() -> str | None:
    try:
        import jax.ffi
    except ImportError as e:
        print(f"XLA FFI handlers not built: jax is not importable ({e})")
        return None
    build_library()
    cmd = ["g++", "-std=c++17", "-O2", "-shared", "-fPIC", "-I", jax.ffi.include_dir(), "-I", INCLUDE,
           "-I", "/usr/local/cuda/include", os.path.join(HERE, "rt_xla_ffi.cc"), "-o", FFI_LIB,
           "-L", PKG, f"-l:{LIB_NAME}", f"-Wl,-rpath,{PKG}"]
    subprocess.run(cmd, check=True)
    return FFI_LIB


if __name__ == "__main__":
    sys.exit(0 if build() is not None or "--allow-missing" in sys.argv else 1)
