"""Build recipe for libgsp_b200.so (the C-ABI library declared in include/gsp_b200.h).

Compiles every CUDA source under csrc/ for sm_100a with nvcc into one shared
library placed next to the Python package (gsp/lib/libgsp_b200.so), so the
built artefact travels with the source tree. The library links the CUDA
runtime statically and has no libtorch dependency.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "gsp", "lib")
LIB_PATH = os.path.join(LIB_DIR, "libgsp_b200.so")
REPO_ROOT = os.path.dirname(HERE)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "-shared", "-cudart", "static",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libgsp_b200.so")
    return cand


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def build(verbose: bool = False, extra_flags: list[str] | None = None) -> str:
    os.makedirs(LIB_DIR, exist_ok=True)
    cmd = [nvcc_path(), *NVCC_FLAGS, *(extra_flags or []),
           "-I", os.path.join(REPO_ROOT, "include"), "-I", CSRC,
           "-o", LIB_PATH, *sources()]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + proc.stdout + proc.stderr)
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout + proc.stderr, file=sys.stderr)
    return LIB_PATH


if __name__ == "__main__":
    flags = sys.argv[1:]
    print(build(verbose=True, extra_flags=flags))
