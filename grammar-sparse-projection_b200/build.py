"""Build recipe for libgsp_b200.so (the C-ABI library declared in include/gsp_b200.h).

Compiles every CUDA source under csrc/ for sm_100a with nvcc into one shared
library placed next to the Python package (gsp/lib/libgsp_b200.so), so the
built artefact travels with the source tree. The library links the CUDA
runtime statically and has no libtorch dependency.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "gsp", "lib")
LIB_PATH = os.path.join(LIB_DIR, "libgsp_b200.so")
REPO_ROOT = os.path.dirname(HERE)

COMPILE_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr",
]
LINK_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libgsp_b200.so")
    return cand


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + proc.stdout + proc.stderr)
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout + proc.stderr, file=sys.stderr)


def build(verbose: bool = False, extra_flags: list[str] | None = None, out: str | None = None) -> str:
    """Compiles each translation unit in parallel (object files in a temporary
    directory), then links them into one shared library at `out` (default
    gsp/lib/libgsp_b200.so)."""
    out = out or LIB_PATH
    os.makedirs(os.path.dirname(out), exist_ok=True)
    nvcc = nvcc_path()
    incs = ["-I", os.path.join(REPO_ROOT, "include"), "-I", CSRC]
    with tempfile.TemporaryDirectory(prefix="gsp_build_") as tmp:
        jobs = []
        for src in sources():
            obj = os.path.join(tmp, os.path.basename(src)[:-3] + ".o")
            jobs.append(([nvcc, *COMPILE_FLAGS, *(extra_flags or []), *incs, "-c", src, "-o", obj], obj))
        workers = max(1, min(len(jobs), os.cpu_count() or 1))
        with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as ex:
            for f in [ex.submit(_run, cmd, verbose) for cmd, _ in jobs]:
                f.result()
        tmp_out = os.path.join(tmp, "lib.so")
        _run([nvcc, *LINK_FLAGS, "-o", tmp_out, *[o for _, o in jobs]], verbose)
        shutil.move(tmp_out, out)
    return out


if __name__ == "__main__":
    flags = sys.argv[1:]
    print(build(verbose=True, extra_flags=flags))
