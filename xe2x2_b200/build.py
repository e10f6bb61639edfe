"""Build libw4.so (all CUDA sources under csrc/) for sm_100a with nvcc.

The library is built in-tree (``xe2x2_b200/libw4.so``) so that it travels with
the repository to the machine that runs it.  A rebuild happens only when a
source or header is newer than the library.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libw4.so")
GENCODE = "arch=compute_100a,code=sm_100a"


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: libw4 cannot be built")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _inputs() -> list[str]:
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + [
        os.path.join(ROOT, "include", "w4.h"), os.path.abspath(__file__)]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _inputs())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [
        _nvcc(), "-O3", "-std=c++17", "-gencode", GENCODE, "-lineinfo",
        "-Xcompiler", "-fPIC", "-shared", "--threads", "0",
        "-I", os.path.join(ROOT, "include"),
        "-o", LIB + ".tmp",
    ]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    cmd += sources()
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("libw4 build failed:\n" + res.stdout + res.stderr)
    if verbose or ptxas_info:
        print(res.stdout + res.stderr, file=sys.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
