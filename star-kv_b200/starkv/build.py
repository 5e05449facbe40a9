"""Build ``libstarkv.so`` in-tree with nvcc for sm_100a (no torch extension machinery:
the library exports a plain C ABI and links only the CUDA runtime)."""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(PKG))
CSRC = os.path.join(os.path.dirname(PKG), "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUT = os.path.join(PKG, "libstarkv.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh")))


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/starkv_abi.cu into starkv/libstarkv.so unless it is newer than every source."""
    srcs = sources() + [os.path.join(INCLUDE, "starkv.h")]
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= max(os.path.getmtime(s) for s in srcs):
        return OUT
    tmp = OUT + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-o", tmp, os.path.join(CSRC, "starkv_abi.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
