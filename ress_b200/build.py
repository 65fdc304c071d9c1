"""Builds libress_sm100.so in-tree with nvcc for sm_100a.

Run as ``python -m ress_b200.build`` (or through ``__graft_entry__.build()``).
The library is the product's only compute path; nothing else is compiled
at import time."""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = [os.path.join(HERE, "csrc", f) for f in ("capi.cu", "score.cu", "select.cu", "attn.cu", "noalloc.cu",
                                                "prologue.cu")]
OUT = os.path.join(HERE, "libress_sm100.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-shared",
    "-I", os.path.join(ROOT, "include"),
]


def needs_build() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = SRC + [os.path.join(HERE, "csrc", "common.cuh"), os.path.join(ROOT, "include", "ress_sm100.h")]
    return any(os.path.getmtime(p) > t for p in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    cmd = [NVCC, *FLAGS, *SRC, "-o", OUT]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(verbose=True, ptxas_info="-v" in sys.argv)
