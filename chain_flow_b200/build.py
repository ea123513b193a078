"""Build libcfb.so (the sm_100a engine) in-tree with nvcc.

    python -m chain_flow_b200.build          # or: python chain_flow_b200/build.py

The shared library lands next to this file (chain_flow_b200/libcfb.so) so it travels with the
source tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libcfb.so"
SOURCES = ["cfb_engine.cu", "cfb_pack.cu", "cfb_gdn.cu", "cfb_wide.cu", "cfb_ring.cu", "cfb_tree.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libcfb.so")
    return cand


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
                    f"-I{INCLUDE}", "-lcudart"]
    if ptxas_info:
        flags += ["-Xptxas", "-v"]
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *flags, *[str(CSRC / s) for s in SOURCES], "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv, ptxas_info="--ptxas" in sys.argv)
    print(f"built {LIB}")
