"""Build the sm_100a groupby library in-tree: winrapids_b200/libtambear_gb.so.

Every CUDA source is compiled with ``nvcc -gencode arch=compute_100a,code=sm_100a``;
objects go to winrapids_b200/_build/ and are rebuilt when a source or header is
newer than its object.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libtambear_gb.so"

SOURCES = ["dense.cu", "table.cu", "partition.cu", "phi.cu", "sort.cu", "group_index.cu", "mask.cu", "bin_stats.cu", "exchange.cu", "gen.cu", "radix.cu", "noalloc.cu", "api.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(INCLUDE), "-I", str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _headers() -> list[Path]:
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp")) + list(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    headers = _headers()
    objs = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD / (src + ".o")
        objs.append(o)
        if _stale(o, [s] + headers) or ptxas_info:
            cmd = [cc, *ARCH, *COMMON, "-c", str(s), "-o", str(o)]
            if ptxas_info and src.endswith(".cu"):
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            subprocess.run(cmd, check=True)
    if _stale(LIB, objs):
        cmd = [cc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB)
