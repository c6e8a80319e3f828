"""Build recipe for the oracle (test infrastructure): oracle/liboracle.so.

gcc, -ffp-contract=off so every f64 operation rounds separately, as the
reference's Rust code does.  The reference's Rust crates cannot be compiled here
(no Rust toolchain).  Its CUDA bin-statistics kernels
(src/winrapids/kernels/bin_stats.cu) compile with nvcc from where they lie: when
the reference tree is present, build_ref() compiles them with the launchers of
oracle/ref_bin_stats.cu into oracle/_ref/libref_bin_stats.so, which the GPU tests
run beside the product kernel (the built library travels with the repository;
the reference tree does not).
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
SRC = [HERE / "oracle.c"]


REF_ROOT = Path("/root/reference")
REF_BIN_STATS = REF_ROOT / "src" / "winrapids" / "kernels" / "bin_stats.cu"
REF_DIR = HERE / "_ref"
REF_BIN_LIB = REF_DIR / "libref_bin_stats.so"


def build_ref(verbose: bool = False) -> Path | None:
    """oracle/_ref/libref_bin_stats.so from the reference's kernel source (None when the
    reference tree is absent and nothing was built before)."""
    if not REF_BIN_STATS.exists():
        return REF_BIN_LIB if REF_BIN_LIB.exists() else None
    launcher = HERE / "ref_bin_stats.cu"
    deps = [launcher, REF_BIN_STATS]
    if REF_BIN_LIB.exists() and all(d.stat().st_mtime <= REF_BIN_LIB.stat().st_mtime for d in deps):
        return REF_BIN_LIB
    REF_DIR.mkdir(exist_ok=True)
    cmd = ["nvcc", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-gencode", "arch=compute_100a,code=sm_100a", f'-DREF_BIN_STATS_CU="{REF_BIN_STATS}"',
           "-o", str(REF_BIN_LIB), str(launcher)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    return REF_BIN_LIB


def build(verbose: bool = False) -> Path:
    deps = SRC + [HERE / "oracle.h"]
    if LIB.exists() and all(d.stat().st_mtime <= LIB.stat().st_mtime for d in deps):
        return LIB
    cmd = ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
           "-o", str(LIB), *map(str, SRC), "-lm", "-lpthread"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
    print(build_ref(verbose=True))
