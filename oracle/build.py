"""Build recipe for the oracle (test infrastructure): oracle/liboracle.so.

gcc, -ffp-contract=off so every f64 operation rounds separately, as the
reference's Rust code does.  The reference itself (Rust) cannot be compiled
here, so there is no oracle/_ref build.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
SRC = [HERE / "oracle.c"]


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
