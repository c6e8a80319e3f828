"""Build recipe for the oracle (test infrastructure): oracle/liboracle.so.

gcc, -ffp-contract=off so every f64 operation rounds separately, as the
reference's Rust code does.  The reference's Rust crates cannot be compiled here
(no Rust toolchain).  Its CUDA bin-statistics kernels
(src/winrapids/kernels/bin_stats.cu) compile with nvcc from where they lie: when
the reference tree is present, build_ref() compiles them with the launchers of
oracle/ref_bin_stats.cu into oracle/_ref/libref_bin_stats.so, which the GPU tests
run beside the product kernel (the built library travels with the repository;
the reference tree does not).  The reference's hash-scatter groupby kernels
(scatter_stats, scatter_stats_smem, scatter_stats_warp) are CUDA C held in a Rust raw
string (crates/tambear/src/hash_scatter.rs, SCATTER_CUDA_SOURCE); build_ref() cuts that
string out of the file at build time into oracle/_ref/hash_scatter_kernels.cu and
compiles it with the launchers of oracle/ref_hash_scatter.cu into
oracle/_ref/libref_hash_scatter.so.

The reference tree is found at the path given by --reference-root, else the
REFERENCE_ROOT environment variable, else the container's read-only mount point.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
SRC = [HERE / "oracle.c"]


DEFAULT_REF_ROOT = "/root/reference"  # where this container mounts the reference tree (read-only)
REF_DIR = HERE / "_ref"
REF_BIN_LIB = REF_DIR / "libref_bin_stats.so"
REF_HS_LIB = REF_DIR / "libref_hash_scatter.so"
REF_HS_SRC = REF_DIR / "hash_scatter_kernels.cu"  # generated: the raw string cut out of hash_scatter.rs


def ref_root(path: str | None = None) -> Path:
    return Path(path or os.environ.get("REFERENCE_ROOT") or DEFAULT_REF_ROOT)


def _nvcc_shared(out: Path, launcher: Path, define: str, verbose: bool) -> None:
    cmd = ["nvcc", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-gencode", "arch=compute_100a,code=sm_100a", define, "-o", str(out), str(launcher)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)


def _fresh(target: Path, deps) -> bool:
    return target.exists() and all(d.stat().st_mtime <= target.stat().st_mtime for d in deps)


def cut_raw_string(rust_file: Path, const_name: str) -> str:
    """The body of `const <const_name>: &str = r#"...";` in a Rust source file."""
    text = rust_file.read_text()
    head = f"const {const_name}: &str = r#\""
    i = text.index(head) + len(head)
    j = text.index('"#;', i)
    return text[i:j]


def build_ref(verbose: bool = False, root: str | None = None) -> Path | None:
    """oracle/_ref/libref_bin_stats.so and oracle/_ref/libref_hash_scatter.so from the reference's
    kernel sources (returns the bin-statistics library; None when the reference tree is absent
    and nothing was built before)."""
    base = ref_root(root)
    bin_stats = base / "src" / "winrapids" / "kernels" / "bin_stats.cu"
    hash_rs = base / "crates" / "tambear" / "src" / "hash_scatter.rs"
    if bin_stats.exists():
        launcher = HERE / "ref_bin_stats.cu"
        if not _fresh(REF_BIN_LIB, [launcher, bin_stats]):
            REF_DIR.mkdir(exist_ok=True)
            _nvcc_shared(REF_BIN_LIB, launcher, f'-DREF_BIN_STATS_CU="{bin_stats}"', verbose)
    if hash_rs.exists():
        launcher = HERE / "ref_hash_scatter.cu"
        if not _fresh(REF_HS_LIB, [launcher, hash_rs]):
            REF_DIR.mkdir(exist_ok=True)
            REF_HS_SRC.write_text(cut_raw_string(hash_rs, "SCATTER_CUDA_SOURCE"))
            _nvcc_shared(REF_HS_LIB, launcher, f'-DREF_HASH_SCATTER_CU="{REF_HS_SRC}"', verbose)
    return REF_BIN_LIB if REF_BIN_LIB.exists() else None


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
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", default=None)
    args = ap.parse_args()
    print(build(verbose=True))
    print(build_ref(verbose=True, root=args.reference_root))
