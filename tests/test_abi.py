"""The C-ABI library loads and exports every symbol include/tambear_gb.h declares (CPU only)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "tambear_gb.h"


def header_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tbgb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def libpath():
    from winrapids_b200 import build

    return build.build()


def test_header_declares_entry_points():
    fns = header_functions()
    assert "tbgb_groupby_dense" in fns and "tbgb_merge_states" in fns
    from winrapids_b200._lib import HEADER_SYMBOLS

    assert sorted(HEADER_SYMBOLS) == fns


def test_library_exports_every_header_symbol(libpath):
    lib = ctypes.CDLL(str(libpath))
    for name in header_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(libpath)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (tbgb_\w+)", out))
    assert set(header_functions()) <= exported


def test_create_without_gpu_fails_loudly(libpath):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import winrapids_b200 as wb

    with pytest.raises(wb.TambearGbError):
        wb.Context(0)


def test_no_oracle_in_product():
    for p in (ROOT / "winrapids_b200").rglob("*"):
        if p.suffix in (".py", ".cu", ".cuh", ".cpp", ".hpp", ".h"):
            text = p.read_text()
            assert "import oracle" not in text and "from oracle" not in text and "liboracle" not in text, p


def test_state_bytes_without_gpu(libpath):
    from winrapids_b200._lib import lib

    assert lib().tbgb_state_bytes(256) == 11 * 256 * 8  # 11 state fields per group
    assert lib().tbgb_state_bytes(0) == 0


def test_rust_bindings_declare_every_header_symbol():
    """rust/src/ffi.rs (the Rust side of the boundary, not compiled here: no Rust toolchain)
    declares every entry point of the header, and the backend names every dispatched entry."""
    ffi = (ROOT / "rust" / "src" / "ffi.rs").read_text()
    declared = set(re.findall(r"pub fn (tbgb_\w+)\s*\(", ffi))
    assert declared == set(header_functions()), sorted(set(header_functions()) ^ declared)
    backend = (ROOT / "rust" / "src" / "backend.rs").read_text()
    for entry in ("scatter_phi", "scatter_multi_phi", "scatter_phi_masked", "scatter_extremum"):
        assert f'"{entry}"' in backend, entry
