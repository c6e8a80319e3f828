"""ctypes binding of include/tambear_gb.h (libtambear_gb.so, built in-tree for sm_100a).

There is no fallback: if the library is missing or no sm_100 device is present,
every entry point raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtambear_gb.so"

STATUS_NAMES = {
    0: "OK",
    1: "Backend",
    2: "Compile",
    3: "Alloc",
    4: "Transfer",
    5: "Dispatch",
    6: "EntryNotFound",
    7: "InvalidArgument",
    8: "KeyOutOfRange",
    9: "TableFull",
    10: "Timeout",
}


class TambearGbError(RuntimeError):
    """A non-OK tbgb_status; `.status` is the numeric code, `.kind` its name."""

    def __init__(self, status: int, message: str):
        self.status = status
        self.kind = STATUS_NAMES.get(status, f"status{status}")
        super().__init__(f"{self.kind}: {message}")


class KeyOutOfRange(TambearGbError):
    pass


class InvalidArgument(TambearGbError):
    pass


class EntryNotFound(TambearGbError):
    pass


def error_for(status: int, message: str) -> TambearGbError:
    if status == 8:
        return KeyOutOfRange(status, message)
    if status == 7:
        return InvalidArgument(status, message)
    if status == 9:
        return TableFull(status, message)
    if status == 6:
        return EntryNotFound(status, message)
    return TambearGbError(status, message)


class TableFull(TambearGbError):
    pass


class Columns(C.Structure):
    """tbgb_columns: value columns a, b, c with the fused expression and filter."""

    _fields_ = [("a", C.c_void_p), ("b", C.c_void_p), ("c", C.c_void_p), ("dtype", C.c_int32),
                ("expr", C.c_int32), ("pred", C.c_int32), ("reserved", C.c_int32), ("threshold", C.c_double)]


DTYPES = {"f64": 0, "f32": 1}
PREDS = {None: 0, "none": 0, ">": 1, ">=": 2, "<": 3, "<=": 4, "not_nan": 5, "finite": 6}
EXPRS = {"a": 0, "a+b": 1, "a-b": 2, "a*b": 3, "a*b+1": 4, "a*b+c": 5}


class Moments(C.Structure):
    _fields_ = [(name, C.c_void_p) for name in
                ("count", "sum", "min", "max", "mean", "m2", "var_pop", "var_samp", "m3", "m4")]


# The grouped moments computed by default; m3 / m4 (HIGHER_FIELDS) cost a little more and are
# computed only when their outputs are requested.
MOMENT_FIELDS = ("count", "sum", "min", "max", "mean", "m2", "var_pop", "var_samp")
HIGHER_FIELDS = ("m3", "m4")

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python winrapids_b200/build.py`")
    L = C.CDLL(str(LIB_PATH))
    vp, i32, i64, u64, f64, sz = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64, C.c_double, C.c_size_t
    st = C.c_int
    sig = {
        "tbgb_create": (st, [C.c_int, C.POINTER(vp)]),
        "tbgb_destroy": (None, [vp]),
        "tbgb_last_error": (C.c_char_p, [vp]),
        "tbgb_device_name": (C.c_char_p, [vp]),
        "tbgb_groupby_dense": (st, [vp, vp, vp, vp, i64, i32, C.POINTER(Moments), vp]),
        "tbgb_sync": (st, [vp, vp]),
        "tbgb_groupby_dense_noalloc": (st, [vp, vp, vp, i64, i32, C.POINTER(Moments), vp]),
        "tbgb_state_bytes": (sz, [i32]),
        "tbgb_groupby_dense_state": (st, [vp, vp, vp, vp, i64, i32, i64, vp, vp]),
        "tbgb_merge_states": (st, [vp, vp, i32, i32, C.POINTER(Moments), vp]),
        "tbgb_workspace_bytes": (sz, [vp, i64, i32]),
        "tbgb_launch_count": (u64, [vp]),
        "tbgb_profile_enable": (st, [vp, C.c_int]),
        "tbgb_kernel_time_ms": (st, [vp, C.POINTER(f64), C.POINTER(i64)]),
        "tbgb_groupby_dense_columns": (st, [vp, vp, C.POINTER(Columns), vp, i64, i32, C.POINTER(Moments), vp]),
        "tbgb_groupby_hash": (st, [vp, vp, C.POINTER(Columns), vp, i64, i64, vp, C.POINTER(Moments), vp, vp]),
        "tbgb_set_table_mode": (st, [vp, C.c_int]),
        "tbgb_hash_partition": (st, [vp, vp, C.POINTER(Columns), vp, i64, i32, vp, vp, vp, vp]),
        "tbgb_radix_value_bytes": (i32, [C.POINTER(Columns)]),
        "tbgb_radix_fallback": (st, [vp, C.POINTER(C.c_uint32)]),
        "tbgb_radix_route": (st, [vp, vp, C.POINTER(Columns), vp, i64, vp, vp, vp, vp]),
        "tbgb_radix_groupby_routed": (st, [vp, i32, C.POINTER(vp), C.POINTER(vp), C.POINTER(i64), i32, vp, i32,
                                           i32, i64, vp, C.POINTER(Moments), vp, vp]),
        "tbgb_scatter_multi_phi_masked": (st, [vp, C.POINTER(i32), i32, vp, vp, vp, vp, i64, i32, vp, vp]),
        "tbgb_scatter_phi": (st, [vp, i32, vp, vp, vp, i64, i32, vp, vp]),
        "tbgb_scatter_multi_phi": (st, [vp, C.POINTER(i32), i32, vp, vp, vp, i64, i32, vp, vp]),
        "tbgb_scatter_phi_masked": (st, [vp, i32, vp, vp, vp, vp, i64, i32, vp, vp]),
        "tbgb_scatter_extremum": (st, [vp, i32, vp, vp, i64, i32, vp, vp]),
        "tbgb_group_index_build": (st, [vp, vp, i64, i32, vp, vp, vp, vp, vp, vp]),
        "tbgb_factorize_i64": (st, [vp, vp, i64, i64, vp, vp, vp, vp]),
        "tbgb_filter_mask": (st, [vp, vp, i32, i64, i32, f64, vp, vp, vp]),
        "tbgb_mask_and": (st, [vp, vp, vp, vp, i64, vp]),
        "tbgb_mask_or": (st, [vp, vp, vp, vp, i64, vp]),
        "tbgb_mask_xor": (st, [vp, vp, vp, vp, i64, vp]),
        "tbgb_mask_not": (st, [vp, vp, vp, i64, i64, vp]),
        "tbgb_mask_popcount": (st, [vp, vp, i64, i64, vp, vp]),
        "tbgb_tile_stats_build": (st, [vp, vp, i32, i64, i64, vp, vp]),
        "tbgb_tile_skip_mask": (st, [vp, vp, i64, i32, f64, vp, vp]),
        "tbgb_mask_skip_tiles": (st, [vp, vp, vp, i64, i64, vp, vp]),
        "tbgb_fused_bin_stats": (st, [vp, vp, i64, i32, vp, i64, vp, vp]),
        "tbgb_exchange_bytes": (C.c_size_t, [i32, i32]),
        "tbgb_exchange_alloc": (st, [vp, i32, i32, C.POINTER(vp)]),
        "tbgb_exchange_free": (st, [vp, vp]),
        "tbgb_peer_export": (st, [vp, vp, vp]),
        "tbgb_peer_import": (st, [vp, vp, C.POINTER(vp)]),
        "tbgb_peer_close": (st, [vp, vp]),
        "tbgb_ipc_alloc": (st, [vp, sz, C.POINTER(vp)]),
        "tbgb_ipc_free": (st, [vp, vp]),
        "tbgb_groupby_dense_sharded": (st, [vp, vp, vp, vp, i64, i32, i64, i32, i32, vp, u64, vp, vp]),
        "tbgb_gen_keys_uniform": (st, [vp, vp, i64, i32, u64, i64, vp]),
        "tbgb_gen_values_uniform": (st, [vp, vp, i64, f64, f64, u64, i64, vp]),
        "tbgb_gen_values_normal": (st, [vp, vp, i64, f64, f64, u64, i64, vp]),
        "tbgb_gen_inject_nonfinite": (st, [vp, vp, i64, f64, f64, u64, i64, vp]),
        "tbgb_gen_keys_cdf": (st, [vp, vp, i64, vp, i64, u64, u64, i64, vp]),
        "tbgb_gen_keys_ids": (st, [vp, vp, i64, i64, u64, u64, i64, vp]),
        "tbgb_gen_values_lognormal_f32": (st, [vp, vp, i64, f64, f64, u64, i64, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


# Every symbol include/tambear_gb.h declares (checked by the CPU test suite).
HEADER_SYMBOLS = (
    "tbgb_create", "tbgb_destroy", "tbgb_last_error", "tbgb_device_name", "tbgb_groupby_dense", "tbgb_sync",
    "tbgb_groupby_dense_noalloc",
    "tbgb_state_bytes", "tbgb_groupby_dense_state", "tbgb_merge_states", "tbgb_workspace_bytes",
    "tbgb_launch_count", "tbgb_profile_enable", "tbgb_kernel_time_ms", "tbgb_gen_keys_uniform", "tbgb_gen_values_uniform", "tbgb_gen_values_normal",
    "tbgb_gen_inject_nonfinite", "tbgb_groupby_dense_columns", "tbgb_groupby_hash", "tbgb_set_table_mode",
    "tbgb_gen_keys_cdf", "tbgb_gen_keys_ids", "tbgb_gen_values_lognormal_f32", "tbgb_hash_partition",
    "tbgb_scatter_multi_phi_masked", "tbgb_scatter_phi", "tbgb_scatter_multi_phi", "tbgb_scatter_phi_masked",
    "tbgb_scatter_extremum", "tbgb_group_index_build", "tbgb_factorize_i64",
    "tbgb_filter_mask", "tbgb_mask_and", "tbgb_mask_or", "tbgb_mask_xor", "tbgb_mask_not", "tbgb_mask_popcount",
    "tbgb_tile_stats_build", "tbgb_tile_skip_mask", "tbgb_mask_skip_tiles", "tbgb_fused_bin_stats",
    "tbgb_exchange_bytes", "tbgb_exchange_alloc", "tbgb_exchange_free", "tbgb_peer_export", "tbgb_peer_import",
    "tbgb_peer_close", "tbgb_groupby_dense_sharded", "tbgb_radix_value_bytes", "tbgb_radix_route",
    "tbgb_radix_groupby_routed", "tbgb_radix_fallback", "tbgb_ipc_alloc", "tbgb_ipc_free",
)

# tbgb_bin_stats field order
BIN_STATS_FIELDS = ("count", "sum", "sum_sq", "min", "max", "first", "last", "mean", "variance", "std")


class BinStats(C.Structure):
    _fields_ = [(f, C.c_void_p) for f in BIN_STATS_FIELDS]

# TileColumnStats (format.rs:60-73) as laid out by tbgb_tile_stats: 40 bytes
TILE_STATS_FIELDS = (("min", "f8"), ("max", "f8"), ("sum", "f8"), ("count", "u4"), ("n_valid", "u4"),
                     ("reserved", "u8"))
TILE_STATS_BYTES = 40

# phi expressions by the reference's source spelling (phi_scatter_eval, compute_engine.rs:593-609)
PHI_IDS = {"v": 0, "v * v": 1, "1.0": 2, "v - r": 3, "(v - r)": 3, "(v - r) * (v - r)": 4, "fabs(v - r)": 5,
           "abs(v - r)": 5, "(v - r) * (v - r) * (v - r)": 6, "(v - r) * (v - r) * (v - r) * (v - r)": 7,
           "v * r": 8, "log(v)": 9, "1.0 / v": 10}
