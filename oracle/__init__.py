"""ctypes wrapper of the oracle (oracle/liboracle.so) -- TEST INFRASTRUCTURE ONLY.

The oracle is a C restatement of the reference's CPU groupby path (see
oracle/oracle.h for the file:line map).  Only tests/, __graft_entry__.smoke()
and the CPU-baseline legs of bench.py use it, as the checker or as the timed
CPU baseline; the product (winrapids_b200/) never imports it.
"""
from __future__ import annotations

import ctypes as C
import math
from pathlib import Path

import numpy as np

from .build import LIB, build

# phi strings accepted by the reference's CPU evaluator (compute_engine.rs:593-609)
PHI_IDS = {
    "v": 0, "v * v": 1, "1.0": 2, "(v - r)": 3, "v - r": 3, "(v - r) * (v - r)": 4,
    "fabs(v - r)": 5, "abs(v - r)": 5, "(v - r) * (v - r) * (v - r)": 6,
    "(v - r) * (v - r) * (v - r) * (v - r)": 7, "v * r": 8, "log(v)": 9, "1.0 / v": 10,
}
PRED_IDS = {"gt": 0, "not_nan": 1, "finite": 2, "lt": 3, "ge": 4, "le": 5}
MAP2_IDS = {"a + b": 0, "a * b": 1, "a - b": 2, "a * b + 1.0": 3}


class OracleError(RuntimeError):
    pass


class _Moments(C.Structure):
    _fields_ = [(f, C.c_void_p) for f in ("counts", "sums", "mins", "maxs", "m2s", "m3s", "m4s")]


_L = None


def lib() -> C.CDLL:
    global _L
    if _L is not None:
        return _L
    build()
    L = C.CDLL(str(LIB))
    vp, i32, i64, f64, u64 = C.c_void_p, C.c_int32, C.c_int64, C.c_double, C.c_uint64
    sig = {
        "orc_exact_sum": (f64, [vp, i64]),
        "orc_scatter_phi": (C.c_int, [C.c_int, vp, vp, vp, i64, i32, vp]),
        "orc_scatter_multi_phi": (C.c_int, [vp, C.c_int, vp, vp, vp, i64, i32, vp]),
        "orc_scatter_phi_masked": (C.c_int, [C.c_int, vp, vp, vp, vp, i64, i32, vp]),
        "orc_scatter_extremum": (C.c_int, [C.c_int, vp, vp, i64, i32, vp]),
        "orc_nan_mask": (i64, [vp, i64, vp]),
        "orc_filter_mask": (None, [C.c_int, f64, vp, i64, vp]),
        "orc_map2": (None, [C.c_int, vp, vp, i64, vp]),
        "orc_mask_and": (None, [vp, vp, i64, vp]),
        "orc_mask_or": (None, [vp, vp, i64, vp]),
        "orc_mask_xor": (None, [vp, vp, i64, vp]),
        "orc_mask_not": (None, [vp, i64, i64, vp]),
        "orc_mask_popcount": (i64, [vp, i64]),
        "orc_tile_stats_build": (None, [vp, i64, i64, vp]),
        "orc_tile_skip": (None, [vp, i64, C.c_int, f64, vp]),
        "orc_bin_stats": (None, [vp, vp, i64, vp, vp, vp, vp, vp, vp, vp]),
        "orc_moments_grouped": (C.c_int, [vp, vp, i64, i32, C.POINTER(_Moments)]),
        "orc_moments_grouped_mt": (C.c_int, [vp, vp, vp, i64, i32, C.c_int, C.POINTER(_Moments)]),
        "orc_moments_grouped_masked": (C.c_int, [vp, vp, vp, i64, i32, C.POINTER(_Moments)]),
        "orc_groupby_i64": (i64, [vp, vp, vp, i64, vp, C.POINTER(_Moments)]),
        "orc_mean": (f64, [f64, f64]),
        "orc_variance": (f64, [f64, f64, C.c_int]),
        "orc_splitmix_at": (u64, [u64, u64]),
        "orc_mix64": (u64, [u64]),
        "orc_column_seed": (u64, [u64, C.c_uint32]),
        "orc_u01": (f64, [u64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _L = L
    return L


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f64(a):
    return np.ascontiguousarray(a, dtype=np.float64)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def _rc(rc):
    if rc == -1:
        raise IndexError("key out of range (the reference panics on this index)")
    if rc != 0:
        raise OracleError(f"oracle returned {rc}")


def exact_sum(x) -> float:
    x = _f64(x)
    return float(lib().orc_exact_sum(_p(x), x.size))


def phi_id(phi: str) -> int:
    try:
        return PHI_IDS[phi]
    except KeyError:
        raise OracleError(f"CPU: unsupported scatter phi '{phi}'") from None


def scatter_phi(phi, keys, values, refs, n_groups):
    k, v = _i32(keys), _f64(values)
    r = None if refs is None else _f64(refs)
    out = np.zeros(n_groups, np.float64)
    _rc(lib().orc_scatter_phi(phi_id(phi), _p(k), _p(v), _p(r), k.size, n_groups, _p(out)))
    return out


def scatter_multi_phi(phis, keys, values, refs, n_groups):
    ids = np.array([phi_id(p) for p in phis], dtype=np.int32)
    k, v = _i32(keys), _f64(values)
    r = None if refs is None else _f64(refs)
    out = np.zeros(len(phis) * n_groups, np.float64)
    _rc(lib().orc_scatter_multi_phi(_p(ids), len(phis), _p(k), _p(v), _p(r), k.size, n_groups, _p(out)))
    return [out[j * n_groups:(j + 1) * n_groups].copy() for j in range(len(phis))]


def scatter_phi_masked(phi, keys, values, refs, mask, n_groups):
    k, v = _i32(keys), _f64(values)
    r = None if refs is None else _f64(refs)
    m = np.ascontiguousarray(mask, dtype=np.uint64)
    out = np.zeros(n_groups, np.float64)
    _rc(lib().orc_scatter_phi_masked(phi_id(phi), _p(k), _p(v), _p(r), _p(m), k.size, n_groups, _p(out)))
    return out


def scatter_extremum(is_max, keys, values, n_groups):
    k, v = _i32(keys), _f64(values)
    out = np.zeros(n_groups, np.float64)
    _rc(lib().orc_scatter_extremum(1 if is_max else 0, _p(k), _p(v), k.size, n_groups, _p(out)))
    return out


def nan_mask(values):
    v = _f64(values)
    m = np.zeros(max(1, (v.size + 63) // 64), np.uint64)
    n_nan = lib().orc_nan_mask(_p(v), v.size, _p(m))
    return m[: (v.size + 63) // 64], int(n_nan)


def filter_mask(pred, threshold, values):
    v = _f64(values)
    m = np.zeros(max(1, (v.size + 63) // 64), np.uint64)
    lib().orc_filter_mask(PRED_IDS[pred], float(threshold), _p(v), v.size, _p(m))
    return m[: (v.size + 63) // 64]


def _words(m):
    return np.ascontiguousarray(m, dtype=np.uint64)


def mask_and(a, b):
    """mask_and (filter_jit.rs:151-154)."""
    a, b = _words(a), _words(b)
    if a.size != b.size:
        raise ValueError("mask_and: length mismatch")
    out = np.empty_like(a)
    lib().orc_mask_and(_p(a), _p(b), a.size, _p(out))
    return out


def mask_or(a, b):
    """mask_or (filter_jit.rs:157-160)."""
    a, b = _words(a), _words(b)
    if a.size != b.size:
        raise ValueError("mask_or: length mismatch")
    out = np.empty_like(a)
    lib().orc_mask_or(_p(a), _p(b), a.size, _p(out))
    return out


def mask_xor(a, b):
    """mask_xor (filter_jit.rs:163-166)."""
    a, b = _words(a), _words(b)
    if a.size != b.size:
        raise ValueError("mask_xor: length mismatch")
    out = np.empty_like(a)
    lib().orc_mask_xor(_p(a), _p(b), a.size, _p(out))
    return out


def mask_not(m, n_rows):
    """mask_not (filter_jit.rs:173-181)."""
    m = _words(m)
    if n_rows % 64 and n_rows // 64 >= m.size:
        raise IndexError("mask_not: n_rows beyond the mask")
    out = np.empty_like(m)
    lib().orc_mask_not(_p(m), m.size, int(n_rows), _p(out))
    return out


def mask_popcount(m, n_rows):
    """mask_popcount (filter_jit.rs:130-144)."""
    m = _words(m)
    if (n_rows + 63) // 64 > m.size:
        raise IndexError("mask_popcount: n_rows beyond the mask")
    return int(lib().orc_mask_popcount(_p(m), int(n_rows)))


TILE_STATS_DTYPE = np.dtype([("min", "<f8"), ("max", "<f8"), ("sum", "<f8"), ("count", "<u4"),
                             ("n_valid", "<u4"), ("reserved", "<u8")])


def tile_stats(values, tile_rows):
    """TileColumnStats::from_slice (format.rs:82-107) of every tile of tile_rows rows."""
    v = _f64(values)
    n_tiles = (v.size + tile_rows - 1) // tile_rows
    out = np.zeros(max(1, n_tiles), TILE_STATS_DTYPE)
    lib().orc_tile_stats_build(_p(v), v.size, int(tile_rows), _p(out))
    return out[:n_tiles]


def tile_skip(stats, pred, threshold):
    """can_skip_gt / _gte / _lt / _lte (format.rs:111-136): 1 where the tile can be skipped."""
    st = np.ascontiguousarray(stats, dtype=TILE_STATS_DTYPE)
    out = np.zeros(max(1, st.size), np.uint8)
    lib().orc_tile_skip(_p(st), st.size, PRED_IDS[pred], float(threshold), _p(out))
    return out[: st.size]


def bin_stats(data, boundaries):
    """fused_bin_stats (bin_stats.cu:25-77) plus the Python wrapper's derived mean / variance /
    std (archive/fintek-contributions/src/fused_bin_stats.py:121-127), serial per bin."""
    d = _f64(data)
    b = np.ascontiguousarray(boundaries, dtype=np.int64)
    nb = max(b.size - 1, 0)
    out = {k: np.zeros(max(nb, 1)) for k in ("sum", "sum_sq", "min", "max", "first", "last")}
    cnt = np.zeros(max(nb, 1), np.int32)
    if nb:
        lib().orc_bin_stats(_p(d), _p(b), nb, _p(out["sum"]), _p(out["sum_sq"]), _p(out["min"]), _p(out["max"]),
                            _p(out["first"]), _p(out["last"]), _p(cnt))
    res = {k: v[:nb] for k, v in out.items()}
    res["count"] = cnt[:nb]
    c = res["count"].astype(np.float64)
    with np.errstate(invalid="ignore", divide="ignore"):
        mean = np.where(c > 0, res["sum"] / np.where(c > 0, c, 1.0), np.nan)
        var = np.where(c > 1, res["sum_sq"] / np.where(c > 0, c, 1.0) - mean * mean, np.nan)
        var = np.where(var < 0.0, 0.0, var)
    res["mean"], res["variance"], res["std"] = mean, var, np.sqrt(var)
    return res


def _fmin(a, b):
    """Rust f64::min: the other operand when one is NaN."""
    if a != a:
        return b
    if b != b:
        return a
    return a if a < b else b


def _fmax(a, b):
    if a != a:
        return b
    if b != b:
        return a
    return a if a > b else b


def tile_global_stats(stats):
    """global_min / global_max / global_sum / global_count / global_mean (format.rs:144-175):
    header-only folds over the tiles (min / max over tiles with n_valid > 0)."""
    mn, mx, s, c = math.inf, -math.inf, 0.0, 0
    for t in stats:
        if int(t["n_valid"]) > 0:
            mn = _fmin(mn, float(t["min"]))
            mx = _fmax(mx, float(t["max"]))
        s += float(t["sum"])
        c += int(t["count"])
    return {"min": mn, "max": mx, "sum": s, "count": c, "mean": (s / c) if c else math.nan}


def map2(expr, a, b):
    a, b = _f64(a), _f64(b)
    out = np.empty_like(a)
    lib().orc_map2(MAP2_IDS[expr], _p(a), _p(b), a.size, _p(out))
    return out


def _alloc(n, m34):
    arrs = {f: np.zeros(n, np.float64) for f in ("counts", "sums", "mins", "maxs", "m2s")}
    if m34:
        arrs["m3s"] = np.zeros(n, np.float64)
        arrs["m4s"] = np.zeros(n, np.float64)
    s = _Moments()
    for f in ("counts", "sums", "mins", "maxs", "m2s", "m3s", "m4s"):
        setattr(s, f, _p(arrs.get(f)))
    return arrs, s


def moments_grouped(values, keys, n_groups, m34=True):
    """DescriptiveEngine::moments_grouped, composed through the scatter primitives."""
    v, k = _f64(values), _i32(keys)
    arrs, s = _alloc(n_groups, m34)
    _rc(lib().orc_moments_grouped(_p(v), _p(k), v.size, n_groups, C.byref(s)))
    return arrs


def moments_grouped_mt(values, keys, n_groups, threads=8, mask=None, m34=False):
    """Same bits as moments_grouped (per-thread Kulisch registers merged in range order)."""
    v, k = _f64(values), _i32(keys)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint64)
    arrs, s = _alloc(n_groups, m34)
    _rc(lib().orc_moments_grouped_mt(_p(v), _p(k), _p(m), v.size, n_groups, int(threads), C.byref(s)))
    return arrs


def moments_grouped_masked(values, keys, mask, n_groups, m34=False):
    v, k = _f64(values), _i32(keys)
    m = np.ascontiguousarray(mask, dtype=np.uint64)
    arrs, s = _alloc(n_groups, m34)
    _rc(lib().orc_moments_grouped_masked(_p(v), _p(k), _p(m), v.size, n_groups, C.byref(s)))
    return arrs


def groupby_i64(keys, values, mask=None, m34=False):
    k = np.ascontiguousarray(keys, dtype=np.int64)
    v = _f64(values)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint64)
    out_keys = np.zeros(max(1, k.size), np.int64)
    arrs, s = _alloc(max(1, k.size), m34)
    ng = int(lib().orc_groupby_i64(_p(k), _p(v), _p(m), k.size, _p(out_keys), C.byref(s)))
    res = {f: a[:ng].copy() for f, a in arrs.items()}
    res["keys"] = out_keys[:ng].copy()
    return res


def group_index_build(keys, max_key):
    """GroupIndex::build (group_index.rs:117-204) in numpy: row_to_group, group_counts,
    group_offsets (with the n sentinel), rows_by_group (stable by group), n_active."""
    k = np.ascontiguousarray(keys, dtype=np.int32)
    G = int(max_key) + 1
    counts = np.bincount(k, minlength=G).astype(np.uint32)
    offsets = np.zeros(G + 1, dtype=np.uint32)
    offsets[1:] = np.cumsum(counts, dtype=np.uint64).astype(np.uint32)
    return {"row_to_group": k.astype(np.uint32), "group_counts": counts, "group_offsets": offsets,
            "rows_by_group": np.argsort(k, kind="stable").astype(np.uint32),
            "n_active": int(np.count_nonzero(counts))}


def factorize_first_seen(keys):
    """Dictionary::encode (dictionary.rs:40-75) over a key column: codes in first-seen order."""
    k = np.ascontiguousarray(keys, dtype=np.int64)
    uniq, first, inv = np.unique(k, return_index=True, return_inverse=True)
    order = np.argsort(first, kind="stable")
    rank = np.empty_like(order)
    rank[order] = np.arange(order.size)
    return rank[inv].astype(np.int32), uniq[order]


def mean(count, total):
    return float(lib().orc_mean(float(count), float(total)))


def variance(count, m2, ddof):
    return float(lib().orc_variance(float(count), float(m2), int(ddof)))


def derived(mom):
    """Mean / var_pop / var_samp arrays from a moments dict (MomentStats, descriptive.rs:97-114)."""
    c, s, m2 = mom["counts"], mom["sums"], mom["m2s"]
    with np.errstate(invalid="ignore", divide="ignore"):
        mean_ = np.where(c == 0.0, np.nan, s / np.where(c == 0.0, 1.0, c))
        vp = np.where(c - 0.0 <= 0.0, np.nan, m2 / np.where(c <= 0.0, 1.0, c))
        vs = np.where(c - 1.0 <= 0.0, np.nan, m2 / np.where(c - 1.0 <= 0.0, 1.0, c - 1.0))
    return {"mean": mean_, "var_pop": vp, "var_samp": vs}


# ---- counter-based SplitMix64 streams (rng.rs:64-85), vectorised in numpy ----------
_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_SALT = 0xD1B54A32D192ED03
M64 = (1 << 64) - 1


def mix64_np(z: np.ndarray) -> np.ndarray:
    z = z.astype(np.uint64, copy=True)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def mix64_int(z: int) -> int:
    z &= M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def column_seed(seed: int, column: int) -> int:
    return mix64_int((seed & M64) ^ ((_SALT * (column + 1)) & M64))


def splitmix_stream(seed: int, start: int, count: int) -> np.ndarray:
    i = np.arange(start + 1, start + count + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return mix64_np(np.uint64(seed & M64) + i * _GAMMA)


def u01_np(x: np.ndarray) -> np.ndarray:
    return (x >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def gen_keys_uniform(n, n_groups, seed, start=0):
    return (splitmix_stream(column_seed(seed, 0), start, n) % np.uint64(n_groups)).astype(np.int32)


def gen_values_uniform(n, lo, hi, seed, start=0):
    return lo + (hi - lo) * u01_np(splitmix_stream(column_seed(seed, 1), start, n))


def gen_values_normal(n, mu, sigma, seed, start=0):
    x = splitmix_stream(column_seed(seed, 1), 2 * start, 2 * n)
    u1 = u01_np(x[0::2])
    u2 = u01_np(x[1::2])
    u1 = np.where(u1 <= 0.0, 1.0 / 9007199254740992.0, u1)
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos((2.0 * np.pi) * u2)
    return mu + sigma * z


def zipf_cdf(n_ids, s):
    """Inverse-CDF table of Zipf(s) over ranks 0..n_ids-1 (p(r) ~ (r+1)^-s); last entry exactly 1.0."""
    w = np.arange(1, n_ids + 1, dtype=np.float64) ** (-float(s))
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    cdf[-1] = 1.0
    return cdf


def gen_keys_cdf(n, cdf, salt, seed, start=0):
    u = u01_np(splitmix_stream(column_seed(seed, 0), start, n))
    rank = np.searchsorted(cdf, u, side="left").astype(np.uint64)
    return mix64_np(rank ^ np.uint64(salt & M64)).view(np.int64)


def gen_keys_ids(n, n_ids, salt, seed, start=0):
    x = splitmix_stream(column_seed(seed, 0), start, n) % np.uint64(n_ids)
    return mix64_np(x ^ np.uint64(salt & M64)).view(np.int64)


def gen_values_lognormal_f32(n, mu, sigma, seed, start=0):
    return np.exp(gen_values_normal(n, mu, sigma, seed, start)).astype(np.float32)


def inject_nonfinite(vals, nan_frac, inf_frac, seed, start=0):
    x = splitmix_stream(column_seed(seed, 2), start, vals.size)
    u = u01_np(x)
    out = vals.copy()
    out[u < nan_frac] = np.nan
    inf_pos = (u >= nan_frac) & (u < nan_frac + inf_frac)
    out[inf_pos] = np.where((x[inf_pos] & np.uint64(1)) == 1, -np.inf, np.inf)
    return out
