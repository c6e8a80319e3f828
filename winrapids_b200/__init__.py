"""B200 (sm_100a) groupby-aggregate path of the WinRapids/Tambear dataframe engine.

Two layers:

* ``Context`` -- thin wrapper over the C ABI (include/tambear_gb.h) working on
  device tensors (torch is used only for device memory and streams);
* the reference's operator API, same names and meaning:
  ``DescriptiveEngine.moments_grouped`` -> ``GroupedMomentStats`` / ``MomentStats``
  (crates/tambear/src/descriptive.rs:67-435).
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import numpy as np

from ._lib import (BIN_STATS_FIELDS, DTYPES, EXPRS, HIGHER_FIELDS, MOMENT_FIELDS, PREDS, TILE_STATS_BYTES,
                   TILE_STATS_FIELDS, BinStats, Columns,
                   EntryNotFound, InvalidArgument, KeyOutOfRange, Moments, TableFull, TambearGbError, error_for, lib)

__all__ = [
    "ComputeEngine", "AccumulateEngine", "HashScatterEngine", "GroupByResult", "Grouping", "Op", "GroupIndex",
    "Context", "DescriptiveEngine", "GroupedMomentStats", "MomentStats", "TambearGbError", "KeyOutOfRange",
    "InvalidArgument", "TableFull", "EntryNotFound", "MOMENT_FIELDS", "HIGHER_FIELDS", "SUMCOUNT_FIELDS",
    "FilterJit", "MaskOp", "Frame", "GroupByBuilder", "from_columns", "fused_bin_stats",
    "fused_multi_column_bin_stats",
]

SUMCOUNT_FIELDS = ("count", "sum", "mean")


def _torch():
    import torch

    return torch


def _ptr(t) -> int | None:
    """Device address of a tensor; an int is taken as an address already (peer mappings)."""
    if t is None or isinstance(t, int):
        return t
    return int(t.data_ptr())


def _stream_handle(stream) -> int | None:
    if stream is None:
        torch = _torch()
        return int(torch.cuda.current_stream().cuda_stream)
    return int(getattr(stream, "cuda_stream", stream))


class Context:
    """One tbgb_ctx on one CUDA device."""

    def __init__(self, device: int = 0):
        self._L = lib()
        h = C.c_void_p()
        st = self._L.tbgb_create(int(device), C.byref(h))
        if st != 0:
            raise error_for(st, f"tbgb_create(device={device}) failed (an sm_100 device is required)")
        self._h = h
        self.device = int(device)

    def close(self):
        if getattr(self, "_h", None):
            self._L.tbgb_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def name(self) -> str:
        return self._L.tbgb_device_name(self._h).decode()

    @property
    def launches(self) -> int:
        return int(self._L.tbgb_launch_count(self._h))

    def _check(self, st: int):
        if st != 0:
            raise error_for(st, self._L.tbgb_last_error(self._h).decode())

    def workspace_bytes(self, n: int, n_groups: int) -> int:
        return int(self._L.tbgb_workspace_bytes(self._h, int(n), int(n_groups)))

    # -- groupby ------------------------------------------------------------------
    @staticmethod
    def moments_struct(out: dict) -> Moments:
        m = Moments()
        for f, _ in Moments._fields_:
            setattr(m, f, _ptr(out.get(f)))
        return m

    def alloc_moments(self, n_groups: int, fields=MOMENT_FIELDS) -> dict:
        torch = _torch()
        return {f: torch.empty(n_groups, dtype=torch.float64, device=f"cuda:{self.device}") for f in fields}

    def groupby_dense(self, keys, vals, n_groups: int, mask=None, out: dict | None = None, stream=None,
                      sync: bool = True) -> dict:
        """Grouped count/sum/min/max/mean/m2/var of device tensors keys (int32) and vals (f64)."""
        n = int(vals.numel())
        if int(keys.numel()) != n:
            raise InvalidArgument(7, "keys and values must have same length")
        if out is None:
            out = self.alloc_moments(n_groups)
        m = self.moments_struct(out)
        self._check(self._L.tbgb_groupby_dense(self._h, _ptr(keys), _ptr(vals), _ptr(mask), n, int(n_groups),
                                               C.byref(m), _stream_handle(stream)))
        if sync:
            self.sync(stream)
        return out

    def sync(self, stream=None):
        self._check(self._L.tbgb_sync(self._h, _stream_handle(stream)))

    def set_table_mode(self, mode: str | int):
        """'auto' (0), 'local' (1: per-CTA shared-memory pre-aggregation), 'direct' (2),
        'bucket' (3: partition first), 'range' (4: dense keys, group ranges held whole in
        shared memory), 'radix' (5: int64 keys, count / sum / mean by radix partitioning) or
        'sweep' (6: dense keys, full moments, rank and sweep); see tbgb_set_table_mode."""
        m = {"auto": 0, "local": 1, "direct": 2, "bucket": 3, "range": 4, "radix": 5, "sweep": 6}.get(mode, mode)
        self._check(self._L.tbgb_set_table_mode(self._h, int(m)))

    @staticmethod
    def columns(a, b=None, c=None, expr: str = "a", pred: str | None = None, threshold: float = 0.0) -> Columns:
        torch = _torch()
        if a.dtype == torch.float64:
            dt = DTYPES["f64"]
        elif a.dtype == torch.float32:
            dt = DTYPES["f32"]
        else:
            raise InvalidArgument(7, f"unsupported value dtype {a.dtype}")
        for t in (b, c):
            if t is not None and t.dtype != a.dtype:
                raise InvalidArgument(7, "columns a, b, c must share one dtype")
        cols = Columns()
        cols.a, cols.b, cols.c = _ptr(a), _ptr(b), _ptr(c)
        cols.dtype, cols.expr, cols.pred, cols.reserved = dt, EXPRS[expr], PREDS[pred], 0
        cols.threshold = float(threshold)
        return cols

    def groupby_dense_columns(self, keys, a, n_groups: int, b=None, c=None, expr: str = "a",
                              pred: str | None = None, threshold: float = 0.0, mask=None,
                              out: dict | None = None, stream=None, sync: bool = True) -> dict:
        """Dense-key groupby of expr(a, b, c) over rows passing mask and pred(a, threshold)."""
        n = int(keys.numel())
        if int(a.numel()) != n:
            raise InvalidArgument(7, "keys and columns must have same length")
        if out is None:
            out = self.alloc_moments(n_groups)
        cols = self.columns(a, b, c, expr, pred, threshold)
        m = self.moments_struct(out)
        self._check(self._L.tbgb_groupby_dense_columns(self._h, _ptr(keys), C.byref(cols), _ptr(mask), n,
                                                       int(n_groups), C.byref(m), _stream_handle(stream)))
        if sync:
            self.sync(stream)
        return out

    def group_index_build(self, keys, max_key: int, stream=None) -> dict:
        """GroupIndex::build of an int32 device key column (u32 outputs as int32 tensors of the
        same bits): row_to_group, group_counts, group_offsets, rows_by_group, n_active."""
        torch = _torch()
        n = int(keys.numel())
        dev = f"cuda:{self.device}"
        G = int(max_key) + 1
        out = {"row_to_group": torch.empty(n, dtype=torch.int32, device=dev),
               "group_counts": torch.empty(G, dtype=torch.int32, device=dev),
               "group_offsets": torch.empty(G + 1, dtype=torch.int32, device=dev),
               "rows_by_group": torch.empty(n, dtype=torch.int32, device=dev)}
        na = torch.zeros(1, dtype=torch.int64, device=dev)
        self._check(self._L.tbgb_group_index_build(self._h, _ptr(keys), n, int(max_key), _ptr(out["row_to_group"]),
                                                   _ptr(out["group_counts"]), _ptr(out["group_offsets"]),
                                                   _ptr(out["rows_by_group"]), _ptr(na), _stream_handle(stream)))
        self.sync(stream)
        out["n_active"] = int(na.item())
        return out

    def factorize_i64(self, keys, max_groups: int, stream=None):
        """Dictionary codes of int64 device keys in first-seen order: (codes int32, uniques int64)."""
        torch = _torch()
        n = int(keys.numel())
        dev = f"cuda:{self.device}"
        codes = torch.empty(n, dtype=torch.int32, device=dev)
        uniques = torch.empty(int(max_groups), dtype=torch.int64, device=dev)
        nu = torch.zeros(1, dtype=torch.int64, device=dev)
        self._check(self._L.tbgb_factorize_i64(self._h, _ptr(keys), n, int(max_groups), _ptr(codes), _ptr(uniques),
                                               _ptr(nu), _stream_handle(stream)))
        self.sync(stream)
        return codes, uniques[:int(nu.item())]

    # ---- row masks (mask-not-filter) and tile statistics ----
    # A device row mask is an int64 tensor of ceil(n_rows / 64) words holding the u64 bit
    # patterns (row i in bit i % 64 of word i // 64).

    def _words_out(self, n_words: int, out):
        torch = _torch()
        if out is None:
            return torch.empty(int(n_words), dtype=torch.int64, device=f"cuda:{self.device}")
        if int(out.numel()) != int(n_words):
            raise InvalidArgument(7, "output mask has the wrong number of words")
        return out

    def filter_mask(self, col, pred: str, threshold: float = 0.0, in_mask=None, out=None, stream=None):
        """FilterJit::filter_mask on a device column (f64 or f32): bit i = in_mask(i) and
        pred(col[i]); col is read only where in_mask is set."""
        torch = _torch()
        n = int(col.numel())
        if pred not in PREDS:
            raise EntryNotFound(6, f"unknown predicate {pred!r}")
        dt = DTYPES["f32"] if col.dtype == torch.float32 else DTYPES["f64"]
        if col.dtype not in (torch.float32, torch.float64):
            raise InvalidArgument(7, "filter column must be f64 or f32")
        m = self._words_out((n + 63) // 64, out)
        self._check(self._L.tbgb_filter_mask(self._h, _ptr(col), dt, n, PREDS[pred], float(threshold),
                                             _ptr(in_mask), _ptr(m), _stream_handle(stream)))
        return m

    def _mask_binary(self, fn, a, b, out, stream):
        if int(a.numel()) != int(b.numel()):
            raise InvalidArgument(7, "mask length mismatch")
        m = self._words_out(a.numel(), out)
        self._check(fn(self._h, _ptr(a), _ptr(b), _ptr(m), int(a.numel()), _stream_handle(stream)))
        return m

    def mask_and(self, a, b, out=None, stream=None):
        return self._mask_binary(self._L.tbgb_mask_and, a, b, out, stream)

    def mask_or(self, a, b, out=None, stream=None):
        return self._mask_binary(self._L.tbgb_mask_or, a, b, out, stream)

    def mask_xor(self, a, b, out=None, stream=None):
        return self._mask_binary(self._L.tbgb_mask_xor, a, b, out, stream)

    def mask_not(self, a, n_rows: int, out=None, stream=None):
        m = self._words_out(a.numel(), out)
        self._check(self._L.tbgb_mask_not(self._h, _ptr(a), _ptr(m), int(a.numel()), int(n_rows),
                                          _stream_handle(stream)))
        return m

    def mask_popcount(self, m, n_rows: int, stream=None) -> int:
        """Set bits of rows [0, n_rows) (synchronises the stream)."""
        torch = _torch()
        cnt = torch.zeros(1, dtype=torch.int64, device=f"cuda:{self.device}")
        self._check(self._L.tbgb_mask_popcount(self._h, _ptr(m), int(m.numel()), int(n_rows), _ptr(cnt),
                                               _stream_handle(stream)))
        self.sync(stream)
        return int(cnt.item())

    def tile_stats(self, col, tile_rows: int = 65536, stream=None):
        """TileColumnStats of every tile of a device column: a uint8 tensor [n_tiles, 40]
        (field layout TILE_STATS_FIELDS; see tile_stats_numpy)."""
        torch = _torch()
        n = int(col.numel())
        if col.dtype not in (torch.float32, torch.float64):
            raise InvalidArgument(7, "tile statistics need an f64 or f32 column")
        n_tiles = (n + int(tile_rows) - 1) // int(tile_rows) if tile_rows >= 1 else 0
        st = torch.empty((max(n_tiles, 0), TILE_STATS_BYTES), dtype=torch.uint8, device=f"cuda:{self.device}")
        dt = DTYPES["f32"] if col.dtype == torch.float32 else DTYPES["f64"]
        self._check(self._L.tbgb_tile_stats_build(self._h, _ptr(col), dt, n, int(tile_rows), _ptr(st),
                                                  _stream_handle(stream)))
        return st

    def tile_skip_mask(self, stats, pred: str, threshold: float, stream=None):
        """1 per tile that no row can pass (pred one of '>', '>=', '<', '<=')."""
        torch = _torch()
        if pred not in PREDS:
            raise EntryNotFound(6, f"unknown predicate {pred!r}")
        n_tiles = int(stats.shape[0])
        skip = torch.empty(n_tiles, dtype=torch.uint8, device=f"cuda:{self.device}")
        self._check(self._L.tbgb_tile_skip_mask(self._h, _ptr(stats), n_tiles, PREDS[pred], float(threshold),
                                                _ptr(skip), _stream_handle(stream)))
        return skip

    def fused_bin_stats(self, data, boundaries, fields=BIN_STATS_FIELDS, stream=None, sync: bool = True,
                        out: dict | None = None) -> dict:
        """Statistics of sorted contiguous bins (tbgb_fused_bin_stats): data is an f64 device
        tensor [n_ticks] or [n_columns, n_ticks], boundaries int64 [n_bins + 1].  Returns
        {field: tensor} with count int32 [n_bins] and the others f64 [n_bins] (one column) or
        [n_columns, n_bins]."""
        torch = _torch()
        if data.dtype != torch.float64:
            raise InvalidArgument(7, "bin statistics need an f64 column")
        if boundaries.dtype != torch.int64:
            raise InvalidArgument(7, "boundaries must be int64")
        data = data.contiguous()
        ncol = 1 if data.dim() == 1 else int(data.shape[0])
        n_ticks = int(data.shape[-1])
        nb = max(int(boundaries.numel()) - 1, 0)
        dev = f"cuda:{self.device}"
        shape = (nb,) if data.dim() == 1 else (ncol, nb)
        if out is None:
            out = {}
            for f in fields:
                out[f] = torch.empty(nb if f == "count" else shape,
                                     dtype=torch.int32 if f == "count" else torch.float64, device=dev)
        bs = BinStats()
        for f in BIN_STATS_FIELDS:
            setattr(bs, f, _ptr(out.get(f)))
        self._check(self._L.tbgb_fused_bin_stats(self._h, _ptr(data), n_ticks, ncol, _ptr(boundaries), nb,
                                                 C.byref(bs), _stream_handle(stream)))
        if sync:
            self.sync(stream)
        return out

    def mask_skip_tiles(self, skip, tile_rows: int, n_rows: int, mask=None, out=None, stream=None):
        """Row mask of the rows outside skipped tiles (and inside `mask` when given)."""
        m = self._words_out((int(n_rows) + 63) // 64, out)
        self._check(self._L.tbgb_mask_skip_tiles(self._h, _ptr(mask), _ptr(skip), int(tile_rows), int(n_rows),
                                                 _ptr(m), _stream_handle(stream)))
        return m

    def groupby_hash_into(self, keys, a, max_groups: int, out_keys, out: dict, n_groups, b=None, c=None,
                          expr: str = "a", pred: str | None = None, threshold: float = 0.0, mask=None,
                          stream=None):
        """Enqueue an int64-key groupby into caller-owned device buffers (no host synchronisation):
        out_keys (int64, max_groups), out {field: f64 tensor}, n_groups (int64, 1 element)."""
        n = int(keys.numel())
        cols = self.columns(a, b, c, expr, pred, threshold)
        m = self.moments_struct(out)
        self._check(self._L.tbgb_groupby_hash(self._h, _ptr(keys), C.byref(cols), _ptr(mask), n, int(max_groups),
                                              _ptr(out_keys), C.byref(m), _ptr(n_groups), _stream_handle(stream)))

    def hash_partition(self, keys, a, n_parts: int, out_keys, out_vals, part_counts, b=None, c=None,
                       expr: str = "a", pred: str | None = None, threshold: float = 0.0, mask=None, stream=None):
        """Enqueue the owner routing of this shard's rows (see tbgb_hash_partition)."""
        cols = self.columns(a, b, c, expr, pred, threshold)
        self._check(self._L.tbgb_hash_partition(self._h, _ptr(keys), C.byref(cols), _ptr(mask), int(keys.numel()),
                                                int(n_parts), _ptr(out_keys), _ptr(out_vals), _ptr(part_counts),
                                                _stream_handle(stream)))

    def radix_fallback(self) -> int:
        """Bits of the last radix call's fallback to the global table (0: none); see
        tbgb_radix_fallback.  Waits for the device."""
        bits = C.c_uint32(0)
        self._check(self._L.tbgb_radix_fallback(self._h, C.byref(bits)))
        return int(bits.value)

    def radix_value_bytes(self, a, b=None, c=None, expr: str = "a", pred: str | None = None,
                          threshold: float = 0.0) -> int:
        """Bytes per value of routed rows: 4 (an f32 column without expression) or 8."""
        return int(self._L.tbgb_radix_value_bytes(C.byref(self.columns(a, b, c, expr, pred, threshold))))

    def radix_route(self, keys, a, out_hashes, out_vals, digit_counts, b=None, c=None, expr: str = "a",
                    pred: str | None = None, threshold: float = 0.0, mask=None, stream=None):
        """Enqueue the owner routing of this shard's rows (see tbgb_radix_route): rows as
        (fmix64(key), value) ordered by the top 9 hash bits; digit_counts (512 int64) per digit."""
        cols = self.columns(a, b, c, expr, pred, threshold)
        self._check(self._L.tbgb_radix_route(self._h, _ptr(keys), C.byref(cols), _ptr(mask), int(keys.numel()),
                                             _ptr(out_hashes), _ptr(out_vals), _ptr(digit_counts),
                                             _stream_handle(stream)))

    def radix_groupby_routed(self, hashes, vals, sender_rows, seg_counts, digit_lo: int, n_digits: int,
                             max_groups: int, out_keys, out: dict, n_groups, value_bytes: int | None = None,
                             stream=None):
        """Enqueue the owner's grouping of routed rows (see tbgb_radix_groupby_routed): count / sum /
        mean into caller-owned buffers.  hashes / vals: per sender, the device address (int) of its
        first routed row -- or one tensor each holding the senders' blocks back to back (a receive
        buffer); sender_rows: rows per sender (host ints); value_bytes: 4 or 8 (taken from the
        tensor when vals is one)."""
        rows = [int(x) for x in sender_rows]
        n = len(rows)
        if not isinstance(hashes, (list, tuple)):
            vb = int(vals.element_size())
            offs = [sum(rows[:i]) for i in range(n)]
            hashes = [int(hashes.data_ptr()) + 8 * o for o in offs]
            vals = [int(vals.data_ptr()) + vb * o for o in offs]
        else:
            vb = int(value_bytes)
        m = self.moments_struct(out)
        hp = (C.c_void_p * n)(*[C.c_void_p(_ptr(p)) for p in hashes])
        vp_ = (C.c_void_p * n)(*[C.c_void_p(_ptr(p)) for p in vals])
        rp = (C.c_int64 * n)(*rows)
        self._check(self._L.tbgb_radix_groupby_routed(self._h, n, hp, vp_, rp, vb, _ptr(seg_counts), int(digit_lo),
                                                      int(n_digits), int(max_groups), _ptr(out_keys), C.byref(m),
                                                      _ptr(n_groups), _stream_handle(stream)))

    def groupby_hash(self, keys, a, max_groups: int, b=None, c=None, expr: str = "a", pred: str | None = None,
                     threshold: float = 0.0, mask=None, fields=MOMENT_FIELDS, stream=None):
        """int64-key groupby; returns (group keys, {field: tensor}) trimmed to the group count
        (group order unspecified).  fields=SUMCOUNT_FIELDS keeps only count/sum/mean."""
        torch = _torch()
        n = int(keys.numel())
        if keys.dtype != torch.int64:
            raise InvalidArgument(7, "hash keys must be int64")
        if int(a.numel()) != n:
            raise InvalidArgument(7, "keys and columns must have same length")
        dev = f"cuda:{self.device}"
        out = self.alloc_moments(int(max_groups), fields)
        out_keys = torch.empty(int(max_groups), dtype=torch.int64, device=dev)
        ng = torch.zeros(1, dtype=torch.int64, device=dev)
        cols = self.columns(a, b, c, expr, pred, threshold)
        m = self.moments_struct(out)
        self._check(self._L.tbgb_groupby_hash(self._h, _ptr(keys), C.byref(cols), _ptr(mask), n, int(max_groups),
                                              _ptr(out_keys), C.byref(m), _ptr(ng), _stream_handle(stream)))
        self.sync(stream)
        g = int(ng.item())
        return out_keys[:g], {k: v[:g] for k, v in out.items()}

    # ---- the exchange step over NVLink peer memory ----
    def exchange_alloc(self, world: int, n_groups: int) -> int:
        """A zeroed exchange buffer (device pointer as an int); free with exchange_free."""
        p = C.c_void_p()
        self._check(self._L.tbgb_exchange_alloc(self._h, int(world), int(n_groups), C.byref(p)))
        return int(p.value)

    def exchange_free(self, ptr: int):
        self._check(self._L.tbgb_exchange_free(self._h, C.c_void_p(ptr)))

    def peer_export(self, ptr: int) -> bytes:
        h = (C.c_uint8 * 64)()
        self._check(self._L.tbgb_peer_export(self._h, C.c_void_p(ptr), h))
        return bytes(h)

    def peer_import(self, handle: bytes) -> int:
        h = (C.c_uint8 * 64).from_buffer_copy(handle)
        p = C.c_void_p()
        self._check(self._L.tbgb_peer_import(self._h, h, C.byref(p)))
        return int(p.value)

    def peer_close(self, ptr: int):
        self._check(self._L.tbgb_peer_close(self._h, C.c_void_p(ptr)))

    def ipc_alloc(self, nbytes: int) -> int:
        """A device buffer in its own allocation, exportable with peer_export; free with ipc_free."""
        p = C.c_void_p()
        self._check(self._L.tbgb_ipc_alloc(self._h, int(nbytes), C.byref(p)))
        return int(p.value)

    def ipc_free(self, ptr: int):
        self._check(self._L.tbgb_ipc_free(self._h, C.c_void_p(ptr)))

    def groupby_dense_sharded(self, keys, vals, n_groups: int, row_offset: int, rank: int, exchange, epoch: int,
                              out: dict, mask=None, stream=None):
        """Enqueue the shard's groupby, the push of its state table into every rank's exchange
        buffer and the rank-ordered merge into `out` (exchange: device pointers of all ranks'
        buffers as mapped here)."""
        arr = (C.c_void_p * len(exchange))(*[C.c_void_p(int(p)) for p in exchange])
        m = self.moments_struct(out)
        self._check(self._L.tbgb_groupby_dense_sharded(self._h, _ptr(keys), _ptr(vals), _ptr(mask),
                                                       int(vals.numel()), int(n_groups), int(row_offset), int(rank),
                                                       len(exchange), arr, int(epoch), C.byref(m),
                                                       _stream_handle(stream)))

    def state_bytes(self, n_groups: int) -> int:
        return int(self._L.tbgb_state_bytes(int(n_groups)))

    def groupby_dense_state(self, keys, vals, n_groups: int, row_offset: int = 0, mask=None, state=None,
                            stream=None):
        torch = _torch()
        n = int(vals.numel())
        if state is None:
            state = torch.empty(self.state_bytes(n_groups) // 8, dtype=torch.float64,
                                device=f"cuda:{self.device}")
        self._check(self._L.tbgb_groupby_dense_state(self._h, _ptr(keys), _ptr(vals), _ptr(mask), n,
                                                     int(n_groups), int(row_offset), _ptr(state),
                                                     _stream_handle(stream)))
        return state

    def merge_states(self, states, n_states: int, n_groups: int, out: dict | None = None, stream=None) -> dict:
        if out is None:
            out = self.alloc_moments(n_groups)
        m = self.moments_struct(out)
        self._check(self._L.tbgb_merge_states(self._h, _ptr(states), int(n_states), int(n_groups), C.byref(m),
                                              _stream_handle(stream)))
        return out

    # -- kernel timing --------------------------------------------------------------
    def profile(self, enable: bool = True):
        self._check(self._L.tbgb_profile_enable(self._h, 1 if enable else 0))

    def kernel_time_ms(self) -> tuple[float, int]:
        ms, cnt = C.c_double(), C.c_int64()
        self._check(self._L.tbgb_kernel_time_ms(self._h, C.byref(ms), C.byref(cnt)))
        return float(ms.value), int(cnt.value)

    # -- synthetic inputs -------------------------------------------------------------
    def gen_keys_uniform(self, keys, n_groups: int, seed: int, first_row: int = 0, stream=None):
        self._check(self._L.tbgb_gen_keys_uniform(self._h, _ptr(keys), int(keys.numel()), int(n_groups),
                                                  int(seed) & (2**64 - 1), int(first_row), _stream_handle(stream)))

    def gen_values_uniform(self, vals, lo: float, hi: float, seed: int, first_row: int = 0, stream=None):
        self._check(self._L.tbgb_gen_values_uniform(self._h, _ptr(vals), int(vals.numel()), float(lo), float(hi),
                                                    int(seed) & (2**64 - 1), int(first_row),
                                                    _stream_handle(stream)))

    def gen_values_normal(self, vals, mu: float, sigma: float, seed: int, first_row: int = 0, stream=None):
        self._check(self._L.tbgb_gen_values_normal(self._h, _ptr(vals), int(vals.numel()), float(mu),
                                                   float(sigma), int(seed) & (2**64 - 1), int(first_row),
                                                   _stream_handle(stream)))

    def gen_keys_cdf(self, keys, cdf, salt: int, seed: int, first_row: int = 0, stream=None):
        self._check(self._L.tbgb_gen_keys_cdf(self._h, _ptr(keys), int(keys.numel()), _ptr(cdf), int(cdf.numel()),
                                              int(salt) & (2**64 - 1), int(seed) & (2**64 - 1), int(first_row),
                                              _stream_handle(stream)))

    def gen_keys_ids(self, keys, n_ids: int, salt: int, seed: int, first_row: int = 0, stream=None):
        self._check(self._L.tbgb_gen_keys_ids(self._h, _ptr(keys), int(keys.numel()), int(n_ids),
                                              int(salt) & (2**64 - 1), int(seed) & (2**64 - 1), int(first_row),
                                              _stream_handle(stream)))

    def gen_values_lognormal_f32(self, vals, mu: float, sigma: float, seed: int, first_row: int = 0, stream=None):
        self._check(self._L.tbgb_gen_values_lognormal_f32(self._h, _ptr(vals), int(vals.numel()), float(mu),
                                                          float(sigma), int(seed) & (2**64 - 1), int(first_row),
                                                          _stream_handle(stream)))

    def gen_inject_nonfinite(self, vals, nan_frac: float, inf_frac: float, seed: int, first_row: int = 0,
                             stream=None):
        self._check(self._L.tbgb_gen_inject_nonfinite(self._h, _ptr(vals), int(vals.numel()), float(nan_frac),
                                                      float(inf_frac), int(seed) & (2**64 - 1), int(first_row),
                                                      _stream_handle(stream)))


# ---------------------------------------------------------------------------------
# The reference's operator API (descriptive.rs)
# ---------------------------------------------------------------------------------

@dataclass
class MomentStats:
    """Per-group sufficient statistics (descriptive.rs:67-254): count, sum, min, max and the
    central moment sums m2, m3, m4."""

    count: float
    sum: float
    min: float
    max: float
    m2: float
    m3: float = 0.0
    m4: float = 0.0

    @staticmethod
    def empty() -> "MomentStats":
        return MomentStats(0.0, 0.0, math.inf, -math.inf, 0.0, 0.0, 0.0)

    def n(self) -> int:
        return int(self.count)

    def mean(self) -> float:
        return math.nan if self.count == 0.0 else self.sum / self.count

    def variance(self, ddof: int) -> float:
        denom = self.count - float(ddof)
        return math.nan if denom <= 0.0 else self.m2 / denom

    def std(self, ddof: int) -> float:
        return math.sqrt(self.variance(ddof)) if not math.isnan(self.variance(ddof)) else math.nan

    def range(self) -> float:
        return math.nan if self.count == 0.0 else self.max - self.min

    def cv(self) -> float:
        m = self.mean()
        if m == 0.0 or self.count < 2.0:
            return math.nan
        return self.std(1) / abs(m)

    def sem(self) -> float:
        return math.nan if self.count < 2.0 else self.std(1) / math.sqrt(self.count)

    def skewness(self, bias: bool) -> float:
        n = self.count
        if n < 1.0 or self.m2 == 0.0:
            return math.nan
        var = self.m2 / n
        g1 = (self.m3 / n) / (var * math.sqrt(var))
        if bias:
            return g1
        return math.nan if n < 3.0 else g1 * math.sqrt(n * (n - 1.0)) / (n - 2.0)

    def kurtosis(self, excess: bool, bias: bool) -> float:
        n = self.count
        if n < 1.0 or self.m2 == 0.0:
            return math.nan
        var = self.m2 / n
        raw = (self.m4 / n) / (var * var)
        if bias:
            return raw - 3.0 if excess else raw
        if n < 4.0:
            return math.nan
        g2 = ((n - 1.0) / ((n - 2.0) * (n - 3.0))) * ((n + 1.0) * (raw - 3.0) + 6.0)
        return g2 if excess else g2 + 3.0

    @staticmethod
    def merge(a: "MomentStats", b: "MomentStats") -> "MomentStats":
        """Parallel merge of two partitions' moments (descriptive.rs:216-253)."""
        na, nb = a.count, b.count
        n = na + nb
        if n == 0.0:
            return MomentStats.empty()
        if na == 0.0:
            return b
        if nb == 0.0:
            return a
        delta = b.sum / nb - a.sum / na
        d2 = delta * delta
        m2 = a.m2 + b.m2 + d2 * na * nb / n
        m3 = a.m3 + b.m3 + d2 * delta * na * nb * (na - nb) / (n * n) + 3.0 * delta * (na * b.m2 - nb * a.m2) / n
        m4 = (a.m4 + b.m4 + d2 * d2 * na * nb * (na * na - na * nb + nb * nb) / (n * n * n)
              + 6.0 * d2 * (na * na * b.m2 + nb * nb * a.m2) / (n * n) + 4.0 * delta * (na * b.m3 - nb * a.m3) / n)
        mn = math.nan if math.isnan(a.min) or math.isnan(b.min) else min(a.min, b.min)
        mx = math.nan if math.isnan(a.max) or math.isnan(b.max) else max(a.max, b.max)
        return MomentStats(n, a.sum + b.sum, mn, mx, m2, m3, m4)


@dataclass
class GroupedMomentStats:
    """Parallel per-group arrays (descriptive.rs:295-330)."""

    n_groups: int
    counts: np.ndarray
    sums: np.ndarray
    mins: np.ndarray
    maxs: np.ndarray
    m2s: np.ndarray
    m3s: np.ndarray
    m4s: np.ndarray

    def group(self, g: int) -> MomentStats:
        return MomentStats(float(self.counts[g]), float(self.sums[g]), float(self.mins[g]), float(self.maxs[g]),
                           float(self.m2s[g]), float(self.m3s[g]), float(self.m4s[g]))

    def means(self) -> np.ndarray:
        with np.errstate(invalid="ignore", divide="ignore"):
            return np.where(self.counts > 0, self.sums / np.where(self.counts > 0, self.counts, 1), np.nan)


class DescriptiveEngine:
    """Grouped descriptive statistics on the B200 path (DescriptiveEngine, descriptive.rs:352-470)."""

    def __init__(self, device: int = 0):
        self.ctx = Context(device)

    def moments_grouped(self, values, keys, n_groups: int) -> GroupedMomentStats:
        torch = _torch()
        values = np.ascontiguousarray(values, dtype=np.float64)
        keys = np.ascontiguousarray(keys, dtype=np.int32)
        if values.shape != keys.shape:
            raise InvalidArgument(7, "values and keys must have same length")
        dev = f"cuda:{self.ctx.device}"
        dv = torch.from_numpy(values).to(dev)
        dk = torch.from_numpy(keys).to(dev)
        out = self.ctx.groupby_dense(dk, dv, n_groups, out=self.ctx.alloc_moments(
            n_groups, ("count", "sum", "min", "max", "m2", "m3", "m4")))
        h = {k: v.cpu().numpy() for k, v in out.items()}
        return GroupedMomentStats(n_groups, h["count"], h["sum"], h["min"], h["max"], h["m2"], h["m3"], h["m4"])

    def mean_grouped(self, values, keys, n_groups: int) -> np.ndarray:
        return self.moments_grouped(values, keys, n_groups).means()


from .engines import AccumulateEngine, ComputeEngine, GroupByResult, Grouping, HashScatterEngine, Op  # noqa: E402
from .group_index import GroupIndex  # noqa: E402
from .frame import FilterJit, Frame, GroupByBuilder, MaskOp, from_columns  # noqa: E402
from .bins import fused_bin_stats, fused_multi_column_bin_stats  # noqa: E402
