/*
 * tambear_gb.h -- C ABI of the B200 (sm_100a) groupby-aggregate path.
 *
 * Drop-in boundary for the reference's groupby/accumulate operator API.  Every
 * entry point takes plain pointers and sizes; no exceptions cross the ABI; all
 * device memory passed in is owned by the caller (the reference's
 * winrapids-store BufferPtr convention, crates/winrapids-store/src/header.rs:138-143),
 * while scratch ("workspace") is owned by the context and sized on demand.
 *
 * Reference interfaces replaced (paths relative to the reference project root):
 *   tbgb_create / tbgb_destroy      tam_gpu::detect() + CudaBackend::new
 *                                   (crates/tam-gpu/src/lib.rs:214, crates/tam-gpu/src/cuda.rs:111)
 *   tbgb_status                     tam_gpu::TamGpuError (crates/tam-gpu/src/error.rs:5-20)
 *   tbgb_groupby_dense              DescriptiveEngine::moments_grouped
 *                                   (crates/tambear/src/descriptive.rs:383-435) and
 *                                   HashScatterEngine::groupby (crates/tambear/src/hash_scatter.rs:367)
 *   tbgb_groupby_dense_state /      MomentStats::merge / SufficientStatistics::merge
 *   tbgb_merge_states               (descriptive.rs:216-253, intermediates.rs:352-377) used
 *                                   across row shards (one partial table per GPU)
 *   tbgb_columns (filter + expr)    FilterJit::filter_mask (crates/tambear/src/filter_jit.rs:71-121,
 *                                   kernel :196-252) and ComputeEngine::map_phi2
 *                                   (crates/tambear/src/compute_engine.rs:198-210, CPU :627-636),
 *                                   fused into the groupby pass as ScatterJit::scatter_multi_phi_masked
 *                                   fuses mask + scatter (crates/tambear/src/scatter_jit.rs:402-495)
 *   tbgb_groupby_dense_columns      the same composition over dense int32 keys, any n_groups
 *   tbgb_groupby_hash               GroupIndex::build (crates/tambear/src/group_index.rs:117-204) +
 *                                   moments_grouped for int64 keys: the reference factorises keys on
 *                                   the host and accepts i32 codes only; here an open-addressing table
 *                                   in HBM groups arbitrary int64 keys in the same pass
 *   tbgb_scatter_phi /              ComputeEngine::scatter_phi / scatter_multi_phi /
 *   tbgb_scatter_multi_phi_masked / scatter_phi_masked (crates/tambear/src/compute_engine.rs:109-154,
 *   tbgb_scatter_extremum           CPU :252-302) and ScatterJit::scatter_multi_phi_masked
 *                                   (scatter_jit.rs:402-495); ComputeEngine::scatter_extremum
 *                                   (compute_engine.rs:165-178, CPU :304-322).  These are the
 *                                   entry names the reference's TamGpu dispatches by (scatter_phi,
 *                                   scatter_multi_phi, scatter_phi_masked, scatter_extremum)
 *   tbgb_group_index_build          GroupIndex::build (crates/tambear/src/group_index.rs:117-204),
 *                                   on the device instead of the host
 *   tbgb_factorize_i64              Dictionary::encode (crates/tambear/src/dictionary.rs:40-75):
 *                                   codes in first-seen order, for int64 keys
 *   tbgb_filter_mask                FilterJit::filter_mask (crates/tambear/src/filter_jit.rs:71-121)
 *   tbgb_mask_and / _or / _xor /    MaskOp::mask_*_gpu (filter_jit.rs:339-440) and the host
 *   tbgb_mask_not / _popcount       mask_and / mask_or / mask_xor / mask_not / mask_popcount (:130-181)
 *   tbgb_tile_stats_build           TileColumnStats::from_slice (crates/tambear/src/format.rs:82-107)
 *   tbgb_tile_skip_mask             tile_skip_mask_gt / _lt (format.rs:182-189), can_skip_* (:111-136)
 *   tbgb_mask_skip_tiles            no counterpart: applies a tile-skip mask to a row mask so the
 *                                   groupby kernels never read skipped tiles
 *   tbgb_fused_bin_stats            fused_bin_stats / fused_bin_stats_multi
 *                                   (src/winrapids/kernels/bin_stats.cu:25-151)
 *   tbgb_groupby_dense_sharded      no counterpart (single GPU): row shards merged over NVLink peer
 *                                   memory, tables pushed into every rank's buffer by plain stores
 *   tbgb_hash_partition             no counterpart in the reference (single GPU); routes rows to
 *                                   the GPU that owns their key for the sharded high-cardinality path
 *   tbgb_radix_route /              no counterpart (single GPU): owner routing by hash digit and the
 *   tbgb_radix_groupby_routed       owner's radix-partitioned grouping of what it received
 *
 * Threading: one context per device; calls on one context are serialised by the
 * caller (the context's workspace is reused by every call); different contexts
 * are independent.
 */
#ifndef TAMBEAR_GB_H
#define TAMBEAR_GB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  1..7 mirror TamGpuError's variants in order. */
typedef enum {
  TBGB_OK = 0,
  TBGB_ERR_BACKEND = 1,           /* TamGpuError::Backend: driver / runtime failure        */
  TBGB_ERR_COMPILE = 2,           /* TamGpuError::Compile: never produced (no runtime JIT) */
  TBGB_ERR_ALLOC = 3,             /* TamGpuError::Alloc                                    */
  TBGB_ERR_TRANSFER = 4,          /* TamGpuError::Transfer                                 */
  TBGB_ERR_DISPATCH = 5,          /* TamGpuError::Dispatch: launch failure                 */
  TBGB_ERR_ENTRY_NOT_FOUND = 6,   /* TamGpuError::EntryNotFound: unknown entry / phi       */
  TBGB_ERR_INVALID_ARGUMENT = 7,  /* TamGpuError::InvalidArgument                          */
  TBGB_ERR_KEY_OUT_OF_RANGE = 8,  /* a key outside [0, n_groups) (the reference panics)    */
  TBGB_ERR_TABLE_FULL = 9,        /* hash table could not place a key                      */
  TBGB_ERR_TIMEOUT = 10           /* a bounded device-side wait gave up                    */
} tbgb_status;

typedef struct tbgb_ctx tbgb_ctx;

/* Create a context on CUDA device `device` (the process's current device is
 * left unchanged).  Fails with TBGB_ERR_BACKEND when no sm_100 device is present:
 * there is no CPU fallback. */
tbgb_status tbgb_create(int device, tbgb_ctx** out);
void tbgb_destroy(tbgb_ctx* ctx);
/* Message for the last failing call on `ctx` (valid until the next call). */
const char* tbgb_last_error(const tbgb_ctx* ctx);
/* "NVIDIA B200 (CUDA sm_100)" style label (TamGpu::name, crates/tam-gpu/src/lib.rs:155). */
const char* tbgb_device_name(const tbgb_ctx* ctx);

/* Per-group outputs of the grouped moments, one double per group each, device
 * pointers owned by the caller; any pointer may be NULL to skip that output.
 * Semantics follow DescriptiveEngine::moments_grouped + MomentStats:
 *   count    rows whose value is not NaN (+-inf rows count)
 *   sum      sum of the finite values (Kulisch skips +-inf), +0.0 when empty
 *   min/max  over non-NaN values, +inf / -inf when empty; +-0 ties resolved as a
 *            sequential `v < acc` scan in row order would
 *   mean     sum / count, NaN when count == 0
 *   m2       sum over finite values of (v - r)^2 with r = sum/count (0.0 when empty)
 *   var_pop  m2 / count, NaN when count == 0;  var_samp  m2 / (count - 1), NaN when count <= 1
 *   m3 / m4  sums over finite values of (v - r)^3 and (v - r)^4, r as for m2 (the m3s / m4s of
 *            GroupedMomentStats, descriptive.rs:421-432); computed only when requested */
typedef struct {
  double* count;
  double* sum;
  double* min;
  double* max;
  double* mean;
  double* m2;
  double* var_pop;
  double* var_samp;
  double* m3;
  double* m4;
} tbgb_moments;

/* Dense-key groupby: keys in [0, n_groups), f64 values, optional row mask
 * (bit i of mask[i/64] set <=> row i participates, filter_jit.rs:202-243 layout;
 * NULL = all rows).  Enqueued on `stream` (a cudaStream_t, NULL = legacy default
 * stream); returns after the launch.  Deferred device errors (key out of range,
 * timeouts) are reported by tbgb_sync.  1 <= n_groups <= 2^31 - 1: up to 512
 * groups run the shared-memory column kernel, more groups the global-table kernel
 * (with tbgb_set_table_mode != 0 the column kernel serves up to 1024 groups). */
tbgb_status tbgb_groupby_dense(tbgb_ctx* ctx, const int32_t* d_keys, const double* d_vals, const uint64_t* d_mask,
                               int64_t n, int32_t n_groups, const tbgb_moments* out, void* stream);

/* ---- value columns with a fused filter and expression ------------------------------
 * The value aggregated for row i is v = expr(a[i], b[i], c[i]) computed in f64 with
 * every operation rounded separately (no fused multiply-add), exactly as the
 * reference's map_phi2 composes `a*b` and then `+ c`.  f32 columns are widened to
 * f64 exactly before any arithmetic.  Row i takes part iff its mask bit is set (or
 * mask is NULL) and pred(a[i], threshold) holds; every comparison with a NaN `a`
 * fails, as in the reference's filter kernels.  Rows whose v is NaN are skipped by
 * every aggregate but, in the hash entry point, still create their key's group. */
typedef enum { TBGB_F64 = 0, TBGB_F32 = 1 } tbgb_dtype;
typedef enum {
  TBGB_PRED_NONE = 0,    /* every row                 */
  TBGB_PRED_GT = 1,      /* a >  threshold            */
  TBGB_PRED_GE = 2,      /* a >= threshold            */
  TBGB_PRED_LT = 3,      /* a <  threshold            */
  TBGB_PRED_LE = 4,      /* a <= threshold            */
  TBGB_PRED_NOT_NAN = 5, /* a is not NaN              */
  TBGB_PRED_FINITE = 6   /* a is finite               */
} tbgb_pred;
typedef enum {
  TBGB_EXPR_A = 0,         /* v = a                   */
  TBGB_EXPR_ADD = 1,       /* v = a + b               */
  TBGB_EXPR_SUB = 2,       /* v = a - b               */
  TBGB_EXPR_MUL = 3,       /* v = a * b               */
  TBGB_EXPR_MUL_PLUS1 = 4, /* v = (a * b) + 1.0       */
  TBGB_EXPR_MUL_ADD = 5    /* v = (a * b) + c         */
} tbgb_expr;
typedef struct {
  const void* a;       /* device column a (n elements of dtype)                 */
  const void* b;       /* device column b, read by ADD / SUB / MUL / MUL_PLUS1 / MUL_ADD */
  const void* c;       /* device column c, read by MUL_ADD                       */
  int32_t dtype;       /* tbgb_dtype of a, b and c                               */
  int32_t expr;        /* tbgb_expr                                              */
  int32_t pred;        /* tbgb_pred, applied to column a                         */
  int32_t reserved;    /* 0                                                      */
  double threshold;
} tbgb_columns;

/* Dense-key groupby of expr(a, b, c) over the rows that pass mask and pred. */
tbgb_status tbgb_groupby_dense_columns(tbgb_ctx* ctx, const int32_t* d_keys, const tbgb_columns* cols,
                                       const uint64_t* d_mask, int64_t n, int32_t n_groups,
                                       const tbgb_moments* out, void* stream);

/* int64-key groupby through an open-addressing table in device memory (any key
 * value, INT64_MIN included).  Groups are the distinct keys among the rows that
 * pass mask and pred.  Group j's key is written to d_out_keys[j] and its outputs to
 * element j of each non-NULL pointer of `out`, j < number of groups, in an order that
 * is not specified (sort by key for a canonical order); the number of groups is
 * written to *d_n_groups (device memory).  At most max_groups groups fit; more
 * distinct keys make tbgb_sync report TBGB_ERR_TABLE_FULL (the outputs are then
 * incomplete).  When out->min, max, m2, var_pop and var_samp are all NULL the table
 * keeps only count and sum (a 32-byte slot instead of 96). */
tbgb_status tbgb_groupby_hash(tbgb_ctx* ctx, const int64_t* d_keys, const tbgb_columns* cols,
                              const uint64_t* d_mask, int64_t n, int64_t max_groups, int64_t* d_out_keys,
                              const tbgb_moments* out, int64_t* d_n_groups, void* stream);

/* ---- scatter primitives over dense int32 keys ----------------------------------------
 * phi expressions of the reference's phi_scatter_eval (compute_engine.rs:593-609), r =
 * refs[key] (0.0 when refs is NULL), each operation rounded separately: */
typedef enum {
  TBGB_PHI_V = 0,        /* v                       */
  TBGB_PHI_VV = 1,       /* v * v                   */
  TBGB_PHI_ONE = 2,      /* 1.0                     */
  TBGB_PHI_VMR = 3,      /* v - r                   */
  TBGB_PHI_VMR2 = 4,     /* (v - r) * (v - r)       */
  TBGB_PHI_ABS_VMR = 5,  /* fabs(v - r)             */
  TBGB_PHI_VMR3 = 6,     /* (v - r)^3 as (d * d) * d */
  TBGB_PHI_VMR4 = 7,     /* (v - r)^4 as d2 * d2    */
  TBGB_PHI_VR = 8,       /* v * r                   */
  TBGB_PHI_LOG = 9,      /* log(v)                  */
  TBGB_PHI_RECIP = 10    /* 1.0 / v                 */
} tbgb_phi;

/* out[j * n_groups + g] = sum over rows i with keys[i] == g (and mask bit i set, when
 * d_mask is not NULL) of phis[j](vals[i], refs[g]), over the finite nonzero terms (the
 * reference's CPU accumulator skips +-0, NaN and +-inf terms), f64 accumulation.
 * 1 <= n_phi <= 5.  Every row's key must lie in [0, n_groups) (masked-out rows are not
 * checked), else tbgb_sync reports TBGB_ERR_KEY_OUT_OF_RANGE.  Unknown phi ids:
 * TBGB_ERR_ENTRY_NOT_FOUND. */
tbgb_status tbgb_scatter_multi_phi_masked(tbgb_ctx* ctx, const int32_t* phis, int32_t n_phi, const int32_t* d_keys,
                                          const double* d_vals, const double* d_refs, const uint64_t* d_mask,
                                          int64_t n, int32_t n_groups, double* d_out, void* stream);
tbgb_status tbgb_scatter_phi(tbgb_ctx* ctx, int32_t phi, const int32_t* d_keys, const double* d_vals,
                             const double* d_refs, int64_t n, int32_t n_groups, double* d_out, void* stream);
tbgb_status tbgb_scatter_multi_phi(tbgb_ctx* ctx, const int32_t* phis, int32_t n_phi, const int32_t* d_keys,
                                   const double* d_vals, const double* d_refs, int64_t n, int32_t n_groups,
                                   double* d_out, void* stream);
tbgb_status tbgb_scatter_phi_masked(tbgb_ctx* ctx, int32_t phi, const int32_t* d_keys, const double* d_vals,
                                    const double* d_refs, const uint64_t* d_mask, int64_t n, int32_t n_groups,
                                    double* d_out, void* stream);
/* out[g] = min (is_max == 0) or max of the non-NaN values of group g by a strict scan in
 * row order (+-0 ties: the first zero), +inf / -inf for groups without one. */
tbgb_status tbgb_scatter_extremum(tbgb_ctx* ctx, int32_t is_max, const int32_t* d_keys, const double* d_vals,
                                  int64_t n, int32_t n_groups, double* d_out, void* stream);

/* ---- key factorisation ---------------------------------------------------------------
 * GroupIndex::build for keys in [0, max_key]: row_to_group[i] = keys[i] (n entries),
 * group_counts[g] (max_key + 1 entries), group_offsets[g] = sum of the counts of groups < g
 * (max_key + 2 entries, the last = n), rows_by_group = row ids ordered by group with the row
 * order kept inside each group (n entries), *d_n_active (device) = groups with a row.  All
 * device memory, caller-owned; u32 like the reference.  n must be in [1, 2^32) (an empty
 * column is TBGB_ERR_INVALID_ARGUMENT, as in the reference); a key outside [0, max_key]
 * makes tbgb_sync report TBGB_ERR_KEY_OUT_OF_RANGE. */
tbgb_status tbgb_group_index_build(tbgb_ctx* ctx, const int32_t* d_keys, int64_t n, int32_t max_key,
                                   uint32_t* d_row_to_group, uint32_t* d_group_counts, uint32_t* d_group_offsets,
                                   uint32_t* d_rows_by_group, int64_t* d_n_active, void* stream);
/* Dictionary codes of int64 keys: distinct keys are numbered 0, 1, ... in the order they are
 * first seen; d_codes[i] = number of keys[i] (n entries), d_uniques[j] = key j (up to
 * max_groups entries), *d_n_uniques (device) = distinct keys (at most max_groups; more make
 * tbgb_sync report TBGB_ERR_TABLE_FULL). */
tbgb_status tbgb_factorize_i64(tbgb_ctx* ctx, const int64_t* d_keys, int64_t n, int64_t max_groups, int32_t* d_codes,
                               int64_t* d_uniques, int64_t* d_n_uniques, void* stream);

/* ---- row masks and tile statistics (mask-not-filter) --------------------------------
 * A row mask for n_rows rows is ceil(n_rows / 64) u64 words in device memory, row i in
 * bit i % 64 of word i / 64, the bits of rows >= n_rows of the last word 0
 * (FilterJit::filter_mask, crates/tambear/src/filter_jit.rs:71-121 and :196-243).  Every
 * groupby entry point takes such a mask (d_mask); the table-path kernels test a row's
 * bit before they read its columns, so rows in all-zero mask regions cost no column
 * reads.  Word pointers must be 8-byte aligned; out may alias an input. */

/* FilterJit::filter_mask (filter_jit.rs:71-121): bit i = in(i) && pred(col[i]) (tbgb_pred; a
 * comparison with NaN fails, TBGB_PRED_NONE passes every row), with in(i) the bit of
 * d_in_mask (NULL: every row).  col[i] is read only where in(i) is set, so a mask from
 * tbgb_mask_skip_tiles keeps skipped tiles unread.  d_mask may alias d_in_mask. */
tbgb_status tbgb_filter_mask(tbgb_ctx* ctx, const void* d_col, int32_t dtype, int64_t n, int32_t pred,
                             double threshold, const uint64_t* d_in_mask, uint64_t* d_mask, void* stream);
/* MaskOp::mask_and_gpu / mask_or_gpu / mask_xor_gpu (filter_jit.rs:339-396): word by
 * word over n_words words. */
tbgb_status tbgb_mask_and(tbgb_ctx* ctx, const uint64_t* d_a, const uint64_t* d_b, uint64_t* d_out, int64_t n_words,
                          void* stream);
tbgb_status tbgb_mask_or(tbgb_ctx* ctx, const uint64_t* d_a, const uint64_t* d_b, uint64_t* d_out, int64_t n_words,
                         void* stream);
tbgb_status tbgb_mask_xor(tbgb_ctx* ctx, const uint64_t* d_a, const uint64_t* d_b, uint64_t* d_out, int64_t n_words,
                          void* stream);
/* MaskOp::mask_not_gpu (filter_jit.rs:397-416): ~a with the bits of rows >= n_rows
 * cleared; n_words must be ceil(n_rows / 64). */
tbgb_status tbgb_mask_not(tbgb_ctx* ctx, const uint64_t* d_a, uint64_t* d_out, int64_t n_words, int64_t n_rows,
                          void* stream);
/* MaskOp::mask_popcount_gpu (filter_jit.rs:418-440), mask_popcount (:130-144): set bits of
 * rows [0, n_rows) into *d_count (device u64); n_words >= ceil(n_rows / 64), later words
 * and the bits of rows >= n_rows are not counted. */
tbgb_status tbgb_mask_popcount(tbgb_ctx* ctx, const uint64_t* d_mask, int64_t n_words, int64_t n_rows,
                               uint64_t* d_count, void* stream);

/* TileColumnStats (crates/tambear/src/format.rs:60-73), 40 bytes. */
typedef struct {
  double min;        /* strict `<` scan from +inf (NaN never wins)                    */
  double max;        /* strict `>` scan from -inf                                     */
  double sum;        /* compensated sum (the serial Kahan result within a few ulps)   */
  uint32_t count;    /* rows of the tile                                              */
  uint32_t n_valid;  /* = count (dense columns)                                       */
  uint64_t reserved; /* 0                                                             */
} tbgb_tile_stats;
/* TileColumnStats::from_slice (format.rs:82-107) for every tile of tile_rows rows
 * (1 <= tile_rows < 2^32; the last tile may be shorter): ceil(n / tile_rows) entries. */
tbgb_status tbgb_tile_stats_build(tbgb_ctx* ctx, const void* d_col, int32_t dtype, int64_t n, int64_t tile_rows,
                                  tbgb_tile_stats* d_stats, void* stream);
/* tile_skip_mask_gt / _lt (format.rs:182-189) and can_skip_gte / _lte (:125-136):
 * d_skip[t] = 1 when no row of tile t can pass pred (TBGB_PRED_GT / GE / LT / LE only). */
tbgb_status tbgb_tile_skip_mask(tbgb_ctx* ctx, const tbgb_tile_stats* d_stats, int64_t n_tiles, int32_t pred,
                                double threshold, uint8_t* d_skip, void* stream);
/* Row mask of the rows outside skipped tiles: d_out = d_mask (every row when NULL) with
 * the rows of tiles t with d_skip[t] != 0 cleared (ceil(n_rows / 64) words; d_skip has
 * ceil(n_rows / tile_rows) entries).  Passing d_out to a groupby skips those tiles' reads. */
tbgb_status tbgb_mask_skip_tiles(tbgb_ctx* ctx, const uint64_t* d_mask, const uint8_t* d_skip, int64_t tile_rows,
                                 int64_t n_rows, uint64_t* d_out, void* stream);

/* ---- statistics of sorted contiguous bins ----------------------------------------
 * fused_bin_stats / fused_bin_stats_multi (src/winrapids/kernels/bin_stats.cu:25-151):
 * bin b is rows [boundaries[b], boundaries[b + 1]) (n_bins + 1 non-decreasing int64
 * boundaries within [0, n_ticks]) of each of n_columns f64 columns (column j at
 * d_data + j * n_ticks).  Outputs are device arrays, NULL to skip: count [n_bins] (int32,
 * < 2^31 rows per bin), the others [n_columns][n_bins]:
 *   sum, sum_sq   plain f64 sums of v and v*v (NaN / infinities propagate)
 *   min, max      strict `<` / `>` scans starting from the bin's first value (a NaN first
 *                 value is the result; a later NaN never wins; ties keep the first row)
 *   first, last   data[lo], data[hi - 1]
 *   mean, variance, std   sum / count, max(sum_sq / count - mean^2, 0) for count > 1 and
 *                 its square root, as the reference's Python wrapper derives them
 *                 (archive/fintek-contributions/src/fused_bin_stats.py:121-127)
 * An empty bin has count 0 and NaN elsewhere.  Counts, extrema, first and last are exact;
 * sums agree with the serial loop to within rounding (the rows are summed in parallel).
 * Boundaries that are not non-decreasing within [0, n_ticks] make tbgb_sync report
 * TBGB_ERR_INVALID_ARGUMENT (their bins' outputs are then unspecified). */
typedef struct {
  int32_t* count;
  double* sum;
  double* sum_sq;
  double* min;
  double* max;
  double* first;
  double* last;
  double* mean;
  double* variance;
  double* std;
} tbgb_bin_stats;
tbgb_status tbgb_fused_bin_stats(tbgb_ctx* ctx, const double* d_data, int64_t n_ticks, int32_t n_columns,
                                 const int64_t* d_boundaries, int64_t n_bins, const tbgb_bin_stats* out,
                                 void* stream);

/* ---- sharded dense groupby over NVLink peer memory (one process per GPU) ----------------
 * The exchange step without a library collective: every rank owns an exchange buffer
 * (tbgb_exchange_alloc: tbgb_exchange_bytes(world, n_groups) bytes, zeroed) and maps every
 * other rank's buffer with tbgb_peer_export / tbgb_peer_import (CUDA IPC handles, 64 bytes,
 * passed between the processes by the caller).  tbgb_groupby_dense_sharded then reduces the
 * rank's rows to its state table, stores it into its slot of every rank's buffer (plain stores
 * over NVLink), raises its flag there, waits until all ranks' flags show `epoch` and folds the
 * tables in rank order into `out` -- the same result as tbgb_groupby_dense_state + all-gather
 * + tbgb_merge_states.  h_exchange is a host array of `world` device pointers (entry q: rank
 * q's buffer as mapped in this process, entry `rank`: the own buffer); `epoch` starts at 1 and
 * increases by one per call on every rank.  A rank that never arrives makes the wait give up
 * after about 2 s: tbgb_sync then reports TBGB_ERR_TIMEOUT.  world <= 8. */
size_t tbgb_exchange_bytes(int32_t world, int32_t n_groups);
tbgb_status tbgb_exchange_alloc(tbgb_ctx* ctx, int32_t world, int32_t n_groups, void** d_buf);
tbgb_status tbgb_exchange_free(tbgb_ctx* ctx, void* d_buf);
tbgb_status tbgb_peer_export(tbgb_ctx* ctx, void* d_buf, uint8_t* handle /* 64 bytes */);
tbgb_status tbgb_peer_import(tbgb_ctx* ctx, const uint8_t* handle /* 64 bytes */, void** d_peer);
tbgb_status tbgb_peer_close(tbgb_ctx* ctx, void* d_peer);
/* A device buffer of `bytes` in its own allocation, so that tbgb_peer_export's handle maps
 * exactly it (e.g. the send buffer of the owner-sharded groupby's routed rows, which the owners
 * read in place); free with tbgb_ipc_free.  No counterpart in the reference (single GPU). */
tbgb_status tbgb_ipc_alloc(tbgb_ctx* ctx, size_t bytes, void** d_buf);
tbgb_status tbgb_ipc_free(tbgb_ctx* ctx, void* d_buf);
tbgb_status tbgb_groupby_dense_sharded(tbgb_ctx* ctx, const int32_t* d_keys, const double* d_vals,
                                       const uint64_t* d_mask, int64_t n, int32_t n_groups, int64_t row_offset,
                                       int32_t rank, int32_t world, void* const* h_exchange, uint64_t epoch,
                                       const tbgb_moments* out, void* stream);

/* ---- sharded int64-key groupby (one process / GPU per shard) ----------------------
 * Routes the rows of this shard that pass mask and pred to their owner part
 * owner(key) = (fmix64(key) >> 32) % n_parts (fmix64: MurmurHash3's 64-bit
 * finaliser), 1 <= n_parts <= 32: the rows of part p are written to
 * d_out_keys / d_out_vals (v = expr(a, b, c) in f64) starting at the sum of the
 * counts of parts < p, in row order; d_part_counts[p] (device memory) receives part
 * p's row count.  Output buffers hold up to n rows.  The caller exchanges the parts
 * (e.g. an NCCL all-to-all, senders concatenated in rank order) and runs
 * tbgb_groupby_hash on what it received: each shard then holds the groups it owns. */
tbgb_status tbgb_hash_partition(tbgb_ctx* ctx, const int64_t* d_keys, const tbgb_columns* cols,
                                const uint64_t* d_mask, int64_t n, int32_t n_parts, int64_t* d_out_keys,
                                double* d_out_vals, int64_t* d_part_counts, void* stream);

/* ---- owner-sharded high-cardinality groupby (count / sum / mean) -------------------------
 * No counterpart in the reference (single GPU, host-side GroupIndex::build,
 * crates/tambear/src/group_index.rs:117-204).  Rows are routed by the top 9 bits of
 * h = fmix64(key) (MurmurHash3's 64-bit finaliser, a bijection): digit d = h >> 55 belongs to rank
 * d * world / 512, so each rank owns a contiguous digit range [ceil(512 r / world),
 * ceil(512 (r + 1) / world)).
 *
 * tbgb_radix_route: the rows of this shard that pass mask and pred, written as (h, v) ordered by
 * digit (all rows of digit 0, then digit 1, ...; order inside a digit unspecified), v = expr(a, b,
 * c) in f64, or the f32 column itself when the columns are f32 without expression
 * (tbgb_radix_value_bytes: 4 or 8 bytes per value).  d_digit_counts (512 int64, device) receives
 * the rows of each digit; the output buffers hold n rows.  The rows for rank r are then one
 * contiguous run, ready for an all-to-all.
 *
 * tbgb_radix_groupby_routed: the owner's side.  Sender i (0 <= i < n_senders <= 64) contributes
 * h_rows[i] rows of digits [digit_lo, digit_lo + n_digits) in digit order, starting at the device
 * addresses h_hashes[i] / h_vals[i] (host arrays): a block of a receive buffer after an
 * all-to-all, or the sender's own routed rows read in place through a peer mapping
 * (tbgb_peer_import), in which case the owner's pass reads them over NVLink and no copy is made.
 * d_seg_counts (device, n_senders * n_digits int64, sender-major) gives the rows of each
 * (sender, digit).  Groups the rows by key (recovered from h) into d_out_keys / out (count, sum,
 * mean only; other outputs must be NULL) and *d_n_groups, with the semantics and errors of
 * tbgb_groupby_hash.  The senders' rows must stay unchanged until the call's stream work is done. */
int32_t tbgb_radix_value_bytes(const tbgb_columns* cols);
tbgb_status tbgb_radix_route(tbgb_ctx* ctx, const int64_t* d_keys, const tbgb_columns* cols, const uint64_t* d_mask,
                             int64_t n, uint64_t* d_out_hashes, void* d_out_vals, int64_t* d_digit_counts,
                             void* stream);
tbgb_status tbgb_radix_groupby_routed(tbgb_ctx* ctx, int32_t n_senders, const uint64_t* const* h_hashes,
                                      const void* const* h_vals, const int64_t* h_rows, int32_t value_bytes,
                                      const int64_t* d_seg_counts, int32_t digit_lo, int32_t n_digits,
                                      int64_t max_groups, int64_t* d_out_keys, const tbgb_moments* out,
                                      int64_t* d_n_groups, void* stream);

/* Diagnostic: whether the last radix-partitioned call on `ctx` (table mode 5, or mode 0 choosing
 * it; or tbgb_radix_groupby_routed) recomputed its result with the global table.  Waits for the
 * device, then *bits = 0 (it did not) or an OR of 1 (a bucket outgrew its region: keys with very
 * many rows) or 2 (a bucket held more distinct keys than its shared-memory table).  Valid until the next groupby call on `ctx`; 0 when
 * no radix call was made.  No counterpart in the reference. */
tbgb_status tbgb_radix_fallback(tbgb_ctx* ctx, uint32_t* bits);

/* Strategy for groupbys the shared-memory column kernel cannot take alone (int64 keys,
 * more than 512 dense groups, filter / expression / f32 columns): 0 = choose by size
 * (default: dense keys take group ranges in shared memory while at most 8 ranges cover
 * them, about 32,900 groups with all moments; otherwise the global table, shared-memory
 * pre-aggregation unless the keys are many); 3 = bucket first (dense keys: stable
 * key-range partition into parts of at most 512 groups, each reduced by the column
 * kernel, up to 16384 groups; int64 keys: stable partition by high hash bits into
 * sub-tables of about 64 MB); 1 = global table with per-CTA shared-memory
 * pre-aggregation (skewed keys); 2 = global table, direct updates (uniform
 * high-cardinality keys); 4 = dense keys split into ranges of groups, each range's
 * accumulators held whole in one CTA's shared memory, the CTAs of one range sharing the
 * rows (falls back to mode 2 beyond 8 ranges; int64 keys as mode 0); 5 = int64 keys with
 * count / sum / mean outputs only and max_groups <= 2^28: radix partitioning (two streaming
 * passes by hash bits, then a shared-memory table per bucket; mode 0 chooses it for at least
 * 2^24 rows and 2^22 <= max_groups <= 2^28), other calls as mode 0; 6 = dense keys with the
 * full moments: rank and sweep (the groups split into as few ranges as keep at least two
 * value columns per group in one CTA's shared memory, up to 8 ranges, about 29,000 groups; each
 * tile's rows ranked into per-group columns with one shared u32 atomic, then one thread per
 * group folds its columns into the group's shared-memory state without atomics; one column
 * without expression and 16-byte aligned keys, else as mode 4), int64 keys as mode 0.  Mode 0
 * takes mode 6 for dense keys with the full moments where one range holds every group with at
 * least four columns (up to about 2,500 groups).  Modes 1, 2, 4 and 6 never bucket. */
tbgb_status tbgb_set_table_mode(tbgb_ctx* ctx, int mode);

/* Waits for `stream` and returns the first deferred device error of the calls
 * enqueued since the previous tbgb_sync (then clears it). */
tbgb_status tbgb_sync(tbgb_ctx* ctx, void* stream);

/* ---- row-sharded execution (one process / GPU per shard) ------------------------
 * A shard computes its mergeable per-group state table (tbgb_state_bytes(n_groups)
 * bytes, caller-owned device memory, including m3 / m4 terms); the caller exchanges the tables (e.g. an
 * NCCL all-gather over NVLink) and folds them in rank order with
 * tbgb_merge_states.  `row_offset` is the global index of the shard's first row
 * (used only to order +-0 ties exactly as the unsharded scan would). */
size_t tbgb_state_bytes(int32_t n_groups);
tbgb_status tbgb_groupby_dense_state(tbgb_ctx* ctx, const int32_t* d_keys, const double* d_vals,
                                     const uint64_t* d_mask, int64_t n, int32_t n_groups, int64_t row_offset,
                                     void* d_state, void* stream);
tbgb_status tbgb_merge_states(tbgb_ctx* ctx, const void* d_states, int32_t n_states, int32_t n_groups,
                              const tbgb_moments* out, void* stream);

/* Dense-key groupby that allocates no device memory and needs no context: for
 * callers that must not have the library allocate at call time (for example a host
 * engine that has already reserved nearly all device memory for its own buffers,
 * or a latency-critical loop that cannot accept cudaMalloc's implicit device
 * synchronisation).  No counterpart in the reference.
 * Same semantics and outputs as tbgb_groupby_dense, on the current device.
 * Limits: 1 <= n_groups <= 256 (TBGB_ERR_INVALID_ARGUMENT otherwise).  Scratch is
 * a fixed device array of about 10.5 MB inside this library.  With CUDA's default
 * lazy module loading that array is mapped on a device by the first call made there,
 * and stays mapped until the process exits: a caller that is about to reserve nearly
 * all of a device's memory makes one call on that device first (n = 0 is enough), or
 * runs with CUDA_MODULE_LOADING=EAGER.  Every call looks up the array's address on the
 * current device (cudaGetSymbolAddress); make the first call on each device before any
 * stream capture.  All calls share the array and it keeps the last call's contents
 * (the call clears what must start empty): calls that overlap on the GPU (other
 * streams, other threads) race and must be serialised by the caller.  The call waits
 * for `stream` and then returns:
 *   TBGB_OK                    outputs written
 *   TBGB_ERR_INVALID_ARGUMENT  n < 0, NULL pointers, n_groups outside [1, 256]
 *   TBGB_ERR_KEY_OUT_OF_RANGE  a selected non-NaN row has a key outside [0, n_groups)
 *   TBGB_ERR_TIMEOUT           a bounded wait inside the kernel gave up
 *   TBGB_ERR_BACKEND           no usable device (not sm_100, the array cannot be mapped)
 *                              or a device-side error bit this entry point does not name
 *   TBGB_ERR_DISPATCH          a launch or the wait for `stream` failed (for example
 *                              the stream already held an error)
 *   TBGB_ERR_TRANSFER          the read-back of the device error word failed
 * There is no context, so no message is kept for tbgb_last_error. */
tbgb_status tbgb_groupby_dense_noalloc(const int32_t* d_keys, const double* d_vals, const uint64_t* d_mask,
                                       int64_t n, int32_t n_groups, const tbgb_moments* out, void* stream);

/* Bytes of device workspace the context holds after a call of this size. */
size_t tbgb_workspace_bytes(const tbgb_ctx* ctx, int64_t n, int32_t n_groups);

/* Number of this library's kernel launches issued through `ctx` so far. */
uint64_t tbgb_launch_count(const tbgb_ctx* ctx);

/* Kernel timing: while enabled, the context records CUDA events on the launching
 * stream around each main groupby kernel.  tbgb_kernel_time_ms waits for them and
 * returns (and resets) the summed duration and the number of timed launches. */
tbgb_status tbgb_profile_enable(tbgb_ctx* ctx, int enable);
tbgb_status tbgb_kernel_time_ms(tbgb_ctx* ctx, double* total_ms, int64_t* launches);

/* ---- synthetic inputs (counter-based SplitMix64 streams) ------------------------
 * Row i of column c uses the i-th output of SplitMix64 seeded with
 * mix64(seed ^ (0xD1B54A32D192ED03 * (c + 1))) (rng.rs:64-85 stream, u01 = (x >> 11) * 2^-53).
 *   keys: x % n_groups                                   (column 0)
 *   uniform values: lo + (hi - lo) * u01                 (column 1)
 *   normal values: mu + sigma * sqrt(-2 ln u1) cos(2 pi u2), u1/u2 = outputs 2i, 2i+1 (column 1)
 * Element j of the output holds row first_row + j, so each shard of a dataset can
 * be generated where it lives. */
tbgb_status tbgb_gen_keys_uniform(tbgb_ctx* ctx, int32_t* d_keys, int64_t n, int32_t n_groups, uint64_t seed,
                                  int64_t first_row, void* stream);
tbgb_status tbgb_gen_values_uniform(tbgb_ctx* ctx, double* d_vals, int64_t n, double lo, double hi,
                                    uint64_t seed, int64_t first_row, void* stream);
tbgb_status tbgb_gen_values_normal(tbgb_ctx* ctx, double* d_vals, int64_t n, double mu, double sigma,
                                   uint64_t seed, int64_t first_row, void* stream);
/* Replace a fraction of values by NaN (u < nan_frac) and +-inf
 * (nan_frac <= u < nan_frac + inf_frac, sign from the low bit), u from column 2. */
tbgb_status tbgb_gen_inject_nonfinite(tbgb_ctx* ctx, double* d_vals, int64_t n, double nan_frac, double inf_frac,
                                      uint64_t seed, int64_t first_row, void* stream);

/* int64 keys through an inverse CDF: u = u01 of column 0, rank = first r with
 * d_cdf[r] >= u (d_cdf: n_ids increasing doubles, the last one 1.0), key =
 * mix64(rank ^ salt).  With a Zipf table this is the fused-pipeline key column. */
tbgb_status tbgb_gen_keys_cdf(tbgb_ctx* ctx, int64_t* d_keys, int64_t n, const double* d_cdf, int64_t n_ids,
                              uint64_t salt, uint64_t seed, int64_t first_row, void* stream);
/* int64 keys uniform over n_ids random ids: key = mix64((x % n_ids) ^ salt), x from column 0. */
tbgb_status tbgb_gen_keys_ids(tbgb_ctx* ctx, int64_t* d_keys, int64_t n, int64_t n_ids, uint64_t salt, uint64_t seed,
                              int64_t first_row, void* stream);
/* f32 LogNormal(mu, sigma): (float)exp(mu + sigma * z), z the normal stream of column 1. */
tbgb_status tbgb_gen_values_lognormal_f32(tbgb_ctx* ctx, float* d_vals, int64_t n, double mu, double sigma,
                                          uint64_t seed, int64_t first_row, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TAMBEAR_GB_H */
