/*
 * oracle.h -- CPU restatement of the reference's groupby-aggregate path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (winrapids_b200/) links,
 * imports or calls this code; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py use it, and only as the
 * checker or the timed CPU baseline.
 *
 * What it restates (paths are relative to the reference project root):
 *   - KulischAccumulator   crates/tambear/src/primitives/specialist/kulisch_accumulator.rs:46-330
 *   - ComputeEngine CPU    crates/tambear/src/compute_engine.rs:232-322 (scatter_phi / _multi /
 *                          _masked / scatter_extremum), phi whitelist :593-609, map2 :627-636
 *   - moments_grouped      crates/tambear/src/descriptive.rs:383-435, nan_mask_count :591-603,
 *                          extremum_grouped_nan_safe :606-620, MomentStats :97-114
 *   - filter mask          crates/tambear/src/filter_jit.rs:196-243 (bit i of word i/64 <-> row i)
 *   - mask algebra         crates/tambear/src/filter_jit.rs:130-181 (mask_and / or / xor / not / popcount)
 *   - tile statistics      crates/tambear/src/format.rs:82-136,182-189 (TileColumnStats::from_slice,
 *                          can_skip_*, tile_skip_mask_gt / _lt)
 *   - bin statistics       src/winrapids/kernels/bin_stats.cu:25-77 (fused_bin_stats, one bin's loop)
 *   - SplitMix64 / u01 / Box-Muller  crates/tambear/src/rng.rs:34-36,64-85,165-176
 *
 * Parity is pinned by the reference's own golden vectors (see tests/test_oracle_golden.py).
 */
#ifndef TAMBEAR_GB_ORACLE_H
#define TAMBEAR_GB_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Kulisch exact accumulator (34 x 128-bit words, radix point 2100 bits above LSB) ---- */
#define ORC_KULISCH_WORDS 34
typedef struct { unsigned __int128 w[ORC_KULISCH_WORDS]; } orc_kulisch;

void   orc_kulisch_init(orc_kulisch* a);
void   orc_kulisch_add(orc_kulisch* a, double x);        /* ignores +-0, NaN, +-inf */
void   orc_kulisch_merge(orc_kulisch* a, const orc_kulisch* b);
double orc_kulisch_to_f64(const orc_kulisch* a);         /* round to nearest even */
double orc_exact_sum(const double* x, int64_t n);        /* Kulisch sum of a slice */

/* ---- phi expressions (compute_engine.rs:593-609) ---- */
enum {
  ORC_PHI_V = 0,           /* "v"                                */
  ORC_PHI_VV = 1,          /* "v * v"                            */
  ORC_PHI_ONE = 2,         /* "1.0"                              */
  ORC_PHI_VMR = 3,         /* "(v - r)" | "v - r"                */
  ORC_PHI_VMR2 = 4,        /* "(v - r) * (v - r)"                */
  ORC_PHI_ABS_VMR = 5,     /* "fabs(v - r)" | "abs(v - r)"       */
  ORC_PHI_VMR3 = 6,        /* "(v - r) * (v - r) * (v - r)"      */
  ORC_PHI_VMR4 = 7,        /* "(v - r) * (v - r) * (v - r) * (v - r)" */
  ORC_PHI_VR = 8,          /* "v * r"                            */
  ORC_PHI_LOG = 9,         /* "log(v)"                           */
  ORC_PHI_RECIP = 10,      /* "1.0 / v"                          */
  ORC_PHI_COUNT_ = 11
};
double orc_phi_eval(int phi, double v, double r);

/* Return codes: 0 ok, -1 key out of range (the reference panics on an
 * out-of-bounds index), -2 bad argument. */
int orc_scatter_phi(int phi, const int32_t* keys, const double* vals, const double* refs /*nullable*/,
                    int64_t n, int32_t n_groups, double* out);
int orc_scatter_multi_phi(const int* phis, int n_phi, const int32_t* keys, const double* vals,
                          const double* refs, int64_t n, int32_t n_groups, double* out /* n_phi*n_groups */);
int orc_scatter_phi_masked(int phi, const int32_t* keys, const double* vals, const double* refs,
                           const uint64_t* mask, int64_t n, int32_t n_groups, double* out);
int orc_scatter_extremum(int is_max, const int32_t* keys, const double* vals, int64_t n,
                         int32_t n_groups, double* out);

/* ---- NaN mask, predicate mask, map2 ---- */
int64_t orc_nan_mask(const double* vals, int64_t n, uint64_t* mask);   /* returns NaN count */
enum { ORC_PRED_GT = 0, ORC_PRED_NOT_NAN = 1, ORC_PRED_FINITE = 2, ORC_PRED_LT = 3, ORC_PRED_GE = 4, ORC_PRED_LE = 5 };
void orc_filter_mask(int pred, double threshold, const double* vals, int64_t n, uint64_t* mask);
enum { ORC_MAP2_ADD = 0, ORC_MAP2_MUL = 1, ORC_MAP2_SUB = 2, ORC_MAP2_MUL_PLUS1 = 3 };
void orc_map2(int op, const double* a, const double* b, int64_t n, double* out);

/* ---- mask algebra (filter_jit.rs:130-181) ---- */
void orc_mask_and(const uint64_t* a, const uint64_t* b, int64_t n_words, uint64_t* out);
void orc_mask_or(const uint64_t* a, const uint64_t* b, int64_t n_words, uint64_t* out);
void orc_mask_xor(const uint64_t* a, const uint64_t* b, int64_t n_words, uint64_t* out);
void orc_mask_not(const uint64_t* a, int64_t n_words, int64_t n_rows, uint64_t* out);
int64_t orc_mask_popcount(const uint64_t* mask, int64_t n_rows);

/* ---- per-tile column statistics (format.rs:60-136,182-189) ---- */
typedef struct {
  double min, max, sum;
  uint32_t count, n_valid;
  uint64_t reserved;
} orc_tile_stats;
/* TileColumnStats::from_slice of every tile of tile_rows rows (serial Kahan sum). */
void orc_tile_stats_build(const double* vals, int64_t n, int64_t tile_rows, orc_tile_stats* out);
/* can_skip_gt / _gte / _lt / _lte with pred ORC_PRED_GT / GE / LT / LE. */
void orc_tile_skip(const orc_tile_stats* st, int64_t n_tiles, int pred, double threshold, uint8_t* skip);

/* ---- statistics of sorted contiguous bins (bin_stats.cu:25-77), serial per bin ---- */
void orc_bin_stats(const double* data, const int64_t* boundaries, int64_t n_bins, double* sum, double* sum_sq,
                   double* mn, double* mx, double* first, double* last, int32_t* count);

/* ---- grouped moments: descriptive.rs:383-435 (counts, sums, mins, maxs, m2s, m3s, m4s) ---- */
typedef struct {
  double *counts, *sums, *mins, *maxs, *m2s, *m3s, *m4s;   /* each n_groups long; m3s/m4s nullable */
} orc_moments;
/* Faithful composition through the scatter primitives (single-threaded, the
 * reference's own execution model). */
int orc_moments_grouped(const double* vals, const int32_t* keys, int64_t n, int32_t n_groups, orc_moments* out);
/* Same result, bit for bit: contiguous row ranges per thread, per-thread Kulisch
 * registers merged in range order, extrema merged first-range-wins. */
int orc_moments_grouped_mt(const double* vals, const int32_t* keys, const uint64_t* mask /*nullable*/,
                           int64_t n, int32_t n_groups, int n_threads, orc_moments* out);
/* Masked variant of the composition (rows whose mask bit is 0 are skipped before
 * the NaN mask is applied), used for filter -> groupby. */
int orc_moments_grouped_masked(const double* vals, const int32_t* keys, const uint64_t* mask,
                               int64_t n, int32_t n_groups, orc_moments* out);

/* ---- int64 keys: factorise (sorted unique, row order kept inside a key), then moments ---- */
/* Returns the number of distinct keys among rows that pass mask (nullable);
 * out_keys must hold up to n entries; out arrays sized like out_keys. */
int64_t orc_groupby_i64(const int64_t* keys, const double* vals, const uint64_t* mask, int64_t n,
                        int64_t* out_keys, orc_moments* out);

/* ---- derived statistics (MomentStats, descriptive.rs:97-114) ---- */
double orc_mean(double count, double sum);
double orc_variance(double count, double m2, int ddof);

/* ---- synthetic input streams (rng.rs SplitMix64 as a counter-based stream) ---- */
uint64_t orc_splitmix_at(uint64_t seed, uint64_t i);   /* i-th output of SplitMix64::new(seed) */
uint64_t orc_mix64(uint64_t z);
uint64_t orc_column_seed(uint64_t seed, uint32_t column);
double   orc_u01(uint64_t x);

#ifdef __cplusplus
}
#endif
#endif
