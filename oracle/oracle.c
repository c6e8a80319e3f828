/*
 * oracle.c -- CPU restatement of the reference's groupby-aggregate path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Build with -ffp-contract=off: the
 * reference evaluates every expression with separately rounded f64 operations.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

typedef unsigned __int128 u128;
typedef __int128 i128;

#define KW ORC_KULISCH_WORDS
#define KWORD_BITS 128
#define KRADIX 2100   /* kulisch_accumulator.rs:57 */

/* ------------------------------------------------------------------------ */
/* KulischAccumulator (kulisch_accumulator.rs:46-330)                          */
/* ------------------------------------------------------------------------ */

void orc_kulisch_init(orc_kulisch* a) { memset(a, 0, sizeof(*a)); }

/* add_shifted_value (kulisch_accumulator.rs:137-181): two data words, then the
 * sign fill, with the same early exit once the carry reaches steady state. */
static void kulisch_add_shifted(orc_kulisch* a, int word_idx, unsigned bit_in_word, i128 signed_mant) {
  const u128 sign_fill = signed_mant < 0 ? ~(u128)0 : (u128)0;
  u128 d0, d1;
  if (bit_in_word == 0) {
    d0 = (u128)signed_mant;
    d1 = sign_fill;
  } else {
    d0 = ((u128)signed_mant) << bit_in_word;
    d1 = (u128)(signed_mant >> (KWORD_BITS - bit_in_word));
  }
  u128 carry = 0;
  for (int i = 0;; ++i) {
    const int idx = word_idx + i;
    if (idx >= KW) break;
    const u128 val = i == 0 ? d0 : (i == 1 ? d1 : sign_fill);
    const u128 w = a->w[idx];
    const u128 s1 = w + val;
    const u128 c1 = s1 < w;
    const u128 s2 = s1 + carry;
    const u128 c2 = s2 < s1;
    a->w[idx] = s2;
    carry = c1 | c2;
    if (i >= 2) {
      if (sign_fill == 0 && carry == 0) break;
      if (sign_fill == ~(u128)0 && carry == 1) break;
    }
  }
}

/* add_f64 (kulisch_accumulator.rs:81-129): +-0, NaN and +-inf are ignored. */
void orc_kulisch_add(orc_kulisch* a, double x) {
  if (x == 0.0 || !isfinite(x)) return;
  uint64_t bits;
  memcpy(&bits, &x, 8);
  const uint64_t sign = bits >> 63;
  const int raw_exp = (int)((bits >> 52) & 0x7FF);
  const uint64_t raw_mant = bits & 0x000FFFFFFFFFFFFFULL;
  uint64_t mant;
  int exp;
  if (raw_exp == 0) {
    mant = raw_mant;
    exp = -1074;
  } else {
    mant = raw_mant | (1ULL << 52);
    exp = raw_exp - 1023 - 52;
  }
  const i128 signed_mant = sign ? -(i128)mant : (i128)mant;
  const int bit_pos = exp + KRADIX;
  kulisch_add_shifted(a, bit_pos / KWORD_BITS, (unsigned)(bit_pos % KWORD_BITS), signed_mant);
}

/* merge (kulisch_accumulator.rs:210-221): word-wise add with carry. */
void orc_kulisch_merge(orc_kulisch* a, const orc_kulisch* b) {
  u128 carry = 0;
  for (int i = 0; i < KW; ++i) {
    const u128 x = a->w[i];
    const u128 s1 = x + b->w[i];
    const u128 c1 = s1 < x;
    const u128 s2 = s1 + carry;
    const u128 c2 = s2 < s1;
    a->w[i] = s2;
    carry = c1 | c2;
  }
}

static int clz128(u128 v) {
  const uint64_t hi = (uint64_t)(v >> 64), lo = (uint64_t)v;
  if (hi) return __builtin_clzll(hi);
  return 64 + __builtin_clzll(lo);
}

static uint64_t extract_bits(const u128* mag, int start, int count) {
  if (count == 0) return 0;
  const int end = start + count - 1;
  const int sw = start / KWORD_BITS, ew = end / KWORD_BITS, sb = start % KWORD_BITS;
  const u128 mask = count == 64 ? (u128)UINT64_MAX : (((u128)1 << count) - 1);
  if (sw >= KW) return 0;
  if (sw == ew || ew >= KW) return (uint64_t)((mag[sw] >> sb) & mask);
  const u128 low = mag[sw] >> sb;
  const u128 high = mag[ew] << (KWORD_BITS - sb);
  return (uint64_t)((low | high) & mask);
}

static int bits_below_are_zero(const u128* mag, int pos) {
  const int wi = pos / KWORD_BITS, bi = pos % KWORD_BITS;
  for (int i = 0; i < wi && i < KW; ++i)
    if (mag[i] != 0) return 0;
  if (wi < KW && bi > 0) {
    const u128 m = ((u128)1 << bi) - 1;
    if ((mag[wi] & m) != 0) return 0;
  }
  return 1;
}

static double from_bits(uint64_t b) {
  double d;
  memcpy(&d, &b, 8);
  return d;
}

/* to_f64 (kulisch_accumulator.rs:225-330): round to nearest, ties to even. */
double orc_kulisch_to_f64(const orc_kulisch* a) {
  const int neg = (i128)a->w[KW - 1] < 0;
  u128 mag[KW];
  if (neg) {
    u128 carry = 1;
    for (int i = 0; i < KW; ++i) {
      const u128 inv = ~a->w[i];
      const u128 s = inv + carry;
      carry = s < inv;
      mag[i] = s;
    }
  } else {
    memcpy(mag, a->w, sizeof(mag));
  }
  int msb = -1;
  for (int i = KW - 1; i >= 0; --i) {
    if (mag[i] != 0) {
      msb = i * KWORD_BITS + (KWORD_BITS - clz128(mag[i])) - 1;
      break;
    }
  }
  if (msb < 0) return neg ? -0.0 : 0.0;
  const int exp_unbiased = msb - KRADIX;
  if (exp_unbiased > 1023) return neg ? -INFINITY : INFINITY;
  const uint64_t sign_bit = neg ? (1ULL << 63) : 0;
  if (exp_unbiased <= -1023) {
    const int SUB_LSB = KRADIX - 1074; /* 1026 */
    if (msb < SUB_LSB) return neg ? -0.0 : 0.0;
    const uint64_t mant_sub = extract_bits(mag, SUB_LSB, 52);
    const uint64_t round = extract_bits(mag, SUB_LSB - 1, 1) & 1;
    const int sticky = !bits_below_are_zero(mag, SUB_LSB - 1);
    uint64_t fm = mant_sub;
    if (round == 1 && (sticky || (fm & 1) == 1)) fm += 1;
    if (fm == (1ULL << 52)) return from_bits(sign_bit | (1ULL << 52));
    return from_bits(sign_bit | fm);
  }
  const uint64_t m52 = extract_bits(mag, msb - 52, 52);
  const uint64_t round = msb >= 53 ? (extract_bits(mag, msb - 53, 1) & 1) : 0;
  const int sticky = msb >= 54 ? !bits_below_are_zero(mag, msb - 53) : 0;
  uint64_t fm = m52;
  int fe = exp_unbiased;
  if (round == 1 && (sticky || (m52 & 1) == 1)) {
    fm += 1;
    if (fm == (1ULL << 52)) {
      fm = 0;
      fe += 1;
      if (fe > 1023) return neg ? -INFINITY : INFINITY;
    }
  }
  return from_bits(sign_bit | ((uint64_t)(fe + 1023) << 52) | fm);
}

double orc_exact_sum(const double* x, int64_t n) {
  orc_kulisch a;
  orc_kulisch_init(&a);
  for (int64_t i = 0; i < n; ++i) orc_kulisch_add(&a, x[i]);
  return orc_kulisch_to_f64(&a);
}

/* ------------------------------------------------------------------------ */
/* phi whitelist (compute_engine.rs:593-609)                                   */
/* ------------------------------------------------------------------------ */

double orc_phi_eval(int phi, double v, double r) {
  switch (phi) {
    case ORC_PHI_V: return v;
    case ORC_PHI_VV: return v * v;
    case ORC_PHI_ONE: return 1.0;
    case ORC_PHI_VMR: return v - r;
    case ORC_PHI_VMR2: return (v - r) * (v - r);
    case ORC_PHI_ABS_VMR: return fabs(v - r);
    case ORC_PHI_VMR3: { const double d = v - r; return d * d * d; }
    case ORC_PHI_VMR4: { const double d = v - r; const double d2 = d * d; return d2 * d2; }
    case ORC_PHI_VR: return v * r;
    case ORC_PHI_LOG: return log(v);
    case ORC_PHI_RECIP: return 1.0 / v;
    default: return NAN;
  }
}

static int keys_in_range(const int32_t* keys, int64_t n, int32_t n_groups) {
  for (int64_t i = 0; i < n; ++i)
    if (keys[i] < 0 || keys[i] >= n_groups) return 0;
  return 1;
}

/* ------------------------------------------------------------------------ */
/* ComputeEngine CPU scatters (compute_engine.rs:232-322)                      */
/* ------------------------------------------------------------------------ */

int orc_scatter_phi(int phi, const int32_t* keys, const double* vals, const double* refs, int64_t n,
                    int32_t n_groups, double* out) {
  if (phi < 0 || phi >= ORC_PHI_COUNT_ || n_groups < 0) return -2;
  if (!keys_in_range(keys, n, n_groups)) return -1;
  orc_kulisch* acc = (orc_kulisch*)calloc((size_t)(n_groups ? n_groups : 1), sizeof(orc_kulisch));
  for (int64_t i = 0; i < n; ++i) {
    const int g = keys[i];
    orc_kulisch_add(&acc[g], orc_phi_eval(phi, vals[i], refs ? refs[g] : 0.0));
  }
  for (int g = 0; g < n_groups; ++g) out[g] = orc_kulisch_to_f64(&acc[g]);
  free(acc);
  return 0;
}

int orc_scatter_multi_phi(const int* phis, int n_phi, const int32_t* keys, const double* vals,
                          const double* refs, int64_t n, int32_t n_groups, double* out) {
  if (n_phi < 1 || n_phi > 5) return -2; /* compute_engine.rs:118 */
  for (int j = 0; j < n_phi; ++j)
    if (phis[j] < 0 || phis[j] >= ORC_PHI_COUNT_) return -2;
  if (!keys_in_range(keys, n, n_groups)) return -1;
  const size_t ng = (size_t)(n_groups ? n_groups : 1);
  orc_kulisch* acc = (orc_kulisch*)calloc(ng * (size_t)n_phi, sizeof(orc_kulisch));
  for (int64_t i = 0; i < n; ++i) {
    const int g = keys[i];
    const double v = vals[i], r = refs ? refs[g] : 0.0;
    for (int j = 0; j < n_phi; ++j) orc_kulisch_add(&acc[(size_t)j * ng + g], orc_phi_eval(phis[j], v, r));
  }
  for (int j = 0; j < n_phi; ++j)
    for (int g = 0; g < n_groups; ++g) out[(size_t)j * n_groups + g] = orc_kulisch_to_f64(&acc[(size_t)j * ng + g]);
  free(acc);
  return 0;
}

int orc_scatter_phi_masked(int phi, const int32_t* keys, const double* vals, const double* refs,
                           const uint64_t* mask, int64_t n, int32_t n_groups, double* out) {
  if (phi < 0 || phi >= ORC_PHI_COUNT_) return -2;
  orc_kulisch* acc = (orc_kulisch*)calloc((size_t)(n_groups ? n_groups : 1), sizeof(orc_kulisch));
  for (int64_t i = 0; i < n; ++i) {
    if (((mask[i / 64] >> (i % 64)) & 1) == 0) continue;
    const int g = keys[i];
    if (g < 0 || g >= n_groups) { free(acc); return -1; }
    orc_kulisch_add(&acc[g], orc_phi_eval(phi, vals[i], refs ? refs[g] : 0.0));
  }
  for (int g = 0; g < n_groups; ++g) out[g] = orc_kulisch_to_f64(&acc[g]);
  free(acc);
  return 0;
}

int orc_scatter_extremum(int is_max, const int32_t* keys, const double* vals, int64_t n, int32_t n_groups,
                         double* out) {
  if (!keys_in_range(keys, n, n_groups)) return -1;
  for (int g = 0; g < n_groups; ++g) out[g] = is_max ? -INFINITY : INFINITY;
  for (int64_t i = 0; i < n; ++i) {
    const int g = keys[i];
    if (is_max) {
      if (vals[i] > out[g]) out[g] = vals[i];
    } else {
      if (vals[i] < out[g]) out[g] = vals[i];
    }
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* masks and map2                                                              */
/* ------------------------------------------------------------------------ */

/* nan_mask_count (descriptive.rs:591-603): bit set iff !is_nan. */
int64_t orc_nan_mask(const double* vals, int64_t n, uint64_t* mask) {
  const int64_t words = (n + 63) / 64;
  memset(mask, 0, (size_t)words * 8);
  int64_t n_nan = 0;
  for (int64_t i = 0; i < n; ++i) {
    if (isnan(vals[i])) n_nan++;
    else mask[i / 64] |= 1ULL << (i % 64);
  }
  return n_nan;
}

/* eval_filter (filter_jit.rs:202-243): bit set iff (row < n) && pred(v);
 * trailing bits of the last word stay 0. */
void orc_filter_mask(int pred, double thr, const double* vals, int64_t n, uint64_t* mask) {
  const int64_t words = (n + 63) / 64;
  memset(mask, 0, (size_t)words * 8);
  for (int64_t i = 0; i < n; ++i) {
    const double v = vals[i];
    int p = 0;
    switch (pred) {
      case ORC_PRED_GT: p = v > thr; break;
      case ORC_PRED_LT: p = v < thr; break;
      case ORC_PRED_GE: p = v >= thr; break;
      case ORC_PRED_LE: p = v <= thr; break;
      case ORC_PRED_NOT_NAN: p = v == v; break;
      case ORC_PRED_FINITE: p = (v == v) && (v * 0.0 == 0.0); break;
      default: p = 0;
    }
    if (p) mask[i / 64] |= 1ULL << (i % 64);
  }
}

/* mask_and / mask_or / mask_xor (filter_jit.rs:151-166): word by word. */
void orc_mask_and(const uint64_t* a, const uint64_t* b, int64_t n_words, uint64_t* out) {
  for (int64_t i = 0; i < n_words; ++i) out[i] = a[i] & b[i];
}
void orc_mask_or(const uint64_t* a, const uint64_t* b, int64_t n_words, uint64_t* out) {
  for (int64_t i = 0; i < n_words; ++i) out[i] = a[i] | b[i];
}
void orc_mask_xor(const uint64_t* a, const uint64_t* b, int64_t n_words, uint64_t* out) {
  for (int64_t i = 0; i < n_words; ++i) out[i] = a[i] ^ b[i];
}

/* mask_not (filter_jit.rs:173-181): flip every word, then keep only the n_rows % 64
 * valid bits of word n_rows / 64 when n_rows is not a multiple of 64. */
void orc_mask_not(const uint64_t* a, int64_t n_words, int64_t n_rows, uint64_t* out) {
  for (int64_t i = 0; i < n_words; ++i) out[i] = ~a[i];
  const int64_t rem = n_rows % 64;
  if (rem != 0) out[n_rows / 64] &= (1ULL << rem) - 1;
}

/* mask_popcount (filter_jit.rs:130-144): full words, then the valid bits of the last. */
int64_t orc_mask_popcount(const uint64_t* mask, int64_t n_rows) {
  const int64_t full = n_rows / 64, rem = n_rows % 64;
  int64_t c = 0;
  for (int64_t i = 0; i < full; ++i) c += __builtin_popcountll(mask[i]);
  if (rem != 0) c += __builtin_popcountll(mask[full] & ((1ULL << rem) - 1));
  return c;
}

/* TileColumnStats::from_slice (format.rs:82-107): strict `<` / `>` scans from +-inf and a
 * Kahan-compensated running sum, in row order. */
void orc_tile_stats_build(const double* vals, int64_t n, int64_t tile_rows, orc_tile_stats* out) {
  const int64_t n_tiles = n > 0 ? (n + tile_rows - 1) / tile_rows : 0;
  for (int64_t t = 0; t < n_tiles; ++t) {
    const int64_t lo = t * tile_rows, hi = lo + tile_rows < n ? lo + tile_rows : n;
    double mn = INFINITY, mx = -INFINITY, sum = 0.0, c = 0.0;
    for (int64_t i = lo; i < hi; ++i) {
      const double v = vals[i];
      if (v < mn) mn = v;
      if (v > mx) mx = v;
      const double y = v - c;
      const double tt = sum + y;
      c = (tt - sum) - y;
      sum = tt;
    }
    out[t].min = mn;
    out[t].max = mx;
    out[t].sum = sum;
    out[t].count = (uint32_t)(hi - lo);
    out[t].n_valid = (uint32_t)(hi - lo);
    out[t].reserved = 0;
  }
}

/* can_skip_gt / _lt / _gte / _lte (format.rs:111-136), tile_skip_mask_gt / _lt (:182-189). */
void orc_tile_skip(const orc_tile_stats* st, int64_t n_tiles, int pred, double thr, uint8_t* skip) {
  for (int64_t t = 0; t < n_tiles; ++t) {
    int s = 0;
    switch (pred) {
      case ORC_PRED_GT: s = st[t].max <= thr; break;
      case ORC_PRED_LT: s = st[t].min >= thr; break;
      case ORC_PRED_GE: s = st[t].max < thr; break;
      case ORC_PRED_LE: s = st[t].min > thr; break;
      default: s = 0;
    }
    skip[t] = (uint8_t)s;
  }
}

/* fused_bin_stats (bin_stats.cu:25-77): per bin, count = hi - lo; an empty bin is NaN
 * everywhere; otherwise sum and sum_sq accumulate in row order, min and max start from the
 * bin's first value with strict `<` / `>`, first / last are the end values.  (The reference
 * kernel is compiled with fused multiply-add contraction on, so its sum_sq rounds once per
 * row; this restatement rounds the product and the sum separately, a last-bit difference.) */
void orc_bin_stats(const double* data, const int64_t* boundaries, int64_t n_bins, double* sum, double* sum_sq,
                   double* mn, double* mx, double* first, double* last, int32_t* count) {
  for (int64_t b = 0; b < n_bins; ++b) {
    const int64_t lo = boundaries[b], hi = boundaries[b + 1];
    count[b] = (int32_t)(hi - lo);
    if (hi - lo == 0) {
      sum[b] = sum_sq[b] = mn[b] = mx[b] = first[b] = last[b] = NAN;
      continue;
    }
    double s = 0.0, q = 0.0, lo_v = data[lo], hi_v = data[lo];
    for (int64_t i = lo; i < hi; ++i) {
      const double v = data[i];
      s += v;
      q += v * v;
      if (v < lo_v) lo_v = v;
      if (v > hi_v) hi_v = v;
    }
    sum[b] = s;
    sum_sq[b] = q;
    mn[b] = lo_v;
    mx[b] = hi_v;
    first[b] = data[lo];
    last[b] = data[hi - 1];
  }
}

/* phi_map2_eval (compute_engine.rs:627-636). */
void orc_map2(int op, const double* a, const double* b, int64_t n, double* out) {
  for (int64_t i = 0; i < n; ++i) {
    switch (op) {
      case ORC_MAP2_ADD: out[i] = a[i] + b[i]; break;
      case ORC_MAP2_MUL: out[i] = a[i] * b[i]; break;
      case ORC_MAP2_SUB: out[i] = a[i] - b[i]; break;
      case ORC_MAP2_MUL_PLUS1: out[i] = a[i] * b[i] + 1.0; break;
      default: out[i] = NAN;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* moments_grouped (descriptive.rs:383-435), composed like the reference        */
/* ------------------------------------------------------------------------ */

static void extremum_nan_safe(const double* vals, const int32_t* keys, int64_t n, int32_t G, double* mins,
                              double* maxs) {
  for (int g = 0; g < G; ++g) { mins[g] = INFINITY; maxs[g] = -INFINITY; }
  for (int64_t i = 0; i < n; ++i) {
    const double v = vals[i];
    if (isnan(v)) continue;
    const int g = keys[i];
    if (v < mins[g]) mins[g] = v;
    if (v > maxs[g]) maxs[g] = v;
  }
}

int orc_moments_grouped(const double* vals, const int32_t* keys, int64_t n, int32_t G, orc_moments* o) {
  if (!keys_in_range(keys, n, G)) return -1;
  const int64_t words = (n + 63) / 64;
  uint64_t* mask = (uint64_t*)malloc((size_t)(words ? words : 1) * 8);
  const int64_t n_nan = orc_nan_mask(vals, n, mask);
  const int has_nan = n_nan > 0;
  double* tmp = (double*)malloc((size_t)(G ? G : 1) * 8 * 3);
  double* means = (double*)malloc((size_t)(G ? G : 1) * 8);
  /* pass 1 */
  if (has_nan) {
    orc_scatter_phi_masked(ORC_PHI_V, keys, vals, NULL, mask, n, G, o->sums);
    orc_scatter_phi_masked(ORC_PHI_ONE, keys, vals, NULL, mask, n, G, o->counts);
    extremum_nan_safe(vals, keys, n, G, o->mins, o->maxs);
  } else {
    const int p1[2] = {ORC_PHI_V, ORC_PHI_ONE};
    orc_scatter_multi_phi(p1, 2, keys, vals, NULL, n, G, tmp);
    memcpy(o->sums, tmp, (size_t)G * 8);
    memcpy(o->counts, tmp + G, (size_t)G * 8);
    orc_scatter_extremum(0, keys, vals, n, G, o->mins);
    orc_scatter_extremum(1, keys, vals, n, G, o->maxs);
  }
  for (int g = 0; g < G; ++g) means[g] = o->counts[g] > 0.0 ? o->sums[g] / o->counts[g] : 0.0;
  /* pass 2 */
  if (has_nan) {
    orc_scatter_phi_masked(ORC_PHI_VMR2, keys, vals, means, mask, n, G, o->m2s);
    if (o->m3s) orc_scatter_phi_masked(ORC_PHI_VMR3, keys, vals, means, mask, n, G, o->m3s);
    if (o->m4s) orc_scatter_phi_masked(ORC_PHI_VMR4, keys, vals, means, mask, n, G, o->m4s);
  } else {
    const int p2[3] = {ORC_PHI_VMR2, ORC_PHI_VMR3, ORC_PHI_VMR4};
    orc_scatter_multi_phi(p2, 3, keys, vals, means, n, G, tmp);
    memcpy(o->m2s, tmp, (size_t)G * 8);
    if (o->m3s) memcpy(o->m3s, tmp + G, (size_t)G * 8);
    if (o->m4s) memcpy(o->m4s, tmp + 2 * (size_t)G, (size_t)G * 8);
  }
  free(mask);
  free(tmp);
  free(means);
  return 0;
}

/* Filtered variant: rows whose filter bit is 0 never reach the groupby; on the
 * remaining rows the composition above applies unchanged. */
int orc_moments_grouped_masked(const double* vals, const int32_t* keys, const uint64_t* fmask, int64_t n,
                               int32_t G, orc_moments* o) {
  int64_t m = 0;
  for (int64_t i = 0; i < n; ++i)
    if ((fmask[i / 64] >> (i % 64)) & 1) m++;
  double* v2 = (double*)malloc((size_t)(m ? m : 1) * 8);
  int32_t* k2 = (int32_t*)malloc((size_t)(m ? m : 1) * 4);
  m = 0;
  for (int64_t i = 0; i < n; ++i)
    if ((fmask[i / 64] >> (i % 64)) & 1) { v2[m] = vals[i]; k2[m] = keys[i]; m++; }
  const int rc = orc_moments_grouped(v2, k2, m, G, o);
  free(v2);
  free(k2);
  return rc;
}

/* ------------------------------------------------------------------------ */
/* Multi-threaded restatement (bit-identical): contiguous row ranges            */
/* ------------------------------------------------------------------------ */

typedef struct {
  const double* vals;
  const int32_t* keys;
  const uint64_t* mask;
  int64_t lo, hi;
  int32_t G;
  int pass;
  const double* means;
  orc_kulisch* k0; /* pass1: sum; pass2: m2 */
  orc_kulisch* k1; /* pass2: m3 */
  orc_kulisch* k2; /* pass2: m4 */
  int64_t* cnt;
  double *mn, *mx;
  int bad_key;
} mt_job;

static void* mt_worker(void* p) {
  mt_job* j = (mt_job*)p;
  for (int64_t i = j->lo; i < j->hi; ++i) {
    if (j->mask && (((j->mask[i / 64] >> (i % 64)) & 1) == 0)) continue;
    const double v = j->vals[i];
    if (isnan(v)) continue;
    const int g = j->keys[i];
    if (g < 0 || g >= j->G) { j->bad_key = 1; return NULL; }
    if (j->pass == 1) {
      orc_kulisch_add(&j->k0[g], v);
      j->cnt[g]++;
      if (v < j->mn[g]) j->mn[g] = v;
      if (v > j->mx[g]) j->mx[g] = v;
    } else {
      const double r = j->means[g];
      orc_kulisch_add(&j->k0[g], orc_phi_eval(ORC_PHI_VMR2, v, r));
      if (j->k1) orc_kulisch_add(&j->k1[g], orc_phi_eval(ORC_PHI_VMR3, v, r));
      if (j->k2) orc_kulisch_add(&j->k2[g], orc_phi_eval(ORC_PHI_VMR4, v, r));
    }
  }
  return NULL;
}

int orc_moments_grouped_mt(const double* vals, const int32_t* keys, const uint64_t* mask, int64_t n, int32_t G,
                           int T, orc_moments* o) {
  if (T < 1) T = 1;
  if (T > 256) T = 256;
  const size_t ng = (size_t)(G ? G : 1);
  mt_job* jobs = (mt_job*)calloc((size_t)T, sizeof(mt_job));
  pthread_t* th = (pthread_t*)calloc((size_t)T, sizeof(pthread_t));
  const int want34 = o->m3s != NULL || o->m4s != NULL;
  for (int t = 0; t < T; ++t) {
    mt_job* j = &jobs[t];
    j->vals = vals; j->keys = keys; j->mask = mask; j->G = G;
    j->lo = n * t / T; j->hi = n * (t + 1) / T;
    j->k0 = (orc_kulisch*)calloc(ng, sizeof(orc_kulisch));
    j->k1 = want34 ? (orc_kulisch*)calloc(ng, sizeof(orc_kulisch)) : NULL;
    j->k2 = want34 ? (orc_kulisch*)calloc(ng, sizeof(orc_kulisch)) : NULL;
    j->cnt = (int64_t*)calloc(ng, 8);
    j->mn = (double*)malloc(ng * 8);
    j->mx = (double*)malloc(ng * 8);
    for (size_t g = 0; g < ng; ++g) { j->mn[g] = INFINITY; j->mx[g] = -INFINITY; }
    j->pass = 1;
  }
  int rc = 0;
  for (int t = 0; t < T; ++t) pthread_create(&th[t], NULL, mt_worker, &jobs[t]);
  for (int t = 0; t < T; ++t) pthread_join(th[t], NULL);
  for (int t = 0; t < T; ++t) if (jobs[t].bad_key) rc = -1;
  double* means = (double*)malloc(ng * 8);
  if (rc == 0) {
    for (int g = 0; g < G; ++g) {
      orc_kulisch s;
      orc_kulisch_init(&s);
      int64_t c = 0;
      double mn = INFINITY, mx = -INFINITY;
      for (int t = 0; t < T; ++t) { /* range order: earlier range wins ties */
        orc_kulisch_merge(&s, &jobs[t].k0[g]);
        c += jobs[t].cnt[g];
        if (jobs[t].mn[g] < mn) mn = jobs[t].mn[g];
        if (jobs[t].mx[g] > mx) mx = jobs[t].mx[g];
      }
      o->sums[g] = orc_kulisch_to_f64(&s);
      o->counts[g] = (double)c;
      o->mins[g] = mn;
      o->maxs[g] = mx;
      means[g] = o->counts[g] > 0.0 ? o->sums[g] / o->counts[g] : 0.0;
    }
    for (int t = 0; t < T; ++t) {
      memset(jobs[t].k0, 0, ng * sizeof(orc_kulisch));
      jobs[t].pass = 2;
      jobs[t].means = means;
    }
    for (int t = 0; t < T; ++t) pthread_create(&th[t], NULL, mt_worker, &jobs[t]);
    for (int t = 0; t < T; ++t) pthread_join(th[t], NULL);
    for (int g = 0; g < G; ++g) {
      orc_kulisch a, b, c;
      orc_kulisch_init(&a); orc_kulisch_init(&b); orc_kulisch_init(&c);
      for (int t = 0; t < T; ++t) {
        orc_kulisch_merge(&a, &jobs[t].k0[g]);
        if (want34) { orc_kulisch_merge(&b, &jobs[t].k1[g]); orc_kulisch_merge(&c, &jobs[t].k2[g]); }
      }
      o->m2s[g] = orc_kulisch_to_f64(&a);
      if (o->m3s) o->m3s[g] = orc_kulisch_to_f64(&b);
      if (o->m4s) o->m4s[g] = orc_kulisch_to_f64(&c);
    }
  }
  for (int t = 0; t < T; ++t) {
    free(jobs[t].k0); free(jobs[t].k1); free(jobs[t].k2);
    free(jobs[t].cnt); free(jobs[t].mn); free(jobs[t].mx);
  }
  free(jobs);
  free(th);
  free(means);
  return rc;
}

/* ------------------------------------------------------------------------ */
/* int64 keys: factorise by sorting (key, row), stream one register per group    */
/* ------------------------------------------------------------------------ */

typedef struct { int64_t key; int64_t row; } kr_pair;

static int cmp_pair(const void* a, const void* b) {
  const kr_pair* x = (const kr_pair*)a;
  const kr_pair* y = (const kr_pair*)b;
  if (x->key != y->key) return x->key < y->key ? -1 : 1;
  return x->row < y->row ? -1 : (x->row > y->row ? 1 : 0);
}

int64_t orc_groupby_i64(const int64_t* keys, const double* vals, const uint64_t* mask, int64_t n,
                        int64_t* out_keys, orc_moments* o) {
  int64_t m = 0;
  kr_pair* p = (kr_pair*)malloc((size_t)(n ? n : 1) * sizeof(kr_pair));
  for (int64_t i = 0; i < n; ++i) {
    if (mask && (((mask[i / 64] >> (i % 64)) & 1) == 0)) continue;
    p[m].key = keys[i];
    p[m].row = i;
    m++;
  }
  qsort(p, (size_t)m, sizeof(kr_pair), cmp_pair);
  int64_t ng = 0;
  for (int64_t s = 0; s < m;) {
    int64_t e = s;
    while (e < m && p[e].key == p[s].key) e++;
    orc_kulisch ks, k2, k3, k4;
    orc_kulisch_init(&ks);
    int64_t c = 0;
    double mn = INFINITY, mx = -INFINITY;
    for (int64_t q = s; q < e; ++q) {
      const double v = vals[p[q].row];
      if (isnan(v)) continue;
      orc_kulisch_add(&ks, v);
      c++;
      if (v < mn) mn = v;
      if (v > mx) mx = v;
    }
    const double sum = orc_kulisch_to_f64(&ks);
    const double cnt = (double)c;
    const double mean = cnt > 0.0 ? sum / cnt : 0.0;
    orc_kulisch_init(&k2); orc_kulisch_init(&k3); orc_kulisch_init(&k4);
    for (int64_t q = s; q < e; ++q) {
      const double v = vals[p[q].row];
      if (isnan(v)) continue;
      orc_kulisch_add(&k2, orc_phi_eval(ORC_PHI_VMR2, v, mean));
      if (o->m3s) orc_kulisch_add(&k3, orc_phi_eval(ORC_PHI_VMR3, v, mean));
      if (o->m4s) orc_kulisch_add(&k4, orc_phi_eval(ORC_PHI_VMR4, v, mean));
    }
    out_keys[ng] = p[s].key;
    o->counts[ng] = cnt;
    o->sums[ng] = sum;
    o->mins[ng] = mn;
    o->maxs[ng] = mx;
    o->m2s[ng] = orc_kulisch_to_f64(&k2);
    if (o->m3s) o->m3s[ng] = orc_kulisch_to_f64(&k3);
    if (o->m4s) o->m4s[ng] = orc_kulisch_to_f64(&k4);
    ng++;
    s = e;
  }
  free(p);
  return ng;
}

/* ------------------------------------------------------------------------ */
/* MomentStats derived values (descriptive.rs:97-114)                          */
/* ------------------------------------------------------------------------ */

double orc_mean(double count, double sum) { return count == 0.0 ? NAN : sum / count; }

double orc_variance(double count, double m2, int ddof) {
  const double denom = count - (double)ddof;
  if (denom <= 0.0) return NAN;
  return m2 / denom;
}

/* ------------------------------------------------------------------------ */
/* SplitMix64 as a counter-based stream (rng.rs:64-85)                          */
/* ------------------------------------------------------------------------ */

uint64_t orc_mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

uint64_t orc_splitmix_at(uint64_t seed, uint64_t i) { return orc_mix64(seed + (i + 1) * 0x9e3779b97f4a7c15ULL); }

uint64_t orc_column_seed(uint64_t seed, uint32_t column) {
  return orc_mix64(seed ^ (0xD1B54A32D192ED03ULL * (uint64_t)(column + 1)));
}

double orc_u01(uint64_t x) { return (double)(x >> 11) / 9007199254740992.0; }
