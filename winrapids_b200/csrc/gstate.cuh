// gstate.cuh -- mergeable per-group moment state (Chan / parallel Welford) and
// the reference's output semantics, shared by the dense and table kernels.
#pragma once
#include <cstdint>

#include "common.cuh"
#include "dense.cuh"

namespace tbgb {

// Order-preserving map of doubles onto u64 (-inf < ... < -0 < +0 < ... < +inf), so
// that integer atomicMin / atomicMax compute floating-point extrema.
__device__ __forceinline__ unsigned long long f2o(double v) {
  const unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(v));
  return (b >> 63) ? ~b : (b | 0x8000000000000000ull);
}
__device__ __forceinline__ double o2f(unsigned long long o) {
  const unsigned long long b = (o >> 63) ? (o & 0x7FFFFFFFFFFFFFFFull) : ~o;
  return __longlong_as_double(static_cast<long long>(b));
}

// ---------------------------------------------------------------------------
// State folding (Chan / parallel Welford) and finalisation
// ---------------------------------------------------------------------------

// m2 / m3 / m4 are central moments of the finite values about their own mean (K + meanoff).
struct GState {
  double nn, nf, K, sumoff, meanoff, m2, mn, mx, m3, m4;
  unsigned long long zf;
};

__device__ __forceinline__ GState gstate_empty() {
  GState s;
  s.nn = 0; s.nf = 0; s.K = 0; s.sumoff = 0; s.meanoff = 0; s.m2 = 0; s.m3 = 0; s.m4 = 0;
  s.mn = pos_inf(); s.mx = neg_inf(); s.zf = ~0ull;
  return s;
}

// Central moments about the mean of n values from their power sums about a shift:
// p1 = sum(d), p2 = sum(d^2), p3 = sum(d^3), p4 = sum(d^4), d = v - K.
__device__ __forceinline__ void central_from_power(double n, double p1, double p2, double p3, double p4,
                                                   double* mu, double* m2, double* m3, double* m4) {
  const double u = p1 / n, u2 = u * u;
  *mu = u;
  *m2 = fmax(p2 - p1 * u, 0.0);
  *m3 = p3 - 3.0 * u * p2 + 2.0 * n * u2 * u;
  *m4 = fmax(p4 - 4.0 * u * p3 + 6.0 * u2 * p2 - 3.0 * n * u2 * u2, 0.0);
}

// A <- A (+) B.
__device__ __forceinline__ void gstate_fold(GState& A, const GState& B) {
  A.nn += B.nn;
  if (B.mn < A.mn) A.mn = B.mn;
  if (B.mx > A.mx) A.mx = B.mx;
  if (B.zf < A.zf) A.zf = B.zf;
  if (B.nf > 0) {
    if (A.nf == 0) {
      A.K = B.K; A.sumoff = B.sumoff; A.meanoff = B.meanoff; A.m2 = B.m2; A.nf = B.nf;
      A.m3 = B.m3; A.m4 = B.m4;
    } else {
      // Chan / Pebay pairwise merge of (n, mean, M2, M3, M4), as MomentStats::merge
      // (descriptive.rs:216-253) with the means kept relative to A's shift.
      const double off = B.K - A.K;
      A.sumoff += B.nf * off + B.sumoff;
      const double cb = off + B.meanoff;
      const double na = A.nf, nb = B.nf, n = na + nb;
      const double delta = cb - A.meanoff, d2 = delta * delta;
      A.m4 += B.m4 + d2 * d2 * (na * nb * (na * na - na * nb + nb * nb) / (n * n * n)) +
              6.0 * d2 * (na * na * B.m2 + nb * nb * A.m2) / (n * n) + 4.0 * delta * (na * B.m3 - nb * A.m3) / n;
      A.m3 += B.m3 + d2 * delta * (na * nb * (na - nb) / (n * n)) + 3.0 * delta * (na * B.m2 - nb * A.m2) / n;
      A.meanoff += delta * (nb / n);
      A.m2 += B.m2 + d2 * (na * nb / n);
      A.nf = n;
    }
  }
}

__device__ __forceinline__ GState gstate_shfl_down(const GState& s, int d) {
  GState o;
  o.nn = __shfl_down_sync(0xffffffffu, s.nn, d);
  o.nf = __shfl_down_sync(0xffffffffu, s.nf, d);
  o.K = __shfl_down_sync(0xffffffffu, s.K, d);
  o.sumoff = __shfl_down_sync(0xffffffffu, s.sumoff, d);
  o.meanoff = __shfl_down_sync(0xffffffffu, s.meanoff, d);
  o.m2 = __shfl_down_sync(0xffffffffu, s.m2, d);
  o.mn = __shfl_down_sync(0xffffffffu, s.mn, d);
  o.mx = __shfl_down_sync(0xffffffffu, s.mx, d);
  o.m3 = __shfl_down_sync(0xffffffffu, s.m3, d);
  o.m4 = __shfl_down_sync(0xffffffffu, s.m4, d);
  o.zf = __shfl_down_sync(0xffffffffu, s.zf, d);
  return o;
}

__device__ __forceinline__ GState gstate_load(const double* st, long long stride, long long idx) {
  GState s;
  s.nn = st[ST_NN * stride + idx];
  s.nf = st[ST_NF * stride + idx];
  s.K = st[ST_K * stride + idx];
  s.sumoff = st[ST_SUMOFF * stride + idx];
  s.meanoff = st[ST_MEANOFF * stride + idx];
  s.m2 = st[ST_M2 * stride + idx];
  s.mn = st[ST_MIN * stride + idx];
  s.mx = st[ST_MAX * stride + idx];
  s.m3 = st[ST_M3 * stride + idx];
  s.m4 = st[ST_M4 * stride + idx];
  s.zf = static_cast<unsigned long long>(__double_as_longlong(st[ST_ZFIRST * stride + idx]));
  return s;
}

__device__ __forceinline__ void gstate_store(double* st, long long stride, long long idx, const GState& s) {
  st[ST_NN * stride + idx] = s.nn;
  st[ST_NF * stride + idx] = s.nf;
  st[ST_K * stride + idx] = s.K;
  st[ST_SUMOFF * stride + idx] = s.sumoff;
  st[ST_MEANOFF * stride + idx] = s.meanoff;
  st[ST_M2 * stride + idx] = s.m2;
  st[ST_MIN * stride + idx] = s.mn;
  st[ST_MAX * stride + idx] = s.mx;
  st[ST_M3 * stride + idx] = s.m3;
  st[ST_M4 * stride + idx] = s.m4;
  st[ST_ZFIRST * stride + idx] = __longlong_as_double(static_cast<long long>(s.zf));
}

// Outputs in the reference's semantics (descriptive.rs:97-114, 416-418).
__device__ __forceinline__ void gstate_finalize(const GState& A, long long g, const tbgb_moments& o) {
  const double nn = A.nn;
  double sum = A.nf > 0 ? A.nf * A.K + A.sumoff : 0.0;
  if (sum == 0.0) sum = 0.0;  // the exact accumulator never yields -0.0 for an exact zero
  const double ref = nn > 0 ? sum / nn : 0.0;
  // moments about r = sum / count (the reference's pass-2 reference, which counts +-inf rows):
  // with e = mean_finite - r, sum (v - r)^k over the finite values follows from M2..M4
  double m2 = 0.0, m3 = 0.0, m4 = 0.0;
  if (A.nf > 0) {
    const double e = (A.K - ref) + A.meanoff, e2 = e * e;
    m2 = A.m2 + A.nf * e2;
    m3 = A.m3 + 3.0 * e * A.m2 + A.nf * e2 * e;
    m4 = A.m4 + 4.0 * e * A.m3 + 6.0 * e2 * A.m2 + A.nf * e2 * e2;
    if (m2 == 0.0) m2 = 0.0;
    if (m3 == 0.0) m3 = 0.0;
    if (m4 == 0.0) m4 = 0.0;
  }
  double mn = A.mn, mx = A.mx;
  if (nn > 0) {
    const double z = (A.zf & 1ull) ? -0.0 : 0.0;
    if (mn == 0.0) mn = z;
    if (mx == 0.0) mx = z;
  }
  if (o.count) o.count[g] = nn;
  if (o.sum) o.sum[g] = sum;
  if (o.min) o.min[g] = mn;
  if (o.max) o.max[g] = mx;
  if (o.mean) o.mean[g] = nn > 0 ? sum / nn : qnan();
  if (o.m2) o.m2[g] = m2;
  if (o.var_pop) o.var_pop[g] = nn > 0 ? m2 / nn : qnan();
  if (o.var_samp) o.var_samp[g] = nn - 1.0 > 0 ? m2 / (nn - 1.0) : qnan();
  if (o.m3) o.m3[g] = m3;
  if (o.m4) o.m4[g] = m4;
}

}  // namespace tbgb
