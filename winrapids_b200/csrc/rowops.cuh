// rowops.cuh -- per-row helpers shared by the table and partition kernels: column
// loads, the fused predicate / expression, key hashing.
#pragma once
#include <cstdint>

#include "common.cuh"
#include "tambear_gb.h"

namespace tbgb {

// MurmurHash3's 64-bit finaliser (public domain): spreads keys over the table.
__device__ __forceinline__ unsigned long long fmix64(unsigned long long k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return k;
}

__device__ __forceinline__ unsigned long long dbits(double v) {
  return static_cast<unsigned long long>(__double_as_longlong(v));
}
__device__ __forceinline__ double bitsd(unsigned long long b) { return __longlong_as_double(static_cast<long long>(b)); }

template <bool F32>
__device__ __forceinline__ double load_val(const void* p, long long i) {
  if constexpr (F32) return static_cast<double>(__ldcs(static_cast<const float*>(p) + i));
  else return __ldcs(static_cast<const double*>(p) + i);
}

template <bool KEY64>
__device__ __forceinline__ long long load_key(const void* p, long long i) {
  if constexpr (KEY64) return __ldcs(static_cast<const long long*>(p) + i);
  else return static_cast<long long>(__ldcs(static_cast<const int*>(p) + i));
}

// Expression of the reference's map_phi2 CPU whitelist (compute_engine.rs:627-636)
// plus `(a*b)+c`; every operation rounded on its own, no contraction.
__device__ __forceinline__ double eval_expr(int expr, double a, double b, double c) {
  switch (expr) {
    case TBGB_EXPR_ADD: return __dadd_rn(a, b);
    case TBGB_EXPR_SUB: return __dsub_rn(a, b);
    case TBGB_EXPR_MUL: return __dmul_rn(a, b);
    case TBGB_EXPR_MUL_PLUS1: return __dadd_rn(__dmul_rn(a, b), 1.0);
    case TBGB_EXPR_MUL_ADD: return __dadd_rn(__dmul_rn(a, b), c);
    default: return a;
  }
}

// Predicate on column a; comparisons with NaN fail (filter_jit.rs:196-243).
__device__ __forceinline__ bool eval_pred(int pred, double a, double t) {
  switch (pred) {
    case TBGB_PRED_GT: return a > t;
    case TBGB_PRED_GE: return a >= t;
    case TBGB_PRED_LT: return a < t;
    case TBGB_PRED_LE: return a <= t;
    case TBGB_PRED_NOT_NAN: return !is_nan(a);
    case TBGB_PRED_FINITE: return is_finite(a);
    default: return true;
  }
}

}  // namespace tbgb
