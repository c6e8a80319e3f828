// gen.cuh -- synthetic input streams (counter-based SplitMix64, rng.rs:64-85).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace tbgb {

constexpr uint64_t kGamma = 0x9e3779b97f4a7c15ULL;
constexpr uint64_t kColumnSalt = 0xD1B54A32D192ED03ULL;

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}
// i-th output (0-based) of SplitMix64::new(seed)
__host__ __device__ __forceinline__ uint64_t splitmix_at(uint64_t seed, uint64_t i) {
  return mix64(seed + (i + 1) * kGamma);
}
__host__ __device__ __forceinline__ uint64_t column_seed(uint64_t seed, uint32_t column) {
  return mix64(seed ^ (kColumnSalt * static_cast<uint64_t>(column + 1)));
}
__host__ __device__ __forceinline__ double u01(uint64_t x) {
  return static_cast<double>(x >> 11) * (1.0 / 9007199254740992.0);
}

cudaError_t gen_keys_uniform(int32_t* keys, long long n, int G, uint64_t seed, long long first, cudaStream_t s);
cudaError_t gen_values_uniform(double* vals, long long n, double lo, double hi, uint64_t seed, long long first,
                               cudaStream_t s);
cudaError_t gen_values_normal(double* vals, long long n, double mu, double sigma, uint64_t seed, long long first,
                              cudaStream_t s);
cudaError_t gen_keys_cdf(int64_t* keys, long long n, const double* cdf, long long n_ids, uint64_t salt, uint64_t seed,
                         long long first, cudaStream_t s);
cudaError_t gen_keys_ids(int64_t* keys, long long n, uint64_t n_ids, uint64_t salt, uint64_t seed, long long first,
                         cudaStream_t s);
cudaError_t gen_values_lognormal_f32(float* vals, long long n, double mu, double sigma, uint64_t seed, long long first,
                                     cudaStream_t s);
cudaError_t gen_inject_nonfinite(double* vals, long long n, double nan_frac, double inf_frac, uint64_t seed,
                                 long long first, cudaStream_t s);

}  // namespace tbgb
