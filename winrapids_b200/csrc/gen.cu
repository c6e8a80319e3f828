// gen.cu -- synthetic input generators for the groupby workloads.
//
// Column c of a workload seeded with `seed` is the SplitMix64 stream of
// column_seed(seed, c); row i reads output i (uniforms) or outputs 2i, 2i+1
// (Box-Muller normals, rng.rs:165-176 uses the cosine branch).  Integer outputs
// (keys, uniform mantissas, NaN/inf positions) are bit-identical to any host
// implementation of the same recipe; normals use CUDA's log/cos and can differ
// from a host libm by an ulp.
#include "gen.cuh"

namespace tbgb {

namespace {

constexpr int kGenThreads = 256;

int gen_blocks(long long n) {
  long long b = (n + kGenThreads - 1) / kGenThreads;
  if (b > 148LL * 64) b = 148LL * 64;
  return b < 1 ? 1 : static_cast<int>(b);
}

__global__ void k_keys_uniform(int32_t* keys, long long n, int G, uint64_t cs, long long first) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    keys[i] = static_cast<int32_t>(splitmix_at(cs, static_cast<uint64_t>(first + i)) % static_cast<uint64_t>(G));
}

__global__ void k_values_uniform(double* v, long long n, double lo, double hi, uint64_t cs, long long first) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    v[i] = __dadd_rn(lo, __dmul_rn(hi - lo, u01(splitmix_at(cs, static_cast<uint64_t>(first + i)))));
}

__global__ void k_values_normal(double* v, long long n, double mu, double sigma, uint64_t cs, long long first) {
  const double two_pi = 6.283185307179586;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint64_t r = static_cast<uint64_t>(first + i);
    double u1 = u01(splitmix_at(cs, 2 * r));
    const double u2 = u01(splitmix_at(cs, 2 * r + 1));
    if (u1 <= 0.0) u1 = 1.0 / 9007199254740992.0;  // the reference redraws u1 <= 1e-300
    const double rad = sqrt(__dmul_rn(-2.0, log(u1)));
    const double z = __dmul_rn(rad, cos(__dmul_rn(two_pi, u2)));
    v[i] = __dadd_rn(mu, __dmul_rn(sigma, z));
  }
}

__global__ void k_inject(double* v, long long n, double nan_frac, double inf_frac, uint64_t cs, long long first) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint64_t x = splitmix_at(cs, static_cast<uint64_t>(first + i));
    const double u = u01(x);
    if (u < nan_frac) v[i] = __longlong_as_double(0x7FF8000000000000LL);
    else if (u < nan_frac + inf_frac)
      v[i] = (x & 1) ? __longlong_as_double(static_cast<long long>(0xFFF0000000000000ULL))
                     : __longlong_as_double(0x7FF0000000000000LL);
  }
}

// int64 keys drawn through an inverse CDF: rank = first r with cdf[r] >= u (the
// table's last entry is 1.0), key = mix64(rank ^ salt) -- random 64-bit ids with the
// rank distribution of the table (Zipf for the fused-pipeline workload).
__global__ void k_keys_cdf(int64_t* keys, long long n, const double* __restrict__ cdf, long long n_ids, uint64_t salt,
                           uint64_t cs, long long first) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const double u = u01(splitmix_at(cs, static_cast<uint64_t>(first + i)));
    long long lo = 0, hi = n_ids - 1;
    while (lo < hi) {
      const long long mid = (lo + hi) >> 1;
      if (cdf[mid] >= u) hi = mid;
      else lo = mid + 1;
    }
    keys[i] = static_cast<int64_t>(mix64(static_cast<uint64_t>(lo) ^ salt));
  }
}

// int64 keys uniform over n_ids random 64-bit ids: key = mix64((x % n_ids) ^ salt).
__global__ void k_keys_ids(int64_t* keys, long long n, uint64_t n_ids, uint64_t salt, uint64_t cs, long long first) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    keys[i] = static_cast<int64_t>(mix64((splitmix_at(cs, static_cast<uint64_t>(first + i)) % n_ids) ^ salt));
}

// f32 LogNormal(mu, sigma): exp of the column's normal stream, rounded to f32.
__global__ void k_values_lognormal_f32(float* v, long long n, double mu, double sigma, uint64_t cs, long long first) {
  const double two_pi = 6.283185307179586;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint64_t r = static_cast<uint64_t>(first + i);
    double u1 = u01(splitmix_at(cs, 2 * r));
    const double u2 = u01(splitmix_at(cs, 2 * r + 1));
    if (u1 <= 0.0) u1 = 1.0 / 9007199254740992.0;
    const double z = __dmul_rn(sqrt(__dmul_rn(-2.0, log(u1))), cos(__dmul_rn(two_pi, u2)));
    v[i] = static_cast<float>(exp(__dadd_rn(mu, __dmul_rn(sigma, z))));
  }
}

}  // namespace

cudaError_t gen_keys_cdf(int64_t* keys, long long n, const double* cdf, long long n_ids, uint64_t salt, uint64_t seed,
                         long long first, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_keys_cdf<<<gen_blocks(n), kGenThreads, 0, s>>>(keys, n, cdf, n_ids, salt, column_seed(seed, 0), first);
  return cudaGetLastError();
}

cudaError_t gen_keys_ids(int64_t* keys, long long n, uint64_t n_ids, uint64_t salt, uint64_t seed, long long first,
                         cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_keys_ids<<<gen_blocks(n), kGenThreads, 0, s>>>(keys, n, n_ids, salt, column_seed(seed, 0), first);
  return cudaGetLastError();
}

cudaError_t gen_values_lognormal_f32(float* vals, long long n, double mu, double sigma, uint64_t seed, long long first,
                                     cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_values_lognormal_f32<<<gen_blocks(n), kGenThreads, 0, s>>>(vals, n, mu, sigma, column_seed(seed, 1), first);
  return cudaGetLastError();
}

cudaError_t gen_keys_uniform(int32_t* keys, long long n, int G, uint64_t seed, long long first, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_keys_uniform<<<gen_blocks(n), kGenThreads, 0, s>>>(keys, n, G, column_seed(seed, 0), first);
  return cudaGetLastError();
}

cudaError_t gen_values_uniform(double* vals, long long n, double lo, double hi, uint64_t seed, long long first,
                               cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_values_uniform<<<gen_blocks(n), kGenThreads, 0, s>>>(vals, n, lo, hi, column_seed(seed, 1), first);
  return cudaGetLastError();
}

cudaError_t gen_values_normal(double* vals, long long n, double mu, double sigma, uint64_t seed, long long first,
                              cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_values_normal<<<gen_blocks(n), kGenThreads, 0, s>>>(vals, n, mu, sigma, column_seed(seed, 1), first);
  return cudaGetLastError();
}

cudaError_t gen_inject_nonfinite(double* vals, long long n, double nan_frac, double inf_frac, uint64_t seed,
                                 long long first, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_inject<<<gen_blocks(n), kGenThreads, 0, s>>>(vals, n, nan_frac, inf_frac, column_seed(seed, 2), first);
  return cudaGetLastError();
}

}  // namespace tbgb
