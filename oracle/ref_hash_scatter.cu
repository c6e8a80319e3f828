// ref_hash_scatter.cu -- TEST INFRASTRUCTURE ONLY: host launchers for the reference's own
// hash-scatter groupby kernels (scatter_stats, scatter_stats_smem, scatter_stats_warp: the
// SCATTER_CUDA_SOURCE raw string of crates/tambear/src/hash_scatter.rs).  The build recipe
// (oracle/build.py) cuts that string out of the reference tree into
// oracle/_ref/hash_scatter_kernels.cu and passes its path as REF_HASH_SCATTER_CU; the result
// is oracle/_ref/libref_hash_scatter.so.  The GPU tests and the bench run it beside the
// product kernel on the same device arrays; nothing in the product loads it.
//
// Launch configuration as HashScatterEngine uses it (hash_scatter.rs:625-731): 256 threads
// per block, one row per thread, ceil(n / 256) blocks; scatter_stats_smem takes
// 3 * n_groups * 8 bytes of dynamic shared memory.  The engine allocates its outputs zeroed
// (alloc_zeros), so the launchers clear them first.  The kernels take `int n`: callers pass
// n < 2^31 rows and keys in [0, n_groups).
#include <cuda_runtime.h>

#include REF_HASH_SCATTER_CU

namespace {

int clear3(double* sums, double* sum_sqs, double* counts, int n_groups, cudaStream_t s) {
  const size_t bytes = static_cast<size_t>(n_groups) * sizeof(double);
  if (cudaMemsetAsync(sums, 0, bytes, s) != cudaSuccess) return 1;
  if (cudaMemsetAsync(sum_sqs, 0, bytes, s) != cudaSuccess) return 1;
  if (cudaMemsetAsync(counts, 0, bytes, s) != cudaSuccess) return 1;
  return 0;
}

}  // namespace

// kind: 0 = scatter_stats (three global atomics per row), 1 = scatter_stats_smem,
// 2 = scatter_stats_warp.  Returns a cudaError_t value (0 = launched).
extern "C" int ref_scatter_stats(int kind, const int* keys, const double* values, double* sums, double* sum_sqs,
                                 double* counts, long long n, int n_groups, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n < 0 || n >= (1ll << 31) || n_groups < 1) return static_cast<int>(cudaErrorInvalidValue);
  if (clear3(sums, sum_sqs, counts, n_groups, s)) return static_cast<int>(cudaGetLastError());
  if (n == 0) return 0;
  const unsigned blocks = static_cast<unsigned>((n + 255) / 256);
  const int ni = static_cast<int>(n);
  if (kind == 0) {
    scatter_stats<<<blocks, 256, 0, s>>>(keys, values, sums, sum_sqs, counts, ni);
  } else if (kind == 1) {
    const size_t smem = static_cast<size_t>(3) * n_groups * 8;
    if (smem > 48 * 1024) {
      if (cudaFuncSetAttribute(scatter_stats_smem, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem)) != cudaSuccess)
        return static_cast<int>(cudaGetLastError());
    }
    scatter_stats_smem<<<blocks, 256, smem, s>>>(keys, values, sums, sum_sqs, counts, ni, n_groups);
  } else if (kind == 2) {
    scatter_stats_warp<<<blocks, 256, 0, s>>>(keys, values, sums, sum_sqs, counts, ni);
  } else {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  return static_cast<int>(cudaGetLastError());
}
