// ref_bin_stats.cu -- TEST INFRASTRUCTURE ONLY: host launchers for the reference's own bin
// statistics kernels (src/winrapids/kernels/bin_stats.cu), compiled from the reference tree
// where it lies (the build recipe passes its path as REF_BIN_STATS_CU) into
// oracle/_ref/libref_bin_stats.so.  The GPU tests run it beside the product kernel on the same
// device arrays; nothing in the product loads it.
//
// Launch configuration as the reference's Python wrapper uses it
// (archive/fintek-contributions/src/fused_bin_stats.py:115-124): one thread per bin (per
// (bin, column) for the multi-column kernel), 256 threads per block.  The kernels trust their
// boundaries, so callers pass only non-decreasing boundaries within [0, n_ticks].
#include <cuda_runtime.h>

#include <cstdint>

#include REF_BIN_STATS_CU

extern "C" int ref_fused_bin_stats(const double* data, const long long* boundaries, double* sum, double* sum_sq,
                                   double* mn, double* mx, double* first, double* last, int* count, int n_bins,
                                   void* stream) {
  if (n_bins <= 0) return 0;
  const int blocks = (n_bins + 255) / 256;
  fused_bin_stats<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(data, boundaries, sum, sum_sq, mn, mx,
                                                                           first, last, count, n_bins);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int ref_fused_bin_stats_multi(const double* data, const long long* boundaries, double* sum,
                                         double* sum_sq, double* mn, double* mx, double* first, double* last,
                                         int* count, int n_bins, int n_columns, long long n_ticks, void* stream) {
  const long long total = static_cast<long long>(n_bins) * n_columns;
  if (total <= 0) return 0;
  const int blocks = static_cast<int>((total + 255) / 256);
  fused_bin_stats_multi<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      data, boundaries, sum, sum_sq, mn, mx, first, last, count, n_bins, n_columns, n_ticks);
  return static_cast<int>(cudaGetLastError());
}
