// bin_stats.cuh -- statistics of sorted contiguous bins (bin_stats.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "tambear_gb.h"

namespace tbgb {

// Scratch bytes of one call (partial states of bins that cross chunk edges).
size_t bin_stats_scratch_bytes(long long n_ticks, int n_columns);

// Bins b = [boundaries[b], boundaries[b + 1]) of each of n_columns columns of n_ticks
// values (column j at data + j * n_ticks); outputs column-major [n_columns][n_bins],
// count [n_bins].
cudaError_t bin_stats_launch(const double* data, long long n_ticks, int n_columns, const int64_t* boundaries,
                             long long n_bins, const tbgb_bin_stats* out, void* scratch, uint32_t* err,
                             int num_sms, cudaStream_t s, uint64_t* launches);

}  // namespace tbgb
