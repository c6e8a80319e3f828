// partition.cuh -- owner routing of rows for the sharded high-cardinality groupby.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "tambear_gb.h"

namespace tbgb {

constexpr int kMaxParts = 32;

struct PartitionArgs {
  const int64_t* keys;
  tbgb_columns cols;
  const uint64_t* mask;  // nullable
  long long n;
  int P;
  int64_t* out_keys;
  double* out_vals;
};

long long partition_tiles(long long n);
size_t partition_scratch_bytes(long long n, int P);
cudaError_t partition_launch(const PartitionArgs& a, unsigned long long* scratch, int64_t* part_counts,
                             cudaStream_t s, uint64_t* launches);

}  // namespace tbgb
