// partition.cuh -- stable partition of rows: owner routing of int64 keys and key-range
// bucketing of dense int32 keys.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "tambear_gb.h"

namespace tbgb {

constexpr int kMaxParts = 32;

struct PartitionArgs {
  const void* keys;      // int64 (owner routing) or int32 (key ranges)
  tbgb_columns cols;
  const uint64_t* mask;  // nullable
  long long n;
  int P;
  bool range;            // key-range bucketing (int32 keys) instead of owner routing
  int width;             // range: groups per part
  int n_groups;          // range: valid keys are [0, n_groups)
  int align_rows;        // part starts rounded up to a multiple of this many rows (>= 1)
  void* out_keys;        // int64 (owner routing) or int32 rebased keys (key ranges)
  double* out_vals;
  uint32_t* err;
};

long long partition_tiles(long long n);
size_t partition_scratch_bytes(long long n, int P);
// Rows the output buffers need (n plus the alignment padding of P parts).
size_t partition_output_rows(long long n, int P, int align_rows);
// part_counts / part_starts: P int64 each (device).
cudaError_t partition_launch(const PartitionArgs& a, unsigned long long* scratch, int64_t* part_counts,
                             int64_t* part_starts, cudaStream_t s, uint64_t* launches);

}  // namespace tbgb
