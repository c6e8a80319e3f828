// group_index.cuh -- group index of dense keys and first-seen codes of int64 keys.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace tbgb {

size_t group_index_scratch_bytes(long long n);
// G = max_key + 1 groups; counts G, offsets G + 1, row_to_group / rows_by_group n entries.
cudaError_t group_index_launch(const int32_t* keys, long long n, int G, uint32_t* row_to_group, uint32_t* counts,
                               uint32_t* offsets, uint32_t* rows_by_group, int64_t* n_active, void* scratch,
                               uint32_t* err, int num_sms, cudaStream_t s, uint64_t* launches);

unsigned long long factorize_slots(long long max_groups);
size_t factorize_scratch_bytes(long long n, long long max_groups);
cudaError_t factorize_launch(const int64_t* keys, long long n, long long max_groups, int32_t* codes,
                             int64_t* uniques, int64_t* n_uniques, void* scratch, uint32_t* err, int num_sms,
                             cudaStream_t s, uint64_t* launches);

}  // namespace tbgb
