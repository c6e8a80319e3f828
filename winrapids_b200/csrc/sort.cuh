// sort.cuh -- stable LSD radix sort of (key, value) pairs on the device.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace tbgb {

// Scratch the counts need for n pairs.
size_t sort_counts_bytes(long long n);
// Sorts the low `bits` bits of the keys (a multiple of 8 passes), stably; keys/vals are
// sorted in place (keys_tmp / vals_tmp: n elements of scratch each).  With vals_are_rows
// the values start as the row index i (vals need not be initialised).  n < 2^32.
cudaError_t sort_pairs_u32(uint32_t* keys, uint32_t* vals, long long n, int bits, uint32_t* keys_tmp,
                           uint32_t* vals_tmp, unsigned int* counts, cudaStream_t s, uint64_t* launches,
                           bool vals_are_rows);
cudaError_t sort_pairs_u64(unsigned long long* keys, uint32_t* vals, long long n, int bits,
                           unsigned long long* keys_tmp, uint32_t* vals_tmp, unsigned int* counts, cudaStream_t s,
                           uint64_t* launches, bool vals_are_rows);

}  // namespace tbgb
