// radix.cuh -- int64-key groupby of count / sum / mean by radix partitioning, for key spaces
// too large for a table that stays in L2 (hundreds of millions of distinct keys).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "tambear_gb.h"

namespace tbgb {

constexpr int kRadixDigits = 512;               // first-pass buckets (the top 9 hash bits)
constexpr int kRadixBuckets = 262144;           // final buckets after the second pass (18 hash bits)
constexpr long long kRadixMaxGroups = 1ll << 28;  // distinct keys one call serves (1024 per bucket)
constexpr int kRadixMaxSenders = 64;            // senders of a routed groupby

struct RadixPlan {
  bool vf32;                  // rows carry the value as f32 (an f32 column without expression)
  unsigned long long cap1;    // rows per first-pass bucket (slack over an even share)
  unsigned long long cap2;    // rows per final bucket
  size_t t1_bytes;            // first-pass buffer: cap1 * 512 hashes + values
  size_t t2_bytes;            // final buffer: cap2 * 65536 hashes + values
  size_t aux_bytes;           // cursors, tile prefix, flags
  int grid_scatter;           // CTAs of the scatter passes
  int grid_agg;               // CTAs of the bucket aggregation
};

// Whether a hash groupby of `n` rows with this column set and these outputs takes the radix
// path in the automatic mode (count / sum / mean only, many groups, many rows).
bool radix_eligible(const tbgb_columns& cols, const tbgb_moments* out, long long n, long long max_groups);

RadixPlan radix_plan(const tbgb_columns& cols, long long n, int num_sms);

struct RadixArgs {
  const int64_t* keys;
  tbgb_columns cols;
  const uint64_t* mask;  // nullable
  long long n;
  long long max_groups;
  int64_t* out_keys;
  tbgb_moments out;      // count / sum / mean (others ignored)
  int64_t* d_n_groups;
  uint32_t* err;         // KERR_TABLE_FULL when more than max_groups keys
};

// Enqueues the three passes (partition by the top 9 hash bits, then by the next 9, then one CTA
// per bucket aggregating in a shared-memory table) and the group count.  `ws` holds
// t1_bytes + t2_bytes + aux_bytes.  `*fallback` (a device word inside ws, returned) is non-zero
// after the passes when a bucket overflowed its slack or its shared-memory table: the caller
// then recomputes the whole result with another strategy, gated on that word.
cudaError_t radix_groupby(const RadixPlan& P, const RadixArgs& a, void* ws, uint32_t** fallback, cudaStream_t s,
                          uint64_t* launches, cudaEvent_t ev0 = nullptr, cudaEvent_t ev1 = nullptr);

// Where the passes keep their buffers inside ws (the fallback table may reuse t2's space).
size_t radix_t2_offset(const RadixPlan& P);

// ---- owner-sharded use: routing on the sender, grouping on the owner -----------------
// Rows carry the value as f32 when the column is f32 and there is no expression.
bool radix_value_f32(const tbgb_columns& cols);
size_t radix_route_aux_bytes();
// The first pass with exact placement (a counting pass first): the rows that pass mask and
// predicate, as (h, v) ordered by the top 9 bits of h; digit_counts (kRadixDigits int64, device)
// receives the rows of each digit.  `aux` holds radix_route_aux_bytes().
cudaError_t radix_route(const RadixArgs& a, unsigned long long* out_h, void* out_v, int64_t* digit_counts, void* aux,
                        int num_sms, cudaStream_t s, uint64_t* launches);

struct RoutedArgs {
  // sender s's rows of digits [digit_lo, digit_lo + n_digits), in digit order, start at hashes[s] /
  // vals[s] (device addresses: this GPU's memory or a peer's buffer mapped here)
  const unsigned long long* hashes[kRadixMaxSenders];
  const void* vals[kRadixMaxSenders];
  const int64_t* seg_counts;         // rows per (sender, digit), sender-major (device)
  int n_senders;
  int digit_lo;
  int n_digits;
  long long n_rows;
  long long max_groups;
  int64_t* out_keys;
  tbgb_moments out;
  int64_t* d_n_groups;
  uint32_t* err;
};
// Plan of the owner's passes over n_rows received rows of n_digits digits (t1 unused).
RadixPlan radix_routed_plan(bool vf32, long long n_rows, int n_digits, int num_sms);
cudaError_t radix_groupby_routed(const RadixPlan& P, const RoutedArgs& r, void* ws, uint32_t** fallback,
                                 cudaStream_t s, uint64_t* launches, cudaEvent_t ev0 = nullptr,
                                 cudaEvent_t ev1 = nullptr);
// A fallback that grouped hashes writes hashes as keys: turn them back into keys (gated).
cudaError_t radix_unhash_keys(int64_t* keys, const int64_t* d_n_groups, long long max_groups, const uint32_t* gate,
                              int num_sms, cudaStream_t s, uint64_t* launches);

}  // namespace tbgb
