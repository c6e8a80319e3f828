// table.cuh -- global-memory accumulator tables: int64 keys (open addressing) and
// dense keys beyond the shared-memory column kernel's range.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "tambear_gb.h"

namespace tbgb {

// Slot words (u64).  FULL slot, 96 bytes: the eight words a row touches share the
// slot's first two 32-byte sectors.
//   KEY  the key (hash mode; EMPTY when free)    K   shift: first finite value seen (bits)
//   NN   non-NaN rows                            NF  finite rows
//   S1   sum(v - K) over finite rows             S2  sum((v - K)^2) over finite rows
//   MN/MX extrema over non-NaN rows, order-preserving u64 encoding
//   ID   output row of the group (hash mode)     ZF  first zero row code (row << 1 | sign)
//   S3/S4 sum((v - K)^3), sum((v - K)^4) over finite rows, when m3 / m4 are requested
// SUMCOUNT slot, 32 bytes (one sector): KEY, NN, SUM (finite values), ID.
// FULL slot words.  FL_NN: non-NaN rows; FL_NI: the +-inf ones among them (finite rows =
// FL_NN - FL_NI: a finite row, the common case, costs one counter update, not two).
enum { FL_KEY = 0, FL_K, FL_NN, FL_NI, FL_S1, FL_S2, FL_MN, FL_MX, FL_ID, FL_ZF, FL_S3, FL_S4, FL_WORDS };
enum { SC_KEY = 0, SC_NN, SC_SUM, SC_ID, SC_WORDS };

constexpr unsigned long long kEmptyKey = 0x8000000000000000ull;  // INT64_MIN marks a free slot
constexpr unsigned long long kNoId = ~0ull;
constexpr int kMaxProbe = 4096;

struct TableArgs {
  const void* keys;      // int32 (dense) or int64 (hash)
  tbgb_columns cols;
  const uint64_t* mask;  // nullable
  long long n;
  long long row_offset;  // global index of row 0 (first-zero codes)
  const int64_t* dev_count;  // when set: n = *dev_count rows starting at row *dev_start (a partition's part)
  const int64_t* dev_start;
  unsigned long long* table;
  unsigned long long slots;   // dense: n_groups; hash: power of two (plus one sentinel slot after them)
  unsigned long long* ngroups;  // hash: distinct-key counter
  long long max_groups;
  uint32_t* err;
  int m34;               // FULL slots: also accumulate sum((v-K)^3), sum((v-K)^4)
  int extrema;           // FULL slots: also track min / max / first zero
  const uint32_t* gate;  // when set, the kernels do nothing unless *gate != 0 (a fallback path)
};

struct TablePlan {
  bool hash;       // int64 keys
  bool full;       // FULL slot (else SUMCOUNT)
  bool local;      // per-CTA shared-memory pre-aggregation
  int ranges;      // dense keys: group ranges held whole in shared memory (range_table_kernel), 0 = none
  int range_groups;  // groups per range
  bool range_gk;   // FULL group ranges: shift and first-zero code in the global slot (fewer ranges)
  int sweep_cols;  // dense FULL keys by rank and sweep (sweep_table_kernel): column depth, 0 = not used
  int num_sms;
  int buckets;     // hash: sub-tables (rows bucketed by their key's high hash bits first), 1 = one table
  unsigned long long slots;       // dense: n_groups; hash: slots of each sub-table (a power of two)
  size_t table_bytes;  // including the sentinel slot and the counter word
  int grid;
  int block;
  size_t smem;
};

size_t table_slot_words(bool full);
// mode: 0 auto, 1 shared-memory pre-aggregation, 2 direct global updates, 4 group ranges in
// shared memory (dense keys); `buckets` > 1 splits a hash table into that many sub-tables
// (power of two); `m34` sizes the group-range slots for sum((v-K)^3) and sum((v-K)^4).
TablePlan table_plan(bool hash, bool full, int mode, long long n_groups_or_max, int num_sms, int buckets = 1,
                     bool m34 = true);
// Sub-table b of a bucketed hash table, and where the distinct-key counter lives.
unsigned long long* table_bucket(const TablePlan& P, unsigned long long* table, int b);
unsigned long long* table_counter(const TablePlan& P, unsigned long long* table);

// Fills every slot with its empty pattern and clears the counter.
// `gate` (nullable): run only when *gate != 0, read on the device.
cudaError_t table_init(const TablePlan& P, unsigned long long* table, cudaStream_t s, uint64_t* launches,
                       const uint32_t* gate = nullptr);
// One pass over the rows.
cudaError_t table_accumulate(const TablePlan& P, const TableArgs& a, cudaStream_t s, uint64_t* launches,
                             cudaEvent_t ev0 = nullptr, cudaEvent_t ev1 = nullptr);
// Dense mode: outputs (or, when state_out != NULL, mergeable states) for groups [0, G).
cudaError_t table_finalize_dense(const TablePlan& P, const unsigned long long* table, long long G,
                                 const tbgb_moments* out, double* state_out, cudaStream_t s, uint64_t* launches);
// Hash mode: the occupied slots, in slot order, to out_keys / out (at most max_groups of
// them); writes the group count.  `scratch` holds table_finalize_scratch_bytes(P).
size_t table_finalize_scratch_bytes(const TablePlan& P);
cudaError_t table_finalize_hash(const TablePlan& P, const unsigned long long* table, long long max_groups,
                                int64_t* out_keys, const tbgb_moments* out, int64_t* d_n_groups,
                                unsigned long long* scratch, cudaStream_t s, uint64_t* launches,
                                const uint32_t* gate = nullptr);

}  // namespace tbgb
