// dense.cuh -- constants and host launchers of the dense-key groupby kernels.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "tambear_gb.h"

namespace tbgb {

constexpr int kDenseThreads = 800;  // threads per CTA (25 warps)
constexpr int kDenseTile = 4096;    // rows per staged tile (one batch of the column buffers)
constexpr int kDenseStages = 2;     // depth of the TMA ring (2 x 48.5 KB in flight per CTA)
constexpr int kDenseMaxGroups = 1024;
constexpr int kDenseColBudget = 14336;  // 2 * C * n_groups doubles of column buffers (112 KiB; C = 28 at 256 groups)

// Mergeable per-group state, stored as structure-of-arrays with ST_COUNT rows.
//   nn       non-NaN rows          nf       finite rows
//   K        shift of this state   sumoff   sum(v - K) over finite rows
//   meanoff  mean(v) - K           m2       sum((v - mean)^2) over finite rows
//   min/max  over non-NaN rows     zfirst   (first zero row << 1 | sign), bits of a u64
//   m3, m4   sum((v - mean)^3), sum((v - mean)^4) over finite rows (0 when not requested)
enum { ST_NN = 0, ST_NF, ST_K, ST_SUMOFF, ST_MEANOFF, ST_M2, ST_MIN, ST_MAX, ST_ZFIRST, ST_M3, ST_M4, ST_COUNT };

// u64 words per group of a CTA's spill state (counts, +-inf counts, shift, power sums, extrema).
constexpr int kDenseSpillFields = 10;

struct DenseLaunch {
  int grid;       // CTAs
  int C;          // column capacity
  int opg;        // owners per group
  int slots;      // n_groups * opg
  int maxslots;   // owner slots per thread (1 or 2)
  size_t smem;    // dynamic shared memory bytes
  size_t part_doubles;  // ST_COUNT * grid * slots
  size_t spill_words;   // per-CTA spill states (u64 words)
};

DenseLaunch dense_plan(int n_groups, int num_sms);
size_t dense_smem_bytes(int G, int C);

// Enqueue the dense moments pipeline.  `part` holds part_doubles, `spill`
// spill_words u64, `zfirst` G u64, `err` one u32.  Writes either final outputs (`out`) or, when `state_out` is not
// NULL, the merged state table of this call (ST_COUNT * G doubles).
struct PushArgs;
cudaError_t dense_moments_launch(const DenseLaunch& L, const int32_t* keys, const double* vals, const uint64_t* mask,
                                 long long n, long long row_offset, int G, double* part, unsigned long long* spill,
                                 unsigned long long* zfirst, uint32_t* err, const tbgb_moments* out, double* state_out,
                                 cudaStream_t stream, uint64_t* launches, cudaEvent_t ev_start = nullptr,
                                 cudaEvent_t ev_stop = nullptr, unsigned* live_scratch = nullptr,
                                 bool state_m34 = true, const PushArgs* push = nullptr);
// push (nullable, with state_out): the fold also stores the state table into the same slot of
// every peer's exchange buffer and its last block raises this rank's flag there (exchange.cuh).
// state_m34 = false: the state table's m3 / m4 are left at zero (cheaper kernel) for callers
// whose final outputs need neither.
// Scratch of the live-tile list of a masked launch over n rows (u32 words).
size_t dense_live_scratch_bytes(long long n);

cudaError_t merge_states_launch(const double* states, int n_states, int G, const tbgb_moments* out,
                                cudaStream_t stream, uint64_t* launches);

}  // namespace tbgb
