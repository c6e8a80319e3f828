// mask.cuh -- row-mask algebra, predicate masks, per-tile column statistics and
// tile-skip masks (mask.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "tambear_gb.h"

namespace tbgb {

enum MaskOpCode { MASK_AND = 0, MASK_OR = 1, MASK_XOR = 2, MASK_NOT = 3 };

// out[i] = a[i] op b[i] for i < n_words; MASK_NOT ignores b and clears the bits of rows
// >= n_rows in the last word.
cudaError_t mask_op_launch(int op, const uint64_t* a, const uint64_t* b, uint64_t* out, long long n_words,
                           long long n_rows, int num_sms, cudaStream_t s, uint64_t* launches);

// *d_count = set bits of rows [0, n_rows).  d_count is zeroed on the stream first.
cudaError_t mask_popcount_launch(const uint64_t* mask, long long n_rows, unsigned long long* d_count, int num_sms,
                                 cudaStream_t s, uint64_t* launches);

// mask bit i = in(i) && pred(col[i]) for i < n (in: every row when in_mask is NULL),
// trailing bits 0 (ceil(n / 64) words); col[i] is read only where in(i) is set.
cudaError_t filter_mask_launch(const void* col, int dtype, long long n, int pred, double threshold,
                               const uint64_t* in_mask, uint64_t* mask, int num_sms, cudaStream_t s,
                               uint64_t* launches);

// TileColumnStats of every tile of tile_rows rows (the last one may be shorter).
cudaError_t tile_stats_launch(const void* col, int dtype, long long n, long long tile_rows, tbgb_tile_stats* out,
                              int num_sms, cudaStream_t s, uint64_t* launches);

// skip[t] = 1 when no row of tile t can pass `pred` (from the tile's min / max).
cudaError_t tile_skip_launch(const tbgb_tile_stats* stats, long long n_tiles, int pred, double threshold,
                             uint8_t* skip, cudaStream_t s, uint64_t* launches);

// out = in (all rows when in is NULL) with the rows of skipped tiles cleared; trailing bits 0.
cudaError_t mask_skip_tiles_launch(const uint64_t* in, const uint8_t* skip, long long tile_rows, long long n_rows,
                                   uint64_t* out, int num_sms, cudaStream_t s, uint64_t* launches);

}  // namespace tbgb
