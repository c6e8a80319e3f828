// partition.cu -- stable partition of rows into parts, for two uses:
//   * owner routing of int64 keys (sharded high-cardinality groupby; no counterpart in the
//     reference, which runs on one GPU): part = (fmix64(key) >> 32) % P, the high hash bits,
//     independent of the low bits a table uses inside a part.  Rows that pass the mask and
//     the predicate are written as (key, v = expr(a, b, c) in f64); NaN rows are kept (they
//     still create their key's group).  The same routing buckets one GPU's rows so that each
//     bucket's table slice is small.
//   * key-range bucketing of dense int32 keys: part = key / width, written as (key - part *
//     width, v), so that each part is a dense groupby of at most `width` groups for the
//     shared-memory column kernel.  NaN rows are dropped (a dense groupby ignores them and
//     never checks their keys); a non-NaN row whose key is outside [0, n_groups) sets
//     KERR_KEY_RANGE and is dropped.
// Each part's rows keep their row order (a stable partition), so every key's rows keep
// their relative order -- which keeps the +-0 tie rule of the extrema exact downstream.
// Parts may be padded to start on a multiple of `align_rows` rows (16-byte aligned part
// starts for the bulk copies of the column kernel).
//
// Three launches over fixed tiles of 65,536 rows: per-tile part counts, one block scanning
// the [part][tile] count matrix into write offsets (plus the part counts and padded part
// starts), and the scatter (per 1024-row step: the lanes of each part found with one match, one
// warp per part scanning the warps' counts, rows written at running offset + prefix +
// rank in warp, from one __match_any_sync over the part ids).  Counting uses the same match.
#include <cstdint>

#include "common.cuh"
#include "partition.cuh"
#include "rowops.cuh"

namespace tbgb {

namespace {

constexpr int PNT = 1024;                // threads per block
constexpr long long PTILE = 65536;       // rows per tile
constexpr int PSTEPS = PTILE / PNT;      // 1024-row steps per tile
constexpr int SCAN_NT = 1024;

__device__ __forceinline__ int owner_of(unsigned long long key, int P) {
  return static_cast<int>((fmix64(key) >> 32) % static_cast<unsigned long long>(P));
}

// Part of row `row`, or -1 when the row is dropped; `key` / `v` receive what is written.
template <bool RANGE, bool F32>
__device__ __forceinline__ int route_row(const PartitionArgs& a, long long row, long long* key, double* v) {
  if (row >= a.n) return -1;
  if (a.mask && !((__ldg(a.mask + (row >> 6)) >> (row & 63)) & 1ull)) return -1;
  const double av = load_val<F32>(a.cols.a, row);
  if (!eval_pred(a.cols.pred, av, a.cols.threshold)) return -1;
  const int expr = a.cols.expr;
  const double bv = expr != TBGB_EXPR_A ? load_val<F32>(a.cols.b, row) : 0.0;
  const double cv = expr == TBGB_EXPR_MUL_ADD ? load_val<F32>(a.cols.c, row) : 0.0;
  *v = eval_expr(expr, av, bv, cv);
  if constexpr (RANGE) {
    if (is_nan(*v)) return -1;
    const int k = __ldcs(static_cast<const int*>(a.keys) + row);
    if (static_cast<unsigned>(k) >= static_cast<unsigned>(a.n_groups)) {
      atomicOr(a.err, KERR_KEY_RANGE);
      return -1;
    }
    const int p = k / a.width;
    *key = k - p * a.width;
    return p;
  } else {
    *key = __ldcs(static_cast<const long long*>(a.keys) + row);
    return owner_of(static_cast<unsigned long long>(*key), a.P);
  }
}

template <bool RANGE, bool F32>
__global__ void __launch_bounds__(PNT) part_count_kernel(PartitionArgs a, long long ntiles,
                                                         unsigned long long* tile_counts) {
  __shared__ unsigned int cnt[kMaxParts];
  const long long t = blockIdx.x;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x < a.P) cnt[threadIdx.x] = 0;
  __syncthreads();
  const long long base = t * PTILE;
  for (int s = 0; s < PSTEPS; ++s) {
    long long key;
    double v;
    const int d = route_row<RANGE, F32>(a, base + static_cast<long long>(s) * PNT + threadIdx.x, &key, &v);
    // the lanes of each part: the lowest adds their number
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    if (d >= 0 && lane == __ffs(peers) - 1) atomicAdd(cnt + d, static_cast<unsigned>(__popc(peers)));
  }
  __syncthreads();
  if (threadIdx.x < a.P) tile_counts[static_cast<long long>(threadIdx.x) * ntiles + t] = cnt[threadIdx.x];
}

// Exclusive scan of the [P][ntiles] count matrix (part-major) in one block; writes the
// offsets in place (unpadded), the per-part totals and the padded part starts.
__global__ void __launch_bounds__(SCAN_NT) part_scan_kernel(unsigned long long* counts, long long len, int P,
                                                            long long ntiles, int align, int64_t* part_counts,
                                                            int64_t* part_starts) {
  __shared__ unsigned long long warp_sums[SCAN_NT / 32];
  __shared__ unsigned long long carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (long long base = 0; base < len; base += SCAN_NT) {
    const long long i = base + threadIdx.x;
    const unsigned long long x = i < len ? counts[i] : 0ull;
    unsigned long long inc = x;
    for (int d = 1; d < 32; d <<= 1) {
      const unsigned long long y = __shfl_up_sync(0xffffffffu, inc, d);
      if (lane >= d) inc += y;
    }
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    if (warp == 0) {
      unsigned long long w = warp_sums[lane];
      for (int d = 1; d < 32; d <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= d) w += y;
      }
      warp_sums[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const unsigned long long before = carry + (warp > 0 ? warp_sums[warp - 1] : 0ull) + inc - x;
    if (i < len) counts[i] = before;
    __syncthreads();
    if (threadIdx.x == SCAN_NT - 1) carry = before + x;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    unsigned long long start = 0;
    for (int p = 0; p < P; ++p) {
      const unsigned long long s0 = counts[static_cast<long long>(p) * ntiles];
      const unsigned long long s1 = p + 1 < P ? counts[static_cast<long long>(p + 1) * ntiles] : carry;
      part_counts[p] = static_cast<int64_t>(s1 - s0);
      part_starts[p] = static_cast<int64_t>(start);
      start += s1 - s0;
      start = (start + align - 1) / align * align;
    }
  }
}

template <bool RANGE, bool F32>
__global__ void __launch_bounds__(PNT) part_scatter_kernel(PartitionArgs a, long long ntiles,
                                                           const unsigned long long* __restrict__ offsets,
                                                           const int64_t* __restrict__ part_starts) {
  constexpr int NW = PNT / 32;
  __shared__ unsigned int wcnt[NW][kMaxParts];  // per warp, per part: rows in this step, then their prefix
  __shared__ unsigned int total[kMaxParts];
  __shared__ unsigned long long running[kMaxParts];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long t = blockIdx.x;
  const int P = a.P;
  if (threadIdx.x < P) {
    const long long d = threadIdx.x;
    running[d] = static_cast<unsigned long long>(part_starts[d]) + offsets[d * ntiles + t] - offsets[d * ntiles];
  }
  const unsigned lt = (1u << lane) - 1u;
  const long long base = t * PTILE;
  for (int s = 0; s < PSTEPS; ++s) {
    long long key = 0;
    double v = 0.0;
    const int d = route_row<RANGE, F32>(a, base + static_cast<long long>(s) * PNT + threadIdx.x, &key, &v);
    // rank among this warp's rows of the same part; the part's lowest lane records their number
    if (lane < P) wcnt[warp][lane] = 0;
    __syncwarp();
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    const unsigned int rank = __popc(peers & lt);
    if (d >= 0 && rank == 0) wcnt[warp][d] = __popc(peers);
    __syncthreads();
    // warp p turns column p of wcnt into exclusive prefixes over the warps (lane = warp index)
    if (warp < P) {
      const unsigned c = wcnt[lane][warp];
      unsigned inc = c;
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
      }
      wcnt[lane][warp] = inc - c;
      if (lane == 31) total[warp] = inc;
    }
    __syncthreads();
    if (d >= 0) {
      const unsigned long long off = running[d] + wcnt[warp][d] + rank;
      if constexpr (RANGE) static_cast<int32_t*>(a.out_keys)[off] = static_cast<int32_t>(key);
      else static_cast<int64_t*>(a.out_keys)[off] = static_cast<int64_t>(key);
      a.out_vals[off] = v;
    }
    __syncthreads();
    if (threadIdx.x < P) running[threadIdx.x] += total[threadIdx.x];
    // the next step's writes of wcnt / total and reads of running are ordered by its first barrier
  }
}

template <bool RANGE, bool F32>
cudaError_t launch_all(const PartitionArgs& a, long long ntiles, unsigned long long* scratch, int64_t* part_counts,
                       int64_t* part_starts, cudaStream_t s) {
  part_count_kernel<RANGE, F32><<<static_cast<unsigned int>(ntiles), PNT, 0, s>>>(a, ntiles, scratch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  part_scan_kernel<<<1, SCAN_NT, 0, s>>>(scratch, ntiles * a.P, a.P, ntiles, a.align_rows, part_counts, part_starts);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  part_scatter_kernel<RANGE, F32><<<static_cast<unsigned int>(ntiles), PNT, 0, s>>>(a, ntiles, scratch, part_starts);
  return cudaGetLastError();
}

__global__ void part_empty_kernel(int64_t* part_counts, int64_t* part_starts, int P) {
  if (threadIdx.x < P) {
    part_counts[threadIdx.x] = 0;
    part_starts[threadIdx.x] = 0;
  }
}

}  // namespace

long long partition_tiles(long long n) { return (n + PTILE - 1) / PTILE; }

size_t partition_scratch_bytes(long long n, int P) {
  const long long t = partition_tiles(n);
  return (static_cast<size_t>(t > 0 ? t : 1) * P * 8 + 255) / 256 * 256;
}

size_t partition_output_rows(long long n, int P, int align_rows) {
  return static_cast<size_t>(n) + static_cast<size_t>(P) * (align_rows > 1 ? align_rows - 1 : 0);
}

cudaError_t partition_launch(const PartitionArgs& a, unsigned long long* scratch, int64_t* part_counts,
                             int64_t* part_starts, cudaStream_t s, uint64_t* launches) {
  const long long ntiles = partition_tiles(a.n);
  if (ntiles == 0) {
    part_empty_kernel<<<1, 32, 0, s>>>(part_counts, part_starts, a.P);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) (*launches)++;
    return e;
  }
  const bool f32 = a.cols.dtype == TBGB_F32;
  cudaError_t e;
  if (a.range) e = f32 ? launch_all<true, true>(a, ntiles, scratch, part_counts, part_starts, s)
                       : launch_all<true, false>(a, ntiles, scratch, part_counts, part_starts, s);
  else e = f32 ? launch_all<false, true>(a, ntiles, scratch, part_counts, part_starts, s)
               : launch_all<false, false>(a, ntiles, scratch, part_counts, part_starts, s);
  if (e == cudaSuccess) *launches += 3;
  return e;
}

}  // namespace tbgb
