// partition.cu -- routes rows to the GPU that owns their key (sharded high-cardinality
// groupby).  No counterpart in the reference, which runs on one GPU.
//
// owner(key) = (fmix64(key) >> 32) % n_parts: the high hash bits, independent of the
// low bits the owner's table slots use.  Rows that pass the mask and the predicate
// are written as (key, v = expr(a, b, c) in f64) grouped by owner, each owner's rows
// in row order (a stable partition), so that after an all-to-all that concatenates
// the senders in rank order every key's rows keep their global order -- which keeps
// the +-0 tie rule of the extrema exact on the owner.
//
// Three launches over fixed tiles of 65,536 rows: per-tile owner counts, one block
// scanning the [owner][tile] count matrix into write offsets, and the stable scatter
// (per 1024-row step: one ballot per owner inside each warp, a prefix over the
// block's warps, rows written at running offset + prefix + rank in warp).
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

// Owner of row `row`, or -1 when the row is filtered out; `v` receives its value.
template <bool F32>
__device__ __forceinline__ int route_row(const PartitionArgs& a, long long row, unsigned long long* key, double* v) {
  if (row >= a.n) return -1;
  if (a.mask && !((__ldg(a.mask + (row >> 6)) >> (row & 63)) & 1ull)) return -1;
  const double av = load_val<F32>(a.cols.a, row);
  if (!eval_pred(a.cols.pred, av, a.cols.threshold)) return -1;
  const int expr = a.cols.expr;
  const double bv = expr != TBGB_EXPR_A ? load_val<F32>(a.cols.b, row) : 0.0;
  const double cv = expr == TBGB_EXPR_MUL_ADD ? load_val<F32>(a.cols.c, row) : 0.0;
  *v = eval_expr(expr, av, bv, cv);
  *key = static_cast<unsigned long long>(__ldcs(a.keys + row));
  return owner_of(*key, a.P);
}

template <bool F32>
__global__ void __launch_bounds__(PNT) part_count_kernel(PartitionArgs a, long long ntiles,
                                                         unsigned long long* tile_counts) {
  __shared__ unsigned int cnt[kMaxParts];
  const long long t = blockIdx.x;
  if (threadIdx.x < a.P) cnt[threadIdx.x] = 0;
  __syncthreads();
  const long long base = t * PTILE;
  for (int s = 0; s < PSTEPS; ++s) {
    unsigned long long key;
    double v;
    const int d = route_row<F32>(a, base + static_cast<long long>(s) * PNT + threadIdx.x, &key, &v);
    if (d >= 0) atomicAdd(cnt + d, 1u);
  }
  __syncthreads();
  if (threadIdx.x < a.P) tile_counts[static_cast<long long>(threadIdx.x) * ntiles + t] = cnt[threadIdx.x];
}

// Exclusive scan of the [P][ntiles] count matrix (owner-major) in one block; writes
// offsets in place and the per-owner totals.
__global__ void __launch_bounds__(SCAN_NT) part_scan_kernel(unsigned long long* counts, long long len, int P,
                                                            long long ntiles, int64_t* part_counts) {
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
  // per-owner totals: offset of the owner's first tile to the next owner's (or the end)
  if (threadIdx.x < P) {
    const int p = threadIdx.x;
    const unsigned long long start = counts[static_cast<long long>(p) * ntiles];
    const unsigned long long end = p + 1 < P ? counts[static_cast<long long>(p + 1) * ntiles] : carry;
    part_counts[p] = static_cast<int64_t>(end - start);
  }
}

template <bool F32>
__global__ void __launch_bounds__(PNT) part_scatter_kernel(PartitionArgs a, long long ntiles,
                                                           const unsigned long long* __restrict__ offsets) {
  __shared__ unsigned int wcnt[PNT / 32][kMaxParts];  // per warp, per owner: rows in this step
  __shared__ unsigned long long running[kMaxParts];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long t = blockIdx.x;
  const int P = a.P;
  if (threadIdx.x < P) running[threadIdx.x] = offsets[static_cast<long long>(threadIdx.x) * ntiles + t];
  const unsigned lt = (1u << lane) - 1u;
  const long long base = t * PTILE;
  for (int s = 0; s < PSTEPS; ++s) {
    unsigned long long key = 0;
    double v = 0.0;
    const int d = route_row<F32>(a, base + static_cast<long long>(s) * PNT + threadIdx.x, &key, &v);
    unsigned int rank = 0;
    for (int p = 0; p < P; ++p) {
      const unsigned bal = __ballot_sync(0xffffffffu, d == p);
      if (d == p) rank = __popc(bal & lt);
      if (lane == 0) wcnt[warp][p] = __popc(bal);
    }
    __syncthreads();
    // warp w's offset for owner p: rows of warps < w in this step
    if (d >= 0) {
      unsigned long long off = running[d];
      for (int w = 0; w < warp; ++w) off += wcnt[w][d];
      a.out_keys[off + rank] = static_cast<int64_t>(key);
      a.out_vals[off + rank] = v;
    }
    __syncthreads();
    if (threadIdx.x < P) {
      unsigned long long tot = 0;
      for (int w = 0; w < PNT / 32; ++w) tot += wcnt[w][threadIdx.x];
      running[threadIdx.x] += tot;
    }
    __syncthreads();
  }
}

}  // namespace

long long partition_tiles(long long n) { return (n + PTILE - 1) / PTILE; }

size_t partition_scratch_bytes(long long n, int P) {
  return static_cast<size_t>(partition_tiles(n) > 0 ? partition_tiles(n) : 1) * P * 8;
}

cudaError_t partition_launch(const PartitionArgs& a, unsigned long long* scratch, int64_t* part_counts,
                             cudaStream_t s, uint64_t* launches) {
  const long long ntiles = partition_tiles(a.n);
  if (ntiles == 0) return cudaMemsetAsync(part_counts, 0, static_cast<size_t>(a.P) * 8, s);
  const bool f32 = a.cols.dtype == TBGB_F32;
  if (f32) part_count_kernel<true><<<static_cast<unsigned int>(ntiles), PNT, 0, s>>>(a, ntiles, scratch);
  else part_count_kernel<false><<<static_cast<unsigned int>(ntiles), PNT, 0, s>>>(a, ntiles, scratch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  part_scan_kernel<<<1, SCAN_NT, 0, s>>>(scratch, ntiles * a.P, a.P, ntiles, part_counts);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (f32) part_scatter_kernel<true><<<static_cast<unsigned int>(ntiles), PNT, 0, s>>>(a, ntiles, scratch);
  else part_scatter_kernel<false><<<static_cast<unsigned int>(ntiles), PNT, 0, s>>>(a, ntiles, scratch);
  e = cudaGetLastError();
  if (e == cudaSuccess) *launches += 3;
  return e;
}

}  // namespace tbgb
