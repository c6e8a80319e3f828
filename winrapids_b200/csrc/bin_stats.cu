// bin_stats.cu -- statistics of sorted contiguous bins: per bin count, sum, sum of squares,
// min, max, first and last value, for one or several columns in one launch.
//
// Restates fused_bin_stats / fused_bin_stats_multi (src/winrapids/kernels/bin_stats.cu:25-151):
// bin b is rows [boundaries[b], boundaries[b + 1]); count = hi - lo; sum and sum_sq are plain
// f64 sums (NaN and infinities propagate); min and max start from the bin's first value and
// take strict `<` / `>` winners in row order (so a NaN first value is the result, a later NaN
// never wins, and among equal values the first row's bits -- +0 versus -0 -- are kept);
// first = data[lo], last = data[hi - 1]; an empty bin has count 0 and NaN elsewhere.  The
// derived mean, variance and std follow the reference's Python wrapper
// (archive/fintek-contributions/src/fused_bin_stats.py:121-127): mean = sum / count,
// variance = max(sum_sq / count - mean^2, 0) for count > 1, std = sqrt(variance).
//
// The reference runs one thread per bin over its rows, which leaves lanes idle on uneven bins
// and serialises a large bin on one thread.  Here the rows are cut into fixed chunks of 16384;
// warps take chunks from an atomic counter (so they finish together) at full occupancy (32
// registers): the warp finds the chunk's first bin with a 32-way search of the boundaries, then
// walks the bins that overlap the chunk.  Runs
// of small bins (<= 16 rows, inside the chunk) are taken one bin per lane; pairs of medium bins
// (<= 2048 rows, inside the chunk) one bin per half-warp; any other bin by the whole warp --
// always with coalesced loads and a butterfly reduction over the lanes that share a bin.
// (Measured on 1e9 ticks in bins of 1..831 rows: one bin per warp 2.79 ms, per quarter-warp 2.14,
// per eighth 2.28, per half-warp 2.06, with chunks handed out dynamically 1.85, and at 8 blocks
// per SM 1.70; the reference's one thread per bin 2.06.)  A bin wholly inside the chunk is written at once; a bin that
// crosses a chunk edge leaves a partial state per chunk (its first chunk's in slot 1, the
// others' in slot 0), and a second kernel merges them (one warp per bin, the extrema's
// first-row rule kept through row offsets).  Sums therefore differ from the serial order in
// the last bits; counts, extrema, first and last are exact.  Every row access is bounded by
// the chunk, so boundaries that are not non-decreasing within [0, n_ticks] cannot fault: a
// per-bin pre-pass flags them (KERR_BOUNDARIES) and writes the empty and invalid bins.
#include <climits>
#include <cstdint>

#include "bin_stats.cuh"
#include "common.cuh"
#include "errbits.hpp"

namespace tbgb {

namespace {

constexpr int BNT = 256;          // threads per block (8 warps)
constexpr int BWARPS = BNT / 32;
constexpr long long BCH = 16384;  // rows per warp chunk
constexpr long long MED = 2048;   // bins of at most this many rows go two at a time, sixteen lanes each
constexpr long long SMALL = 16;   // bins of at most this many rows go one per lane

struct BinPart {
  double sum, sq, mn, mx;
  unsigned int mno, mxo;  // row offsets (from the bin's first row) of the extrema
  long long bin;          // -1: slot unused
};

struct BinAcc {
  double sum, sq, mn, mx;
  unsigned int mno, mxo;

  __device__ __forceinline__ void init() {
    sum = 0.0;
    sq = 0.0;
    mn = pos_inf();
    mx = neg_inf();
    mno = UINT_MAX;
    mxo = UINT_MAX;
  }
  __device__ __forceinline__ void add(double v, unsigned int off) {
    sum += v;
    sq = fma(v, v, sq);
    if (v < mn) { mn = v; mno = off; }
    if (v > mx) { mx = v; mxo = off; }
  }
  __device__ __forceinline__ void merge(double s, double q, double m0, unsigned o0, double m1, unsigned o1) {
    sum += s;
    sq += q;
    if (m0 < mn || (m0 == mn && o0 < mno)) { mn = m0; mno = o0; }
    if (m1 > mx || (m1 == mx && o1 < mxo)) { mx = m1; mxo = o1; }
  }
  // over aligned groups of `width` lanes (width a power of two <= 32)
  __device__ __forceinline__ void group_reduce(int width) {
    for (int o = width >> 1; o > 0; o >>= 1) {
      const double s = __shfl_xor_sync(0xffffffffu, sum, o);
      const double q = __shfl_xor_sync(0xffffffffu, sq, o);
      const double m0 = __shfl_xor_sync(0xffffffffu, mn, o);
      const double m1 = __shfl_xor_sync(0xffffffffu, mx, o);
      const unsigned o0 = __shfl_xor_sync(0xffffffffu, mno, o);
      const unsigned o1 = __shfl_xor_sync(0xffffffffu, mxo, o);
      merge(s, q, m0, o0, m1, o1);
    }
  }
  __device__ __forceinline__ void warp_reduce() {
    for (int o = 16; o > 0; o >>= 1) {
      const double s = __shfl_xor_sync(0xffffffffu, sum, o);
      const double q = __shfl_xor_sync(0xffffffffu, sq, o);
      const double m0 = __shfl_xor_sync(0xffffffffu, mn, o);
      const double m1 = __shfl_xor_sync(0xffffffffu, mx, o);
      const unsigned o0 = __shfl_xor_sync(0xffffffffu, mno, o);
      const unsigned o1 = __shfl_xor_sync(0xffffffffu, mxo, o);
      merge(s, q, m0, o0, m1, o1);
    }
  }
};

struct BinArgs {
  const double* data;
  long long n;
  int ncol;
  const long long* B;
  long long nb;
  tbgb_bin_stats out;
  BinPart* part;  // [n_chunks][2][ncol]
  long long n_chunks;
  unsigned long long* next_chunk;  // per column: chunks handed out so far (zeroed before the launch)
  uint32_t* err;
};

__device__ __forceinline__ void write_empty(const BinArgs& a, long long b, int col) {
  const long long i = static_cast<long long>(col) * a.nb + b;
  const double nan = qnan();
  if (col == 0 && a.out.count) a.out.count[b] = 0;
  if (a.out.sum) a.out.sum[i] = nan;
  if (a.out.sum_sq) a.out.sum_sq[i] = nan;
  if (a.out.min) a.out.min[i] = nan;
  if (a.out.max) a.out.max[i] = nan;
  if (a.out.first) a.out.first[i] = nan;
  if (a.out.last) a.out.last[i] = nan;
  if (a.out.mean) a.out.mean[i] = nan;
  if (a.out.variance) a.out.variance[i] = nan;
  if (a.out.std) a.out.std[i] = nan;
}

// Outputs of bin b (rows [lo, hi), 0 <= lo < hi <= n) of column `col` from its reduced state.
__device__ __forceinline__ void write_bin(const BinArgs& a, const double* x, long long b, long long lo, long long hi,
                                          int col, const BinAcc& acc) {
  const long long i = static_cast<long long>(col) * a.nb + b;
  const long long count = hi - lo;
  const double first = x[lo], last = x[hi - 1];
  if (col == 0 && a.out.count) a.out.count[b] = static_cast<int32_t>(count);
  if (a.out.sum) a.out.sum[i] = acc.sum;
  if (a.out.sum_sq) a.out.sum_sq[i] = acc.sq;
  // the scans start from the first value: a NaN first value is the result
  if (a.out.min) a.out.min[i] = is_nan(first) ? first : acc.mn;
  if (a.out.max) a.out.max[i] = is_nan(first) ? first : acc.mx;
  if (a.out.first) a.out.first[i] = first;
  if (a.out.last) a.out.last[i] = last;
  if (a.out.mean || a.out.variance || a.out.std) {
    const double c = static_cast<double>(count);
    const double mean = acc.sum / c;
    double var = qnan();
    if (count > 1) {
      var = acc.sq / c - mean * mean;
      if (var < 0.0) var = 0.0;
    }
    if (a.out.mean) a.out.mean[i] = mean;
    if (a.out.variance) a.out.variance[i] = var;
    if (a.out.std) a.out.std[i] = sqrt(var);
  }
}

// Validates every bin and writes the empty (and invalid) ones.
__global__ void __launch_bounds__(BNT) bin_prepass_kernel(BinArgs a) {
  const long long stride = static_cast<long long>(gridDim.x) * BNT;
  for (long long b = static_cast<long long>(blockIdx.x) * BNT + threadIdx.x; b < a.nb; b += stride) {
    const long long lo = a.B[b], hi = a.B[b + 1];
    const bool bad = lo < 0 || hi < lo || hi > a.n || hi - lo > INT32_MAX;
    if (bad) atomicOr(a.err, KERR_BOUNDARIES);
    if (bad || lo == hi)
      for (int c = 0; c < a.ncol; ++c) write_empty(a, b, c);
  }
}

// Smallest b in [0, nb) with B[b + 1] > row (nb when none), by 32-way steps of the warp.
__device__ __forceinline__ long long first_bin_after(const long long* B, long long nb, long long row, int lane) {
  long long lo = 0, hi = nb;  // the answer is in [lo, hi]; hi stands for "none below"
  while (hi - lo > 32) {
    const long long stride = (hi - lo + 31) / 32;
    long long p = lo + (lane + 1) * stride - 1;
    if (p > hi - 1) p = hi - 1;
    const unsigned bal = __ballot_sync(0xffffffffu, B[p + 1] > row);
    if (bal == 0) {
      lo = lo + 32 * stride;
      if (lo > hi) lo = hi;
    } else {
      const int j = __ffs(bal) - 1;
      const long long pj = __shfl_sync(0xffffffffu, p, j);
      const long long pprev = j > 0 ? __shfl_sync(0xffffffffu, p, j - 1) : lo - 1;
      lo = pprev + 1;
      hi = pj;
    }
  }
  const long long p = lo + lane;
  const unsigned bal = __ballot_sync(0xffffffffu, p < hi && B[p + 1] > row);
  return bal ? lo + (__ffs(bal) - 1) : hi;
}

__global__ void __launch_bounds__(BNT, 8) bin_chunk_kernel(BinArgs a) {
  const int lane = threadIdx.x & 31;
  const int col = blockIdx.y;
  const double* x = a.data + static_cast<long long>(col) * a.n;
  for (;;) {
    unsigned long long cc = 0;
    if (lane == 0) cc = atomicAdd(a.next_chunk + col, 1ull);
    const long long c = static_cast<long long>(__shfl_sync(0xffffffffu, cc, 0));
    if (c >= a.n_chunks) break;
    const long long c0 = c * BCH;
    const long long c1 = c0 + BCH < a.n ? c0 + BCH : a.n;
    BinPart* slots = a.part + (c * 2) * a.ncol + col;  // slot s at slots[s * ncol]
    if (lane == 0) {
      slots[0].bin = -1;
      slots[a.ncol].bin = -1;
    }
    long long b = first_bin_after(a.B, a.nb, c0, lane);
    while (b < a.nb) {
      // a run of small bins inside the chunk: one bin per lane
      const long long bi = b + lane;
      long long lo_i = 0, hi_i = 0;
      bool small = false;
      if (bi < a.nb) {
        lo_i = a.B[bi];
        hi_i = a.B[bi + 1];
        small = lo_i >= c0 && hi_i <= c1 && hi_i >= lo_i && hi_i - lo_i <= SMALL;
      }
      const unsigned big = __ballot_sync(0xffffffffu, !small);
      const int run = big ? __ffs(big) - 1 : 32;
      if (run == 0) {
        // two bins inside the chunk of at most MED rows: sixteen lanes each
        const int g = lane >> 4, gl = lane & 15;
        const long long bg = b + g;
        long long lo_g = 0, hi_g = 0;
        bool med = false;
        if (bg < a.nb) {
          lo_g = a.B[bg];
          hi_g = a.B[bg + 1];
          med = lo_g >= c0 && hi_g <= c1 && hi_g >= lo_g && hi_g - lo_g <= MED;
        }
        if (__all_sync(0xffffffffu, med)) {
          BinAcc acc;
          acc.init();
#pragma unroll 4
          for (long long r = lo_g + gl; r < hi_g; r += 16) acc.add(__ldcs(x + r), static_cast<unsigned>(r - lo_g));
          acc.group_reduce(16);
          if (gl == 0 && hi_g > lo_g) write_bin(a, x, bg, lo_g, hi_g, col, acc);
          b += 2;
          continue;
        }
      }
      if (run > 0) {
        if (lane < run && hi_i > lo_i) {
          BinAcc acc;
          acc.init();
          for (long long r = lo_i; r < hi_i; ++r) acc.add(x[r], static_cast<unsigned>(r - lo_i));
          write_bin(a, x, bi, lo_i, hi_i, col, acc);
        }
        b += run;
        continue;
      }
      // bin b: larger, or crossing a chunk edge -- the whole warp
      const long long lo = a.B[b], hi = a.B[b + 1];
      if (lo >= c1) break;
      const long long s = lo > c0 ? lo : c0;
      const long long e = hi < c1 ? hi : c1;
      if (s < e) {
        BinAcc acc;
        acc.init();
#pragma unroll 4
        for (long long r = s + lane; r < e; r += 32) acc.add(__ldcs(x + r), static_cast<unsigned>(r - lo));
        acc.warp_reduce();
        if (lane == 0) {
          if (lo >= c0 && hi <= c1) {
            write_bin(a, x, b, lo, hi, col, acc);
          } else {
            BinPart& p = slots[(lo < c0 ? 0 : 1) * a.ncol];
            p.sum = acc.sum;
            p.sq = acc.sq;
            p.mn = acc.mn;
            p.mx = acc.mx;
            p.mno = acc.mno;
            p.mxo = acc.mxo;
            p.bin = b;
          }
        }
      }
      ++b;
    }
  }
}

// One warp per chunk: a bin that starts in chunk c and continues past it is finished here from
// its partial states (slot 1 of chunk c, slot 0 of the chunks it runs on through).
__global__ void __launch_bounds__(BNT) bin_combine_kernel(BinArgs a) {
  const int lane = threadIdx.x & 31;
  const int col = blockIdx.y;
  const double* x = a.data + static_cast<long long>(col) * a.n;
  const long long nw = static_cast<long long>(gridDim.x) * BWARPS;
  for (long long c = static_cast<long long>(blockIdx.x) * BWARPS + (threadIdx.x >> 5); c < a.n_chunks; c += nw) {
    const BinPart& head = a.part[(c * 2 + 1) * a.ncol + col];
    const long long b = head.bin;
    if (b < 0) continue;
    const long long lo = a.B[b], hi = a.B[b + 1];
    if (lo < 0 || hi <= lo || hi > a.n) continue;  // invalid boundaries (flagged by the pre-pass)
    const long long c_last = (hi - 1) / BCH;
    BinAcc acc;
    acc.init();
    if (lane == 0) acc.merge(head.sum, head.sq, head.mn, head.mno, head.mx, head.mxo);
    for (long long j = c + 1 + lane; j <= c_last && j < a.n_chunks; j += 32) {
      const BinPart& p = a.part[(j * 2) * a.ncol + col];
      if (p.bin == b) acc.merge(p.sum, p.sq, p.mn, p.mno, p.mx, p.mxo);
    }
    acc.warp_reduce();
    if (lane == 0) write_bin(a, x, b, lo, hi, col, acc);
  }
}

int chunk_grid(long long n_chunks, int num_sms) {
  static int per_sm = 0;
  if (per_sm == 0) {
    int x = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&x, bin_chunk_kernel, BNT, 0) != cudaSuccess || x < 1) x = 1;
    per_sm = x;
  }
  long long blocks = (n_chunks + BWARPS - 1) / BWARPS;
  const long long cap = static_cast<long long>(num_sms > 0 ? num_sms : 148) * per_sm;
  if (blocks > cap) blocks = cap;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

}  // namespace

size_t bin_stats_scratch_bytes(long long n_ticks, int n_columns) {
  const long long n_chunks = (n_ticks + BCH - 1) / BCH;
  return static_cast<size_t>(n_chunks > 0 ? n_chunks : 1) * 2 * static_cast<size_t>(n_columns) * sizeof(BinPart) +
         static_cast<size_t>(n_columns) * 8;
}

cudaError_t bin_stats_launch(const double* data, long long n_ticks, int n_columns, const int64_t* boundaries,
                             long long n_bins, const tbgb_bin_stats* out, void* scratch, uint32_t* err,
                             int num_sms, cudaStream_t s, uint64_t* launches) {
  if (n_bins <= 0) return cudaSuccess;
  BinArgs a;
  a.data = data;
  a.n = n_ticks;
  a.ncol = n_columns;
  a.B = reinterpret_cast<const long long*>(boundaries);
  a.nb = n_bins;
  a.out = *out;
  a.part = static_cast<BinPart*>(scratch);
  a.n_chunks = (n_ticks + BCH - 1) / BCH;
  a.next_chunk = reinterpret_cast<unsigned long long*>(static_cast<char*>(scratch) +
                 static_cast<size_t>(a.n_chunks > 0 ? a.n_chunks : 1) * 2 * n_columns * sizeof(BinPart));
  a.err = err;
  long long pb = (n_bins + BNT - 1) / BNT;
  if (pb > 65536) pb = 65536;
  bin_prepass_kernel<<<static_cast<unsigned>(pb), BNT, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  (*launches)++;
  if (a.n_chunks == 0) return cudaSuccess;
  e = cudaMemsetAsync(a.next_chunk, 0, static_cast<size_t>(n_columns) * 8, s);
  if (e != cudaSuccess) return e;
  const dim3 grid(chunk_grid(a.n_chunks, num_sms), static_cast<unsigned>(n_columns));
  bin_chunk_kernel<<<grid, BNT, 0, s>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  bin_combine_kernel<<<grid, BNT, 0, s>>>(a);
  e = cudaGetLastError();
  if (e == cudaSuccess) *launches += 2;
  return e;
}

}  // namespace tbgb
