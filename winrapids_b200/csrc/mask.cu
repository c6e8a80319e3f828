// mask.cu -- mask-not-filter plumbing: row masks, their algebra, per-tile column
// statistics and tile-skip masks.
//
// A row mask holds row i in bit (i % 64) of word i / 64, the bits of rows >= n of the
// last word 0 (FilterJit::filter_mask, crates/tambear/src/filter_jit.rs:71-121, kernel
// layout :196-243).  The algebra follows MaskOp (filter_jit.rs:262-440, kernels :459-537)
// and the host functions mask_and / mask_or / mask_xor / mask_not / mask_popcount
// (:130-181): AND / OR / XOR word by word, NOT with the last word's trailing bits
// cleared, popcount over rows [0, n_rows).
//
// Tile statistics restate TileColumnStats::from_slice (crates/tambear/src/format.rs:60-107):
// per tile min and max by strict `<` / `>` scans from +inf / -inf (NaN never wins, so an
// all-NaN tile keeps +inf / -inf; among equal values the first row's bits are kept,
// which decides +0 versus -0), a Kahan-compensated sum, count = n_valid = rows of the
// tile.  The sum is computed here as a compensated parallel sum (within a few ulps of
// the serial Kahan result for finite values); non-finite values give what the serial
// Kahan loop gives: NaN if any value is NaN or if a value follows an infinity in the
// tile, the infinity itself when a single infinity is the tile's last value.
// Tile-skip masks restate can_skip_gt / _gte / _lt / _lte (:111-136) and
// tile_skip_mask_gt / _lt (:182-189).  The reference only counts skippable tiles; here
// mask_skip_tiles clears a skipped tile's rows in a row mask, and the table and
// partition kernels test a row's mask bit before they load its columns, so the rows of
// skipped tiles are never read.
#include <climits>
#include <cstdint>

#include "common.cuh"
#include "mask.cuh"
#include "rowops.cuh"

namespace tbgb {

namespace {

constexpr int MNT = 256;      // threads per block of the word-wise kernels
constexpr int TS_NT = 512;    // threads per block of the tile-statistics kernel
constexpr int MUNROLL = 4;    // words in flight per thread

int word_grid(long long items, int num_sms) {
  long long blocks = (items + static_cast<long long>(MNT) * MUNROLL - 1) / (static_cast<long long>(MNT) * MUNROLL);
  const long long cap = static_cast<long long>(num_sms > 0 ? num_sms : 148) * 8;
  if (blocks > cap) blocks = cap;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

template <int OP>
__device__ __forceinline__ unsigned long long apply_op(unsigned long long x, unsigned long long y) {
  if constexpr (OP == MASK_AND) return x & y;
  else if constexpr (OP == MASK_OR) return x | y;
  else if constexpr (OP == MASK_XOR) return x ^ y;
  else return ~x;
}

// In place (out == a or out == b) is allowed: each word is read and written by one thread,
// its loads before its store.
template <int OP>
__global__ void __launch_bounds__(MNT) mask_op_kernel(const unsigned long long* a, const unsigned long long* b,
                                                      unsigned long long* out, long long n_words,
                                                      unsigned long long last_keep) {
  const long long stride = static_cast<long long>(gridDim.x) * MNT;
  for (long long i0 = static_cast<long long>(blockIdx.x) * MNT + threadIdx.x; i0 < n_words;
       i0 += stride * MUNROLL) {
    unsigned long long x[MUNROLL], y[MUNROLL];
#pragma unroll
    for (int u = 0; u < MUNROLL; ++u) {
      const long long i = i0 + u * stride;
      x[u] = 0;
      y[u] = 0;
      if (i < n_words) {
        x[u] = __ldcs(a + i);
        if constexpr (OP != MASK_NOT) y[u] = __ldcs(b + i);
      }
    }
#pragma unroll
    for (int u = 0; u < MUNROLL; ++u) {
      const long long i = i0 + u * stride;
      if (i < n_words) {
        unsigned long long r = apply_op<OP>(x[u], y[u]);
        if (OP == MASK_NOT && i == n_words - 1) r &= last_keep;
        __stcs(out + i, r);
      }
    }
  }
}

__global__ void __launch_bounds__(MNT) mask_popcount_kernel(const unsigned long long* mask, long long n_words,
                                                            unsigned long long last_keep,
                                                            unsigned long long* count) {
  const long long stride = static_cast<long long>(gridDim.x) * MNT;
  unsigned long long c = 0;
  for (long long i = static_cast<long long>(blockIdx.x) * MNT + threadIdx.x; i < n_words; i += stride) {
    unsigned long long w = __ldcs(mask + i);
    if (i == n_words - 1) w &= last_keep;
    c += static_cast<unsigned long long>(__popcll(w));
  }
  for (int o = 16; o > 0; o >>= 1) c += __shfl_down_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0 && c) atomicAdd(count, c);
}

// One warp builds 32 words (2048 rows) per step: 64 ballots over 32 consecutive rows each
// (coalesced loads), lane j keeping word j.  With an input mask, lane j first loads input
// word j; a row whose input bit is 0 is not read (a warp whose 32 rows are all out issues
// no load).  In place (mask == in_mask) is safe: the words are read before any is written.
template <bool F32>
__global__ void __launch_bounds__(MNT) filter_mask_kernel(const void* col, long long n, int pred, double threshold,
                                                          const unsigned long long* in_mask,
                                                          unsigned long long* mask, long long n_words) {
  const int lane = threadIdx.x & 31;
  const long long warp = (static_cast<long long>(blockIdx.x) * MNT + threadIdx.x) >> 5;
  const long long nwarps = static_cast<long long>(gridDim.x) * (MNT / 32);
  for (long long w0 = warp * 32; w0 < n_words; w0 += nwarps * 32) {
    const long long row0 = w0 * 64;
    const unsigned long long inw = !in_mask ? ~0ull : (w0 + lane < n_words ? in_mask[w0 + lane] : 0ull);
    if (__all_sync(0xffffffffu, inw == 0ull)) {  // 2048 rows none of which is selected
      if (w0 + lane < n_words) mask[w0 + lane] = 0ull;
      continue;
    }
    unsigned long long word = 0;
#pragma unroll 16
    for (int k = 0; k < 64; ++k) {
      const long long row = row0 + static_cast<long long>(k) * 32 + lane;
      // this row's input bit: word k/2 (held by lane k/2), bit (k & 1) * 32 + lane
      const unsigned long long src = __shfl_sync(0xffffffffu, inw, k >> 1);
      bool p = false;
      if (row < n && ((src >> ((k & 1) * 32 + lane)) & 1ull)) p = eval_pred(pred, load_val<F32>(col, row), threshold);
      const unsigned bal = __ballot_sync(0xffffffffu, p);
      if (lane == (k >> 1)) word |= static_cast<unsigned long long>(bal) << ((k & 1) * 32);
    }
    __syncwarp();
    if (w0 + lane < n_words) mask[w0 + lane] = word;
  }
}

// Error-free sum of two doubles (Knuth's TwoSum).
__device__ __forceinline__ void two_sum(double a, double b, double* s, double* e) {
  const double x = __dadd_rn(a, b);
  const double bv = __dsub_rn(x, a);
  const double av = __dsub_rn(x, bv);
  *s = x;
  *e = __dadd_rn(__dsub_rn(a, av), __dsub_rn(b, bv));
}

struct TileAcc {
  double mn, mx;             // strict-scan extrema
  long long mnr, mxr;        // first row holding them (LLONG_MAX: the initial +-inf)
  double s, c;               // compensated sum of the finite values
  long long first_inf;       // first row holding an infinity (LLONG_MAX: none)
  double inf_val;            // that infinity
  int nan;                   // a NaN was seen
  int n_inf;                 // infinities seen
};

__device__ __forceinline__ void acc_merge(TileAcc& a, const TileAcc& b) {
  if (b.mn < a.mn || (b.mn == a.mn && b.mnr < a.mnr)) { a.mn = b.mn; a.mnr = b.mnr; }
  if (b.mx > a.mx || (b.mx == a.mx && b.mxr < a.mxr)) { a.mx = b.mx; a.mxr = b.mxr; }
  double s, e;
  two_sum(a.s, b.s, &s, &e);
  a.s = s;
  a.c = __dadd_rn(__dadd_rn(a.c, b.c), e);
  if (b.first_inf < a.first_inf) { a.first_inf = b.first_inf; a.inf_val = b.inf_val; }
  a.nan |= b.nan;
  a.n_inf += b.n_inf;
}

__device__ __forceinline__ TileAcc acc_shfl_down(const TileAcc& a, int o) {
  TileAcc b;
  b.mn = __shfl_down_sync(0xffffffffu, a.mn, o);
  b.mx = __shfl_down_sync(0xffffffffu, a.mx, o);
  b.mnr = __shfl_down_sync(0xffffffffu, a.mnr, o);
  b.mxr = __shfl_down_sync(0xffffffffu, a.mxr, o);
  b.s = __shfl_down_sync(0xffffffffu, a.s, o);
  b.c = __shfl_down_sync(0xffffffffu, a.c, o);
  b.first_inf = __shfl_down_sync(0xffffffffu, a.first_inf, o);
  b.inf_val = __shfl_down_sync(0xffffffffu, a.inf_val, o);
  b.nan = __shfl_down_sync(0xffffffffu, a.nan, o);
  b.n_inf = __shfl_down_sync(0xffffffffu, a.n_inf, o);
  return b;
}

// One block per tile (grid-stride over tiles); blockDim.x is a multiple of 32, <= TS_NT.
template <bool F32>
__global__ void __launch_bounds__(TS_NT) tile_stats_kernel(const void* col, long long n, long long tile_rows,
                                                           long long n_tiles, tbgb_tile_stats* out) {
  __shared__ TileAcc part[TS_NT / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x) {
    const long long lo = t * tile_rows;
    const long long hi = lo + tile_rows < n ? lo + tile_rows : n;
    TileAcc a;
    a.mn = pos_inf(); a.mx = neg_inf();
    a.mnr = LLONG_MAX; a.mxr = LLONG_MAX;
    a.s = 0.0; a.c = 0.0;
    a.first_inf = LLONG_MAX; a.inf_val = 0.0;
    a.nan = 0; a.n_inf = 0;
    for (long long r = lo + threadIdx.x; r < hi; r += blockDim.x) {
      const double v = load_val<F32>(col, r);
      if (v < a.mn) { a.mn = v; a.mnr = r; }
      if (v > a.mx) { a.mx = v; a.mxr = r; }
      if (is_finite(v)) {
        double s, e;
        two_sum(a.s, v, &s, &e);
        a.s = s;
        a.c = __dadd_rn(a.c, e);
      } else if (is_nan(v)) {
        a.nan = 1;
      } else {
        if (r < a.first_inf) { a.first_inf = r; a.inf_val = v; }
        a.n_inf += 1;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const TileAcc b = acc_shfl_down(a, o);
      if (lane + o < 32) acc_merge(a, b);
    }
    if (lane == 0) part[warp] = a;
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < nwarps; ++w) acc_merge(a, part[w]);
      double sum;
      if (a.nan) sum = qnan();
      else if (a.n_inf == 0) sum = __dadd_rn(a.s, a.c);
      else if (a.n_inf == 1 && a.first_inf == hi - 1) sum = a.inf_val;
      else sum = qnan();
      tbgb_tile_stats st;
      st.min = a.mn;
      st.max = a.mx;
      st.sum = sum;
      st.count = static_cast<uint32_t>(hi - lo);
      st.n_valid = static_cast<uint32_t>(hi - lo);
      st.reserved = 0;
      out[t] = st;
    }
    __syncthreads();  // part[] is rewritten by the next tile
  }
}

__global__ void __launch_bounds__(MNT) tile_skip_kernel(const tbgb_tile_stats* stats, long long n_tiles, int pred,
                                                        double t, uint8_t* skip) {
  const long long stride = static_cast<long long>(gridDim.x) * MNT;
  for (long long i = static_cast<long long>(blockIdx.x) * MNT + threadIdx.x; i < n_tiles; i += stride) {
    const double mn = stats[i].min, mx = stats[i].max;
    bool s;
    switch (pred) {
      case TBGB_PRED_GT: s = mx <= t; break;
      case TBGB_PRED_GE: s = mx < t; break;
      case TBGB_PRED_LT: s = mn >= t; break;
      default: s = mn > t; break;  // TBGB_PRED_LE (the host admits no other predicate)
    }
    skip[i] = s ? 1 : 0;
  }
}

__global__ void __launch_bounds__(MNT) mask_skip_tiles_kernel(const unsigned long long* in, const uint8_t* skip,
                                                              long long tile_rows, long long n_rows,
                                                              long long n_words, unsigned long long* out) {
  const long long stride = static_cast<long long>(gridDim.x) * MNT;
  const int rem = static_cast<int>(n_rows & 63);
  for (long long w = static_cast<long long>(blockIdx.x) * MNT + threadIdx.x; w < n_words; w += stride) {
    const long long r0 = w * 64;
    const long long rl = r0 + 63 < n_rows ? r0 + 63 : n_rows - 1;
    const long long t0 = r0 / tile_rows, t1 = rl / tile_rows;
    unsigned long long keep;
    if (t0 == t1) {
      keep = skip[t0] ? 0ull : ~0ull;
    } else {
      keep = 0;
      for (int b = 0; r0 + b <= rl; ++b)
        if (!skip[(r0 + b) / tile_rows]) keep |= 1ull << b;
    }
    unsigned long long v = in ? (in[w] & keep) : keep;
    if (rem && w == n_words - 1) v &= (1ull << rem) - 1ull;
    out[w] = v;
  }
}

unsigned long long last_word_keep(long long n_rows) {
  const int rem = static_cast<int>(n_rows & 63);
  return rem ? (1ull << rem) - 1ull : ~0ull;
}

}  // namespace

cudaError_t mask_op_launch(int op, const uint64_t* a, const uint64_t* b, uint64_t* out, long long n_words,
                           long long n_rows, int num_sms, cudaStream_t s, uint64_t* launches) {
  if (n_words <= 0) return cudaSuccess;
  const auto* A = reinterpret_cast<const unsigned long long*>(a);
  const auto* B = reinterpret_cast<const unsigned long long*>(b);
  auto* O = reinterpret_cast<unsigned long long*>(out);
  const int g = word_grid(n_words, num_sms);
  const unsigned long long keep = last_word_keep(n_rows);
  switch (op) {
    case MASK_AND: mask_op_kernel<MASK_AND><<<g, MNT, 0, s>>>(A, B, O, n_words, keep); break;
    case MASK_OR: mask_op_kernel<MASK_OR><<<g, MNT, 0, s>>>(A, B, O, n_words, keep); break;
    case MASK_XOR: mask_op_kernel<MASK_XOR><<<g, MNT, 0, s>>>(A, B, O, n_words, keep); break;
    default: mask_op_kernel<MASK_NOT><<<g, MNT, 0, s>>>(A, B, O, n_words, keep); break;
  }
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

cudaError_t mask_popcount_launch(const uint64_t* mask, long long n_rows, unsigned long long* d_count, int num_sms,
                                 cudaStream_t s, uint64_t* launches) {
  cudaError_t e = cudaMemsetAsync(d_count, 0, sizeof(unsigned long long), s);
  if (e != cudaSuccess || n_rows <= 0) return e;
  const long long n_words = (n_rows + 63) / 64;
  mask_popcount_kernel<<<word_grid(n_words, num_sms), MNT, 0, s>>>(
      reinterpret_cast<const unsigned long long*>(mask), n_words, last_word_keep(n_rows), d_count);
  e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

cudaError_t filter_mask_launch(const void* col, int dtype, long long n, int pred, double threshold,
                               const uint64_t* in_mask, uint64_t* mask, int num_sms, cudaStream_t s,
                               uint64_t* launches) {
  if (n <= 0) return cudaSuccess;
  const long long n_words = (n + 63) / 64;
  const long long chunks = (n_words + 31) / 32;  // 32 words per warp step
  long long blocks = (chunks + (MNT / 32) - 1) / (MNT / 32);
  const long long cap = static_cast<long long>(num_sms > 0 ? num_sms : 148) * 8;
  if (blocks > cap) blocks = cap;
  auto* M = reinterpret_cast<unsigned long long*>(mask);
  const auto* I = reinterpret_cast<const unsigned long long*>(in_mask);
  if (dtype == TBGB_F32)
    filter_mask_kernel<true><<<static_cast<int>(blocks), MNT, 0, s>>>(col, n, pred, threshold, I, M, n_words);
  else
    filter_mask_kernel<false><<<static_cast<int>(blocks), MNT, 0, s>>>(col, n, pred, threshold, I, M, n_words);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

cudaError_t tile_stats_launch(const void* col, int dtype, long long n, long long tile_rows, tbgb_tile_stats* out,
                              int num_sms, cudaStream_t s, uint64_t* launches) {
  if (n <= 0) return cudaSuccess;
  const long long n_tiles = (n + tile_rows - 1) / tile_rows;
  const int nt = tile_rows >= TS_NT ? TS_NT : static_cast<int>((tile_rows + 31) / 32 * 32);
  long long blocks = n_tiles;
  const long long cap = static_cast<long long>(num_sms > 0 ? num_sms : 148) * (2048 / nt);
  if (blocks > cap) blocks = cap;
  if (dtype == TBGB_F32)
    tile_stats_kernel<true><<<static_cast<int>(blocks), nt, 0, s>>>(col, n, tile_rows, n_tiles, out);
  else
    tile_stats_kernel<false><<<static_cast<int>(blocks), nt, 0, s>>>(col, n, tile_rows, n_tiles, out);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

cudaError_t tile_skip_launch(const tbgb_tile_stats* stats, long long n_tiles, int pred, double threshold,
                             uint8_t* skip, cudaStream_t s, uint64_t* launches) {
  if (n_tiles <= 0) return cudaSuccess;
  long long blocks = (n_tiles + MNT - 1) / MNT;
  if (blocks > 65536) blocks = 65536;
  tile_skip_kernel<<<static_cast<int>(blocks), MNT, 0, s>>>(stats, n_tiles, pred, threshold, skip);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

cudaError_t mask_skip_tiles_launch(const uint64_t* in, const uint8_t* skip, long long tile_rows, long long n_rows,
                                   uint64_t* out, int num_sms, cudaStream_t s, uint64_t* launches) {
  if (n_rows <= 0) return cudaSuccess;
  const long long n_words = (n_rows + 63) / 64;
  long long blocks = (n_words + MNT - 1) / MNT;
  const long long cap = static_cast<long long>(num_sms > 0 ? num_sms : 148) * 8;
  if (blocks > cap) blocks = cap;
  mask_skip_tiles_kernel<<<static_cast<int>(blocks), MNT, 0, s>>>(
      reinterpret_cast<const unsigned long long*>(in), skip, tile_rows, n_rows, n_words,
      reinterpret_cast<unsigned long long*>(out));
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

}  // namespace tbgb
