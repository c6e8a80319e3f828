// radix.cu -- int64-key groupby (count, sum, mean) by radix partitioning.
//
// A single open-addressing table over hundreds of millions of keys lives far outside L2 and
// the TLB's reach: every row then pays a random DRAM sector and a TLB miss.  Here the rows are
// instead moved twice, in streaming passes, until each bucket's keys fit one CTA's shared
// memory:
//   pass 1  rows -> 512 buckets by the top 9 bits of h = fmix64(key)   (mask, predicate and
//           expression applied here; rows that fail them are dropped)
//   pass 2  each of those -> 512 buckets by the next 9 bits            (262,144 buckets)
//   pass 3  one CTA per bucket: a shared-memory table of 2,048 slots keyed by the low 46 bits of
//           h (the top 18 are the bucket) takes the bucket's rows, then writes its groups.  A
//           slot is the key (claimed by a 64-bit compare-and-swap), a u32 count and the sum: for
//           f32 values an exact 64-bit fixed-point sum in two u32 words (below), for f64 values
//           an f64 sum.  An f32 row costs one probe read and three 32-bit adds.
// fmix64 (MurmurHash3's finaliser) is a bijection, so the rows carry h instead of the key and
// pass 3 recovers each group's key by inverting it.  A row is (h, value): 12 bytes for an f32
// column without an expression, 16 otherwise.
//
// Each pass-1/2 CTA stages a tile of 4,096 rows: per row a shared-memory atomic gives its rank
// among the tile's rows of the same bucket, one global atomic per (tile, bucket) claims a run in
// the bucket's region, the rows are reordered by bucket in shared memory and then written as
// runs (consecutive threads, consecutive addresses).  Buckets have fixed regions with slack
// over an even share (tens of standard deviations for hashed keys); a bucket that still
// overflows -- heavily skewed or adversarial keys -- or a final bucket with more distinct keys
// than its table takes sets the fallback word, the remaining passes stop early, and the caller
// recomputes the result with the global-table strategy gated on that word.
//
// No counterpart in the reference, which groups int64 keys on the host (GroupIndex::build,
// crates/tambear/src/group_index.rs:117-204, i32 codes only); the outputs follow the same
// semantics as the global table: count = non-NaN rows, sum = sum of finite values, mean =
// sum / count (NaN when count is 0), and a key whose rows are all NaN is a group of count 0.
#include <cmath>
#include <cstdint>
#include <type_traits>

#include "common.cuh"
#include "radix.cuh"
#include "rowops.cuh"

namespace tbgb {

namespace {

constexpr int RX_NT = 512;                     // threads per scatter CTA
constexpr int RX_TILE = 4096;                  // rows per scatter tile
constexpr int RX_PER = RX_TILE / RX_NT;        // rows per thread per tile
constexpr int D1_BITS = 9, D2_BITS = 9;        // digits of pass 1 and pass 2
constexpr int BUCKET_BITS = D1_BITS + D2_BITS;  // final buckets: the top 18 bits of h
constexpr int KEY_BITS = 64 - BUCKET_BITS;      // bits of h a table slot keeps (46)
constexpr unsigned long long kKeyMask = (1ull << KEY_BITS) - 1;
constexpr int AGG_NT = 512;                    // threads per aggregation CTA
constexpr int AGG_SLOTS = 2048;                // shared-memory table slots per bucket
constexpr int AGG_MAX_PROBE = 512;             // probes before a row gives up (fallback)
constexpr int AGG_UNROLL = 2;
constexpr unsigned long long kFree = ~0ull;  // a free slot (never a 46-bit key)
static_assert(kRadixBuckets == (1 << BUCKET_BITS), "bucket count");
static_assert(kRadixDigits == (1 << D1_BITS), "first-pass digits");

static_assert(RX_TILE <= 65536, "ranks are packed in 16 bits");

__host__ __device__ constexpr unsigned long long inverse_odd(unsigned long long c) {
  unsigned long long x = c;  // Newton's iteration for the inverse mod 2^64 (3 correct bits to start)
  for (int i = 0; i < 6; ++i) x *= 2ull - c * x;
  return x;
}
static_assert(0xff51afd7ed558ccdull * inverse_odd(0xff51afd7ed558ccdull) == 1ull, "inverse");
static_assert(0xc4ceb9fe1a85ec53ull * inverse_odd(0xc4ceb9fe1a85ec53ull) == 1ull, "inverse");

// fmix64's inverse: each x ^= x >> 33 undoes itself (33 >= 64 / 2), each multiply by an odd
// constant is undone by its inverse mod 2^64.
__device__ __forceinline__ unsigned long long unfmix64(unsigned long long h) {
  constexpr unsigned long long i2 = inverse_odd(0xc4ceb9fe1a85ec53ull);
  constexpr unsigned long long i1 = inverse_odd(0xff51afd7ed558ccdull);
  h ^= h >> 33;
  h *= i2;
  h ^= h >> 33;
  h *= i1;
  h ^= h >> 33;
  return h;
}

constexpr int kMaxSeg = 4096;  // second-pass segments: (sender, digit) pairs of a routed groupby
constexpr int kMaxSenders = kRadixMaxSenders;

struct SenderBases {  // first row of each sender's routed rows (addresses)
  unsigned long long h[kMaxSenders];
  unsigned long long v[kMaxSenders];
};

struct Aux {  // device bookkeeping inside the workspace
  unsigned long long cur1[kRadixDigits];
  unsigned long long cur2[kRadixBuckets];
  unsigned long long route_base[kRadixDigits];  // exact placement of a routing pass
  unsigned long long route_cap[kRadixDigits];
  unsigned long long seg_h[kMaxSeg];            // address of a segment's first hash
  unsigned long long seg_v[kMaxSeg];            // address of its first value
  long long seg_count[kMaxSeg];
  int seg_digit[kMaxSeg];                       // destination digit, relative to the first owned one
  long long seg_tiles[kMaxSeg + 1];
  unsigned long long n_groups;
  uint32_t fallback;
  uint32_t pad[13];
};

struct RxScatter {
  // pass 1: the caller's rows
  const int64_t* keys;
  tbgb_columns cols;
  const uint64_t* mask;
  long long n;
  // pass 2: segments of rows ordered by the previous digit (the first pass's buffer, or routed rows
  // in the senders' buffers), each at its own address
  const unsigned long long* seg_h;
  const unsigned long long* seg_v;
  const long long* seg_count;
  const int* seg_digit;
  const long long* seg_tiles;  // exclusive prefix of tiles per segment, n_seg + 1 entries
  int n_seg;
  int shift;                   // digit = (h >> shift) & 255
  // destination
  unsigned long long* dst_h;
  void* dst_v;
  unsigned long long* cursor;  // rows claimed per destination bucket
  unsigned long long cap;      // rows per destination bucket region (when out_base is NULL)
  const unsigned long long* out_base;  // nullable: first row of each destination bucket
  const unsigned long long* out_cap;   // with out_base: rows of each destination bucket
  uint32_t* fallback;
  int stage;                   // 1: full, 16-byte aligned tiles arrive by TMA bulk copy (local sources)
};

// Plain sources (SRC 0, 2) stage whole tiles into shared memory with a bulk copy issued one tile
// ahead: the copy of a CTA's next tile runs while the current tile is ranked, reordered and
// written, so the row loads leave the tile's critical path.
template <int SRC>
__host__ __device__ constexpr bool scatter_staged() { return SRC != 1; }

// The reordered tile (hashes and values as two arrays), and for staged sources the tile being
// copied in (keys or hashes, values).
template <int SRC, bool VF32>
__host__ __device__ constexpr size_t scatter_smem() {
  constexpr size_t vb = VF32 ? 4 : 8;
  return static_cast<size_t>(RX_TILE) * (8 + vb) * (scatter_staged<SRC>() ? 2 : 1) + 16;
}

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Bounded wait on a stage's bulk copy (limit_ns; a copy that never lands sends the call to the
// fallback instead of hanging the CTA).
__device__ __forceinline__ bool stage_wait(uint64_t* bar, uint32_t parity, uint32_t* fallback, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (globaltimer_ns() - t0 > limit_ns) {
      atomicOr(fallback, 4u);
      return false;
    }
  }
}

// SRC: 0 = the caller's key and value columns as they are, 1 = the caller's columns with mask /
// predicate / expression, 2 = segments of a partitioned buffer.  VF32: rows carry an f32 value.
// F32IN: the caller's columns are f32.
template <int SRC, bool VF32, bool F32IN, int DBITS>
__global__ void __launch_bounds__(RX_NT, 2) rx_scatter_kernel(RxScatter a) {
  using VT = typename std::conditional<VF32, float, double>::type;
  using ST = typename std::conditional<SRC == 0, int64_t, unsigned long long>::type;  // staged key / hash
  constexpr int ND = 1 << DBITS;  // destination digits of this pass
  constexpr bool STAGED = scatter_staged<SRC>();
  static_assert(ND <= RX_NT, "one thread per digit in phase B");
  extern __shared__ __align__(16) unsigned char rx_sm[];
  // the tile reordered by bucket (hashes, values); the bucket is recomputed from the hash when the
  // runs are written out
  unsigned long long* sh_h = reinterpret_cast<unsigned long long*>(rx_sm);
  VT* sh_v = reinterpret_cast<VT*>(rx_sm + RX_TILE * 8);
  // staged sources: the tile in flight (keys or hashes, values) and its mbarrier
  ST* st_k = reinterpret_cast<ST*>(rx_sm + RX_TILE * (8 + sizeof(VT)));
  VT* st_v = reinterpret_cast<VT*>(rx_sm + RX_TILE * (16 + sizeof(VT)));
  uint64_t* st_bar = reinterpret_cast<uint64_t*>(rx_sm + RX_TILE * (16 + 2 * sizeof(VT)));
  __shared__ unsigned int hist[ND];
  __shared__ unsigned int lstart[ND];
  __shared__ unsigned int wlim[ND];
  __shared__ unsigned long long gdst[ND];
  __shared__ unsigned int wsum[ND / 32];
  __shared__ unsigned int tile_total;
  constexpr unsigned int DMASK = ND - 1;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // an earlier pass overflowed, or the call was sent to the fallback before the passes
  if (*reinterpret_cast<volatile const uint32_t*>(a.fallback)) return;
  if (tid < ND) hist[tid] = 0;
  const long long ntiles = SRC == 2 ? a.seg_tiles[a.n_seg] : (a.n + RX_TILE - 1) / RX_TILE;
  VT* dst_v = static_cast<VT*>(a.dst_v);
  int seg = 0;
  // Source addresses of tile t when it is a full, 16-byte aligned tile of a staged source (every
  // thread decides the same way); `sg` walks the segments forward like the tile loop does.
  auto stage_src = [&](long long t, int& sg, const ST*& sk, const VT*& sv) -> bool {
    if (!STAGED || !a.stage || t >= ntiles) return false;
    if constexpr (SRC == 2) {
      while (__ldg(a.seg_tiles + sg + 1) <= t) ++sg;
      const long long r0 = (t - __ldg(a.seg_tiles + sg)) * RX_TILE;
      if (__ldg(a.seg_count + sg) - r0 < RX_TILE) return false;
      sk = reinterpret_cast<const ST*>(__ldg(a.seg_h + sg)) + r0;
      sv = reinterpret_cast<const VT*>(__ldg(a.seg_v + sg)) + r0;
    } else {
      const long long r0 = t * RX_TILE;
      if (a.n - r0 < RX_TILE) return false;
      sk = reinterpret_cast<const ST*>(a.keys) + r0;
      sv = static_cast<const VT*>(a.cols.a) + r0;
    }
    return aligned16(sk) && aligned16(sv);
  };
  // st_tile: the tile whose copy the stage holds or receives (-1: none); st_off: a copy did not land
  // in time, so this CTA issues no more (the call already falls back) and loads rows directly
  __shared__ long long st_tile;
  __shared__ int st_off;
  uint32_t st_phase = 0;
  int sg_next = 0;        // segment cursor of the copies issued ahead (thread 0)
  int st_pending = -1;    // thread 0: parity of a copy whose wait gave up, still to be waited out
  if (tid == 0) {
    st_tile = -1;
    st_off = 0;
  }
  if (STAGED && tid == 0) {
    mbar_init(st_bar, 1);
    mbar_fence_init();
    const ST* sk = nullptr;
    const VT* sv = nullptr;
    if (stage_src(blockIdx.x, sg_next, sk, sv)) {
      mbar_arrive_expect_tx(st_bar, RX_TILE * (8 + sizeof(VT)));
      bulk_g2s(st_k, sk, RX_TILE * 8, st_bar);
      bulk_g2s(st_v, sv, RX_TILE * sizeof(VT), st_bar);
      st_tile = blockIdx.x;
    }
  }
  __syncthreads();
  for (long long t = blockIdx.x; t < ntiles; t += gridDim.x) {
    long long row0, rows;
    unsigned long long obase = 0;  // first destination bucket of this tile's source segment
    const unsigned long long* src_h = nullptr;
    const VT* src_v = nullptr;
    if constexpr (SRC == 2) {
      while (__ldg(a.seg_tiles + seg + 1) <= t) ++seg;
      const long long tin = t - __ldg(a.seg_tiles + seg);
      row0 = tin * RX_TILE;
      rows = __ldg(a.seg_count + seg) - row0;
      src_h = reinterpret_cast<const unsigned long long*>(__ldg(a.seg_h + seg));
      src_v = reinterpret_cast<const VT*>(__ldg(a.seg_v + seg));
      obase = static_cast<unsigned long long>(__ldg(a.seg_digit + seg)) * ND;
    } else {
      row0 = t * RX_TILE;
      rows = a.n - row0;
    }
    if (rows > RX_TILE) rows = RX_TILE;

    // ---- phase A: load, hash, rank inside the tile
    unsigned long long hv[RX_PER];
    VT vv[RX_PER];
    unsigned int rk[RX_PER];  // bit 31 valid, bits 16-24 digit, bits 0-15 rank
    bool staged = false;
    if constexpr (STAGED) {
      staged = st_tile == t;  // the same in every thread: written by thread 0 between barriers
      if (staged) {
        if (!stage_wait(st_bar, st_phase, a.fallback, 2000000000ull)) {
          staged = false;  // this thread's rows then come from global memory
          st_off = 1;
          if (tid == 0) st_pending = static_cast<int>(st_phase);
        }
        st_phase ^= 1u;
      }
    }
    if constexpr (SRC == 2) {
      if (staged) {
#pragma unroll
        for (int j = 0; j < RX_PER; ++j) {
          hv[j] = st_k[j * RX_NT + tid];
          vv[j] = st_v[j * RX_NT + tid];
        }
      } else {
#pragma unroll
        for (int j = 0; j < RX_PER; ++j) {
          const int li = j * RX_NT + tid;
          if (li < rows) {
            hv[j] = __ldcs(src_h + row0 + li);
            vv[j] = __ldcs(src_v + row0 + li);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < RX_PER; ++j) {
        const int li = j * RX_NT + tid;
        rk[j] = 0;
        if (li < rows) {
          const unsigned d = static_cast<unsigned>(hv[j] >> a.shift) & DMASK;
          rk[j] = 0x80000000u | (d << 16) | atomicAdd(hist + d, 1u);
        }
      }
    } else if constexpr (SRC == 0) {
      if (staged) {
#pragma unroll
        for (int j = 0; j < RX_PER; ++j) {
          hv[j] = static_cast<unsigned long long>(st_k[j * RX_NT + tid]);
          vv[j] = st_v[j * RX_NT + tid];
        }
      } else {
#pragma unroll
        for (int j = 0; j < RX_PER; ++j) {
          const int li = j * RX_NT + tid;
          if (li < rows) {
            hv[j] = static_cast<unsigned long long>(__ldcs(a.keys + row0 + li));
            vv[j] = __ldcs(static_cast<const VT*>(a.cols.a) + row0 + li);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < RX_PER; ++j) {
        const int li = j * RX_NT + tid;
        rk[j] = 0;
        if (li < rows) {
          hv[j] = fmix64(hv[j]);
          const unsigned d = static_cast<unsigned>(hv[j] >> (64 - DBITS));
          rk[j] = 0x80000000u | (d << 16) | atomicAdd(hist + d, 1u);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < RX_PER; ++j) {
        const int li = j * RX_NT + tid;
        rk[j] = 0;
        if (li >= rows) continue;
        const long long row = row0 + li;
        if (a.mask && !((__ldg(a.mask + (row >> 6)) >> (row & 63)) & 1ull)) continue;
        const double av = load_val<F32IN>(a.cols.a, row);
        if (!eval_pred(a.cols.pred, av, a.cols.threshold)) continue;
        if constexpr (VF32) {
          vv[j] = static_cast<float>(av);  // an f32 column without expression: exact
        } else {
          const int expr = a.cols.expr;
          const double bv = expr != TBGB_EXPR_A ? load_val<F32IN>(a.cols.b, row) : 0.0;
          const double cv = expr == TBGB_EXPR_MUL_ADD ? load_val<F32IN>(a.cols.c, row) : 0.0;
          vv[j] = eval_expr(expr, av, bv, cv);
        }
        hv[j] = fmix64(static_cast<unsigned long long>(__ldcs(a.keys + row)));
        const unsigned d = static_cast<unsigned>(hv[j] >> (64 - DBITS));
        rk[j] = 0x80000000u | (d << 16) | atomicAdd(hist + d, 1u);
      }
    }
    __syncthreads();
    // every thread has read the stage: copy the CTA's next tile into it
    if (STAGED && tid == 0) {
      st_tile = -1;
      const ST* sk = nullptr;
      const VT* sv = nullptr;
      if (!st_off && stage_src(t + gridDim.x, sg_next, sk, sv)) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(st_bar, RX_TILE * (8 + sizeof(VT)));
        bulk_g2s(st_k, sk, RX_TILE * 8, st_bar);
        bulk_g2s(st_v, sv, RX_TILE * sizeof(VT), st_bar);
        st_tile = t + gridDim.x;
      }
    }

    // ---- phase B: claim a run per bucket, offsets of the buckets inside the tile
    unsigned int c = 0, inc = 0;
    if (tid < ND) {
      c = hist[tid];
      hist[tid] = 0;
      unsigned long long g = 0;
      unsigned int w = 0;
      if (c) {
        const unsigned long long b = obase + tid;
        const unsigned long long pos = atomicAdd(a.cursor + b, static_cast<unsigned long long>(c));
        const unsigned long long cap = a.out_base ? a.out_cap[b] : a.cap;
        if (pos < cap) w = cap - pos < c ? static_cast<unsigned int>(cap - pos) : c;
        if (w < c) atomicOr(a.fallback, 1u);
        g = (a.out_base ? a.out_base[b] : b * a.cap) + pos;
      }
      gdst[tid] = g;
      wlim[tid] = w;
      inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
      }
      if (lane == 31) wsum[warp] = inc;
    }
    __syncthreads();
    if (tid < ND) {
      unsigned int before = inc - c;
      for (int w = 0; w < warp; ++w) before += wsum[w];
      lstart[tid] = before;
      if (tid == ND - 1) tile_total = before + c;
    }
    __syncthreads();

    // ---- phase C: reorder the tile by bucket in shared memory
#pragma unroll
    for (int j = 0; j < RX_PER; ++j) {
      if (rk[j] >> 31) {
        const unsigned d = (rk[j] >> 16) & DMASK;
        const unsigned p = lstart[d] + (rk[j] & 0xFFFFu);
        sh_h[p] = hv[j];
        sh_v[p] = vv[j];
      }
    }
    __syncthreads();

    // ---- phase D: write each bucket's run (consecutive threads, consecutive addresses)
    const unsigned int tot = tile_total;
    for (unsigned int p = tid; p < tot; p += RX_NT) {
      const unsigned long long h = sh_h[p];
      const unsigned d = SRC == 2 ? static_cast<unsigned>(h >> a.shift) & DMASK : static_cast<unsigned>(h >> (64 - DBITS));
      const unsigned i = p - lstart[d];
      if (i < wlim[d]) {
        const unsigned long long dst = gdst[d] + i;
        a.dst_h[dst] = h;
        dst_v[dst] = sh_v[p];
      }
    }
    // the next tile's first barrier orders these reads before lstart / gdst / sh_* change
  }
  // a copy whose wait gave up may still be in flight into this CTA's shared memory: wait once
  // more (bounded) before the CTA exits
  if (STAGED && tid == 0 && st_pending >= 0) stage_wait(st_bar, static_cast<uint32_t>(st_pending), a.fallback, 500000000ull);
}

// Segments of pass 2 (one per first-pass bucket): addresses, rows written, tiles.
__global__ void rx_segments_kernel(Aux* x, unsigned long long cap1, const unsigned long long* t1h, const char* t1v,
                                   int value_bytes) {
  __shared__ long long tiles[kRadixDigits];
  const int d = threadIdx.x;
  unsigned long long c = x->cur1[d];
  if (c > cap1) c = cap1;
  x->seg_h[d] = reinterpret_cast<unsigned long long>(t1h + d * cap1);
  x->seg_v[d] = reinterpret_cast<unsigned long long>(t1v + d * cap1 * value_bytes);
  x->seg_count[d] = static_cast<long long>(c);
  x->seg_digit[d] = d;
  tiles[d] = static_cast<long long>((c + RX_TILE - 1) / RX_TILE);
  __syncthreads();
  if (d == 0) {
    long long s = 0;
    for (int i = 0; i < kRadixDigits; ++i) {
      x->seg_tiles[i] = s;
      s += tiles[i];
    }
    x->seg_tiles[kRadixDigits] = s;
  }
}

// Rows per top digit of a routing pass (the rows that pass mask and predicate).
template <bool PLAIN, bool F32IN>
__global__ void __launch_bounds__(RX_NT) rx_count_kernel(RxScatter a) {
  __shared__ unsigned int hist[kRadixDigits];
  const int tid = threadIdx.x;
  if (tid < kRadixDigits) hist[tid] = 0;
  __syncthreads();
  const long long stride = static_cast<long long>(gridDim.x) * RX_NT;
  for (long long row = static_cast<long long>(blockIdx.x) * RX_NT + tid; row < a.n; row += stride) {
    if constexpr (!PLAIN) {
      if (a.mask && !((__ldg(a.mask + (row >> 6)) >> (row & 63)) & 1ull)) continue;
      if (!eval_pred(a.cols.pred, load_val<F32IN>(a.cols.a, row), a.cols.threshold)) continue;
    }
    const unsigned long long h = fmix64(static_cast<unsigned long long>(__ldcs(a.keys + row)));
    atomicAdd(hist + (h >> (64 - D1_BITS)), 1u);
  }
  __syncthreads();
  if (tid < kRadixDigits && hist[tid]) atomicAdd(a.cursor + tid, static_cast<unsigned long long>(hist[tid]));
}

// Exact placement of a routing pass: digit d's rows start after those of the digits below it.
__global__ void rx_route_bases_kernel(Aux* x, int64_t* digit_counts) {
  if (threadIdx.x == 0) {
    unsigned long long s = 0;
    for (int d = 0; d < kRadixDigits; ++d) {
      const unsigned long long c = x->cur1[d];
      x->route_base[d] = s;
      x->route_cap[d] = c;
      digit_counts[d] = static_cast<int64_t>(c);
      s += c;
      x->cur1[d] = 0;  // the scatter claims from zero again
    }
  }
}

// Segments of a routed groupby: sender s's rows of digits [digit_lo, digit_lo + n_digits) start
// at B.h[s] / B.v[s], in digit order; counts[s * n_digits + j].  Segments are numbered digit-major
// (digit j of every sender, then digit j + 1), so the second pass's tiles alternate between the
// senders' buffers: peers' rows over NVLink and local rows from HBM are read at the same time.
__global__ void rx_routed_segments_kernel(Aux* x, const int64_t* counts, SenderBases B, int n_senders, int n_digits,
                                          int value_bytes) {
  if (threadIdx.x == 0) {
    unsigned long long off[kMaxSenders];
    for (int s = 0; s < n_senders; ++s) off[s] = 0;
    long long tiles = 0;
    int i = 0;
    for (int j = 0; j < n_digits; ++j) {
      for (int s = 0; s < n_senders; ++s, ++i) {
        const long long c0 = counts[static_cast<long long>(s) * n_digits + j];
        const long long c = c0 > 0 ? c0 : 0;
        x->seg_h[i] = B.h[s] + off[s] * 8;
        x->seg_v[i] = B.v[s] + off[s] * static_cast<unsigned long long>(value_bytes);
        x->seg_count[i] = c;
        x->seg_digit[i] = j;
        x->seg_tiles[i] = tiles;
        off[s] += static_cast<unsigned long long>(c);
        tiles += (c + RX_TILE - 1) / RX_TILE;
      }
    }
    x->seg_tiles[i] = tiles;
  }
}

// Group keys of a fallback that grouped the hashes themselves: each output key is a hash; turn
// it back into the key (runs only when the fallback ran).
__global__ void rx_unhash_kernel(int64_t* keys, const int64_t* d_n_groups, long long max_groups,
                                 const uint32_t* gate) {
  if (*gate == 0u) return;
  long long g = *d_n_groups;
  if (g > max_groups) g = max_groups;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < g; i += stride)
    keys[i] = static_cast<int64_t>(unfmix64(static_cast<unsigned long long>(keys[i])));
}

struct RxAgg {
  const unsigned long long* src_h;
  const void* src_v;
  const unsigned long long* cursor;
  int n_buckets;               // buckets of this call (all 65,536, or an owner's share)
  int bucket0;                 // bucket index of local bucket 0 (the top 17 bits of its hashes)
  unsigned long long cap;
  long long max_groups;
  int64_t* out_keys;
  tbgb_moments out;
  unsigned long long* n_groups;
  uint32_t* fallback;
};

// f32 values are summed exactly in 64-bit fixed point with FX_SHIFT = 36 fraction bits, held as
// two u32 words a slot: on B200 a 32-bit shared-memory atomic add runs about six times faster
// than a 64-bit one (f64 or u64 alike), and the carry out of the low word follows from the value
// the low word's atomic returns, so the sum is exact whatever the order of the adds.  An f32 of
// magnitude >= 2^-13 is a multiple of 2^-36 (24 significant bits), so v * 2^36 is an integer;
// values outside [2^-13, 2^E), E chosen so that a bucket's sum stays inside 63 bits, take an f64
// atomic into a second per-slot sum.  The output is the fixed-point total (exact) rounded once to
// f64, plus that f64 sum.
constexpr int FX_SHIFT = 36;
constexpr double kFxMin = 0x1p-13;  // smallest magnitude whose f32 value is a multiple of 2^-36

template <bool VF32>
constexpr size_t agg_smem() {
  return static_cast<size_t>(AGG_SLOTS) * (VF32 ? (8 + 8 + 4 + 4 + 4) : (8 + 8 + 4));
}

template <bool VF32>
__global__ void __launch_bounds__(AGG_NT, 3) rx_agg_kernel(RxAgg a) {
  using VT = typename std::conditional<VF32, float, double>::type;
  extern __shared__ __align__(16) unsigned char ag_sm[];
  unsigned long long* tk = reinterpret_cast<unsigned long long*>(ag_sm);  // key (low 46 bits of h)
  // f64 values: the sum of finite values; f32 values: the sum of those outside the fixed range
  double* ts = reinterpret_cast<double*>(tk + AGG_SLOTS);
  unsigned int* tc = reinterpret_cast<unsigned int*>(ts + AGG_SLOTS);     // non-NaN rows
  unsigned int* flo = tc + AGG_SLOTS;                                     // f32: fixed-point sum, low word
  unsigned int* fhi = flo + AGG_SLOTS;                                    //      and high word
  __shared__ unsigned int wcount[AGG_NT / 32];
  __shared__ unsigned long long gbase;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  volatile const uint32_t* fb = a.fallback;
  if (*fb) return;  // an earlier pass overflowed
  const VT* src_v = static_cast<const VT*>(a.src_v);
  // magnitudes below fx_lim keep a bucket's fixed-point sum (at most cap rows) inside 63 bits
  const int cap_bits = 64 - __clzll(a.cap | 1ull);
  const double fx_lim = ldexp(1.0, 63 - FX_SHIFT - cap_bits);
  // the table starts empty; each bucket's output loop empties the slots it used
  for (int i = tid; i < AGG_SLOTS; i += AGG_NT) {
    tk[i] = kFree;
    ts[i] = 0.0;
    tc[i] = 0u;
    if constexpr (VF32) {
      flo[i] = 0u;
      fhi[i] = 0u;
    }
  }
  __syncthreads();
  for (int b = blockIdx.x; b < a.n_buckets; b += gridDim.x) {
    const unsigned long long base = static_cast<unsigned long long>(b) * a.cap;
    unsigned long long rows = a.cursor[b];
    if (rows > a.cap) rows = a.cap;
    for (unsigned long long p0 = 0; p0 < rows; p0 += static_cast<unsigned long long>(AGG_NT) * AGG_UNROLL) {
      unsigned long long hv[AGG_UNROLL];
      double vv[AGG_UNROLL];
#pragma unroll
      for (int u = 0; u < AGG_UNROLL; ++u) {
        const unsigned long long p = p0 + static_cast<unsigned long long>(u) * AGG_NT + tid;
        if (p < rows) {
          hv[u] = a.src_h[base + p];
          vv[u] = static_cast<double>(src_v[base + p]);
        }
      }
#pragma unroll
      for (int u = 0; u < AGG_UNROLL; ++u) {
        const unsigned long long p = p0 + static_cast<unsigned long long>(u) * AGG_NT + tid;
        if (p >= rows) continue;
        const unsigned long long key = hv[u] & kKeyMask;
        unsigned int slot = static_cast<unsigned int>(hv[u]) & (AGG_SLOTS - 1);
        int found = -1;
        for (int probe = 0; probe < AGG_MAX_PROBE; ++probe) {
          unsigned long long w = tk[slot];
          if (w == kFree) w = atomicCAS(tk + slot, kFree, key);
          if (w == kFree || w == key) {  // claimed it, or found it
            found = static_cast<int>(slot);
            break;
          }
          slot = (slot + 1) & (AGG_SLOTS - 1);
        }
        if (found < 0) {
          atomicOr(a.fallback, 2u);  // more distinct keys than the table takes: recompute elsewhere
          continue;
        }
        const double v = vv[u];
        if (!is_nan(v)) atomicAdd(tc + found, 1u);  // a NaN row makes its group, uncounted
        if constexpr (VF32) {
          const double av = fabs(v);
          if (av >= kFxMin && av < fx_lim) {
            const unsigned long long q = static_cast<unsigned long long>(__double2ll_rn(v * 0x1p36));  // exact
            const unsigned int xl = static_cast<unsigned int>(q), xh = static_cast<unsigned int>(q >> 32);
            const unsigned int old = atomicAdd(flo + found, xl);
            const unsigned int hi = xh + (old + xl < old ? 1u : 0u);  // carry out of the low word
            if (hi) atomicAdd(fhi + found, hi);
          } else if (is_finite(v) && v != 0.0) {
            atomicAdd(ts + found, v);
          }
        } else {
          if (is_finite(v)) atomicAdd(ts + found, v);
        }
      }
    }
    __syncthreads();
    // the occupied slots, compacted in slot order: warp w takes slots k * AGG_NT + w * 32 + lane
    unsigned int mine = 0;
    for (int k = 0; k < AGG_SLOTS / AGG_NT; ++k)
      mine += __popc(__ballot_sync(0xffffffffu, tk[k * AGG_NT + tid] != kFree));
    if (lane == 0) wcount[warp] = mine;
    __syncthreads();
    if (warp == 0) {
      const unsigned int cnt = lane < AGG_NT / 32 ? wcount[lane] : 0u;
      unsigned int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (lane < AGG_NT / 32) wcount[lane] = incl - cnt;
      if (lane == 31) gbase = atomicAdd(a.n_groups, static_cast<unsigned long long>(incl));
    }
    __syncthreads();
    unsigned long long pos = gbase + wcount[warp];
    const unsigned long long top = static_cast<unsigned long long>(b + a.bucket0) << KEY_BITS;
    for (int k = 0; k < AGG_SLOTS / AGG_NT; ++k) {
      const int i = k * AGG_NT + tid;
      const unsigned long long w = tk[i];
      const bool occ = w != kFree;
      const unsigned bal = __ballot_sync(0xffffffffu, occ);
      if (occ) {
        const unsigned long long j = pos + __popc(bal & ((1u << lane) - 1u));
        if (j < static_cast<unsigned long long>(a.max_groups)) {
          const double cnt = static_cast<double>(tc[i]);
          double sum = ts[i];
          if constexpr (VF32) {
            const long long fx = static_cast<long long>((static_cast<unsigned long long>(fhi[i]) << 32) | flo[i]);
            sum = ldexp(static_cast<double>(fx), -FX_SHIFT) + sum;
          }
          a.out_keys[j] = static_cast<int64_t>(unfmix64(top | w));
          if (a.out.count) a.out.count[j] = cnt;
          if (a.out.sum) a.out.sum[j] = sum;
          if (a.out.mean) a.out.mean[j] = cnt > 0.0 ? sum / cnt : qnan();
        }
        // empty the slot for the next bucket (only this thread reads it from here on)
        tk[i] = kFree;
        ts[i] = 0.0;
        tc[i] = 0u;
        if constexpr (VF32) {
          flo[i] = 0u;
          fhi[i] = 0u;
        }
      }
      pos += __popc(bal);
    }
    __syncthreads();  // the next bucket's rows reach the table only after every slot was emptied
  }
}

__global__ void rx_finish_kernel(const Aux* x, long long max_groups, int64_t* d_n_groups, uint32_t* err) {
  if (x->fallback) return;  // the fallback strategy writes the group count
  unsigned long long g = x->n_groups;
  if (g > static_cast<unsigned long long>(max_groups)) {
    atomicOr(err, KERR_TABLE_FULL);
    g = static_cast<unsigned long long>(max_groups);
  }
  *d_n_groups = static_cast<int64_t>(g);
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

unsigned long long round16(unsigned long long x) { return (x + 15) / 16 * 16; }


// Rows of a bucket's region: its even share e plus slack.  A bucket's rows arrive in clumps (all
// rows of a key land in one bucket), so its row count varies with the keys' multiplicity, not
// only as a Poisson count of rows: with about 7.5 rows a key the standard deviation is about
// 2.9 sqrt(e) (250 rows on a final bucket of 7,600 at 2^28 keys of 7.5 rows).  40 sqrt(e) is ten deviations for keys of up
// to about 15 rows each; heavier keys overflow into the fallback.
unsigned long long bucket_cap(unsigned long long e, unsigned long long margin) {
  return round16(e + static_cast<unsigned long long>(40.0 * std::sqrt(static_cast<double>(e))) + margin);
}

template <int SRC, bool VF32, bool F32IN>
cudaError_t launch_scatter(const RxScatter& s, int grid, cudaStream_t st) {
  auto k = rx_scatter_kernel<SRC, VF32, F32IN, SRC == 2 ? D2_BITS : D1_BITS>;
  constexpr size_t smem = scatter_smem<SRC, VF32>();
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return e;
  k<<<grid, RX_NT, smem, st>>>(s);
  return cudaGetLastError();
}

template <bool VF32>
cudaError_t launch_agg(const RxAgg& g, int grid, cudaStream_t st) {
  auto k = rx_agg_kernel<VF32>;
  constexpr size_t smem = agg_smem<VF32>();
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return e;
  k<<<grid, AGG_NT, smem, st>>>(g);
  return cudaGetLastError();
}

int agg_blocks_per_sm(bool vf32) {
  static int cached[2] = {0, 0};
  int& c = cached[vf32 ? 1 : 0];
  if (c == 0) {
    int v = 0;
    const size_t smem = vf32 ? agg_smem<true>() : agg_smem<false>();
    auto k = vf32 ? rx_agg_kernel<true> : rx_agg_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, k, AGG_NT, smem);
    c = (e == cudaSuccess && v > 0) ? v : 1;
  }
  return c;
}

int scatter_blocks_per_sm(bool vf32) {
  static int cached[2] = {0, 0};
  int& c = cached[vf32 ? 1 : 0];
  if (c == 0) {
    int v = 0;
    const size_t smem = vf32 ? scatter_smem<2, true>() : scatter_smem<2, false>();
    cudaError_t e = vf32 ? cudaFuncSetAttribute(rx_scatter_kernel<2, true, true, D2_BITS>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem))
                         : cudaFuncSetAttribute(rx_scatter_kernel<2, false, false, D2_BITS>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e == cudaSuccess) {
      e = vf32 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, rx_scatter_kernel<2, true, true, D2_BITS>, RX_NT, smem)
               : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, rx_scatter_kernel<2, false, false, D2_BITS>, RX_NT, smem);
    }
    c = (e == cudaSuccess && v > 0) ? v : 1;
  }
  return c;
}

}  // namespace

bool radix_eligible(const tbgb_columns& cols, const tbgb_moments* out, long long n, long long max_groups) {
  (void)cols;
  if (!out || out->min || out->max || out->m2 || out->var_pop || out->var_samp || out->m3 || out->m4) return false;
  return n >= (1ll << 24) && max_groups >= (1ll << 22) && max_groups <= kRadixMaxGroups;
}

RadixPlan radix_plan(const tbgb_columns& cols, long long n, int num_sms) {
  RadixPlan P{};
  P.vf32 = cols.dtype == TBGB_F32 && cols.expr == TBGB_EXPR_A;
  const unsigned long long rows = static_cast<unsigned long long>(n > 0 ? n : 0);
  const unsigned long long e1 = rows / kRadixDigits, e2 = rows / kRadixBuckets;
  P.cap1 = bucket_cap(e1, 4096);
  P.cap2 = bucket_cap(e2, 256);
  const size_t row_bytes = 8 + (P.vf32 ? 4 : 8);
  P.t1_bytes = align256(static_cast<size_t>(P.cap1) * kRadixDigits * 8) +
               align256(static_cast<size_t>(P.cap1) * kRadixDigits * (row_bytes - 8));
  P.t2_bytes = align256(static_cast<size_t>(P.cap2) * kRadixBuckets * 8) +
               align256(static_cast<size_t>(P.cap2) * kRadixBuckets * (row_bytes - 8));
  P.aux_bytes = align256(sizeof(Aux));
  P.grid_scatter = num_sms * scatter_blocks_per_sm(P.vf32);
  P.grid_agg = num_sms * agg_blocks_per_sm(P.vf32);
  return P;
}

size_t radix_t2_offset(const RadixPlan& P) { return P.aux_bytes + P.t1_bytes; }

cudaError_t radix_groupby(const RadixPlan& P, const RadixArgs& a, void* ws, uint32_t** fallback, cudaStream_t s,
                          uint64_t* launches, cudaEvent_t ev0, cudaEvent_t ev1) {
  char* w = static_cast<char*>(ws);
  Aux* x = reinterpret_cast<Aux*>(w);
  const size_t vb = P.vf32 ? 4 : 8;
  unsigned long long* t1h = reinterpret_cast<unsigned long long*>(w + P.aux_bytes);
  void* t1v = w + P.aux_bytes + align256(static_cast<size_t>(P.cap1) * kRadixDigits * 8);
  unsigned long long* t2h = reinterpret_cast<unsigned long long*>(w + radix_t2_offset(P));
  void* t2v = w + radix_t2_offset(P) + align256(static_cast<size_t>(P.cap2) * kRadixBuckets * 8);
  (void)vb;
  *fallback = &x->fallback;
  cudaError_t e = cudaMemsetAsync(x, 0, sizeof(Aux), s);
  if (e != cudaSuccess) return e;
  if (ev0) cudaEventRecord(ev0, s);

  RxScatter p1{};
  p1.keys = a.keys;
  p1.cols = a.cols;
  p1.mask = a.mask;
  p1.n = a.n;
  p1.dst_h = t1h;
  p1.dst_v = t1v;
  p1.cursor = x->cur1;
  p1.cap = P.cap1;
  p1.fallback = &x->fallback;
  p1.stage = 1;  // local sources: full tiles arrive by bulk copy
  const bool plain = a.mask == nullptr && a.cols.pred == TBGB_PRED_NONE && a.cols.expr == TBGB_EXPR_A;
  const bool f32in = a.cols.dtype == TBGB_F32;
  if (a.n > 0) {
    if (plain) e = f32in ? launch_scatter<0, true, true>(p1, P.grid_scatter, s)
                         : launch_scatter<0, false, false>(p1, P.grid_scatter, s);
    else if (P.vf32) e = launch_scatter<1, true, true>(p1, P.grid_scatter, s);
    else e = f32in ? launch_scatter<1, false, true>(p1, P.grid_scatter, s)
                   : launch_scatter<1, false, false>(p1, P.grid_scatter, s);
    if (e != cudaSuccess) return e;
    (*launches)++;
  }
  rx_segments_kernel<<<1, kRadixDigits, 0, s>>>(x, P.cap1, t1h, static_cast<const char*>(t1v), P.vf32 ? 4 : 8);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  (*launches)++;

  RxScatter p2{};
  p2.seg_h = x->seg_h;
  p2.seg_v = x->seg_v;
  p2.seg_count = x->seg_count;
  p2.seg_digit = x->seg_digit;
  p2.seg_tiles = x->seg_tiles;
  p2.n_seg = kRadixDigits;
  p2.shift = KEY_BITS;
  p2.dst_h = t2h;
  p2.dst_v = t2v;
  p2.cursor = x->cur2;
  p2.cap = P.cap2;
  p2.fallback = &x->fallback;
  p2.stage = 1;  // local sources: full tiles arrive by bulk copy
  if (a.n > 0) {
    e = P.vf32 ? launch_scatter<2, true, true>(p2, P.grid_scatter, s)
               : launch_scatter<2, false, false>(p2, P.grid_scatter, s);
    if (e != cudaSuccess) return e;
    (*launches)++;
  }

  RxAgg g{};
  g.src_h = t2h;
  g.src_v = t2v;
  g.cursor = x->cur2;
  g.n_buckets = kRadixBuckets;
  g.bucket0 = 0;
  g.cap = P.cap2;
  g.max_groups = a.max_groups;
  g.out_keys = a.out_keys;
  g.out = a.out;
  g.n_groups = &x->n_groups;
  g.fallback = &x->fallback;
  if (a.n > 0) {
    e = P.vf32 ? launch_agg<true>(g, P.grid_agg, s) : launch_agg<false>(g, P.grid_agg, s);
    if (e != cudaSuccess) return e;
    (*launches)++;
  }
  if (ev1) cudaEventRecord(ev1, s);
  rx_finish_kernel<<<1, 1, 0, s>>>(x, a.max_groups, a.d_n_groups, a.err);
  e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

size_t radix_route_aux_bytes() { return align256(sizeof(Aux)); }

bool radix_value_f32(const tbgb_columns& cols) { return cols.dtype == TBGB_F32 && cols.expr == TBGB_EXPR_A; }

cudaError_t radix_route(const RadixArgs& a, unsigned long long* out_h, void* out_v, int64_t* digit_counts, void* aux,
                        int num_sms, cudaStream_t s, uint64_t* launches) {
  Aux* x = static_cast<Aux*>(aux);
  cudaError_t e = cudaMemsetAsync(x, 0, sizeof(Aux), s);
  if (e != cudaSuccess) return e;
  RxScatter p1{};
  p1.keys = a.keys;
  p1.cols = a.cols;
  p1.mask = a.mask;
  p1.n = a.n;
  p1.dst_h = out_h;
  p1.dst_v = out_v;
  p1.cursor = x->cur1;
  p1.out_base = x->route_base;
  p1.out_cap = x->route_cap;
  p1.fallback = &x->fallback;
  p1.stage = 1;  // local sources: full tiles arrive by bulk copy
  const bool plain = a.mask == nullptr && a.cols.pred == TBGB_PRED_NONE && a.cols.expr == TBGB_EXPR_A;
  const bool f32in = a.cols.dtype == TBGB_F32;
  const bool vf32 = radix_value_f32(a.cols);
  if (a.n > 0) {
    long long blocks = (a.n + RX_NT - 1) / RX_NT;
    const long long cap = static_cast<long long>(num_sms) * 4;
    if (blocks > cap) blocks = cap;
    if (plain) rx_count_kernel<true, false><<<static_cast<unsigned>(blocks), RX_NT, 0, s>>>(p1);
    else if (f32in) rx_count_kernel<false, true><<<static_cast<unsigned>(blocks), RX_NT, 0, s>>>(p1);
    else rx_count_kernel<false, false><<<static_cast<unsigned>(blocks), RX_NT, 0, s>>>(p1);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    (*launches)++;
  }
  rx_route_bases_kernel<<<1, 32, 0, s>>>(x, digit_counts);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  (*launches)++;
  if (a.n > 0) {
    const int grid = num_sms * scatter_blocks_per_sm(vf32);
    if (plain) e = f32in ? launch_scatter<0, true, true>(p1, grid, s) : launch_scatter<0, false, false>(p1, grid, s);
    else if (vf32) e = launch_scatter<1, true, true>(p1, grid, s);
    else e = f32in ? launch_scatter<1, false, true>(p1, grid, s) : launch_scatter<1, false, false>(p1, grid, s);
    if (e != cudaSuccess) return e;
    (*launches)++;
  }
  return cudaSuccess;
}

RadixPlan radix_routed_plan(bool vf32, long long n_rows, int n_digits, int num_sms) {
  RadixPlan P{};
  P.vf32 = vf32;
  const unsigned long long rows = static_cast<unsigned long long>(n_rows > 0 ? n_rows : 0);
  const unsigned long long nb = static_cast<unsigned long long>(n_digits) << D2_BITS;
  const unsigned long long e2 = rows / nb;
  P.cap1 = 0;
  P.cap2 = bucket_cap(e2, 256);
  const size_t vb = vf32 ? 4 : 8;
  P.t1_bytes = 0;
  P.t2_bytes = align256(static_cast<size_t>(P.cap2) * nb * 8) + align256(static_cast<size_t>(P.cap2) * nb * vb);
  P.aux_bytes = align256(sizeof(Aux));
  P.grid_scatter = num_sms * scatter_blocks_per_sm(vf32);
  P.grid_agg = num_sms * agg_blocks_per_sm(P.vf32);
  return P;
}

cudaError_t radix_groupby_routed(const RadixPlan& P, const RoutedArgs& r, void* ws, uint32_t** fallback,
                                 cudaStream_t s, uint64_t* launches, cudaEvent_t ev0, cudaEvent_t ev1) {
  char* w = static_cast<char*>(ws);
  Aux* x = reinterpret_cast<Aux*>(w);
  const unsigned long long nb = static_cast<unsigned long long>(r.n_digits) << D2_BITS;
  unsigned long long* t2h = reinterpret_cast<unsigned long long*>(w + radix_t2_offset(P));
  void* t2v = w + radix_t2_offset(P) + align256(static_cast<size_t>(P.cap2) * nb * 8);
  *fallback = &x->fallback;
  cudaError_t e = cudaMemsetAsync(x, 0, sizeof(Aux), s);
  if (e != cudaSuccess) return e;
  if (ev0) cudaEventRecord(ev0, s);
  const int n_seg = r.n_senders * r.n_digits;
  SenderBases B{};
  for (int i = 0; i < r.n_senders; ++i) {
    B.h[i] = reinterpret_cast<unsigned long long>(r.hashes[i]);
    B.v[i] = reinterpret_cast<unsigned long long>(r.vals[i]);
  }
  rx_routed_segments_kernel<<<1, 32, 0, s>>>(x, r.seg_counts, B, r.n_senders, r.n_digits, P.vf32 ? 4 : 8);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  (*launches)++;
  RxScatter p2{};
  p2.seg_h = x->seg_h;
  p2.seg_v = x->seg_v;
  p2.seg_count = x->seg_count;
  p2.seg_digit = x->seg_digit;
  p2.seg_tiles = x->seg_tiles;
  p2.n_seg = n_seg;
  p2.shift = KEY_BITS;
  p2.dst_h = t2h;
  p2.dst_v = t2v;
  p2.cursor = x->cur2;
  p2.cap = P.cap2;
  p2.fallback = &x->fallback;
  p2.stage = 0;  // peers' buffers are read with plain loads over NVLink
  if (r.n_rows > 0) {
    e = P.vf32 ? launch_scatter<2, true, true>(p2, P.grid_scatter, s)
               : launch_scatter<2, false, false>(p2, P.grid_scatter, s);
    if (e != cudaSuccess) return e;
    (*launches)++;
  }
  RxAgg g{};
  g.src_h = t2h;
  g.src_v = t2v;
  g.cursor = x->cur2;
  g.n_buckets = static_cast<int>(nb);
  g.bucket0 = r.digit_lo << D2_BITS;
  g.cap = P.cap2;
  g.max_groups = r.max_groups;
  g.out_keys = r.out_keys;
  g.out = r.out;
  g.n_groups = &x->n_groups;
  g.fallback = &x->fallback;
  if (r.n_rows > 0) {
    e = P.vf32 ? launch_agg<true>(g, P.grid_agg, s) : launch_agg<false>(g, P.grid_agg, s);
    if (e != cudaSuccess) return e;
    (*launches)++;
  }
  if (ev1) cudaEventRecord(ev1, s);
  rx_finish_kernel<<<1, 1, 0, s>>>(x, r.max_groups, r.d_n_groups, r.err);
  e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

cudaError_t radix_unhash_keys(int64_t* keys, const int64_t* d_n_groups, long long max_groups, const uint32_t* gate,
                              int num_sms, cudaStream_t s, uint64_t* launches) {
  rx_unhash_kernel<<<num_sms * 4, 256, 0, s>>>(keys, d_n_groups, max_groups, gate);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

}  // namespace tbgb
