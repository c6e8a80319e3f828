// dense.cu -- dense-key groupby moments for low cardinality (n_groups <= 1024).
//
// Semantics: DescriptiveEngine::moments_grouped (crates/tambear/src/descriptive.rs:383-435)
// with the NaN mask of nan_mask_count (:591-603) and the extrema of
// scatter_extremum / extremum_grouped_nan_safe (compute_engine.rs:304-322,
// descriptive.rs:606-620).  One pass over the data instead of the reference's two:
// per (CTA, group) the kernel keeps the finite count, a shift K, S1 = sum(v-K),
// S2 = sum((v-K)^2), min and max, plus +-inf counts; the partial states are merged
// with Chan's formula (descriptive.rs:216-253, intermediates.rs:352-377) in a fixed
// order, so the merge itself does not depend on which CTA finishes first.
//
// One persistent 800-thread CTA per SM, warp-specialised:
//   * TMA bulk copies (cp.async.bulk + mbarrier, no multicast) stream 4096-row
//     tiles of keys / values / mask words into a 2-deep shared-memory ring, and
//     bulk L2 prefetches run 4 tiles further ahead so that enough bytes are in
//     flight to cover loaded HBM latency without more shared memory (4096-row tiles
//     measured 13% faster than 2048-row tiles in a 4-deep ring: each owner's per-tile
//     bookkeeping is paid half as often and a column holds 16 rows per group on
//     average instead of 8, so the owner warps diverge less);
//   * warps 0-15 ("scatter") rank each finite row inside its group with a shared
//     u32 atomic and store the value into column `rank` of a [C][n_groups]
//     buffer (two buffers, alternating per tile); rows ranked >= C go to a
//     per-buffer shared spill list (and, if that fills, to a per-CTA spill state
//     in global memory, which also counts +-inf rows);
//   * one team of 8 owner warps sweeps the two column buffers in turn and keeps
//     each group's accumulators in registers (branch-free: the columns hold finite
//     values only; several accumulator chains per group, loads kept in flight).
//     16 scatter warps and one owner team measured faster than 8 scatter warps and
//     two owner teams (10^9 rows: 2.74 against 2.78 ms; the masked pushdown 0.47
//     against 0.58 ms): the scatter's shared atomics need the warps to hide their
//     latency, while one team keeps up with the sweeps;
//   * a producer warp refills the ring.
//   Hand-offs use mbarriers (tile full / column full / column empty) and named
//   barriers inside each warp group, so the two roles overlap instead of meeting
//   at CTA-wide barriers.
#include <cstdint>
#include <type_traits>

#include "common.cuh"
#include "dense.cuh"
#include "exchange.cuh"
#include "gstate.cuh"

namespace tbgb {

constexpr int NT = kDenseThreads;   // 800: 8 scatter + 2 x 8 owner + 1 producer warp
constexpr int NSC = 512;            // scatter threads (warps 0-15)
constexpr int NOW = 256;            // owner threads per team (warps 16-23)
constexpr int TEAMS = 1;            // one team sweeps the column buffers of all batches in turn
constexpr int SCATTER_WARPS = NSC / 32;
constexpr int PRODUCER_WARP = (NSC + TEAMS * NOW) / 32;  // warp 24
// 25 warps put up to 7 warps on one SM sub-partition: 72 registers per thread.
constexpr int TILE = kDenseTile;    // rows per staged tile
constexpr int STAGES = kDenseStages;
constexpr int RPS = TILE / NSC;     // rows per scatter thread per tile (16, taken four at a time)
constexpr int CHUNK = 2 * NSC;      // rows covered by one vector access of all scatter threads
static_assert(RPS % 4 == 0, "scatter mapping takes rows four at a time");

constexpr uint32_t KEY_BYTES = TILE * 4;
constexpr uint32_t VAL_BYTES = TILE * 8;
constexpr uint32_t MASK_BYTES = TILE / 8;
constexpr uint32_t STAGE_BYTES = KEY_BYTES + VAL_BYTES + MASK_BYTES;
static_assert(STAGE_BYTES % 16 == 0, "bulk copy sizes must be 16-byte multiples");

constexpr int PF_AHEAD = 4;     // tiles prefetched into L2 beyond the shared ring
constexpr int SPL = 256;        // shared spill-list entries per column buffer

constexpr int BAR_OWNER = 2;    // named barrier of the owner warps
constexpr unsigned long long K_UNSET = 0x7FF8000000000001ull;  // NaN payload no finite value has
constexpr uint32_t NO_RANK = 0xFFFFFFFFu;

// spill state, per CTA, SoA over groups (u64 words)
// (the third and fourth power sums exist only when m3 / m4 are computed: SP_BASE fields otherwise)
enum { SP_N = 0, SP_NINFP, SP_NINFN, SP_K, SP_S1, SP_S2, SP_MN, SP_MX, SP_BASE, SP_S3 = SP_BASE, SP_S4, SP_COUNT };
static_assert(SP_COUNT == kDenseSpillFields, "spill state size exported in dense.cuh");
template <bool M34>
__host__ __device__ constexpr int spill_fields() { return M34 ? SP_COUNT : SP_BASE; }

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// Barrier among `n` threads that also ORs a predicate across them.
__device__ __forceinline__ bool bar_red_or(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bounded wait that also gives up when the other warp group raised `abort`.
// Waiting threads sleep in try_wait (suspend hint) rather than spin.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, uint32_t* err, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > 2000000000ull) {
      atomicOr(err, KERR_TIMEOUT);
      return false;
    }
  }
}

struct DenseArgs {
  const int32_t* keys;
  const double* vals;
  const uint64_t* mask;  // nullable (MASKED template flag)
  long long n;
  long long row_offset;  // global index of row 0 (zero-tie ordering across shards)
  int G, C, opg, slots;
  double* part;                // owner partials [ST_COUNT][gridDim.x * TEAMS * slots]
  unsigned long long* spill;   // [gridDim.x][SP_COUNT][G]
  unsigned long long* zfirst;  // [G], preset to ~0
  uint32_t* err;
  // masked launches: tiles with a selected row (bit j of live_bits[w] = tile 32w + j) and the
  // exclusive prefix of their counts (live_pre[live_words] = all of them); NULL: every tile
  const unsigned* live_bits;
  const unsigned* live_pre;
  long long live_words;
};

// Walks the live tiles from a given rank (0-based among all live tiles) in increasing order.
struct LiveCursor {
  const unsigned* bits;
  long long w, nw;
  unsigned cur;
  __device__ __forceinline__ void init(const unsigned* b, const unsigned* pre, long long nw_, long long rank) {
    bits = b;
    nw = nw_;
    long long lo = 0, hi = nw_;  // the last word with pre[w] <= rank
    while (hi - lo > 1) {
      const long long mid = (lo + hi) >> 1;
      if (static_cast<long long>(pre[mid]) <= rank) lo = mid;
      else hi = mid;
    }
    w = lo;
    cur = nw_ > 0 ? b[lo] : 0u;
    for (long long s = rank - static_cast<long long>(pre[lo]); s > 0 && cur; --s) cur &= cur - 1u;
  }
  __device__ __forceinline__ long long next() {
    while (cur == 0u && w + 1 < nw) cur = bits[++w];
    const int j = __ffs(cur) - 1;
    cur &= cur - 1u;
    return w * 32 + j;
  }
};

size_t dense_smem_bytes(int G, int C) {
  const size_t gp = (static_cast<size_t>(G) + 3) & ~size_t(3);
  return static_cast<size_t>(STAGES) * STAGE_BYTES + 2 * static_cast<size_t>(C) * G * 8 + 2 * SPL * 8 +
         2 * gp * 4 + 2 * SPL * 4 + 16 + (2 * STAGES + 4) * 8 + 16;
}

// Column capacity (rows per group in one column buffer) and owners per group for G groups.
__host__ __device__ constexpr int dense_cols(int G) {
  return (kDenseColBudget / 2) / G > TILE ? TILE : ((kDenseColBudget / 2) / G < 1 ? 1 : (kDenseColBudget / 2) / G);
}
__host__ __device__ constexpr int dense_opg(int G) { return G >= NOW ? 1 : NOW / G; }

DenseLaunch dense_plan(int G, int num_sms) {
  DenseLaunch L{};
  L.grid = num_sms;
  L.C = dense_cols(G);
  L.opg = dense_opg(G);
  L.slots = G * L.opg;
  const int ms = (L.slots + NOW - 1) / NOW;
  L.maxslots = ms <= 1 ? 1 : (ms <= 2 ? 2 : 4);
  L.smem = dense_smem_bytes(G, L.C);
  L.part_doubles = static_cast<size_t>(ST_COUNT) * L.grid * TEAMS * L.slots;
  L.spill_words = static_cast<size_t>(SP_COUNT) * L.grid * G;
  return L;
}

// Rare path: a finite row that found its column full.
template <bool M34>
__device__ __forceinline__ void spill_add(unsigned long long* sp, int G, int g, double v) {
  const unsigned long long vb = static_cast<unsigned long long>(__double_as_longlong(v));
  const unsigned long long kb = atomicCAS(sp + SP_K * G + g, K_UNSET, vb);
  const double K = kb == K_UNSET ? v : __longlong_as_double(static_cast<long long>(kb));
  const double d = v - K;
  atomicAdd(reinterpret_cast<double*>(sp + SP_S1 * G + g), d);
  atomicAdd(reinterpret_cast<double*>(sp + SP_S2 * G + g), d * d);
  // (written as in the two-moment kernel: how this rare path is written changed the
  // scheduling of the whole kernel measurably)
  if constexpr (M34) {
    atomicAdd(reinterpret_cast<double*>(sp + SP_S3 * G + g), d * d * d);
    atomicAdd(reinterpret_cast<double*>(sp + SP_S4 * G + g), (d * d) * (d * d));
  }
  atomicAdd(sp + SP_N * G + g, 1ull);
  atomicMin(sp + SP_MN * G + g, f2o(v));
  atomicMax(sp + SP_MX * G + g, f2o(v));
}

// Register accumulators of one owner slot; NCH independent chains shorten the
// dependency path through S1/S2.
template <int NCH>
struct OwnerAcc {
  double K, s1[NCH], s2[NCH], mn, mx;
  unsigned long long nf;
  bool kset;
  __device__ __forceinline__ void init() {
    K = 0.0;
#pragma unroll
    for (int j = 0; j < NCH; ++j) { s1[j] = 0.0; s2[j] = 0.0; }
    mn = pos_inf(); mx = neg_inf(); nf = 0; kset = false;
  }
  __device__ __forceinline__ void quad(double x0, double x1, double x2, double x3) {
    const double d0 = x0 - K, d1 = x1 - K, d2 = x2 - K, d3 = x3 - K;
    s1[0 % NCH] += d0;
    s2[0 % NCH] = fma(d0, d0, s2[0 % NCH]);
    s1[1 % NCH] += d1;
    s2[1 % NCH] = fma(d1, d1, s2[1 % NCH]);
    s1[2 % NCH] += d2;
    s2[2 % NCH] = fma(d2, d2, s2[2 % NCH]);
    s1[3 % NCH] += d3;
    s2[3 % NCH] = fma(d3, d3, s2[3 % NCH]);
    // extrema by plain compares (no NaN reaches a column); +-0 ties are settled
    // later from the first-zero tracker
    const bool l01 = x0 < x1, l23 = x2 < x3;
    const double lo01 = l01 ? x0 : x1, hi01 = l01 ? x1 : x0;
    const double lo23 = l23 ? x2 : x3, hi23 = l23 ? x3 : x2;
    const double lo = lo01 < lo23 ? lo01 : lo23, hi = hi01 > hi23 ? hi01 : hi23;
    mn = lo < mn ? lo : mn;
    mx = hi > mx ? hi : mx;
  }
  __device__ __forceinline__ void one(double x) {
    const double d = x - K;
    s1[0] += d;
    s2[0] = fma(d, d, s2[0]);
    mn = x < mn ? x : mn;
    mx = x > mx ? x : mx;
  }
  // Sweep entries sub, sub+opg, ... < c of one group's column (finite values
  // only), keeping the next four loads in flight while the current four are added.
  __device__ __forceinline__ void sweep(const double* cg, int c, int sub, int opg, int G) {
    if (c <= sub) return;
    const size_t step = static_cast<size_t>(opg) * G;
    const double* p = cg + static_cast<size_t>(sub) * G;
    const int m = (c - sub + opg - 1) / opg;  // values of this sub-owner
    if (!kset) { K = p[0]; kset = true; }
    int i = 0;
    if (m >= 4) {
      double y0 = p[0], y1 = p[step], y2 = p[2 * step], y3 = p[3 * step];
      for (; i + 8 <= m; i += 4) {
        const double x0 = y0, x1 = y1, x2 = y2, x3 = y3;
        const double* q = p + static_cast<size_t>(i + 4) * step;
        y0 = q[0];
        y1 = q[step];
        y2 = q[2 * step];
        y3 = q[3 * step];
        quad(x0, x1, x2, x3);
      }
      quad(y0, y1, y2, y3);
      i += 4;
    }
    for (; i < m; ++i) one(p[static_cast<size_t>(i) * step]);
    nf += static_cast<unsigned long long>(m);
  }
  __device__ __forceinline__ void add1(double x) {
    if (!kset) { K = x; kset = true; }
    one(x);
    nf += 1;
  }
  __device__ __forceinline__ double sum_s1() const {
    double r = 0.0;
#pragma unroll
    for (int j = 0; j < NCH; ++j) r += s1[j];
    return r;
  }
  __device__ __forceinline__ double sum_s2() const {
    double r = 0.0;
#pragma unroll
    for (int j = 0; j < NCH; ++j) r += s2[j];
    return r;
  }
};

// The accumulator of an owner slot when m3 / m4 are requested: the third and fourth
// power sums as well (kept apart from OwnerAcc so that the common path is unchanged).
template <int NCH>
struct OwnerAcc4 {
  double K, s1[NCH], s2[NCH], s3[NCH], s4[NCH], mn, mx;
  unsigned long long nf;
  bool kset;
  __device__ __forceinline__ void init() {
    K = 0.0;
#pragma unroll
    for (int j = 0; j < NCH; ++j) { s1[j] = 0.0; s2[j] = 0.0; s3[j] = 0.0; s4[j] = 0.0; }
    mn = pos_inf(); mx = neg_inf(); nf = 0; kset = false;
  }
  __device__ __forceinline__ void pw(int j, double d) {
    const double dd = d * d;
    s1[j] += d;
    s2[j] += dd;
    s3[j] = fma(dd, d, s3[j]);
    s4[j] = fma(dd, dd, s4[j]);
  }
  __device__ __forceinline__ void quad(double x0, double x1, double x2, double x3) {
    pw(0 % NCH, x0 - K);
    pw(1 % NCH, x1 - K);
    pw(2 % NCH, x2 - K);
    pw(3 % NCH, x3 - K);
    const bool l01 = x0 < x1, l23 = x2 < x3;
    const double lo01 = l01 ? x0 : x1, hi01 = l01 ? x1 : x0;
    const double lo23 = l23 ? x2 : x3, hi23 = l23 ? x3 : x2;
    const double lo = lo01 < lo23 ? lo01 : lo23, hi = hi01 > hi23 ? hi01 : hi23;
    mn = lo < mn ? lo : mn;
    mx = hi > mx ? hi : mx;
  }
  __device__ __forceinline__ void one(double x) {
    pw(0, x - K);
    mn = x < mn ? x : mn;
    mx = x > mx ? x : mx;
  }
  __device__ __forceinline__ void sweep(const double* cg, int c, int sub, int opg, int G) {
    if (c <= sub) return;
    const size_t step = static_cast<size_t>(opg) * G;
    const double* p = cg + static_cast<size_t>(sub) * G;
    const int m = (c - sub + opg - 1) / opg;
    if (!kset) { K = p[0]; kset = true; }
    int i = 0;
    if (m >= 4) {
      double y0 = p[0], y1 = p[step], y2 = p[2 * step], y3 = p[3 * step];
      for (; i + 8 <= m; i += 4) {
        const double x0 = y0, x1 = y1, x2 = y2, x3 = y3;
        const double* q = p + static_cast<size_t>(i + 4) * step;
        y0 = q[0];
        y1 = q[step];
        y2 = q[2 * step];
        y3 = q[3 * step];
        quad(x0, x1, x2, x3);
      }
      quad(y0, y1, y2, y3);
      i += 4;
    }
    for (; i < m; ++i) one(p[static_cast<size_t>(i) * step]);
    nf += static_cast<unsigned long long>(m);
  }
  __device__ __forceinline__ void add1(double x) {
    if (!kset) { K = x; kset = true; }
    one(x);
    nf += 1;
  }
  __device__ __forceinline__ double sum_s1() const {
    double r = 0.0;
#pragma unroll
    for (int j = 0; j < NCH; ++j) r += s1[j];
    return r;
  }
  __device__ __forceinline__ double sum_s2() const {
    double r = 0.0;
#pragma unroll
    for (int j = 0; j < NCH; ++j) r += s2[j];
    return r;
  }
  __device__ __forceinline__ double sum_s3() const {
    double r = 0.0;
#pragma unroll
    for (int j = 0; j < NCH; ++j) r += s3[j];
    return r;
  }
  __device__ __forceinline__ double sum_s4() const {
    double r = 0.0;
#pragma unroll
    for (int j = 0; j < NCH; ++j) r += s4[j];
    return r;
  }
};

template <int NCH, bool M34>
using OwnerAccT = typename std::conditional<M34, OwnerAcc4<NCH>, OwnerAcc<NCH>>::type;

// GC > 0: an instantiation for exactly GC groups.  With the group count (and so the column
// capacity and the owners per group) known at compile time, the column address rank * G + key
// and the owners' column strides fold into shifts and immediate offsets: 10^9 rows over 256
// groups took 2.55 ms against 2.75 ms with the counts read from the arguments.
template <int MAXSLOTS, bool MASKED, bool TMA, bool M34, int GC = 0>
__global__ void __launch_bounds__(NT, 1) dense_moments_kernel(DenseArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x;
  const int G = GC ? GC : a.G, C = GC ? dense_cols(GC) : a.C;
  const int opg = GC ? dense_opg(GC) : a.opg;
  const int gp = (G + 3) & ~3;
  double* col0 = reinterpret_cast<double*>(smem + STAGES * STAGE_BYTES);
  double* col1 = col0 + static_cast<size_t>(C) * G;
  double* splv0 = col1 + static_cast<size_t>(C) * G;  // spill-list values [2][SPL]
  uint32_t* cnt0 = reinterpret_cast<uint32_t*>(splv0 + 2 * SPL);
  uint32_t* cnt1 = cnt0 + gp;
  int* splk0 = reinterpret_cast<int*>(cnt1 + gp);      // spill-list keys [2][SPL]
  // spill-list counts, one per batch modulo 4: batch k uses splc[k & 3]; the owners of
  // batch k clear splc[(k + 2) & 3], which batch k - 2 used and batch k + 2 will use
  uint32_t* splc = reinterpret_cast<uint32_t*>(splk0 + 2 * SPL);
  uint64_t* full = reinterpret_cast<uint64_t*>(splc + 4);  // [STAGES] tile landed
  uint64_t* empty = full + STAGES;                            // [STAGES] tile consumed
  uint64_t* colfull = empty + STAGES;                         // [2] column buffer written
  uint64_t* colempty = colfull + 2;                           // [2] column buffer swept
  volatile int* abort = reinterpret_cast<volatile int*>(colempty + 2);

  const long long ntiles = a.n / TILE;
  const int P = gridDim.x, b = blockIdx.x;
  long long t_begin = ntiles * b / P, t_end = ntiles * (b + 1) / P;
  if constexpr (MASKED) {
    // ranks among the live tiles: every CTA takes an equal share of the tiles that have a row
    if (a.live_bits) {
      const long long nl = a.live_pre[a.live_words];
      t_begin = nl * b / P;
      t_end = nl * (b + 1) / P;
    }
  }
  const long long mytiles = t_end - t_begin;
  const bool has_tail = (b == P - 1) && (a.n % TILE) != 0;
  const long long nbatch = mytiles + (has_tail ? 1 : 0);
  unsigned long long* sp = a.spill + static_cast<size_t>(b) * spill_fields<M34>() * G;

  // Unmasked staged launches: the first tiles' bulk copies leave before the rest of the setup
  // (the mbarriers first), so the ring fills while the counters and spill states are cleared.
  constexpr bool EARLY = TMA && !MASKED;
  if (EARLY && tid == PRODUCER_WARP * 32) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], SCATTER_WARPS); }
    mbar_fence_init();
    for (int s = 0; s < STAGES && s < mytiles; ++s) {
      unsigned char* st = smem + static_cast<size_t>(s) * STAGE_BYTES;
      mbar_arrive_expect_tx(&full[s], KEY_BYTES + VAL_BYTES);
      bulk_g2s(st, a.keys + (t_begin + s) * TILE, KEY_BYTES, &full[s]);
      bulk_g2s(st + KEY_BYTES, a.vals + (t_begin + s) * TILE, VAL_BYTES, &full[s]);
    }
  }
  for (int i = tid; i < 2 * gp; i += NT) cnt0[i] = 0;
  if (tid < 4) splc[tid] = 0;
  for (int g = tid; g < G; g += NT) {
    sp[SP_N * G + g] = 0;
    sp[SP_NINFP * G + g] = 0;
    sp[SP_NINFN * G + g] = 0;
    sp[SP_K * G + g] = K_UNSET;
    sp[SP_S1 * G + g] = 0;
    sp[SP_S2 * G + g] = 0;
    sp[SP_MN * G + g] = ~0ull;
    sp[SP_MX * G + g] = 0;
    if constexpr (M34) {
      sp[SP_S3 * G + g] = 0;
      sp[SP_S4 * G + g] = 0;
    }
  }
  if (tid == 0) {
    if (!EARLY)
      for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], SCATTER_WARPS); }
    for (int s = 0; s < 2; ++s) { mbar_init(&colfull[s], SCATTER_WARPS); mbar_init(&colempty[s], NOW / 32); }
    static_assert(TEAMS == 1, "one owner team sweeps both column buffers");
    *abort = 0;
    mbar_fence_init();
  }
  __syncthreads();

  const uint32_t tx_bytes = KEY_BYTES + VAL_BYTES + (MASKED ? MASK_BYTES : 0);
  auto issue = [&](int s, long long tile) {
    unsigned char* st = smem + static_cast<size_t>(s) * STAGE_BYTES;
    mbar_arrive_expect_tx(&full[s], tx_bytes);
    bulk_g2s(st, a.keys + tile * TILE, KEY_BYTES, &full[s]);
    bulk_g2s(st + KEY_BYTES, a.vals + tile * TILE, VAL_BYTES, &full[s]);
    if (MASKED) bulk_g2s(st + KEY_BYTES + VAL_BYTES, a.mask + tile * (TILE / 64), MASK_BYTES, &full[s]);
  };
  auto prefetch = [&](long long tile) {
    bulk_prefetch_l2(a.keys + tile * TILE, KEY_BYTES);
    bulk_prefetch_l2(a.vals + tile * TILE, VAL_BYTES);
    if (MASKED) bulk_prefetch_l2(a.mask + tile * (TILE / 64), MASK_BYTES);
  };

  const int warp = tid >> 5, lane = tid & 31;
  if (warp == PRODUCER_WARP) {
    // ------------------------------------------------------------ producer warp
    // Refills each stage as soon as all scatter warps released it, and keeps
    // PF_AHEAD further tiles streaming into L2.
    if constexpr (MASKED) {
      // With a live-tile list the producer issues (and prefetches) only tiles that have a
      // selected row: tiles whose mask words are all zero are never read.
      if (TMA && lane == 0 && a.live_bits) {
        LiveCursor ic, pc;
        ic.init(a.live_bits, a.live_pre, a.live_words, t_begin);
        pc.init(a.live_bits, a.live_pre, a.live_words, t_begin + (mytiles > STAGES ? STAGES : mytiles));
        long long issued = 0;
        for (int st = 0; st < STAGES && st < mytiles; ++st) issue(st, ic.next());
        issued = mytiles < STAGES ? mytiles : STAGES;
        for (long long j = STAGES; j < STAGES + PF_AHEAD && j < mytiles; ++j) prefetch(pc.next());
        bool failed = false;
        for (long long k = 0; k + STAGES < mytiles; ++k) {
          const int st = static_cast<int>(k % STAGES);
          if (!wait_or_abort(&empty[st], static_cast<uint32_t>((k / STAGES) & 1), a.err, abort)) {
            failed = true;
            *abort = 1;
            break;
          }
          fence_proxy_async_smem();
          issue(st, ic.next());
          ++issued;
          if (k + STAGES + PF_AHEAD < mytiles) prefetch(pc.next());
        }
        if (failed || *abort) {
          // leave no bulk copy in flight into this CTA's shared memory (bounded waits)
          for (long long j = issued - STAGES < 0 ? 0 : issued - STAGES; j < issued; ++j) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&full[j % STAGES], static_cast<uint32_t>((j / STAGES) & 1))) {
              if (globaltimer_ns() - t0 > 500000000ull) break;
            }
          }
        }
      } else if (TMA && lane == 0) {
        long long issued = 0;
        for (int s = 0; s < STAGES && s < mytiles; ++s) issue(s, t_begin + s);
        issued = mytiles < STAGES ? mytiles : STAGES;
        for (long long j = STAGES; j < STAGES + PF_AHEAD && j < mytiles; ++j) prefetch(t_begin + j);
        bool failed = false;
        for (long long k = 0; k + STAGES < mytiles; ++k) {
          const int st = static_cast<int>(k % STAGES);
          if (!wait_or_abort(&empty[st], static_cast<uint32_t>((k / STAGES) & 1), a.err, abort)) {
            failed = true;
            *abort = 1;
            break;
          }
          fence_proxy_async_smem();
          issue(st, t_begin + k + STAGES);
          ++issued;
          if (k + STAGES + PF_AHEAD < mytiles) prefetch(t_begin + k + STAGES + PF_AHEAD);
        }
        if (failed || *abort) {
          for (long long j = issued - STAGES < 0 ? 0 : issued - STAGES; j < issued; ++j) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&full[j % STAGES], static_cast<uint32_t>((j / STAGES) & 1))) {
              if (globaltimer_ns() - t0 > 500000000ull) break;
            }
          }
        }
      }
    } else if (TMA && lane == 0) {
      long long issued = 0;
      // the first STAGES tiles were issued before the setup (EARLY)
      issued = mytiles < STAGES ? mytiles : STAGES;
      for (long long j = STAGES; j < STAGES + PF_AHEAD && j < mytiles; ++j) prefetch(t_begin + j);
      bool failed = false;
      for (long long k = 0; k + STAGES < mytiles; ++k) {
        const int st = static_cast<int>(k % STAGES);
        if (!wait_or_abort(&empty[st], static_cast<uint32_t>((k / STAGES) & 1), a.err, abort)) {
          failed = true;
          *abort = 1;
          break;
        }
        fence_proxy_async_smem();
        issue(st, t_begin + k + STAGES);
        ++issued;
        if (k + STAGES + PF_AHEAD < mytiles) prefetch(t_begin + k + STAGES + PF_AHEAD);
      }
      if (failed || *abort) {
        // leave no bulk copy in flight into this CTA's shared memory (bounded waits)
        for (long long j = issued - STAGES < 0 ? 0 : issued - STAGES; j < issued; ++j) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[j % STAGES], static_cast<uint32_t>((j / STAGES) & 1))) {
            if (globaltimer_ns() - t0 > 500000000ull) break;
          }
        }
      }
    }
  } else if (warp < SCATTER_WARPS) {
    // ------------------------------------------------------------ scatter warps
    // Each warp runs independently: it signals stage release and column
    // completion with one mbarrier arrival per warp.  A thread's 16 rows of a tile
    // are handled four at a time (register budget of a 25-warp CTA).
    const int t = tid;
    LiveCursor sc;
    if constexpr (MASKED) {
      if (a.live_bits) sc.init(a.live_bits, a.live_pre, a.live_words, t_begin);
    }
    for (long long k = 0; k < nbatch; ++k) {
      const int bs = static_cast<int>(k & 1);
      double* col = bs ? col1 : col0;
      uint32_t* cnt = bs ? cnt1 : cnt0;
      double* splv = splv0 + bs * SPL;
      int* splk = splk0 + bs * SPL;
      bool ok = true;
      if (k >= 2) ok = wait_or_abort(&colempty[bs], static_cast<uint32_t>(((k >> 1) - 1) & 1), a.err, abort);
      const bool tail = k >= mytiles;
      long long row0 = tail ? ntiles * TILE : (t_begin + k) * TILE;
      if constexpr (MASKED) {
        if (a.live_bits && !tail) row0 = sc.next() * TILE;
      }
      const int s = static_cast<int>(k % STAGES);
      const bool staged = TMA && !tail;
      if (staged) ok = ok && wait_or_abort(&full[s], static_cast<uint32_t>((k / STAGES) & 1), a.err, abort);
      if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0) *abort = 1;
        break;
      }
      const unsigned char* st = smem + static_cast<size_t>(s) * STAGE_BYTES;
#pragma unroll
      for (int h = 0; h < RPS / 4; ++h) {
        constexpr int R = 4;
        int kk[R];
        double vv[R];
        uint32_t mb = 0;
        if (staged) {
#pragma unroll
          for (int cc = 0; cc < R / 2; ++cc) {
            const int c = 2 * h + cc;
            const int2 kp = reinterpret_cast<const int2*>(st)[c * NSC + t];
            const double2 vp = reinterpret_cast<const double2*>(st + KEY_BYTES)[c * NSC + t];
            kk[2 * cc] = kp.x; kk[2 * cc + 1] = kp.y;
            vv[2 * cc] = vp.x; vv[2 * cc + 1] = vp.y;
            if (MASKED) {
              const int r = c * CHUNK + 2 * t;
              const uint64_t w = reinterpret_cast<const uint64_t*>(st + KEY_BYTES + VAL_BYTES)[r >> 6];
              mb |= static_cast<uint32_t>((w >> (r & 63)) & 3ull) << (2 * cc);
            } else {
              mb |= 3u << (2 * cc);
            }
          }
        } else {
#pragma unroll
          for (int cc = 0; cc < R / 2; ++cc) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const long long r = row0 + (2 * h + cc) * CHUNK + 2 * t + j;
              if (r < a.n) {
                kk[2 * cc + j] = a.keys[r];
                vv[2 * cc + j] = a.vals[r];
                const bool m = MASKED ? ((a.mask[r >> 6] >> (r & 63)) & 1ull) != 0 : true;
                mb |= (m ? 1u : 0u) << (2 * cc + j);
              } else {
                kk[2 * cc + j] = 0;
                vv[2 * cc + j] = 0.0;
              }
            }
          }
        }
        // the stage's rows are in registers: release it to the producer
        if (h == RPS / 4 - 1) {
          __syncwarp();
          if (staged && lane == 0) mbar_arrive(&empty[s]);
        }
        // Fast path: every row of the warp is unmasked with an in-range key and a
        // finite non-zero value (one predicated compare chain per row, one vote).
        bool good = !MASKED || mb == 0xFu;
#pragma unroll
        for (int i = 0; i < R; ++i)
          good = good && static_cast<unsigned>(kk[i]) < static_cast<unsigned>(G) && fabs(vv[i]) > 0.0 &&
                 fabs(vv[i]) < pos_inf();
        const bool all_good = __all_sync(0xffffffffu, good);
        uint32_t over = 0, rare = 0;
        if (all_good) {
          uint32_t rk[R];
#pragma unroll
          for (int i = 0; i < R; ++i) rk[i] = atomicAdd(&cnt[kk[i]], 1u);
#pragma unroll
          for (int i = 0; i < R; ++i) {
            if (rk[i] < static_cast<uint32_t>(C)) col[static_cast<size_t>(rk[i]) * G + kk[i]] = vv[i];
            else over |= 1u << i;
          }
        } else {
          // general path: finite rows with an in-range key take the column; rows with
          // an out-of-range key, +-inf or a zero value also need the slow path below
          uint32_t fin = 0;
#pragma unroll
          for (int i = 0; i < R; ++i) {
            const double x = vv[i];
            const bool m = (mb >> i) & 1u;
            const bool inr = static_cast<unsigned>(kk[i]) < static_cast<unsigned>(G);
            const bool f = is_finite(x);
            fin |= static_cast<uint32_t>(m && inr && f) << i;
            rare |= static_cast<uint32_t>(m && !is_nan(x) && (!inr || !f || x == 0.0)) << i;
          }
          uint32_t rk[R];
#pragma unroll
          for (int i = 0; i < R; ++i) rk[i] = ((fin >> i) & 1u) ? atomicAdd(&cnt[kk[i]], 1u) : NO_RANK;
#pragma unroll
          for (int i = 0; i < R; ++i) {
            if (rk[i] < static_cast<uint32_t>(C)) col[static_cast<size_t>(rk[i]) * G + kk[i]] = vv[i];
            else if (rk[i] != NO_RANK) over |= 1u << i;
          }
        }
        if (rare | over) {
          for (int i = 0; i < R; ++i) {
            const int g = kk[i];
            const double x = vv[i];
            if ((over >> i) & 1u) {
              const uint32_t slot = atomicAdd(&splc[k & 3], 1u);
              if (slot < SPL) { splk[slot] = g; splv[slot] = x; }
              else spill_add<M34>(sp, G, g, x);
            }
            if (!((rare >> i) & 1u)) continue;
            if (static_cast<unsigned>(g) >= static_cast<unsigned>(G)) {
              atomicOr(a.err, KERR_KEY_RANGE);
            } else if (x == 0.0) {
              const long long r = row0 + (2 * h + (i >> 1)) * CHUNK + 2 * t + (i & 1);
              atomicMin(&a.zfirst[g], zero_code(a.row_offset + r, x));
            } else {
              atomicAdd(sp + (x > 0 ? SP_NINFP : SP_NINFN) * G + g, 1ull);
            }
          }
        }
      }
      // this warp's rows of tile k are in column buffer bs
      __syncwarp();
      if (lane == 0) mbar_arrive(&colfull[bs]);
    }
  } else {
    // ------------------------------------------------------------ owner warps
    const int team = (tid - NSC) / NOW;
    const int o = tid - NSC - team * NOW;  // owner index within the team
    constexpr int NCH = MAXSLOTS == 1 ? (M34 ? 2 : 4) : (MAXSLOTS == 2 && !M34 ? 2 : 1);
    OwnerAccT<NCH, M34> acc[MAXSLOTS];
    int og[MAXSLOTS], osub[MAXSLOTS];
#pragma unroll
    for (int q = 0; q < MAXSLOTS; ++q) {
      acc[q].init();
      const int slot = o + q * NOW;
      if (slot < a.slots) { osub[q] = slot / G; og[q] = slot - osub[q] * G; }
      else { og[q] = -1; osub[q] = 0; }
    }
    // With one owner per group (n_groups >= owner threads) each count has a single
    // reader and the owner warps run independently; otherwise the sub-owners of a
    // group meet at a named barrier before its count is reset.
    const bool shared_counts = opg > 1;
    for (long long k = team; k < nbatch; k += TEAMS) {
      const int bs = static_cast<int>(k & 1);
      const double* col = bs ? col1 : col0;
      uint32_t* cnt = bs ? cnt1 : cnt0;
      const double* splv = splv0 + bs * SPL;
      const int* splk = splk0 + bs * SPL;
      const bool ok = wait_or_abort(&colfull[bs], static_cast<uint32_t>((k >> 1) & 1), a.err, abort);
      int c[MAXSLOTS];
#pragma unroll
      for (int q = 0; q < MAXSLOTS; ++q) {
        const int g = og[q] < 0 ? 0 : og[q];
        const int v = static_cast<int>(cnt[g]);
        c[q] = v < C ? v : C;
      }
      const uint32_t ns = splc[k & 3];
      const int nspill = static_cast<int>(ns < SPL ? ns : SPL);
      if (shared_counts) {
        if (bar_red_or(BAR_OWNER + team, NOW, !ok || *abort)) {
          if (!ok) *abort = 1;
          break;
        }
      } else if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0) *abort = 1;
        break;
      }
#pragma unroll
      for (int q = 0; q < MAXSLOTS; ++q)
        if (og[q] >= 0 && osub[q] == 0) cnt[og[q]] = 0;
#pragma unroll
      for (int q = 0; q < MAXSLOTS; ++q)
        if (og[q] >= 0) acc[q].sweep(col + og[q], c[q], osub[q], opg, G);
      for (int e = 0; e < nspill; ++e) {  // rows that overflowed their column (rare)
        const int key = splk[e];
#pragma unroll
        for (int q = 0; q < MAXSLOTS; ++q)
          if (og[q] == key && osub[q] == 0) acc[q].add1(splv[e]);
      }
      if (o == 0) splc[(k + 2) & 3] = 0;
      // this warp is done with column buffer bs (and, when counts are shared,
      // every owner has read them before the first reset above)
      __syncwarp();
      if (lane == 0) mbar_arrive(&colempty[bs]);
    }
    // partial states of this CTA's owners
    const long long stride = static_cast<long long>(P) * TEAMS * a.slots;
#pragma unroll
    for (int q = 0; q < MAXSLOTS; ++q) {
      if (og[q] < 0) continue;
      const long long idx = (static_cast<long long>(b) * TEAMS + team) * a.slots + (o + q * NOW);
      const auto& A = acc[q];
      const double s1 = A.sum_s1(), s2 = A.sum_s2();
      double meanoff = 0.0, m2 = 0.0, m3 = 0.0, m4 = 0.0;
      if (A.nf > 0) {
        if constexpr (M34) {
          central_from_power(static_cast<double>(A.nf), s1, s2, A.sum_s3(), A.sum_s4(), &meanoff, &m2, &m3, &m4);
        } else {
          meanoff = s1 / static_cast<double>(A.nf);
          m2 = fmax(s2 - s1 * meanoff, 0.0);
        }
      }
      a.part[ST_NN * stride + idx] = static_cast<double>(A.nf);
      a.part[ST_NF * stride + idx] = static_cast<double>(A.nf);
      a.part[ST_K * stride + idx] = A.K;
      a.part[ST_SUMOFF * stride + idx] = s1;
      a.part[ST_MEANOFF * stride + idx] = meanoff;
      a.part[ST_M2 * stride + idx] = m2;
      a.part[ST_MIN * stride + idx] = A.mn;
      a.part[ST_MAX * stride + idx] = A.mx;
      if constexpr (M34) {
        a.part[ST_M3 * stride + idx] = m3;
        a.part[ST_M4 * stride + idx] = m4;
      }
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Folding the per-CTA partials (state helpers in gstate.cuh)
// ---------------------------------------------------------------------------

// The spill state of one CTA for group g as a mergeable state.
__device__ __forceinline__ GState spill_state(const unsigned long long* sp, int G, int g, bool m34) {
  GState s = gstate_empty();
  const unsigned long long n = sp[SP_N * G + g];
  const unsigned long long np = sp[SP_NINFP * G + g], nm = sp[SP_NINFN * G + g];
  s.nn = static_cast<double>(n + np + nm);
  if (n > 0) {
    s.nf = static_cast<double>(n);
    s.K = __longlong_as_double(static_cast<long long>(sp[SP_K * G + g]));
    s.sumoff = __longlong_as_double(static_cast<long long>(sp[SP_S1 * G + g]));
    central_from_power(s.nf, s.sumoff, __longlong_as_double(static_cast<long long>(sp[SP_S2 * G + g])),
                       m34 ? __longlong_as_double(static_cast<long long>(sp[SP_S3 * G + g])) : 0.0,
                       m34 ? __longlong_as_double(static_cast<long long>(sp[SP_S4 * G + g])) : 0.0, &s.meanoff, &s.m2,
                       &s.m3, &s.m4);
    s.mn = o2f(sp[SP_MN * G + g]);
    s.mx = o2f(sp[SP_MX * G + g]);
  }
  if (nm > 0) s.mn = neg_inf();
  if (np > 0) s.mx = pos_inf();
  if (n == 0 && nm == 0 && np > 0) s.mn = pos_inf();
  if (n == 0 && np == 0 && nm > 0) s.mx = neg_inf();
  return s;
}

// One warp per group: lane l folds partials l, l+32, ... (each CTA contributes
// TEAMS * opg owner partials and one spill partial), then a fixed shuffle tree
// folds the lanes.
// One block per group: every thread folds a few of the group's partial states (the CTAs' owner
// partials and spill states), warps shuffle, and the eight warp results fold as a three-level tree
// (a fixed order: the same bits every run).  Chains stay short because a merge has a long latency
// (its divisions): a warp per group, or a warp per slice of partials, walked chains of dozens of
// dependent merges and ran 2-4 times longer.
constexpr int FOLD_NT = 256;

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void __launch_bounds__(FOLD_NT) dense_fold_kernel(const double* __restrict__ part,
                                                             const unsigned long long* __restrict__ spill, int P,
                                                             int G, int opg,
                                                             const unsigned long long* __restrict__ zfirst,
                                                             tbgb_moments out, double* state_out, int m34,
                                                             PushArgs push) {
  __shared__ GState warp_state[FOLD_NT / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = blockIdx.x;
  if (g >= G) return;  // uniform over the block
  const int slots = G * opg;
  const long long stride = static_cast<long long>(P) * TEAMS * slots;
  const int per = TEAMS * opg + 1;
  const int nparts = P * per;
  GState A = gstate_empty();
  for (int i = threadIdx.x; i < nparts; i += FOLD_NT) {
    const int p = i / per, j = i - p * per;
    GState B;
    if (j < TEAMS * opg) {
      // partial of team j / opg, sub-owner j % opg
      const long long idx = static_cast<long long>(p) * TEAMS * slots + static_cast<long long>(j / opg) * slots +
                            static_cast<long long>(j % opg) * G + g;
      B.nn = part[ST_NN * stride + idx];
      B.nf = part[ST_NF * stride + idx];
      B.K = part[ST_K * stride + idx];
      B.sumoff = part[ST_SUMOFF * stride + idx];
      B.meanoff = part[ST_MEANOFF * stride + idx];
      B.m2 = part[ST_M2 * stride + idx];
      B.mn = part[ST_MIN * stride + idx];
      B.mx = part[ST_MAX * stride + idx];
      B.m3 = m34 ? part[ST_M3 * stride + idx] : 0.0;  // written only by the M34 kernels
      B.m4 = m34 ? part[ST_M4 * stride + idx] : 0.0;
      B.zf = ~0ull;
    } else {
      B = spill_state(spill + static_cast<size_t>(p) * (m34 ? SP_COUNT : SP_BASE) * G, G, g, m34 != 0);
    }
    gstate_fold(A, B);
  }
  for (int d = 1; d < 32; d <<= 1) {
    const GState B = gstate_shfl_down(A, d);
    if ((lane & (2 * d - 1)) == 0) gstate_fold(A, B);
  }
  if (lane == 0) warp_state[warp] = A;
  __syncthreads();
  for (int d = 1; d < FOLD_NT / 32; d <<= 1) {
    if (threadIdx.x < FOLD_NT / 32 && (threadIdx.x & (2 * d - 1)) == 0) gstate_fold(warp_state[threadIdx.x],
                                                                                   warp_state[threadIdx.x + d]);
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    A = warp_state[0];
    A.zf = zfirst[g];
    if (state_out) gstate_store(state_out, G, g, A);
    else gstate_finalize(A, g, out);
    warp_state[0] = A;
  }
  if (push.world > 0) {
    // the fused exchange: the group's state goes straight into this rank's slot of every peer
    // (plain stores over NVLink; thread q stores into peer q), then the last block to finish
    // raises this rank's flag in every buffer
    __syncthreads();
    if (threadIdx.x < push.world && threadIdx.x != push.rank) gstate_store(push.slot[threadIdx.x], G, g, warp_state[0]);
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned int done = atomicAdd(push.counter, 1u);
      if (done == static_cast<unsigned int>(gridDim.x) - 1u) {
        __threadfence_system();
        for (int q = 0; q < push.world; ++q) st_release_sys_u64(push.flag[q], push.epoch);
        *push.counter = 0u;  // the next step's fold (stream-ordered after this one) counts from zero
      }
    }
  }
}

// Fold R state tables (table r at states + r * ST_COUNT * G) in rank order.
__global__ void __launch_bounds__(256) merge_states_kernel(const double* __restrict__ states, int R, int G,
                                                            tbgb_moments out) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= G) return;
  GState A = gstate_empty();
  for (int r = 0; r < R; ++r) {
    const GState B = gstate_load(states + static_cast<size_t>(r) * ST_COUNT * G, G, g);
    gstate_fold(A, B);
  }
  gstate_finalize(A, g, out);
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------

template <int MAXSLOTS, bool MASKED, bool TMA, bool M34, int GC = 0>
static cudaError_t launch_main(const DenseLaunch& L, const DenseArgs& a, cudaStream_t stream) {
  auto kern = dense_moments_kernel<MAXSLOTS, MASKED, TMA, M34, GC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(L.smem));
  if (e != cudaSuccess) return e;
  kern<<<L.grid, NT, L.smem, stream>>>(a);
  return cudaGetLastError();
}

// Staged (TMA) launches of the common group counts run an instantiation for that count.
template <int MAXSLOTS, bool MASKED, bool M34>
static cudaError_t launch_staged(const DenseLaunch& L, const DenseArgs& a, cudaStream_t stream) {
  if constexpr (MAXSLOTS == 1) {
    if (a.G == 256) return launch_main<1, MASKED, true, M34, 256>(L, a, stream);
    if (a.G == 128) return launch_main<1, MASKED, true, M34, 128>(L, a, stream);
  } else if constexpr (MAXSLOTS == 2) {
    if (a.G == 512) return launch_main<2, MASKED, true, M34, 512>(L, a, stream);
  }
  return launch_main<MAXSLOTS, MASKED, true, M34>(L, a, stream);
}

template <int MAXSLOTS, bool M34>
static cudaError_t launch_slots(const DenseLaunch& L, const DenseArgs& a, bool masked, bool aligned,
                                cudaStream_t stream) {
  if (masked)
    return aligned ? launch_staged<MAXSLOTS, true, M34>(L, a, stream)
                   : launch_main<MAXSLOTS, true, false, M34>(L, a, stream);
  return aligned ? launch_staged<MAXSLOTS, false, M34>(L, a, stream)
                 : launch_main<MAXSLOTS, false, false, M34>(L, a, stream);
}

template <bool M34>
static cudaError_t launch_m(const DenseLaunch& L, const DenseArgs& a, bool masked, bool aligned, cudaStream_t stream) {
  if (L.maxslots == 1) return launch_slots<1, M34>(L, a, masked, aligned, stream);
  if (L.maxslots == 2) return launch_slots<2, M34>(L, a, masked, aligned, stream);
  return launch_slots<4, M34>(L, a, masked, aligned, stream);
}

constexpr int LT_NT = 256;
constexpr int LS_NT = 1024;

// Bit j of bits[w]: full tile 32w + j has a selected row; cnt[w] = popcount(bits[w]).
__global__ void __launch_bounds__(LT_NT) live_tiles_kernel(const uint64_t* __restrict__ mask, long long ntiles,
                                                           unsigned* bits, unsigned* cnt, long long nw) {
  const int lane = threadIdx.x & 31;
  const long long warp = (static_cast<long long>(blockIdx.x) * LT_NT + threadIdx.x) >> 5;
  const long long nwarps = static_cast<long long>(gridDim.x) * (LT_NT / 32);
  for (long long w = warp; w < nw; w += nwarps) {
    const long long t = w * 32 + lane;
    bool any = false;
    if (t < ntiles) {
      const uint64_t* mw = mask + t * (TILE / 64);
      uint64_t acc = 0;
#pragma unroll 8
      for (int i = 0; i < TILE / 64; ++i) acc |= __ldg(mw + i);
      any = acc != 0;
    }
    const unsigned bal = __ballot_sync(0xffffffffu, any);
    if (lane == 0) {
      bits[w] = bal;
      cnt[w] = static_cast<unsigned>(__popc(bal));
    }
  }
}

// pre[w] = cnt[0] + ... + cnt[w - 1] for w <= nw (one block).
__global__ void __launch_bounds__(LS_NT) live_scan_kernel(const unsigned* __restrict__ cnt, long long nw,
                                                          unsigned* pre) {
  __shared__ unsigned warp_sums[LS_NT / 32];
  __shared__ unsigned carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (long long base = 0; base < nw; base += LS_NT) {
    const long long i = base + threadIdx.x;
    const unsigned x = i < nw ? cnt[i] : 0u;
    unsigned inc = x;
    for (int d = 1; d < 32; d <<= 1) {
      const unsigned y = __shfl_up_sync(0xffffffffu, inc, d);
      if (lane >= d) inc += y;
    }
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    if (warp == 0) {
      unsigned ws = warp_sums[lane];
      for (int d = 1; d < 32; d <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, ws, d);
        if (lane >= d) ws += y;
      }
      warp_sums[lane] = ws;
    }
    __syncthreads();
    const unsigned before = carry + (warp > 0 ? warp_sums[warp - 1] : 0u) + inc - x;
    if (i < nw) pre[i] = before;
    __syncthreads();
    if (threadIdx.x == LS_NT - 1) carry = before + x;
    __syncthreads();
  }
  if (threadIdx.x == 0) pre[nw] = carry;
}

size_t dense_live_scratch_bytes(long long n) {
  const long long nw = (n / TILE + 31) / 32;
  return static_cast<size_t>(3 * nw + 1) * sizeof(unsigned);
}

cudaError_t dense_moments_launch(const DenseLaunch& L, const int32_t* keys, const double* vals, const uint64_t* mask,
                                 long long n, long long row_offset, int G, double* part, unsigned long long* spill,
                                 unsigned long long* zfirst, uint32_t* err, const tbgb_moments* out, double* state_out,
                                 cudaStream_t stream, uint64_t* launches, cudaEvent_t ev_start, cudaEvent_t ev_stop,
                                 unsigned* live_scratch, bool state_m34, const PushArgs* push) {
  DenseArgs a;
  a.keys = keys; a.vals = vals; a.mask = mask; a.n = n; a.row_offset = row_offset;
  a.G = G; a.C = L.C; a.opg = L.opg; a.slots = L.slots;
  a.part = part; a.spill = spill; a.zfirst = zfirst; a.err = err;
  a.live_bits = nullptr; a.live_pre = nullptr; a.live_words = 0;
  const bool aligned = (reinterpret_cast<uintptr_t>(keys) % 16 == 0) && (reinterpret_cast<uintptr_t>(vals) % 16 == 0) &&
                       (mask == nullptr || reinterpret_cast<uintptr_t>(mask) % 16 == 0);
  const bool masked = mask != nullptr;
  cudaError_t e;
  if (ev_start) cudaEventRecord(ev_start, stream);
  const long long ntiles = n / TILE;
  if (masked && aligned && live_scratch && ntiles > 0) {
    // list the tiles that have a selected row, so that the kernel never reads the others
    const long long nw = (ntiles + 31) / 32;
    unsigned* bits = live_scratch;
    unsigned* cnt = bits + nw;
    unsigned* pre = cnt + nw;
    long long blocks = (nw * 32 + LT_NT - 1) / LT_NT;
    const long long cap = static_cast<long long>(L.grid) * 8;
    if (blocks > cap) blocks = cap;
    live_tiles_kernel<<<static_cast<unsigned>(blocks), LT_NT, 0, stream>>>(mask, ntiles, bits, cnt, nw);
    live_scan_kernel<<<1, LS_NT, 0, stream>>>(cnt, nw, pre);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    *launches += 2;
    a.live_bits = bits;
    a.live_pre = pre;
    a.live_words = nw;
  }
  const bool m34 = (state_out != nullptr && state_m34) || (out && (out->m3 || out->m4));
  e = m34 ? launch_m<true>(L, a, masked, aligned, stream) : launch_m<false>(L, a, masked, aligned, stream);
  if (e != cudaSuccess) return e;
  if (ev_stop) cudaEventRecord(ev_stop, stream);
  (*launches)++;
  tbgb_moments o = out ? *out : tbgb_moments{};
  PushArgs pa{};
  if (push && state_out) pa = *push;
  dense_fold_kernel<<<G, FOLD_NT, 0, stream>>>(part, spill, L.grid, G, L.opg, zfirst, o, state_out, m34 ? 1 : 0,
                                               pa);
  e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

cudaError_t merge_states_launch(const double* states, int n_states, int G, const tbgb_moments* out, cudaStream_t stream,
                                uint64_t* launches) {
  merge_states_kernel<<<(G + 255) / 256, 256, 0, stream>>>(states, n_states, G, *out);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

}  // namespace tbgb
