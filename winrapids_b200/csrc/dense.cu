// dense.cu -- dense-key groupby moments for low cardinality (n_groups <= 1024).
//
// Semantics: DescriptiveEngine::moments_grouped (crates/tambear/src/descriptive.rs:383-435)
// with the NaN mask of nan_mask_count (:591-603) and the extrema of
// scatter_extremum / extremum_grouped_nan_safe (compute_engine.rs:304-322,
// descriptive.rs:606-620).  One pass over the data instead of the reference's two:
// per (CTA, group owner) the kernel keeps the non-NaN count, finite count, shift
// K, S1 = sum(v-K), S2 = sum((v-K)^2), min and max; partial states are merged with
// Chan's formula (descriptive.rs:216-253, intermediates.rs:352-377) in a fixed
// order, so results do not depend on which CTA finishes first.
//
// Data path per CTA (one persistent 512-thread CTA per SM):
//   * TMA bulk copies (cp.async.bulk, mbarrier completion, no multicast) stage
//     2048-row tiles of keys, values and mask words into a 4-deep shared ring;
//   * every thread ranks its 4 rows inside their groups with a shared-memory u32
//     atomic and stores the value into column `rank` of a [C][n_groups] buffer;
//   * owner threads (n_groups * opg of them) sweep their group's column and update
//     register accumulators; rows ranked >= C go through further rounds of the
//     same buffer, so heavy key skew stays correct (only slower).
#include <cstdint>

#include "common.cuh"
#include "dense.cuh"

namespace tbgb {

constexpr int DT = kDenseThreads;
constexpr int TILE = kDenseTile;
constexpr int STAGES = kDenseStages;
constexpr int RPT = TILE / DT;  // rows per thread per tile
static_assert(RPT == 4, "thread -> row mapping assumes 4 rows per thread");

constexpr uint32_t KEY_BYTES = TILE * 4;
constexpr uint32_t VAL_BYTES = TILE * 8;
constexpr uint32_t MASK_BYTES = TILE / 8;
constexpr uint32_t STAGE_BYTES = KEY_BYTES + VAL_BYTES + MASK_BYTES;
static_assert(STAGE_BYTES % 16 == 0, "bulk copy sizes must be 16-byte multiples");
constexpr uint32_t NO_RANK = 0xFFFFFFFFu;

struct OwnerAcc {
  unsigned long long nn;  // non-NaN rows
  unsigned long long nf;  // finite rows
  double K, s1, s2, mn, mx;
  bool kset;
  __device__ __forceinline__ void init() {
    nn = 0; nf = 0; K = 0.0; s1 = 0.0; s2 = 0.0; mn = pos_inf(); mx = neg_inf(); kset = false;
  }
  __device__ __forceinline__ void add(double v) {
    nn += 1;
    if (is_finite(v)) {
      if (!kset) { K = v; kset = true; }
      const double d = v - K;
      s1 += d;
      s2 = fma(d, d, s2);
      nf += 1;
    }
    mn = fmin(mn, v);
    mx = fmax(mx, v);
  }
};

struct DenseArgs {
  const int32_t* keys;
  const double* vals;
  const uint64_t* mask;  // nullable (MASKED template flag)
  long long n;
  long long row_offset;  // global index of row 0 (zero-tie ordering across shards)
  int G, C, opg, slots;
  double* part;                // [ST_COUNT][gridDim.x * slots]
  unsigned long long* zfirst;  // [G], preset to ~0
  uint32_t* err;
};

size_t dense_smem_bytes(int G, int C) {
  const size_t gp = (static_cast<size_t>(G) + 3) & ~size_t(3);
  return static_cast<size_t>(STAGES) * STAGE_BYTES + static_cast<size_t>(C) * G * 8 + 2 * gp * 4 + STAGES * 8;
}

DenseLaunch dense_plan(int G, int num_sms) {
  DenseLaunch L{};
  L.grid = num_sms;
  int C = kDenseColBudget / G;
  if (C > TILE) C = TILE;
  if (C < 1) C = 1;
  L.C = C;
  L.opg = G >= DT ? 1 : DT / G;
  L.slots = G * L.opg;
  L.maxslots = (L.slots + DT - 1) / DT;
  L.smem = dense_smem_bytes(G, C);
  L.part_doubles = static_cast<size_t>(ST_COUNT) * L.grid * L.slots;
  return L;
}

template <int MAXSLOTS>
__device__ __forceinline__ void owner_sweep(const DenseArgs& a, const double* col, const uint32_t* cnt, int round,
                                            OwnerAcc (&acc)[MAXSLOTS], const int (&og)[MAXSLOTS],
                                            const int (&osub)[MAXSLOTS]) {
#pragma unroll
  for (int q = 0; q < MAXSLOTS; ++q) {
    const int g = og[q];
    if (g < 0) continue;
    int c = static_cast<int>(cnt[g]) - round * a.C;
    c = c < 0 ? 0 : (c > a.C ? a.C : c);
    const double* cg = col + g;
    int e = osub[q];
    // two independent loads in flight per iteration
    for (; e + a.opg < c; e += 2 * a.opg) {
      const double x0 = cg[static_cast<size_t>(e) * a.G];
      const double x1 = cg[static_cast<size_t>(e + a.opg) * a.G];
      acc[q].add(x0);
      acc[q].add(x1);
    }
    if (e < c) acc[q].add(cg[static_cast<size_t>(e) * a.G]);
  }
}

template <int MAXSLOTS, bool MASKED, bool TMA>
__global__ void __launch_bounds__(DT, 1) dense_moments_kernel(DenseArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x;
  const int G = a.G;
  const int gp = (G + 3) & ~3;
  double* col = reinterpret_cast<double*>(smem + STAGES * STAGE_BYTES);
  uint32_t* cnt = reinterpret_cast<uint32_t*>(col + static_cast<size_t>(a.C) * G);
  uint64_t* bars = reinterpret_cast<uint64_t*>(cnt + 2 * gp);

  const long long ntiles = a.n / TILE;
  const int P = gridDim.x, b = blockIdx.x;
  const long long t_begin = ntiles * b / P, t_end = ntiles * (b + 1) / P;
  const long long mytiles = t_end - t_begin;
  const bool has_tail = (b == P - 1) && (a.n % TILE) != 0;

  OwnerAcc acc[MAXSLOTS];
  int og[MAXSLOTS], osub[MAXSLOTS];
#pragma unroll
  for (int q = 0; q < MAXSLOTS; ++q) {
    acc[q].init();
    const int o = tid + q * DT;
    if (o < a.slots) { osub[q] = o / G; og[q] = o - osub[q] * G; }
    else { og[q] = -1; osub[q] = 0; }
  }
  for (int i = tid; i < 2 * gp; i += DT) cnt[i] = 0;

  const uint32_t tx_bytes = KEY_BYTES + VAL_BYTES + (MASKED ? MASK_BYTES : 0);
  auto issue = [&](int s, long long tile) {
    unsigned char* st = smem + static_cast<size_t>(s) * STAGE_BYTES;
    mbar_arrive_expect_tx(&bars[s], tx_bytes);
    bulk_g2s(st, a.keys + tile * TILE, KEY_BYTES, &bars[s]);
    bulk_g2s(st + KEY_BYTES, a.vals + tile * TILE, VAL_BYTES, &bars[s]);
    if (MASKED) bulk_g2s(st + KEY_BYTES + VAL_BYTES, a.mask + tile * (TILE / 64), MASK_BYTES, &bars[s]);
  };
  if (TMA && tid == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (TMA && tid == 0) {
    for (int s = 0; s < STAGES && s < mytiles; ++s) issue(s, t_begin + s);
  }

  int cb = 0;
  bool failed = false;
  long long li_fail = 0;
  // One tile: rank rows into the column buffer (round 0), barrier, owner sweep,
  // overflow rounds; ends with a barrier after which col/cnt[cb] may be reused.
  auto run_tile = [&](const int (&k)[RPT], const double (&v)[RPT], uint32_t mbits, long long row0, bool ok_in,
                      int stage_to_refill, long long refill_tile) -> bool {
    uint32_t* cur = cnt + cb * gp;
    uint32_t* nxt = cnt + (cb ^ 1) * gp;
    uint32_t rank[RPT];
    bool pend = false;
#pragma unroll
    for (int j = 0; j < RPT; ++j) {
      rank[j] = NO_RANK;
      const int g = k[j];
      const double x = v[j];
      bool ok = ok_in && ((mbits >> j) & 1u) && !is_nan(x);
      if (ok && static_cast<unsigned>(g) >= static_cast<unsigned>(G)) {
        atomicOr(a.err, KERR_KEY_RANGE);
        ok = false;
      }
      if (ok) {
        if (x == 0.0) atomicMin(&a.zfirst[g], zero_code(a.row_offset + row0 + j, x));
        const uint32_t r = atomicAdd(&cur[g], 1u);
        rank[j] = r;
        if (r < static_cast<uint32_t>(a.C)) col[static_cast<size_t>(r) * G + g] = x;
        else pend = true;
      }
    }
    // barrier A: tile consumed from the stage; columns and counts complete
    if (__syncthreads_or(!ok_in)) return false;
    if (TMA && tid == 0 && stage_to_refill >= 0) {
      fence_proxy_async_smem();
      issue(stage_to_refill, refill_tile);
    }
    for (int i = tid; i < G; i += DT) nxt[i] = 0;
    owner_sweep<MAXSLOTS>(a, col, cur, 0, acc, og, osub);
    int round = 0;
    // barrier B (and overflow rounds while any group exceeded C rows)
    while (__syncthreads_or(pend)) {
      ++round;
      const uint32_t lo = static_cast<uint32_t>(round) * a.C, hi = lo + a.C;
      pend = false;
#pragma unroll
      for (int j = 0; j < RPT; ++j) {
        if (rank[j] == NO_RANK || rank[j] < lo) continue;
        if (rank[j] < hi) col[static_cast<size_t>(rank[j] - lo) * G + k[j]] = v[j];
        else pend = true;
      }
      __syncthreads();
      owner_sweep<MAXSLOTS>(a, col, cur, round, acc, og, osub);
    }
    cb ^= 1;
    return true;
  };

  for (long long li = 0; li < mytiles && !failed; ++li) {
    const long long tile = t_begin + li;
    const long long row0 = tile * TILE + tid * RPT;
    int k[RPT];
    double v[RPT];
    uint32_t mbits = 0xFu;
    bool ok = true;
    int refill = -1;
    if (TMA) {
      const int s = static_cast<int>(li % STAGES);
      const uint32_t par = static_cast<uint32_t>((li / STAGES) & 1);
      ok = mbar_wait_bounded(&bars[s], par, a.err);
      const unsigned char* st = smem + static_cast<size_t>(s) * STAGE_BYTES;
      const int4 kk = reinterpret_cast<const int4*>(st)[tid];
      const double2 v0 = reinterpret_cast<const double2*>(st + KEY_BYTES)[2 * tid];
      const double2 v1 = reinterpret_cast<const double2*>(st + KEY_BYTES)[2 * tid + 1];
      k[0] = kk.x; k[1] = kk.y; k[2] = kk.z; k[3] = kk.w;
      v[0] = v0.x; v[1] = v0.y; v[2] = v1.x; v[3] = v1.y;
      if (MASKED) {
        const uint64_t w = reinterpret_cast<const uint64_t*>(st + KEY_BYTES + VAL_BYTES)[(tid * RPT) >> 6];
        mbits = static_cast<uint32_t>(w >> ((tid * RPT) & 63)) & 0xFu;
      }
      if (li + STAGES < mytiles) refill = s;
    } else {
#pragma unroll
      for (int j = 0; j < RPT; ++j) { k[j] = a.keys[row0 + j]; v[j] = a.vals[row0 + j]; }
      if (MASKED) {
        const uint64_t w = a.mask[row0 >> 6];
        mbits = static_cast<uint32_t>(w >> (row0 & 63)) & 0xFu;
      }
    }
    if (!run_tile(k, v, mbits, tile * TILE + tid * RPT, ok, refill, tile + STAGES)) {
      failed = true;
      li_fail = li;
    }
  }

  if (failed) {
    // A staged copy did not complete in time: wait (bounded) for the copies this
    // CTA may still have in flight, then leave; the host reports TBGB_ERR_TIMEOUT.
    if (TMA && tid == 0) {
      // tiles li_fail .. li_fail+STAGES-1 were issued and not consumed
      for (long long t = li_fail; t < li_fail + STAGES && t < mytiles; ++t) {
        const int s = static_cast<int>(t % STAGES);
        const uint32_t par = static_cast<uint32_t>((t / STAGES) & 1);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&bars[s], par)) {
          if (globaltimer_ns() - t0 > 500000000ull) break;
        }
      }
    }
    __syncthreads();
    return;
  }

  if (has_tail) {
    const long long tail0 = ntiles * TILE;
    const long long row0 = tail0 + tid * RPT;
    int k[RPT];
    double v[RPT];
    uint32_t mbits = 0;
#pragma unroll
    for (int j = 0; j < RPT; ++j) {
      const long long r = row0 + j;
      if (r < a.n) {
        k[j] = a.keys[r];
        v[j] = a.vals[r];
        const bool m = MASKED ? ((a.mask[r >> 6] >> (r & 63)) & 1ull) != 0 : true;
        mbits |= (m ? 1u : 0u) << j;
      } else {
        k[j] = 0;
        v[j] = 0.0;
      }
    }
    run_tile(k, v, mbits, row0, true, -1, 0);
  }

  // partial states of this CTA's owners
  const long long stride = static_cast<long long>(P) * a.slots;
#pragma unroll
  for (int q = 0; q < MAXSLOTS; ++q) {
    if (og[q] < 0) continue;
    const long long idx = static_cast<long long>(b) * a.slots + (tid + q * DT);
    const OwnerAcc& A = acc[q];
    double meanoff = 0.0, m2 = 0.0;
    if (A.nf > 0) {
      const double nf = static_cast<double>(A.nf);
      meanoff = A.s1 / nf;
      m2 = fmax(A.s2 - A.s1 * meanoff, 0.0);
    }
    a.part[ST_NN * stride + idx] = static_cast<double>(A.nn);
    a.part[ST_NF * stride + idx] = static_cast<double>(A.nf);
    a.part[ST_K * stride + idx] = A.K;
    a.part[ST_SUMOFF * stride + idx] = A.s1;
    a.part[ST_MEANOFF * stride + idx] = meanoff;
    a.part[ST_M2 * stride + idx] = m2;
    a.part[ST_MIN * stride + idx] = A.mn;
    a.part[ST_MAX * stride + idx] = A.mx;
  }
}

// ---------------------------------------------------------------------------
// State folding (Chan / parallel Welford) and finalisation
// ---------------------------------------------------------------------------

struct GState {
  double nn, nf, K, sumoff, meanoff, m2, mn, mx;
  unsigned long long zf;
};

__device__ __forceinline__ GState gstate_empty() {
  GState s;
  s.nn = 0; s.nf = 0; s.K = 0; s.sumoff = 0; s.meanoff = 0; s.m2 = 0;
  s.mn = pos_inf(); s.mx = neg_inf(); s.zf = ~0ull;
  return s;
}

// A <- A (+) B.  A holds the earlier rows.
__device__ __forceinline__ void gstate_fold(GState& A, const GState& B) {
  A.nn += B.nn;
  if (B.mn < A.mn) A.mn = B.mn;
  if (B.mx > A.mx) A.mx = B.mx;
  if (B.zf < A.zf) A.zf = B.zf;
  if (B.nf > 0) {
    if (A.nf == 0) {
      A.K = B.K; A.sumoff = B.sumoff; A.meanoff = B.meanoff; A.m2 = B.m2; A.nf = B.nf;
    } else {
      const double off = B.K - A.K;
      A.sumoff += B.nf * off + B.sumoff;
      const double cb = off + B.meanoff;
      const double n = A.nf + B.nf;
      const double delta = cb - A.meanoff;
      A.meanoff += delta * (B.nf / n);
      A.m2 += B.m2 + delta * delta * (A.nf * B.nf / n);
      A.nf = n;
    }
  }
}

__device__ __forceinline__ GState gstate_shfl_down(const GState& s, int d) {
  GState o;
  o.nn = __shfl_down_sync(0xffffffffu, s.nn, d);
  o.nf = __shfl_down_sync(0xffffffffu, s.nf, d);
  o.K = __shfl_down_sync(0xffffffffu, s.K, d);
  o.sumoff = __shfl_down_sync(0xffffffffu, s.sumoff, d);
  o.meanoff = __shfl_down_sync(0xffffffffu, s.meanoff, d);
  o.m2 = __shfl_down_sync(0xffffffffu, s.m2, d);
  o.mn = __shfl_down_sync(0xffffffffu, s.mn, d);
  o.mx = __shfl_down_sync(0xffffffffu, s.mx, d);
  o.zf = __shfl_down_sync(0xffffffffu, s.zf, d);
  return o;
}

__device__ __forceinline__ GState gstate_load(const double* st, long long stride, long long idx) {
  GState s;
  s.nn = st[ST_NN * stride + idx];
  s.nf = st[ST_NF * stride + idx];
  s.K = st[ST_K * stride + idx];
  s.sumoff = st[ST_SUMOFF * stride + idx];
  s.meanoff = st[ST_MEANOFF * stride + idx];
  s.m2 = st[ST_M2 * stride + idx];
  s.mn = st[ST_MIN * stride + idx];
  s.mx = st[ST_MAX * stride + idx];
  s.zf = static_cast<unsigned long long>(__double_as_longlong(st[ST_ZFIRST * stride + idx]));
  return s;
}

__device__ __forceinline__ void gstate_store(double* st, long long stride, long long idx, const GState& s) {
  st[ST_NN * stride + idx] = s.nn;
  st[ST_NF * stride + idx] = s.nf;
  st[ST_K * stride + idx] = s.K;
  st[ST_SUMOFF * stride + idx] = s.sumoff;
  st[ST_MEANOFF * stride + idx] = s.meanoff;
  st[ST_M2 * stride + idx] = s.m2;
  st[ST_MIN * stride + idx] = s.mn;
  st[ST_MAX * stride + idx] = s.mx;
  st[ST_ZFIRST * stride + idx] = __longlong_as_double(static_cast<long long>(s.zf));
}

// Outputs in the reference's semantics (descriptive.rs:97-114, 416-418).
__device__ __forceinline__ void gstate_finalize(const GState& A, int g, const tbgb_moments& o) {
  const double nn = A.nn;
  double sum = A.nf > 0 ? A.nf * A.K + A.sumoff : 0.0;
  if (sum == 0.0) sum = 0.0;  // the exact accumulator never yields -0.0 for an exact zero
  const double ref = nn > 0 ? sum / nn : 0.0;
  double m2 = 0.0;
  if (A.nf > 0) {
    const double dev = (A.K - ref) + A.meanoff;
    m2 = A.m2 + A.nf * dev * dev;
    if (m2 == 0.0) m2 = 0.0;
  }
  double mn = A.mn, mx = A.mx;
  if (nn > 0) {
    const double z = (A.zf & 1ull) ? -0.0 : 0.0;
    if (mn == 0.0) mn = z;
    if (mx == 0.0) mx = z;
  }
  if (o.count) o.count[g] = nn;
  if (o.sum) o.sum[g] = sum;
  if (o.min) o.min[g] = mn;
  if (o.max) o.max[g] = mx;
  if (o.mean) o.mean[g] = nn > 0 ? sum / nn : qnan();
  if (o.m2) o.m2[g] = m2;
  if (o.var_pop) o.var_pop[g] = nn > 0 ? m2 / nn : qnan();
  if (o.var_samp) o.var_samp[g] = nn - 1.0 > 0 ? m2 / (nn - 1.0) : qnan();
}

// One warp per group: lane l folds partials l, l+32, ... in order, then a fixed
// shuffle tree folds the lanes (lane order = row order of the partials).
__global__ void __launch_bounds__(256) dense_fold_kernel(const double* __restrict__ part, long long stride, int P,
                                                          int G, int opg, const unsigned long long* __restrict__ zfirst,
                                                          tbgb_moments out, double* state_out) {
  const int lane = threadIdx.x & 31;
  const int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (g >= G) return;
  const int slots = G * opg;
  const int nparts = P * opg;
  GState A = gstate_empty();
  for (int i = lane; i < nparts; i += 32) {
    const int p = i / opg, sub = i - (i / opg) * opg;
    const long long idx = static_cast<long long>(p) * slots + static_cast<long long>(sub) * G + g;
    GState B;
    B.nn = part[ST_NN * stride + idx];
    B.nf = part[ST_NF * stride + idx];
    B.K = part[ST_K * stride + idx];
    B.sumoff = part[ST_SUMOFF * stride + idx];
    B.meanoff = part[ST_MEANOFF * stride + idx];
    B.m2 = part[ST_M2 * stride + idx];
    B.mn = part[ST_MIN * stride + idx];
    B.mx = part[ST_MAX * stride + idx];
    B.zf = ~0ull;
    gstate_fold(A, B);
  }
  // lanes hold interleaved partials; fold them in lane order with a fixed tree
  for (int d = 1; d < 32; d <<= 1) {
    const GState B = gstate_shfl_down(A, d);
    if ((lane & (2 * d - 1)) == 0) gstate_fold(A, B);
  }
  if (lane == 0) {
    A.zf = zfirst[g];
    if (state_out) gstate_store(state_out, G, g, A);
    else gstate_finalize(A, g, out);
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

template <int MAXSLOTS, bool MASKED, bool TMA>
static cudaError_t launch_main(const DenseLaunch& L, const DenseArgs& a, cudaStream_t stream) {
  auto kern = dense_moments_kernel<MAXSLOTS, MASKED, TMA>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(L.smem));
  if (e != cudaSuccess) return e;
  kern<<<L.grid, DT, L.smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t dense_moments_launch(const DenseLaunch& L, const int32_t* keys, const double* vals, const uint64_t* mask,
                                 long long n, long long row_offset, int G, double* part, unsigned long long* zfirst,
                                 uint32_t* err, const tbgb_moments* out, double* state_out, cudaStream_t stream,
                                 uint64_t* launches, cudaEvent_t ev_start, cudaEvent_t ev_stop) {
  DenseArgs a;
  a.keys = keys; a.vals = vals; a.mask = mask; a.n = n; a.row_offset = row_offset;
  a.G = G; a.C = L.C; a.opg = L.opg; a.slots = L.slots;
  a.part = part; a.zfirst = zfirst; a.err = err;
  const bool aligned = (reinterpret_cast<uintptr_t>(keys) % 16 == 0) && (reinterpret_cast<uintptr_t>(vals) % 16 == 0) &&
                       (mask == nullptr || reinterpret_cast<uintptr_t>(mask) % 16 == 0);
  const bool masked = mask != nullptr;
  cudaError_t e;
  if (ev_start) cudaEventRecord(ev_start, stream);
  if (L.maxslots == 1) {
    if (masked) e = aligned ? launch_main<1, true, true>(L, a, stream) : launch_main<1, true, false>(L, a, stream);
    else e = aligned ? launch_main<1, false, true>(L, a, stream) : launch_main<1, false, false>(L, a, stream);
  } else {
    if (masked) e = aligned ? launch_main<2, true, true>(L, a, stream) : launch_main<2, true, false>(L, a, stream);
    else e = aligned ? launch_main<2, false, true>(L, a, stream) : launch_main<2, false, false>(L, a, stream);
  }
  if (e != cudaSuccess) return e;
  if (ev_stop) cudaEventRecord(ev_stop, stream);
  (*launches)++;
  tbgb_moments o = out ? *out : tbgb_moments{};
  const long long stride = static_cast<long long>(L.grid) * L.slots;
  const int blocks = (G * 32 + 255) / 256;
  dense_fold_kernel<<<blocks, 256, 0, stream>>>(part, stride, L.grid, G, L.opg, zfirst, o, state_out);
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
