// table.cu -- groupby through an accumulator table in device memory.
//
// Covers what the shared-memory column kernel (dense.cu) cannot: int64 keys of any
// value (an open-addressing hash table in HBM; the reference factorises keys on the
// host, group_index.rs:117-204, and accepts i32 codes only), dense keys with more
// than 1024 groups, f32 columns, and the filter / expression fused into the pass
// (filter_jit.rs:196-252 mask semantics, map_phi2 compute_engine.rs:198-210 and its
// CPU arithmetic :627-636, fused like scatter_jit.rs:402-495).
//
// Per group the table keeps non-NaN and finite row counts, a shift K (the first
// finite value that reached the slot), S1 = sum(v - K), S2 = sum((v - K)^2), the
// extrema as order-preserving u64 (so integer atomicMin / atomicMax apply) and the
// first zero row; the finaliser turns a slot into the same mergeable state and the
// same outputs as the dense kernel (gstate.cuh), so sum, mean and m2 follow
// descriptive.rs:383-435 and extrema the strict `<` / `>` scans of
// compute_engine.rs:304-322.
//
// Persistent CTAs of 1024 threads stream rows with coalesced evict-first loads, one
// row per thread per step (measured: more rows per thread, with their loads and first
// probes issued together, ran slower -- the larger body stalls on instruction fetch).
// Rows either update the global table with atomics, or -- for skewed keys -- first go to a
// per-CTA shared-memory table of a few thousand slots that absorbs the hot keys and
// is merged into the global table once at the end (shifted sums re-centred on the
// global slot's K).  Rows whose key is not admitted to the shared table (it is full)
// take the global path, so any key distribution is handled.
#include <cstdint>

#include "common.cuh"
#include "gstate.cuh"
#include "rowops.cuh"
#include "table.cuh"

namespace tbgb {

namespace {

constexpr int TNT = 1024;           // threads per CTA
constexpr int TR = 1;               // rows per thread per tile (more per thread measured slower: a larger body)
constexpr int TTILE = TNT * TR;     // rows per tile
constexpr int LS_FULL = 2048;       // shared-table slots with the FULL layout (64 B each)
constexpr int LS_SC = 4096;         // shared-table slots with the SUMCOUNT layout (20 B each)
constexpr int LPROBE = 8;           // shared-table probe limit
constexpr int kRangeSmemBytes = 225 * 1024;  // shared memory of one group range's table
constexpr int kMaxRanges = 8;       // more ranges: every CTA would read too many keys it drops
constexpr unsigned long long K_UNSET = 0x7FF8000000000001ull;  // NaN payload no finite value has

template <bool FULL>
__host__ __device__ constexpr int slot_words() { return FULL ? int(FL_WORDS) : int(SC_WORDS); }

// Assigns the output row of a newly inserted hash slot.
__device__ __forceinline__ void assign_id(const TableArgs& a, unsigned long long* p, int wid) {
  const unsigned long long id = atomicAdd(a.ngroups, 1ull);
  p[wid] = id;
  if (id >= static_cast<unsigned long long>(a.max_groups)) atomicOr(a.err, KERR_TABLE_FULL);
}

// Slot of `key` in the hash table, inserting it when absent; -1 when the probe
// limit is reached (reported as KERR_TABLE_FULL).  INT64_MIN, the free-slot
// marker, lives in the sentinel slot after the table, claimed through its ID word.
template <bool FULL>
__device__ __forceinline__ long long hash_slot_from(const TableArgs& a, unsigned long long key,
                                                    unsigned long long h, unsigned long long cur) {
  constexpr int W = slot_words<FULL>();
  constexpr int ID = FULL ? FL_ID : SC_ID;
  unsigned long long* T = a.table;
  if (key == kEmptyKey) {
    unsigned long long* p = T + a.slots * W;
    if (__ldcg(p + ID) == kNoId && atomicCAS(p + ID, kNoId, kNoId - 1) == kNoId) assign_id(a, p, ID);
    return static_cast<long long>(a.slots);
  }
  const unsigned long long m = a.slots - 1;
  for (int probe = 0; probe < kMaxProbe; ++probe) {
    if (probe > 0) cur = __ldcg(T + h * W);
    if (cur == key) return static_cast<long long>(h);
    if (cur == kEmptyKey) {
      const unsigned long long old = atomicCAS(T + h * W, kEmptyKey, key);
      if (old == kEmptyKey) {
        assign_id(a, T + h * W, ID);
        return static_cast<long long>(h);
      }
      if (old == key) return static_cast<long long>(h);
    }
    h = (h + 1) & m;
  }
  atomicOr(a.err, KERR_TABLE_FULL);
  return -1;
}

// K of a slot: the first finite value that reached it.
__device__ __forceinline__ double slot_shift(unsigned long long* kw, double v) {
  unsigned long long kb = __ldcg(kw);
  if (kb == K_UNSET) {
    kb = atomicCAS(kw, K_UNSET, dbits(v));
    if (kb == K_UNSET) kb = dbits(v);
  }
  return bitsd(kb);
}

// One non-NaN row into a global slot.
template <bool FULL>
__device__ __forceinline__ void global_row(unsigned long long* p, double v, long long grow, bool m34, bool extrema) {
  if constexpr (FULL) {
    atomicAdd(p + FL_NN, 1ull);
    if (is_finite(v)) {
      const double d = v - slot_shift(p + FL_K, v), dd = d * d;
      atomicAdd(reinterpret_cast<double*>(p + FL_S1), d);
      atomicAdd(reinterpret_cast<double*>(p + FL_S2), dd);
      if (m34) {
        atomicAdd(reinterpret_cast<double*>(p + FL_S3), dd * d);
        atomicAdd(reinterpret_cast<double*>(p + FL_S4), dd * dd);
      }
    } else {
      atomicAdd(p + FL_NI, 1ull);
    }
    if (extrema) {
      const unsigned long long o = f2o(v);
      if (o < __ldcg(p + FL_MN)) atomicMin(p + FL_MN, o);
      if (o > __ldcg(p + FL_MX)) atomicMax(p + FL_MX, o);
      if (v == 0.0) atomicMin(p + FL_ZF, zero_code(grow, v));
    }
  } else {
    atomicAdd(p + SC_NN, 1ull);
    if (is_finite(v)) atomicAdd(reinterpret_cast<double*>(p + SC_SUM), v);
  }
}

// Accumulators of a shared-memory table, one array entry per slot: the per-row update
// and the merge of a slot into a global slot.
template <bool FULL>
struct SlotArrays {
  unsigned long long* K;     // FULL
  double* s1;                // FULL: sum(v - K); SUMCOUNT: sum(v)
  double* s2;                // FULL
  double* s3;                // FULL: sum((v - K)^3)
  double* s4;                // FULL: sum((v - K)^4)
  unsigned long long* mn;    // FULL
  unsigned long long* mx;    // FULL
  unsigned long long* zf;    // FULL
  // FULL: non-NaN rows (low 32-bit word) and +-inf rows (high word); finite rows = the difference.
  // A row costs one 32-bit atomic (the high word only for the rare +-inf rows): 32-bit shared-memory
  // atomics run well ahead of 64-bit ones.
  unsigned long long* cnt;
  uint32_t* nn;              // SUMCOUNT: non-NaN rows

  __device__ __forceinline__ void clear(int s) {
    s1[s] = 0.0;
    if constexpr (!FULL) nn[s] = 0;
    if constexpr (FULL) {
      if (K) K[s] = K_UNSET;
      s2[s] = 0.0;
      if (s3) s3[s] = 0.0;
      if (s4) s4[s] = 0.0;
      if (mn) mn[s] = f2o(pos_inf());
      if (mx) mx[s] = f2o(neg_inf());
      if (zf) zf[s] = ~0ull;
      cnt[s] = 0;
    }
  }

  __device__ __forceinline__ void row(int s, double v, long long grow, bool m34, bool extrema) {
    if constexpr (FULL) {
      const bool fin = is_finite(v);
      atomicAdd(reinterpret_cast<unsigned int*>(cnt + s), 1u);
      if (!fin) atomicAdd(reinterpret_cast<unsigned int*>(cnt + s) + 1, 1u);
      if (fin) {
        unsigned long long kb = *reinterpret_cast<volatile unsigned long long*>(K + s);
        if (kb == K_UNSET) {
          kb = atomicCAS(K + s, K_UNSET, dbits(v));
          if (kb == K_UNSET) kb = dbits(v);
        }
        const double d = v - bitsd(kb), dd = d * d;
        atomicAdd(s1 + s, d);
        atomicAdd(s2 + s, dd);
        if (m34) {
          atomicAdd(s3 + s, dd * d);
          atomicAdd(s4 + s, dd * dd);
        }
      }
      if (extrema) {
        const unsigned long long o = f2o(v);
        if (o < *reinterpret_cast<volatile unsigned long long*>(mn + s)) atomicMin(mn + s, o);
        if (o > *reinterpret_cast<volatile unsigned long long*>(mx + s)) atomicMax(mx + s, o);
        if (v == 0.0) atomicMin(zf + s, zero_code(grow, v));
      }
    } else {
      atomicAdd(nn + s, 1u);
      if (is_finite(v)) atomicAdd(s1 + s, v);
    }
  }

  // Merges slot s into global slot p: power sums re-centred from the local shift K_l to
  // the global K_g, sum (d + off)^k with off = K_l - K_g.
  __device__ __forceinline__ void flush(int s, unsigned long long* p, bool m34, bool extrema) {
    if constexpr (FULL) {
      const unsigned long long n_nn = cnt[s] & 0xFFFFFFFFull, n_inf = cnt[s] >> 32, n_f = n_nn - n_inf;
      if (n_nn) atomicAdd(p + FL_NN, n_nn);
      if (n_inf) atomicAdd(p + FL_NI, n_inf);
      if (n_f) {
        const double Kl = bitsd(K[s]);
        const double Kg = slot_shift(p + FL_K, Kl);
        const double off = Kl - Kg, a1 = s1[s], a2 = s2[s], nfd = static_cast<double>(n_f);
        const double o2 = off * off;
        atomicAdd(reinterpret_cast<double*>(p + FL_S1), a1 + nfd * off);
        atomicAdd(reinterpret_cast<double*>(p + FL_S2), a2 + off * (2.0 * a1 + nfd * off));
        if (m34) {
          const double a3 = s3[s], a4 = s4[s];
          atomicAdd(reinterpret_cast<double*>(p + FL_S3), a3 + 3.0 * off * a2 + 3.0 * o2 * a1 + nfd * o2 * off);
          atomicAdd(reinterpret_cast<double*>(p + FL_S4),
                    a4 + 4.0 * off * a3 + 6.0 * o2 * a2 + 4.0 * o2 * off * a1 + nfd * o2 * o2);
        }
      }
      if (n_nn && extrema) {
        if (mn[s] < __ldcg(p + FL_MN)) atomicMin(p + FL_MN, mn[s]);
        if (mx[s] > __ldcg(p + FL_MX)) atomicMax(p + FL_MX, mx[s]);
        if (zf[s] != ~0ull) atomicMin(p + FL_ZF, zf[s]);
      }
    } else {
      if (nn[s]) {
        atomicAdd(p + SC_NN, static_cast<unsigned long long>(nn[s]));
        atomicAdd(reinterpret_cast<double*>(p + SC_SUM), s1[s]);
      }
    }
  }
};

// Per-CTA shared-memory hash table of a few thousand slots (LSV: slots, a power of two).
template <bool FULL, int LSV = (FULL ? LS_FULL : LS_SC)>
struct LocalTable : SlotArrays<FULL> {
  static constexpr int LS = LSV;
  static constexpr int LIMIT = LS * 3 / 4;  // admission stops at this fill
  unsigned long long* key;
  uint32_t* fill;

  static constexpr size_t bytes() {
    return FULL ? static_cast<size_t>(LS) * (10 * 8) + 16 : static_cast<size_t>(LS) * (2 * 8 + 4) + 16;
  }

  __device__ __forceinline__ void carve(unsigned char* sm) {
    unsigned char* q = sm;
    key = reinterpret_cast<unsigned long long*>(q); q += LS * 8;
    if constexpr (FULL) {
      this->K = reinterpret_cast<unsigned long long*>(q); q += LS * 8;
      this->s1 = reinterpret_cast<double*>(q); q += LS * 8;
      this->s2 = reinterpret_cast<double*>(q); q += LS * 8;
      this->s3 = reinterpret_cast<double*>(q); q += LS * 8;
      this->s4 = reinterpret_cast<double*>(q); q += LS * 8;
      this->mn = reinterpret_cast<unsigned long long*>(q); q += LS * 8;
      this->mx = reinterpret_cast<unsigned long long*>(q); q += LS * 8;
      this->zf = reinterpret_cast<unsigned long long*>(q); q += LS * 8;
      this->cnt = reinterpret_cast<unsigned long long*>(q); q += LS * 8;
    } else {
      this->s1 = reinterpret_cast<double*>(q); q += LS * 8;
      this->nn = reinterpret_cast<uint32_t*>(q); q += LS * 4;
    }
    fill = reinterpret_cast<uint32_t*>(q);
  }

  __device__ __forceinline__ void init(int tid) {
    for (int s = tid; s < LS; s += TNT) {
      key[s] = kEmptyKey;
      this->clear(s);
    }
    if (tid == 0) *fill = 0;
  }

  // Slot of `k` (inserted if there is room), or -1.
  __device__ __forceinline__ int find(unsigned long long k) {
    if (k == kEmptyKey) return -1;
    volatile unsigned long long* vk = key;
    unsigned int h = static_cast<unsigned int>(fmix64(k)) & (LS - 1);
    for (int probe = 0; probe < LPROBE; ++probe) {
      const unsigned long long cur = vk[h];
      if (cur == k) return static_cast<int>(h);
      if (cur == kEmptyKey) {
        if (*reinterpret_cast<volatile uint32_t*>(fill) >= static_cast<uint32_t>(LIMIT)) return -1;
        const unsigned long long old = atomicCAS(key + h, kEmptyKey, k);
        if (old == kEmptyKey) {
          atomicAdd(fill, 1u);
          return static_cast<int>(h);
        }
        if (old == k) return static_cast<int>(h);
      }
      h = (h + 1) & (LS - 1);
    }
    return -1;
  }
};

// M34 / EXT: the m3 / m4 sums and the extrema (with the first-zero code) are compiled in only
// where the call asks for them, which keeps the common bodies small (instruction fetch stalls
// dominated a body that carried every path).
template <bool KEY64, bool F32, bool FULL, bool LOCAL, bool M34, bool EXT>
__global__ void __launch_bounds__(TNT, 1) table_kernel(TableArgs a) {
  extern __shared__ __align__(16) unsigned char sm[];
  if (a.gate && *a.gate == 0u) return;
  // The rows: the call's columns, or one part of a partition (plain f64 values, no mask)
  // whose row count and first row are read from device memory.
  long long n = a.n;
  const char* keys = static_cast<const char*>(a.keys);
  const char* col_a = static_cast<const char*>(a.cols.a);
  if (a.dev_count) {
    const long long start = *a.dev_start;
    n = *a.dev_count;
    keys += start * (KEY64 ? 8 : 4);
    col_a += start * (F32 ? 4 : 8);
  }
  constexpr int W = slot_words<FULL>();
  const int tid = threadIdx.x;
  LocalTable<FULL> lt;
  if constexpr (LOCAL) {
    lt.carve(sm);
    lt.init(tid);
    __syncthreads();
  }
  const int expr = a.cols.expr, pred = a.cols.pred;
  const double thr = a.cols.threshold;
  const bool need_b = expr != TBGB_EXPR_A, need_c = expr == TBGB_EXPR_MUL_ADD;
  const uint64_t* mask = a.mask;
  unsigned long long* T = a.table;
  const unsigned long long hmask = a.slots - 1;

  // The row loads run one step ahead: the next step's key and columns are in flight while
  // this step's row probes and updates the table.
  const long long step = static_cast<long long>(gridDim.x) * TTILE;
  long long nk[TR];
  double na[TR], nb[TR], nc[TR];
  bool nin[TR];  // inside the rows and selected by the mask; other rows' columns are not read
  auto load_rows = [&](long long b0) {
#pragma unroll
    for (int r = 0; r < TR; ++r) {
      const long long row = b0 + r * TNT + tid;
      nk[r] = 0; na[r] = 0.0; nb[r] = 0.0; nc[r] = 0.0;
      nin[r] = row < n;
      if (nin[r] && mask) nin[r] = (__ldg(mask + (row >> 6)) >> (row & 63)) & 1ull;
      if (nin[r]) {
        nk[r] = load_key<KEY64>(keys, row);
        na[r] = load_val<F32>(col_a, row);
        if (need_b) nb[r] = load_val<F32>(a.cols.b, row);
        if (need_c) nc[r] = load_val<F32>(a.cols.c, row);
      }
    }
  };
  load_rows(static_cast<long long>(blockIdx.x) * TTILE);
  for (long long base = static_cast<long long>(blockIdx.x) * TTILE; base < n; base += step) {
    long long kk[TR];
    double va[TR], vb[TR], vc[TR];
    bool in[TR];
#pragma unroll
    for (int r = 0; r < TR; ++r) {
      kk[r] = nk[r]; va[r] = na[r]; vb[r] = nb[r]; vc[r] = nc[r]; in[r] = nin[r];
    }
    load_rows(base + step);
    // filter + expression; `live` rows have passed mask and predicate
    bool live[TR];
    double v[TR];
#pragma unroll
    for (int r = 0; r < TR; ++r) {
      bool ok = in[r];
      if (ok) ok = eval_pred(pred, va[r], thr);
      if (ok && !KEY64 && static_cast<unsigned long long>(kk[r]) >= a.slots) {
        atomicOr(a.err, KERR_KEY_RANGE);
        ok = false;
      }
      v[r] = eval_expr(expr, va[r], vb[r], vc[r]);
      // dense keys need no slot for NaN rows; hash keys still create their group
      if (!KEY64 && is_nan(v[r])) ok = false;
      live[r] = ok;
    }
    // shared-table admission
    int ls[TR];
#pragma unroll
    for (int r = 0; r < TR; ++r) {
      ls[r] = -1;
      if constexpr (LOCAL) {
        if (live[r]) ls[r] = lt.find(static_cast<unsigned long long>(kk[r]));
      }
    }
    // first probe of every global-path row, issued together
    unsigned long long hh[TR], cur[TR];
#pragma unroll
    for (int r = 0; r < TR; ++r) {
      hh[r] = 0; cur[r] = 0;
      if constexpr (KEY64) {
        if (live[r] && ls[r] < 0) {
          hh[r] = fmix64(static_cast<unsigned long long>(kk[r])) & hmask;
          if (static_cast<unsigned long long>(kk[r]) != kEmptyKey) cur[r] = __ldcg(T + hh[r] * W);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < TR; ++r) {
      if (!live[r]) continue;
      const long long grow = a.row_offset + base + r * TNT + tid;
      if constexpr (LOCAL) {
        if (ls[r] >= 0) {
          if (!is_nan(v[r])) lt.row(ls[r], v[r], grow, M34, EXT);
          continue;
        }
      }
      long long gs;
      if constexpr (KEY64) {
        gs = hash_slot_from<FULL>(a, static_cast<unsigned long long>(kk[r]), hh[r], cur[r]);
        if (gs < 0) continue;
      } else {
        gs = kk[r];
      }
      if (!is_nan(v[r]))
        global_row<FULL>(T + static_cast<unsigned long long>(gs) * W, v[r], grow, M34, EXT);
    }
  }

  if constexpr (LOCAL) {
    __syncthreads();
    for (int s = tid; s < LocalTable<FULL>::LS; s += TNT) {
      const unsigned long long k = lt.key[s];
      if (k == kEmptyKey) continue;
      long long gs;
      if constexpr (KEY64) {
        const unsigned long long h = fmix64(k) & hmask;
        gs = hash_slot_from<FULL>(a, k, h, __ldcg(T + h * W));
        if (gs < 0) continue;
      } else {
        gs = static_cast<long long>(k);
      }
      lt.flush(s, T + static_cast<unsigned long long>(gs) * W, M34, EXT);
    }
  }
}

// ---- int64 keys, shared-memory pre-aggregation with full warps ---------------------------
// table_kernel runs one row per lane: with a filter about half the lanes idle, and a warp whose
// lanes split between the shared table and the global one runs both paths one after the other
// (in the fused pipeline ncu counted 11 active lanes per warp instruction).  Here each warp
// queues its live rows in a shared-memory ring and takes them 32 at a time: every lane probes
// the shared table; rows it cannot take are queued again and go to the global table 32 at a
// time, with the first probe's key and shift words loaded together.  Extrema are not compiled
// in (table_kernel keeps that variant), so the slot arrays skip min / max / first-zero.
constexpr int QN = 64;  // ring entries per warp: fewer than 32 pending + 32 pushed

// Slots of the queued kernel's table: with the five FULL arrays (no m3 / m4) 4096 slots still
// fit beside the rings, which keeps more of a long-tailed key set in shared memory.
template <bool FULL, bool M34>
__host__ __device__ constexpr int queue_slots() { return FULL ? (M34 ? LS_FULL : 2 * LS_FULL) : LS_SC; }

template <bool FULL, bool M34>
__host__ __device__ constexpr size_t queue_table_bytes() {
  return FULL ? static_cast<size_t>(queue_slots<FULL, M34>()) * 8 * (M34 ? 7 : 5) + 16
              : static_cast<size_t>(queue_slots<FULL, M34>()) * 20 + 16;
}
constexpr size_t kQueueRingBytes = static_cast<size_t>(2) * (TNT / 32) * QN * 16;

template <bool FULL, int LSV>
__device__ __forceinline__ unsigned char* carve_queue_table(LocalTable<FULL, LSV>& lt, unsigned char* sm, bool m34) {
  constexpr int LS = LSV;
  unsigned char* q = sm;
  lt.key = reinterpret_cast<unsigned long long*>(q); q += LS * 8;
  if constexpr (FULL) {
    lt.K = reinterpret_cast<unsigned long long*>(q); q += LS * 8;
    lt.s1 = reinterpret_cast<double*>(q); q += LS * 8;
    lt.s2 = reinterpret_cast<double*>(q); q += LS * 8;
    lt.cnt = reinterpret_cast<unsigned long long*>(q); q += LS * 8;
    lt.s3 = lt.s4 = nullptr;
    if (m34) {
      lt.s3 = reinterpret_cast<double*>(q); q += LS * 8;
      lt.s4 = reinterpret_cast<double*>(q); q += LS * 8;
    }
    lt.mn = lt.mx = lt.zf = nullptr;
  } else {
    lt.s1 = reinterpret_cast<double*>(q); q += LS * 8;
    lt.nn = reinterpret_cast<uint32_t*>(q); q += LS * 4;
  }
  lt.fill = reinterpret_cast<uint32_t*>(q);
  return q + 16;
}

// One non-NaN row into global slot p; kb: the slot's shift word as loaded with the first probe
// (K_UNSET: not known, read it again).  The shift is set once, so a loaded value stays valid.
template <bool FULL, bool M34>
__device__ __forceinline__ void global_row_k(unsigned long long* p, double v, unsigned long long kb) {
  if constexpr (FULL) {
    atomicAdd(p + FL_NN, 1ull);
    if (is_finite(v)) {
      const double K = kb != K_UNSET ? bitsd(kb) : slot_shift(p + FL_K, v);
      const double d = v - K, dd = d * d;
      atomicAdd(reinterpret_cast<double*>(p + FL_S1), d);
      atomicAdd(reinterpret_cast<double*>(p + FL_S2), dd);
      if constexpr (M34) {
        atomicAdd(reinterpret_cast<double*>(p + FL_S3), dd * d);
        atomicAdd(reinterpret_cast<double*>(p + FL_S4), dd * dd);
      }
    } else {
      atomicAdd(p + FL_NI, 1ull);
    }
  } else {
    atomicAdd(p + SC_NN, 1ull);
    if (is_finite(v)) atomicAdd(reinterpret_cast<double*>(p + SC_SUM), v);
  }
}

template <bool F32, bool FULL, bool M34>
__global__ void __launch_bounds__(TNT, 1) table_queue_kernel(TableArgs a) {
  extern __shared__ __align__(16) unsigned char sm[];
  if (a.gate && *a.gate == 0u) return;
  constexpr int W = slot_words<FULL>();
  constexpr unsigned FULLMASK = 0xFFFFFFFFu;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned below = (1u << lane) - 1u;
  using LT = LocalTable<FULL, queue_slots<FULL, M34>()>;
  LT lt;
  unsigned char* rq = carve_queue_table(lt, sm, M34);
  rq += (16 - reinterpret_cast<uintptr_t>(rq) % 16) % 16;
  // this warp's rings: rows waiting for the shared table (lk / lv), rows for the global table (gk / gv)
  unsigned long long* lk = reinterpret_cast<unsigned long long*>(rq) + static_cast<size_t>(warp) * QN;
  double* lv = reinterpret_cast<double*>(rq) + static_cast<size_t>(TNT / 32 + warp) * QN;
  unsigned long long* gk = reinterpret_cast<unsigned long long*>(rq) + static_cast<size_t>(2 * (TNT / 32) + warp) * QN;
  double* gv = reinterpret_cast<double*>(rq) + static_cast<size_t>(3 * (TNT / 32) + warp) * QN;
  lt.init(tid);
  __syncthreads();

  const long long n = a.n;
  const char* keys = static_cast<const char*>(a.keys);
  const char* col_a = static_cast<const char*>(a.cols.a);
  const int expr = a.cols.expr, pred = a.cols.pred;
  const double thr = a.cols.threshold;
  const bool need_b = expr != TBGB_EXPR_A, need_c = expr == TBGB_EXPR_MUL_ADD;
  const uint64_t* mask = a.mask;
  unsigned long long* T = a.table;
  const unsigned long long hmask = a.slots - 1;
  unsigned lhead = 0, ltail = 0, ghead = 0, gtail = 0;  // ring positions (the same in every lane)

  auto push = [&](unsigned long long* rk, double* rv, unsigned& head, bool live, unsigned long long k, double v) {
    const unsigned bal = __ballot_sync(FULLMASK, live);
    if (live) {
      const unsigned i = (head + __popc(bal & below)) & (QN - 1);
      rk[i] = k;
      rv[i] = v;
    }
    head += __popc(bal);
    __syncwarp();
  };
  // cnt (<= 32) rows from the global ring: first probe with the key and shift words together
  auto global_batch = [&](unsigned cnt) {
    const bool act = static_cast<unsigned>(lane) < cnt;
    unsigned long long k = 0;
    double v = 0.0;
    if (act) {
      const unsigned i = (gtail + lane) & (QN - 1);
      k = gk[i];
      v = gv[i];
    }
    gtail += cnt;
    __syncwarp();
    if (act) {
      const unsigned long long h = fmix64(k) & hmask;
      unsigned long long cur = 0, kb = K_UNSET;
      if (k != kEmptyKey) {
        cur = __ldcg(T + h * W);
        if constexpr (FULL) kb = __ldcg(T + h * W + FL_K);
      }
      const long long gs = hash_slot_from<FULL>(a, k, h, cur);
      if (gs >= 0 && !is_nan(v)) {
        if (static_cast<unsigned long long>(gs) != h) kb = K_UNSET;
        global_row_k<FULL, M34>(T + static_cast<unsigned long long>(gs) * W, v, kb);
      }
    }
  };
  // cnt (<= 32) rows from the shared-table ring; the ones the table cannot take are queued again
  auto local_batch = [&](unsigned cnt) {
    const bool act = static_cast<unsigned>(lane) < cnt;
    unsigned long long k = 0;
    double v = 0.0;
    if (act) {
      const unsigned i = (ltail + lane) & (QN - 1);
      k = lk[i];
      v = lv[i];
    }
    ltail += cnt;
    __syncwarp();
    int ls = -1;
    if (act) ls = lt.find(k);
    bool mine = act && ls >= 0 && !is_nan(v);  // the lane updates the shared table itself
    if constexpr (FULL) {
      // Skewed keys put several lanes of a batch on one slot.  The largest such group is summed
      // across the warp first and applied once by its lowest lane, which takes those same-address
      // atomics (serialised within the instruction and across warps) off the hottest slots.
      const unsigned g = __match_any_sync(FULLMASK, mine ? ls : -1 - lane);
      const unsigned sz = mine ? static_cast<unsigned>(__popc(g)) : 0u;
      const unsigned best = __reduce_max_sync(FULLMASK, (sz << 5) | (31u - static_cast<unsigned>(lane)));
      if ((best >> 5) >= 2u) {
        const int bl = 31 - static_cast<int>(best & 31u);
        const unsigned bg = __shfl_sync(FULLMASK, g, bl);
        const int slot = __shfl_sync(FULLMASK, ls, bl);
        const bool in = (bg >> lane) & 1u;
        const bool fin = in && is_finite(v);
        const unsigned finm = __ballot_sync(FULLMASK, fin);
        const int leader = __ffs(bg) - 1;
        const double v0 = __shfl_sync(FULLMASK, v, finm ? __ffs(finm) - 1 : 0);
        unsigned long long kb = K_UNSET;
        if (lane == leader && finm) {  // the slot's shift, set by the group's first finite row when unset
          kb = *reinterpret_cast<volatile unsigned long long*>(lt.K + slot);
          if (kb == K_UNSET) {
            kb = atomicCAS(lt.K + slot, K_UNSET, dbits(v0));
            if (kb == K_UNSET) kb = dbits(v0);
          }
        }
        kb = __shfl_sync(FULLMASK, kb, leader);
        const double d = fin ? v - bitsd(kb) : 0.0, dd = d * d;
        double s1 = d, s2 = dd, s3 = 0.0, s4 = 0.0;
        if constexpr (M34) {
          s3 = dd * d;
          s4 = dd * dd;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          s1 += __shfl_xor_sync(FULLMASK, s1, off);
          s2 += __shfl_xor_sync(FULLMASK, s2, off);
          if constexpr (M34) {
            s3 += __shfl_xor_sync(FULLMASK, s3, off);
            s4 += __shfl_xor_sync(FULLMASK, s4, off);
          }
        }
        if (lane == leader) {
          unsigned int* c32 = reinterpret_cast<unsigned int*>(lt.cnt + slot);
          atomicAdd(c32, static_cast<unsigned>(__popc(bg)));
          const unsigned ninf = static_cast<unsigned>(__popc(bg & ~finm));
          if (ninf) atomicAdd(c32 + 1, ninf);
          if (finm) {
            atomicAdd(lt.s1 + slot, s1);
            atomicAdd(lt.s2 + slot, s2);
            if constexpr (M34) {
              atomicAdd(lt.s3 + slot, s3);
              atomicAdd(lt.s4 + slot, s4);
            }
          }
        }
        if (in) mine = false;
      }
    }
    if (mine) lt.row(ls, v, 0, M34, false);
    push(gk, gv, ghead, act && ls < 0, k, v);
    if (ghead - gtail >= 32u) global_batch(32u);
  };

  // Each thread takes a pair of adjacent rows per step (one 16-byte load per column when the
  // columns are 16-byte aligned); the loads run one step ahead, as in table_kernel.
  constexpr int QR = 2;
  const long long step = static_cast<long long>(gridDim.x) * TNT * QR;
  // (a row mask keeps the per-row loads: the columns of rows it drops are not read)
  const bool vec = !F32 && mask == nullptr && ((reinterpret_cast<uintptr_t>(keys) | reinterpret_cast<uintptr_t>(col_a) |
                             reinterpret_cast<uintptr_t>(need_b ? a.cols.b : nullptr) |
                             reinterpret_cast<uintptr_t>(need_c ? a.cols.c : nullptr)) & 15u) == 0;
  long long nk[QR];
  double na[QR], nb[QR], nc[QR];
  bool nin[QR];
  auto load_rows = [&](long long r0) {  // rows r0, r0 + 1
#pragma unroll
    for (int r = 0; r < QR; ++r) {
      nk[r] = 0; na[r] = 0.0; nb[r] = 0.0; nc[r] = 0.0;
      nin[r] = r0 + r < n;
    }
    if (vec && r0 + 1 < n) {
      const longlong2 k2 = __ldcs(reinterpret_cast<const longlong2*>(keys) + (r0 >> 1));
      const double2 a2 = __ldcs(reinterpret_cast<const double2*>(col_a) + (r0 >> 1));
      nk[0] = k2.x; nk[1] = k2.y; na[0] = a2.x; na[1] = a2.y;
      if (need_b) {
        const double2 b2 = __ldcs(reinterpret_cast<const double2*>(a.cols.b) + (r0 >> 1));
        nb[0] = b2.x; nb[1] = b2.y;
      }
      if (need_c) {
        const double2 c2 = __ldcs(reinterpret_cast<const double2*>(a.cols.c) + (r0 >> 1));
        nc[0] = c2.x; nc[1] = c2.y;
      }
    } else {
#pragma unroll
      for (int r = 0; r < QR; ++r) {
        if (nin[r] && mask) nin[r] = (__ldg(mask + ((r0 + r) >> 6)) >> ((r0 + r) & 63)) & 1ull;
        if (nin[r]) {
          nk[r] = load_key<true>(keys, r0 + r);
          na[r] = load_val<F32>(col_a, r0 + r);
          if (need_b) nb[r] = load_val<F32>(a.cols.b, r0 + r);
          if (need_c) nc[r] = load_val<F32>(a.cols.c, r0 + r);
        }
      }
    }
  };
  load_rows(static_cast<long long>(blockIdx.x) * TNT * QR + 2 * tid);
  for (long long base = static_cast<long long>(blockIdx.x) * TNT * QR; base < n; base += step) {
    long long k[QR];
    double va[QR], vb[QR], vc[QR];
    bool in[QR];
#pragma unroll
    for (int r = 0; r < QR; ++r) {
      k[r] = nk[r]; va[r] = na[r]; vb[r] = nb[r]; vc[r] = nc[r]; in[r] = nin[r];
    }
    load_rows(base + step + 2 * tid);
#pragma unroll
    for (int r = 0; r < QR; ++r) {
      const bool live = in[r] && eval_pred(pred, va[r], thr);
      push(lk, lv, lhead, live, static_cast<unsigned long long>(k[r]), eval_expr(expr, va[r], vb[r], vc[r]));
      if (lhead - ltail >= 32u) local_batch(32u);
    }
  }
  if (lhead != ltail) local_batch(lhead - ltail);
  while (ghead != gtail) global_batch(ghead - gtail < 32u ? ghead - gtail : 32u);

  __syncthreads();
  for (int s = tid; s < LT::LS; s += TNT) {
    const unsigned long long k = lt.key[s];
    if (k == kEmptyKey) continue;
    const unsigned long long h = fmix64(k) & hmask;
    const long long gs = hash_slot_from<FULL>(a, k, h, __ldcg(T + h * W));
    if (gs < 0) continue;
    lt.flush(s, T + static_cast<unsigned long long>(gs) * W, M34, false);
  }
}

// ---- dense keys: group ranges held whole in shared memory ---------------------------------
// The G groups are split into R ranges of at most Gr groups, each small enough for a
// shared-memory table indexed by key (no hashing, no admission limit).  CTA b owns range
// b % R and walks tiles b / R, b / R + P, ... (P = grid / R): the R CTAs that read one tile
// run side by side, so the tile crosses HBM about once and the other reads hit L2.  A CTA
// reads the keys of all its tiles and the value columns only around rows in its range;
// range 0 also takes rows whose key is outside [0, G), so that a selected one raises
// KERR_KEY_RANGE as in table_kernel.  At the end every CTA merges its slots into the global
// table (SlotArrays::flush), whose finaliser gives the outputs.
constexpr int RROWS = 4;              // rows per thread per step: one 16-byte key load
constexpr int RTILE = TNT * RROWS;    // rows per CTA per step

// Shared bytes of a group's slot.  GK (FULL only): the shift K and the first-zero code stay in
// the group's global slot (FL_K, FL_ZF), 16 bytes less a group in shared memory.
template <bool FULL>
__host__ __device__ constexpr int range_slot_bytes(bool m34, bool gk = false) {
  return FULL ? 8 * ((gk ? 5 : 7) + (m34 ? 2 : 0)) : 12;
}

template <bool FULL, bool GK>
__device__ __forceinline__ void range_carve(SlotArrays<FULL>& t, unsigned char* q, int Gr, bool m34) {
  if constexpr (FULL) {
    t.cnt = reinterpret_cast<unsigned long long*>(q); q += Gr * 8;
    t.K = nullptr;
    if (!GK) { t.K = reinterpret_cast<unsigned long long*>(q); q += Gr * 8; }
    t.s1 = reinterpret_cast<double*>(q); q += Gr * 8;
    t.s2 = reinterpret_cast<double*>(q); q += Gr * 8;
    t.mn = reinterpret_cast<unsigned long long*>(q); q += Gr * 8;
    t.mx = reinterpret_cast<unsigned long long*>(q); q += Gr * 8;
    t.zf = nullptr;
    if (!GK) { t.zf = reinterpret_cast<unsigned long long*>(q); q += Gr * 8; }
    t.s3 = nullptr;
    t.s4 = nullptr;
    if (m34) {
      t.s3 = reinterpret_cast<double*>(q); q += Gr * 8;
      t.s4 = reinterpret_cast<double*>(q);
    }
    t.nn = nullptr;
  } else {
    t.s1 = reinterpret_cast<double*>(q); q += Gr * 8;
    t.nn = reinterpret_cast<uint32_t*>(q);
  }
}

// Four consecutive values of a column starting at row0 (a multiple of four): one or two
// 16-byte loads when `vec` (the column 16-byte aligned, all four rows inside), else one
// load per selected row.
template <bool F32>
__device__ __forceinline__ void range_load4(const void* col, long long row0, bool vec, unsigned sel, double* v) {
  if (vec) {
    if constexpr (F32) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(col) + row0));
      v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    } else {
      const double2* p = reinterpret_cast<const double2*>(static_cast<const double*>(col) + row0);
      const double2 lo = __ldg(p), hi = __ldg(p + 1);
      v[0] = lo.x; v[1] = lo.y; v[2] = hi.x; v[3] = hi.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < RROWS; ++j) {
      v[j] = 0.0;
      if ((sel >> j) & 1u) {
        if constexpr (F32) v[j] = static_cast<double>(__ldg(static_cast<const float*>(col) + row0 + j));
        else v[j] = __ldg(static_cast<const double*>(col) + row0 + j);
      }
    }
  }
}

// Position of the n-th (0-based) set bit of m; m holds more than n set bits.
__device__ __forceinline__ int nth_set_bit(unsigned m, int n) {
  int r = 0;
  int c = __popc(m & 0xFFFFu);
  if (n >= c) { n -= c; m >>= 16; r += 16; }
  c = __popc(m & 0xFFu);
  if (n >= c) { n -= c; m >>= 8; r += 8; }
  c = __popc(m & 0xFu);
  if (n >= c) { n -= c; m >>= 4; r += 4; }
  c = __popc(m & 0x3u);
  if (n >= c) { n -= c; m >>= 2; r += 2; }
  if (n >= static_cast<int>(m & 1u)) r += 1;
  return r;
}

// GK slot update: the shared accumulators are sums about the global slot's K (p + FL_K, the
// first finite value that reached the group), and zeros go to the global first-zero code.
__device__ __forceinline__ void row_gk(SlotArrays<true>& t, int s, unsigned long long* p, double v, long long grow,
                                       bool m34, bool extrema) {
  const bool fin = is_finite(v);
  atomicAdd(reinterpret_cast<unsigned int*>(t.cnt + s), 1u);
  if (!fin) atomicAdd(reinterpret_cast<unsigned int*>(t.cnt + s) + 1, 1u);
  if (fin) {
    const double d = v - slot_shift(p + FL_K, v), dd = d * d;
    atomicAdd(t.s1 + s, d);
    atomicAdd(t.s2 + s, dd);
    if (m34) {
      atomicAdd(t.s3 + s, dd * d);
      atomicAdd(t.s4 + s, dd * dd);
    }
  }
  if (extrema) {
    const unsigned long long o = f2o(v);
    if (o < *reinterpret_cast<volatile unsigned long long*>(t.mn + s)) atomicMin(t.mn + s, o);
    if (o > *reinterpret_cast<volatile unsigned long long*>(t.mx + s)) atomicMax(t.mx + s, o);
    if (v == 0.0) atomicMin(p + FL_ZF, zero_code(grow, v));
  }
}

// GK merge of slot s into global slot p: the sums already share its K.
__device__ __forceinline__ void flush_gk(const SlotArrays<true>& t, int s, unsigned long long* p, bool m34,
                                         bool extrema) {
  const unsigned long long n_nn = t.cnt[s] & 0xFFFFFFFFull, n_inf = t.cnt[s] >> 32, n_f = n_nn - n_inf;
  if (n_nn) atomicAdd(p + FL_NN, n_nn);
  if (n_inf) atomicAdd(p + FL_NI, n_inf);
  if (n_f) {
    atomicAdd(reinterpret_cast<double*>(p + FL_S1), t.s1[s]);
    atomicAdd(reinterpret_cast<double*>(p + FL_S2), t.s2[s]);
    if (m34) {
      atomicAdd(reinterpret_cast<double*>(p + FL_S3), t.s3[s]);
      atomicAdd(reinterpret_cast<double*>(p + FL_S4), t.s4[s]);
    }
  }
  if (n_nn && extrema) {
    if (t.mn[s] < __ldcg(p + FL_MN)) atomicMin(p + FL_MN, t.mn[s]);
    if (t.mx[s] > __ldcg(p + FL_MX)) atomicMax(p + FL_MX, t.mx[s]);
  }
}

// One row the CTA took: predicate, key check, expression, NaN drop, then the slot update.
template <bool FULL, bool GK>
__device__ __forceinline__ void range_row(SlotArrays<FULL>& t, const TableArgs& a, int key, long long g0,
                                          unsigned long long uG, double av, double bv, double cv, long long row,
                                          bool m34, bool extrema) {
  if (!eval_pred(a.cols.pred, av, a.cols.threshold)) return;
  const unsigned long long k = static_cast<unsigned long long>(static_cast<long long>(key));
  if (k >= uG) {
    atomicOr(a.err, KERR_KEY_RANGE);
    return;
  }
  const double v = eval_expr(a.cols.expr, av, bv, cv);
  if (is_nan(v)) return;
  const int s = static_cast<int>(k - static_cast<unsigned long long>(g0));
  if constexpr (GK) row_gk(t, s, a.table + k * slot_words<true>(), v, a.row_offset + row, m34, extrema);
  else t.row(s, v, a.row_offset + row, m34, extrema);
}

template <bool F32>
__device__ __forceinline__ double range_load1(const void* col, long long row) {
  if constexpr (F32) return static_cast<double>(__ldg(static_cast<const float*>(col) + row));
  else return __ldg(static_cast<const double*>(col) + row);
}

// COMPACT (more than one range): a lane takes about 1 / R of its rows, so before the updates
// the warp gathers its selected rows onto consecutive lanes (ballots per row slot, the n-th
// set bit, key shuffles) and every lane then loads and updates one row per round.
template <bool F32, bool FULL, bool COMPACT, bool GK>
__global__ void __launch_bounds__(TNT, 1) range_table_kernel(TableArgs a, int R, int Gr, int vec_ok) {
  static_assert(FULL || !GK, "the global shift applies to FULL slots");
  extern __shared__ __align__(16) unsigned char sm[];
  constexpr int W = slot_words<FULL>();
  const int tid = threadIdx.x, lane = tid & 31;
  const int r = static_cast<int>(blockIdx.x % R);
  const long long P = gridDim.x / R, p = blockIdx.x / R;
  const long long G = static_cast<long long>(a.slots);
  const long long g0 = static_cast<long long>(r) * Gr;
  const long long left = G - g0;
  const int gr = left < Gr ? static_cast<int>(left) : Gr;
  const bool m34 = a.m34 != 0, extrema = a.extrema != 0;
  SlotArrays<FULL> t;
  range_carve<FULL, GK>(t, sm, Gr, m34);
  for (int s = tid; s < gr; s += TNT) t.clear(s);
  __syncthreads();

  const long long n = a.n;
  const int* keys = static_cast<const int*>(a.keys);
  const int expr = a.cols.expr;
  const bool need_b = expr != TBGB_EXPR_A, need_c = expr == TBGB_EXPR_MUL_ADD;
  const uint64_t* mask = a.mask;
  const unsigned long long ugr = static_cast<unsigned long long>(gr), uG = static_cast<unsigned long long>(G);

  for (long long base = p * RTILE; base < n; base += P * RTILE) {
    const long long row0 = base + static_cast<long long>(tid) * RROWS;
    if (!COMPACT && row0 >= n) continue;  // COMPACT: every lane stays for the warp's ballots
    const bool whole = row0 + RROWS <= n;
    const bool vec = vec_ok && whole;
    int kk[RROWS] = {0, 0, 0, 0};
    if (vec) {
      const int4 k4 = __ldg(reinterpret_cast<const int4*>(keys + row0));
      kk[0] = k4.x; kk[1] = k4.y; kk[2] = k4.z; kk[3] = k4.w;
    } else {
#pragma unroll
      for (int j = 0; j < RROWS; ++j)
        if (row0 + j < n) kk[j] = __ldg(keys + row0 + j);
    }
    unsigned sel = 0;  // bit j: row row0 + j is this CTA's
#pragma unroll
    for (int j = 0; j < RROWS; ++j) {
      const unsigned long long k = static_cast<unsigned long long>(static_cast<long long>(kk[j]));
      bool take = row0 + j < n && k - static_cast<unsigned long long>(g0) < ugr;
      if (r == 0 && row0 + j < n && k >= uG) take = true;
      sel |= static_cast<unsigned>(take) << j;
    }
    // the four rows share one mask word (row0 is a multiple of four)
    if (sel && mask) sel &= static_cast<unsigned>(__ldg(mask + (row0 >> 6)) >> (row0 & 63)) & 0xFu;
    if constexpr (COMPACT) {
      // selected rows in (slot j, lane) order; round q gives lane L the (q * 32 + L)-th
      unsigned bj[RROWS];
      int cum[RROWS + 1];
      cum[0] = 0;
#pragma unroll
      for (int j = 0; j < RROWS; ++j) {
        bj[j] = __ballot_sync(0xffffffffu, (sel >> j) & 1u);
        cum[j + 1] = cum[j] + __popc(bj[j]);
      }
      const long long wrow0 = row0 - static_cast<long long>(lane) * RROWS;  // the warp's first row
      for (int q = 0; q < cum[RROWS]; q += 32) {
        const int i = q + lane;
        const bool act = i < cum[RROWS];
        const int j = (i >= cum[1]) + (i >= cum[2]) + (i >= cum[3]);
        const unsigned m = j == 0 ? bj[0] : j == 1 ? bj[1] : j == 2 ? bj[2] : bj[3];
        const int src = act ? nth_set_bit(m, i - cum[j]) : lane;
        const int k0 = __shfl_sync(0xffffffffu, kk[0], src), k1 = __shfl_sync(0xffffffffu, kk[1], src);
        const int k2 = __shfl_sync(0xffffffffu, kk[2], src), k3 = __shfl_sync(0xffffffffu, kk[3], src);
        if (act) {
          const int key = j == 0 ? k0 : j == 1 ? k1 : j == 2 ? k2 : k3;
          const long long row = wrow0 + static_cast<long long>(src) * RROWS + j;
          const double av = range_load1<F32>(a.cols.a, row);
          const double bv = need_b ? range_load1<F32>(a.cols.b, row) : 0.0;
          const double cv = need_c ? range_load1<F32>(a.cols.c, row) : 0.0;
          range_row<FULL, GK>(t, a, key, g0, uG, av, bv, cv, row, m34, extrema);
        }
      }
    } else {
      if (!sel) continue;
      double va[RROWS], vb[RROWS] = {0.0, 0.0, 0.0, 0.0}, vc[RROWS] = {0.0, 0.0, 0.0, 0.0};
      range_load4<F32>(a.cols.a, row0, vec, sel, va);
      if (need_b) range_load4<F32>(a.cols.b, row0, vec, sel, vb);
      if (need_c) range_load4<F32>(a.cols.c, row0, vec, sel, vc);
#pragma unroll
      for (int j = 0; j < RROWS; ++j)
        if ((sel >> j) & 1u)
          range_row<FULL, GK>(t, a, kk[j], g0, uG, va[j], vb[j], vc[j], row0 + j, m34, extrema);
    }
  }

  __syncthreads();
  for (int s = tid; s < gr; s += TNT) {
    unsigned long long* p = a.table + static_cast<unsigned long long>(g0 + s) * W;
    if constexpr (GK) flush_gk(t, s, p, m34, extrema);
    else t.flush(s, p, m34, extrema);
  }
}

__global__ void table_init_kernel(unsigned long long* T, unsigned long long nslots, int full, const uint32_t* gate) {
  if (gate && *gate == 0u) return;
  const unsigned long long i0 = blockIdx.x * static_cast<unsigned long long>(blockDim.x) + threadIdx.x;
  const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
  if (full) {
    const unsigned long long mn0 = f2o(pos_inf()), mx0 = f2o(neg_inf());
    for (unsigned long long s = i0; s < nslots; s += stride) {
      ulonglong2* p = reinterpret_cast<ulonglong2*>(T + s * FL_WORDS);
      p[0] = make_ulonglong2(kEmptyKey, K_UNSET);  // KEY, K
      p[1] = make_ulonglong2(0ull, 0ull);          // NN, NI
      p[2] = make_ulonglong2(0ull, 0ull);          // S1, S2 (+0.0)
      p[3] = make_ulonglong2(mn0, mx0);            // MN, MX
      p[4] = make_ulonglong2(kNoId, ~0ull);        // ID, ZF
      p[5] = make_ulonglong2(0ull, 0ull);          // S3, S4
    }
  } else {
    for (unsigned long long s = i0; s < nslots; s += stride) {
      ulonglong2* p = reinterpret_cast<ulonglong2*>(T + s * SC_WORDS);
      p[0] = make_ulonglong2(kEmptyKey, 0ull);     // KEY, NN
      p[1] = make_ulonglong2(0ull, kNoId);         // SUM, ID
    }
  }
  if (i0 == 0) T[nslots * (full ? FL_WORDS : SC_WORDS)] = 0ull;  // distinct-key counter
}

// A FULL slot as a mergeable state.
__device__ __forceinline__ GState slot_state(const unsigned long long* p) {
  GState s = gstate_empty();
  s.nn = static_cast<double>(p[FL_NN]);
  const unsigned long long nf = p[FL_NN] - p[FL_NI];
  if (nf > 0) {
    s.nf = static_cast<double>(nf);
    s.K = bitsd(p[FL_K]);
    s.sumoff = bitsd(p[FL_S1]);
    central_from_power(s.nf, s.sumoff, bitsd(p[FL_S2]), bitsd(p[FL_S3]), bitsd(p[FL_S4]), &s.meanoff, &s.m2, &s.m3,
                       &s.m4);
  }
  s.mn = o2f(p[FL_MN]);
  s.mx = o2f(p[FL_MX]);
  s.zf = p[FL_ZF];
  return s;
}

__device__ __forceinline__ void sumcount_finalize(const unsigned long long* p, long long j, const tbgb_moments& o) {
  const double nn = static_cast<double>(p[SC_NN]);
  double sum = bitsd(p[SC_SUM]);
  if (sum == 0.0) sum = 0.0;
  if (o.count) o.count[j] = nn;
  if (o.sum) o.sum[j] = sum;
  if (o.mean) o.mean[j] = nn > 0 ? sum / nn : qnan();
}

__global__ void table_finalize_dense_kernel(const unsigned long long* __restrict__ T, long long G, int full,
                                            tbgb_moments out, double* state_out) {
  for (long long g = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; g < G;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    if (full) {
      const GState s = slot_state(T + g * FL_WORDS);
      if (state_out) gstate_store(state_out, G, g, s);
      else gstate_finalize(s, g, out);
    } else {
      sumcount_finalize(T + g * SC_WORDS, g, out);
    }
  }
}

// ---- compaction of a hash table's occupied slots, in slot order --------------------------
// Sub-tables of `slots` slots each are followed by their sentinel slot; the distinct-key
// counter follows the last.  Blocks of FIN_CHUNK slots count their occupied slots, one block
// scans the counts, then every block writes its groups contiguously from its offset (a
// ballot-ranked block scan per 256 slots), so the outputs are written in long runs.
constexpr int FIN_NT = 256;
constexpr int FIN_CHUNK = FIN_NT * 16;

__device__ __forceinline__ bool slot_occupied(const unsigned long long* T, unsigned long long i,
                                              unsigned long long slots, int W, int ID) {
  const unsigned long long* p = T + i * W;
  return (i % (slots + 1)) < slots ? p[0] != kEmptyKey : p[ID] != kNoId;
}

__global__ void __launch_bounds__(FIN_NT) table_occ_count_kernel(const unsigned long long* __restrict__ T,
                                                                 unsigned long long slots, unsigned long long total,
                                                                 int full, unsigned long long* counts,
                                                                 const uint32_t* gate) {
  if (gate && *gate == 0u) return;
  const int W = full ? FL_WORDS : SC_WORDS, ID = full ? FL_ID : SC_ID;
  const unsigned long long nchunks = (total + FIN_CHUNK - 1) / FIN_CHUNK;
  __shared__ unsigned int ws[FIN_NT / 32];
  for (unsigned long long chunk = blockIdx.x; chunk < nchunks; chunk += gridDim.x) {
    const unsigned long long i0 = chunk * FIN_CHUNK;
    unsigned int c = 0;
    for (int k = 0; k < FIN_CHUNK / FIN_NT; ++k) {
      const unsigned long long i = i0 + static_cast<unsigned long long>(k) * FIN_NT + threadIdx.x;
      if (i < total && slot_occupied(T, i, slots, W, ID)) ++c;
    }
    for (int o = 16; o > 0; o >>= 1) c += __shfl_down_sync(0xffffffffu, c, o);
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long t = 0;
      for (int w = 0; w < FIN_NT / 32; ++w) t += ws[w];
      counts[chunk] = t;
    }
    __syncthreads();
  }
}

// Exclusive scan of `len` counts in one block (in place); the total goes to *n_groups,
// clipped to max_groups.
__global__ void __launch_bounds__(1024) table_occ_scan_kernel(unsigned long long* counts, long long len,
                                                             long long max_groups, int64_t* n_groups,
                                                             const uint32_t* gate) {
  if (gate && *gate == 0u) return;
  __shared__ unsigned long long warp_sums[32];
  __shared__ unsigned long long carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (long long base = 0; base < len; base += 1024) {
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
      warp_sums[lane] = w;
    }
    __syncthreads();
    const unsigned long long before = carry + (warp > 0 ? warp_sums[warp - 1] : 0ull) + inc - x;
    if (i < len) counts[i] = before;
    __syncthreads();
    if (threadIdx.x == 1023) carry = before + x;
    __syncthreads();
  }
  if (threadIdx.x == 0)
    *n_groups = static_cast<int64_t>(carry < static_cast<unsigned long long>(max_groups) ? carry : max_groups);
}

__global__ void __launch_bounds__(FIN_NT) table_compact_kernel(const unsigned long long* __restrict__ T,
                                                               unsigned long long slots, unsigned long long total,
                                                               int full, const unsigned long long* __restrict__ offsets,
                                                               long long max_groups, int64_t* out_keys,
                                                               tbgb_moments out, const uint32_t* gate) {
  if (gate && *gate == 0u) return;
  const int W = full ? FL_WORDS : SC_WORDS, ID = full ? FL_ID : SC_ID;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ unsigned int wpre[FIN_NT / 32];
  const unsigned long long nchunks = (total + FIN_CHUNK - 1) / FIN_CHUNK;
  for (unsigned long long chunk = blockIdx.x; chunk < nchunks; chunk += gridDim.x) {
  unsigned long long pos = offsets[chunk];
  const unsigned long long i0 = chunk * FIN_CHUNK;
  for (int k = 0; k < FIN_CHUNK / FIN_NT; ++k) {
    const unsigned long long i = i0 + static_cast<unsigned long long>(k) * FIN_NT + threadIdx.x;
    const bool occ = i < total && slot_occupied(T, i, slots, W, ID);
    const unsigned bal = __ballot_sync(0xffffffffu, occ);
    if (lane == 0) wpre[warp] = __popc(bal);
    __syncthreads();
    unsigned int before = 0, all = 0;
    for (int w = 0; w < FIN_NT / 32; ++w) {
      const unsigned int c = wpre[w];
      before += w < warp ? c : 0u;
      all += c;
    }
    if (occ) {
      const unsigned long long j = pos + before + __popc(bal & ((1u << lane) - 1u));
      if (j < static_cast<unsigned long long>(max_groups)) {
        const unsigned long long* p = T + i * W;
        out_keys[j] = static_cast<int64_t>(p[0]);
        if (full) gstate_finalize(slot_state(p), static_cast<long long>(j), out);
        else sumcount_finalize(p, static_cast<long long>(j), out);
      }
    }
    pos += all;
    __syncthreads();
  }
  }
}

// ---- dense keys beyond the column kernel: rank and sweep with the state in shared memory ----
// For G > 512 dense groups (count / sum / mean / m2 / variances / extrema, optionally m3 / m4) of
// one column with an optional predicate.  The groups are split into R ranges of Gr groups whose
// state (packed counts, shift K, power sums, ordered min / max, first-zero code) lives in shared
// memory, structure of arrays; CTA b owns range b % R and walks 8192-row tiles b / R,
// b / R + P, ... (the R CTAs reading a tile run side by side: the keys cross HBM once).  Per tile:
//   rank   every row of the range takes its rank inside its group with one shared u32 atomic
//          and stores its value into column `rank` of a [C][Gr] buffer; rows ranked >= C, zeros
//          (the first-zero code needs the row) and +-inf rows update the state directly with
//          shared atomics (no owner runs meanwhile);
//   sweep  thread t owns groups t, t + 1024, ...: it folds the group's column entries into the
//          group's state with plain loads and stores, no atomics, and clears the rank counter.
// Two CTA barriers a tile.  The next tile's keys are loaded at the start of the rank phase and
// its values at its end, so both are in flight across the barriers and the sweep.  At the end
// the CTA merges its state into the global table (SlotArrays::flush).
constexpr int SW_TILE = 8192;             // rows per tile
constexpr int SW_RPT = SW_TILE / TNT;     // rows per thread per tile (two 16-byte key loads)
constexpr int SW_MAXC = 32;               // column depth cap
constexpr int SW_AHEAD = 3;               // tiles ahead of the current one prefetched into L2
constexpr size_t kSweepSmemBytes = 227 * 1024;

__host__ __device__ constexpr int sweep_state_bytes(bool m34) { return m34 ? 72 : 56; }

struct SweepPlan {
  int R;      // ranges
  int Gr;     // groups per range
  int C;      // column depth
  size_t smem;
};

// R ranges with at least two columns each (0 ranges: the shapes this kernel does not take).
// max_ranges 1 (the automatic choice): every CTA of a range reads all the keys of its tiles, so
// beyond one range the group-range table kernel, which reads fewer of them per row, measured
// faster (3,000 groups: 1.76 against 1.62 ms; 10,000: 4.04 against 2.75 ms), while one range with
// at least four columns beat it (1,000 groups: 1.08 against 2.03 ms; 2,000: 1.28 against 1.63).
SweepPlan sweep_plan(long long G, bool m34, int num_sms, int max_ranges, int min_cols) {
  SweepPlan S{};
  for (int R = 1; R <= max_ranges && R <= num_sms; ++R) {
    const long long Gr = (G + R - 1) / R;
    const long long per = static_cast<long long>(kSweepSmemBytes) / Gr - sweep_state_bytes(m34) - 4;
    const long long C = per / 8;
    if (C >= min_cols) {
      S.R = static_cast<int>((G + Gr - 1) / Gr);
      S.Gr = static_cast<int>(Gr);
      S.C = static_cast<int>(C < SW_MAXC ? C : SW_MAXC);
      S.smem = static_cast<size_t>(Gr) * (sweep_state_bytes(m34) + 4 + 8 * S.C) + 64;
      return S;
    }
  }
  return S;
}

template <bool F32, bool M34>
__global__ void __launch_bounds__(TNT, 1) sweep_table_kernel(TableArgs a, int R, int Gr, int C, int every) {
  extern __shared__ __align__(16) unsigned char sm[];
  if (a.gate && *a.gate == 0u) return;
  constexpr int W = slot_words<true>();
  const int tid = threadIdx.x;
  const int range = static_cast<int>(blockIdx.x) % R;
  const int P = static_cast<int>(gridDim.x) / R;
  const long long G = static_cast<long long>(a.slots);
  const long long g0 = static_cast<long long>(range) * Gr;
  const int Gq = static_cast<int>(G - g0 < Gr ? G - g0 : Gr);  // groups of this range
  // shared memory: state arrays, rank counters, columns
  SlotArrays<true> st{};
  unsigned char* q = sm;
  st.cnt = reinterpret_cast<unsigned long long*>(q); q += static_cast<size_t>(Gr) * 8;
  st.K = reinterpret_cast<unsigned long long*>(q); q += static_cast<size_t>(Gr) * 8;
  st.s1 = reinterpret_cast<double*>(q); q += static_cast<size_t>(Gr) * 8;
  st.s2 = reinterpret_cast<double*>(q); q += static_cast<size_t>(Gr) * 8;
  st.mn = reinterpret_cast<unsigned long long*>(q); q += static_cast<size_t>(Gr) * 8;
  st.mx = reinterpret_cast<unsigned long long*>(q); q += static_cast<size_t>(Gr) * 8;
  st.zf = reinterpret_cast<unsigned long long*>(q); q += static_cast<size_t>(Gr) * 8;
  st.s3 = st.s4 = nullptr;
  if constexpr (M34) {
    st.s3 = reinterpret_cast<double*>(q); q += static_cast<size_t>(Gr) * 8;
    st.s4 = reinterpret_cast<double*>(q); q += static_cast<size_t>(Gr) * 8;
  }
  double* col = reinterpret_cast<double*>(q); q += static_cast<size_t>(C) * Gr * 8;
  unsigned int* rk = reinterpret_cast<unsigned int*>(q);
  for (int j = tid; j < Gr; j += TNT) {
    st.clear(j);
    rk[j] = 0u;
  }
  __syncthreads();

  const long long n = a.n;
  const int* keys = static_cast<const int*>(a.keys);
  const uint64_t* mask = a.mask;
  const int pred = a.cols.pred;
  const double thr = a.cols.threshold;
  const long long ntiles = (n + SW_TILE - 1) / SW_TILE;
  const int ig0 = static_cast<int>(g0);
  const unsigned uGq = static_cast<unsigned>(Gq), uG = static_cast<unsigned>(G);
  // this thread's e-th row of a tile: two 4-row chunks 4096 rows apart (tile-relative, 32-bit)
  auto lrow = [&](int e) { return (e >> 2) * (TNT * 4) + 4 * tid + (e & 3); };
  auto tile_rows = [&](long long t) {
    return t < ntiles ? static_cast<int>(n - t * SW_TILE < SW_TILE ? n - t * SW_TILE : SW_TILE) : 0;
  };
  auto selected = [&](long long row) { return !mask || ((__ldg(mask + (row >> 6)) >> (row & 63)) & 1ull); };
  int ck[SW_RPT], nk[SW_RPT];
  double cv[SW_RPT], nv[SW_RPT];
  auto load_keys = [&](long long t, int* kk) {
    const int rows = tile_rows(t);
    const int* kt = keys + t * SW_TILE;
#pragma unroll
    for (int h = 0; h < SW_RPT / 4; ++h) {
      const int l0 = lrow(4 * h);
      if (l0 + 3 < rows) {
        const int4 k4 = __ldcs(reinterpret_cast<const int4*>(kt + l0));
        kk[4 * h] = k4.x; kk[4 * h + 1] = k4.y; kk[4 * h + 2] = k4.z; kk[4 * h + 3] = k4.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) kk[4 * h + e] = l0 + e < rows ? __ldcs(kt + l0 + e) : ig0 - 1;
      }
    }
  };
  // values of this range's rows (rows past the end carry key g0 - 1: outside every range's test)
  auto load_vals = [&](long long t, const int* kk, double* vv) {
#pragma unroll
    for (int e = 0; e < SW_RPT; ++e) {
      vv[e] = 0.0;
      if (static_cast<unsigned>(kk[e] - ig0) < uGq) {
        const long long row = t * SW_TILE + lrow(e);
        if (selected(row)) vv[e] = load_val<F32>(a.cols.a, row);
      }
    }
  };
  // bulk L2 prefetch of a later tile's keys and values (one thread; sizes rounded down to 16 bytes)
  const int vsz = F32 ? 4 : 8;
  const bool valign = (reinterpret_cast<uintptr_t>(a.cols.a) & 15u) == 0;
  auto prefetch = [&](long long t2) {
    if (tid == 0 && t2 < ntiles) {
      const long long r0 = t2 * SW_TILE;
      const long long rows = tile_rows(t2);
      const uint32_t kbytes = static_cast<uint32_t>((rows * 4) & ~15ll);
      if (kbytes) bulk_prefetch_l2(keys + r0, kbytes);
      const uint32_t vbytes = static_cast<uint32_t>((rows * vsz) & ~15ll);
      if (valign && vbytes) bulk_prefetch_l2(static_cast<const char*>(a.cols.a) + r0 * vsz, vbytes);
    }
  };
  long long tile = blockIdx.x / R;
  prefetch(tile + P);
  load_keys(tile, ck);
  load_vals(tile, ck, cv);
  int since = 0;  // tiles ranked since the last sweep
  for (; tile < ntiles; tile += P) {
    prefetch(tile + SW_AHEAD * P);
    load_keys(tile + P, nk);
    // ---- rank
#pragma unroll
    for (int e = 0; e < SW_RPT; ++e) {
      const unsigned j = static_cast<unsigned>(ck[e] - ig0);
      if (j >= uGq) {
        // a key outside [0, G) (range 0 checks): an error when the row is selected
        if (range == 0 && static_cast<unsigned>(ck[e]) >= uG && lrow(e) < tile_rows(tile)) {
          const long long row = tile * SW_TILE + lrow(e);
          if (selected(row) && eval_pred(pred, load_val<F32>(a.cols.a, row), thr)) atomicOr(a.err, KERR_KEY_RANGE);
        }
        continue;
      }
      const double v = cv[e];
      if (!eval_pred(pred, v, thr) || is_nan(v)) continue;
      if (mask && !selected(tile * SW_TILE + lrow(e))) continue;
      if (is_finite(v) && v != 0.0) {
        const unsigned r = atomicAdd(rk + j, 1u);
        if (r < static_cast<unsigned>(C)) {
          col[r * static_cast<unsigned>(Gr) + j] = v;
          continue;
        }
      }
      // overflow, zero or +-inf: straight into the state
      st.row(static_cast<int>(j), v, a.row_offset + tile * SW_TILE + lrow(e), M34, true);
    }
    load_vals(tile + P, nk, nv);
#pragma unroll
    for (int e = 0; e < SW_RPT; ++e) {
      ck[e] = nk[e];
      cv[e] = nv[e];
    }
    if (++since < every && tile + P < ntiles) continue;  // columns still have room: rank another tile first
    since = 0;
    __syncthreads();
    // ---- sweep
    for (int j = tid; j < Gq; j += TNT) {
      const unsigned cnt = rk[j];
      if (cnt == 0u) continue;
      rk[j] = 0u;
      const int m = cnt < static_cast<unsigned>(C) ? static_cast<int>(cnt) : C;
      unsigned long long kb = st.K[j];
      double s1 = st.s1[j], s2 = st.s2[j], s3 = 0.0, s4 = 0.0;
      if constexpr (M34) {
        s3 = st.s3[j];
        s4 = st.s4[j];
      }
      double mn = o2f(st.mn[j]), mx = o2f(st.mx[j]);
      if (kb == K_UNSET) kb = dbits(col[j]);
      const double K = bitsd(kb);
      for (int r = 0; r < m; ++r) {
        const double v = col[static_cast<size_t>(r) * Gr + j];
        const double d = v - K, dd = d * d;
        s1 += d;
        s2 += dd;
        if constexpr (M34) {
          s3 += dd * d;
          s4 += dd * dd;
        }
        mn = v < mn ? v : mn;  // finite, non-zero values: the numeric order is the ordered-bits order
        mx = v > mx ? v : mx;
      }
      st.K[j] = kb;
      st.s1[j] = s1;
      st.s2[j] = s2;
      if constexpr (M34) {
        st.s3[j] = s3;
        st.s4[j] = s4;
      }
      st.mn[j] = f2o(mn);
      st.mx[j] = f2o(mx);
      st.cnt[j] += static_cast<unsigned long long>(m);  // non-NaN rows, low word
    }
    __syncthreads();
  }
  // merge into the global table
  unsigned long long* T = a.table;
  for (int j = tid; j < Gq; j += TNT) st.flush(j, T + static_cast<unsigned long long>(g0 + j) * W, M34, true);
}

template <bool F32>
cudaError_t launch_sweep(const TablePlan& P, const TableArgs& a, cudaStream_t s) {
  auto k = a.m34 ? sweep_table_kernel<F32, true> : sweep_table_kernel<F32, false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(P.smem));
  if (e != cudaSuccess) return e;
  // tiles ranked between sweeps: the columns about half full on average for uniform keys
  // (rows ranked past the columns take the shared atomics instead)
  const long long G = static_cast<long long>(a.slots);
  long long every = static_cast<long long>(P.sweep_cols) * G / (2ll * SW_TILE);
  every = every < 1 ? 1 : (every > 8 ? 8 : every);
  k<<<P.grid, TNT, P.smem, s>>>(a, P.ranges, P.range_groups, P.sweep_cols, static_cast<int>(every));
  return cudaGetLastError();
}

template <bool F32, bool FULL>
cudaError_t launch_queue(const TablePlan& P, const TableArgs& a, cudaStream_t s) {
  const bool m34 = FULL && a.m34;
  auto k = m34 ? table_queue_kernel<F32, FULL, true> : table_queue_kernel<F32, FULL, false>;
  const size_t smem = (m34 ? queue_table_bytes<FULL, true>() : queue_table_bytes<FULL, false>()) + 16 + kQueueRingBytes;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  k<<<P.grid, TNT, smem, s>>>(a);
  return cudaGetLastError();
}

template <bool KEY64, bool F32, bool FULL, bool LOCAL>
cudaError_t launch_table(const TablePlan& P, const TableArgs& a, cudaStream_t s) {
  // int64 keys into a per-CTA shared table: the full-warp variant, unless extrema are asked for
  // or the rows are a partition's part (row count on the device)
  if constexpr (KEY64 && LOCAL) {
    if (!(FULL && a.extrema) && a.dev_count == nullptr) return launch_queue<F32, FULL>(P, a, s);
  }
  auto k = table_kernel<KEY64, F32, FULL, LOCAL, false, false>;
  if constexpr (FULL) {
    if (a.m34 && a.extrema) k = table_kernel<KEY64, F32, FULL, LOCAL, true, true>;
    else if (a.m34) k = table_kernel<KEY64, F32, FULL, LOCAL, true, false>;
    else if (a.extrema) k = table_kernel<KEY64, F32, FULL, LOCAL, false, true>;
  }
  if (P.smem > 0) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(P.smem));
    if (e != cudaSuccess) return e;
  }
  k<<<P.grid, P.block, P.smem, s>>>(a);
  return cudaGetLastError();
}

template <bool F32, bool FULL>
cudaError_t launch_range(const TablePlan& P, const TableArgs& a, int vec, cudaStream_t s) {
  auto k = P.ranges > 1 ? range_table_kernel<F32, FULL, true, false> : range_table_kernel<F32, FULL, false, false>;
  if constexpr (FULL) {
    if (P.range_gk)
      k = P.ranges > 1 ? range_table_kernel<F32, true, true, true> : range_table_kernel<F32, true, false, true>;
  }
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(P.smem));
  if (e != cudaSuccess) return e;
  k<<<P.grid, P.block, P.smem, s>>>(a, P.ranges, P.range_groups, vec);
  return cudaGetLastError();
}

template <bool KEY64, bool F32>
cudaError_t launch_table_kf(const TablePlan& P, const TableArgs& a, cudaStream_t s) {
  if (P.full)
    return P.local ? launch_table<KEY64, F32, true, true>(P, a, s) : launch_table<KEY64, F32, true, false>(P, a, s);
  return P.local ? launch_table<KEY64, F32, false, true>(P, a, s) : launch_table<KEY64, F32, false, false>(P, a, s);
}

unsigned long long next_pow2(unsigned long long x) {
  unsigned long long p = 1;
  while (p < x) p <<= 1;
  return p;
}

}  // namespace

size_t table_slot_words(bool full) { return full ? size_t(FL_WORDS) : size_t(SC_WORDS); }

TablePlan table_plan(bool hash, bool full, int mode, long long groups, int num_sms, int buckets, bool m34) {
  TablePlan P{};
  P.hash = hash;
  P.full = full;
  P.buckets = hash && buckets > 1 ? buckets : 1;
  const long long limit = full ? LocalTable<true>::LIMIT : LocalTable<false>::LIMIT;
  if (hash) {
    const unsigned long long want = static_cast<unsigned long long>(groups) * 2;
    const unsigned long long total = next_pow2(want < 1024 ? 1024 : want);
    P.slots = total / P.buckets >= 256 ? total / P.buckets : 256;
  } else {
    P.slots = static_cast<unsigned long long>(groups);
  }
  if (mode == 1) P.local = true;
  else if (mode == 2) P.local = false;
  else P.local = hash ? groups <= (1ll << 22) : groups <= limit;
  const unsigned long long words =
      static_cast<unsigned long long>(P.buckets) * (P.slots + (hash ? 1 : 0)) * table_slot_words(full) + 1;
  P.table_bytes = (words * 8 + 255) / 256 * 256;
  P.grid = num_sms;
  P.num_sms = num_sms;
  P.block = TNT;
  P.smem = P.local ? (full ? LocalTable<true>::bytes() : LocalTable<false>::bytes()) : 0;
  // dense keys, full moments: rank and sweep (mode 6, and the default where it fits)
  if (!hash && full && (mode == 0 || mode == 6)) {
    const SweepPlan S = mode == 6 ? sweep_plan(groups, m34, num_sms, kMaxRanges, 2) : sweep_plan(groups, m34, num_sms, 1, 4);
    if (S.R > 0) {
      P.local = false;
      P.ranges = S.R;
      P.range_groups = S.Gr;
      P.sweep_cols = S.C;
      P.grid = num_sms / S.R * S.R;
      P.smem = S.smem;
      return P;
    }
  }
  // dense keys: group ranges in shared memory (mode 4, and the default while R stays small)
  if (!hash && (mode == 0 || mode == 4)) {
    long long per = full ? range_slot_bytes<true>(m34) : range_slot_bytes<false>(m34);
    long long R0 = (groups + kRangeSmemBytes / per - 1) / (kRangeSmemBytes / per);
    bool gk = false;
    if (full) {  // the global shift when it saves a range
      const long long per_gk = range_slot_bytes<true>(m34, true);
      const long long R_gk = (groups + kRangeSmemBytes / per_gk - 1) / (kRangeSmemBytes / per_gk);
      if (R_gk < R0) {
        per = per_gk;
        R0 = R_gk;
        gk = true;
      }
    }
    if (R0 <= kMaxRanges && R0 <= num_sms) {
      const long long Gr = (groups + R0 - 1) / R0;
      const long long R = (groups + Gr - 1) / Gr;  // every range holds at least one group
      P.local = false;
      P.range_gk = gk;
      P.ranges = static_cast<int>(R);
      P.range_groups = static_cast<int>(Gr);
      P.grid = static_cast<int>(num_sms / R * R);
      P.smem = static_cast<size_t>(Gr * per);
    }
  }
  return P;
}

unsigned long long* table_bucket(const TablePlan& P, unsigned long long* table, int b) {
  return table + static_cast<unsigned long long>(b) * (P.slots + (P.hash ? 1 : 0)) * table_slot_words(P.full);
}

unsigned long long* table_counter(const TablePlan& P, unsigned long long* table) {
  return table_bucket(P, table, P.buckets);
}

cudaError_t table_init(const TablePlan& P, unsigned long long* table, cudaStream_t s, uint64_t* launches,
                       const uint32_t* gate) {
  const unsigned long long nslots = static_cast<unsigned long long>(P.buckets) * (P.slots + (P.hash ? 1 : 0));
  unsigned long long blocks = (nslots + 255) / 256;
  const unsigned long long cap = gate ? static_cast<unsigned long long>(P.grid > 0 ? P.grid : 148) * 16 : 65536ull;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  table_init_kernel<<<static_cast<unsigned int>(blocks), 256, 0, s>>>(table, nslots, P.full ? 1 : 0, gate);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

cudaError_t table_accumulate(const TablePlan& P, const TableArgs& a, cudaStream_t s, uint64_t* launches,
                             cudaEvent_t ev0, cudaEvent_t ev1) {
  if (a.n == 0 && !a.dev_count) return cudaSuccess;
  const bool f32 = a.cols.dtype == TBGB_F32;
  if (ev0) cudaEventRecord(ev0, s);
  cudaError_t e;
  if (P.sweep_cols > 0) {
    // rank and sweep: one column without expression, 16-byte aligned keys, packed 32-bit counts
    // per CTA that cannot wrap; other calls take the group-range kernel planned for them
    const bool ok = !a.dev_count && a.cols.expr == TBGB_EXPR_A && (reinterpret_cast<uintptr_t>(a.keys) & 15u) == 0 &&
                    a.n / (P.grid / P.ranges) + SW_TILE < (1ll << 32);
    if (ok) {
      e = f32 ? launch_sweep<true>(P, a, s) : launch_sweep<false>(P, a, s);
      if (e != cudaSuccess) return e;
      if (ev1) cudaEventRecord(ev1, s);
      (*launches)++;
      return cudaSuccess;
    }
    const TablePlan Q = table_plan(false, true, 4, static_cast<long long>(a.slots), P.num_sms, 1, a.m34 != 0);
    return table_accumulate(Q, a, s, launches, nullptr, ev1);
  }
  // group ranges: a CTA's packed 32-bit row counts must not wrap
  const bool range = P.ranges > 0 && !a.dev_count &&
                     a.n / (P.grid / P.ranges) + RTILE < (1ll << 32);
  if (P.ranges > 0 && !range) {
    TablePlan D = P;
    D.ranges = 0;
    D.smem = 0;
    D.grid = P.grid > 0 ? P.grid : 1;
    e = f32 ? launch_table_kf<false, true>(D, a, s) : launch_table_kf<false, false>(D, a, s);
  } else if (range) {
    const auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    const int expr = a.cols.expr;
    const int vec = al(a.keys) && al(a.cols.a) && (expr == TBGB_EXPR_A || al(a.cols.b)) &&
                    (expr != TBGB_EXPR_MUL_ADD || al(a.cols.c));
    if (P.full) e = f32 ? launch_range<true, true>(P, a, vec, s) : launch_range<false, true>(P, a, vec, s);
    else e = f32 ? launch_range<true, false>(P, a, vec, s) : launch_range<false, false>(P, a, vec, s);
  } else if (P.hash) e = f32 ? launch_table_kf<true, true>(P, a, s) : launch_table_kf<true, false>(P, a, s);
  else e = f32 ? launch_table_kf<false, true>(P, a, s) : launch_table_kf<false, false>(P, a, s);
  if (e != cudaSuccess) return e;
  if (ev1) cudaEventRecord(ev1, s);
  (*launches)++;
  return cudaSuccess;
}

cudaError_t table_finalize_dense(const TablePlan& P, const unsigned long long* table, long long G,
                                 const tbgb_moments* out, double* state_out, cudaStream_t s, uint64_t* launches) {
  long long blocks = (G + 255) / 256;
  if (blocks > 65536) blocks = 65536;
  tbgb_moments o = out ? *out : tbgb_moments{};
  table_finalize_dense_kernel<<<static_cast<unsigned int>(blocks), 256, 0, s>>>(table, G, P.full ? 1 : 0, o,
                                                                                 state_out);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

size_t table_finalize_scratch_bytes(const TablePlan& P) {
  const unsigned long long total = static_cast<unsigned long long>(P.buckets) * (P.slots + 1);
  return ((total + FIN_CHUNK - 1) / FIN_CHUNK * 8 + 255) / 256 * 256;
}

cudaError_t table_finalize_hash(const TablePlan& P, const unsigned long long* table, long long max_groups,
                                int64_t* out_keys, const tbgb_moments* out, int64_t* d_n_groups,
                                unsigned long long* scratch, cudaStream_t s, uint64_t* launches,
                                const uint32_t* gate) {
  const unsigned long long total = static_cast<unsigned long long>(P.buckets) * (P.slots + 1);
  const unsigned long long nblk = (total + FIN_CHUNK - 1) / FIN_CHUNK;
  const int full = P.full ? 1 : 0;
  // grid-stride over the chunks: a gated launch that finds its gate closed costs a few CTAs only
  const unsigned long long cap = static_cast<unsigned long long>(P.grid > 0 ? P.grid : 148) * 16;
  const unsigned int grid = static_cast<unsigned int>(nblk < cap ? nblk : cap);
  table_occ_count_kernel<<<grid, FIN_NT, 0, s>>>(table, P.slots, total, full, scratch, gate);
  table_occ_scan_kernel<<<1, 1024, 0, s>>>(scratch, static_cast<long long>(nblk), max_groups, d_n_groups, gate);
  table_compact_kernel<<<grid, FIN_NT, 0, s>>>(table, P.slots, total, full, scratch, max_groups, out_keys, *out,
                                               gate);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) *launches += 3;
  return e;
}

}  // namespace tbgb
