// api.cpp -- C ABI of the groupby path (include/tambear_gb.h).
#include <cuda_runtime.h>

#include <climits>
#include <cstdio>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "bin_stats.cuh"
#include "dense.cuh"
#include "exchange.cuh"
#include "errbits.hpp"
#include "gen.cuh"
#include "group_index.cuh"
#include "mask.cuh"
#include "partition.cuh"
#include "phi.cuh"
#include "radix.cuh"
#include "table.cuh"
#include "tambear_gb.h"

struct tbgb_ctx {
  int device = 0;
  int num_sms = 0;
  std::string name;
  std::string last_error;
  void* ws = nullptr;  // workspace: partial states, zero trackers
  size_t ws_bytes = 0;
  void* ws_mask = nullptr;  // row mask of a predicate evaluated ahead of the column kernel
  size_t ws_mask_bytes = 0;
  uint32_t* err = nullptr;  // deferred kernel error bits (persist until tbgb_sync)
  uint64_t launches = 0;
  int table_mode = 0;    // tbgb_set_table_mode
  bool profile = false;  // record events around main kernels
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> events;
  const uint32_t* radix_gate = nullptr;  // fallback word of the last radix call (inside ws)
};

namespace {

// Makes ctx->device current for the duration of an entry point.
struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

tbgb_status fail(tbgb_ctx* ctx, tbgb_status st, const std::string& msg) {
  if (ctx) ctx->last_error = msg;
  return st;
}

tbgb_status cuda_fail(tbgb_ctx* ctx, tbgb_status st, const char* what, cudaError_t e) {
  return fail(ctx, st, std::string(what) + ": " + cudaGetErrorString(e));
}

tbgb_status ensure_ws(tbgb_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->ws_bytes) return TBGB_OK;
  if (ctx->ws) {
    cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
  }
  const size_t extra = bytes / 4 < (size_t(256) << 20) ? bytes / 4 : (size_t(256) << 20);  // room to grow
  size_t want = bytes + extra;
  cudaError_t e = cudaMalloc(&ctx->ws, want);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_ALLOC, "workspace allocation", e);
  ctx->ws_bytes = want;
  return TBGB_OK;
}

tbgb_status ensure_ws_mask(tbgb_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->ws_mask_bytes) return TBGB_OK;
  if (ctx->ws_mask) {
    cudaFree(ctx->ws_mask);
    ctx->ws_mask = nullptr;
    ctx->ws_mask_bytes = 0;
  }
  const size_t want = (bytes + bytes / 4 + 255) / 256 * 256;
  cudaError_t e = cudaMalloc(&ctx->ws_mask, want);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_ALLOC, "mask workspace allocation", e);
  ctx->ws_mask_bytes = want;
  return TBGB_OK;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// A device pointer the kernels read as `bytes`-wide elements must be aligned to them.
bool misaligned(const void* p, size_t bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) != 0; }

struct DenseWs {
  double* part;
  unsigned long long* spill;
  unsigned long long* zfirst;
  unsigned* live;  // live-tile list of a masked launch
  size_t bytes;
};

DenseWs dense_ws_layout(void* base, const tbgb::DenseLaunch& L, int G, int64_t n_masked = 0) {
  DenseWs w{};
  const size_t part_bytes = align_up(L.part_doubles * 8, 256);
  const size_t spill_bytes = align_up(L.spill_words * 8, 256);
  const size_t zf_bytes = align_up(static_cast<size_t>(G) * 8, 256);
  char* p = static_cast<char*>(base);
  w.part = reinterpret_cast<double*>(p);
  w.spill = reinterpret_cast<unsigned long long*>(p + part_bytes);
  w.zfirst = reinterpret_cast<unsigned long long*>(p + part_bytes + spill_bytes);
  w.live = n_masked > 0 ? reinterpret_cast<unsigned*>(p + part_bytes + spill_bytes + zf_bytes) : nullptr;
  w.bytes = part_bytes + spill_bytes + zf_bytes +
            (n_masked > 0 ? align_up(tbgb::dense_live_scratch_bytes(n_masked), 256) : 0);
  return w;
}

tbgb_status check_dense_args(tbgb_ctx* ctx, const int32_t* keys, const double* vals, int64_t n, int32_t G) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (G < 1 || G > tbgb::kDenseMaxGroups)
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_groups must be in [1, 1024] for the column kernel");
  if (n > 0 && (!keys || !vals)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "keys/values pointer is NULL");
  return TBGB_OK;
}

tbgb_status profile_events(tbgb_ctx* ctx, cudaEvent_t* e0, cudaEvent_t* e1) {
  *e0 = nullptr;
  *e1 = nullptr;
  if (!ctx->profile) return TBGB_OK;
  if (cudaEventCreate(e0) != cudaSuccess || cudaEventCreate(e1) != cudaSuccess)
    return fail(ctx, TBGB_ERR_BACKEND, "cudaEventCreate failed");
  ctx->events.emplace_back(*e0, *e1);
  return TBGB_OK;
}

tbgb_status dense_common(tbgb_ctx* ctx, const int32_t* keys, const double* vals, const uint64_t* mask, int64_t n,
                         int32_t G, int64_t row_offset, const tbgb_moments* out, double* state_out, void* stream,
                         bool state_m34 = true, const tbgb::PushArgs* push = nullptr) {
  tbgb_status st = check_dense_args(ctx, keys, vals, n, G);
  if (st != TBGB_OK) return st;
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  const tbgb::DenseLaunch L = tbgb::dense_plan(G, ctx->num_sms);
  const int64_t n_masked = mask ? n : 0;
  DenseWs w = dense_ws_layout(nullptr, L, G, n_masked);
  st = ensure_ws(ctx, w.bytes);
  if (st != TBGB_OK) return st;
  w = dense_ws_layout(ctx->ws, L, G, n_masked);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(w.zfirst, 0xFF, static_cast<size_t>(G) * 8, s);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "memset", e);
  cudaEvent_t e0, e1;
  st = profile_events(ctx, &e0, &e1);
  if (st != TBGB_OK) return st;
  e = tbgb::dense_moments_launch(L, keys, vals, mask, n, row_offset, G, w.part, w.spill, w.zfirst, ctx->err, out,
                                 state_out, s, &ctx->launches, e0, e1, w.live, state_m34, push);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "dense groupby launch", e);
  return TBGB_OK;
}

bool wants_full(const tbgb_moments* out) {
  return !out || out->min || out->max || out->m2 || out->var_pop || out->var_samp || out->m3 || out->m4;
}

tbgb_status check_columns(tbgb_ctx* ctx, const tbgb_columns* c, int64_t n) {
  if (!c) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "columns descriptor is NULL");
  if (c->dtype != TBGB_F64 && c->dtype != TBGB_F32) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "unknown dtype");
  if (c->expr < TBGB_EXPR_A || c->expr > TBGB_EXPR_MUL_ADD)
    return fail(ctx, TBGB_ERR_ENTRY_NOT_FOUND, "unknown expression id");
  if (c->pred < TBGB_PRED_NONE || c->pred > TBGB_PRED_FINITE)
    return fail(ctx, TBGB_ERR_ENTRY_NOT_FOUND, "unknown predicate id");
  if (n > 0) {
    if (!c->a) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "column a is NULL");
    if (c->expr != TBGB_EXPR_A && !c->b) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "column b is NULL");
    if (c->expr == TBGB_EXPR_MUL_ADD && !c->c) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "column c is NULL");
    const size_t eb = c->dtype == TBGB_F32 ? 4 : 8;
    if (misaligned(c->a, eb) || misaligned(c->b, eb) || misaligned(c->c, eb))
      return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "column pointer not aligned to its element size");
  }
  return TBGB_OK;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// int64-key count / sum / mean by radix partitioning (radix.cu); when a bucket overflows, the
// global table recomputes the whole result, its kernels gated on the radix passes' fallback word
// (they return at once when it is zero).  The fallback table lives where the second pass's
// buffer was.
tbgb_status radix_hash(tbgb_ctx* ctx, const int64_t* keys, const tbgb_columns* cols, const uint64_t* mask, int64_t n,
                       long long groups, int64_t* out_keys, const tbgb_moments* out, int64_t* d_n_groups,
                       void* stream) {
  const tbgb::RadixPlan R = tbgb::radix_plan(*cols, n, ctx->num_sms);
  const tbgb::TablePlan P = tbgb::table_plan(true, false, 0, groups, ctx->num_sms, 1, false);
  const size_t fb_bytes = align256(P.table_bytes) + align256(tbgb::table_finalize_scratch_bytes(P));
  const size_t t2_region = R.t2_bytes > fb_bytes ? R.t2_bytes : fb_bytes;
  tbgb_status st = ensure_ws(ctx, tbgb::radix_t2_offset(R) + t2_region);
  if (st != TBGB_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaEvent_t e0, e1;
  st = profile_events(ctx, &e0, &e1);
  if (st != TBGB_OK) return st;
  tbgb::RadixArgs ra{};
  ra.keys = keys;
  ra.cols = *cols;
  ra.mask = mask;
  ra.n = n;
  ra.max_groups = groups;
  ra.out_keys = out_keys;
  ra.out = *out;
  ra.d_n_groups = d_n_groups;
  ra.err = ctx->err;
  uint32_t* gate = nullptr;
  cudaError_t e = tbgb::radix_groupby(R, ra, ctx->ws, &gate, s, &ctx->launches, e0, e1);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "radix groupby launch", e);
  ctx->radix_gate = gate;
  char* w = static_cast<char*>(ctx->ws) + tbgb::radix_t2_offset(R);
  unsigned long long* T = reinterpret_cast<unsigned long long*>(w);
  unsigned long long* fin = reinterpret_cast<unsigned long long*>(w + align256(P.table_bytes));
  e = tbgb::table_init(P, T, s, &ctx->launches, gate);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "fallback table init", e);
  tbgb::TableArgs a{};
  a.keys = keys;
  a.cols = *cols;
  a.mask = mask;
  a.n = n;
  a.slots = P.slots;
  a.ngroups = tbgb::table_counter(P, T);
  a.max_groups = groups;
  a.err = ctx->err;
  a.table = T;
  a.gate = gate;
  e = tbgb::table_accumulate(P, a, s, &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "fallback table launch", e);
  e = tbgb::table_finalize_hash(P, T, groups, out_keys, out, d_n_groups, fin, s, &ctx->launches, gate);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "fallback table finalize", e);
  return TBGB_OK;
}

// The column set of a plain f64 value column (no filter, no expression).
tbgb_columns plain_f64(const double* vals) {
  tbgb_columns c{};
  c.a = vals;
  c.dtype = TBGB_F64;
  c.expr = TBGB_EXPR_A;
  c.pred = TBGB_PRED_NONE;
  return c;
}

// Bucket count of a hash table: sub-tables of about 64 MB keep a bucket's probes inside
// L2 and the TLB's reach; at most kMaxParts (the partition's limit).
int hash_buckets(tbgb_ctx* ctx, bool full, long long groups) {
  // opt-in: with 2^28 keys, 32 sub-tables of 512 MB measured no faster than one 16 GB table
  if (ctx->table_mode != 3) return 1;
  const tbgb::TablePlan one = tbgb::table_plan(true, full, 0, groups, ctx->num_sms, 1);
  const size_t target = size_t(64) << 20;
  int b = 1;
  while (b < tbgb::kMaxParts && one.table_bytes / b > target) b <<= 1;
  return b < 2 ? 2 : b;
}

// Global-table groupby: dense keys (hash == false, `groups` = n_groups) or int64
// keys (`groups` = max_groups).  int64 keys with a large table are first routed to
// sub-tables by their high hash bits (a stable partition that also applies the filter
// and the expression), then each sub-table takes its rows.
tbgb_status table_common(tbgb_ctx* ctx, bool hash, const void* keys, const tbgb_columns* cols, const uint64_t* mask,
                         int64_t n, long long groups, int64_t row_offset, int64_t* out_keys,
                         const tbgb_moments* out, double* state_out, int64_t* d_n_groups, void* stream,
                         bool state_m34 = true) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (groups < 1) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "the group count must be >= 1");
  if (n > 0 && !keys) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "keys pointer is NULL");
  tbgb_status st = check_columns(ctx, cols, n);
  if (st != TBGB_OK) return st;
  if (n / (ctx->num_sms > 0 ? ctx->num_sms : 1) >= (1ll << 31))
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "too many rows for one call (split the rows)");
  const bool full = state_out != nullptr || wants_full(out);
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  if (hash && !full && groups <= tbgb::kRadixMaxGroups &&
      (ctx->table_mode == 5 ||
       ((ctx->table_mode == 0 || ctx->table_mode == 6) && tbgb::radix_eligible(*cols, out, n, groups))))
    return radix_hash(ctx, static_cast<const int64_t*>(keys), cols, mask, n, groups, out_keys, out, d_n_groups,
                      stream);
  const int B = hash ? hash_buckets(ctx, full, groups) : 1;
  const int mode = ctx->table_mode == 3 ? 0 : ctx->table_mode;
  const bool m34 = full && ((state_out != nullptr && state_m34) || (out && (out->m3 || out->m4)));
  const tbgb::TablePlan P = tbgb::table_plan(hash, full, mode, groups, ctx->num_sms, B, m34);
  // workspace: table | partition scratch | part counts | part starts | routed keys | routed values
  const size_t t_bytes = align256(P.table_bytes);
  const size_t sc_bytes = B > 1 ? align256(tbgb::partition_scratch_bytes(n, B)) : 0;
  const size_t pc_bytes = B > 1 ? 256 : 0;
  const size_t rows = B > 1 ? tbgb::partition_output_rows(n, B, 1) : 0;
  const size_t pk_bytes = align256(rows * 8), pv_bytes = align256(rows * 8);
  const size_t fin_bytes = hash ? align256(tbgb::table_finalize_scratch_bytes(P)) : 0;
  st = ensure_ws(ctx, t_bytes + sc_bytes + 2 * pc_bytes + pk_bytes + pv_bytes + fin_bytes);
  if (st != TBGB_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* w = static_cast<char*>(ctx->ws);
  unsigned long long* T = reinterpret_cast<unsigned long long*>(w);
  unsigned long long* scratch = reinterpret_cast<unsigned long long*>(w + t_bytes);
  int64_t* pcounts = reinterpret_cast<int64_t*>(w + t_bytes + sc_bytes);
  int64_t* pstarts = reinterpret_cast<int64_t*>(w + t_bytes + sc_bytes + pc_bytes);
  int64_t* pkeys = reinterpret_cast<int64_t*>(w + t_bytes + sc_bytes + 2 * pc_bytes);
  double* pvals = reinterpret_cast<double*>(w + t_bytes + sc_bytes + 2 * pc_bytes + pk_bytes);
  unsigned long long* fin = reinterpret_cast<unsigned long long*>(w + t_bytes + sc_bytes + 2 * pc_bytes + pk_bytes +
                                                                  pv_bytes);
  cudaEvent_t e0, e1;
  st = profile_events(ctx, &e0, &e1);
  if (st != TBGB_OK) return st;
  if (e0) cudaEventRecord(e0, s);
  cudaError_t e = tbgb::table_init(P, T, s, &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "table init", e);
  tbgb::TableArgs a{};
  a.row_offset = row_offset;
  a.slots = P.slots;
  a.ngroups = tbgb::table_counter(P, T);
  a.max_groups = groups;
  a.err = ctx->err;
  a.m34 = m34;
  a.extrema = full && (state_out != nullptr || !out || out->min || out->max);
  if (B == 1) {
    a.keys = keys;
    a.cols = *cols;
    a.mask = mask;
    a.n = n;
    a.table = T;
    e = tbgb::table_accumulate(P, a, s, &ctx->launches);
    if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "table groupby launch", e);
  } else {
    tbgb::PartitionArgs pa{};
    pa.keys = keys;
    pa.cols = *cols;
    pa.mask = mask;
    pa.n = n;
    pa.P = B;
    pa.range = false;
    pa.align_rows = 1;
    pa.out_keys = pkeys;
    pa.out_vals = pvals;
    pa.err = ctx->err;
    e = tbgb::partition_launch(pa, scratch, pcounts, pstarts, s, &ctx->launches);
    if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "bucket partition launch", e);
    a.keys = pkeys;
    a.cols = plain_f64(pvals);
    a.mask = nullptr;
    a.n = 0;
    for (int b = 0; b < B; ++b) {
      a.table = tbgb::table_bucket(P, T, b);
      a.dev_count = pcounts + b;
      a.dev_start = pstarts + b;
      e = tbgb::table_accumulate(P, a, s, &ctx->launches);
      if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "table groupby launch", e);
    }
  }
  if (e1) cudaEventRecord(e1, s);
  if (hash) e = tbgb::table_finalize_hash(P, T, groups, out_keys, out, d_n_groups, fin, s, &ctx->launches);
  else e = tbgb::table_finalize_dense(P, T, groups, out, state_out, s, &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "table finalize launch", e);
  return TBGB_OK;
}

// Groups per key-range part: the column kernel's two-slot owner variant covers up to 512.
constexpr int kBucketGroups = 512;

// Key-range bucketing serves dense groupbys of up to kMaxParts * kBucketGroups groups when the
// context asks for it (mode 3).
bool use_buckets(const tbgb_ctx* ctx, long long G) {
  // opt-in: on the 10,000-group stress shape the partition pass costs more than the column
  // kernel saves over the shared-memory table (measured)
  return ctx->table_mode == 3 && G <= static_cast<long long>(tbgb::kMaxParts) * kBucketGroups;
}

// Above 512 groups each owner thread of the column kernel keeps four slots and spills them to
// local memory; the global-table kernel with shared-memory pre-aggregation is then faster
// (1000 groups, 2e8 rows: 2.9 ms against 4.9 ms), so the default mode sends it those.
constexpr int kColumnFastGroups = 512;

bool column_kernel_for(const tbgb_ctx* ctx, int32_t G) {
  return G >= 1 && G <= tbgb::kDenseMaxGroups && (ctx->table_mode != 0 || G <= kColumnFastGroups);
}

// Dense keys in [0, G) with G up to kMaxParts * kBucketGroups (or any filter / expression / f32
// columns): a stable key-range partition into parts of at most kBucketGroups groups (applying
// mask, predicate and expression, dropping NaN rows), then the shared-memory column
// kernel on each part, writing that part's slice of the outputs.
tbgb_status bucketed_dense(tbgb_ctx* ctx, const int32_t* keys, const tbgb_columns* cols, const uint64_t* mask,
                           int64_t n, int32_t G, const tbgb_moments* out, void* stream) {
  if (n > 0 && !keys) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "keys pointer is NULL");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  const int nb = (G + kBucketGroups - 1) / kBucketGroups;
  const int W = (G + nb - 1) / nb;
  const tbgb::DenseLaunch L = tbgb::dense_plan(W, ctx->num_sms);
  DenseWs dw = dense_ws_layout(nullptr, L, W);
  const int align = 4;  // part starts on 16-byte boundaries of the int32 keys (32 of the values)
  const size_t rows = tbgb::partition_output_rows(n, nb, align);
  const size_t sc_bytes = align256(tbgb::partition_scratch_bytes(n, nb));
  const size_t pk_bytes = align256(rows * 4), pv_bytes = align256(rows * 8);
  const size_t d_bytes = align256(dw.bytes);
  tbgb_status st = ensure_ws(ctx, d_bytes + sc_bytes + 512 + pk_bytes + pv_bytes);
  if (st != TBGB_OK) return st;
  char* w = static_cast<char*>(ctx->ws);
  dw = dense_ws_layout(w, L, W);
  unsigned long long* scratch = reinterpret_cast<unsigned long long*>(w + d_bytes);
  int64_t* pcounts = reinterpret_cast<int64_t*>(w + d_bytes + sc_bytes);
  int64_t* pstarts = pcounts + 32;
  int32_t* pkeys = reinterpret_cast<int32_t*>(w + d_bytes + sc_bytes + 512);
  double* pvals = reinterpret_cast<double*>(w + d_bytes + sc_bytes + 512 + pk_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaEvent_t e0, e1;
  st = profile_events(ctx, &e0, &e1);
  if (st != TBGB_OK) return st;
  if (e0) cudaEventRecord(e0, s);
  tbgb::PartitionArgs pa{};
  pa.keys = keys;
  pa.cols = *cols;
  pa.mask = mask;
  pa.n = n;
  pa.P = nb;
  pa.range = true;
  pa.width = W;
  pa.n_groups = G;
  pa.align_rows = align;
  pa.out_keys = pkeys;
  pa.out_vals = pvals;
  pa.err = ctx->err;
  cudaError_t e = tbgb::partition_launch(pa, scratch, pcounts, pstarts, s, &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "key-range partition launch", e);
  // The column kernel takes its row count at launch: read the part sizes (a few dozen bytes).
  int64_t hc[tbgb::kMaxParts], hs[tbgb::kMaxParts];
  e = cudaMemcpyAsync(hc, pcounts, static_cast<size_t>(nb) * 8, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(hs, pstarts, static_cast<size_t>(nb) * 8, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_TRANSFER, "part sizes", e);
  for (int b = 0; b < nb; ++b) {
    const int Gb = (b + 1) * W <= G ? W : G - b * W;
    const tbgb::DenseLaunch Lb = tbgb::dense_plan(Gb, ctx->num_sms);
    tbgb_moments ob = *out;
    double** f[] = {&ob.count, &ob.sum, &ob.min, &ob.max, &ob.mean, &ob.m2, &ob.var_pop, &ob.var_samp, &ob.m3, &ob.m4};
    for (double** q : f)
      if (*q) *q += static_cast<size_t>(b) * W;
    e = cudaMemsetAsync(dw.zfirst, 0xFF, static_cast<size_t>(Gb) * 8, s);
    if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "memset", e);
    e = tbgb::dense_moments_launch(Lb, pkeys + hs[b], pvals + hs[b], nullptr, hc[b], 0, Gb, dw.part, dw.spill,
                                   dw.zfirst, ctx->err, &ob, nullptr, s, &ctx->launches);
    if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "dense groupby launch", e);
  }
  if (e1) cudaEventRecord(e1, s);
  return TBGB_OK;
}

}  // namespace

extern "C" {

tbgb_status tbgb_create(int device, tbgb_ctx** out) {
  if (!out) return TBGB_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) return TBGB_ERR_BACKEND;
  if (device < 0 || device >= count) return TBGB_ERR_INVALID_ARGUMENT;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return TBGB_ERR_BACKEND;
  if (prop.major != 10) return TBGB_ERR_BACKEND;  // built for sm_100a only
  tbgb_ctx* ctx = new tbgb_ctx();
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  ctx->name = std::string(prop.name) + " (CUDA sm_" + std::to_string(prop.major) + std::to_string(prop.minor) + ")";
  DeviceGuard dg(device);
  if (!dg.ok || cudaMalloc(&ctx->err, sizeof(uint32_t)) != cudaSuccess ||
      cudaMemset(ctx->err, 0, sizeof(uint32_t)) != cudaSuccess) {
    delete ctx;
    return TBGB_ERR_ALLOC;
  }
  *out = ctx;
  return TBGB_OK;
}

void tbgb_destroy(tbgb_ctx* ctx) {
  if (!ctx) return;
  {
    DeviceGuard dg(ctx->device);
    for (auto& pr : ctx->events) {
      cudaEventDestroy(pr.first);
      cudaEventDestroy(pr.second);
    }
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->ws_mask) cudaFree(ctx->ws_mask);
    if (ctx->err) cudaFree(ctx->err);
  }
  delete ctx;
}

const char* tbgb_last_error(const tbgb_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

const char* tbgb_device_name(const tbgb_ctx* ctx) { return ctx ? ctx->name.c_str() : ""; }

uint64_t tbgb_launch_count(const tbgb_ctx* ctx) { return ctx ? ctx->launches : 0; }

tbgb_status tbgb_profile_enable(tbgb_ctx* ctx, int enable) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  ctx->profile = enable != 0;
  return TBGB_OK;
}

tbgb_status tbgb_kernel_time_ms(tbgb_ctx* ctx, double* total_ms, int64_t* launches) {
  if (!ctx || !total_ms || !launches) return TBGB_ERR_INVALID_ARGUMENT;
  DeviceGuard dg(ctx->device);
  double tot = 0.0;
  tbgb_status st = TBGB_OK;
  for (auto& pr : ctx->events) {
    float ms = 0.f;
    if (st == TBGB_OK) {
      cudaError_t e = cudaEventSynchronize(pr.second);
      if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, pr.first, pr.second);
      if (e != cudaSuccess) st = cuda_fail(ctx, TBGB_ERR_BACKEND, "event timing", e);
    }
    tot += ms;
    cudaEventDestroy(pr.first);
    cudaEventDestroy(pr.second);
  }
  *launches = static_cast<int64_t>(ctx->events.size());
  *total_ms = tot;
  ctx->events.clear();
  return st;
}

size_t tbgb_workspace_bytes(const tbgb_ctx* ctx, int64_t n, int32_t n_groups) {
  (void)n;
  if (!ctx || n_groups < 1) return 0;
  if (n_groups > tbgb::kDenseMaxGroups)
    return tbgb::table_plan(false, true, ctx->table_mode, n_groups, ctx->num_sms).table_bytes;
  const tbgb::DenseLaunch L = tbgb::dense_plan(n_groups, ctx->num_sms);
  return dense_ws_layout(nullptr, L, n_groups).bytes;
}

tbgb_status tbgb_set_table_mode(tbgb_ctx* ctx, int mode) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (mode < 0 || mode > 6) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "table mode must be 0 to 6");
  ctx->table_mode = mode;
  return TBGB_OK;
}

tbgb_status tbgb_groupby_dense(tbgb_ctx* ctx, const int32_t* d_keys, const double* d_vals, const uint64_t* d_mask,
                               int64_t n, int32_t n_groups, const tbgb_moments* out, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (!out) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "out is NULL");
  if (n_groups > tbgb::kDenseMaxGroups || (n_groups >= 1 && !column_kernel_for(ctx, n_groups))) {
    if (n > 0 && !d_vals) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "values pointer is NULL");
    const tbgb_columns c = plain_f64(d_vals);
    if (use_buckets(ctx, n_groups)) return bucketed_dense(ctx, d_keys, &c, d_mask, n, n_groups, out, stream);
    return table_common(ctx, false, d_keys, &c, d_mask, n, n_groups, 0, nullptr, out, nullptr, nullptr, stream);
  }
  return dense_common(ctx, d_keys, d_vals, d_mask, n, n_groups, 0, out, nullptr, stream);
}

tbgb_status tbgb_groupby_dense_columns(tbgb_ctx* ctx, const int32_t* d_keys, const tbgb_columns* cols,
                                       const uint64_t* d_mask, int64_t n, int32_t n_groups,
                                       const tbgb_moments* out, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (!out) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "out is NULL");
  tbgb_status st = check_columns(ctx, cols, n);
  if (st != TBGB_OK) return st;
  const bool plain = cols->dtype == TBGB_F64 && cols->expr == TBGB_EXPR_A && cols->pred == TBGB_PRED_NONE;
  if (plain && column_kernel_for(ctx, n_groups))
    return dense_common(ctx, d_keys, static_cast<const double*>(cols->a), d_mask, n, n_groups, 0, out, nullptr,
                        stream);
  // A predicate on a plain f64 column with few groups: the predicate as a row mask (reading
  // column a only where d_mask selects), then the masked column kernel, which skips tiles
  // whose mask words are all zero.
  const bool filtered = cols->dtype == TBGB_F64 && cols->expr == TBGB_EXPR_A && cols->pred != TBGB_PRED_NONE;
  if (filtered && ctx->table_mode == 0 && column_kernel_for(ctx, n_groups) && n > 0) {
    if (misaligned(d_mask, 8)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "mask not 8-byte aligned");
    DeviceGuard dg(ctx->device);
    if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
    st = ensure_ws_mask(ctx, static_cast<size_t>((n + 63) / 64) * 8);
    if (st != TBGB_OK) return st;
    uint64_t* m = static_cast<uint64_t*>(ctx->ws_mask);
    cudaError_t e = tbgb::filter_mask_launch(cols->a, TBGB_F64, n, cols->pred, cols->threshold, d_mask, m,
                                             ctx->num_sms, static_cast<cudaStream_t>(stream), &ctx->launches);
    if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "filter mask launch", e);
    return dense_common(ctx, d_keys, static_cast<const double*>(cols->a), m, n, n_groups, 0, out, nullptr, stream);
  }
  if (n_groups >= 1 && use_buckets(ctx, n_groups))
    return bucketed_dense(ctx, d_keys, cols, d_mask, n, n_groups, out, stream);
  return table_common(ctx, false, d_keys, cols, d_mask, n, n_groups, 0, nullptr, out, nullptr, nullptr, stream);
}

tbgb_status tbgb_groupby_hash(tbgb_ctx* ctx, const int64_t* d_keys, const tbgb_columns* cols,
                              const uint64_t* d_mask, int64_t n, int64_t max_groups, int64_t* d_out_keys,
                              const tbgb_moments* out, int64_t* d_n_groups, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (!out || !d_out_keys || !d_n_groups)
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "out, out_keys and n_groups must not be NULL");
  if (max_groups < 1 || max_groups > (1ll << 40))
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "max_groups must be in [1, 2^40]");
  return table_common(ctx, true, d_keys, cols, d_mask, n, max_groups, 0, d_out_keys, out, nullptr, d_n_groups,
                      stream);
}

size_t tbgb_state_bytes(int32_t n_groups) {
  return n_groups > 0 ? static_cast<size_t>(tbgb::ST_COUNT) * n_groups * sizeof(double) : 0;
}

namespace {

// A shard's mergeable state table; with m34 = false its m3 / m4 stay zero (the cheaper kernels).
tbgb_status dense_state(tbgb_ctx* ctx, const int32_t* d_keys, const double* d_vals, const uint64_t* d_mask, int64_t n,
                        int32_t n_groups, int64_t row_offset, void* d_state, void* stream, bool m34) {
  if (!d_state) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "state buffer is NULL");
  if (row_offset < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "row_offset must be >= 0");
  if (n_groups > tbgb::kDenseMaxGroups) {
    if (n > 0 && !d_vals) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "values pointer is NULL");
    const tbgb_columns c = plain_f64(d_vals);
    return table_common(ctx, false, d_keys, &c, d_mask, n, n_groups, row_offset, nullptr, nullptr,
                        static_cast<double*>(d_state), nullptr, stream, m34);
  }
  return dense_common(ctx, d_keys, d_vals, d_mask, n, n_groups, row_offset, nullptr, static_cast<double*>(d_state),
                      stream, m34);
}

}  // namespace

tbgb_status tbgb_groupby_dense_state(tbgb_ctx* ctx, const int32_t* d_keys, const double* d_vals,
                                     const uint64_t* d_mask, int64_t n, int32_t n_groups, int64_t row_offset,
                                     void* d_state, void* stream) {
  return dense_state(ctx, d_keys, d_vals, d_mask, n, n_groups, row_offset, d_state, stream, true);
}

size_t tbgb_exchange_bytes(int32_t world, int32_t n_groups) {
  if (world < 1 || world > tbgb::kMaxRanks || n_groups < 1) return 0;
  return tbgb::exchange_bytes(world, n_groups);
}

tbgb_status tbgb_exchange_alloc(tbgb_ctx* ctx, int32_t world, int32_t n_groups, void** d_buf) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (!d_buf || world < 1 || world > tbgb::kMaxRanks || n_groups < 1)
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "exchange_alloc: bad arguments (world <= 8)");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  const size_t bytes = tbgb::exchange_bytes(world, n_groups);
  cudaError_t e = cudaMalloc(d_buf, bytes);  // its own allocation: an IPC handle maps exactly this buffer
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_ALLOC, "exchange buffer", e);
  e = cudaMemset(*d_buf, 0, bytes);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_BACKEND, "exchange buffer memset", e);
  return TBGB_OK;
}

tbgb_status tbgb_exchange_free(tbgb_ctx* ctx, void* d_buf) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  DeviceGuard dg(ctx->device);
  if (d_buf) cudaFree(d_buf);
  return TBGB_OK;
}

tbgb_status tbgb_ipc_alloc(tbgb_ctx* ctx, size_t bytes, void** d_buf) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (!d_buf || bytes == 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "ipc_alloc: bad arguments");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  cudaError_t e = cudaMalloc(d_buf, bytes);  // its own allocation: an IPC handle maps exactly this buffer
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_ALLOC, "ipc buffer", e);
  return TBGB_OK;
}

tbgb_status tbgb_ipc_free(tbgb_ctx* ctx, void* d_buf) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  DeviceGuard dg(ctx->device);
  if (d_buf) cudaFree(d_buf);
  return TBGB_OK;
}

tbgb_status tbgb_peer_export(tbgb_ctx* ctx, void* d_buf, uint8_t* handle) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (!d_buf || !handle) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "peer_export: NULL pointer");
  DeviceGuard dg(ctx->device);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, d_buf);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_BACKEND, "cudaIpcGetMemHandle", e);
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle, &h, sizeof(h));
  return TBGB_OK;
}

tbgb_status tbgb_peer_import(tbgb_ctx* ctx, const uint8_t* handle, void** d_peer) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (!handle || !d_peer) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "peer_import: NULL pointer");
  DeviceGuard dg(ctx->device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(d_peer, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_BACKEND, "cudaIpcOpenMemHandle", e);
  return TBGB_OK;
}

tbgb_status tbgb_peer_close(tbgb_ctx* ctx, void* d_peer) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  DeviceGuard dg(ctx->device);
  if (d_peer) cudaIpcCloseMemHandle(d_peer);
  return TBGB_OK;
}

tbgb_status tbgb_groupby_dense_sharded(tbgb_ctx* ctx, const int32_t* d_keys, const double* d_vals,
                                       const uint64_t* d_mask, int64_t n, int32_t n_groups, int64_t row_offset,
                                       int32_t rank, int32_t world, void* const* h_exchange, uint64_t epoch,
                                       const tbgb_moments* out, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (!out || !h_exchange) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (world < 1 || world > tbgb::kMaxRanks || rank < 0 || rank >= world)
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "rank / world out of range (world <= 8)");
  if (epoch < 1) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "epoch must start at 1");
  if (n_groups < 1) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_groups must be >= 1");
  tbgb::PeerPtrs peers{};
  for (int q = 0; q < world; ++q) {
    if (!h_exchange[q] || misaligned(h_exchange[q], 256))
      return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "exchange buffer NULL or not 256-byte aligned");
    peers.p[q] = h_exchange[q];
  }
  const int parity = static_cast<int>(epoch & 1ull);
  double* own_slot = reinterpret_cast<double*>(static_cast<char*>(h_exchange[rank]) +
                                               tbgb::exchange_slot_offset(world, n_groups, parity, rank));
  // this shard's state table, written straight into its slot of the own buffer (without the
  // third and fourth moments unless `out` asks for them: the merge of the others never reads them)
  const bool m34 = out->m3 != nullptr || out->m4 != nullptr;
  cudaError_t e = cudaSuccess;
  DeviceGuard dg(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_groups <= tbgb::kDenseMaxGroups) {
    // the column kernel's fold stores the table into every peer's slot and raises the flags
    const tbgb::PushArgs push = tbgb::exchange_push_args(peers, world, rank, n_groups, epoch);
    if (row_offset < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "row_offset must be >= 0");
    tbgb_status st = dense_common(ctx, d_keys, d_vals, d_mask, n, n_groups, row_offset, nullptr, own_slot, stream,
                                  m34, &push);
    if (st != TBGB_OK) return st;
  } else {
    tbgb_status st = dense_state(ctx, d_keys, d_vals, d_mask, n, n_groups, row_offset, own_slot, stream, m34);
    if (st != TBGB_OK) return st;
    e = tbgb::exchange_push_launch(peers, world, rank, n_groups, epoch, s, &ctx->launches);
  }
  if (e == cudaSuccess)
    e = tbgb::exchange_merge_launch(h_exchange[rank], world, n_groups, epoch, ctx->err, out, s, &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "exchange launch", e);
  return TBGB_OK;
}

tbgb_status tbgb_merge_states(tbgb_ctx* ctx, const void* d_states, int32_t n_states, int32_t n_groups,
                              const tbgb_moments* out, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (!d_states || !out || n_states < 1 || n_groups < 1)
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "merge_states: bad arguments");
  DeviceGuard dg(ctx->device);
  cudaError_t e = tbgb::merge_states_launch(static_cast<const double*>(d_states), n_states, n_groups, out,
                                            static_cast<cudaStream_t>(stream), &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "merge_states launch", e);
  return TBGB_OK;
}

tbgb_status tbgb_scatter_multi_phi_masked(tbgb_ctx* ctx, const int32_t* phis, int32_t n_phi, const int32_t* d_keys,
                                          const double* d_vals, const double* d_refs, const uint64_t* d_mask,
                                          int64_t n, int32_t n_groups, double* d_out, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (!phis || n_phi < 1 || n_phi > tbgb::kMaxPhi)
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "between 1 and 5 phi expressions per call");
  for (int j = 0; j < n_phi; ++j)
    if (phis[j] < TBGB_PHI_V || phis[j] > TBGB_PHI_RECIP)
      return fail(ctx, TBGB_ERR_ENTRY_NOT_FOUND, "unknown phi id " + std::to_string(phis[j]));
  if (n < 0 || n_groups < 1) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n must be >= 0 and n_groups >= 1");
  if (!d_out || (n > 0 && (!d_keys || !d_vals)))
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "keys / values / out pointer is NULL");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  cudaError_t e = tbgb::phi_scatter_launch(phis, n_phi, d_keys, d_vals, d_refs, d_mask, n, n_groups, d_out, ctx->err,
                                           ctx->num_sms, static_cast<cudaStream_t>(stream), &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "scatter launch", e);
  return TBGB_OK;
}

tbgb_status tbgb_scatter_phi(tbgb_ctx* ctx, int32_t phi, const int32_t* d_keys, const double* d_vals,
                             const double* d_refs, int64_t n, int32_t n_groups, double* d_out, void* stream) {
  return tbgb_scatter_multi_phi_masked(ctx, &phi, 1, d_keys, d_vals, d_refs, nullptr, n, n_groups, d_out, stream);
}

tbgb_status tbgb_scatter_multi_phi(tbgb_ctx* ctx, const int32_t* phis, int32_t n_phi, const int32_t* d_keys,
                                   const double* d_vals, const double* d_refs, int64_t n, int32_t n_groups,
                                   double* d_out, void* stream) {
  return tbgb_scatter_multi_phi_masked(ctx, phis, n_phi, d_keys, d_vals, d_refs, nullptr, n, n_groups, d_out,
                                       stream);
}

tbgb_status tbgb_scatter_phi_masked(tbgb_ctx* ctx, int32_t phi, const int32_t* d_keys, const double* d_vals,
                                    const double* d_refs, const uint64_t* d_mask, int64_t n, int32_t n_groups,
                                    double* d_out, void* stream) {
  if (ctx && n > 0 && !d_mask) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "mask is NULL");
  return tbgb_scatter_multi_phi_masked(ctx, &phi, 1, d_keys, d_vals, d_refs, d_mask, n, n_groups, d_out, stream);
}

tbgb_status tbgb_scatter_extremum(tbgb_ctx* ctx, int32_t is_max, const int32_t* d_keys, const double* d_vals,
                                  int64_t n, int32_t n_groups, double* d_out, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n < 0 || n_groups < 1) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n must be >= 0 and n_groups >= 1");
  if (!d_out || (n > 0 && (!d_keys || !d_vals)))
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "keys / values / out pointer is NULL");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  tbgb_status st = ensure_ws(ctx, static_cast<size_t>(n_groups) * 16);
  if (st != TBGB_OK) return st;
  cudaError_t e = tbgb::extremum_launch(is_max != 0, d_keys, d_vals, n, n_groups, d_out,
                                        static_cast<unsigned long long*>(ctx->ws), ctx->err, ctx->num_sms,
                                        static_cast<cudaStream_t>(stream), &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "extremum launch", e);
  return TBGB_OK;
}

tbgb_status tbgb_group_index_build(tbgb_ctx* ctx, const int32_t* d_keys, int64_t n, int32_t max_key,
                                   uint32_t* d_row_to_group, uint32_t* d_group_counts, uint32_t* d_group_offsets,
                                   uint32_t* d_rows_by_group, int64_t* d_n_active, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n <= 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "GroupIndex::build called on empty column");
  if (n >= (1ll << 32)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "row ids are u32: n must be < 2^32");
  if (max_key < 0 || max_key == INT32_MAX) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "max_key out of range");
  if (!d_keys || !d_row_to_group || !d_group_counts || !d_group_offsets || !d_rows_by_group || !d_n_active)
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "NULL pointer");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  tbgb_status st = ensure_ws(ctx, tbgb::group_index_scratch_bytes(n));
  if (st != TBGB_OK) return st;
  cudaError_t e = tbgb::group_index_launch(d_keys, n, max_key + 1, d_row_to_group, d_group_counts, d_group_offsets,
                                           d_rows_by_group, d_n_active, ctx->ws, ctx->err, ctx->num_sms,
                                           static_cast<cudaStream_t>(stream), &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "group index launch", e);
  return TBGB_OK;
}

tbgb_status tbgb_factorize_i64(tbgb_ctx* ctx, const int64_t* d_keys, int64_t n, int64_t max_groups, int32_t* d_codes,
                               int64_t* d_uniques, int64_t* d_n_uniques, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n < 0 || n >= (1ll << 32)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n must be in [0, 2^32)");
  if (max_groups < 1 || max_groups > INT32_MAX) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "max_groups out of range");
  if (!d_uniques || !d_n_uniques || (n > 0 && (!d_keys || !d_codes)))
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "NULL pointer");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  tbgb_status st = ensure_ws(ctx, tbgb::factorize_scratch_bytes(n, max_groups));
  if (st != TBGB_OK) return st;
  cudaError_t e = tbgb::factorize_launch(d_keys, n, max_groups, d_codes, d_uniques, d_n_uniques, ctx->ws, ctx->err,
                                         ctx->num_sms, static_cast<cudaStream_t>(stream), &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "factorize launch", e);
  return TBGB_OK;
}

// ---- statistics of sorted contiguous bins ----

tbgb_status tbgb_fused_bin_stats(tbgb_ctx* ctx, const double* d_data, int64_t n_ticks, int32_t n_columns,
                                 const int64_t* d_boundaries, int64_t n_bins, const tbgb_bin_stats* out,
                                 void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (!out) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "out is NULL");
  if (n_ticks < 0 || n_bins < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_ticks and n_bins must be >= 0");
  if (n_columns < 1 || n_columns > 65535) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_columns must be in [1, 65535]");
  if (n_ticks > 0 && !d_data) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "data is NULL");
  if (!d_boundaries) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "boundaries is NULL");
  const void* ptrs[] = {d_data, d_boundaries, out->sum, out->sum_sq, out->min, out->max, out->first, out->last,
                        out->mean, out->variance, out->std};
  for (const void* p : ptrs)
    if (misaligned(p, 8)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "pointer not 8-byte aligned");
  if (misaligned(out->count, 4)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "count not 4-byte aligned");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  tbgb_status st = ensure_ws(ctx, tbgb::bin_stats_scratch_bytes(n_ticks, n_columns));
  if (st != TBGB_OK) return st;
  cudaEvent_t e0, e1;
  st = profile_events(ctx, &e0, &e1);
  if (st != TBGB_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (e0) cudaEventRecord(e0, s);
  cudaError_t e = tbgb::bin_stats_launch(d_data, n_ticks, n_columns, d_boundaries, n_bins, out, ctx->ws, ctx->err,
                                         ctx->num_sms, s, &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "bin stats launch", e);
  if (e1) cudaEventRecord(e1, s);
  return TBGB_OK;
}

// ---- row masks and tile statistics ----

namespace {

tbgb_status check_words(tbgb_ctx* ctx, const void* p, int64_t n_words, const char* what) {
  if (n_words > 0 && !p) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, std::string(what) + " is NULL");
  if (misaligned(p, 8)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, std::string(what) + " is not 8-byte aligned");
  return TBGB_OK;
}

tbgb_status mask_binary(tbgb_ctx* ctx, int op, const uint64_t* a, const uint64_t* b, uint64_t* out, int64_t n_words,
                        void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n_words < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_words < 0");
  tbgb_status st = check_words(ctx, a, n_words, "mask a");
  if (st == TBGB_OK) st = check_words(ctx, b, n_words, "mask b");
  if (st == TBGB_OK) st = check_words(ctx, out, n_words, "output mask");
  if (st != TBGB_OK) return st;
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  cudaError_t e = tbgb::mask_op_launch(op, a, b, out, n_words, n_words * 64, ctx->num_sms,
                                       static_cast<cudaStream_t>(stream), &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "mask launch", e);
  return TBGB_OK;
}

tbgb_status check_rows_words(tbgb_ctx* ctx, int64_t n_words, int64_t n_rows) {
  if (n_rows < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_rows < 0");
  if (n_words != (n_rows + 63) / 64) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_words must be ceil(n_rows / 64)");
  return TBGB_OK;
}

}  // namespace

tbgb_status tbgb_filter_mask(tbgb_ctx* ctx, const void* d_col, int32_t dtype, int64_t n, int32_t pred,
                             double threshold, const uint64_t* d_in_mask, uint64_t* d_mask, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n < 0");
  if (dtype != TBGB_F64 && dtype != TBGB_F32) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "unknown dtype");
  if (pred < TBGB_PRED_NONE || pred > TBGB_PRED_FINITE) return fail(ctx, TBGB_ERR_ENTRY_NOT_FOUND, "unknown predicate id");
  if (n > 0 && !d_col) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "column is NULL");
  if (misaligned(d_col, dtype == TBGB_F32 ? 4 : 8))
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "column pointer not aligned to its element size");
  tbgb_status st = check_words(ctx, d_mask, (n + 63) / 64, "mask");
  if (st != TBGB_OK) return st;
  if (misaligned(d_in_mask, 8)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "input mask not 8-byte aligned");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  cudaError_t e = tbgb::filter_mask_launch(d_col, dtype, n, pred, threshold, d_in_mask, d_mask, ctx->num_sms,
                                           static_cast<cudaStream_t>(stream), &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "filter mask launch", e);
  return TBGB_OK;
}

tbgb_status tbgb_mask_and(tbgb_ctx* ctx, const uint64_t* d_a, const uint64_t* d_b, uint64_t* d_out, int64_t n_words,
                          void* stream) {
  return mask_binary(ctx, tbgb::MASK_AND, d_a, d_b, d_out, n_words, stream);
}

tbgb_status tbgb_mask_or(tbgb_ctx* ctx, const uint64_t* d_a, const uint64_t* d_b, uint64_t* d_out, int64_t n_words,
                         void* stream) {
  return mask_binary(ctx, tbgb::MASK_OR, d_a, d_b, d_out, n_words, stream);
}

tbgb_status tbgb_mask_xor(tbgb_ctx* ctx, const uint64_t* d_a, const uint64_t* d_b, uint64_t* d_out, int64_t n_words,
                          void* stream) {
  return mask_binary(ctx, tbgb::MASK_XOR, d_a, d_b, d_out, n_words, stream);
}

tbgb_status tbgb_mask_not(tbgb_ctx* ctx, const uint64_t* d_a, uint64_t* d_out, int64_t n_words, int64_t n_rows,
                          void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  tbgb_status st = check_rows_words(ctx, n_words, n_rows);
  if (st == TBGB_OK) st = check_words(ctx, d_a, n_words, "mask");
  if (st == TBGB_OK) st = check_words(ctx, d_out, n_words, "output mask");
  if (st != TBGB_OK) return st;
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  cudaError_t e = tbgb::mask_op_launch(tbgb::MASK_NOT, d_a, nullptr, d_out, n_words, n_rows, ctx->num_sms,
                                       static_cast<cudaStream_t>(stream), &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "mask launch", e);
  return TBGB_OK;
}

tbgb_status tbgb_mask_popcount(tbgb_ctx* ctx, const uint64_t* d_mask, int64_t n_words, int64_t n_rows,
                               uint64_t* d_count, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n_rows < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_rows < 0");
  if (n_words < (n_rows + 63) / 64) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_words < ceil(n_rows / 64)");
  tbgb_status st = check_words(ctx, d_mask, n_words, "mask");
  if (st == TBGB_OK) st = check_words(ctx, d_count, 1, "count");
  if (st != TBGB_OK) return st;
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  cudaError_t e = tbgb::mask_popcount_launch(d_mask, n_rows, reinterpret_cast<unsigned long long*>(d_count),
                                             ctx->num_sms, static_cast<cudaStream_t>(stream), &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "popcount launch", e);
  return TBGB_OK;
}

tbgb_status tbgb_tile_stats_build(tbgb_ctx* ctx, const void* d_col, int32_t dtype, int64_t n, int64_t tile_rows,
                                  tbgb_tile_stats* d_stats, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n < 0");
  if (tile_rows < 1 || tile_rows > static_cast<int64_t>(UINT32_MAX))
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "tile_rows must be in [1, 2^32)");
  if (dtype != TBGB_F64 && dtype != TBGB_F32) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "unknown dtype");
  if (n > 0 && (!d_col || !d_stats)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (misaligned(d_col, dtype == TBGB_F32 ? 4 : 8) || misaligned(d_stats, 8))
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "pointer not aligned");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  cudaError_t e = tbgb::tile_stats_launch(d_col, dtype, n, tile_rows, d_stats, ctx->num_sms,
                                          static_cast<cudaStream_t>(stream), &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "tile stats launch", e);
  return TBGB_OK;
}

tbgb_status tbgb_tile_skip_mask(tbgb_ctx* ctx, const tbgb_tile_stats* d_stats, int64_t n_tiles, int32_t pred,
                                double threshold, uint8_t* d_skip, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n_tiles < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_tiles < 0");
  if (pred != TBGB_PRED_GT && pred != TBGB_PRED_GE && pred != TBGB_PRED_LT && pred != TBGB_PRED_LE)
    return fail(ctx, TBGB_ERR_ENTRY_NOT_FOUND, "tile skipping needs a >, >=, < or <= predicate");
  if (n_tiles > 0 && (!d_stats || !d_skip)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (misaligned(d_stats, 8)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "stats not 8-byte aligned");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  cudaError_t e = tbgb::tile_skip_launch(d_stats, n_tiles, pred, threshold, d_skip,
                                         static_cast<cudaStream_t>(stream), &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "tile skip launch", e);
  return TBGB_OK;
}

tbgb_status tbgb_mask_skip_tiles(tbgb_ctx* ctx, const uint64_t* d_mask, const uint8_t* d_skip, int64_t tile_rows,
                                 int64_t n_rows, uint64_t* d_out, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n_rows < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_rows < 0");
  if (tile_rows < 1) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "tile_rows < 1");
  const int64_t n_words = (n_rows + 63) / 64;
  if (n_rows > 0 && !d_skip) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "skip is NULL");
  if (misaligned(d_mask, 8)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "mask not 8-byte aligned");
  tbgb_status st = check_words(ctx, d_out, n_words, "output mask");
  if (st != TBGB_OK) return st;
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  cudaError_t e = tbgb::mask_skip_tiles_launch(d_mask, d_skip, tile_rows, n_rows, d_out, ctx->num_sms,
                                               static_cast<cudaStream_t>(stream), &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "mask skip-tiles launch", e);
  return TBGB_OK;
}

tbgb_status tbgb_hash_partition(tbgb_ctx* ctx, const int64_t* d_keys, const tbgb_columns* cols,
                                const uint64_t* d_mask, int64_t n, int32_t n_parts, int64_t* d_out_keys,
                                double* d_out_vals, int64_t* d_part_counts, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (n_parts < 1 || n_parts > tbgb::kMaxParts)
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_parts must be in [1, 32]");
  if (!d_part_counts) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "part_counts is NULL");
  if (n > 0 && (!d_keys || !d_out_keys || !d_out_vals))
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "keys / output pointers are NULL");
  tbgb_status st = check_columns(ctx, cols, n);
  if (st != TBGB_OK) return st;
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  const size_t sc_bytes = align256(tbgb::partition_scratch_bytes(n, n_parts));
  st = ensure_ws(ctx, sc_bytes + 256);
  if (st != TBGB_OK) return st;
  tbgb::PartitionArgs a{};
  a.keys = d_keys;
  a.cols = *cols;
  a.mask = d_mask;
  a.n = n;
  a.P = n_parts;
  a.range = false;
  a.align_rows = 1;
  a.out_keys = d_out_keys;
  a.out_vals = d_out_vals;
  a.err = ctx->err;
  char* w = static_cast<char*>(ctx->ws);
  cudaError_t e = tbgb::partition_launch(a, reinterpret_cast<unsigned long long*>(w), d_part_counts,
                                         reinterpret_cast<int64_t*>(w + sc_bytes), static_cast<cudaStream_t>(stream),
                                         &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "hash partition launch", e);
  return TBGB_OK;
}

int32_t tbgb_radix_value_bytes(const tbgb_columns* cols) {
  if (!cols) return 0;
  return tbgb::radix_value_f32(*cols) ? 4 : 8;
}

tbgb_status tbgb_radix_route(tbgb_ctx* ctx, const int64_t* d_keys, const tbgb_columns* cols, const uint64_t* d_mask,
                             int64_t n, uint64_t* d_out_hashes, void* d_out_vals, int64_t* d_digit_counts,
                             void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (!d_digit_counts) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "digit_counts is NULL");
  if (n > 0 && (!d_keys || !d_out_hashes || !d_out_vals))
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "keys / output pointers are NULL");
  if (misaligned(d_keys, 8) || misaligned(d_out_hashes, 8) ||
      misaligned(d_out_vals, static_cast<size_t>(tbgb_radix_value_bytes(cols))))
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "pointer not aligned to its element size");
  tbgb_status st = check_columns(ctx, cols, n);
  if (st != TBGB_OK) return st;
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  st = ensure_ws(ctx, tbgb::radix_route_aux_bytes());
  if (st != TBGB_OK) return st;
  tbgb::RadixArgs a{};
  a.keys = d_keys;
  a.cols = *cols;
  a.mask = d_mask;
  a.n = n;
  cudaError_t e = tbgb::radix_route(a, reinterpret_cast<unsigned long long*>(d_out_hashes), d_out_vals,
                                    d_digit_counts, ctx->ws, ctx->num_sms, static_cast<cudaStream_t>(stream),
                                    &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "radix route launch", e);
  return TBGB_OK;
}

tbgb_status tbgb_radix_groupby_routed(tbgb_ctx* ctx, int32_t n_senders, const uint64_t* const* h_hashes,
                                      const void* const* h_vals, const int64_t* h_rows, int32_t value_bytes,
                                      const int64_t* d_seg_counts, int32_t digit_lo, int32_t n_digits,
                                      int64_t max_groups, int64_t* d_out_keys, const tbgb_moments* out,
                                      int64_t* d_n_groups, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (!out || !d_out_keys || !d_n_groups || !d_seg_counts)
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "out, out_keys, n_groups and seg_counts must not be NULL");
  if (out->min || out->max || out->m2 || out->var_pop || out->var_samp || out->m3 || out->m4)
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "the routed groupby computes count, sum and mean only");
  if (value_bytes != 4 && value_bytes != 8) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "value_bytes must be 4 or 8");
  if (n_senders < 1 || n_senders > tbgb::kRadixMaxSenders || n_digits < 1 || digit_lo < 0 ||
      digit_lo + n_digits > tbgb::kRadixDigits || static_cast<long long>(n_senders) * n_digits > 4096)
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "bad sender / digit ranges (1..64 senders, digits within [0, 512), "
                                                "senders x digits <= 4096)");
  if (!h_hashes || !h_vals || !h_rows) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "sender arrays must not be NULL");
  long long n_rows = 0;
  for (int i = 0; i < n_senders; ++i) {
    if (h_rows[i] < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "a sender's row count is negative");
    if (h_rows[i] > 0 && (!h_hashes[i] || !h_vals[i]))
      return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "row pointers are NULL");
    if (misaligned(h_hashes[i], 8) || misaligned(h_vals[i], static_cast<size_t>(value_bytes)))
      return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "pointer not aligned to its element size");
    n_rows += h_rows[i];
  }
  if (max_groups < 1 || max_groups > (1ll << 40))
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "max_groups must be in [1, 2^40]");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  const bool vf32 = value_bytes == 4;
  const tbgb::RadixPlan R = tbgb::radix_routed_plan(vf32, n_rows, n_digits, ctx->num_sms);
  const tbgb::TablePlan P = tbgb::table_plan(true, false, 0, max_groups, ctx->num_sms, 1, false);
  const size_t fb_bytes = align256(P.table_bytes) + align256(tbgb::table_finalize_scratch_bytes(P));
  const size_t t2_region = R.t2_bytes > fb_bytes ? R.t2_bytes : fb_bytes;
  tbgb_status st = ensure_ws(ctx, tbgb::radix_t2_offset(R) + t2_region);
  if (st != TBGB_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaEvent_t e0, e1;
  st = profile_events(ctx, &e0, &e1);
  if (st != TBGB_OK) return st;
  tbgb::RoutedArgs r{};
  for (int i = 0; i < n_senders; ++i) {
    r.hashes[i] = reinterpret_cast<const unsigned long long*>(h_hashes[i]);
    r.vals[i] = h_vals[i];
  }
  r.seg_counts = d_seg_counts;
  r.n_senders = n_senders;
  r.digit_lo = digit_lo;
  r.n_digits = n_digits;
  r.n_rows = n_rows;
  r.max_groups = max_groups;
  r.out_keys = d_out_keys;
  r.out = *out;
  r.d_n_groups = d_n_groups;
  r.err = ctx->err;
  uint32_t* gate = nullptr;
  cudaError_t e = tbgb::radix_groupby_routed(R, r, ctx->ws, &gate, s, &ctx->launches, e0, e1);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "routed radix groupby launch", e);
  ctx->radix_gate = gate;
  // fallback (gated): group the hashes themselves in the global table, then turn them into keys
  char* w = static_cast<char*>(ctx->ws) + tbgb::radix_t2_offset(R);
  unsigned long long* T = reinterpret_cast<unsigned long long*>(w);
  unsigned long long* fin = reinterpret_cast<unsigned long long*>(w + align256(P.table_bytes));
  e = tbgb::table_init(P, T, s, &ctx->launches, gate);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "fallback table init", e);
  for (int i = 0; i < n_senders; ++i) {  // one gated pass over each sender's rows
    if (h_rows[i] == 0) continue;
    tbgb::TableArgs a{};
    a.keys = reinterpret_cast<const int64_t*>(h_hashes[i]);
    a.cols.a = h_vals[i];
    a.cols.dtype = vf32 ? TBGB_F32 : TBGB_F64;
    a.cols.expr = TBGB_EXPR_A;
    a.cols.pred = TBGB_PRED_NONE;
    a.n = h_rows[i];
    a.slots = P.slots;
    a.ngroups = tbgb::table_counter(P, T);
    a.max_groups = max_groups;
    a.err = ctx->err;
    a.table = T;
    a.gate = gate;
    e = tbgb::table_accumulate(P, a, s, &ctx->launches);
    if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "fallback table launch", e);
  }
  e = tbgb::table_finalize_hash(P, T, max_groups, d_out_keys, out, d_n_groups, fin, s, &ctx->launches, gate);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "fallback table finalize", e);
  e = tbgb::radix_unhash_keys(d_out_keys, d_n_groups, max_groups, gate, ctx->num_sms, s, &ctx->launches);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "fallback key launch", e);
  return TBGB_OK;
}

tbgb_status tbgb_radix_fallback(tbgb_ctx* ctx, uint32_t* bits) {
  if (!ctx || !bits) return TBGB_ERR_INVALID_ARGUMENT;
  *bits = 0;
  if (!ctx->radix_gate) return TBGB_OK;
  DeviceGuard dg(ctx->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(bits, ctx->radix_gate, sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_TRANSFER, "reading the radix fallback word", e);
  return TBGB_OK;
}

tbgb_status tbgb_sync(tbgb_ctx* ctx, void* stream) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  DeviceGuard dg(ctx->device);
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "stream synchronize", e);
  uint32_t bits = 0;
  e = cudaMemcpy(&bits, ctx->err, sizeof(bits), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_TRANSFER, "status read", e);
  if (bits == 0) return TBGB_OK;
  cudaMemset(ctx->err, 0, sizeof(uint32_t));
  if (bits & tbgb::KERR_KEY_RANGE) return fail(ctx, TBGB_ERR_KEY_OUT_OF_RANGE, "a key is outside [0, n_groups)");
  if (bits & tbgb::KERR_TABLE_FULL) return fail(ctx, TBGB_ERR_TABLE_FULL, "hash table full");
  if (bits & tbgb::KERR_TIMEOUT) return fail(ctx, TBGB_ERR_TIMEOUT, "device-side wait timed out");
  if (bits & tbgb::KERR_BOUNDARIES)
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "bin boundaries are not non-decreasing within [0, n_ticks]");
  if (bits & tbgb::KERR_MISALIGNED) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "a staged column is not 16-byte aligned");
  return fail(ctx, TBGB_ERR_BACKEND, "unknown device error bits " + std::to_string(bits));
}

// ---- generators ------------------------------------------------------------------

#define GEN_ENTRY(call)                                                              \
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;                                        \
  if (n < 0 || first_row < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n, first_row must be >= 0"); \
  DeviceGuard dg(ctx->device);                                                       \
  cudaError_t e = (call);                                                            \
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "generator", e);    \
  ctx->launches++;                                                                   \
  return TBGB_OK;

tbgb_status tbgb_gen_keys_uniform(tbgb_ctx* ctx, int32_t* d_keys, int64_t n, int32_t n_groups, uint64_t seed,
                                  int64_t first_row, void* stream) {
  if (n_groups < 1) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_groups must be >= 1");
  GEN_ENTRY(tbgb::gen_keys_uniform(d_keys, n, n_groups, seed, first_row, static_cast<cudaStream_t>(stream)))
}

tbgb_status tbgb_gen_values_uniform(tbgb_ctx* ctx, double* d_vals, int64_t n, double lo, double hi, uint64_t seed,
                                    int64_t first_row, void* stream) {
  GEN_ENTRY(tbgb::gen_values_uniform(d_vals, n, lo, hi, seed, first_row, static_cast<cudaStream_t>(stream)))
}

tbgb_status tbgb_gen_values_normal(tbgb_ctx* ctx, double* d_vals, int64_t n, double mu, double sigma, uint64_t seed,
                                   int64_t first_row, void* stream) {
  GEN_ENTRY(tbgb::gen_values_normal(d_vals, n, mu, sigma, seed, first_row, static_cast<cudaStream_t>(stream)))
}

tbgb_status tbgb_gen_inject_nonfinite(tbgb_ctx* ctx, double* d_vals, int64_t n, double nan_frac, double inf_frac,
                                      uint64_t seed, int64_t first_row, void* stream) {
  GEN_ENTRY(tbgb::gen_inject_nonfinite(d_vals, n, nan_frac, inf_frac, seed, first_row,
                                       static_cast<cudaStream_t>(stream)))
}

tbgb_status tbgb_gen_keys_cdf(tbgb_ctx* ctx, int64_t* d_keys, int64_t n, const double* d_cdf, int64_t n_ids,
                              uint64_t salt, uint64_t seed, int64_t first_row, void* stream) {
  if (n_ids < 1 || (n > 0 && !d_cdf)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "bad cdf table");
  GEN_ENTRY(tbgb::gen_keys_cdf(d_keys, n, d_cdf, n_ids, salt, seed, first_row, static_cast<cudaStream_t>(stream)))
}

tbgb_status tbgb_gen_keys_ids(tbgb_ctx* ctx, int64_t* d_keys, int64_t n, int64_t n_ids, uint64_t salt, uint64_t seed,
                              int64_t first_row, void* stream) {
  if (n_ids < 1) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_ids must be >= 1");
  GEN_ENTRY(tbgb::gen_keys_ids(d_keys, n, static_cast<uint64_t>(n_ids), salt, seed, first_row,
                               static_cast<cudaStream_t>(stream)))
}

tbgb_status tbgb_gen_values_lognormal_f32(tbgb_ctx* ctx, float* d_vals, int64_t n, double mu, double sigma,
                                          uint64_t seed, int64_t first_row, void* stream) {
  GEN_ENTRY(tbgb::gen_values_lognormal_f32(d_vals, n, mu, sigma, seed, first_row, static_cast<cudaStream_t>(stream)))
}

}  // extern "C"
