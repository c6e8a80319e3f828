// api.cpp -- C ABI of the groupby path (include/tambear_gb.h).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "dense.cuh"
#include "errbits.hpp"
#include "gen.cuh"
#include "tambear_gb.h"

struct tbgb_ctx {
  int device = 0;
  int num_sms = 0;
  std::string name;
  std::string last_error;
  void* ws = nullptr;  // workspace: partial states, zero trackers
  size_t ws_bytes = 0;
  uint32_t* err = nullptr;  // deferred kernel error bits (persist until tbgb_sync)
  uint64_t launches = 0;
  bool profile = false;  // record events around main kernels
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> events;
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
  size_t want = bytes + bytes / 4;
  cudaError_t e = cudaMalloc(&ctx->ws, want);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_ALLOC, "workspace allocation", e);
  ctx->ws_bytes = want;
  return TBGB_OK;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct DenseWs {
  double* part;
  unsigned long long* spill;
  unsigned long long* zfirst;
  size_t bytes;
};

DenseWs dense_ws_layout(void* base, const tbgb::DenseLaunch& L, int G) {
  DenseWs w{};
  const size_t part_bytes = align_up(L.part_doubles * 8, 256);
  const size_t spill_bytes = align_up(L.spill_words * 8, 256);
  char* p = static_cast<char*>(base);
  w.part = reinterpret_cast<double*>(p);
  w.spill = reinterpret_cast<unsigned long long*>(p + part_bytes);
  w.zfirst = reinterpret_cast<unsigned long long*>(p + part_bytes + spill_bytes);
  w.bytes = part_bytes + spill_bytes + align_up(static_cast<size_t>(G) * 8, 256);
  return w;
}

tbgb_status check_dense_args(tbgb_ctx* ctx, const int32_t* keys, const double* vals, int64_t n, int32_t G) {
  if (!ctx) return TBGB_ERR_INVALID_ARGUMENT;
  if (n < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n must be >= 0");
  if (G < 1 || G > tbgb::kDenseMaxGroups)
    return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "n_groups must be in [1, 1024] for the dense kernel");
  if (n > 0 && (!keys || !vals)) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "keys/values pointer is NULL");
  return TBGB_OK;
}

tbgb_status dense_common(tbgb_ctx* ctx, const int32_t* keys, const double* vals, const uint64_t* mask, int64_t n,
                         int32_t G, int64_t row_offset, const tbgb_moments* out, double* state_out, void* stream) {
  tbgb_status st = check_dense_args(ctx, keys, vals, n, G);
  if (st != TBGB_OK) return st;
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, TBGB_ERR_BACKEND, "cudaSetDevice failed");
  const tbgb::DenseLaunch L = tbgb::dense_plan(G, ctx->num_sms);
  DenseWs w = dense_ws_layout(nullptr, L, G);
  st = ensure_ws(ctx, w.bytes);
  if (st != TBGB_OK) return st;
  w = dense_ws_layout(ctx->ws, L, G);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(w.zfirst, 0xFF, static_cast<size_t>(G) * 8, s);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "memset", e);
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (ctx->profile) {
    if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess)
      return fail(ctx, TBGB_ERR_BACKEND, "cudaEventCreate failed");
    ctx->events.emplace_back(e0, e1);
  }
  e = tbgb::dense_moments_launch(L, keys, vals, mask, n, row_offset, G, w.part, w.spill, w.zfirst, ctx->err, out,
                                 state_out, s, &ctx->launches, e0, e1);
  if (e != cudaSuccess) return cuda_fail(ctx, TBGB_ERR_DISPATCH, "dense groupby launch", e);
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
  if (!ctx || n_groups < 1 || n_groups > tbgb::kDenseMaxGroups) return 0;
  const tbgb::DenseLaunch L = tbgb::dense_plan(n_groups, ctx->num_sms);
  return dense_ws_layout(nullptr, L, n_groups).bytes;
}

tbgb_status tbgb_groupby_dense(tbgb_ctx* ctx, const int32_t* d_keys, const double* d_vals, const uint64_t* d_mask,
                               int64_t n, int32_t n_groups, const tbgb_moments* out, void* stream) {
  if (!out) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "out is NULL");
  return dense_common(ctx, d_keys, d_vals, d_mask, n, n_groups, 0, out, nullptr, stream);
}

size_t tbgb_state_bytes(int32_t n_groups) {
  return n_groups > 0 ? static_cast<size_t>(tbgb::ST_COUNT) * n_groups * sizeof(double) : 0;
}

tbgb_status tbgb_groupby_dense_state(tbgb_ctx* ctx, const int32_t* d_keys, const double* d_vals,
                                     const uint64_t* d_mask, int64_t n, int32_t n_groups, int64_t row_offset,
                                     void* d_state, void* stream) {
  if (!d_state) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "state buffer is NULL");
  if (row_offset < 0) return fail(ctx, TBGB_ERR_INVALID_ARGUMENT, "row_offset must be >= 0");
  return dense_common(ctx, d_keys, d_vals, d_mask, n, n_groups, row_offset, nullptr, static_cast<double*>(d_state),
                      stream);
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

}  // extern "C"
