/*
 * tambear_gb.h -- C ABI of the B200 (sm_100a) groupby-aggregate path.
 *
 * Drop-in boundary for the reference's groupby/accumulate operator API.  Every
 * entry point takes plain pointers and sizes; no exceptions cross the ABI; all
 * device memory passed in is owned by the caller (the reference's
 * winrapids-store BufferPtr convention, crates/winrapids-store/src/header.rs:138-143),
 * while scratch ("workspace") is owned by the context and sized on demand.
 *
 * Reference interfaces replaced (paths relative to the reference project root):
 *   tbgb_create / tbgb_destroy      tam_gpu::detect() + CudaBackend::new
 *                                   (crates/tam-gpu/src/lib.rs:214, crates/tam-gpu/src/cuda.rs:111)
 *   tbgb_status                     tam_gpu::TamGpuError (crates/tam-gpu/src/error.rs:5-20)
 *   tbgb_groupby_dense              DescriptiveEngine::moments_grouped
 *                                   (crates/tambear/src/descriptive.rs:383-435) and
 *                                   HashScatterEngine::groupby (crates/tambear/src/hash_scatter.rs:367)
 *   tbgb_groupby_dense_state /      MomentStats::merge / SufficientStatistics::merge
 *   tbgb_merge_states               (descriptive.rs:216-253, intermediates.rs:352-377) used
 *                                   across row shards (one partial table per GPU)
 *
 * Threading: one context per device; calls on one context are serialised by the
 * caller (the context's workspace is reused by every call); different contexts
 * are independent.
 */
#ifndef TAMBEAR_GB_H
#define TAMBEAR_GB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  1..7 mirror TamGpuError's variants in order. */
typedef enum {
  TBGB_OK = 0,
  TBGB_ERR_BACKEND = 1,           /* TamGpuError::Backend: driver / runtime failure        */
  TBGB_ERR_COMPILE = 2,           /* TamGpuError::Compile: never produced (no runtime JIT) */
  TBGB_ERR_ALLOC = 3,             /* TamGpuError::Alloc                                    */
  TBGB_ERR_TRANSFER = 4,          /* TamGpuError::Transfer                                 */
  TBGB_ERR_DISPATCH = 5,          /* TamGpuError::Dispatch: launch failure                 */
  TBGB_ERR_ENTRY_NOT_FOUND = 6,   /* TamGpuError::EntryNotFound: unknown entry / phi       */
  TBGB_ERR_INVALID_ARGUMENT = 7,  /* TamGpuError::InvalidArgument                          */
  TBGB_ERR_KEY_OUT_OF_RANGE = 8,  /* a key outside [0, n_groups) (the reference panics)    */
  TBGB_ERR_TABLE_FULL = 9,        /* hash table could not place a key                      */
  TBGB_ERR_TIMEOUT = 10           /* a bounded device-side wait gave up                    */
} tbgb_status;

typedef struct tbgb_ctx tbgb_ctx;

/* Create a context on CUDA device `device` (the process's current device is
 * left unchanged).  Fails with TBGB_ERR_BACKEND when no sm_100 device is present:
 * there is no CPU fallback. */
tbgb_status tbgb_create(int device, tbgb_ctx** out);
void tbgb_destroy(tbgb_ctx* ctx);
/* Message for the last failing call on `ctx` (valid until the next call). */
const char* tbgb_last_error(const tbgb_ctx* ctx);
/* "NVIDIA B200 (CUDA sm_100)" style label (TamGpu::name, crates/tam-gpu/src/lib.rs:155). */
const char* tbgb_device_name(const tbgb_ctx* ctx);

/* Per-group outputs of the grouped moments, one double per group each, device
 * pointers owned by the caller; any pointer may be NULL to skip that output.
 * Semantics follow DescriptiveEngine::moments_grouped + MomentStats:
 *   count    rows whose value is not NaN (+-inf rows count)
 *   sum      sum of the finite values (Kulisch skips +-inf), +0.0 when empty
 *   min/max  over non-NaN values, +inf / -inf when empty; +-0 ties resolved as a
 *            sequential `v < acc` scan in row order would
 *   mean     sum / count, NaN when count == 0
 *   m2       sum over finite values of (v - r)^2 with r = sum/count (0.0 when empty)
 *   var_pop  m2 / count, NaN when count == 0;  var_samp  m2 / (count - 1), NaN when count <= 1 */
typedef struct {
  double* count;
  double* sum;
  double* min;
  double* max;
  double* mean;
  double* m2;
  double* var_pop;
  double* var_samp;
} tbgb_moments;

/* Dense-key groupby: keys in [0, n_groups), f64 values, optional row mask
 * (bit i of mask[i/64] set <=> row i participates, filter_jit.rs:202-243 layout;
 * NULL = all rows).  Enqueued on `stream` (a cudaStream_t, NULL = legacy default
 * stream); returns after the launch.  Deferred device errors (key out of range,
 * timeouts) are reported by tbgb_sync.  Requires 1 <= n_groups <= 1024 in this
 * version (TBGB_ERR_INVALID_ARGUMENT otherwise). */
tbgb_status tbgb_groupby_dense(tbgb_ctx* ctx, const int32_t* d_keys, const double* d_vals, const uint64_t* d_mask,
                               int64_t n, int32_t n_groups, const tbgb_moments* out, void* stream);

/* Waits for `stream` and returns the first deferred device error of the calls
 * enqueued since the previous tbgb_sync (then clears it). */
tbgb_status tbgb_sync(tbgb_ctx* ctx, void* stream);

/* ---- row-sharded execution (one process / GPU per shard) ------------------------
 * A shard computes its mergeable per-group state table (tbgb_state_bytes(n_groups)
 * bytes, caller-owned device memory); the caller exchanges the tables (e.g. an
 * NCCL all-gather over NVLink) and folds them in rank order with
 * tbgb_merge_states.  `row_offset` is the global index of the shard's first row
 * (used only to order +-0 ties exactly as the unsharded scan would). */
size_t tbgb_state_bytes(int32_t n_groups);
tbgb_status tbgb_groupby_dense_state(tbgb_ctx* ctx, const int32_t* d_keys, const double* d_vals,
                                     const uint64_t* d_mask, int64_t n, int32_t n_groups, int64_t row_offset,
                                     void* d_state, void* stream);
tbgb_status tbgb_merge_states(tbgb_ctx* ctx, const void* d_states, int32_t n_states, int32_t n_groups,
                              const tbgb_moments* out, void* stream);

/* Dense-key groupby that allocates no device memory and needs no context: for
 * callers that must not have the library allocate at call time (for example a host
 * engine that has already reserved nearly all device memory for its own buffers,
 * or a latency-critical loop that cannot accept cudaMalloc's implicit device
 * synchronisation).  No counterpart in the reference.
 * Same semantics and outputs as tbgb_groupby_dense, on the current device.
 * Limits: 1 <= n_groups <= 256 (TBGB_ERR_INVALID_ARGUMENT otherwise).  Scratch is
 * a fixed device array of about 8.5 MB inside this library, held by every GPU that
 * loads the library until the process exits.  The first call on a device looks up
 * that array's address (make it before any stream capture).  All calls share the
 * array: calls that overlap on the GPU (other streams, other threads) race and
 * must be serialised by the caller.  The call waits for `stream` and returns any
 * device-side error (e.g. TBGB_ERR_KEY_OUT_OF_RANGE). */
tbgb_status tbgb_groupby_dense_noalloc(const int32_t* d_keys, const double* d_vals, const uint64_t* d_mask,
                                       int64_t n, int32_t n_groups, const tbgb_moments* out, void* stream);

/* Bytes of device workspace the context holds after a call of this size. */
size_t tbgb_workspace_bytes(const tbgb_ctx* ctx, int64_t n, int32_t n_groups);

/* Number of this library's kernel launches issued through `ctx` so far. */
uint64_t tbgb_launch_count(const tbgb_ctx* ctx);

/* Kernel timing: while enabled, the context records CUDA events on the launching
 * stream around each main groupby kernel.  tbgb_kernel_time_ms waits for them and
 * returns (and resets) the summed duration and the number of timed launches. */
tbgb_status tbgb_profile_enable(tbgb_ctx* ctx, int enable);
tbgb_status tbgb_kernel_time_ms(tbgb_ctx* ctx, double* total_ms, int64_t* launches);

/* ---- synthetic inputs (counter-based SplitMix64 streams) ------------------------
 * Row i of column c uses the i-th output of SplitMix64 seeded with
 * mix64(seed ^ (0xD1B54A32D192ED03 * (c + 1))) (rng.rs:64-85 stream, u01 = (x >> 11) * 2^-53).
 *   keys: x % n_groups                                   (column 0)
 *   uniform values: lo + (hi - lo) * u01                 (column 1)
 *   normal values: mu + sigma * sqrt(-2 ln u1) cos(2 pi u2), u1/u2 = outputs 2i, 2i+1 (column 1)
 * Element j of the output holds row first_row + j, so each shard of a dataset can
 * be generated where it lives. */
tbgb_status tbgb_gen_keys_uniform(tbgb_ctx* ctx, int32_t* d_keys, int64_t n, int32_t n_groups, uint64_t seed,
                                  int64_t first_row, void* stream);
tbgb_status tbgb_gen_values_uniform(tbgb_ctx* ctx, double* d_vals, int64_t n, double lo, double hi,
                                    uint64_t seed, int64_t first_row, void* stream);
tbgb_status tbgb_gen_values_normal(tbgb_ctx* ctx, double* d_vals, int64_t n, double mu, double sigma,
                                   uint64_t seed, int64_t first_row, void* stream);
/* Replace a fraction of values by NaN (u < nan_frac) and +-inf
 * (nan_frac <= u < nan_frac + inf_frac, sign from the low bit), u from column 2. */
tbgb_status tbgb_gen_inject_nonfinite(tbgb_ctx* ctx, double* d_vals, int64_t n, double nan_frac, double inf_frac,
                                      uint64_t seed, int64_t first_row, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TAMBEAR_GB_H */
