//! Raw declarations of every entry point of include/tambear_gb.h (the C ABI of
//! libtambear_gb.so, sm_100a).  Device pointers are plain `*const T` / `*mut T`; `stream`
//! is a `cudaStream_t` (null = the legacy default stream).
//!
//! Not compiled here: no Rust toolchain in this build environment.  `tests/test_abi.py`
//! checks that the library exports every symbol the header declares; this file mirrors the
//! header one to one.
#![allow(non_camel_case_types, dead_code)]

use std::os::raw::{c_char, c_int, c_void};

/// Opaque context: one per device, calls on one context serialised by the caller.
#[repr(C)]
pub struct tbgb_ctx {
    _private: [u8; 0],
}

/// 0 ok; 1..7 mirror `TamGpuError` (crates/tam-gpu/src/error.rs:5-20) in order;
/// 8 key out of range, 9 table full, 10 bounded device-side wait gave up.
pub type tbgb_status = c_int;
pub const TBGB_OK: tbgb_status = 0;
pub const TBGB_ERR_BACKEND: tbgb_status = 1;
pub const TBGB_ERR_COMPILE: tbgb_status = 2;
pub const TBGB_ERR_ALLOC: tbgb_status = 3;
pub const TBGB_ERR_TRANSFER: tbgb_status = 4;
pub const TBGB_ERR_DISPATCH: tbgb_status = 5;
pub const TBGB_ERR_ENTRY_NOT_FOUND: tbgb_status = 6;
pub const TBGB_ERR_INVALID_ARGUMENT: tbgb_status = 7;
pub const TBGB_ERR_KEY_OUT_OF_RANGE: tbgb_status = 8;
pub const TBGB_ERR_TABLE_FULL: tbgb_status = 9;
pub const TBGB_ERR_TIMEOUT: tbgb_status = 10;

/// Per-group outputs (device, caller-owned, one f64 per group each; null = not wanted).
#[repr(C)]
#[derive(Clone, Copy)]
pub struct tbgb_moments {
    pub count: *mut f64,
    pub sum: *mut f64,
    pub min: *mut f64,
    pub max: *mut f64,
    pub mean: *mut f64,
    pub m2: *mut f64,
    pub var_pop: *mut f64,
    pub var_samp: *mut f64,
    pub m3: *mut f64,
    pub m4: *mut f64,
}

impl Default for tbgb_moments {
    fn default() -> Self {
        let z = std::ptr::null_mut();
        Self { count: z, sum: z, min: z, max: z, mean: z, m2: z, var_pop: z, var_samp: z, m3: z, m4: z }
    }
}

pub const TBGB_F64: i32 = 0;
pub const TBGB_F32: i32 = 1;

pub const TBGB_PRED_NONE: i32 = 0;
pub const TBGB_PRED_GT: i32 = 1;
pub const TBGB_PRED_GE: i32 = 2;
pub const TBGB_PRED_LT: i32 = 3;
pub const TBGB_PRED_LE: i32 = 4;
pub const TBGB_PRED_NOT_NAN: i32 = 5;
pub const TBGB_PRED_FINITE: i32 = 6;

pub const TBGB_EXPR_A: i32 = 0;
pub const TBGB_EXPR_ADD: i32 = 1;
pub const TBGB_EXPR_SUB: i32 = 2;
pub const TBGB_EXPR_MUL: i32 = 3;
pub const TBGB_EXPR_MUL_PLUS1: i32 = 4;
pub const TBGB_EXPR_MUL_ADD: i32 = 5;

/// Value columns with the fused filter (on column a) and expression.
#[repr(C)]
#[derive(Clone, Copy)]
pub struct tbgb_columns {
    pub a: *const c_void,
    pub b: *const c_void,
    pub c: *const c_void,
    pub dtype: i32,
    pub expr: i32,
    pub pred: i32,
    pub reserved: i32,
    pub threshold: f64,
}

impl tbgb_columns {
    /// A plain f64 value column: no filter, no expression.
    pub fn plain_f64(vals: *const f64) -> Self {
        Self {
            a: vals as *const c_void,
            b: std::ptr::null(),
            c: std::ptr::null(),
            dtype: TBGB_F64,
            expr: TBGB_EXPR_A,
            pred: TBGB_PRED_NONE,
            reserved: 0,
            threshold: 0.0,
        }
    }
}

/// phi ids of `phi_scatter_eval` (crates/tambear/src/compute_engine.rs:593-609).
pub const TBGB_PHI_V: i32 = 0;
pub const TBGB_PHI_VV: i32 = 1;
pub const TBGB_PHI_ONE: i32 = 2;
pub const TBGB_PHI_VMR: i32 = 3;
pub const TBGB_PHI_VMR2: i32 = 4;
pub const TBGB_PHI_ABS_VMR: i32 = 5;
pub const TBGB_PHI_VMR3: i32 = 6;
pub const TBGB_PHI_VMR4: i32 = 7;
pub const TBGB_PHI_VR: i32 = 8;
pub const TBGB_PHI_LOG: i32 = 9;
pub const TBGB_PHI_RECIP: i32 = 10;

/// `TileColumnStats` (crates/tambear/src/format.rs:60-73), 40 bytes.
#[repr(C)]
#[derive(Clone, Copy, Default)]
pub struct tbgb_tile_stats {
    pub min: f64,
    pub max: f64,
    pub sum: f64,
    pub count: u32,
    pub n_valid: u32,
    pub reserved: u64,
}

/// Outputs of the segmented bin statistics (null = not wanted).
#[repr(C)]
#[derive(Clone, Copy)]
pub struct tbgb_bin_stats {
    pub count: *mut i32,
    pub sum: *mut f64,
    pub sum_sq: *mut f64,
    pub min: *mut f64,
    pub max: *mut f64,
    pub first: *mut f64,
    pub last: *mut f64,
    pub mean: *mut f64,
    pub variance: *mut f64,
    pub std: *mut f64,
}

extern "C" {
    // ---- context -----------------------------------------------------------------------
    pub fn tbgb_create(device: c_int, out: *mut *mut tbgb_ctx) -> tbgb_status;
    pub fn tbgb_destroy(ctx: *mut tbgb_ctx);
    pub fn tbgb_last_error(ctx: *const tbgb_ctx) -> *const c_char;
    pub fn tbgb_device_name(ctx: *const tbgb_ctx) -> *const c_char;
    pub fn tbgb_sync(ctx: *mut tbgb_ctx, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_set_table_mode(ctx: *mut tbgb_ctx, mode: c_int) -> tbgb_status;
    pub fn tbgb_workspace_bytes(ctx: *const tbgb_ctx, n: i64, n_groups: i32) -> usize;
    pub fn tbgb_launch_count(ctx: *const tbgb_ctx) -> u64;
    pub fn tbgb_profile_enable(ctx: *mut tbgb_ctx, enable: c_int) -> tbgb_status;
    pub fn tbgb_kernel_time_ms(ctx: *mut tbgb_ctx, total_ms: *mut f64, launches: *mut i64) -> tbgb_status;

    // ---- grouped moments ---------------------------------------------------------------
    pub fn tbgb_groupby_dense(ctx: *mut tbgb_ctx, keys: *const i32, vals: *const f64, mask: *const u64, n: i64,
                              n_groups: i32, out: *const tbgb_moments, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_groupby_dense_columns(ctx: *mut tbgb_ctx, keys: *const i32, cols: *const tbgb_columns,
                                      mask: *const u64, n: i64, n_groups: i32, out: *const tbgb_moments,
                                      stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_groupby_hash(ctx: *mut tbgb_ctx, keys: *const i64, cols: *const tbgb_columns, mask: *const u64,
                             n: i64, max_groups: i64, out_keys: *mut i64, out: *const tbgb_moments,
                             n_groups: *mut i64, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_groupby_dense_noalloc(keys: *const i32, vals: *const f64, mask: *const u64, n: i64, n_groups: i32,
                                      out: *const tbgb_moments, stream: *mut c_void) -> tbgb_status;

    // ---- scatter primitives (the entry names TamGpu dispatches by) ------------------------
    pub fn tbgb_scatter_phi(ctx: *mut tbgb_ctx, phi: i32, keys: *const i32, vals: *const f64, refs: *const f64,
                            n: i64, n_groups: i32, out: *mut f64, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_scatter_multi_phi(ctx: *mut tbgb_ctx, phis: *const i32, n_phi: i32, keys: *const i32,
                                  vals: *const f64, refs: *const f64, n: i64, n_groups: i32, out: *mut f64,
                                  stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_scatter_phi_masked(ctx: *mut tbgb_ctx, phi: i32, keys: *const i32, vals: *const f64,
                                   refs: *const f64, mask: *const u64, n: i64, n_groups: i32, out: *mut f64,
                                   stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_scatter_multi_phi_masked(ctx: *mut tbgb_ctx, phis: *const i32, n_phi: i32, keys: *const i32,
                                         vals: *const f64, refs: *const f64, mask: *const u64, n: i64,
                                         n_groups: i32, out: *mut f64, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_scatter_extremum(ctx: *mut tbgb_ctx, is_max: i32, keys: *const i32, vals: *const f64, n: i64,
                                 n_groups: i32, out: *mut f64, stream: *mut c_void) -> tbgb_status;

    // ---- group index and dictionary codes -------------------------------------------------
    pub fn tbgb_group_index_build(ctx: *mut tbgb_ctx, keys: *const i32, n: i64, max_key: i32,
                                  row_to_group: *mut u32, group_counts: *mut u32, group_offsets: *mut u32,
                                  rows_by_group: *mut u32, n_active: *mut i64, stream: *mut c_void)
                                  -> tbgb_status;
    pub fn tbgb_factorize_i64(ctx: *mut tbgb_ctx, keys: *const i64, n: i64, max_groups: i64, codes: *mut i32,
                              uniques: *mut i64, n_uniques: *mut i64, stream: *mut c_void) -> tbgb_status;

    // ---- masks and tile statistics --------------------------------------------------------
    pub fn tbgb_filter_mask(ctx: *mut tbgb_ctx, col: *const c_void, dtype: i32, n: i64, pred: i32, threshold: f64,
                            in_mask: *const u64, mask: *mut u64, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_mask_and(ctx: *mut tbgb_ctx, a: *const u64, b: *const u64, out: *mut u64, n_words: i64,
                         stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_mask_or(ctx: *mut tbgb_ctx, a: *const u64, b: *const u64, out: *mut u64, n_words: i64,
                        stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_mask_xor(ctx: *mut tbgb_ctx, a: *const u64, b: *const u64, out: *mut u64, n_words: i64,
                         stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_mask_not(ctx: *mut tbgb_ctx, a: *const u64, out: *mut u64, n_words: i64, n_rows: i64,
                         stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_mask_popcount(ctx: *mut tbgb_ctx, mask: *const u64, n_words: i64, n_rows: i64, count: *mut u64,
                              stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_tile_stats_build(ctx: *mut tbgb_ctx, col: *const c_void, dtype: i32, n: i64, tile_rows: i64,
                                 stats: *mut tbgb_tile_stats, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_tile_skip_mask(ctx: *mut tbgb_ctx, stats: *const tbgb_tile_stats, n_tiles: i64, pred: i32,
                               threshold: f64, skip: *mut u8, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_mask_skip_tiles(ctx: *mut tbgb_ctx, mask: *const u64, skip: *const u8, tile_rows: i64, n_rows: i64,
                                out: *mut u64, stream: *mut c_void) -> tbgb_status;

    // ---- segmented bin statistics ---------------------------------------------------------
    pub fn tbgb_fused_bin_stats(ctx: *mut tbgb_ctx, data: *const f64, n_ticks: i64, n_columns: i32,
                                boundaries: *const i64, n_bins: i64, out: *const tbgb_bin_stats,
                                stream: *mut c_void) -> tbgb_status;

    // ---- row shards: states, peer-memory exchange, owner routing -------------------------
    pub fn tbgb_state_bytes(n_groups: i32) -> usize;
    pub fn tbgb_groupby_dense_state(ctx: *mut tbgb_ctx, keys: *const i32, vals: *const f64, mask: *const u64,
                                    n: i64, n_groups: i32, row_offset: i64, state: *mut c_void,
                                    stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_merge_states(ctx: *mut tbgb_ctx, states: *const c_void, n_states: i32, n_groups: i32,
                             out: *const tbgb_moments, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_exchange_bytes(world: i32, n_groups: i32) -> usize;
    pub fn tbgb_exchange_alloc(ctx: *mut tbgb_ctx, world: i32, n_groups: i32, buf: *mut *mut c_void) -> tbgb_status;
    pub fn tbgb_exchange_free(ctx: *mut tbgb_ctx, buf: *mut c_void) -> tbgb_status;
    pub fn tbgb_peer_export(ctx: *mut tbgb_ctx, buf: *mut c_void, handle: *mut u8 /* 64 bytes */) -> tbgb_status;
    pub fn tbgb_peer_import(ctx: *mut tbgb_ctx, handle: *const u8 /* 64 bytes */, peer: *mut *mut c_void)
                            -> tbgb_status;
    pub fn tbgb_peer_close(ctx: *mut tbgb_ctx, peer: *mut c_void) -> tbgb_status;
    pub fn tbgb_ipc_alloc(ctx: *mut tbgb_ctx, bytes: usize, buf: *mut *mut c_void) -> tbgb_status;
    pub fn tbgb_ipc_free(ctx: *mut tbgb_ctx, buf: *mut c_void) -> tbgb_status;
    pub fn tbgb_groupby_dense_sharded(ctx: *mut tbgb_ctx, keys: *const i32, vals: *const f64, mask: *const u64,
                                      n: i64, n_groups: i32, row_offset: i64, rank: i32, world: i32,
                                      exchange: *const *mut c_void, epoch: u64, out: *const tbgb_moments,
                                      stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_hash_partition(ctx: *mut tbgb_ctx, keys: *const i64, cols: *const tbgb_columns, mask: *const u64,
                               n: i64, n_parts: i32, out_keys: *mut i64, out_vals: *mut f64,
                               part_counts: *mut i64, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_radix_value_bytes(cols: *const tbgb_columns) -> i32;
    pub fn tbgb_radix_fallback(ctx: *mut tbgb_ctx, bits: *mut u32) -> tbgb_status;
    pub fn tbgb_radix_route(ctx: *mut tbgb_ctx, keys: *const i64, cols: *const tbgb_columns, mask: *const u64,
                            n: i64, out_hashes: *mut u64, out_vals: *mut c_void, digit_counts: *mut i64,
                            stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_radix_groupby_routed(ctx: *mut tbgb_ctx, n_senders: i32, hashes: *const *const u64,
                                     vals: *const *const c_void, rows: *const i64, value_bytes: i32,
                                     seg_counts: *const i64, digit_lo: i32, n_digits: i32, max_groups: i64,
                                     out_keys: *mut i64, out: *const tbgb_moments, n_groups: *mut i64,
                                     stream: *mut c_void) -> tbgb_status;

    // ---- synthetic inputs (counter-based SplitMix64 streams) ------------------------------
    pub fn tbgb_gen_keys_uniform(ctx: *mut tbgb_ctx, keys: *mut i32, n: i64, n_groups: i32, seed: u64,
                                 first_row: i64, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_gen_values_uniform(ctx: *mut tbgb_ctx, vals: *mut f64, n: i64, lo: f64, hi: f64, seed: u64,
                                   first_row: i64, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_gen_values_normal(ctx: *mut tbgb_ctx, vals: *mut f64, n: i64, mu: f64, sigma: f64, seed: u64,
                                  first_row: i64, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_gen_inject_nonfinite(ctx: *mut tbgb_ctx, vals: *mut f64, n: i64, nan_frac: f64, inf_frac: f64,
                                     seed: u64, first_row: i64, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_gen_keys_cdf(ctx: *mut tbgb_ctx, keys: *mut i64, n: i64, cdf: *const f64, n_ids: i64, salt: u64,
                             seed: u64, first_row: i64, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_gen_keys_ids(ctx: *mut tbgb_ctx, keys: *mut i64, n: i64, n_ids: i64, salt: u64, seed: u64,
                             first_row: i64, stream: *mut c_void) -> tbgb_status;
    pub fn tbgb_gen_values_lognormal_f32(ctx: *mut tbgb_ctx, vals: *mut f32, n: i64, mu: f64, sigma: f64,
                                         seed: u64, first_row: i64, stream: *mut c_void) -> tbgb_status;
}
