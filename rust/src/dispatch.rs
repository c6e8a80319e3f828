//! The `PrimitiveOp::Scatter` arm of winrapids-compiler's CUDA dispatcher
//! (`CudaKernelDispatcher::dispatch`, crates/winrapids-compiler/src/cuda_dispatch.rs:199,
//! today the "not yet dispatched" error arm).  Inputs arrive as `BufferPtr { device_ptr,
//! byte_size }` (crates/winrapids-store/src/header.rs:138-143); the step's params name the
//! aggregate.  The arm calls the B200 groupby and returns the output's `BufferPtr`; the
//! dispatcher keeps the output allocation alive, as it does for its fused outputs.
//!
//! Not compiled here: no Rust toolchain in this build environment.
//!
//! Wiring (in cuda_dispatch.rs, before the `other =>` arm):
//! ```ignore
//! PrimitiveOp::Scatter => {
//!     let (ptr, owned) = tam_gpu_b200::dispatch::scatter_step(&self.b200, params, input_ptrs)?;
//!     self.fused_outputs.push(owned);
//!     Ok(ptr)
//! }
//! ```
use std::os::raw::c_void;

use winrapids_store::header::BufferPtr;

use crate::backend::{phi_id, B200Backend};
use crate::ffi;

/// Device memory the dispatcher must keep alive while the store refers to it.
pub struct OwnedOutput {
    pub ptr: *mut c_void,
    pub bytes: usize,
}
unsafe impl Send for OwnedOutput {}
impl Drop for OwnedOutput {
    fn drop(&mut self) {
        extern "C" {
            fn cudaFree(p: *mut c_void) -> i32;
        }
        if !self.ptr.is_null() {
            unsafe { cudaFree(self.ptr) };
        }
    }
}

fn param<'a>(params: &'a [(String, String)], key: &str) -> Option<&'a str> {
    params.iter().find(|(k, _)| k == key).map(|(_, v)| v.as_str())
}

/// One Scatter step.  Inputs: `[keys:i32, values:f64]` (+ `mask:u64` when the step has
/// `masked=1`).  Params: `n_groups`, and `agg` = one of `sum`, `count`, `mean`, `min`, `max`,
/// `var` (ddof 1), `var_pop`, or `phi` = a phi spelling of phi_scatter_eval (summed per group).
/// Output: one f64 per group.
pub fn scatter_step(
    b200: &B200Backend,
    params: &[(String, String)],
    inputs: &[BufferPtr],
) -> Result<(BufferPtr, OwnedOutput), Box<dyn std::error::Error>> {
    extern "C" {
        fn cudaMalloc(p: *mut *mut c_void, bytes: usize) -> i32;
    }
    if inputs.len() < 2 {
        return Err("Scatter needs keys and values".into());
    }
    let n_groups: i32 = param(params, "n_groups").ok_or("Scatter step missing 'n_groups'")?.parse()?;
    let masked = param(params, "masked") == Some("1");
    let keys = inputs[0].device_ptr as *const i32;
    let n = (inputs[0].byte_size / 4) as i64;
    let vals = inputs[1].device_ptr as *const f64;
    if (inputs[1].byte_size / 8) as i64 != n {
        return Err("Scatter: keys and values differ in length".into());
    }
    let mask = if masked {
        inputs.get(2).ok_or("masked Scatter needs a mask input")?.device_ptr as *const u64
    } else {
        std::ptr::null()
    };
    let bytes = n_groups as usize * 8;
    let mut out: *mut c_void = std::ptr::null_mut();
    if unsafe { cudaMalloc(&mut out, bytes) } != 0 {
        return Err("Scatter: output allocation failed".into());
    }
    let owned = OwnedOutput { ptr: out, bytes };
    let o = out as *mut f64;
    b200.with_ctx(|ctx| {
        let st = if let Some(phi) = param(params, "phi") {
            let id = phi_id(phi)?;
            unsafe {
                if masked {
                    ffi::tbgb_scatter_phi_masked(ctx, id, keys, vals, std::ptr::null(), mask, n, n_groups, o,
                                                 std::ptr::null_mut())
                } else {
                    ffi::tbgb_scatter_phi(ctx, id, keys, vals, std::ptr::null(), n, n_groups, o, std::ptr::null_mut())
                }
            }
        } else {
            let mut m = ffi::tbgb_moments::default();
            match param(params, "agg").unwrap_or("sum") {
                "sum" => m.sum = o,
                "count" => m.count = o,
                "mean" => m.mean = o,
                "min" => m.min = o,
                "max" => m.max = o,
                "var" => m.var_samp = o,
                "var_pop" => m.var_pop = o,
                other => {
                    return Err(tam_gpu::TamGpuError::EntryNotFound(format!("Scatter aggregate '{other}'")))
                }
            }
            unsafe { ffi::tbgb_groupby_dense(ctx, keys, vals, mask, n, n_groups, &m, std::ptr::null_mut()) }
        };
        if st != ffi::TBGB_OK {
            return Err(tam_gpu::TamGpuError::Dispatch(format!("Scatter step failed with status {st}")));
        }
        let st = unsafe { ffi::tbgb_sync(ctx, std::ptr::null_mut()) };
        if st != ffi::TBGB_OK {
            return Err(tam_gpu::TamGpuError::Dispatch(format!("Scatter step failed with status {st}")));
        }
        Ok(())
    })?;
    Ok((BufferPtr { device_ptr: out as u64, byte_size: bytes as u64 }, owned))
}
