//! `B200Backend`: the reference's `TamGpu` trait (crates/tam-gpu/src/lib.rs:148-199) over
//! libtambear_gb.so.  Kernels are chosen by entry name, as `CpuBackend::compile` does
//! (crates/tam-gpu/src/cpu.rs:101-194): `compile` parses the phi list (and, for the engine's
//! CUDA sources, `#define PARAM_N`) out of the source text and returns a tag; `dispatch` calls
//! the matching C entry point with the buffers in the reference's order.  No NVRTC, no source
//! is compiled at run time: grid / block / shared_mem are ignored (the library sizes its own
//! launches for sm_100a).
//!
//! Not compiled here: no Rust toolchain in this build environment.
use std::ffi::CStr;
use std::os::raw::c_void;
use std::sync::Mutex;

use tam_gpu::{Backend, Buffer, Kernel, ShaderLang, TamGpu, TamGpuError, TamResult};

use crate::ffi;

// The few CUDA runtime calls the buffer plumbing needs (libcudart, linked by build.rs).
extern "C" {
    fn cudaMalloc(ptr: *mut *mut c_void, bytes: usize) -> i32;
    fn cudaFree(ptr: *mut c_void) -> i32;
    fn cudaMemset(ptr: *mut c_void, value: i32, bytes: usize) -> i32;
    fn cudaMemcpy(dst: *mut c_void, src: *const c_void, bytes: usize, kind: i32) -> i32;
    fn cudaDeviceSynchronize() -> i32;
    fn cudaSetDevice(device: i32) -> i32;
}
const H2D: i32 = 1;
const D2H: i32 = 2;

/// Device allocation owned by a `tam_gpu::Buffer` (freed on drop, like `CudaBackend`'s buffers).
pub struct B200Buffer {
    pub ptr: *mut c_void,
    pub bytes: usize,
}
unsafe impl Send for B200Buffer {}
unsafe impl Sync for B200Buffer {}
impl Drop for B200Buffer {
    fn drop(&mut self) {
        if !self.ptr.is_null() {
            unsafe { cudaFree(self.ptr) };
        }
    }
}

/// What `compile` resolved: the entry and its phi ids (or the extremum direction).
#[derive(Clone, Debug)]
pub struct B200Kernel {
    pub entry: String,
    pub phis: Vec<i32>,
    pub is_max: bool,
    pub n: Option<usize>,
}

pub struct B200Backend {
    ctx: Mutex<*mut ffi::tbgb_ctx>,
    device: i32,
    name: String,
}
unsafe impl Send for B200Backend {}
unsafe impl Sync for B200Backend {}

/// `tbgb_status` -> `TamGpuError`: 1..7 are TamGpuError's variants in order; the library's
/// own statuses (8 key out of range, 9 table full, 10 timeout) map to InvalidArgument /
/// Alloc / Backend with the library's message.
fn status(ctx: *mut ffi::tbgb_ctx, st: ffi::tbgb_status) -> TamResult<()> {
    if st == ffi::TBGB_OK {
        return Ok(());
    }
    let msg = unsafe {
        let p = ffi::tbgb_last_error(ctx);
        if p.is_null() { String::new() } else { CStr::from_ptr(p).to_string_lossy().into_owned() }
    };
    Err(match st {
        ffi::TBGB_ERR_BACKEND | ffi::TBGB_ERR_TIMEOUT => TamGpuError::Backend(msg),
        ffi::TBGB_ERR_COMPILE => TamGpuError::Compile(msg),
        ffi::TBGB_ERR_ALLOC | ffi::TBGB_ERR_TABLE_FULL => TamGpuError::Alloc(msg),
        ffi::TBGB_ERR_TRANSFER => TamGpuError::Transfer(msg),
        ffi::TBGB_ERR_DISPATCH => TamGpuError::Dispatch(msg),
        ffi::TBGB_ERR_ENTRY_NOT_FOUND => TamGpuError::EntryNotFound(msg),
        _ => TamGpuError::InvalidArgument(format!("status {st}: {msg}")),
    })
}

/// phi spellings of `phi_scatter_eval` (crates/tambear/src/compute_engine.rs:593-609).
pub fn phi_id(phi: &str) -> TamResult<i32> {
    let p: String = phi.split_whitespace().collect::<Vec<_>>().join(" ");
    Ok(match p.as_str() {
        "v" => ffi::TBGB_PHI_V,
        "v * v" => ffi::TBGB_PHI_VV,
        "1.0" => ffi::TBGB_PHI_ONE,
        "v - r" | "(v - r)" => ffi::TBGB_PHI_VMR,
        "(v - r) * (v - r)" => ffi::TBGB_PHI_VMR2,
        "fabs(v - r)" | "abs(v - r)" => ffi::TBGB_PHI_ABS_VMR,
        "(v - r) * (v - r) * (v - r)" => ffi::TBGB_PHI_VMR3,
        "(v - r) * (v - r) * (v - r) * (v - r)" => ffi::TBGB_PHI_VMR4,
        "v * r" => ffi::TBGB_PHI_VR,
        "log(v)" => ffi::TBGB_PHI_LOG,
        "1.0 / v" => ffi::TBGB_PHI_RECIP,
        other => return Err(TamGpuError::EntryNotFound(format!("phi '{other}' has no B200 kernel"))),
    })
}

/// The phi list of a kernel source, in either spelling the reference emits:
/// the CPU registry's first-line comment (`// Scatter multi-phi kernel: v|v * v|1.0`), or the
/// CUDA emitters' `// phi = <expr>` line / `atomicAdd(&out<j>[g], (<expr>));` lines
/// (crates/tambear/src/compute_engine.rs:689-760).
fn parse_phis(source: &str) -> Vec<String> {
    let mut phis = Vec::new();
    for line in source.lines() {
        let l = line.trim();
        if let Some(rest) = l.strip_prefix("// phi = ") {
            phis.push(rest.trim().to_string());
        } else if l.starts_with("atomicAdd(&out") {
            if let (Some(a), Some(b)) = (l.find(", ("), l.rfind("));")) {
                if a + 3 <= b {
                    phis.push(l[a + 3..b].trim().to_string());
                }
            }
        }
    }
    if phis.is_empty() {
        if let Some(rest) = source.lines().next().and_then(|f| f.rsplit("kernel: ").next()) {
            phis = rest.split('|').map(|s| s.trim().to_string()).filter(|s| !s.is_empty()).collect();
        }
    }
    phis
}

fn parse_param_n(source: &str) -> Option<usize> {
    source.lines().find_map(|l| l.trim().strip_prefix("#define PARAM_N ").and_then(|v| v.trim().parse().ok()))
}

impl B200Backend {
    /// A backend on CUDA device `device`; fails (no CPU fallback) without an sm_100 device.
    pub fn new(device: i32) -> TamResult<Self> {
        let mut ctx: *mut ffi::tbgb_ctx = std::ptr::null_mut();
        let st = unsafe { ffi::tbgb_create(device, &mut ctx) };
        if st != ffi::TBGB_OK {
            return Err(TamGpuError::Backend(format!("tbgb_create({device}) failed with status {st}")));
        }
        let name = unsafe { CStr::from_ptr(ffi::tbgb_device_name(ctx)).to_string_lossy().into_owned() };
        Ok(Self { ctx: Mutex::new(ctx), device, name })
    }

    /// The context for one call (calls on one context are serialised, as the ABI requires).
    pub fn with_ctx<R>(&self, f: impl FnOnce(*mut ffi::tbgb_ctx) -> TamResult<R>) -> TamResult<R> {
        let guard = self.ctx.lock().map_err(|_| TamGpuError::Backend("context lock poisoned".into()))?;
        f(*guard)
    }

    fn dev(buf: &Buffer) -> TamResult<&B200Buffer> {
        buf.downcast_inner::<B200Buffer>()
            .ok_or_else(|| TamGpuError::InvalidArgument("buffer does not belong to the B200 backend".into()))
    }
}

impl Drop for B200Backend {
    fn drop(&mut self) {
        if let Ok(g) = self.ctx.lock() {
            unsafe { ffi::tbgb_destroy(*g) };
        }
    }
}

impl TamGpu for B200Backend {
    fn name(&self) -> String {
        self.name.clone()
    }

    fn backend(&self) -> Backend {
        Backend::Cuda
    }

    fn shader_lang(&self) -> ShaderLang {
        ShaderLang::Cuda
    }

    fn compile(&self, source: &str, entry: &str) -> TamResult<Kernel> {
        let k = match entry {
            "scatter_phi" | "scatter_phi_masked" | "scatter_multi_phi" | "scatter_multi_phi_masked" => {
                let phis = parse_phis(source);
                if phis.is_empty() {
                    return Err(TamGpuError::Compile(format!("{entry}: no phi expression in the source")));
                }
                if !entry.contains("multi") && phis.len() != 1 {
                    return Err(TamGpuError::Compile(format!("{entry}: expected one phi, found {}", phis.len())));
                }
                B200Kernel {
                    entry: entry.to_string(),
                    phis: phis.iter().map(|p| phi_id(p)).collect::<TamResult<Vec<_>>>()?,
                    is_max: false,
                    n: parse_param_n(source),
                }
            }
            "scatter_extremum" => B200Kernel {
                entry: entry.to_string(),
                phis: vec![],
                is_max: source.contains("(max)") || source.contains("fmax"),
                n: parse_param_n(source),
            },
            other => {
                return Err(TamGpuError::EntryNotFound(format!(
                    "B200Backend has no kernel '{other}'. Supported: scatter_phi, scatter_multi_phi, \
                     scatter_phi_masked, scatter_multi_phi_masked, scatter_extremum"
                )))
            }
        };
        Ok(Kernel::new(Box::new(k), entry))
    }

    fn alloc(&self, bytes: usize) -> TamResult<Buffer> {
        let mut p: *mut c_void = std::ptr::null_mut();
        unsafe {
            cudaSetDevice(self.device);
            if bytes > 0 && cudaMalloc(&mut p, bytes) != 0 {
                return Err(TamGpuError::Alloc(format!("cudaMalloc({bytes}) failed")));
            }
            if bytes > 0 && cudaMemset(p, 0, bytes) != 0 {
                cudaFree(p);
                return Err(TamGpuError::Alloc("cudaMemset failed".into()));
            }
        }
        Ok(Buffer::new(Box::new(B200Buffer { ptr: p, bytes }), bytes))
    }

    fn free(&self, buf: Buffer) -> TamResult<()> {
        drop(buf);
        Ok(())
    }

    fn copy_h2d(&self, src: &[u8], dst: &Buffer) -> TamResult<()> {
        let d = Self::dev(dst)?;
        if src.len() > d.bytes {
            return Err(TamGpuError::InvalidArgument("host slice larger than the buffer".into()));
        }
        match unsafe { cudaMemcpy(d.ptr, src.as_ptr() as *const c_void, src.len(), H2D) } {
            0 => Ok(()),
            e => Err(TamGpuError::Transfer(format!("cudaMemcpy H2D failed ({e})"))),
        }
    }

    fn copy_d2h(&self, src: &Buffer, dst: &mut [u8]) -> TamResult<()> {
        let s = Self::dev(src)?;
        if dst.len() > s.bytes {
            return Err(TamGpuError::InvalidArgument("host slice larger than the buffer".into()));
        }
        match unsafe { cudaMemcpy(dst.as_mut_ptr() as *mut c_void, s.ptr, dst.len(), D2H) } {
            0 => Ok(()),
            e => Err(TamGpuError::Transfer(format!("cudaMemcpy D2H failed ({e})"))),
        }
    }

    /// Buffers in the reference's order (crates/tam-gpu/src/cpu.rs:9-20, compute_engine.rs:360-510):
    /// scatter_phi `[keys, values, refs, out]`; scatter_multi_phi `[keys, values, refs, out0..]`;
    /// scatter_phi_masked `[keys, values, refs, mask, out]`; scatter_multi_phi_masked
    /// `[keys, values, refs, mask, out0..]`; scatter_extremum `[keys, values, out]` (out
    /// pre-filled with -inf / +inf, which the library's result overwrites).
    fn dispatch(&self, kernel: &Kernel, _grid: [u32; 3], _block: [u32; 3], bufs: &[&Buffer],
                _shared_mem: u32) -> TamResult<()> {
        let k = kernel
            .downcast_inner::<B200Kernel>()
            .ok_or_else(|| TamGpuError::Dispatch("kernel was not compiled by the B200 backend".into()))?;
        let need = |m: usize| -> TamResult<()> {
            if bufs.len() < m {
                Err(TamGpuError::Dispatch(format!("{} needs {m} buffers, got {}", k.entry, bufs.len())))
            } else {
                Ok(())
            }
        };
        let ptr = |i: usize| -> TamResult<*mut c_void> { Ok(Self::dev(bufs[i])?.ptr) };
        let keys_n = |i: usize| -> TamResult<i64> {
            let n = (Self::dev(bufs[i])?.bytes / 4) as i64;
            Ok(k.n.map(|p| p as i64).unwrap_or(n).min(n))
        };
        let null = std::ptr::null_mut::<c_void>();
        self.with_ctx(|ctx| {
            let st = match k.entry.as_str() {
                "scatter_phi" | "scatter_phi_masked" => {
                    let masked = k.entry.ends_with("masked");
                    need(if masked { 5 } else { 4 })?;
                    let out_i = if masked { 4 } else { 3 };
                    let g = (Self::dev(bufs[out_i])?.bytes / 8) as i32;
                    let n = keys_n(0)?;
                    unsafe {
                        if masked {
                            ffi::tbgb_scatter_phi_masked(ctx, k.phis[0], ptr(0)? as _, ptr(1)? as _, ptr(2)? as _,
                                                         ptr(3)? as _, n, g, ptr(4)? as _, null)
                        } else {
                            ffi::tbgb_scatter_phi(ctx, k.phis[0], ptr(0)? as _, ptr(1)? as _, ptr(2)? as _, n, g,
                                                  ptr(3)? as _, null)
                        }
                    }
                }
                "scatter_multi_phi" | "scatter_multi_phi_masked" => {
                    let masked = k.entry.ends_with("masked");
                    let first = if masked { 4 } else { 3 };
                    let m = k.phis.len();
                    need(first + m)?;
                    let g = (Self::dev(bufs[first])?.bytes / 8) as i32;
                    let n = keys_n(0)?;
                    // the library writes the n_phi outputs contiguously: one scratch, then copies
                    let scratch = self.alloc(m * g as usize * 8)?;
                    let sp = Self::dev(&scratch)?.ptr;
                    let st = unsafe {
                        if masked {
                            ffi::tbgb_scatter_multi_phi_masked(ctx, k.phis.as_ptr(), m as i32, ptr(0)? as _,
                                                               ptr(1)? as _, ptr(2)? as _, ptr(3)? as _, n, g,
                                                               sp as _, null)
                        } else {
                            ffi::tbgb_scatter_multi_phi(ctx, k.phis.as_ptr(), m as i32, ptr(0)? as _,
                                                        ptr(1)? as _, ptr(2)? as _, n, g, sp as _, null)
                        }
                    };
                    status(ctx, st)?;
                    status(ctx, unsafe { ffi::tbgb_sync(ctx, null) })?;
                    for j in 0..m {
                        let src = unsafe { (sp as *mut u8).add(j * g as usize * 8) } as *const c_void;
                        if unsafe { cudaMemcpy(ptr(first + j)?, src, g as usize * 8, 3 /* D2D */) } != 0 {
                            return Err(TamGpuError::Transfer("output copy failed".into()));
                        }
                    }
                    ffi::TBGB_OK
                }
                "scatter_extremum" => {
                    need(3)?;
                    let g = (Self::dev(bufs[2])?.bytes / 8) as i32;
                    let n = keys_n(0)?;
                    unsafe {
                        ffi::tbgb_scatter_extremum(ctx, k.is_max as i32, ptr(0)? as _, ptr(1)? as _, n, g,
                                                   ptr(2)? as _, null)
                    }
                }
                other => return Err(TamGpuError::EntryNotFound(other.to_string())),
            };
            status(ctx, st)
        })
    }

    fn sync(&self) -> TamResult<()> {
        self.with_ctx(|ctx| {
            status(ctx, unsafe { ffi::tbgb_sync(ctx, std::ptr::null_mut()) })?;
            match unsafe { cudaDeviceSynchronize() } {
                0 => Ok(()),
                e => Err(TamGpuError::Backend(format!("cudaDeviceSynchronize failed ({e})"))),
            }
        })
    }
}
