//! tam-gpu-b200: the reference's GPU seams over libtambear_gb.so (include/tambear_gb.h).
//!
//! * [`ffi`]: every entry point of the C ABI.
//! * [`backend::B200Backend`]: `tam_gpu::TamGpu` (crates/tam-gpu/src/lib.rs:148-199) with
//!   entry-name dispatch, so `ComputeEngine`, `DescriptiveEngine` and `AccumulateEngine` run
//!   on it unchanged (`tam_gpu::detect()` would return it ahead of the CUDA backend on sm_100).
//! * [`dispatch::scatter_step`]: the `PrimitiveOp::Scatter` arm of winrapids-compiler's
//!   `CudaKernelDispatcher` (crates/winrapids-compiler/src/cuda_dispatch.rs:199).
//!
//! Not compiled here: no Rust toolchain in this build environment.
pub mod backend;
pub mod dispatch;
pub mod ffi;

pub use backend::B200Backend;
