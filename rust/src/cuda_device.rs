//! Host change 3: CUDA devices in `EngineDevice` (src/device.rs:34-61), the
//! module a maintainer merges into src/device.rs.  Not compiled in this
//! repository (no Rust toolchain here).
//!
//! ```ignore
//! pub enum EngineDevice {
//!     Cpu { cores: usize },
//!     Gpu { device: Arc<wgpu::Device>, queue: Arc<wgpu::Queue> },
//!     // ... the reference's other variants ...
//!     /// One B200 (or any sm_100a GPU) driven by libclove_cuda.so.
//!     Cuda { ordinal: i32 },
//! }
//! ```
use crate::cuda_backend::cuda_devices;

/// `EngineDevice::init` prefers CUDA devices when the library finds any
/// (replaces the adapter probe of src/device.rs:79-150 for the CUDA build):
/// one `Cuda { ordinal }` per GPU, sequences sharded over them with the
/// reference's `distribute_batch` rule (src/distributed.rs:184-200).
pub fn cuda_ordinals_or_none() -> Option<Vec<i32>> {
    match cuda_devices() {
        Ok(v) if !v.is_empty() => Some(v),
        _ => None,
    }
}
