//! Host change 4: `clove_paged_attention` of src/ffi.rs:247-266 keeps its
//! signature and forwards CUDA tensors to `CudaBackend`; tensors of the other
//! backends keep their old route.  Not compiled in this repository (no Rust
//! toolchain here).  The same C-level behaviour is what libclove_cuda.so
//! exports itself under include/clove_ffi.h (ffi.cu), which a C or Python
//! caller can use without the crate.
//!
//! In src/ffi.rs the body becomes:
//!
//! ```ignore
//! #[unsafe(no_mangle)]
//! pub unsafe extern "C" fn clove_paged_attention(q: CTensor, k: CTensor, v: CTensor, kv: CTensor,
//!                                                bt: CTensor, cl: CTensor) -> CTensor {
//!     unsafe {
//!         if is_cuda(as_node(kv)) {
//!             return match cuda_paged_attention(as_node(q), as_node(k), as_node(v), as_node(kv),
//!                                               as_node(bt), as_node(cl)) {
//!                 Ok(t) => into_raw(t),
//!                 Err(e) => { set_ffi_error(e); std::ptr::null_mut() } // NULL + text, no abort
//!             };
//!         }
//!         into_raw(WgpuBackend::paged_attention(as_node(q), as_node(k), as_node(v), as_node(kv),
//!                                               as_node(bt), as_node(cl)))
//!     }
//! }
//! ```
use std::os::raw::c_void;

use crate::cuda_backend::{CudaBackend, CudaBuffer};
use crate::cuda_ffi::CLOVE_DTYPE_F32;

/// Allocates the f32 [B, Hq * D] output, runs the append + decode on the
/// default stream, and reports the decode's device check flags as an error
/// (a clamped block id is an error, not a result).
pub fn cuda_paged_attention(backend: &CudaBackend, q: &CudaBuffer, k: &CudaBuffer, v: &CudaBuffer, kv: &CudaBuffer,
                            bt: &CudaBuffer, cl: &CudaBuffer) -> Result<CudaBuffer, String> {
    let batch = cl.shape[0];
    let width = q.shape[1];
    let mut out = CudaBuffer {
        ptr: unsafe { crate::cuda_rt::malloc(q.device, batch * width * 4)? },
        bytes: batch * width * 4,
        dtype: CLOVE_DTYPE_F32,
        device: q.device,
        shape: vec![batch, width],
    };
    let max_ctx = bt.shape[1] * kv.shape[2]; // table capacity: no device-to-host read of the lengths
    let stream: *mut c_void = std::ptr::null_mut();
    backend.paged_attention_raw(q, k, v, kv, bt, cl, &mut out, max_ctx, stream)?;
    match backend.decode_flags(kv, stream)? {
        0 => Ok(out),
        f => Err(format!("paged_attention: device check flags {f:#x}")),
    }
}
