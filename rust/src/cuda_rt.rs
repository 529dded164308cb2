//! The few CUDA runtime calls the crate's CUDA backend makes itself (buffer
//! allocation for tensors and the decode scratch).  Not compiled in this
//! repository (no Rust toolchain here).
use std::os::raw::{c_int, c_void};

#[link(name = "cudart")]
unsafe extern "C" {
    fn cudaSetDevice(device: c_int) -> c_int;
    fn cudaMalloc(ptr: *mut *mut c_void, bytes: usize) -> c_int;
    fn cudaMemset(ptr: *mut c_void, value: c_int, bytes: usize) -> c_int;
    fn cudaFree(ptr: *mut c_void) -> c_int;
}

pub unsafe fn malloc(device: i32, bytes: usize) -> Result<*mut c_void, String> {
    let mut p: *mut c_void = std::ptr::null_mut();
    unsafe {
        if cudaSetDevice(device) != 0 || cudaMalloc(&mut p, bytes.max(256)) != 0 {
            return Err(format!("cudaMalloc of {bytes} bytes on device {device} failed"));
        }
    }
    Ok(p)
}

/// The decode scratch must start zero-filled (its check-flag words).
pub unsafe fn malloc_zeroed(device: i32, bytes: usize) -> Result<*mut c_void, String> {
    let p = unsafe { malloc(device, bytes)? };
    if unsafe { cudaMemset(p, 0, bytes) } != 0 {
        unsafe { cudaFree(p) };
        return Err("cudaMemset failed".into());
    }
    Ok(p)
}

pub unsafe fn free(p: *mut c_void) {
    unsafe { cudaFree(p) };
}
