//! The CUDA side of Clove's PagedAttention path: the module a maintainer adds
//! as src/cuda_backend.rs.  Not compiled in this repository (no Rust
//! toolchain here); every call below is an entry point of
//! include/clove_cuda.h, and the Python mirror (clove_b200/backend.py,
//! clove_b200/ops.py) exercises the same calls in the tests.
//!
//! The four host changes the path needs:
//!   1. src/backend.rs: `TensorData` (src/backend.rs:164-168) gains
//!      `Cuda(CudaBuffer)`, and `CudaBackend` implements `Backend` with
//!      `paged_attention` (trait method src/backend.rs:249-256) running
//!      `CudaBackend::paged_attention_raw` below.  Every other trait method of
//!      `CudaBackend` panics with "unsupported on CudaBackend": no op of this
//!      backend falls back to the CPU.
//!   2. src/nn.rs: `PagedAttention::forward` (src/nn.rs:531-546) is unchanged;
//!      its block tables and context lengths are `TensorData::Cuda` int32
//!      tensors kept on the device and updated in place (`DeviceTables`).
//!   3. src/device.rs: `EngineDevice::Cuda { ordinal }`, enumerated by
//!      `cuda_devices()` (replaces the adapter probe of `init`, src/device.rs:79-150).
//!   4. src/ffi.rs: `clove_paged_attention` (src/ffi.rs:247-266) keeps its
//!      signature and forwards CUDA tensors to `CudaBackend` (cuda_ffi_routing.rs).
use std::collections::HashMap;
use std::ffi::CStr;
use std::os::raw::{c_char, c_int, c_void};
use std::sync::Mutex;

use crate::cuda_ffi::*;

/// A device allocation owned by a `TensorData::Cuda` tensor.
pub struct CudaBuffer {
    pub ptr: *mut c_void,
    pub bytes: usize,
    pub dtype: c_int, // CLOVE_DTYPE_* or 32 for int32
    pub device: i32,
    pub shape: Vec<usize>,
}
unsafe impl Send for CudaBuffer {}
unsafe impl Sync for CudaBuffer {}

/// The library's error text for a failed call (never an abort).
pub fn last_error() -> String {
    let mut buf = [0 as c_char; 512];
    unsafe {
        clove_cuda_get_last_error(buf.as_mut_ptr(), buf.len());
        CStr::from_ptr(buf.as_ptr()).to_string_lossy().into_owned()
    }
}

fn check(rc: c_int) -> Result<(), String> {
    if rc == CLOVE_OK { Ok(()) } else { Err(format!("clove_cuda error {rc}: {}", last_error())) }
}

/// Device ordinals for `EngineDevice::Cuda { ordinal }` (host change 3).
pub fn cuda_devices() -> Result<Vec<i32>, String> {
    let mut n: c_int = 0;
    check(unsafe { clove_cuda_init(&mut n) })?;
    Ok((0..n).collect())
}

/// A kv_cache tensor [2, num_blocks, block_size, num_kv_heads, head_dim]
/// wrapped once as a pool handle (the tensor maps of the decode's bulk copies
/// are encoded at wrap time).
pub struct Pool {
    raw: CPool,
    pub head_dim: usize,
    pub device: i32,
    workspace: *mut c_void, // zero-filled scratch (clove_cuda_decode_workspace_size), grown on demand
    workspace_bytes: usize,
}
unsafe impl Send for Pool {}

impl Pool {
    pub fn wrap(kv: &CudaBuffer) -> Result<Pool, String> {
        let s = &kv.shape;
        if s.len() != 5 || s[0] != 2 {
            return Err("kv_cache must be [2, num_blocks, block_size, num_kv_heads, head_dim]".into());
        }
        let plane = kv.bytes / 2;
        let mut raw: CPool = std::ptr::null_mut();
        check(unsafe {
            clove_cuda_pool_wrap(kv.device, kv.ptr, (kv.ptr as *mut u8).add(plane) as *mut c_void, s[1] as c_int,
                                 s[2] as c_int, s[3] as c_int, s[4] as c_int, kv.dtype, &mut raw)
        })?;
        Ok(Pool { raw, head_dim: s[4], device: kv.device, workspace: std::ptr::null_mut(), workspace_bytes: 0 })
    }

    fn ensure_workspace(&mut self, batch: usize, hq: usize, max_ctx: usize) -> Result<(), String> {
        let need = unsafe { clove_cuda_decode_workspace_size(self.raw, batch as c_int, hq as c_int, max_ctx as c_int) };
        if need > self.workspace_bytes {
            unsafe {
                // cuda_rt: the crate's thin binding of cudaMalloc / cudaMemset / cudaFree
                if !self.workspace.is_null() {
                    crate::cuda_rt::free(self.workspace);
                }
                self.workspace = crate::cuda_rt::malloc_zeroed(self.device, need)?;
            }
            self.workspace_bytes = need;
        }
        Ok(())
    }
}

impl Drop for Pool {
    fn drop(&mut self) {
        unsafe {
            if !self.workspace.is_null() {
                crate::cuda_rt::free(self.workspace);
            }
            clove_cuda_pool_destroy(self.raw);
        }
    }
}

/// Pools cached by kv_cache pointer, so a decode loop wraps its cache once.
pub struct CudaBackend {
    pools: Mutex<HashMap<usize, Pool>>,
}

impl CudaBackend {
    pub fn new() -> Self {
        CudaBackend { pools: Mutex::new(HashMap::new()) }
    }

    /// The body of `Backend::paged_attention` for CUDA tensors (host change 1):
    /// appends k, v at each sequence's slot `context_lens[b]` and decodes q
    /// over `context_lens[b] + 1` tokens, writing `out` f32 [B, Hq * D].
    /// `max_ctx` bounds the attended lengths (the table width times the
    /// block size when the lengths live only on the device).
    #[allow(clippy::too_many_arguments)]
    pub fn paged_attention_raw(&self, q: &CudaBuffer, k: &CudaBuffer, v: &CudaBuffer, kv_cache: &CudaBuffer,
                               block_tables: &CudaBuffer, context_lens: &CudaBuffer, out: &mut CudaBuffer,
                               max_ctx: usize, stream: *mut c_void) -> Result<(), String> {
        let mut pools = self.pools.lock().unwrap();
        let key = kv_cache.ptr as usize;
        if !pools.contains_key(&key) {
            pools.insert(key, Pool::wrap(kv_cache)?);
        }
        let pool = pools.get_mut(&key).unwrap();
        let batch = context_lens.shape[0];
        let hq = q.shape[1] / pool.head_dim;
        pool.ensure_workspace(batch, hq, max_ctx)?;
        check(unsafe {
            clove_cuda_paged_append_decode(pool.raw, q.ptr, k.ptr, v.ptr, hq as c_int, block_tables.ptr as *mut i32,
                                           block_tables.shape[1] as c_int, context_lens.ptr as *mut i32,
                                           batch as c_int, 1.0 / (pool.head_dim as f32).sqrt(), max_ctx as c_int,
                                           out.ptr as *mut f32, pool.workspace, pool.workspace_bytes, stream)
        })
    }

    /// Device check flags of the last decode on this cache (bad block ids,
    /// context lengths beyond max_ctx, a bounded wait that ran out).
    pub fn decode_flags(&self, kv_cache: &CudaBuffer, stream: *mut c_void) -> Result<i32, String> {
        let pools = self.pools.lock().unwrap();
        let pool = pools.get(&(kv_cache.ptr as usize)).ok_or("no decode ran on this cache")?;
        let mut flags: c_int = 0;
        let rc = unsafe { clove_cuda_decode_status(pool.workspace, stream, &mut flags) };
        if rc == CLOVE_OK || rc == CLOVE_ERR_DEVICE_CHECK { Ok(flags) } else { Err(last_error()) }
    }
}

/// Device-resident block tables and context lengths of a running batch
/// (host change 2): int32 buffers allocated once and updated in place by
/// the block manager (include/clove_blocks.h), never copied per step.
pub struct DeviceTables {
    pub block_tables: CudaBuffer, // int32 [B, max_blocks_per_seq]
    pub context_lens: CudaBuffer, // int32 [B]
}
