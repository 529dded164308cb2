//! `extern "C"` declarations of libclove_cuda.so (include/clove_cuda.h), the
//! module a maintainer adds as src/cuda_ffi.rs.  Generated from the header's
//! declarations (every entry point it declares), so the two cannot drift.
//! Not compiled in this repository (no Rust toolchain here).
#![allow(non_camel_case_types, dead_code)]
use std::os::raw::{c_char, c_float, c_int, c_void};

pub type CPool = *mut c_void;

/// clove_pool_info_t
#[repr(C)]
pub struct CPoolInfo {
    pub device: c_int,
    pub num_blocks: c_int,
    pub block_size: c_int,
    pub num_kv_heads: c_int,
    pub head_dim: c_int,
    pub dtype: c_int,
    pub owns_memory: c_int,
    pub k_cache: *mut c_void,
    pub v_cache: *mut c_void,
    pub plane_bytes: usize,
}

pub const CLOVE_OK: c_int = 0;
pub const CLOVE_ERR_WORKSPACE: c_int = -5;
pub const CLOVE_ERR_DEVICE_CHECK: c_int = -6;
pub const CLOVE_DTYPE_F32: c_int = 0;
pub const CLOVE_DTYPE_F16: c_int = 16;
pub const CLOVE_DTYPE_BF16: c_int = 160;

#[link(name = "clove_cuda")]
unsafe extern "C" {
    pub fn clove_cuda_init(num_devices: *mut c_int) -> c_int;
    pub fn clove_cuda_get_last_error(buf: *mut c_char, n: usize) -> c_int;
    pub fn clove_cuda_pool_create(device: c_int, num_blocks: c_int, block_size: c_int, num_kv_heads: c_int, head_dim: c_int, dtype: c_int, out: *mut CPool) -> c_int;
    pub fn clove_cuda_pool_wrap(device: c_int, k_cache: *mut c_void, v_cache: *mut c_void, num_blocks: c_int, block_size: c_int, num_kv_heads: c_int, head_dim: c_int, dtype: c_int, out: *mut CPool) -> c_int;
    pub fn clove_cuda_pool_destroy(pool: CPool) -> c_int;
    pub fn clove_cuda_pool_status(pool: CPool, stream: *mut c_void, flags: *mut c_int) -> c_int;
    pub fn clove_cuda_pool_info(pool: CPool, info: *mut CPoolInfo) -> c_int;
    pub fn clove_cuda_reshape_and_cache(pool: CPool, k: *mut c_void, v: *mut c_void, slot_mapping: *mut i32, num_tokens: c_int, stream: *mut c_void) -> c_int;
    pub fn clove_cuda_gather_kv(pool: CPool, block_tables: *mut i32, bt_stride: c_int, context_lens: *mut i32, batch: c_int, max_ctx: c_int, k_out: *mut c_void, v_out: *mut c_void, stream: *mut c_void) -> c_int;
    pub fn clove_cuda_decode_workspace_size(pool: CPool, batch: c_int, num_q_heads: c_int, max_ctx: c_int) -> usize;
    pub fn clove_cuda_paged_decode(pool: CPool, q: *mut c_void, num_q_heads: c_int, block_tables: *mut i32, bt_stride: c_int, context_lens: *mut i32, batch: c_int, scale: c_float, max_ctx: c_int, out: *mut c_float, workspace: *mut c_void, workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn clove_cuda_paged_append_decode(pool: CPool, q: *mut c_void, k_new: *mut c_void, v_new: *mut c_void, num_q_heads: c_int, block_tables: *mut i32, bt_stride: c_int, context_lens: *mut i32, batch: c_int, scale: c_float, max_ctx: c_int, out: *mut c_float, workspace: *mut c_void, workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn clove_cuda_prefill_workspace_size(pool: CPool, num_tokens: c_int, num_q_heads: c_int, bt_stride: c_int, max_ctx: c_int) -> usize;
    pub fn clove_cuda_paged_prefill(pool: CPool, q: *mut c_void, k: *mut c_void, v: *mut c_void, cu_seqlens: *mut i32, block_tables: *mut i32, bt_stride: c_int, context_lens: *mut i32, batch: c_int, num_tokens: c_int, num_q_heads: c_int, scale: c_float, rope_theta: c_float, max_ctx: c_int, out: *mut c_float, workspace: *mut c_void, workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn clove_cuda_qkv_packed_bytes(n_out: c_int, hidden: c_int) -> usize;
    pub fn clove_cuda_qkv_pack_weights(dtype: c_int, w_t: *mut c_void, n_out: c_int, hidden: c_int, packed: *mut c_void, stream: *mut c_void) -> c_int;
    pub fn clove_cuda_qkv_workspace_size(pool: CPool, batch: c_int, hidden: c_int, num_q_heads: c_int) -> usize;
    pub fn clove_cuda_qkv_append(pool: CPool, x: *mut c_void, w_packed: *mut c_void, bias: *mut c_float, batch: c_int, hidden: c_int, num_q_heads: c_int, block_tables: *mut i32, bt_stride: c_int, context_lens: *mut i32, rope_theta: c_float, q_out: *mut c_void, context_lens_out: *mut i32, workspace: *mut c_void, workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn clove_cuda_paged_append_decode_noalloc(pool: CPool, q: *mut c_void, k_new: *mut c_void, v_new: *mut c_void, num_q_heads: c_int, block_tables: *mut i32, bt_stride: c_int, context_lens: *mut i32, batch: c_int, scale: c_float, max_ctx: c_int, out: *mut c_float, stream: *mut c_void) -> c_int;
    pub fn clove_cuda_noalloc_status(device: c_int, stream: *mut c_void, flags: *mut c_int) -> c_int;
    pub fn clove_cuda_peer_gather_buffer_bytes(slice_bytes: usize, world: c_int) -> usize;
    pub fn clove_cuda_peer_buffer_alloc(device: c_int, bytes: usize, ptr: *mut *mut c_void, ipc_handle: *mut c_void) -> c_int;
    pub fn clove_cuda_peer_buffer_open(device: c_int, ipc_handle: *const c_void, ptr: *mut *mut c_void) -> c_int;
    pub fn clove_cuda_peer_buffer_close(ptr: *mut c_void) -> c_int;
    pub fn clove_cuda_peer_buffer_free(ptr: *mut c_void) -> c_int;
    pub fn clove_cuda_peer_gather(src: *const c_void, slice_bytes: usize, peer_bufs: *const *mut c_void, rank: c_int, world: c_int, out: *mut c_void, stream: *mut c_void) -> c_int;
    pub fn clove_cuda_peer_gather_status(own_buf: *mut c_void, slice_bytes: usize, world: c_int, stream: *mut c_void, flags: *mut c_int) -> c_int;
    pub fn clove_cuda_decode_status(workspace: *mut c_void, stream: *mut c_void, flags: *mut c_int) -> c_int;
    pub fn clove_cuda_set_decode_variant(variant: c_int) -> c_int;
    pub fn clove_cuda_launch_count() -> u64;
    pub fn clove_cuda_debug_set(wait_limit: u32, inject_stall: c_int) -> c_int;
    pub fn clove_cuda_debug_phase_timing(enable: c_int) -> c_int;
    pub fn clove_cuda_debug_phase_ms(plan_ms: *mut c_float, decode_ms: *mut c_float, combine_ms: *mut c_float) -> c_int;
    pub fn clove_cuda_debug_trace(buffer: *mut c_void) -> c_int;
}
