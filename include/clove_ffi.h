/*
 * clove_ffi.h — the reference-facing tensor-handle FFI of libclove_cuda.so.
 *
 * Mirrors the opaque-pointer C ABI of the reference (src/ffi.rs:35-113,
 * src/ffi.rs:247-266): tensors are opaque handles created from host data,
 * read back to host memory and freed by the caller; clove_paged_attention
 * takes the six tensors of Backend::paged_attention (src/backend.rs:249-256)
 * and returns a new tensor.  Differences, all deliberate:
 *   - handles live on a CUDA device (the reference's are CPU or wgpu);
 *   - a tensor has a dtype (CLOVE_DTYPE_* or CLOVE_DTYPE_I32) and any rank;
 *   - errors return NULL / a negative status and set the text read by
 *     clove_cuda_get_last_error instead of panicking (src/backend.rs:2937).
 *
 * Device memory for handles comes from a per-device size-keyed cache (freed
 * buffers are kept for reuse, the idea of the reference's BufferPool,
 * src/device.rs:177-222), so a decode loop does not call cudaMalloc per step.
 * All copies and kernels run on the legacy default stream; clove_tensor_data
 * and clove_paged_attention synchronise it.
 */
#ifndef CLOVE_FFI_H
#define CLOVE_FFI_H

#include <stddef.h>
#include <stdint.h>

#include "clove_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#define CLOVE_DTYPE_I32 32

typedef struct clove_tensor* CTensor;

/* src/ffi.rs:71-87 — a 2-D f32 tensor [rows, cols] from host data, on device
 * 0.  NULL data -> NULL. */
CTensor clove_tensor_create(const float* data, size_t rows, size_t cols);

/* Any-rank tensor from host data (NULL data: uninitialised) on `device`. */
CTensor clove_tensor_create_nd(const void* data, const int64_t* shape, int ndim, int dtype, int device);

/* Wrap existing device memory (not owned; never freed by the library). */
CTensor clove_tensor_from_device(void* device_ptr, const int64_t* shape, int ndim, int dtype, int device);

/* src/ffi.rs:89-97 — NULL is a no-op. */
void clove_tensor_free(CTensor t);

/* src/ffi.rs:99-113 — copy the tensor's bytes to host memory `out`
 * (synchronises the default stream).  NULL arguments are a no-op. */
void clove_tensor_data(CTensor t, void* out);

/* Shape query: writes up to 8 dims; returns ndim, or -1 for a NULL handle. */
int clove_tensor_shape(CTensor t, int64_t* shape);

/* src/ffi.rs:247-266 — Backend::paged_attention on the CUDA path:
 *   q  [B, Hq*D]   k, v [B, Hkv*D]   (pool dtype)
 *   kv [2, num_blocks, block_size, Hkv, D] (K plane, V plane)
 *   bt int32 [B, max_blocks_per_seq]   cl int32 [B] (lengths before this token)
 * Appends k, v at slot bt[b][cl_b/bs]*bs + cl_b%bs, attends over cl_b + 1
 * tokens with scale 1/sqrt(D) and returns a new f32 [B, Hq*D] tensor.  The
 * call waits for the decode (the reference's op is synchronous) and checks
 * the kernels' device flags: a block id outside the pool, a context length
 * beyond the block table or a pipeline wait that ran out returns NULL with
 * the flags in clove_cuda_get_last_error's text, never a clamped result.
 * NULL on any error.  When cl was made from host data its maximum sizes the
 * scratch; otherwise the table width does (no device-to-host read). */
CTensor clove_paged_attention(CTensor q, CTensor k, CTensor v, CTensor kv, CTensor bt, CTensor cl);

/* Bytes currently held by the handle cache of `device` (for tests). */
size_t clove_tensor_cache_bytes(int device);

#ifdef __cplusplus
}
#endif

#endif /* CLOVE_FFI_H */
