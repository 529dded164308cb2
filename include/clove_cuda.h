/*
 * clove_cuda.h — C ABI of the B200-native PagedAttention decode library
 * (libclove_cuda.so, built for sm_100a).
 *
 * The reference (rakeshpdey/clove, Rust) exposes the hot path as
 *   Backend::paged_attention(q, k, v, kv_cache, block_tables, context_lens)
 *     src/backend.rs:249-256
 *   PagedAttention::forward(x, kv_cache, block_tables, context_lens)
 *     src/nn.rs:531-546
 *   clove_paged_attention(q, k, v, kv, bt, cl) -> CTensor
 *     src/ffi.rs:247-266
 * and has no working implementation of it (the eager backend panics at
 * src/backend.rs:2937-2948; the lazy WGSL kernel at src/lazy.rs:5243-5275 is a
 * placeholder).  The entry points below are what a Rust `CudaBackend`
 * declares in an `extern "C"` block to replace those three.
 *
 * Conventions
 *   - Every function returns an int status (CLOVE_OK == 0, negative on
 *     error) and never aborts; clove_cuda_get_last_error() gives the text.
 *   - All tensor pointers are device pointers on the pool's device unless a
 *     function says otherwise.  Calls are asynchronous on `stream`
 *     (a cudaStream_t; NULL = legacy default stream).
 *   - KV cache layout (per plane, K and V):  [num_blocks, block_size,
 *     num_kv_heads, head_dim], row-major — the layout documented at
 *     src/nn.rs:534 with the KV-head count made explicit for GQA.
 *   - block_tables: int32 [batch, bt_stride] (src/nn.rs:535; the reference
 *     hardcodes a stride of 1024 at src/lazy.rs:5264, here it is a parameter).
 *   - context_lens: int32 [batch] (src/nn.rs:536).
 *   - q: [batch, num_q_heads, head_dim] in the pool dtype; out: float32
 *     [batch, num_q_heads, head_dim] (the reference output is f32,
 *     src/lazy.rs:5252).  Query head hq reads KV head hq / (num_q_heads /
 *     num_kv_heads).
 *   - Scale: the caller passes it; the reference uses 1/sqrt(head_dim)
 *     (src/lazy.rs:5267, src/nn/attention.rs:64).
 */
#ifndef CLOVE_CUDA_H
#define CLOVE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define CLOVE_OK                 0
#define CLOVE_ERR_INVALID_ARG   -1  /* bad shape, null pointer, misalignment   */
#define CLOVE_ERR_UNSUPPORTED   -2  /* head_dim / group / dtype not built       */
#define CLOVE_ERR_CUDA          -3  /* a CUDA runtime call failed               */
#define CLOVE_ERR_OOM           -4  /* device allocation failed (pool create)   */
#define CLOVE_ERR_WORKSPACE     -5  /* workspace too small                      */
#define CLOVE_ERR_DEVICE_CHECK  -6  /* a kernel flagged bad indices (see flags) */
#define CLOVE_ERR_NO_DEVICE     -7  /* no CUDA device / ordinal out of range    */

/* ---- device-side check flags, reported by clove_cuda_decode_status ------ */
#define CLOVE_FLAG_BLOCK_OOB     1  /* a block-table entry outside [0, num_blocks) */
#define CLOVE_FLAG_CTX_RANGE     2  /* a context length < 0 or > max_ctx          */
#define CLOVE_FLAG_SLOT_OOB      4  /* a slot_mapping entry >= num_blocks*block_size */
#define CLOVE_FLAG_TIMEOUT       8  /* a bounded pipeline wait ran out            */

/* ---- dtypes: the reference's FFI precision codes (src/ffi.rs:305-313) ---- */
#define CLOVE_DTYPE_F32    0
#define CLOVE_DTYPE_F16   16
#define CLOVE_DTYPE_BF16 160

typedef struct clove_pool* clove_pool_t;

typedef struct clove_pool_info {
    int device;
    int num_blocks;
    int block_size;
    int num_kv_heads;
    int head_dim;
    int dtype;
    int owns_memory;      /* 1: created by pool_create, 0: wrapped */
    void* k_cache;        /* device pointer, plane K */
    void* v_cache;        /* device pointer, plane V */
    size_t plane_bytes;   /* bytes of one plane */
} clove_pool_info_t;

/* Number of visible CUDA devices (replaces the adapter enumeration of
 * EngineDevice::init, src/device.rs:79-150, and MultiGPUOrchestrator::new,
 * src/distributed.rs:58-120). */
int clove_cuda_init(int* num_devices);

/* Last error text of the calling thread (empty string if none). */
int clove_cuda_get_last_error(char* buf, size_t n);

/* Device-resident KV block pool: one allocation [2, num_blocks, block_size,
 * num_kv_heads, head_dim] (K plane then V plane), owned by the handle.
 * The reference passes a caller-made kv_cache tensor (src/nn.rs:534) and has
 * no allocator; its only pool is the size-keyed BufferPool
 * (src/device.rs:177-222). */
int clove_cuda_pool_create(int device, int num_blocks, int block_size,
                           int num_kv_heads, int head_dim, int dtype,
                           clove_pool_t* out);

/* Wrap caller-owned K and V planes (each [num_blocks, block_size,
 * num_kv_heads, head_dim], 16-byte aligned) without taking ownership. */
int clove_cuda_pool_wrap(int device, void* k_cache, void* v_cache,
                         int num_blocks, int block_size, int num_kv_heads,
                         int head_dim, int dtype, clove_pool_t* out);

int clove_cuda_pool_destroy(clove_pool_t pool);

/* Synchronise `stream`, read and clear the check flags that the append and
 * gather kernels of this pool raised since the last call (CLOVE_FLAG_*). */
int clove_cuda_pool_status(clove_pool_t pool, void* stream, int* flags);
int clove_cuda_pool_info(clove_pool_t pool, clove_pool_info_t* info);

/* KV append (reshape-and-cache): for each token i with slot s =
 * slot_mapping[i] >= 0, copy k[i, :, :] -> K[s / block_size, s % block_size]
 * and v[i] -> V[...], bit for bit.  k, v: [num_tokens, num_kv_heads,
 * head_dim] in the pool dtype.  Negative slots are skipped (padding).  The
 * reference passes the new k, v to paged_attention (src/nn.rs:539-543,
 * src/lazy.rs:5247-5248) but never writes them to the cache. */
int clove_cuda_reshape_and_cache(clove_pool_t pool, const void* k,
                                 const void* v, const int32_t* slot_mapping,
                                 int num_tokens, void* stream);

/* Block-table gather (debug / parity): k_out, v_out: [batch, max_ctx,
 * num_kv_heads, head_dim] in the pool dtype; token t of sequence b is read
 * from physical block block_tables[b*bt_stride + t/block_size], offset
 * t % block_size — the indexing of src/lazy.rs:5259-5270 with explicit heads
 * and table stride.  Rows t >= context_lens[b] are zero-filled. */
int clove_cuda_gather_kv(clove_pool_t pool, const int32_t* block_tables,
                         int bt_stride, const int32_t* context_lens,
                         int batch, int max_ctx, void* k_out, void* v_out,
                         void* stream);

/* Bytes of scratch workspace paged_decode / paged_append_decode need for
 * this head count (the batch and context-length arguments are kept for the
 * interface: the decode splits its work evenly over a fixed number of CTAs,
 * each keeping at most two partial states, so the scratch does not grow with
 * them; a few MB). */
size_t clove_cuda_decode_workspace_size(clove_pool_t pool, int batch,
                                        int num_q_heads, int max_ctx);

/* Decode: for every sequence b and query head hq,
 *   out[b,hq,:] = softmax_t(scale * <q[b,hq,:], K_t>) . V_t
 * over the context_lens[b] cached tokens of sequence b (semantics of
 * src/nn/attention.rs:52-69; gather of src/lazy.rs:5259-5270).  A sequence
 * with context length 0 gets a zero output row.  `workspace` (device memory,
 * >= clove_cuda_decode_workspace_size bytes, 256-byte aligned) is scratch:
 * ZERO-FILLED before its first use (its check-flag words), after which calls
 * on one stream keep sharing it; the call allocates nothing. */
int clove_cuda_paged_decode(clove_pool_t pool, const void* q, int num_q_heads,
                            const int32_t* block_tables, int bt_stride,
                            const int32_t* context_lens, int batch,
                            float scale, int max_ctx, float* out,
                            void* workspace, size_t workspace_bytes,
                            void* stream);

/* Append + decode in one launch (the CudaBackend body of
 * Backend::paged_attention, src/backend.rs:249-256): context_lens holds the
 * lengths BEFORE this step; k_new, v_new: [batch, num_kv_heads, head_dim] are
 * written to slot block_tables[b][ctx_b / block_size]*block_size +
 * ctx_b % block_size, then the sequence attends over ctx_b + 1 tokens.
 * context_lens is not modified (the caller advances it). */
int clove_cuda_paged_append_decode(clove_pool_t pool, const void* q,
                                   const void* k_new, const void* v_new,
                                   int num_q_heads,
                                   const int32_t* block_tables, int bt_stride,
                                   const int32_t* context_lens, int batch,
                                   float scale, int max_ctx, float* out,
                                   void* workspace, size_t workspace_bytes,
                                   void* stream);

/* Prefill into the paged cache (the step before decode; the reference's
 * FlashAttention step, src/lazy.rs:4821-4923, causal, RoPE on q and k, scale
 * 1/sqrt(head_dim)).  The prompt tokens of `batch` sequences are packed:
 * q [num_tokens, num_q_heads, D], k, v [num_tokens, num_kv_heads, D] in the
 * pool dtype; sequence b owns tokens cu_seqlens[b] .. cu_seqlens[b+1]-1 (int32
 * [batch+1], device) at positions context_lens[b] + i (context_lens: cached
 * tokens before the prompt; 0 for a fresh prompt).  With rope_theta > 0, q
 * and k are rotated in adjacent pairs (2i, 2i+1) by pos * theta^(-2i/D)
 * (theta 10000 in the reference); 0 disables RoPE.  K and V (rotated K) are
 * written to their slots through block_tables; out f32 [num_tokens,
 * num_q_heads, D] is each token's causal attention over its sequence's cache
 * up to and including itself.  max_ctx bounds context_lens[b] + prompt
 * length.  Scratch: clove_cuda_prefill_workspace_size bytes. */
size_t clove_cuda_prefill_workspace_size(clove_pool_t pool, int num_tokens,
                                         int num_q_heads, int bt_stride,
                                         int max_ctx);
int clove_cuda_paged_prefill(clove_pool_t pool, const void* q, const void* k,
                             const void* v, const int32_t* cu_seqlens,
                             const int32_t* block_tables, int bt_stride,
                             const int32_t* context_lens, int batch,
                             int num_tokens, int num_q_heads, float scale,
                             float rope_theta, int max_ctx, float* out,
                             void* workspace, size_t workspace_bytes,
                             void* stream);

/* Fused Q/K/V projection + KV append (one decode step) on the tensor cores.
 * Replaces the three Linear calls of PagedAttention::forward
 * (src/nn.rs:538-540; Linear y = x W + b, src/nn.rs:102-123) and the append
 * that the paged-attention op must do with their k, v.
 *
 * Weights are packed once (per weight update) into the kernel's streaming
 * layout: clove_cuda_qkv_pack_weights takes W^T [n_out, hidden] (pool dtype,
 * row-major: the reference's W_q | W_k | W_v, each [hidden, out],
 * transposed and stacked; n_out = (num_q_heads + 2 num_kv_heads) * head_dim)
 * and writes clove_cuda_qkv_packed_bytes(n_out, hidden) bytes: 128-feature x
 * 64-element tiles, each 16 KB contiguous in the 128-byte-swizzled order the
 * tensor cores read, zero-padded at the edges.
 *
 * clove_cuda_qkv_append:
 *   x         [batch, hidden], pool dtype (bf16/f16), 16-byte aligned
 *   w_packed  the packed weights above, 16-byte aligned
 *   bias      f32 [n_out] (b_q | b_k | b_v), or null
 * Writes q_out [batch, num_q_heads, head_dim] (pool dtype, 16-byte aligned)
 * and stores k, v at slot context_lens[b] of sequence b through
 * block_tables.  With rope_theta > 0, q and k are rotated by position
 * context_lens[b] (the pairing of clove_cuda_paged_prefill).
 * context_lens_out (optional, int32 [batch], not aliasing context_lens)
 * receives context_lens + 1: the lengths to decode over with
 * clove_cuda_paged_decode.  Bad slots are
 * skipped and flagged in the pool's status word, like
 * clove_cuda_reshape_and_cache.  Scratch: clove_cuda_qkv_workspace_size
 * bytes, 256-byte aligned, ZERO-FILLED before its first use; every call
 * leaves it zeroed again (its per-tile counters), including one whose
 * bounded waits ran out (CLOVE_FLAG_TIMEOUT in the pool's status word), so
 * one buffer serves all later calls on a stream.  f32 pools return
 * CLOVE_ERR_UNSUPPORTED. */
size_t clove_cuda_qkv_packed_bytes(int n_out, int hidden);
int clove_cuda_qkv_pack_weights(int dtype, const void* w_t, int n_out,
                                int hidden, void* packed, void* stream);
size_t clove_cuda_qkv_workspace_size(clove_pool_t pool, int batch, int hidden,
                                     int num_q_heads);
int clove_cuda_qkv_append(clove_pool_t pool, const void* x,
                          const void* w_packed, const float* bias, int batch,
                          int hidden, int num_q_heads,
                          const int32_t* block_tables, int bt_stride,
                          const int32_t* context_lens, float rope_theta,
                          void* q_out, int32_t* context_lens_out,
                          void* workspace, size_t workspace_bytes,
                          void* stream);

/* Append + decode for callers that cannot allocate device memory when they
 * decode (an engine that hands all of HBM to its KV pool at start-up, a host
 * whose device memory comes only from an allocator it may not call on the
 * serving path).  No counterpart in the reference.  Same arguments and
 * results as clove_cuda_paged_append_decode, minus the workspace: scratch
 * comes from a fixed 16 MiB array in the library's device code, placed on a
 * GPU when the library's device code is first loaded there and kept until
 * the process exits.  Returns CLOVE_ERR_WORKSPACE when the call needs more
 * than that (see clove_cuda_decode_workspace_size).  All calls on a GPU
 * share the array: calls that overlap on the GPU race, so serialise them.
 * The first call on a device looks up the array's address (a failed lookup
 * is retried by the next call); make it before any stream capture.  Device
 * check flags go to the array and are read with clove_cuda_noalloc_status.
 * The call allocates nothing. */
int clove_cuda_paged_append_decode_noalloc(clove_pool_t pool, const void* q,
                                           const void* k_new, const void* v_new,
                                           int num_q_heads,
                                           const int32_t* block_tables,
                                           int bt_stride,
                                           const int32_t* context_lens,
                                           int batch, float scale, int max_ctx,
                                           float* out, void* stream);

/* ---- output exchange over NVLink peer memory (KV-head split) ---------- */
/* The reference assembles per-shard results through host memory
 * (MultiGPUOrchestrator::synchronize_gradients, src/distributed.rs:204-300);
 * these replace that step for the head-split decode with P2P stores between
 * the ranks' GPUs.  One process per GPU; every rank allocates a receive
 * buffer, publishes its IPC handle (e.g. through torch.distributed), opens
 * the peers' handles and keeps a device array of the world's buffer
 * pointers (its own at index rank). */
#define CLOVE_IPC_HANDLE_BYTES 64

/* Receive-buffer bytes for slices of `slice_bytes` over `world` ranks. */
size_t clove_cuda_peer_gather_buffer_bytes(size_t slice_bytes, int world);

/* cudaMalloc `bytes` on `device`, zero them and write the allocation's IPC
 * handle (CLOVE_IPC_HANDLE_BYTES) to `ipc_handle`. */
int clove_cuda_peer_buffer_alloc(int device, size_t bytes, void** ptr, void* ipc_handle);
/* Map a peer's buffer from its IPC handle into this process (on `device`). */
int clove_cuda_peer_buffer_open(int device, const void* ipc_handle, void** ptr);
/* Unmap a buffer from clove_cuda_peer_buffer_open. */
int clove_cuda_peer_buffer_close(void* ptr);
/* Free a buffer from clove_cuda_peer_buffer_alloc (after the peers closed it). */
int clove_cuda_peer_buffer_free(void* ptr);

/* All-gather of equal slices: out[r * slice_bytes ...] receives rank r's
 * `src` on every rank (the layout of an all-gather into one tensor).
 * peer_bufs: device array of `world` receive-buffer pointers as mapped in
 * this process.  Every rank must make the same sequence of calls with the
 * same slice_bytes; the kernel waits (bounded) for the peers' slices, so the
 * ranks' calls must be able to run at the same time (one GPU per rank).
 * slice_bytes, src and out: multiples of 16 bytes.  Capturable in a CUDA
 * graph.  A wait that runs out sets CLOVE_FLAG_TIMEOUT (read it with
 * clove_cuda_peer_gather_status) and leaves that peer's part of `out`
 * undefined; the ranks' delivery counts are then out of step, so every rank
 * must replace its receive buffer before the next call. */
int clove_cuda_peer_gather(const void* src, size_t slice_bytes, void* const* peer_bufs, int rank,
                           int world, void* out, void* stream);
/* Synchronise `stream`, read and clear the flags of this rank's receive
 * buffer; CLOVE_ERR_DEVICE_CHECK if any was set. */
int clove_cuda_peer_gather_status(void* own_buf, size_t slice_bytes, int world, void* stream,
                                  int* flags);

/* Check flags (CLOVE_FLAG_*) of the most recent
 * clove_cuda_paged_append_decode_noalloc call on `device`: synchronises
 * `stream`, reads and clears the flag word of the built-in scratch, like
 * clove_cuda_decode_status does for a caller workspace.  No counterpart in
 * the reference. */
int clove_cuda_noalloc_status(int device, void* stream, int* flags);

/* Synchronise `stream` and read the device check flags (CLOVE_FLAG_*) that
 * the most recent completed decode call on `workspace` raised (each call
 * publishes its own flags when it completes); the word is cleared after
 * reading.  Returns CLOVE_ERR_DEVICE_CHECK if any flag was set, CLOVE_OK
 * otherwise. */
int clove_cuda_decode_status(void* workspace, void* stream, int* flags);

/* Kernel-variant selection for decode: 0 = automatic (default), 1 = force
 * the CUDA-core kernel, 2 = force the tensor-core kernel (bf16/f16 with
 * group >= 4 only).  Process-wide; for tests and measurement. */
int clove_cuda_set_decode_variant(int variant);

/* Number of kernels the library launched since load (for the bench's
 * launch count). */
uint64_t clove_cuda_launch_count(void);

/* Testing hook (failure detection without a GPU fault).  wait_limit: polls
 * after which a pipeline wait gives up (0 = the default, seconds of wall
 * time; a peer-gather receive gives up after wait_limit x 64 ns);
 * inject_stall = 1 makes producers skip one stage's copy (decode: the first
 * stage of every CTA's first piece; fused projection: the first
 * stage of the first CTA), so the consumers' bounded waits run out: the call
 * then completes, reports CLOVE_FLAG_TIMEOUT through clove_cuda_decode_status
 * (the pool's status for the projection), and its output is undefined.
 * Process-wide; never set it in production. */
int clove_cuda_debug_set(uint32_t wait_limit, int inject_stall);

/* Measurement hook: with enable = 1, every decode call records CUDA events
 * around its plan, decode and combine launches; clove_cuda_debug_phase_ms
 * waits for the most recent timed call and returns the three durations in
 * milliseconds (combine = 0 when the call needed no split-K merge).  The
 * events sit between the launches, so timed calls lose the overlap of
 * programmatically chained launches.  Process-wide; for the benchmark. */
int clove_cuda_debug_phase_timing(int enable);
int clove_cuda_debug_phase_ms(float* plan_ms, float* decode_ms,
                              float* combine_ms);

/* Measurement hook of timeline builds (compiled with -DCLOVE_TRACE): decode
 * calls write %globaltimer stamps of the plan, every CTA and every work unit
 * into `buffer` (device memory, at least (16 + 4*4096 + 3*65536) u64, plan
 * and combine slots 0..3 preset by the caller); NULL stops it.  Returns
 * CLOVE_ERR_UNSUPPORTED in the product build, which records nothing. */
int clove_cuda_debug_trace(void* buffer);

#ifdef __cplusplus
}
#endif

#endif /* CLOVE_CUDA_H */
