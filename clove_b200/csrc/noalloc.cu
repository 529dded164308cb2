// Append + decode without a caller-supplied workspace.
//
// Some callers cannot allocate device memory at the point where they decode:
// an engine that has carved all of HBM into its KV pool up front, a host
// runtime whose only device memory comes from a foreign allocator it may not
// call on the serving path, or a plugin host that forbids cudaMalloc after
// start-up.  clove_cuda_paged_append_decode_noalloc serves them: it runs the
// same append + decode as clove_cuda_paged_append_decode, with its scratch in
// a fixed array of this library's device code.  The array is placed in a
// GPU's memory when the library's device code is first loaded on that GPU
// (with CUDA's lazy module loading: at the first use of any of the library's
// kernels or symbols there) and stays until the process exits.
//
// Limits and rules:
//   - The scratch is kNoAllocScratchBytes (16 MiB) per GPU; calls whose
//     workspace need (clove_cuda_decode_workspace_size) exceeds it are
//     rejected with CLOVE_ERR_WORKSPACE.
//   - Every call on a GPU shares the one array and it keeps what the last
//     call left there.  Each call writes every per-CTA descriptor and partial
//     state it later reads, and its combine kernel leaves the flag word
//     cleared for the next call, so leftovers of an earlier (larger or
//     smaller) call are never read.  The array starts zeroed (static device
//     memory).  Calls that overlap on the GPU (other streams, other host
//     threads) race on it: serialise them.
//   - The first call on a device looks up the array's device address (with
//     that device current) and caches it; make that first call before any
//     stream capture.  A failed lookup is not cached: the next call retries.
//   - Device check flags (bad block ids, context lengths, a bounded wait that
//     ran out) land in the array, as they land in a caller's workspace;
//     clove_cuda_noalloc_status reads and clears those of the last call.
#include <mutex>

#include "host.h"

namespace clove {

constexpr size_t kNoAllocScratchBytes = 16u << 20;
constexpr int kMaxDevices = 64;

// The scratch.  In host code this name is only a stand-in for the symbol,
// never a device address: kernels get the address from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static void* g_scratch_ptr[kMaxDevices] = {};
static std::mutex g_scratch_mu;

// Device address of the scratch on `device` (which must be current).  Only a
// successful lookup is cached; after a failure (e.g. a first call made during
// stream capture) the error is cleared and the next call tries again.
static void* scratch_on(int device, cudaError_t* err) {
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  *err = cudaSuccess;
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (*err == cudaSuccess) {
      g_scratch_ptr[device] = p;
    } else {
      cudaGetLastError();
    }
  }
  return g_scratch_ptr[device];
}

// The scratch address on `device`, made current for the lookup and then
// restored.  Returns a CLOVE_* status.
static int scratch_for(int device, const char* who, void** ws) {
  if (device < 0 || device >= kMaxDevices) {
    set_last_error("%s: device %d beyond %d", who, device, kMaxDevices);
    return CLOVE_ERR_NO_DEVICE;
  }
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  if (prev != device && cudaSetDevice(device) != cudaSuccess) {
    cudaGetLastError();
    set_last_error("%s: cudaSetDevice(%d) failed", who, device);
    return CLOVE_ERR_CUDA;
  }
  cudaError_t e = cudaSuccess;
  *ws = scratch_on(device, &e);
  if (prev >= 0 && prev != device) cudaSetDevice(prev);
  if (!*ws) {
    set_last_error("%s: cudaGetSymbolAddress: %s", who, cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  return CLOVE_OK;
}

}  // namespace clove

using namespace clove;

extern "C" {

int clove_cuda_paged_append_decode_noalloc(clove_pool_t pool, const void* q, const void* k_new,
                                           const void* v_new, int num_q_heads, const int32_t* block_tables,
                                           int bt_stride, const int32_t* context_lens, int batch, float scale,
                                           int max_ctx, float* out, void* stream) {
  if (!pool) {
    set_last_error("paged_append_decode_noalloc: null pool");
    return CLOVE_ERR_INVALID_ARG;
  }
  if (batch <= 0 || num_q_heads <= 0 || max_ctx < 1) {
    // Same argument checks (and messages) as the workspace entry point.
    return clove_cuda_paged_append_decode(pool, q, k_new, v_new, num_q_heads, block_tables, bt_stride,
                                          context_lens, batch, scale, max_ctx, out, nullptr, 0, stream);
  }
  const size_t need = clove_cuda_decode_workspace_size(pool, batch, num_q_heads, max_ctx);
  if (need > kNoAllocScratchBytes) {
    set_last_error(
        "paged_append_decode_noalloc: this call needs %zu bytes of scratch, the built-in scratch holds %zu "
        "(use clove_cuda_paged_append_decode with a workspace)",
        need, kNoAllocScratchBytes);
    return CLOVE_ERR_WORKSPACE;
  }
  void* ws = nullptr;
  const int rc = scratch_for(pool->device, "paged_append_decode_noalloc", &ws);
  if (rc != CLOVE_OK) return rc;
  return clove_cuda_paged_append_decode(pool, q, k_new, v_new, num_q_heads, block_tables, bt_stride, context_lens,
                                        batch, scale, max_ctx, out, ws, kNoAllocScratchBytes, stream);
}

int clove_cuda_noalloc_status(int device, void* stream, int* flags) {
  void* ws = nullptr;
  const int rc = scratch_for(device, "noalloc_status", &ws);
  if (rc != CLOVE_OK) return rc;
  return clove_cuda_decode_status(ws, stream, flags);
}

}  // extern "C"
