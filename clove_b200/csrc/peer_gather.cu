// Output exchange of the KV-head split over NVLink peer memory: every rank
// stores its slice straight into every peer's receive buffer (P2P stores
// through NVSwitch), raises a per-source counter in the peer's buffer with a
// system-scope release, and copies what its peers delivered into `out`
// ([world][slice] like an all-gather) once their counters say it landed.
//
// The reference exchanges per-shard buffers through host memory
// (MultiGPUOrchestrator::synchronize_gradients, src/distributed.rs:204-300:
// copy to a staging buffer, map, combine on the CPU, ring over TCP); this is
// the device-side replacement for the head-split decode's output assembly.
//
// Receive buffer of each rank (allocated here, mapped into the peers with
// CUDA IPC handles; no multicast object, no cluster-multicast load):
//   data   [2][world][slot]   slot = slice rounded up to 256 B; calls
//                             alternate between the two halves
//   count  [world] u32        chunks received from each source, monotonic
//   state  u32 calls, u32 done, i32 flags   (local bookkeeping)
// A rank can only be one call ahead of a peer (its call n+1 waits for the
// peer's call n+1 sends, which the peer issues after its call n finished),
// so two halves keep a sender from overwriting data a receiver still copies.
#include <cstdint>
#include <cstring>

#include "host.h"

namespace clove {
namespace {

constexpr int kGatherThreads = 256;
constexpr size_t kGatherChunk = 8192;  // bytes per CTA and peer
constexpr int kMaxChunks = 64;

struct GatherLayout {
  size_t slot, data, count_off, state_off, total;
};

GatherLayout gather_layout(size_t slice, int world) {
  GatherLayout g;
  g.slot = (slice + 255) & ~size_t(255);
  g.data = 2 * (size_t)world * g.slot;
  g.count_off = g.data;
  g.state_off = g.count_off + 4 * (size_t)world;
  g.total = g.data + ((4 * (size_t)world + 12 + 255) & ~size_t(255));
  return g;
}

int gather_chunks(size_t slice) {
  size_t c = (slice + kGatherChunk - 1) / kGatherChunk;
  return (int)(c < 1 ? 1 : (c > kMaxChunks ? kMaxChunks : c));
}

struct GatherArgs {
  const uint4* src;
  uint4* out;
  char* const* bufs;  // device array: bufs[r] = rank r's receive buffer as mapped here
  size_t slice16;     // slice in 16-byte words
  size_t slot, count_off, state_off;
  int rank, world, chunks;
  uint64_t wait_ns;   // how long a receive waits before it gives up
};


__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Words [lo, hi) of chunk c out of `chunks` equal pieces of n words.
__device__ __forceinline__ void chunk_range(size_t n, int c, int chunks, size_t& lo, size_t& hi) {
  size_t per = (n + chunks - 1) / chunks;
  lo = per * c;
  hi = lo + per < n ? lo + per : n;
  if (lo > n) lo = n;
}

// grid (chunks, world): CTA (c, p) moves chunk c of the exchange with rank p.
__global__ void __launch_bounds__(kGatherThreads) peer_gather_kernel(GatherArgs a) {
  const int c = blockIdx.x, p = blockIdx.y;
  char* own = a.bufs[a.rank];
  uint32_t* state = reinterpret_cast<uint32_t*>(own + a.state_off);
  griddep_wait();  // the slice is the previous kernel's output
  const uint32_t call = state[0] + 1;  // read by every CTA before the last one bumps it
  const size_t half = (size_t)(call & 1) * a.world * a.slot;
  size_t lo, hi;
  chunk_range(a.slice16, c, a.chunks, lo, hi);
  uint4* out = a.out + (size_t)p * a.slice16;

  if (p == a.rank) {
    for (size_t i = lo + threadIdx.x; i < hi; i += kGatherThreads) out[i] = a.src[i];
  } else {
    // Send: this rank's chunk into peer p's half, at this rank's slot.
    uint4* dst = reinterpret_cast<uint4*>(a.bufs[p] + half + (size_t)a.rank * a.slot);
    for (size_t i = lo + threadIdx.x; i < hi; i += kGatherThreads) dst[i] = a.src[i];
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0)
      red_release_sys_add(reinterpret_cast<uint32_t*>(a.bufs[p] + a.count_off) + a.rank, 1u);
    // Receive: wait until peer p delivered all its chunks of this call.
    __shared__ int ok;
    if (threadIdx.x == 0) {
      const uint32_t* cnt = reinterpret_cast<const uint32_t*>(own + a.count_off) + p;
      const uint32_t target = call * (uint32_t)a.chunks;
      int got = 0;
      const uint64_t t0 = gtime();
      for (;;) {
        if ((int32_t)(ld_acquire_sys(cnt) - target) >= 0) {
          got = 1;
          break;
        }
        if (gtime() - t0 > a.wait_ns) break;
        __nanosleep(64);
      }
      if (!got) atomicOr(reinterpret_cast<int*>(state + 2), CLOVE_FLAG_TIMEOUT);
      ok = got;
    }
    __syncthreads();
    if (ok) {
      const uint4* rx = reinterpret_cast<const uint4*>(own + half + (size_t)p * a.slot);
      for (size_t i = lo + threadIdx.x; i < hi; i += kGatherThreads) out[i] = rx[i];
    }
  }
  // The last CTA to finish advances the call counter.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(state + 1, 1u) == gridDim.x * gridDim.y - 1) {
      state[1] = 0;
      state[0] = call;
    }
  }
}

}  // namespace
}  // namespace clove

using namespace clove;

extern "C" {

size_t clove_cuda_peer_gather_buffer_bytes(size_t slice_bytes, int world) {
  if (world < 1) return 0;
  return gather_layout(slice_bytes, world).total;
}

int clove_cuda_peer_buffer_alloc(int device, size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) {
    set_last_error("peer_buffer_alloc: null pointer or zero size");
    return CLOVE_ERR_INVALID_ARG;
  }
  *ptr = nullptr;
  if (cudaSetDevice(device) != cudaSuccess) {
    set_last_error("peer_buffer_alloc: no device %d", device);
    return CLOVE_ERR_NO_DEVICE;
  }
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    set_last_error("peer_buffer_alloc: cudaMalloc of %zu bytes failed", bytes);
    return CLOVE_ERR_OOM;
  }
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any peer can map it
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    set_last_error("peer_buffer_alloc: %s", cudaGetErrorString(e));
    cudaFree(p);
    return CLOVE_ERR_CUDA;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == CLOVE_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return CLOVE_OK;
}

int clove_cuda_peer_buffer_open(int device, const void* ipc_handle, void** ptr) {
  if (!ptr || !ipc_handle) {
    set_last_error("peer_buffer_open: null pointer");
    return CLOVE_ERR_INVALID_ARG;
  }
  *ptr = nullptr;
  if (cudaSetDevice(device) != cudaSuccess) {
    set_last_error("peer_buffer_open: no device %d", device);
    return CLOVE_ERR_NO_DEVICE;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_last_error("peer_buffer_open: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  return CLOVE_OK;
}

int clove_cuda_peer_buffer_close(void* ptr) {
  if (!ptr) return CLOVE_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    set_last_error("peer_buffer_close: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  return CLOVE_OK;
}

int clove_cuda_peer_buffer_free(void* ptr) {
  if (!ptr) return CLOVE_OK;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    set_last_error("peer_buffer_free: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  return CLOVE_OK;
}

int clove_cuda_peer_gather(const void* src, size_t slice_bytes, void* const* peer_bufs, int rank,
                           int world, void* out, void* stream) {
  if (!src || !peer_bufs || !out || world < 1 || rank < 0 || rank >= world) {
    set_last_error("peer_gather: null pointer or rank %d outside world %d", rank, world);
    return CLOVE_ERR_INVALID_ARG;
  }
  if (slice_bytes == 0) return CLOVE_OK;
  if (slice_bytes % 16 || (reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(out)) % 16) {
    set_last_error("peer_gather: slice size and pointers must be multiples of 16 bytes");
    return CLOVE_ERR_INVALID_ARG;
  }
  GatherLayout g = gather_layout(slice_bytes, world);
  GatherArgs a;
  a.src = static_cast<const uint4*>(src);
  a.out = static_cast<uint4*>(out);
  a.bufs = reinterpret_cast<char* const*>(peer_bufs);
  a.slice16 = slice_bytes / 16;
  a.slot = g.slot;
  a.count_off = g.count_off;
  a.state_off = g.state_off;
  a.rank = rank;
  a.world = world;
  a.chunks = gather_chunks(slice_bytes);
  a.wait_ns = (uint64_t)debug_wait_limit() * 64;  // the default limit: about a second

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.chunks, (unsigned)world, 1);
  cfg.blockDim = dim3(kGatherThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, peer_gather_kernel, a);
  if (e != cudaSuccess) {
    set_last_error("peer_gather launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(1);
  return CLOVE_OK;
}

int clove_cuda_peer_gather_status(void* own_buf, size_t slice_bytes, int world, void* stream,
                                  int* flags) {
  if (!own_buf || world < 1) {
    set_last_error("peer_gather_status: null buffer or world < 1");
    return CLOVE_ERR_INVALID_ARG;
  }
  GatherLayout g = gather_layout(slice_bytes, world);
  int* word = reinterpret_cast<int*>(static_cast<char*>(own_buf) + g.state_off + 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0;
  cudaError_t e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemcpy(&v, word, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && v) e = cudaMemset(word, 0, sizeof(int));
  if (e != cudaSuccess) {
    set_last_error("peer_gather_status: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  if (flags) *flags = v;
  return v ? CLOVE_ERR_DEVICE_CHECK : CLOVE_OK;
}

}  // extern "C"
