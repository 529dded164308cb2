// Tensor-handle FFI (include/clove_ffi.h): the reference-facing C ABI of the
// decode path, over the clove_cuda_* entry points.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <new>
#include <unordered_map>
#include <vector>

#include "../../include/clove_ffi.h"
#include "host.h"

struct clove_tensor {
  void* ptr = nullptr;
  size_t bytes = 0;         // requested bytes
  size_t cap = 0;           // allocation size (cache key)
  std::vector<int64_t> shape;
  int dtype = CLOVE_DTYPE_F32;
  int device = 0;
  bool owns = false;
  std::vector<int32_t> host_i32;  // host copy of small int32 tensors made from host data
  clove_pool_t pool = nullptr;    // lazily wrapped when used as a kv cache
};

namespace {

using clove::set_last_error;

int elem_bytes(int dtype) {
  switch (dtype) {
    case CLOVE_DTYPE_F32: return 4;
    case CLOVE_DTYPE_I32: return 4;
    case CLOVE_DTYPE_BF16: return 2;
    case CLOVE_DTYPE_F16: return 2;
    default: return 0;
  }
}

// Per-device size-keyed cache of device buffers.
struct DeviceCache {
  std::mutex mu;
  std::unordered_map<size_t, std::vector<void*>> free_lists;
  size_t held = 0;
  void* workspace = nullptr;  // cudaMallocAsync'd on the legacy stream (stream-ordered free on growth)
  size_t workspace_bytes = 0;
  int32_t* flags_host = nullptr;  // pinned word: the check flags of the last decode, read after it
};

constexpr int kMaxDev = 64;
DeviceCache g_cache[kMaxDev];

size_t round_cap(size_t n) { return std::max<size_t>(256, (n + 255) & ~size_t(255)); }

struct DevGuard {
  int prev = -1;
  bool ok = true;
  explicit DevGuard(int d) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != d) ok = cudaSetDevice(d) == cudaSuccess;
  }
  ~DevGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

void* cache_alloc(int device, size_t cap) {
  DeviceCache& c = g_cache[device];
  {
    std::lock_guard<std::mutex> lk(c.mu);
    auto it = c.free_lists.find(cap);
    if (it != c.free_lists.end() && !it->second.empty()) {
      void* p = it->second.back();
      it->second.pop_back();
      c.held -= cap;
      return p;
    }
  }
  void* p = nullptr;
  if (cudaMalloc(&p, cap) == cudaSuccess) return p;
  // out of memory with buffers parked in the cache: give them back and retry once
  cudaGetLastError();
  {
    std::lock_guard<std::mutex> lk(c.mu);
    for (auto& kv : c.free_lists)
      for (void* q : kv.second) cudaFree(q);
    c.free_lists.clear();
    c.held = 0;
  }
  if (cudaMalloc(&p, cap) == cudaSuccess) return p;
  cudaGetLastError();
  return nullptr;
}

void cache_release(int device, void* p, size_t cap) {
  DeviceCache& c = g_cache[device];
  std::lock_guard<std::mutex> lk(c.mu);
  c.free_lists[cap].push_back(p);
  c.held += cap;
}

size_t numel(const std::vector<int64_t>& s) {
  size_t n = 1;
  for (int64_t d : s) n *= (size_t)d;
  return n;
}

CTensor make_tensor(const int64_t* shape, int ndim, int dtype, int device) {
  if (ndim < 0 || ndim > 8 || (ndim > 0 && !shape) || elem_bytes(dtype) == 0 || device < 0 || device >= kMaxDev) {
    set_last_error("tensor: bad shape, dtype %d or device %d", dtype, device);
    return nullptr;
  }
  clove_tensor* t = new (std::nothrow) clove_tensor();
  if (!t) return nullptr;
  t->shape.assign(shape, shape + ndim);
  for (int64_t d : t->shape)
    if (d < 0) {
      delete t;
      set_last_error("tensor: negative dimension");
      return nullptr;
    }
  t->dtype = dtype;
  t->device = device;
  t->bytes = numel(t->shape) * (size_t)elem_bytes(dtype);
  return t;
}

}  // namespace

extern "C" {

CTensor clove_tensor_create_nd(const void* data, const int64_t* shape, int ndim, int dtype, int device) {
  CTensor t = make_tensor(shape, ndim, dtype, device);
  if (!t) return nullptr;
  DevGuard g(device);
  if (!g.ok) {
    delete t;
    set_last_error("tensor: cudaSetDevice(%d) failed", device);
    return nullptr;
  }
  t->cap = round_cap(t->bytes);
  t->ptr = cache_alloc(device, t->cap);
  if (!t->ptr) {
    delete t;
    set_last_error("tensor: device allocation of %zu bytes failed", t->cap);
    return nullptr;
  }
  t->owns = true;
  if (data && t->bytes) {
    if (cudaMemcpyAsync(t->ptr, data, t->bytes, cudaMemcpyHostToDevice, 0) != cudaSuccess) {
      clove_tensor_free(t);
      set_last_error("tensor: host-to-device copy failed");
      return nullptr;
    }
    if (dtype == CLOVE_DTYPE_I32 && t->bytes <= (1u << 20)) {
      const int32_t* src = static_cast<const int32_t*>(data);
      t->host_i32.assign(src, src + t->bytes / 4);
    }
  }
  return t;
}

CTensor clove_tensor_create(const float* data, size_t rows, size_t cols) {
  if (!data) return nullptr;
  const int64_t shape[2] = {(int64_t)rows, (int64_t)cols};
  return clove_tensor_create_nd(data, shape, 2, CLOVE_DTYPE_F32, 0);
}

CTensor clove_tensor_from_device(void* device_ptr, const int64_t* shape, int ndim, int dtype, int device) {
  if (!device_ptr) {
    set_last_error("tensor_from_device: null pointer");
    return nullptr;
  }
  CTensor t = make_tensor(shape, ndim, dtype, device);
  if (!t) return nullptr;
  t->ptr = device_ptr;
  t->owns = false;
  return t;
}

void clove_tensor_free(CTensor t) {
  if (!t) return;
  if (t->pool) clove_cuda_pool_destroy(t->pool);
  if (t->owns && t->ptr) cache_release(t->device, t->ptr, t->cap);
  delete t;
}

void clove_tensor_data(CTensor t, void* out) {
  if (!t || !out) return;
  DevGuard g(t->device);
  if (cudaMemcpyAsync(out, t->ptr, t->bytes, cudaMemcpyDeviceToHost, 0) != cudaSuccess ||
      cudaStreamSynchronize(0) != cudaSuccess)
    set_last_error("tensor_data: device-to-host copy failed");
}

int clove_tensor_shape(CTensor t, int64_t* shape) {
  if (!t) return -1;
  if (shape)
    for (size_t i = 0; i < t->shape.size(); ++i) shape[i] = t->shape[i];
  return (int)t->shape.size();
}

size_t clove_tensor_cache_bytes(int device) {
  if (device < 0 || device >= kMaxDev) return 0;
  std::lock_guard<std::mutex> lk(g_cache[device].mu);
  return g_cache[device].held;
}

CTensor clove_paged_attention(CTensor q, CTensor k, CTensor v, CTensor kv, CTensor bt, CTensor cl) {
  if (!q || !k || !v || !kv || !bt || !cl) {
    set_last_error("paged_attention: null tensor");
    return nullptr;
  }
  // kv [2, num_blocks, block_size, Hkv, D]
  if (kv->shape.size() != 5 || kv->shape[0] != 2) {
    set_last_error("paged_attention: kv_cache must be [2, num_blocks, block_size, num_kv_heads, head_dim]");
    return nullptr;
  }
  const int nb = (int)kv->shape[1], bs = (int)kv->shape[2], hkv = (int)kv->shape[3], d = (int)kv->shape[4];
  const int dev = kv->device;
  if (q->device != dev || k->device != dev || v->device != dev || bt->device != dev || cl->device != dev) {
    set_last_error("paged_attention: tensors on different devices");
    return nullptr;
  }
  if (q->dtype != kv->dtype || k->dtype != kv->dtype || v->dtype != kv->dtype) {
    set_last_error("paged_attention: q, k, v must have the kv_cache dtype");
    return nullptr;
  }
  if (bt->dtype != CLOVE_DTYPE_I32 || cl->dtype != CLOVE_DTYPE_I32 || bt->shape.size() != 2 ||
      cl->shape.size() != 1) {
    set_last_error("paged_attention: block_tables int32 [B, M], context_lens int32 [B]");
    return nullptr;
  }
  const int batch = (int)cl->shape[0];
  if (q->shape.empty() || (int)q->shape[0] != batch || (int)bt->shape[0] != batch) {
    set_last_error("paged_attention: batch mismatch between q, block_tables and context_lens");
    return nullptr;
  }
  const size_t per_seq_q = numel(q->shape) / std::max(batch, 1);
  if (per_seq_q % d) {
    set_last_error("paged_attention: q row of %zu elements is not a multiple of head_dim %d", per_seq_q, d);
    return nullptr;
  }
  const int hq = (int)(per_seq_q / d);
  if (numel(k->shape) != (size_t)batch * hkv * d || numel(v->shape) != (size_t)batch * hkv * d) {
    set_last_error("paged_attention: k, v must hold [B, %d * %d] elements", hkv, d);
    return nullptr;
  }
  DevGuard g(dev);
  if (!kv->pool) {
    const size_t plane = (size_t)nb * bs * hkv * d * elem_bytes(kv->dtype);
    int rc = clove_cuda_pool_wrap(dev, kv->ptr, static_cast<char*>(kv->ptr) + plane, nb, bs, hkv, d, kv->dtype,
                                  &kv->pool);
    if (rc) return nullptr;
  }
  // max_ctx (tokens attended): from the host copy of context_lens when the
  // tensor was made from host data, else the block table's capacity (no
  // device-to-host read on the call path; the kernels flag lengths beyond it).
  long long max_ctx = (long long)bt->shape[1] * bs;
  if ((int)cl->host_i32.size() == batch) {
    long long m = 1;
    for (int32_t c : cl->host_i32) m = std::max<long long>(m, (long long)c + 1);
    max_ctx = std::min(max_ctx, m);
  }
  if (max_ctx < 1) max_ctx = 1;
  if (max_ctx > INT32_MAX) {
    set_last_error("paged_attention: block table of %lld tokens per sequence is too large", max_ctx);
    return nullptr;
  }
  const int64_t oshape[2] = {batch, (int64_t)hq * d};
  CTensor out = clove_tensor_create_nd(nullptr, oshape, 2, CLOVE_DTYPE_F32, dev);
  if (!out) return nullptr;
  const size_t need = clove_cuda_decode_workspace_size(kv->pool, batch, hq, (int)max_ctx);
  DeviceCache& c = g_cache[dev];
  void* ws = nullptr;
  size_t ws_bytes = 0;
  int32_t* flags_host = nullptr;
  {
    std::lock_guard<std::mutex> lk(c.mu);
    if (!c.flags_host && cudaMallocHost(reinterpret_cast<void**>(&c.flags_host), sizeof(int32_t)) != cudaSuccess) {
      c.flags_host = nullptr;
      cudaGetLastError();
    }
    if (c.workspace_bytes < need) {
      // Stream-ordered: queued decodes on the legacy stream finish with the
      // old buffer before it is released; the host does not wait.
      if (c.workspace) cudaFreeAsync(c.workspace, 0);
      c.workspace = nullptr;
      c.workspace_bytes = 0;
      if (cudaMallocAsync(&c.workspace, round_cap(need), 0) == cudaSuccess &&
          cudaMemsetAsync(c.workspace, 0, round_cap(need), 0) == cudaSuccess) {  // decode scratch starts zeroed
        c.workspace_bytes = round_cap(need);
      } else {
        c.workspace = nullptr;
        cudaGetLastError();
      }
    }
    ws = c.workspace;
    ws_bytes = c.workspace_bytes;
    flags_host = c.flags_host;
  }
  if (!ws || !flags_host) {
    clove_tensor_free(out);
    set_last_error("paged_attention: workspace allocation of %zu bytes failed", need);
    return nullptr;
  }
  const float scale = 1.0f / std::sqrt((float)d);
  int rc = clove_cuda_paged_append_decode(kv->pool, q->ptr, k->ptr, v->ptr, hq, static_cast<const int32_t*>(bt->ptr),
                                          (int)bt->shape[1], static_cast<const int32_t*>(cl->ptr), batch, scale,
                                          (int)max_ctx, static_cast<float*>(out->ptr), ws, ws_bytes, nullptr);
  if (rc) {
    clove_tensor_free(out);
    return nullptr;
  }
  // Device-side checks: the decode's check-flag word (bad block ids, context
  // lengths beyond the table, a pipeline wait that ran out).  The reference
  // op is synchronous and aborts on bad input; here the call waits for the
  // decode and returns NULL with the flags in the error text instead of a
  // silently clamped result.
  // (word 1 of the scratch: the flags of the call that just completed)
  if (cudaMemcpyAsync(flags_host, static_cast<int32_t*>(ws) + 1, sizeof(int32_t), cudaMemcpyDeviceToHost, 0) !=
          cudaSuccess ||
      cudaStreamSynchronize(0) != cudaSuccess) {
    clove_tensor_free(out);
    set_last_error("paged_attention: %s", cudaGetErrorString(cudaGetLastError()));
    return nullptr;
  }
  if (*flags_host) {
    const int f = *flags_host;
    clove_tensor_free(out);
    set_last_error("paged_attention: device check flags 0x%x:%s%s%s%s", f,
                   (f & CLOVE_FLAG_BLOCK_OOB) ? " block id outside the pool;" : "",
                   (f & CLOVE_FLAG_CTX_RANGE) ? " context length outside [0, block table capacity);" : "",
                   (f & CLOVE_FLAG_SLOT_OOB) ? " slot outside the pool;" : "",
                   (f & CLOVE_FLAG_TIMEOUT) ? " a pipeline wait ran out;" : "");
    return nullptr;
  }
  return out;
}

}  // extern "C"
