// The C ABI (include/clove_cuda.h): argument validation, pool lifecycle,
// tensor-map encoding and error reporting around the kernel launchers.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>

#include "host.h"

namespace clove {

static thread_local char g_last_error[512] = {0};
static std::atomic<uint64_t> g_launches{0};
static std::atomic<int> g_variant{0};
static std::atomic<uint32_t> g_wait_limit{1u << 24};
static std::atomic<int> g_inject_stall{0};

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

void count_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }
int decode_variant() { return g_variant.load(std::memory_order_relaxed); }
uint32_t debug_wait_limit() { return g_wait_limit.load(std::memory_order_relaxed); }
int debug_inject_stall() { return g_inject_stall.load(std::memory_order_relaxed); }

static int cuda_fail(const char* what, cudaError_t e) {
  set_last_error("%s: %s", what, cudaGetErrorString(e));
  return CLOVE_ERR_CUDA;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda directly.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

static int encode_plane_map(CUtensorMap* map, void* base, const clove_pool& p, bool swizzled) {
  auto fn = tensor_map_encoder();
  if (!fn) {
    set_last_error("cuTensorMapEncodeTiled unavailable from the driver");
    return CLOVE_ERR_CUDA;
  }
  CUtensorMapDataType dt = p.dtype == CLOVE_DTYPE_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                           : p.dtype == CLOVE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r;
  if (!swizzled) {
    // 3-D, dims innermost first: head_dim, kv head, token slot (block*block_size+off)
    cuuint64_t dims[3] = {(cuuint64_t)p.head_dim, (cuuint64_t)p.num_kv_heads,
                          (cuuint64_t)p.num_blocks * (cuuint64_t)p.block_size};
    cuuint64_t strides[2] = {(cuuint64_t)p.head_dim * p.elem_bytes,
                             (cuuint64_t)p.num_kv_heads * p.head_dim * p.elem_bytes};
    cuuint32_t box[3] = {(cuuint32_t)p.head_dim, 1u, (cuuint32_t)p.block_size};
    cuuint32_t estr[3] = {1, 1, 1};
    r = fn(map, dt, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    // 4-D for the 128-byte swizzle: head_dim split into 64-element (128-byte)
    // halves (d_lo, d_hi), kv head, token slot.  One box = a whole
    // [block_size, head_dim] tile, laid out as 128-byte rows (token, d_hi).
    const int nh = p.head_dim / 64;
    cuuint64_t dims[4] = {64, (cuuint64_t)nh, (cuuint64_t)p.num_kv_heads,
                          (cuuint64_t)p.num_blocks * (cuuint64_t)p.block_size};
    cuuint64_t strides[3] = {128, (cuuint64_t)p.head_dim * p.elem_bytes,
                             (cuuint64_t)p.num_kv_heads * p.head_dim * p.elem_bytes};
    cuuint32_t box[4] = {64, (cuuint32_t)nh, 1u, (cuuint32_t)p.block_size};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    r = fn(map, dt, 4, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (%d) for head_dim %d block_size %d", (int)r, p.head_dim,
                   p.block_size);
    return CLOVE_ERR_INVALID_ARG;
  }
  return CLOVE_OK;
}

static int elem_bytes_of(int dtype) {
  switch (dtype) {
    case CLOVE_DTYPE_F32: return 4;
    case CLOVE_DTYPE_BF16: return 2;
    case CLOVE_DTYPE_F16: return 2;
    default: return 0;
  }
}

// RAII device switch: the calls may come from any thread with any device
// current.
struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

static int check_pool_shape(int device, int num_blocks, int block_size, int num_kv_heads, int head_dim,
                            int dtype) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
    set_last_error("no CUDA device");
    return CLOVE_ERR_NO_DEVICE;
  }
  if (device < 0 || device >= n) {
    set_last_error("device %d out of range [0, %d)", device, n);
    return CLOVE_ERR_NO_DEVICE;
  }
  if (num_blocks <= 0 || block_size <= 0 || block_size > 256 || num_kv_heads <= 0 || head_dim <= 0) {
    set_last_error("pool shape (%d, %d, %d, %d) invalid", num_blocks, block_size, num_kv_heads, head_dim);
    return CLOVE_ERR_INVALID_ARG;
  }
  if (block_size < 4 || (block_size & (block_size - 1))) {
    set_last_error("block_size %d must be a power of two in [4, 256]", block_size);
    return CLOVE_ERR_UNSUPPORTED;
  }
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) {
    set_last_error("head_dim %d not built (64, 128, 256)", head_dim);
    return CLOVE_ERR_UNSUPPORTED;
  }
  if (elem_bytes_of(dtype) == 0) {
    set_last_error("dtype code %d (0 = f32, 16 = f16, 160 = bf16)", dtype);
    return CLOVE_ERR_UNSUPPORTED;
  }
  if ((long long)num_blocks * block_size > 0x7fffffffLL) {
    set_last_error("num_blocks * block_size exceeds int32 slot range");
    return CLOVE_ERR_INVALID_ARG;
  }
  return CLOVE_OK;
}

static int finish_pool(clove_pool* p) {
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, p->device);
  if (e != cudaSuccess) return cuda_fail("cudaGetDeviceProperties", e);
  p->num_sms = prop.multiProcessorCount;
  e = cudaMalloc(&p->flags, 256);
  if (e != cudaSuccess) return cuda_fail("cudaMalloc(flags)", e);
  e = cudaMemset(p->flags, 0, 256);
  if (e != cudaSuccess) return cuda_fail("cudaMemset(flags)", e);
  int rc = encode_plane_map(&p->tm_k, p->k_cache, *p, false);
  if (rc) return rc;
  rc = encode_plane_map(&p->tm_v, p->v_cache, *p, false);
  if (rc) return rc;
  p->has_swizzled = 0;
  if (p->elem_bytes == 2 && p->head_dim % 64 == 0 && p->block_size >= 8) {
    rc = encode_plane_map(&p->tm_k_sw, p->k_cache, *p, true);
    if (rc) return rc;
    rc = encode_plane_map(&p->tm_v_sw, p->v_cache, *p, true);
    if (rc) return rc;
    p->has_swizzled = 1;
  }
  return CLOVE_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace clove

using namespace clove;

extern "C" {

int clove_cuda_init(int* num_devices) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (num_devices) *num_devices = (e == cudaSuccess) ? n : 0;
  if (e != cudaSuccess) {
    set_last_error("cudaGetDeviceCount: %s", cudaGetErrorString(e));
    return CLOVE_ERR_NO_DEVICE;
  }
  if (n == 0) {
    set_last_error("no CUDA device");
    return CLOVE_ERR_NO_DEVICE;
  }
  return CLOVE_OK;
}

int clove_cuda_get_last_error(char* buf, size_t n) {
  if (!buf || n == 0) return CLOVE_ERR_INVALID_ARG;
  snprintf(buf, n, "%s", g_last_error);
  return CLOVE_OK;
}

int clove_cuda_pool_create(int device, int num_blocks, int block_size, int num_kv_heads, int head_dim, int dtype,
                           clove_pool_t* out) {
  if (!out) {
    set_last_error("pool_create: null out");
    return CLOVE_ERR_INVALID_ARG;
  }
  *out = nullptr;
  int rc = check_pool_shape(device, num_blocks, block_size, num_kv_heads, head_dim, dtype);
  if (rc) return rc;
  DeviceGuard g(device);
  if (!g.ok) return cuda_fail("cudaSetDevice", cudaGetLastError());
  clove_pool* p = new (std::nothrow) clove_pool();
  if (!p) return CLOVE_ERR_OOM;
  p->device = device;
  p->num_blocks = num_blocks;
  p->block_size = block_size;
  p->num_kv_heads = num_kv_heads;
  p->head_dim = head_dim;
  p->dtype = dtype;
  p->elem_bytes = elem_bytes_of(dtype);
  p->owns_memory = 1;
  p->plane_bytes = (size_t)num_blocks * block_size * num_kv_heads * head_dim * p->elem_bytes;
  void* base = nullptr;
  cudaError_t e = cudaMalloc(&base, 2 * p->plane_bytes);
  if (e != cudaSuccess) {
    delete p;
    set_last_error("pool_create: cudaMalloc(%zu): %s", 2 * p->plane_bytes, cudaGetErrorString(e));
    return CLOVE_ERR_OOM;
  }
  p->k_cache = base;
  p->v_cache = static_cast<unsigned char*>(base) + p->plane_bytes;
  rc = finish_pool(p);
  if (rc) {
    clove_cuda_pool_destroy(p);
    return rc;
  }
  *out = p;
  return CLOVE_OK;
}

int clove_cuda_pool_wrap(int device, void* k_cache, void* v_cache, int num_blocks, int block_size,
                         int num_kv_heads, int head_dim, int dtype, clove_pool_t* out) {
  if (!out || !k_cache || !v_cache) {
    set_last_error("pool_wrap: null pointer");
    return CLOVE_ERR_INVALID_ARG;
  }
  *out = nullptr;
  int rc = check_pool_shape(device, num_blocks, block_size, num_kv_heads, head_dim, dtype);
  if (rc) return rc;
  if (!aligned16(k_cache) || !aligned16(v_cache)) {
    set_last_error("pool_wrap: cache planes must be 16-byte aligned");
    return CLOVE_ERR_INVALID_ARG;
  }
  DeviceGuard g(device);
  if (!g.ok) return cuda_fail("cudaSetDevice", cudaGetLastError());
  clove_pool* p = new (std::nothrow) clove_pool();
  if (!p) return CLOVE_ERR_OOM;
  p->device = device;
  p->num_blocks = num_blocks;
  p->block_size = block_size;
  p->num_kv_heads = num_kv_heads;
  p->head_dim = head_dim;
  p->dtype = dtype;
  p->elem_bytes = elem_bytes_of(dtype);
  p->owns_memory = 0;
  p->plane_bytes = (size_t)num_blocks * block_size * num_kv_heads * head_dim * p->elem_bytes;
  p->k_cache = k_cache;
  p->v_cache = v_cache;
  rc = finish_pool(p);
  if (rc) {
    clove_cuda_pool_destroy(p);
    return rc;
  }
  *out = p;
  return CLOVE_OK;
}

int clove_cuda_pool_destroy(clove_pool_t pool) {
  if (!pool) return CLOVE_OK;
  DeviceGuard g(pool->device);
  if (pool->owns_memory && pool->k_cache) cudaFree(pool->k_cache);
  if (pool->flags) cudaFree(pool->flags);
  delete pool;
  return CLOVE_OK;
}

int clove_cuda_pool_info(clove_pool_t pool, clove_pool_info_t* info) {
  if (!pool || !info) {
    set_last_error("pool_info: null pointer");
    return CLOVE_ERR_INVALID_ARG;
  }
  info->device = pool->device;
  info->num_blocks = pool->num_blocks;
  info->block_size = pool->block_size;
  info->num_kv_heads = pool->num_kv_heads;
  info->head_dim = pool->head_dim;
  info->dtype = pool->dtype;
  info->owns_memory = pool->owns_memory;
  info->k_cache = pool->k_cache;
  info->v_cache = pool->v_cache;
  info->plane_bytes = pool->plane_bytes;
  return CLOVE_OK;
}

int clove_cuda_pool_status(clove_pool_t pool, void* stream, int* flags) {
  if (!pool) {
    set_last_error("pool_status: null pool");
    return CLOVE_ERR_INVALID_ARG;
  }
  DeviceGuard g(pool->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, pool->flags, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemsetAsync(pool->flags, 0, sizeof(int), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail("pool_status", e);
  if (flags) *flags = host;
  if (host) {
    set_last_error("device check flags 0x%x", host);
    return CLOVE_ERR_DEVICE_CHECK;
  }
  return CLOVE_OK;
}

int clove_cuda_reshape_and_cache(clove_pool_t pool, const void* k, const void* v, const int32_t* slot_mapping,
                                 int num_tokens, void* stream) {
  if (!pool || num_tokens < 0) {
    set_last_error("reshape_and_cache: bad pool or num_tokens");
    return CLOVE_ERR_INVALID_ARG;
  }
  if (num_tokens == 0) return CLOVE_OK;
  if (!k || !v || !slot_mapping) {
    set_last_error("reshape_and_cache: null pointer");
    return CLOVE_ERR_INVALID_ARG;
  }
  if (!aligned16(k) || !aligned16(v)) {
    set_last_error("reshape_and_cache: k and v must be 16-byte aligned");
    return CLOVE_ERR_INVALID_ARG;
  }
  DeviceGuard g(pool->device);
  const int row_bytes = pool->num_kv_heads * pool->head_dim * pool->elem_bytes;
  cudaError_t e = launch_reshape_and_cache(k, v, pool->k_cache, pool->v_cache, slot_mapping, num_tokens, row_bytes,
                                           (long long)pool->num_blocks * pool->block_size, pool->flags,
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("reshape_and_cache launch", e);
  count_launches(1);
  return CLOVE_OK;
}

int clove_cuda_gather_kv(clove_pool_t pool, const int32_t* block_tables, int bt_stride, const int32_t* context_lens,
                         int batch, int max_ctx, void* k_out, void* v_out, void* stream) {
  if (!pool || batch < 0 || max_ctx < 0 || bt_stride <= 0) {
    set_last_error("gather_kv: bad arguments");
    return CLOVE_ERR_INVALID_ARG;
  }
  if (batch == 0 || max_ctx == 0) return CLOVE_OK;
  if (!block_tables || !context_lens || !k_out || !v_out || !aligned16(k_out) || !aligned16(v_out)) {
    set_last_error("gather_kv: null or misaligned pointer");
    return CLOVE_ERR_INVALID_ARG;
  }
  if (batch > 65535) {
    set_last_error("gather_kv: batch %d > 65535", batch);
    return CLOVE_ERR_INVALID_ARG;
  }
  DeviceGuard g(pool->device);
  const int row_bytes = pool->num_kv_heads * pool->head_dim * pool->elem_bytes;
  cudaError_t e = launch_gather_kv(pool->k_cache, pool->v_cache, block_tables, bt_stride, context_lens, batch,
                                   max_ctx, pool->block_size, pool->num_blocks, row_bytes, k_out, v_out, pool->flags,
                                   static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("gather_kv launch", e);
  count_launches(1);
  return CLOVE_OK;
}

size_t clove_cuda_decode_workspace_size(clove_pool_t pool, int batch, int num_q_heads, int max_ctx) {
  if (!pool || batch <= 0 || num_q_heads <= 0 || max_ctx < 0) return 0;
  return decode_layout(*pool, batch, num_q_heads, max_ctx).total;
}

static int decode_common(clove_pool_t pool, const void* q, const void* k_new, const void* v_new, int num_q_heads,
                         const int32_t* block_tables, int bt_stride, const int32_t* context_lens, int batch,
                         float scale, int max_ctx, float* out, void* workspace, size_t workspace_bytes,
                         void* stream, const char* who) {
  if (!pool) {
    set_last_error("%s: null pool", who);
    return CLOVE_ERR_INVALID_ARG;
  }
  if (batch < 0 || num_q_heads <= 0 || max_ctx < 0 || bt_stride <= 0) {
    set_last_error("%s: batch %d, num_q_heads %d, max_ctx %d, bt_stride %d", who, batch, num_q_heads, max_ctx,
                   bt_stride);
    return CLOVE_ERR_INVALID_ARG;
  }
  if (num_q_heads % pool->num_kv_heads != 0) {
    set_last_error("%s: num_q_heads %d not a multiple of num_kv_heads %d", who, num_q_heads, pool->num_kv_heads);
    return CLOVE_ERR_INVALID_ARG;
  }
  if (num_q_heads / pool->num_kv_heads > 8) {
    set_last_error("%s: group size %d > 8 not built", who, num_q_heads / pool->num_kv_heads);
    return CLOVE_ERR_UNSUPPORTED;
  }
  if ((long long)max_ctx > (long long)bt_stride * pool->block_size) {
    set_last_error("%s: max_ctx %d exceeds block table capacity %d x %d", who, max_ctx, bt_stride,
                   pool->block_size);
    return CLOVE_ERR_INVALID_ARG;
  }
  if (k_new && max_ctx < 1) {
    set_last_error("%s: max_ctx must be >= 1 with append", who);
    return CLOVE_ERR_INVALID_ARG;
  }
  if (batch == 0) return CLOVE_OK;
  if (!q || !block_tables || !context_lens || !out || !workspace) {
    set_last_error("%s: null pointer", who);
    return CLOVE_ERR_INVALID_ARG;
  }
  if (!aligned16(q) || !aligned16(out) || (reinterpret_cast<uintptr_t>(workspace) & 255u)) {
    set_last_error("%s: q/out must be 16-byte aligned, workspace 256-byte aligned", who);
    return CLOVE_ERR_INVALID_ARG;
  }
  if (k_new && (!v_new || !aligned16(k_new) || !aligned16(v_new))) {
    set_last_error("%s: k_new/v_new null or not 16-byte aligned", who);
    return CLOVE_ERR_INVALID_ARG;
  }
  DeviceGuard g(pool->device);
  if (!g.ok) return cuda_fail("cudaSetDevice", cudaGetLastError());
  DecodeCall c;
  c.q = q;
  c.k_new = k_new;
  c.v_new = v_new;
  c.num_q_heads = num_q_heads;
  c.block_tables = block_tables;
  c.bt_stride = bt_stride;
  c.context_lens = context_lens;
  c.batch = batch;
  c.scale = scale;
  c.max_ctx = max_ctx;
  c.out = out;
  c.workspace = workspace;
  c.workspace_bytes = workspace_bytes;
  if (max_ctx == 0) {
    // Every sequence is empty: the output is all zeros.
    cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float) * (size_t)batch * num_q_heads * pool->head_dim,
                                    static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? CLOVE_OK : cuda_fail("cudaMemsetAsync", e);
  }
  return launch_decode(*pool, c, static_cast<cudaStream_t>(stream));
}

int clove_cuda_paged_decode(clove_pool_t pool, const void* q, int num_q_heads, const int32_t* block_tables,
                            int bt_stride, const int32_t* context_lens, int batch, float scale, int max_ctx,
                            float* out, void* workspace, size_t workspace_bytes, void* stream) {
  return decode_common(pool, q, nullptr, nullptr, num_q_heads, block_tables, bt_stride, context_lens, batch, scale,
                       max_ctx, out, workspace, workspace_bytes, stream, "paged_decode");
}

int clove_cuda_paged_append_decode(clove_pool_t pool, const void* q, const void* k_new, const void* v_new,
                                   int num_q_heads, const int32_t* block_tables, int bt_stride,
                                   const int32_t* context_lens, int batch, float scale, int max_ctx, float* out,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  if (!k_new || !v_new) {
    set_last_error("paged_append_decode: null k_new/v_new");
    return CLOVE_ERR_INVALID_ARG;
  }
  return decode_common(pool, q, k_new, v_new, num_q_heads, block_tables, bt_stride, context_lens, batch, scale,
                       max_ctx, out, workspace, workspace_bytes, stream, "paged_append_decode");
}

int clove_cuda_decode_status(void* workspace, void* stream, int* flags) {
  if (!workspace) {
    set_last_error("decode_status: null workspace");
    return CLOVE_ERR_INVALID_ARG;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // word 1 of the workspace: the flags the last completed call published
  // (its combine kernel moves them there from the accumulating word 0)
  int32_t* last = static_cast<int32_t*>(workspace) + 1;
  int host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, last, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemsetAsync(last, 0, sizeof(int), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail("decode_status", e);
  if (flags) *flags = host;
  if (host) {
    set_last_error("device check flags 0x%x", host);
    return CLOVE_ERR_DEVICE_CHECK;
  }
  return CLOVE_OK;
}

int clove_cuda_set_decode_variant(int variant) {
  if (variant < 0 || variant > 2) {
    set_last_error("set_decode_variant: %d not in {0, 1, 2}", variant);
    return CLOVE_ERR_INVALID_ARG;
  }
  g_variant.store(variant);
  return CLOVE_OK;
}

uint64_t clove_cuda_launch_count(void) { return g_launches.load(); }

int clove_cuda_debug_phase_timing(int enable) {
  set_phase_timing(enable);
  return CLOVE_OK;
}

int clove_cuda_debug_phase_ms(float* plan_ms, float* decode_ms, float* combine_ms) {
  return read_phase_ms(plan_ms, decode_ms, combine_ms);
}

int clove_cuda_debug_trace(void* buffer) {
  set_trace_buffer(buffer);
  return kTrace ? CLOVE_OK : CLOVE_ERR_UNSUPPORTED;
}

int clove_cuda_debug_set(uint32_t wait_limit, int inject_stall) {
  g_wait_limit.store(wait_limit ? wait_limit : (1u << 24));
  g_inject_stall.store(inject_stall ? 1 : 0);
  return CLOVE_OK;
}

}  // extern "C"
