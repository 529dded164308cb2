// Prefill into the paged cache: the prompt tokens of each sequence are
// (optionally) rotated with RoPE, written to their cache slots, and attend
// causally over the sequence's cache — prior context plus the prompt up to
// themselves.
//
// The attention reuses the decode pipeline: every new token is a query row
// whose context is the sequence's cache up to and including its own
// position.  A prep kernel writes the rotated K/V into the slots, the rotated
// queries into the workspace, and expands one block-table row and context
// length per token; the decode kernels (plan -> decode -> combine) then run
// over those rows.  The rows of one sequence read the same K/V tiles, which
// the 126 MB L2 serves for all but the longest prompts.
//
// Semantics follow the reference's FlashAttention step (src/lazy.rs:4821-4923:
// causal mask, RoPE on q and k, scale 1/sqrt(head_dim)) with the exact
// exponential in place of its polynomial approximation (lazy.rs:4846-4851).
#include <algorithm>
#include <cstdlib>
#include <cmath>

#include "../../include/clove_cuda.h"
#include "common.cuh"

#include "host.h"

namespace clove {

struct PrefillPrepArgs {
  const void* q;   // [T, Hq, D]
  const void* k;   // [T, Hkv, D]
  const void* v;
  const int32_t* cu_seqlens;    // [B + 1]
  const int32_t* block_tables;  // [B, bt_stride]
  const int32_t* context_lens;  // [B] cached tokens before the prompt
  void* k_cache;
  void* v_cache;
  void* q_rot;            // out [T, Hq, D]
  int32_t* row_tables;    // out [T, bt_stride]
  int32_t* row_lens;      // out [T] = position + 1
  int32_t* flags;
  int batch, num_tokens, hq, hkv, D, bs, bt_stride, num_blocks, max_ctx;
  float rope_theta;       // 0: no rotation
  int write_rows;         // 1: fill row_tables / row_lens (the decode-reuse path reads them)
};

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// Rotate one head row in place semantics: out[2i], out[2i+1] from in[2i],
// in[2i+1] by angle pos * theta^(-2i/D) (pairs of adjacent elements, the
// pairing of src/lazy.rs:4834-4842).
template <typename T>
__device__ void rope_row(const T* in, T* out, int D, int pos, float theta, int lane0, int stride) {
  for (int i = lane0; i < D / 2; i += stride) {
    const float x0 = Elem<T>::to_f(in[2 * i]), x1 = Elem<T>::to_f(in[2 * i + 1]);
    if (theta > 0.f) {
      const float ang = (float)pos * powf(theta, -2.f * (float)i / (float)D);
      float sn, cs;
      sincosf(ang, &sn, &cs);
      out[2 * i] = from_f<T>(x0 * cs - x1 * sn);
      out[2 * i + 1] = from_f<T>(x0 * sn + x1 * cs);
    } else {
      out[2 * i] = in[2 * i];
      out[2 * i + 1] = in[2 * i + 1];
    }
  }
}

// Rotate 8 consecutive elements (4 adjacent pairs starting at pair i0) of a
// 16-byte vector with the token's per-pair (cos, sin).
template <typename T>
__device__ __forceinline__ uint4 rope8(uint4 in, const float* cs, const float* sn, int i0) {
  const T* x = reinterpret_cast<const T*>(&in);
  uint4 out;
  T* y = reinterpret_cast<T*>(&out);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float x0 = Elem<T>::to_f(x[2 * j]), x1 = Elem<T>::to_f(x[2 * j + 1]);
    y[2 * j] = from_f<T>(x0 * cs[i0 + j] - x1 * sn[i0 + j]);
    y[2 * j + 1] = from_f<T>(x0 * sn[i0 + j] + x1 * cs[i0 + j]);
  }
  return out;
}

// One CTA per prompt token (16-bit pools; f32 pools take rope_row below).
// The token's rotation angles, pos * theta^(-2i/D) for pair i (the pairing of
// src/lazy.rs:4834-4842), are computed once into shared memory and applied to
// every head with 16-byte loads and stores.
template <typename T>
__global__ void __launch_bounds__(128) prefill_prep_kernel(const PrefillPrepArgs p) {
  __shared__ float cs[128], sn[128];  // D / 2 <= 128
  const int t = blockIdx.x;
  // sequence of token t: largest b with cu_seqlens[b] <= t
  int lo = 0, hi = p.batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(p.cu_seqlens + mid) <= t) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  const int pos = __ldg(p.context_lens + b) + (t - __ldg(p.cu_seqlens + b));
  const int32_t* bt = p.block_tables + (size_t)b * p.bt_stride;
  const bool in_range = pos >= 0 && pos < p.max_ctx && pos / p.bs < p.bt_stride;
  if (p.write_rows) {
    // expanded table row and length (the decode-reuse path treats every
    // prompt token as a decode row)
    for (int j = threadIdx.x; j < p.bt_stride; j += blockDim.x) p.row_tables[(size_t)t * p.bt_stride + j] = bt[j];
    if (threadIdx.x == 0) p.row_lens[t] = in_range ? pos + 1 : 0;
  }
  if (threadIdx.x == 0 && !in_range) atomicOr(p.flags, CLOVE_FLAG_CTX_RANGE);
  const bool rot = p.rope_theta > 0.f;
  if (rot) {
    for (int i = threadIdx.x; i < p.D / 2; i += blockDim.x) {
      const float ang = (float)pos * powf(p.rope_theta, -2.f * (float)i / (float)p.D);
      sincosf(ang, &sn[i], &cs[i]);
    }
    __syncthreads();
  }
  constexpr int EPV = 16 / (int)sizeof(T);  // elements per 16-byte vector
  const int vpr = p.D / EPV;                // vectors per head row
  // rotated query rows
  {
    const uint4* qs = reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) + (size_t)t * p.hq * p.D);
    uint4* qd = reinterpret_cast<uint4*>(static_cast<T*>(p.q_rot) + (size_t)t * p.hq * p.D);
    for (int u = threadIdx.x; u < p.hq * vpr; u += blockDim.x) {
      const uint4 x = __ldg(qs + u);
      qd[u] = rot ? rope8<T>(x, cs, sn, (u % vpr) * (EPV / 2)) : x;
    }
  }
  // K (rotated) and V into the slot
  const int phys = in_range ? __ldg(bt + pos / p.bs) : -1;
  if (in_range && (phys < 0 || phys >= p.num_blocks) && threadIdx.x == 0) atomicOr(p.flags, CLOVE_FLAG_BLOCK_OOB);
  if (in_range && phys >= 0 && phys < p.num_blocks) {
    const size_t row = ((size_t)phys * p.bs + pos % p.bs) * p.hkv * p.D;
    const uint4* ks = reinterpret_cast<const uint4*>(static_cast<const T*>(p.k) + (size_t)t * p.hkv * p.D);
    const uint4* vs = reinterpret_cast<const uint4*>(static_cast<const T*>(p.v) + (size_t)t * p.hkv * p.D);
    uint4* kc = reinterpret_cast<uint4*>(static_cast<T*>(p.k_cache) + row);
    uint4* vc = reinterpret_cast<uint4*>(static_cast<T*>(p.v_cache) + row);
    for (int u = threadIdx.x; u < p.hkv * vpr; u += blockDim.x) {
      const uint4 x = __ldg(ks + u);
      kc[u] = rot ? rope8<T>(x, cs, sn, (u % vpr) * (EPV / 2)) : x;
      vc[u] = __ldg(vs + u);
    }
  }
  // Launched as a programmatic dependent of the tensor-core path's plan
  // kernel (which it does not read): wait for it here, at the end, so that
  // this grid's completion implies the plan's for the kernel after it.
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// f32 pools: the same with element-wise rotation.
__global__ void __launch_bounds__(128) prefill_prep_f32_kernel(const PrefillPrepArgs p) {
  using T = float;
  const int t = blockIdx.x;
  int lo = 0, hi = p.batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(p.cu_seqlens + mid) <= t) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  const int pos = __ldg(p.context_lens + b) + (t - __ldg(p.cu_seqlens + b));
  const int32_t* bt = p.block_tables + (size_t)b * p.bt_stride;
  const bool in_range = pos >= 0 && pos < p.max_ctx && pos / p.bs < p.bt_stride;
  if (p.write_rows) {
    for (int j = threadIdx.x; j < p.bt_stride; j += blockDim.x) p.row_tables[(size_t)t * p.bt_stride + j] = bt[j];
    if (threadIdx.x == 0) p.row_lens[t] = in_range ? pos + 1 : 0;
  }
  if (threadIdx.x == 0 && !in_range) atomicOr(p.flags, CLOVE_FLAG_CTX_RANGE);
  const T* qs = static_cast<const T*>(p.q) + (size_t)t * p.hq * p.D;
  T* qd = static_cast<T*>(p.q_rot) + (size_t)t * p.hq * p.D;
  for (int h = 0; h < p.hq; ++h) rope_row<T>(qs + h * p.D, qd + h * p.D, p.D, pos, p.rope_theta, threadIdx.x, blockDim.x);
  if (!in_range) return;
  const int phys = __ldg(bt + pos / p.bs);
  if (phys < 0 || phys >= p.num_blocks) {
    if (threadIdx.x == 0) atomicOr(p.flags, CLOVE_FLAG_BLOCK_OOB);
    return;
  }
  const size_t row = ((size_t)phys * p.bs + pos % p.bs) * p.hkv * p.D;
  const T* ks = static_cast<const T*>(p.k) + (size_t)t * p.hkv * p.D;
  const T* vs = static_cast<const T*>(p.v) + (size_t)t * p.hkv * p.D;
  T* kc = static_cast<T*>(p.k_cache) + row;
  T* vc = static_cast<T*>(p.v_cache) + row;
  for (int h = 0; h < p.hkv; ++h) rope_row<T>(ks + h * p.D, kc + h * p.D, p.D, pos, p.rope_theta, threadIdx.x, blockDim.x);
  for (int i = threadIdx.x; i < p.hkv * p.D; i += blockDim.x) vc[i] = vs[i];
}

struct PrefillLayout {
  size_t off_q, off_tables, off_lens, off_decode, total;
};

static size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

static PrefillLayout prefill_layout(const clove_pool& pool, int num_tokens, int num_q_heads, int bt_stride,
                                    int max_ctx) {
  PrefillLayout L;
  size_t off = 0;
  L.off_q = off;
  off = al256(off + (size_t)num_tokens * num_q_heads * pool.head_dim * pool.elem_bytes);
  L.off_tables = off;
  off = al256(off + (size_t)num_tokens * bt_stride * 4);
  L.off_lens = off;
  off = al256(off + (size_t)num_tokens * 4);
  L.off_decode = off;
  off += std::max(decode_layout(pool, num_tokens, num_q_heads, max_ctx).total, prefill_mma_scratch_bytes(num_tokens));
  L.total = off;
  return L;
}

}  // namespace clove

using namespace clove;

extern "C" {

size_t clove_cuda_prefill_workspace_size(clove_pool_t pool, int num_tokens, int num_q_heads, int bt_stride,
                                         int max_ctx) {
  if (!pool || num_tokens <= 0 || num_q_heads <= 0 || bt_stride <= 0 || max_ctx <= 0) return 0;
  return prefill_layout(*pool, num_tokens, num_q_heads, bt_stride, max_ctx).total;
}

int clove_cuda_paged_prefill(clove_pool_t pool, const void* q, const void* k, const void* v,
                             const int32_t* cu_seqlens, const int32_t* block_tables, int bt_stride,
                             const int32_t* context_lens, int batch, int num_tokens, int num_q_heads, float scale,
                             float rope_theta, int max_ctx, float* out, void* workspace, size_t workspace_bytes,
                             void* stream) {
  if (!pool || batch <= 0 || num_tokens < 0 || num_q_heads <= 0 || bt_stride <= 0 || max_ctx <= 0 ||
      rope_theta < 0.f) {
    set_last_error("paged_prefill: bad arguments");
    return CLOVE_ERR_INVALID_ARG;
  }
  if (num_tokens == 0) return CLOVE_OK;
  if (!q || !k || !v || !cu_seqlens || !block_tables || !context_lens || !out || !workspace ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u)) {
    set_last_error("paged_prefill: null pointer or workspace not 256-byte aligned");
    return CLOVE_ERR_INVALID_ARG;
  }
  if (pool->elem_bytes == 2 && ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                                 reinterpret_cast<uintptr_t>(v)) & 15u)) {
    set_last_error("paged_prefill: q, k, v must be 16-byte aligned");
    return CLOVE_ERR_INVALID_ARG;
  }
  if (num_q_heads % pool->num_kv_heads || (long long)max_ctx > (long long)bt_stride * pool->block_size) {
    set_last_error("paged_prefill: num_q_heads / max_ctx inconsistent with the pool and tables");
    return CLOVE_ERR_INVALID_ARG;
  }
  const PrefillLayout L = prefill_layout(*pool, num_tokens, num_q_heads, bt_stride, max_ctx);
  if (workspace_bytes < L.total) {
    set_last_error("paged_prefill: workspace %zu bytes < required %zu", workspace_bytes, L.total);
    return CLOVE_ERR_WORKSPACE;
  }
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != pool->device) cudaSetDevice(pool->device);
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  PrefillPrepArgs p;
  p.q = q;
  p.k = k;
  p.v = v;
  p.cu_seqlens = cu_seqlens;
  p.block_tables = block_tables;
  p.context_lens = context_lens;
  p.k_cache = pool->k_cache;
  p.v_cache = pool->v_cache;
  p.q_rot = ws + L.off_q;
  p.row_tables = reinterpret_cast<int32_t*>(ws + L.off_tables);
  p.row_lens = reinterpret_cast<int32_t*>(ws + L.off_lens);
  p.flags = pool->flags;
  p.batch = batch;
  p.num_tokens = num_tokens;
  p.hq = num_q_heads;
  p.hkv = pool->num_kv_heads;
  p.D = pool->head_dim;
  p.bs = pool->block_size;
  p.bt_stride = bt_stride;
  p.num_blocks = pool->num_blocks;
  p.max_ctx = max_ctx;
  p.rope_theta = rope_theta;
  // the expanded per-token tables are read only by the decode-reuse path
  const bool tc_path = decode_variant() == 0 && prefill_tc_supported(*pool, num_q_heads);
  const bool mma_path = decode_variant() != 1 && pool->elem_bytes == 2 && pool->has_swizzled &&
                        pool->block_size >= 8 && num_q_heads / pool->num_kv_heads <= 16 &&
                        (pool->head_dim == 64 || pool->head_dim == 128);
  p.write_rows = (tc_path || mma_path) ? 0 : 1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The 2-CTA kernel (M = 256 over an SM pair) for prompts averaging 1024
  // tokens or more; the one-CTA kernel's units of two tiles waste less on
  // short prompts.  CLOVE_PREFILL_CTAS = 1 or 2 (read per call) forces one.
  int ctas = 0;
  if (const char* v = std::getenv("CLOVE_PREFILL_CTAS")) ctas = std::atoi(v);
  if (ctas != 1 && ctas != 2) ctas = (long long)num_tokens >= 1024LL * batch ? 2 : 1;
  cudaError_t e = cudaSuccess;
  if (tc_path) {
    // the tensor-core path's work list first (it reads only the lengths),
    // then the prep kernel as its programmatic dependent, so the two overlap
    const int rc = ctas == 2 ? launch_prefill_tc2(*pool, ws + L.off_q, out, cu_seqlens, context_lens, block_tables,
                                                  bt_stride, batch, num_tokens, num_q_heads, scale, max_ctx,
                                                  ws + L.off_decode, s, kPrefillPlanOnly)
                             : launch_prefill_tc(*pool, ws + L.off_q, out, cu_seqlens, context_lens, block_tables,
                                                 bt_stride, batch, num_tokens, num_q_heads, scale, max_ctx,
                                                 ws + L.off_decode, s, kPrefillPlanOnly);
    if (rc != CLOVE_OK) {
      if (prev >= 0 && prev != pool->device) cudaSetDevice(prev);
      return rc;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)num_tokens);
    cfg.blockDim = dim3(128);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = pool->dtype == CLOVE_DTYPE_BF16 ? cudaLaunchKernelEx(&cfg, prefill_prep_kernel<__nv_bfloat16>, p)
                                        : cudaLaunchKernelEx(&cfg, prefill_prep_kernel<__half>, p);
  } else {
    switch (pool->dtype) {
      case CLOVE_DTYPE_F32: prefill_prep_f32_kernel<<<num_tokens, 128, 0, s>>>(p); break;
      case CLOVE_DTYPE_BF16: prefill_prep_kernel<__nv_bfloat16><<<num_tokens, 128, 0, s>>>(p); break;
      default: prefill_prep_kernel<__half><<<num_tokens, 128, 0, s>>>(p); break;
    }
    e = cudaGetLastError();
  }
  if (prev >= 0 && prev != pool->device) cudaSetDevice(prev);
  if (e != cudaSuccess) {
    set_last_error("paged_prefill prep launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(1);
  // Tensor-core prefill where the shape is covered: tcgen05 (prefill_tc.cu)
  // first, then the warp-MMA kernel (16-bit pools, head_dim 64/128, group
  // <= 16), unless the CUDA-core variant is forced; otherwise every prompt
  // token runs as a decode query row over the cache.
  if (decode_variant() != 1) {
    int prev2 = -1;
    cudaGetDevice(&prev2);
    if (prev2 != pool->device) cudaSetDevice(pool->device);
    int rc = CLOVE_ERR_UNSUPPORTED;
    // 5th-generation tensor cores where the shape is covered (16-bit pools,
    // head_dim 128, group dividing 128, block_size dividing 128), unless the
    // warp-MMA variant is forced (2)
    if (tc_path && ctas == 2)
      rc = launch_prefill_tc2(*pool, ws + L.off_q, out, cu_seqlens, context_lens, block_tables, bt_stride, batch,
                              num_tokens, num_q_heads, scale, max_ctx, ws + L.off_decode, s, kPrefillKernelOnly);
    else if (tc_path)
      rc = launch_prefill_tc(*pool, ws + L.off_q, out, cu_seqlens, context_lens, block_tables, bt_stride, batch,
                             num_tokens, num_q_heads, scale, max_ctx, ws + L.off_decode, s, kPrefillKernelOnly);
    if (rc == CLOVE_ERR_UNSUPPORTED)
      rc = launch_prefill_mma(*pool, ws + L.off_q, out, cu_seqlens, context_lens, block_tables, bt_stride, batch,
                              num_tokens, num_q_heads, scale, max_ctx, ws + L.off_decode, s);
    if (prev2 >= 0 && prev2 != pool->device) cudaSetDevice(prev2);
    if (rc != CLOVE_ERR_UNSUPPORTED) return rc;
  }
  return clove_cuda_paged_decode(pool, ws + L.off_q, num_q_heads, p.row_tables, bt_stride, p.row_lens, num_tokens,
                                 scale, max_ctx, out, ws + L.off_decode, L.total - L.off_decode, stream);
}

}  // extern "C"
