// Shared device helpers for the sm_100a PagedAttention kernels: dtype
// conversion, mbarrier / bulk-tensor (TMA) PTX wrappers with bounded waits,
// and the parameter blocks the kernels take.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/clove_cuda.h"

namespace clove {

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
};

// Load N consecutive elements (N*sizeof(T) bytes, naturally aligned) and widen
// to float.  N*sizeof(T) is 4, 8 or 16 bytes in every instantiation.
template <typename T, int N>
__device__ __forceinline__ void load_vec_f32(const T* p, float (&o)[N]) {
  constexpr int BYTES = N * (int)sizeof(T);
  static_assert(BYTES == 4 || BYTES == 8 || BYTES == 16 || BYTES == 32, "vector width");
  if constexpr (BYTES == 32) {
    load_vec_f32<T, N / 2>(p, reinterpret_cast<float(&)[N / 2]>(o[0]));
    load_vec_f32<T, N / 2>(p + N / 2, reinterpret_cast<float(&)[N / 2]>(o[N / 2]));
  } else if constexpr (sizeof(T) == 4) {
    if constexpr (N == 4) {
      float4 v = *reinterpret_cast<const float4*>(p);
      o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
    } else if constexpr (N == 2) {
      float2 v = *reinterpret_cast<const float2*>(p);
      o[0] = v.x; o[1] = v.y;
    } else {
      o[0] = Elem<T>::to_f(p[0]);
    }
  } else {
    // 16-bit types: move raw words, then widen pairs.
    constexpr int W = BYTES / 4;
    uint32_t w[W];
    if constexpr (W == 4) {
      uint4 v = *reinterpret_cast<const uint4*>(p);
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else if constexpr (W == 2) {
      uint2 v = *reinterpret_cast<const uint2*>(p);
      w[0] = v.x; w[1] = v.y;
    } else {
      w[0] = *reinterpret_cast<const uint32_t*>(p);
    }
#pragma unroll
    for (int i = 0; i < W; ++i) {
      T lo, hi;
      uint16_t l16 = (uint16_t)(w[i] & 0xffffu), h16 = (uint16_t)(w[i] >> 16);
      lo = *reinterpret_cast<T*>(&l16);
      hi = *reinterpret_cast<T*>(&h16);
      o[2 * i] = Elem<T>::to_f(lo);
      o[2 * i + 1] = Elem<T>::to_f(hi);
    }
  }
}

// ---------------------------------------------------------------------------
// mbarrier + bulk tensor copy (TMA) wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialisation may start before the previous kernel on the stream has
// finished; griddep_wait blocks the calling thread until that kernel has
// completed and its writes are visible.  griddep_launch_dependents lets the
// next such kernel be scheduled (it still waits before reading anything).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Upper bound on try_wait polls before a wait is declared stuck.  Each poll
// may suspend the thread for a hardware-chosen interval, so this is seconds of
// wall time: far beyond any legitimate wait, short enough to never hang a GPU.
constexpr uint32_t kWaitLimit = 1u << 24;

// Bounded wait on `bar` completing the phase with `parity`.  Returns false
// (and sets CLOVE_FLAG_TIMEOUT in *err) if the limit ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err,
                                                  uint32_t limit = kWaitLimit) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  atomicOr(err, CLOVE_FLAG_TIMEOUT);
  return false;
}

// L2 eviction policy for streamed KV tiles: they are read once per step.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Fetch a tensor map (a __grid_constant__ kernel parameter) into the
// descriptor cache ahead of its first bulk tensor copy.
__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 3-D tiled bulk tensor load global -> shared, completion counted on `bar`.
// Coordinates are in elements, innermost first.  c0 is always 0 here (a tile
// starts at the beginning of a head row), which satisfies the 16-byte rule
// for the innermost coordinate.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Plain (non-tensor) bulk copy global -> shared; both addresses 16-byte
// aligned and the size a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// 4-D tiled bulk tensor load (the swizzled K/V maps); c0 = 0 always.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Make this thread's generic-proxy global writes visible to later async-proxy
// (TMA) reads.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named-barrier OR reduction: returns nonzero in every participating thread
// if `pred` was nonzero in any of them.
__device__ __forceinline__ int named_bar_or(int id, int nthreads, int pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\tselp.s32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(pred), "r"(id), "r"(nthreads)
      : "memory");
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------------------
// kernel parameter blocks
// ---------------------------------------------------------------------------
// Floats per softmax state row (acc[D], m, l) in shared scratch and in the
// partials: padded to a multiple of 4 so rows start 16-byte aligned.
__host__ __device__ constexpr int state_stride(int head_dim) { return head_dim + 4; }

struct DecodeArgs {
  const void* q;             // [B, Hq, D] pool dtype
  const void* k_new;         // [B, Hkv, D] or null (no append)
  const void* v_new;
  void* k_cache;             // plane K [NB, bs, Hkv, D] (written only by the append)
  void* v_cache;
  const int32_t* block_tables;
  const int32_t* context_lens;
  float* out;                // [B, Hq, D] f32
  float* partials;           // [num_ctas, 2, group, state_stride(D)] f32: a CTA's first / last piece when split
  int4* desc;                // [num_ctas]: segment at the CTA's range start {b, h, offset, blocks}
  int32_t* err;              // device check flags raised by this call (accumulated)
  int32_t* err_last;         // flags of the last completed call (published by the combine)
  long long* total;          // work W of this call in (segment, block) units (CTA 0 writes it)
  int bt_stride;
  int batch;
  int num_kv_heads;
  int num_blocks;
  int block_size;
  int num_ctas;              // P: decode CTAs (the partition's divisor)
  int seg_cost;              // alpha: stream positions charged per segment for a piece's fixed cost
  int max_ctx;
  int group;                 // query heads per KV head (runtime, <= template G)
  int append;                // 1: context_lens are pre-append lengths
  int nstage;                // pipeline depth (a multiple of ncw)
  int ncw;                   // consumer warps that take stages (<= the kernel's NCW)
  int stage_blocks;          // blocks per pipeline stage (1..4)
  int nscr;                  // merge scratch buffers (1 or 2)
  uint32_t wait_limit;       // polls before a pipeline wait is declared stuck
  int inject_stall;          // test hook: the first stage of each CTA's first piece is never filled
  float qscale;              // scale * log2(e)
  unsigned long long* trace; // timeline buffer (trace builds only; null otherwise)
};

// Timeline tracing for measurement builds (compiled with -DCLOVE_TRACE; the
// product build contains none of it).  u64 slots of the buffer:
//   [0] plan start, [1] plan end, [2] first combine CTA start, [3] last
//   combine CTA end; [kTraceCta + 4 cta + k]: decode CTA k = 0 entry, 1 past
//   griddepcontrol.wait, 2 producer done, 3 last consumer done;
//   [kTraceUnit + 3 u + k]: piece u = 16 cta + (piece index within the
//   CTA, < 16) k = 0 posted, 1 merged, 2 (cta << 32) | blocks.  Times from
//   %globaltimer (ns).  The Q/K/V projection kernels use [kTraceCta + 8 cta
//   + k]: k = 0 entry, 1 producer past griddepcontrol.wait, 2 first stage
//   landed, 3 last MMA issued, 4 epilogue done.
#ifdef CLOVE_TRACE
constexpr bool kTrace = true;
#else
constexpr bool kTrace = false;
#endif
constexpr int kTraceCta = 16;
constexpr int kTraceMaxCta = 4096;
constexpr int kTraceUnit = kTraceCta + 4 * kTraceMaxCta;
constexpr int kTraceMaxUnit = 65536;

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

}  // namespace clove
