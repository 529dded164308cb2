// Host-side declarations shared by the C-ABI layer and the kernel launchers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/clove_cuda.h"
#include "common.cuh"

// The pool handle behind clove_pool_t.
struct clove_pool {
  int device;
  int num_blocks;
  int block_size;
  int num_kv_heads;
  int head_dim;
  int dtype;
  int elem_bytes;
  int owns_memory;
  void* k_cache;
  void* v_cache;
  size_t plane_bytes;
  int32_t* flags;   // device word for the append / gather kernels' check flags
  int num_sms;
  CUtensorMap tm_k;  // 3-D maps {head_dim, num_kv_heads, num_blocks*block_size}
  CUtensorMap tm_v;
  // 16-bit pools only: head_dim split into 64-element boxes with the 128-byte
  // swizzle (the tensor-core kernel's conflict-free shared-memory layout).
  CUtensorMap tm_k_sw;
  CUtensorMap tm_v_sw;
  int has_swizzled;
};

namespace clove {

// Decode CTAs per SM are capped here; the workspace holds per-CTA state for
// num_sms * kMaxCtasPerSm CTAs.
constexpr int kMaxCtasPerSm = 4;

// Workspace carve-up for one decode call; offsets in bytes from the base.
// It does not depend on the batch or the context lengths: the partition
// leaves at most two partial states per decode CTA.
struct DecodeLayout {
  int max_ctas;
  size_t off_err, off_desc, off_partials;
  size_t total;
};

DecodeLayout decode_layout(const clove_pool& pool, int batch, int num_q_heads, int max_ctx);

struct DecodeCall {
  const void* q;
  const void* k_new;  // null: plain decode
  const void* v_new;
  int num_q_heads;
  const int32_t* block_tables;
  int bt_stride;
  const int32_t* context_lens;
  int batch;
  float scale;
  int max_ctx;
  float* out;
  void* workspace;
  size_t workspace_bytes;
};

// Returns a CLOVE_* status; sets the thread's last-error text on failure.
int launch_decode(const clove_pool& pool, const DecodeCall& call, cudaStream_t stream);

cudaError_t launch_reshape_and_cache(const void* k, const void* v, void* k_cache, void* v_cache,
                                     const int32_t* slot_mapping, int num_tokens, int row_bytes,
                                     long long num_slots, int32_t* flags, cudaStream_t stream);
cudaError_t launch_gather_kv(const void* k_cache, const void* v_cache, const int32_t* block_tables,
                             int bt_stride, const int32_t* context_lens, int batch, int max_ctx,
                             int block_size, int num_blocks, int row_bytes, void* k_out, void* v_out,
                             int32_t* flags, cudaStream_t stream);

// Launch a decode kernel as a programmatic dependent of the previous kernel
// on the stream (the plan): it may start early and must execute
// griddepcontrol.wait before reading the plan's outputs.
template <typename Kern, typename Args>
cudaError_t launch_dependent(Kern kern, unsigned grid, unsigned threads, size_t smem, cudaStream_t stream,
                             const CUtensorMap& tk, const CUtensorMap& tv, const Args& a) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tk, tv, a);
}

size_t prefill_mma_scratch_bytes(int num_tokens);
// What a tensor-core prefill launch issues: its plan kernel (the work list),
// the attention kernel (a programmatic dependent of the kernel before it), or both.
constexpr int kPrefillPlanOnly = 1, kPrefillKernelOnly = 2, kPrefillBoth = 3;
bool prefill_tc_supported(const clove_pool& pool, int num_q_heads);
int launch_prefill_tc(const clove_pool& pool, const void* q_rot, float* out, const int32_t* cu_seqlens,
                      const int32_t* context_lens, const int32_t* block_tables, int bt_stride, int batch,
                      int num_tokens, int num_q_heads, float scale, int max_ctx, void* ws, cudaStream_t stream,
                      int phase);
int launch_prefill_tc2(const clove_pool& pool, const void* q_rot, float* out, const int32_t* cu_seqlens,
                       const int32_t* context_lens, const int32_t* block_tables, int bt_stride, int batch,
                       int num_tokens, int num_q_heads, float scale, int max_ctx, void* ws, cudaStream_t stream,
                      int phase);
int launch_prefill_mma(const clove_pool& pool, const void* q_rot, float* out, const int32_t* cu_seqlens,
                       const int32_t* context_lens, const int32_t* block_tables, int bt_stride, int batch,
                       int num_tokens, int num_q_heads, float scale, int max_ctx, void* ws, cudaStream_t stream);

// cuTensorMapEncodeTiled from the driver (null if unavailable)
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// error text / launch accounting (capi.cu)
void set_last_error(const char* fmt, ...);
void count_launches(int n);
int decode_variant();  // 0 auto, 1 simt, 2 mma
uint32_t debug_wait_limit();
int debug_inject_stall();
void set_phase_timing(int on);  // decode_kernels.cu
int read_phase_ms(float* plan_ms, float* decode_ms, float* combine_ms);
void set_trace_buffer(void* buf);  // decode_kernels.cu
unsigned long long* trace_buffer();

}  // namespace clove
