// KV append (reshape-and-cache) and block-table gather kernels.
//
// Both are pure data movement, bound by HBM bandwidth.  A token's K (or V)
// row for all KV heads is contiguous in the cache layout
// [num_blocks, block_size, num_kv_heads, head_dim], so each token moves one
// contiguous row of num_kv_heads * head_dim elements; the copies use 16-byte
// vector accesses (row bytes are a multiple of 16 for every supported shape).
#include "common.cuh"

namespace clove {

// One CTA per token-chunk; warps stride over the 16-byte words of the row.
// Grid: (ceil(num_tokens / TOK_PER_CTA), 2) — y selects the K or V plane.
constexpr int kAppendThreads = 256;

__global__ void __launch_bounds__(kAppendThreads)
reshape_and_cache_kernel(const uint4* __restrict__ k, const uint4* __restrict__ v,
                         uint4* __restrict__ k_cache, uint4* __restrict__ v_cache,
                         const int32_t* __restrict__ slot_mapping, int num_tokens,
                         int row_words, long long num_slots, int32_t* __restrict__ flags) {
  const uint4* src = blockIdx.y == 0 ? k : v;
  uint4* dst = blockIdx.y == 0 ? k_cache : v_cache;
  // Each CTA covers a contiguous range of (token, word) pairs.
  long long total = (long long)num_tokens * row_words;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    int tok = (int)(i / row_words);
    int w = (int)(i - (long long)tok * row_words);
    int slot = __ldg(slot_mapping + tok);
    if (slot < 0) continue;  // padding token
    if ((long long)slot >= num_slots) {
      if (w == 0) atomicOr(flags, CLOVE_FLAG_SLOT_OOB);
      continue;
    }
    dst[(long long)slot * row_words + w] = __ldg(src + i);
  }
}

// Gather [B, max_ctx, row] from the paged cache through the block tables.
__global__ void __launch_bounds__(256)
gather_kv_kernel(const uint4* __restrict__ k_cache, const uint4* __restrict__ v_cache,
                 const int32_t* __restrict__ block_tables, int bt_stride,
                 const int32_t* __restrict__ context_lens, int max_ctx, int block_size,
                 int num_blocks, int row_words, uint4* __restrict__ k_out, uint4* __restrict__ v_out,
                 int32_t* __restrict__ flags) {
  const uint4* src = blockIdx.z == 0 ? k_cache : v_cache;
  uint4* dst = blockIdx.z == 0 ? k_out : v_out;
  int b = blockIdx.y;
  int ctx = __ldg(context_lens + b);
  if (ctx < 0 || ctx > max_ctx || ctx > bt_stride * block_size) {
    if (blockIdx.x == 0 && threadIdx.x == 0 && blockIdx.z == 0) atomicOr(flags, CLOVE_FLAG_CTX_RANGE);
    ctx = max(0, min(ctx, min(max_ctx, bt_stride * block_size)));
  }
  long long total = (long long)max_ctx * row_words;
  uint4* drow = dst + (long long)b * total;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    int t = (int)(i / row_words);
    int w = (int)(i - (long long)t * row_words);
    uint4 val = make_uint4(0, 0, 0, 0);
    if (t < ctx) {
      int logical = t / block_size;
      int off = t - logical * block_size;
      int phys = __ldg(block_tables + (long long)b * bt_stride + logical);
      if (phys >= 0 && phys < num_blocks) {
        val = __ldg(src + ((long long)phys * block_size + off) * row_words + w);
      } else if (w == 0) {
        atomicOr(flags, CLOVE_FLAG_BLOCK_OOB);
      }
    }
    drow[i] = val;
  }
}

cudaError_t launch_reshape_and_cache(const void* k, const void* v, void* k_cache, void* v_cache,
                                     const int32_t* slot_mapping, int num_tokens, int row_bytes,
                                     long long num_slots, int32_t* flags, cudaStream_t stream) {
  int row_words = row_bytes / 16;
  long long total = (long long)num_tokens * row_words;
  long long blocks = (total + kAppendThreads - 1) / kAppendThreads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  dim3 grid((unsigned)blocks, 2);
  reshape_and_cache_kernel<<<grid, kAppendThreads, 0, stream>>>(
      (const uint4*)k, (const uint4*)v, (uint4*)k_cache, (uint4*)v_cache, slot_mapping, num_tokens,
      row_words, num_slots, flags);
  return cudaGetLastError();
}

cudaError_t launch_gather_kv(const void* k_cache, const void* v_cache, const int32_t* block_tables,
                             int bt_stride, const int32_t* context_lens, int batch, int max_ctx,
                             int block_size, int num_blocks, int row_bytes, void* k_out, void* v_out,
                             int32_t* flags, cudaStream_t stream) {
  int row_words = row_bytes / 16;
  long long per_seq = (long long)max_ctx * row_words;
  long long bx = (per_seq + 255) / 256;
  if (bx > 1024) bx = 1024;
  if (bx < 1) bx = 1;
  dim3 grid((unsigned)bx, batch, 2);
  gather_kv_kernel<<<grid, 256, 0, stream>>>((const uint4*)k_cache, (const uint4*)v_cache, block_tables,
                                             bt_stride, context_lens, max_ctx, block_size, num_blocks,
                                             row_words, (uint4*)k_out, (uint4*)v_out, flags);
  return cudaGetLastError();
}

}  // namespace clove
