// KV block manager (include/clove_blocks.h): host-side allocation of the
// paged pool's blocks to sequences, with reference-counted sharing and
// copy-on-write, plus the GPU block-copy kernel.
#include <algorithm>
#include <new>
#include <vector>

#include "../../include/clove_blocks.h"
#include "host.h"

struct clove_blocks {
  int num_blocks = 0;
  int block_size = 0;
  std::vector<int32_t> free_list;          // stack; top = next block handed out
  std::vector<int32_t> refcount;           // per physical block
  std::vector<std::vector<int32_t>> seq_blocks;
  std::vector<int32_t> seq_len;            // -1: sequence not in use
};

namespace {

using clove::set_last_error;

bool valid_seq(const clove_blocks* m, int seq) {
  return m && seq >= 0 && seq < (int)m->seq_len.size();
}

int blocks_for(int len, int bs) { return (len + bs - 1) / bs; }

int32_t take_block(clove_blocks* m) {
  const int32_t b = m->free_list.back();
  m->free_list.pop_back();
  m->refcount[b] = 1;
  return b;
}

void drop_block(clove_blocks* m, int32_t b) {
  if (--m->refcount[b] == 0) m->free_list.push_back(b);
}

}  // namespace

extern "C" {

int clove_blocks_create(int num_blocks, int block_size, int max_seqs, clove_blocks_t* out) {
  if (!out || num_blocks <= 0 || block_size <= 0 || max_seqs <= 0) {
    set_last_error("blocks_create: bad arguments");
    return CLOVE_ERR_INVALID_ARG;
  }
  clove_blocks* m = new (std::nothrow) clove_blocks();
  if (!m) return CLOVE_ERR_OOM;
  m->num_blocks = num_blocks;
  m->block_size = block_size;
  m->free_list.resize(num_blocks);
  for (int i = 0; i < num_blocks; ++i) m->free_list[i] = num_blocks - 1 - i;  // block 0 on top
  m->refcount.assign(num_blocks, 0);
  m->seq_blocks.resize(max_seqs);
  m->seq_len.assign(max_seqs, -1);
  *out = m;
  return CLOVE_OK;
}

int clove_blocks_destroy(clove_blocks_t m) {
  delete m;
  return CLOVE_OK;
}

int clove_blocks_add(clove_blocks_t m, int seq, int len) {
  if (!valid_seq(m, seq) || m->seq_len[seq] >= 0 || len < 0) {
    set_last_error("blocks_add: sequence %d unknown or in use, or len %d < 0", seq, len);
    return CLOVE_ERR_NO_SEQ;
  }
  const int need = blocks_for(len, m->block_size);
  if (need > (int)m->free_list.size()) {
    set_last_error("blocks_add: %d blocks needed, %zu free", need, m->free_list.size());
    return CLOVE_ERR_NO_BLOCKS;
  }
  m->seq_blocks[seq].clear();
  for (int i = 0; i < need; ++i) m->seq_blocks[seq].push_back(take_block(m));
  m->seq_len[seq] = len;
  return CLOVE_OK;
}

int clove_blocks_reserve(clove_blocks_t m, int seq, int len, int32_t* src, int32_t* dst, int* n_copies) {
  if (!valid_seq(m, seq) || m->seq_len[seq] < 0 || len < m->seq_len[seq] || !n_copies) {
    set_last_error("blocks_reserve: sequence %d unknown, or len %d shrinks it", seq, len);
    return CLOVE_ERR_NO_SEQ;
  }
  const int cap = *n_copies;
  *n_copies = 0;
  std::vector<int32_t>& bl = m->seq_blocks[seq];
  const int old_len = m->seq_len[seq];
  const int need = blocks_for(len, m->block_size);
  const int grow = std::max(0, need - (int)bl.size());
  // Shared blocks that receive new tokens (positions old_len .. len-1) must
  // be privatised first.
  std::vector<int> cow;
  if (len > old_len) {
    const int first = old_len / m->block_size, last = std::min((len - 1) / m->block_size, (int)bl.size() - 1);
    for (int j = first; j <= last; ++j)
      if (m->refcount[bl[j]] > 1) cow.push_back(j);
  }
  if (grow + (int)cow.size() > (int)m->free_list.size()) {
    set_last_error("blocks_reserve: %d blocks needed, %zu free", grow + (int)cow.size(), m->free_list.size());
    return CLOVE_ERR_NO_BLOCKS;
  }
  if ((int)cow.size() > cap || (!cow.empty() && (!src || !dst))) {
    set_last_error("blocks_reserve: %zu copy pairs, room for %d", cow.size(), cap);
    return CLOVE_ERR_INVALID_ARG;
  }
  for (int j : cow) {
    const int32_t fresh = take_block(m);
    src[*n_copies] = bl[j];
    dst[*n_copies] = fresh;
    ++*n_copies;
    drop_block(m, bl[j]);
    bl[j] = fresh;
  }
  for (int i = 0; i < grow; ++i) bl.push_back(take_block(m));
  m->seq_len[seq] = len;
  return CLOVE_OK;
}

int clove_blocks_fork(clove_blocks_t m, int parent, int child) {
  if (!valid_seq(m, parent) || !valid_seq(m, child) || m->seq_len[parent] < 0 || m->seq_len[child] >= 0) {
    set_last_error("blocks_fork: parent %d must be in use and child %d free", parent, child);
    return CLOVE_ERR_NO_SEQ;
  }
  m->seq_blocks[child] = m->seq_blocks[parent];
  for (int32_t b : m->seq_blocks[child]) ++m->refcount[b];
  m->seq_len[child] = m->seq_len[parent];
  return CLOVE_OK;
}

int clove_blocks_free(clove_blocks_t m, int seq) {
  if (!valid_seq(m, seq) || m->seq_len[seq] < 0) {
    set_last_error("blocks_free: sequence %d not in use", seq);
    return CLOVE_ERR_NO_SEQ;
  }
  for (int32_t b : m->seq_blocks[seq]) drop_block(m, b);
  m->seq_blocks[seq].clear();
  m->seq_len[seq] = -1;
  return CLOVE_OK;
}

int clove_blocks_num_free(clove_blocks_t m) { return m ? (int)m->free_list.size() : -1; }

int clove_blocks_seq_len(clove_blocks_t m, int seq) { return valid_seq(m, seq) ? m->seq_len[seq] : -1; }

int clove_blocks_seq_blocks(clove_blocks_t m, int seq) {
  return valid_seq(m, seq) && m->seq_len[seq] >= 0 ? (int)m->seq_blocks[seq].size() : -1;
}

int clove_blocks_export(clove_blocks_t m, const int32_t* seqs, int n, int stride, int32_t* tables, int32_t* lens) {
  if (!m || n < 0 || stride <= 0 || (n && (!seqs || !tables || !lens))) {
    set_last_error("blocks_export: bad arguments");
    return CLOVE_ERR_INVALID_ARG;
  }
  for (int i = 0; i < n; ++i) {
    const int s = seqs[i];
    if (!valid_seq(m, s) || m->seq_len[s] < 0) {
      set_last_error("blocks_export: sequence %d not in use", s);
      return CLOVE_ERR_NO_SEQ;
    }
    const std::vector<int32_t>& bl = m->seq_blocks[s];
    if ((int)bl.size() > stride) {
      set_last_error("blocks_export: sequence %d has %zu blocks > stride %d", s, bl.size(), stride);
      return CLOVE_ERR_INVALID_ARG;
    }
    int32_t* row = tables + (size_t)i * stride;
    std::fill(row, row + stride, -1);
    std::copy(bl.begin(), bl.end(), row);
    lens[i] = m->seq_len[s];
  }
  return CLOVE_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// GPU block copy: one CTA per (pair, plane); 16-byte words.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) copy_blocks_kernel(uint4* k_cache, uint4* v_cache, const int32_t* src,
                                                          const int32_t* dst, int block_words, int num_blocks,
                                                          int32_t* flags) {
  const int i = blockIdx.x;
  uint4* plane = blockIdx.y == 0 ? k_cache : v_cache;
  const int s = src[i], d = dst[i];
  if (s < 0 || s >= num_blocks || d < 0 || d >= num_blocks) {
    if (threadIdx.x == 0 && blockIdx.y == 0) atomicOr(flags, CLOVE_FLAG_BLOCK_OOB);
    return;
  }
  const uint4* from = plane + (size_t)s * block_words;
  uint4* to = plane + (size_t)d * block_words;
  for (int w = threadIdx.x; w < block_words; w += blockDim.x) to[w] = from[w];
}

extern "C" int clove_cuda_copy_blocks(clove_pool_t pool, const int32_t* src, const int32_t* dst, int n,
                                      void* stream) {
  if (!pool || n < 0) {
    set_last_error("copy_blocks: bad arguments");
    return CLOVE_ERR_INVALID_ARG;
  }
  if (n == 0) return CLOVE_OK;
  if (!src || !dst) {
    set_last_error("copy_blocks: null pointer");
    return CLOVE_ERR_INVALID_ARG;
  }
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != pool->device) cudaSetDevice(pool->device);
  const int block_words = (int)((size_t)pool->block_size * pool->num_kv_heads * pool->head_dim * pool->elem_bytes / 16);
  copy_blocks_kernel<<<dim3((unsigned)n, 2), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(pool->k_cache), static_cast<uint4*>(pool->v_cache), src, dst, block_words,
      pool->num_blocks, pool->flags);
  cudaError_t e = cudaGetLastError();
  if (prev >= 0 && prev != pool->device) cudaSetDevice(prev);
  if (e != cudaSuccess) {
    set_last_error("copy_blocks launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  clove::count_launches(1);
  return CLOVE_OK;
}
