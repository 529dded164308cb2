/*
 * clove_blocks.h — KV block manager for the device-resident paged cache.
 *
 * The reference has no block allocator: block_tables is a caller-supplied
 * tensor (src/nn.rs:535) and its only pool is the size-keyed BufferPool of
 * whole buffers (src/device.rs:177-222).  This manager owns the mapping
 * sequence -> physical blocks of one clove_pool_t, so a serving loop can grow,
 * fork and free sequences and hand the decode its block tables:
 *   - free list of physical blocks (host side; lowest ids first);
 *   - per-block reference counts: forked sequences share their prefix blocks;
 *   - copy-on-write: before a sequence appends into a block it shares, the
 *     manager gives it a private copy and reports the (src, dst) pair, which
 *     clove_cuda_copy_blocks copies on the GPU;
 *   - export of int32 block tables / context lengths for a batch.
 * The manager is host state only (no device memory of its own); it is not
 * thread-safe — one manager per serving thread.
 */
#ifndef CLOVE_BLOCKS_H
#define CLOVE_BLOCKS_H

#include <stddef.h>
#include <stdint.h>

#include "clove_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#define CLOVE_ERR_NO_BLOCKS -8  /* pool exhausted */
#define CLOVE_ERR_NO_SEQ    -9  /* unknown or already-used sequence id */

typedef struct clove_blocks* clove_blocks_t;

/* A manager for `num_blocks` blocks of `block_size` tokens; sequence ids are
 * 0 .. max_seqs-1. */
int clove_blocks_create(int num_blocks, int block_size, int max_seqs, clove_blocks_t* out);
int clove_blocks_destroy(clove_blocks_t m);

/* Start sequence `seq` with `len` tokens of capacity (blocks allocated). */
int clove_blocks_add(clove_blocks_t m, int seq, int len);

/* Make room for `len` tokens in total (allocating blocks as needed) and set
 * the sequence's length.  When the block that will receive token len-1 is
 * shared with another sequence, it is replaced by a fresh block and the pair
 * (old, new) is appended to src/dst (capacity *n_copies on input, count on
 * output); the caller copies those blocks (clove_cuda_copy_blocks) before it
 * writes.  Fails with CLOVE_ERR_NO_BLOCKS, leaving the sequence unchanged,
 * when the pool cannot supply the blocks. */
int clove_blocks_reserve(clove_blocks_t m, int seq, int len, int32_t* src, int32_t* dst, int* n_copies);

/* New sequence `child` sharing all blocks of `parent` (same length). */
int clove_blocks_fork(clove_blocks_t m, int parent, int child);

/* Release a sequence's blocks (reference counts drop; blocks at zero return
 * to the free list). */
int clove_blocks_free(clove_blocks_t m, int seq);

/* Free blocks, and a sequence's length / block count (-1 if unknown). */
int clove_blocks_num_free(clove_blocks_t m);
int clove_blocks_seq_len(clove_blocks_t m, int seq);
int clove_blocks_seq_blocks(clove_blocks_t m, int seq);

/* Block tables and lengths of a batch of sequences, host int32:
 * tables [n, stride] (unused entries -1), lens [n].  Fails if a sequence has
 * more than `stride` blocks. */
int clove_blocks_export(clove_blocks_t m, const int32_t* seqs, int n, int stride, int32_t* tables,
                        int32_t* lens);

/* GPU: copy whole blocks src[i] -> dst[i] of both planes of `pool`, bit for
 * bit (the copy-on-write step).  src, dst: device int32 [n]. */
int clove_cuda_copy_blocks(clove_pool_t pool, const int32_t* src, const int32_t* dst, int n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CLOVE_BLOCKS_H */
