// Shared by the prefill kernels: the arguments and the longest-first work
// list of (sequence, query tile) items (prefill_plan_kernel, defined in
// prefill_mma.cu).
#pragma once

#include "common.cuh"

namespace clove {

constexpr int kPfBins = 256;  // size bins of the longest-first ordering

struct PrefillArgs {
  const void* q;                // rotated queries [T, Hq, D]
  float* out;                   // [T, Hq, D]
  const int32_t* cu_seqlens;    // [B + 1]
  const int32_t* context_lens;  // [B]
  const int32_t* block_tables;  // [B, bt_stride]
  int2* items;                  // (b, tile)
  int32_t* n_items;
  int32_t* unit_counter;
  int32_t* err;
  int bt_stride, batch, hq, hkv, group, bs, num_blocks, tq, nstage, sb, max_ctx;
  uint32_t wait_limit;
  float qscale;                 // scale * log2(e)
  int inject_stall;             // test hook (tensor-core prefill): one K/V step is never filled
  unsigned long long* trace;    // step timeline of CTA 0 (trace builds only; null otherwise)
};

// Work list: every (sequence, tile of p.tq prompt tokens), ordered by key
// count descending (counting sort over kPfBins bins); zeroes the claim counter.
__global__ void prefill_plan_kernel(PrefillArgs p);

}  // namespace clove
