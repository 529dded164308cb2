// Pieces shared by the decode kernels (CUDA-core and tensor-core consumers):
// the work-unit walk, the TMA producer warp, and the epilogue that merges
// consumer-warp softmax states and performs the split-K combine.
//
// Pipeline.  A stage holds `sb` consecutive logical blocks of one unit (K and
// V tiles, each [block_size, head_dim] of one KV head), i.e. TT = sb *
// block_size tokens.  Stages are numbered continuously over all units a CTA
// walks; stage g lives in ring slot g % nstage with mbarrier phase
// (g / nstage) & 1.  Each stage is consumed by exactly one consumer warp,
// which arrives on its `empty` barrier (count 1) when done.
#pragma once

#include "common.cuh"

namespace clove {

__device__ __forceinline__ int clamp_ctx(const int32_t* ctx_lens, int b, int max_ctx, int append) {
  int c = __ldg(ctx_lens + b);
  c = max(0, min(c, max_ctx - append));
  return c + append;
}

struct Unit {
  int b, c, h;
  int L;        // tokens the sequence attends over
  int blk0;     // first logical block of the chunk
  int nblk;     // blocks in this chunk
  int nstages;  // stages in this chunk
};

__device__ __forceinline__ Unit load_unit(const DecodeArgs& a, int u, int sb) {
  Unit x;
  const int2 it = a.items[u / a.num_kv_heads];
  x.h = u - (u / a.num_kv_heads) * a.num_kv_heads;
  x.b = it.x;
  x.c = it.y;
  x.L = clamp_ctx(a.context_lens, x.b, a.max_ctx, a.append);
  const int cb = __ldg(a.chunk_blocks);
  x.blk0 = x.c * cb;
  x.nblk = min(cb, (x.L + a.block_size - 1) / a.block_size - x.blk0);
  x.nstages = (x.nblk + sb - 1) / sb;
  return x;
}

// Shared-memory carve-up: [ring: nstage x (K tiles | V tiles)] [barriers]
// [scratch].  Every region starts 128-byte aligned (bulk tensor copies want
// 128-byte aligned destinations).
struct SmemPlan {
  int tile_stride;   // bytes of one [block_size, head_dim] tile, 128-aligned
  int stage_bytes;   // 2 * sb tiles
  int ring_bytes;
  int bar_bytes;
  int scratch_bytes;
  int total;         // + 128 alignment slack
};

__host__ __device__ inline SmemPlan smem_plan(int block_size, int head_dim, int elem_bytes, int sb, int nstage,
                                             int scratch_bytes) {
  SmemPlan s;
  s.tile_stride = (block_size * head_dim * elem_bytes + 127) & ~127;
  s.stage_bytes = 2 * sb * s.tile_stride;
  s.ring_bytes = s.stage_bytes * nstage;
  s.bar_bytes = ((2 * nstage * 8 + 64) + 127) & ~127;
  s.scratch_bytes = (scratch_bytes + 127) & ~127;
  s.total = s.ring_bytes + s.bar_bytes + s.scratch_bytes + 128;
  return s;
}

// K tiles of a stage are at [0, sb) * tile_stride, V tiles at
// [sb, 2 sb) * tile_stride; consecutive tiles are contiguous when
// block_size * head_dim * elem_bytes is a multiple of 128 (always true for the
// supported shapes), so a stage's K (and V) rows form one dense
// [sb * block_size, head_dim] array.

// Fused reshape-and-cache of the new token for head h (called by the
// producer warp before it issues the copies of the unit's last chunk).
template <typename T, int D>
__device__ __forceinline__ void append_row(const DecodeArgs& a, const Unit& x, int lane) {
  const int bs = a.block_size;
  const int pos = x.L - 1;
  const int phys = __ldg(a.block_tables + (size_t)x.b * a.bt_stride + pos / bs);
  if (phys < 0 || phys >= a.num_blocks) {
    if (lane == 0) atomicOr(a.err, CLOVE_FLAG_BLOCK_OOB);
  } else {
    const size_t row = (((size_t)phys * bs + (pos % bs)) * a.num_kv_heads + x.h) * D;
    const size_t src = ((size_t)x.b * a.num_kv_heads + x.h) * D;
    constexpr int WORDS = D * (int)sizeof(T) / 16;
    const uint4* ks = reinterpret_cast<const uint4*>(static_cast<const T*>(a.k_new) + src);
    const uint4* vs = reinterpret_cast<const uint4*>(static_cast<const T*>(a.v_new) + src);
    uint4* kd = reinterpret_cast<uint4*>(static_cast<T*>(a.k_cache) + row);
    uint4* vd = reinterpret_cast<uint4*>(static_cast<T*>(a.v_cache) + row);
    for (int w = lane; w < WORDS; w += 32) {
      kd[w] = __ldg(ks + w);
      vd[w] = __ldg(vs + w);
    }
    fence_proxy_async_global();
  }
  __syncwarp();
}

// The producer warp: walks the CTA's units and streams their K/V tiles into
// the ring.  Only lane 0 issues copies; the warp loads block-table entries 32
// at a time and broadcasts them.  On a stuck wait it raises the abort flag and
// drains its own in-flight copies (bounded) before returning.
//
// NBOX: boxes per tile.  1 = one [block_size, head_dim] box (dense rows);
// D/64 = head_dim split into 64-element (128-byte) boxes written with the
// 128-byte swizzle, sub-tile hb at tile offset hb * block_size * 128.
template <typename T, int D, int NBOX>
__device__ void produce(const DecodeArgs& a, const CUtensorMap* tm_k, const CUtensorMap* tm_v,
                        unsigned char* ring, const SmemPlan& sp, int sb, uint64_t* full, uint64_t* empty,
                        volatile int* s_abort, int n_units) {
  const int lane = threadIdx.x & 31;
  const int bs = a.block_size;
  const uint32_t tile_bytes = (uint32_t)(bs * D * (int)sizeof(T));
  const uint64_t pol = policy_evict_first();
  int slot = 0;
  uint32_t phase = 0;
  bool aborted = false;
  for (int u = blockIdx.x; u < n_units && !aborted; u += gridDim.x) {
    const Unit x = load_unit(a, u, sb);
    if (a.append && x.c == a.seq_chunks[x.b] - 1) append_row<T, D>(a, x, lane);
    const int32_t* bt = a.block_tables + (size_t)x.b * a.bt_stride + x.blk0;
    int my = 0;
    for (int s = 0; s < x.nstages && !aborted; ++s) {
      const int j0 = s * sb;  // first block of this stage within the chunk
      if ((j0 & 31) == 0) {
        my = 0;
        if (j0 + lane < x.nblk) {
          my = __ldg(bt + j0 + lane);
          if (my < 0 || my >= a.num_blocks) {
            atomicOr(a.err, CLOVE_FLAG_BLOCK_OOB);
            my = 0;
          }
        }
      }
      const int nb = min(sb, x.nblk - j0);
      int ok = 1;
      int phys[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) phys[i] = __shfl_sync(0xffffffffu, my, (j0 + i) & 31);
      if (lane == 0) {
        if (*s_abort || !mbar_wait_bounded(&empty[slot], phase ^ 1, a.err)) {
          ok = 0;
          *s_abort = 1;
        } else {
          mbar_arrive_expect_tx(&full[slot], 2u * tile_bytes * (uint32_t)nb);
          unsigned char* st = ring + (size_t)slot * sp.stage_bytes;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (i < nb) {
#pragma unroll
              for (int hb = 0; hb < NBOX; ++hb) {
                const int off = hb * (D / NBOX) * (int)sizeof(T) * bs;
                tma_load_3d(st + i * sp.tile_stride + off, tm_k, &full[slot], hb * (D / NBOX), x.h, phys[i] * bs,
                            pol);
                tma_load_3d(st + (sb + i) * sp.tile_stride + off, tm_v, &full[slot], hb * (D / NBOX), x.h,
                            phys[i] * bs, pol);
              }
            }
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) aborted = true;
      if (++slot == a.nstage) {
        slot = 0;
        phase ^= 1;
      }
    }
  }
  if (aborted && lane == 0) {
    // Drain: the last nstage issues may still be in flight.
    int s = slot;
    uint32_t ph = phase;
    for (int k = 0; k < a.nstage; ++k) {
      if (--s < 0) {
        s = a.nstage - 1;
        ph ^= 1;
      }
      for (uint32_t i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(&full[s], ph)) break;
    }
  }
}

// Epilogue of one unit, run by all NCT consumer threads (ct in [0, NCT)).
// scratch holds NW partial softmax states [NW][G][D + 2] = (acc[D], m, l) in
// the log2 domain.  A sequence in one chunk is finished here; otherwise the
// merged chunk state goes to the workspace partials and the CTA that finishes
// the last chunk of (b, h) — found with an atomic counter, no waiting —
// merges all chunks and writes the output.
template <int D, int G, int NW, int NCT>
__device__ void finish_unit(const DecodeArgs& a, const Unit& x, const float* scratch, volatile int* s_last,
                            int ct) {
  const int group = a.group;
  const int Hkv = a.num_kv_heads;
  const int Hq = Hkv * group;
  const int nchunks = a.seq_chunks[x.b];
  float* part_base = a.partials + (((size_t)x.b * Hkv + x.h) * a.max_chunks) * G * (D + 2);
  for (int idx = ct; idx < group * D; idx += NCT) {
    const int g = idx / D, d = idx - (idx / D) * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, scratch[(w * G + g) * (D + 2) + D]);
    float Ls = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float mw = scratch[(w * G + g) * (D + 2) + D];
      if (mw != -INFINITY) {
        const float f = exp2f(mw - M);
        Ls = fmaf(scratch[(w * G + g) * (D + 2) + D + 1], f, Ls);
        O = fmaf(scratch[(w * G + g) * (D + 2) + d], f, O);
      }
    }
    if (nchunks == 1) {
      a.out[((size_t)x.b * Hq + (size_t)x.h * group + g) * D + d] = O / Ls;
    } else {
      float* P = part_base + ((size_t)x.c * G + g) * (D + 2);
      P[d] = O;
      if (d == 0) {
        P[D] = M;
        P[D + 1] = Ls;
      }
    }
  }
  if (nchunks > 1) {
    __threadfence();
    named_bar_sync(1, NCT);
    if (ct == 0) {
      const int prev = atomicAdd(a.counters + (size_t)x.b * Hkv + x.h, 1);
      *s_last = (prev == nchunks - 1);
    }
    named_bar_sync(1, NCT);
    if (*s_last) {
      __threadfence();
      for (int idx = ct; idx < group * D; idx += NCT) {
        const int g = idx / D, d = idx - (idx / D) * D;
        float M = -INFINITY;
        for (int cc = 0; cc < nchunks; ++cc)
          M = fmaxf(M, __ldcg(part_base + ((size_t)cc * G + g) * (D + 2) + D));
        float Ls = 0.f, O = 0.f;
        for (int cc = 0; cc < nchunks; ++cc) {
          const float* P = part_base + ((size_t)cc * G + g) * (D + 2);
          const float f = exp2f(__ldcg(P + D) - M);
          Ls = fmaf(__ldcg(P + D + 1), f, Ls);
          O = fmaf(__ldcg(P + d), f, O);
        }
        a.out[((size_t)x.b * Hq + (size_t)x.h * group + g) * D + d] = O / Ls;
      }
      if (ct == 0) a.counters[(size_t)x.b * Hkv + x.h] = 0;
    }
  }
}

}  // namespace clove
