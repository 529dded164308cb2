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

// Units travel from the producer to the consumers through a small ring of
// shared-memory slots (kUnitRing deep): the unit's metadata plus a copy of
// its query rows, brought in by one bulk copy.  Consumers never touch global
// memory at a unit boundary.
constexpr int kUnitRing = 2;

struct UnitSlot {
  Unit x;
  int nchunks;  // chunks of sequence x.b
  int valid;    // 0: no more work
};

// Shared-memory carve-up: [ring: nstage x (K tiles | V tiles)] [barriers]
// [unit slots] [query buffers] [2 scratch buffers].  Every region starts 128-byte
// aligned (bulk tensor copies want 128-byte aligned destinations).
struct SmemPlan {
  int tile_stride;   // bytes of one [block_size, head_dim] tile, 128-aligned
  int stage_bytes;   // 2 * sb tiles
  int ring_bytes;
  int bar_bytes;     // full/empty per stage, ufull/uempty per unit slot, scr_empty x2, misc ints
  int slot_bytes;    // kUnitRing unit slots
  int q_stride;      // bytes of one query buffer (group * head_dim elements max)
  int scratch_bytes; // one scratch buffer (consumer-warp states of one unit)
  int total;         // + 128 alignment slack
};

__host__ __device__ inline SmemPlan smem_plan(int block_size, int head_dim, int elem_bytes, int sb, int nstage,
                                             int scratch_bytes, int q_bytes) {
  SmemPlan s;
  s.tile_stride = (block_size * head_dim * elem_bytes + 127) & ~127;
  s.stage_bytes = 2 * sb * s.tile_stride;
  s.ring_bytes = s.stage_bytes * nstage;
  s.bar_bytes = ((2 * nstage + 2 * kUnitRing + 2) * 8 + 64 + 127) & ~127;
  s.slot_bytes = (kUnitRing * (int)sizeof(UnitSlot) + 127) & ~127;
  s.q_stride = (q_bytes + 127) & ~127;
  s.scratch_bytes = (scratch_bytes + 127) & ~127;
  s.total = s.ring_bytes + s.bar_bytes + s.slot_bytes + kUnitRing * s.q_stride + 2 * s.scratch_bytes + 128;
  return s;
}

// Pointers into the carve-up, from the aligned base.
struct SmemPtrs {
  unsigned char* ring;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* ufull;
  uint64_t* uempty;
  uint64_t* scr_empty;  // [2]: scratch buffer free again (arrived by the warp that merged it)
  volatile int* misc;   // [0] abort
  int* arrive;          // [2]: consumer warps done with the unit in scratch buffer k
  UnitSlot* slots;
  unsigned char* qbuf;  // kUnitRing x q_stride
  float* scratch;       // 2 x scratch_floats
  int scratch_floats;
};

__device__ __forceinline__ SmemPtrs smem_ptrs(unsigned char* base, const SmemPlan& sp, int nstage) {
  SmemPtrs p;
  p.ring = base;
  p.full = reinterpret_cast<uint64_t*>(base + sp.ring_bytes);
  p.empty = p.full + nstage;
  p.ufull = p.empty + nstage;
  p.uempty = p.ufull + kUnitRing;
  p.scr_empty = p.uempty + kUnitRing;
  p.misc = reinterpret_cast<volatile int*>(p.scr_empty + 2);
  p.arrive = const_cast<int*>(p.misc) + 2;
  p.slots = reinterpret_cast<UnitSlot*>(base + sp.ring_bytes + sp.bar_bytes);
  p.qbuf = base + sp.ring_bytes + sp.bar_bytes + sp.slot_bytes;
  p.scratch = reinterpret_cast<float*>(p.qbuf + kUnitRing * sp.q_stride);
  p.scratch_floats = sp.scratch_bytes / 4;
  return p;
}

// Barrier initialisation (thread 0), then a CTA barrier.  ncw_all: consumer
// warps in the CTA (each arrives on uempty once per unit).
__device__ __forceinline__ void init_barriers(const SmemPtrs& p, int nstage, int ncw_all) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < nstage; ++s) {
      mbar_init(&p.full[s], 1);
      mbar_init(&p.empty[s], 1);
    }
    for (int k = 0; k < kUnitRing; ++k) {
      mbar_init(&p.ufull[k], 1);
      mbar_init(&p.uempty[k], ncw_all);
    }
    mbar_init(&p.scr_empty[0], 1);
    mbar_init(&p.scr_empty[1], 1);
    p.misc[0] = 0;
    p.arrive[0] = 0;
    p.arrive[1] = 0;
    fence_barrier_init();
  }
  __syncthreads();
  // Launched as a programmatic dependent of the plan kernel: from here on the
  // kernel reads the plan's outputs, so wait for that grid to finish.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The split-K combine kernel that follows may be scheduled now; it waits
  // for this grid to finish before it reads anything.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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

// The producer warp.  It claims units from the plan's longest-first list
// with an atomic counter, posts each one (metadata + a bulk copy of its query
// rows) to the unit ring, performs the fused append when the unit holds the
// sequence's last chunk, then streams the unit's K/V tiles into the stage
// ring.  Halfway through a unit's stages (once the ring is primed) it claims
// the next unit and loads its metadata and first block-table entries, so a
// unit boundary costs no global round trip on the critical path.  Only lane
// 0 issues copies.  On a stuck wait it raises the abort flag and drains its
// own in-flight copies (bounded) before returning.
//
// NBOX: 1 = one 3-D [block_size, head_dim] box per tile (dense rows); 2 =
// one 4-D box per tile written with the 128-byte swizzle as
// 128-byte rows (token, 64-dim half).
template <typename T, int D, int NBOX>
__device__ void produce(const DecodeArgs& a, const CUtensorMap* tm_k, const CUtensorMap* tm_v, const SmemPtrs& sm,
                        const SmemPlan& sp, int sb, int n_units) {
  const int lane = threadIdx.x & 31;
  const int bs = a.block_size;
  const uint32_t tile_bytes = (uint32_t)(bs * D * (int)sizeof(T));
  const uint32_t q_bytes = (uint32_t)(a.group * D * (int)sizeof(T));
  const int Hq = a.num_kv_heads * a.group;
  const uint64_t pol = policy_evict_first();
  int slot = 0, uk = 0;
  uint32_t phase = 0, uphase = 0;
  bool aborted = false;

  // Block-table entries, 32 at a time (lane i holds entry j0 + i); entries
  // outside the pool are flagged and replaced by block 0 (never followed).
  auto table = [&](const Unit& x, int j0) {
    const bool in = j0 + lane < x.nblk;
    int v = in ? __ldg(a.block_tables + (size_t)x.b * a.bt_stride + x.blk0 + j0 + lane) : 0;
    if (in && (v < 0 || v >= a.num_blocks)) {
      atomicOr(a.err, CLOVE_FLAG_BLOCK_OOB);
      v = 0;
    }
    return v;
  };
  auto claim = [&](int& u, Unit& x, int& bt0) {
    int v = 0;
    if (lane == 0) v = atomicAdd(a.unit_counter, 1);
    u = __shfl_sync(0xffffffffu, v, 0);
    if (u < n_units) {
      x = load_unit(a, u, sb);
      bt0 = table(x, 0);
    }
  };

  int u, bt0 = 0;
  Unit x;
  claim(u, x, bt0);
  while (!aborted) {
    // ---- post the unit (or the end marker) to the unit ring ----
    int ok = 1;
    if (lane == 0) {
      if (*sm.misc || !mbar_wait_bounded(&sm.uempty[uk], uphase ^ 1, a.err, a.wait_limit)) {
        ok = 0;
        *sm.misc = 1;
      } else if (u >= n_units) {
        sm.slots[uk].valid = 0;
        mbar_arrive(&sm.ufull[uk]);
      } else {
        sm.slots[uk].x = x;
        sm.slots[uk].nchunks = a.seq_chunks[x.b];
        sm.slots[uk].valid = 1;
        mbar_arrive_expect_tx(&sm.ufull[uk], q_bytes);
        const T* qsrc = static_cast<const T*>(a.q) + ((size_t)x.b * Hq + (size_t)x.h * a.group) * D;
        bulk_load(sm.qbuf + uk * sp.q_stride, qsrc, q_bytes, &sm.ufull[uk]);
      }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) {
      aborted = true;
      break;
    }
    if (u >= n_units) break;
    if (++uk == kUnitRing) {
      uk = 0;
      uphase ^= 1;
    }

    if (a.append && x.c == a.seq_chunks[x.b] - 1) append_row<T, D>(a, x, lane);
    int my = bt0;
    int u2 = n_units, bt2 = 0;
    Unit x2;
    const int claim_at = min(x.nstages - 1, a.nstage / 2);
    for (int s = 0; s < x.nstages && !aborted; ++s) {
      const int j0 = s * sb;  // first block of this stage within the chunk
      if ((j0 & 31) == 0 && j0 > 0) my = table(x, j0);
      const int nb = min(sb, x.nblk - j0);
      int phys[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) phys[i] = __shfl_sync(0xffffffffu, my, (j0 + i) & 31);
      ok = 1;
      if (lane == 0) {
        if (*sm.misc || !mbar_wait_bounded(&sm.empty[slot], phase ^ 1, a.err, a.wait_limit)) {
          ok = 0;
          *sm.misc = 1;
        } else if (a.inject_stall && u == 0 && s == 0) {
          // test hook: the first stage of the first unit is never filled, so
          // its consumer's wait runs out
        } else {
          mbar_arrive_expect_tx(&sm.full[slot], 2u * tile_bytes * (uint32_t)nb);
          unsigned char* st = sm.ring + (size_t)slot * sp.stage_bytes;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (i < nb) {
              if constexpr (NBOX == 1) {
                tma_load_3d(st + i * sp.tile_stride, tm_k, &sm.full[slot], 0, x.h, phys[i] * bs, pol);
                tma_load_3d(st + (sb + i) * sp.tile_stride, tm_v, &sm.full[slot], 0, x.h, phys[i] * bs, pol);
              } else {
                tma_load_4d(st + i * sp.tile_stride, tm_k, &sm.full[slot], 0, 0, x.h, phys[i] * bs, pol);
                tma_load_4d(st + (sb + i) * sp.tile_stride, tm_v, &sm.full[slot], 0, 0, x.h, phys[i] * bs, pol);
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
      if (s == claim_at) claim(u2, x2, bt2);
    }
    u = u2;
    x = x2;
    bt0 = bt2;
  }
  if (aborted && lane == 0) {
    // Drain: the last nstage stage issues and the last unit-slot posts may
    // still be in flight.
    int s = slot;
    uint32_t ph = phase;
    for (int k = 0; k < a.nstage; ++k) {
      if (--s < 0) {
        s = a.nstage - 1;
        ph ^= 1;
      }
      for (uint32_t i = 0; i < a.wait_limit; ++i)
        if (mbar_try_wait(&sm.full[s], ph)) break;
    }
    int k2 = uk;
    uint32_t uph = uphase;
    for (int k = 0; k < kUnitRing; ++k) {
      if (--k2 < 0) {
        k2 = kUnitRing - 1;
        uph ^= 1;
      }
      for (uint32_t i = 0; i < a.wait_limit; ++i)
        if (mbar_try_wait(&sm.ufull[k2], uph)) break;
    }
  }
}

// Consumer side of the unit ring: wait (per warp, bounded) for the next
// posted unit.  Returns false at the end marker or when the kernel must stop
// (a stuck wait anywhere raises misc[0]; every warp then leaves at its next
// wait, so no warp is ever left at a barrier).
__device__ __forceinline__ bool wait_unit(const DecodeArgs& a, const SmemPtrs& sm, int uk, uint32_t uphase,
                                          UnitSlot& out) {
  if (sm.misc[0] || !mbar_wait_bounded(&sm.ufull[uk], uphase, a.err, a.wait_limit)) {
    sm.misc[0] = 1;
    return false;
  }
  out = sm.slots[uk];
  return out.valid != 0;
}

__device__ __forceinline__ bool wait_or_abort(const DecodeArgs& a, const SmemPtrs& sm, uint64_t* bar,
                                              uint32_t parity) {
  if (sm.misc[0] || !mbar_wait_bounded(bar, parity, a.err, a.wait_limit)) {
    sm.misc[0] = 1;
    return false;
  }
  return true;
}

// Merge the NW consumer-warp states of one unit (scratch [NW][G][D + 2] =
// (acc[D], m, l), log2 domain), run by one warp.  A sequence in one chunk is
// finished here; otherwise the merged chunk state goes to the workspace
// partials [B*Hkv, max_chunks, group, D + 2] and the combine kernel finishes
// the sequence.
template <int D, int G, int NW>
__device__ void merge_unit(const DecodeArgs& a, const Unit& x, int nchunks, const float* scratch, int lane) {
  const int group = a.group;
  const int Hkv = a.num_kv_heads;
  const int Hq = Hkv * group;
  float* part_base = a.partials + (((size_t)x.b * Hkv + x.h) * a.max_chunks) * group * (D + 2);
  for (int idx = lane; idx < group * D; idx += 32) {
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
      float* P = part_base + ((size_t)x.c * group + g) * (D + 2);
      P[d] = O;
      if (d == 0) {
        P[D] = M;
        P[D + 1] = Ls;
      }
    }
  }
}

// Unit hand-off, run by every consumer warp after it wrote its state into
// scratch buffer sbuf: release the unit slot, count the warp in, and if it
// is the last of the NW warps, merge the unit and free the buffer.  No warp
// waits for another here.
template <int D, int G, int NW>
__device__ __forceinline__ void hand_off(const DecodeArgs& a, const SmemPtrs& sm, const UnitSlot& us, int sbuf,
                                         int uk, int lane) {
  __syncwarp();
  int last = 0;
  if (lane == 0) {
    __threadfence_block();
    last = atomicAdd(&sm.arrive[sbuf], 1) == NW - 1;
    mbar_arrive(&sm.uempty[uk]);  // this warp no longer reads the unit's slot
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) {
    __threadfence_block();
    merge_unit<D, G, NW>(a, us.x, us.nchunks, sm.scratch + sbuf * sm.scratch_floats, lane);
    __syncwarp();
    if (lane == 0) {
      sm.arrive[sbuf] = 0;
      mbar_arrive(&sm.scr_empty[sbuf]);
    }
  }
}

}  // namespace clove
