// Pieces shared by the decode kernels (CUDA-core and tensor-core consumers):
// the work partition, the TMA producer warp, and the epilogue that merges
// consumer-warp softmax states.
//
// Work partition (equal work per CTA).  The KV reads of a call form one
// stream of segments, one per (sequence b, KV head h) in b-major, h-minor
// order.  Segment (b, h) is alpha + nblk(b) positions long, nblk(b) =
// ceil(L_b / block_size) (no positions at all when nblk(b) = 0): alpha
// leading positions that carry no data and stand for the fixed cost of
// starting a piece (query load, state hand-off), then one position per
// block; W = num_kv_heads * sum_b (alpha + nblk(b)).  CTA c of P owns stream
// positions [c W / P, (c + 1) W / P): every CTA gets the same cost (+-1
// position) of blocks plus piece starts, so all finish together, whatever
// the mix of lengths.  Every CTA
// computes W and its start itself (partition_prologue: two block-wide scans
// of context_lens), so no planning launch precedes the decode.  A CTA walks
// its range as pieces: a piece is the part of one segment inside the range.
// A piece that is a whole segment writes its output rows directly; a segment
// split by a CTA boundary leaves one partial softmax state per piece, at most
// two per CTA (its first and its last piece), merged by the combine kernel.
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
  int u;         // trace id: 16 * cta + piece index within the CTA
  int b, h;
  int L;         // tokens the sequence attends over
  int blk0;      // first logical block of the piece
  int nblk;      // blocks in this piece
  int nstages;   // stages in this piece
  int complete;  // 1: the piece is its whole segment (output written directly)
  int slot;      // partial slot when split: 0 = the CTA's first piece, 1 = its last
  int last;      // 1: the piece holds the segment's last block (it performs the append)
};

// Units travel from the producer to the consumers through a small ring of
// shared-memory slots (kUnitRing deep): the unit's metadata plus a copy of
// its query rows, brought in by one bulk copy.  Consumers never touch global
// memory at a unit boundary.
constexpr int kUnitRing = 2;

struct UnitSlot {
  Unit x;
  int valid;  // 0: no more work
};

// Where a CTA's range starts (partition_prologue's result).
struct WalkStart {
  long long lo, hi;  // stream range [lo, hi)
  int b, h, off;     // segment (b, h) and position of lo within it (alpha leading positions
                     // included); b < 0: empty range
};

// Stream position bookkeeping shared with the combine kernel.
__host__ __device__ __forceinline__ long long range_begin(long long c, long long W, long long P) { return c * W / P; }
// The CTA whose range holds stream position x (0 <= x < W).
__host__ __device__ __forceinline__ long long cta_of(long long x, long long W, long long P) {
  return ((x + 1) * P + W - 1) / W - 1;
}

// Block-wide exclusive scan of one int per thread (all threads of the CTA
// take part, blockDim.x a multiple of 32, at most 1024); *total gets the sum.
__device__ __forceinline__ int block_excl_scan(int n, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = n;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) warp_tot[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const int excl = x - n + (warp > 0 ? warp_tot[warp - 1] : 0);
  *total = warp_tot[nw - 1];
  __syncthreads();
  return excl;
}

// Shared-memory carve-up: [ring: nstage x (K tiles | V tiles)] [barriers]
// [unit slots] [query buffers] [1 or 2 scratch buffers].  Every region starts 128-byte
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

// scratch_bytes: one merge scratch buffer (consumer warps x group rows x
// state_stride floats); nscr buffers of it.  q_bytes: one unit's query rows.
__host__ __device__ inline SmemPlan smem_plan(int block_size, int head_dim, int elem_bytes, int sb, int nstage,
                                             int scratch_bytes, int q_bytes, int nscr) {
  SmemPlan s;
  s.tile_stride = (block_size * head_dim * elem_bytes + 127) & ~127;
  s.stage_bytes = 2 * sb * s.tile_stride;
  s.ring_bytes = s.stage_bytes * nstage;
  s.bar_bytes = ((2 * nstage + 2 * kUnitRing + 2) * 8 + 64 + 127) & ~127;
  s.slot_bytes = (kUnitRing * (int)sizeof(UnitSlot) + 127) & ~127;
  s.q_stride = (q_bytes + 127) & ~127;
  s.scratch_bytes = (scratch_bytes + 127) & ~127;
  s.total = s.ring_bytes + s.bar_bytes + s.slot_bytes + kUnitRing * s.q_stride + nscr * s.scratch_bytes + 128;
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
  // Launched as a programmatic dependent of the previous kernel on the
  // stream: it may have started before that kernel finished, so wait for it
  // before reading any input (context lengths, tables, q, the cache).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The combine kernel that follows may be scheduled now; it waits for this
  // grid to finish before it reads anything.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// The equal-work partition, run by every thread of every decode CTA right
// after init_barriers.  Pass 1 sums nblk(b) over the batch (and zeroes the
// output rows of empty sequences, sequence b by CTA b % P; CTA 0 flags
// context lengths outside [0, max_ctx]); pass 2 finds the segment holding the
// CTA's first position.  CTA c records that segment in desc[c] for the
// combine; CTA 0 records W.  D: head_dim.
template <int D>
__device__ void partition_prologue(const DecodeArgs& a, WalkStart* out) {
  __shared__ int warp_tot[32];
  __shared__ long long s_sum;
  __shared__ int s_found;
  const int tid = threadIdx.x, lane = tid & 31;
  const int nt = blockDim.x;
  const int bs = a.block_size;
  const int H = a.num_kv_heads;
  const int row_floats = H * a.group * D;
  if (tid == 0) {
    s_sum = 0;
    s_found = 0;
  }
  __syncthreads();
  long long mine = 0;
  for (int b = tid; b < a.batch; b += nt) {
    const int raw = __ldg(a.context_lens + b);
    const int L = clamp_ctx(a.context_lens, b, a.max_ctx, a.append);
    if (blockIdx.x == 0 && raw != L - a.append) atomicOr(a.err, CLOVE_FLAG_CTX_RANGE);
    const int nb = (L + bs - 1) / bs;
    mine += nb > 0 ? nb + a.seg_cost : 0;
    if (L == 0 && b % a.num_ctas == (int)blockIdx.x) {
      float* row = a.out + (size_t)b * row_floats;
      if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
        for (int i = 0; i < row_floats / 4; ++i) reinterpret_cast<float4*>(row)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      } else {
        for (int i = 0; i < row_floats; ++i) row[i] = 0.f;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
  if (lane == 0 && mine) atomicAdd(reinterpret_cast<unsigned long long*>(&s_sum), (unsigned long long)mine);
  __syncthreads();
  const long long W = s_sum * H;
  const long long P = a.num_ctas;
  const long long lo = range_begin(blockIdx.x, W, P), hi = range_begin(blockIdx.x + 1, W, P);
  if (tid == 0) {
    out->lo = lo;
    out->hi = hi;
    out->b = -1;
    out->h = 0;
    out->off = 0;
    if (blockIdx.x == 0) *a.total = W;
  }
  if (lo < hi) {
    // pass 2: segment of position lo (sequence b spans [H pre_b, H pre_{b+1}))
    long long carry = 0;
    for (int base = 0; base < a.batch; base += nt) {
      const int b = base + tid;
      const int nb = b < a.batch ? (clamp_ctx(a.context_lens, b, a.max_ctx, a.append) + bs - 1) / bs : 0;
      const int len = nb > 0 ? nb + a.seg_cost : 0;  // stream positions of each of b's segments
      int tot;
      const int excl = block_excl_scan(len, warp_tot, &tot);
      const long long s0 = (carry + excl) * H;
      if (len > 0 && s0 <= lo && lo < s0 + (long long)len * H) {
        const long long r = lo - s0;
        out->b = b;
        out->h = (int)(r / len);
        out->off = (int)(r - (r / len) * len);
        s_found = 1;
      }
      carry += tot;
      __syncthreads();
      if (s_found) break;
    }
  }
  __syncthreads();
  if (tid == 0)
    a.desc[blockIdx.x] =
        out->b >= 0
            ? make_int4(out->b, out->h, out->off,
                        (clamp_ctx(a.context_lens, out->b, a.max_ctx, a.append) + bs - 1) / bs + a.seg_cost)
            : make_int4(-1, 0, 0, 0);
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

// The producer warp.  It walks the CTA's stream range (partition_prologue)
// piece by piece, posts each piece (metadata + a bulk copy of its query rows)
// to the unit ring, performs the fused append when the piece holds its
// segment's last block, then streams the piece's K/V tiles into the stage
// ring.  Halfway through a piece's stages (once the ring is primed) it works
// out the next piece and loads its first block-table entries, so a piece
// boundary costs no global round trip on the critical path.  Only lane 0
// issues copies.  On a stuck wait it raises the abort flag and drains its own
// in-flight copies (bounded) before returning.
//
// NBOX: 1 = one 3-D [block_size, head_dim] box per tile (dense rows); 2 =
// one 4-D box per tile written with the 128-byte swizzle as
// 128-byte rows (token, 64-dim half).
template <typename T, int D, int NBOX>
__device__ void produce(const DecodeArgs& a, const CUtensorMap* tm_k, const CUtensorMap* tm_v, const SmemPtrs& sm,
                        const SmemPlan& sp, int sb, const WalkStart& ws) {
  const int lane = threadIdx.x & 31;
  const int bs = a.block_size;
  const int H = a.num_kv_heads;
  const uint32_t tile_bytes = (uint32_t)(bs * D * (int)sizeof(T));
  const uint32_t q_bytes = (uint32_t)(a.group * D * (int)sizeof(T));
  const int Hq = H * a.group;
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

  // walk state: segment (b, h) of len = alpha + nb stream positions, the
  // position within it (off), the stream position (pos)
  const int alpha = a.seg_cost;
  int b = ws.b, h = ws.h, off = ws.off, npiece = 0;
  long long pos = ws.lo;
  int L = b >= 0 ? clamp_ctx(a.context_lens, b, a.max_ctx, a.append) : 0;
  int nb = (L + bs - 1) / bs;
  // The next piece of the walk (segment parts of the range that hold blocks),
  // then advance past it.
  auto next_piece = [&](Unit& x, int& bt0) -> bool {
    while (b >= 0 && pos < ws.hi) {
      const int len = nb + alpha;
      const int span = (int)min((long long)(len - off), ws.hi - pos);
      const int r0 = max(off, alpha), r1 = off + span;  // positions of this segment in the range
      const bool piece = r1 > r0;
      if (piece) {
        x.u = 16 * (int)blockIdx.x + min(npiece, 15);
        x.b = b;
        x.h = h;
        x.L = L;
        x.blk0 = r0 - alpha;
        x.nblk = r1 - r0;
        x.nstages = (x.nblk + sb - 1) / sb;
        x.complete = r0 == alpha && r1 == len;
        x.slot = npiece == 0 ? 0 : 1;
        x.last = r1 == len;
      }
      pos += span;
      off += span;
      if (off == len && pos < ws.hi) {  // next segment with work (empty sequences have none)
        off = 0;
        if (++h == H) {
          h = 0;
          do {
            if (++b >= a.batch) {  // (cannot happen while pos < hi; bounds the walk regardless)
              b = -1;
              break;
            }
            L = clamp_ctx(a.context_lens, b, a.max_ctx, a.append);
            nb = (L + bs - 1) / bs;
          } while (nb == 0);
        }
      }
      if (piece) {
        bt0 = table(x, 0);
        if constexpr (kTrace) {
          if (a.trace && lane == 0 && x.u < kTraceMaxUnit) {
            a.trace[kTraceUnit + 3 * x.u] = gtime();
            a.trace[kTraceUnit + 3 * x.u + 2] = ((unsigned long long)blockIdx.x << 32) | (unsigned)x.nblk;
          }
        }
        ++npiece;
        return true;
      }
    }
    return false;
  };

  int bt0 = 0;
  Unit x;
  bool have = next_piece(x, bt0);
  bool first = true;
  while (!aborted) {
    // ---- post the piece (or the end marker) to the unit ring ----
    int ok = 1;
    if (lane == 0) {
      if (*sm.misc || !mbar_wait_bounded(&sm.uempty[uk], uphase ^ 1, a.err, a.wait_limit)) {
        ok = 0;
        *sm.misc = 1;
      } else if (!have) {
        sm.slots[uk].valid = 0;
        mbar_arrive(&sm.ufull[uk]);
      } else {
        sm.slots[uk].x = x;
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
    if (!have) break;
    if (++uk == kUnitRing) {
      uk = 0;
      uphase ^= 1;
    }

    if (a.append && x.last) append_row<T, D>(a, x, lane);
    int my = bt0;
    int bt2 = 0;
    Unit x2;
    bool have2 = false;
    const int claim_at = min(x.nstages - 1, a.nstage / 2);
    for (int s = 0; s < x.nstages && !aborted; ++s) {
      const int j0 = s * sb;  // first block of this stage within the piece
      if ((j0 & 31) == 0 && j0 > 0) my = table(x, j0);
      const int nbs = min(sb, x.nblk - j0);
      int phys[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) phys[i] = __shfl_sync(0xffffffffu, my, (j0 + i) & 31);
      ok = 1;
      if (lane == 0) {
        if (*sm.misc || !mbar_wait_bounded(&sm.empty[slot], phase ^ 1, a.err, a.wait_limit)) {
          ok = 0;
          *sm.misc = 1;
        } else if (a.inject_stall && first && s == 0) {
          // test hook: the first stage of each CTA's first piece is never
          // filled, so its consumer's (bounded) wait runs out
        } else {
          mbar_arrive_expect_tx(&sm.full[slot], 2u * tile_bytes * (uint32_t)nbs);
          unsigned char* st = sm.ring + (size_t)slot * sp.stage_bytes;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (i < nbs) {
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
      if (s == claim_at) have2 = next_piece(x2, bt2);
    }
    have = have2;
    x = x2;
    bt0 = bt2;
    first = false;
  }
  if constexpr (kTrace) {
    if (a.trace && lane == 0 && blockIdx.x < kTraceMaxCta) a.trace[kTraceCta + 4 * blockIdx.x + 2] = gtime();
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

// Merge the NW consumer-warp states of one piece (scratch [NW][group][S] with
// S = state_stride(D): acc[D], m, l in the log2 domain), run by one warp.
// Lane (g, w) first works out warp w's weight for row g, f = 2^(m_w - M),
// and L = sum_w f l_w; the rows are then summed four dims per lane with
// 16-byte loads.  A complete segment is finished here (out = sum f acc / L);
// a split one leaves its merged state (sum f acc, M, L) in the CTA's partial
// slot [num_ctas, 2, group, S] for the combine kernel.
template <int D, int G, int NW>
__device__ void merge_unit(const DecodeArgs& a, const Unit& x, const float* scratch, int lane) {
  constexpr int S = state_stride(D);
  static_assert(G * NW <= 32, "one lane per (row, warp) state");
  const int group = a.group;
  const int Hq = a.num_kv_heads * group;
  const int lg = lane / NW, lw = lane - (lane / NW) * NW;
  float mw = -INFINITY, lsw = 0.f;
  if (lg < group) {
    mw = scratch[(lw * group + lg) * S + D];
    lsw = scratch[(lw * group + lg) * S + D + 1];
  }
  // row reductions over the NW lanes lg * NW .. lg * NW + NW - 1 (NW need
  // not be a power of two; lanes past G * NW compute unused values)
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < NW; ++w) M = fmaxf(M, __shfl_sync(0xffffffffu, mw, (lg * NW + w) & 31));
  const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
  const float fl = f * lsw;
  float Lr = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) Lr += __shfl_sync(0xffffffffu, fl, (lg * NW + w) & 31);
  float* part_base = a.partials + ((size_t)blockIdx.x * 2 + x.slot) * group * S;
  float* out_base = a.out + ((size_t)x.b * Hq + (size_t)x.h * group) * D;
  const bool out_vec = (reinterpret_cast<uintptr_t>(a.out) & 15) == 0;
  for (int g = 0; g < group; ++g) {
    float fw[NW];
#pragma unroll
    for (int w = 0; w < NW; ++w) fw[w] = __shfl_sync(0xffffffffu, f, g * NW + w);
    const float Lg = __shfl_sync(0xffffffffu, Lr, g * NW);
    const float Mg = __shfl_sync(0xffffffffu, M, g * NW);
    const float inv = 1.f / Lg;
    for (int d4 = lane; d4 < D / 4; d4 += 32) {
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float4 v = *reinterpret_cast<const float4*>(scratch + (w * group + g) * S + 4 * d4);
        o.x = fmaf(fw[w], v.x, o.x);
        o.y = fmaf(fw[w], v.y, o.y);
        o.z = fmaf(fw[w], v.z, o.z);
        o.w = fmaf(fw[w], v.w, o.w);
      }
      if (x.complete) {
        float* dst = out_base + (size_t)g * D + 4 * d4;
        const float4 r = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
        if (out_vec) {
          *reinterpret_cast<float4*>(dst) = r;
        } else {
          dst[0] = r.x;
          dst[1] = r.y;
          dst[2] = r.z;
          dst[3] = r.w;
        }
      } else {
        *reinterpret_cast<float4*>(part_base + (size_t)g * S + 4 * d4) = o;
      }
    }
    if (!x.complete && lane == 0) {
      part_base[(size_t)g * S + D] = Mg;
      part_base[(size_t)g * S + D + 1] = Lg;
    }
  }
}

// Unit hand-off, run by every consumer warp after it wrote its state into
// scratch buffer sbuf: release the unit slot, count the warp in, and if it
// is the last of the NW warps, merge the piece and free the buffer.  No warp
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
    merge_unit<D, G, NW>(a, us.x, sm.scratch + sbuf * sm.scratch_floats, lane);
    if constexpr (kTrace) {
      if (a.trace && lane == 0 && us.x.u < kTraceMaxUnit) a.trace[kTraceUnit + 3 * us.x.u + 1] = gtime();
    }
    __syncwarp();
    if (lane == 0) {
      sm.arrive[sbuf] = 0;
      mbar_arrive(&sm.scr_empty[sbuf]);
    }
  }
}

}  // namespace clove
