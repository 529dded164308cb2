// PagedAttention decode for sm_100a.
//
// Work decomposition (decode_common.cuh): the call's KV reads form one stream
// of (sequence, KV head) segments, each as many blocks long as its sequence;
// decode CTA c of P streams positions [c W / P, (c + 1) W / P), so every CTA
// reads the same number of K/V blocks.  A piece (the part of one segment in
// one CTA's range) is consumed for all query heads of the GQA group, so K/V
// are read from HBM exactly once.
//
// Two launches per call, chained with programmatic dependent launch:
//   decode kernel   persistent, P = SMs x resident CTAs.  Every CTA first
//                   computes the partition itself (two block-wide scans of
//                   context_lens), then one producer warp streams K/V tiles
//                   (one block of one head = a [block_size, head_dim] box)
//                   into a shared-memory ring with bulk tensor copies (TMA)
//                   and mbarriers, and consumer warps compute QK^T, an fp32
//                   online softmax and P.V.  Whole segments write their
//                   output rows; a segment split by a CTA boundary leaves a
//                   partial (m, l, acc) per piece.
//   combine kernel  merges the partials of split segments with a
//                   log-sum-exp combine, and publishes the call's check flags.
//
// With append (fused reshape-and-cache), the piece that holds a segment's
// last block writes the new token's K/V row of that head into its slot before
// it issues the tile copies (ordered with a proxy fence), so the tile it then
// reads already holds the new token.
//
// Semantics follow the reference's documented op: softmax(q.K^T * scale).V
// (src/nn/attention.rs:52-69), scale 1/sqrt(head_dim) supplied by the caller
// (src/lazy.rs:5267), block-table gather of src/lazy.rs:5259-5270.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "decode_common.cuh"
#include "host.h"
#include "mma_decode.cuh"

namespace clove {

// ---------------------------------------------------------------------------
// the CUDA-core decode kernel
// ---------------------------------------------------------------------------
// T: KV/Q element type.  D: head_dim.  G: max query heads per KV head
// (runtime a.group <= G).  NCW: consumer warps.
//
// A stage (TT = 16 or block_size tokens) is consumed by one warp; warps take
// a unit's stages round-robin and keep private (m, l, acc) softmax states,
// merged in the epilogue.  Inside a warp, per pass of P = min(TT, 32) tokens:
//   QK^T   lanes split the tokens: LPT = 32/P lanes per token, each lane
//          covering D/LPT dims of its token's K row, with q (pre-scaled,
//          f32) read from shared memory; an LPT-lane butterfly finishes the
//          dot product.  Each lane walks its 16-byte chunks starting at a
//          lane-dependent rotation so the 8 lanes of a shared-memory phase
//          hit distinct banks.
//   softmax the pass max is a warp max; the running max / correction are
//          warp-uniform; the row sum l is kept per lane and reduced once per
//          unit.
//   P.V    lanes split head_dim (E = D/32 dims each); for every token the
//          probability is broadcast with a shuffle and the V row is one
//          conflict-free warp-wide shared-memory read.
template <typename T, int D, int G, int NCW>
__global__ void __launch_bounds__((NCW + 1) * 32)
    paged_decode_simt_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                             const DecodeArgs a) {
  constexpr int E = D / 32;
  constexpr int EPC = 16 / (int)sizeof(T);  // elements per 16-byte chunk
  const int bs = a.block_size;
  const int sb = a.stage_blocks;
  const int TT = sb * bs;
  const int P = TT < 32 ? TT : 32;
  const int LPT = 32 / P;
  const int DL = D / LPT;
  const int CH = DL / EPC;
  const int group = a.group;

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const SmemPlan sp = smem_plan(bs, D, (int)sizeof(T), sb, a.nstage,
                                NCW * group * state_stride(D) * (int)sizeof(float), group * D * (int)sizeof(T),
                                a.nscr);
  const SmemPtrs sm = smem_ptrs(smem, sp, a.nstage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if constexpr (kTrace) {
    if (a.trace && threadIdx.x == 0 && blockIdx.x < kTraceMaxCta) a.trace[kTraceCta + 4 * blockIdx.x] = gtime();
  }
  init_barriers(sm, a.nstage, NCW);
  __shared__ WalkStart walk;
  partition_prologue<D>(a, &walk);
  if constexpr (kTrace) {
    if (a.trace && threadIdx.x == 0 && blockIdx.x < kTraceMaxCta) a.trace[kTraceCta + 4 * blockIdx.x + 1] = gtime();
  }

  if (warp == 0) {
    produce<T, D, 1>(a, &tm_k, &tm_v, sm, sp, sb, walk);
    return;
  }

  const int cw = warp - 1;
  const int tk_l = lane / LPT;    // token of this lane within a pass
  const int part = lane % LPT;    // which D/LPT slice of that token
  int gbase = 0;                  // stages of earlier units (CTA-wide count)
  int uk = 0, n_done = 0;
  uint32_t uphase = 0;
  UnitSlot us;

  while (wait_unit(a, sm, uk, uphase, us)) {
    const Unit x = us.x;
    const T* qs = reinterpret_cast<const T*>(sm.qbuf + uk * sp.q_stride);  // the unit's raw query rows

    float m[G], l[G], acc[G][E];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m[g] = -INFINITY;
      l[g] = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[g][e] = 0.f;
    }

    bool aborted = false;
    // Stage gs belongs to warp gs % ncw.  nstage is a multiple of ncw, so
    // ring slot gs % nstage is only ever consumed by that warp, which takes
    // its slots' fills in order: a parity wait can never alias an older,
    // still-incomplete fill of the same slot.
    const int ncw = a.ncw;
    for (int j = cw < ncw ? ((cw - gbase) % ncw + ncw) % ncw : x.nstages; j < x.nstages; j += ncw) {
      const int gs = gbase + j;
      const int slot = gs % a.nstage;
      const uint32_t par = (uint32_t)(gs / a.nstage) & 1u;
      if (sm.misc[0] || !mbar_wait_bounded(&sm.full[slot], par, a.err, a.wait_limit)) {
        sm.misc[0] = 1;
        aborted = true;
        break;
      }
      const T* Ks = reinterpret_cast<const T*>(sm.ring + (size_t)slot * sp.stage_bytes);
      const T* Vs = reinterpret_cast<const T*>(sm.ring + (size_t)slot * sp.stage_bytes + sb * sp.tile_stride);
      // tokens of this stage: up to the piece's end (a piece may end inside
      // a stage of sb blocks, before its sequence does) and the sequence's
      const int ntok = min(TT, min((x.blk0 + x.nblk) * bs, x.L) - (x.blk0 + j * sb) * bs);
      for (int p0 = 0; p0 < ntok; p0 += P) {
        const int tk = p0 + tk_l;
        // ---- scores ----
        float s[G];
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] = 0.f;
        const T* krow = Ks + (size_t)tk * D + part * DL;
        const T* qrow = qs + part * DL;
        for (int c = 0; c < CH; ++c) {
          const int cc = (c + lane) & (CH - 1);
          float kf[EPC];
          load_vec_f32<T, EPC>(krow + cc * EPC, kf);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            if (g < group) {
              float qf[EPC];
              load_vec_f32<T, EPC>(qrow + g * D + cc * EPC, qf);
#pragma unroll
              for (int e = 0; e < EPC; ++e) s[g] = fmaf(qf[e], kf[e], s[g]);
            }
          }
        }
        const bool valid = tk < ntok;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          for (int o = 1; o < LPT; o <<= 1) s[g] += __shfl_xor_sync(0xffffffffu, s[g], o);
          s[g] = valid ? s[g] * a.qscale : -INFINITY;
        }
        // ---- online softmax (warp-uniform max / correction) ----
        float pe[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float mp = s[g];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, o));
          const float mn = fmaxf(m[g], mp);
          const float corr = exp2f(m[g] - mn);
          m[g] = mn;
          l[g] *= corr;
#pragma unroll
          for (int e = 0; e < E; ++e) acc[g][e] *= corr;
          pe[g] = valid ? exp2f(s[g] - mn) : 0.f;
          if (part == 0) l[g] += pe[g];
        }
        // ---- P.V ----
        const int nt = min(P, ntok - p0);
        const T* vbase = Vs + (size_t)p0 * D + lane * E;
        for (int t = 0; t < nt; ++t) {
          float vf[E];
          load_vec_f32<T, E>(vbase + (size_t)t * D, vf);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float pt = __shfl_sync(0xffffffffu, pe[g], t * LPT);
#pragma unroll
            for (int e = 0; e < E; ++e) acc[g][e] = fmaf(pt, vf[e], acc[g][e]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[slot]);
    }
    if (aborted) return;  // the abort flag is up; every other warp leaves at its next wait
    gbase += x.nstages;

    // ---- publish this warp's state (rows < group) into scratch, hand off ----
    const int sbuf = n_done % a.nscr;
    if (!wait_or_abort(a, sm, &sm.scr_empty[sbuf], ((uint32_t)(n_done / a.nscr) & 1u) ^ 1u)) return;
    float* my_scr = sm.scratch + sbuf * sm.scratch_floats + (size_t)cw * group * state_stride(D);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (g >= group) break;  // the scratch holds `group` rows per warp
      const float lsum = warp_sum(l[g]);
#pragma unroll
      for (int e = 0; e < E; ++e) my_scr[g * state_stride(D) + lane * E + e] = acc[g][e];
      if (lane == 0) {
        my_scr[g * state_stride(D) + D] = m[g];
        my_scr[g * state_stride(D) + D + 1] = lsum;
      }
    }
    hand_off<D, G, NCW>(a, sm, us, sbuf, uk, lane);
    ++n_done;
    if (++uk == kUnitRing) {
      uk = 0;
      uphase ^= 1;
    }
  }
  if constexpr (kTrace) {
    if (a.trace && lane == 0 && blockIdx.x < kTraceMaxCta)
      atomicMax(a.trace + kTraceCta + 4 * blockIdx.x + 3, gtime());
  }
}

// ---------------------------------------------------------------------------
// combine
// ---------------------------------------------------------------------------
// Segments split by CTA boundaries: segment s is split iff some boundary
// range_begin(c), 0 < c < P, falls strictly inside it; its pieces are those
// of CTAs cta_of(S) .. cta_of(S + len - 1).  The CTA whose range starts at
// (or before) S keeps its piece in partial slot 1 (its last piece) unless its
// range starts exactly at S (slot 0); every later CTA keeps it in slot 0 (its
// first piece).  Combine CTAs stride over the boundaries c and merge the
// segment whose first interior boundary is c.
constexpr int kCombineThreads = 128;
constexpr int kCombineMaxPieces = 1024;  // >= P (decode CTAs) - checked on the host

// Pieces merged per pass (more are merged in passes, carrying a running state).
constexpr int kCombinePass = 256;

// Merge the np partial states listed in pieces[] (partial slot indices
// c * 2 + slot) of segment (b, h) and write outputs [o_begin, o_end) of its
// rows (output o = row o / (D/4), dims 4 (o % (D/4)) ..).  All threads of the
// CTA take part; per pass, every load of a phase is independent of the
// others, so a pass costs a few memory round trips whatever the piece count:
//   1. (m, l) of every (piece, row) into shared memory;
//   2. per row g: M = max_i m_i, w_i = 2^(m_i - M), L = sum_i w_i l_i;
//   3. each thread sums four dims of one row over all pieces (16-byte loads).
template <int D>
__device__ void combine_segment(const DecodeArgs& a, int b, int h, const int* pieces, int np, float* pm, float* pl,
                                float* run, float* rowv, int o_begin, int o_end) {
  constexpr int S = state_stride(D);
  constexpr int NW = kCombineThreads / 32;
  const int group = a.group;
  const int Hq = a.num_kv_heads * group;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* rowM = rowv;         // [8] reference max of the pass
  float* rowL = rowv + 8;     // [8] sum of weights times l (running)
  float* rowR = rowv + 16;    // [8] factor on the running state
  for (int base = 0; base < np; base += kCombinePass) {
    const int n = min(kCombinePass, np - base);
    const bool first = base == 0, last = base + n >= np;
    for (int i = tid; i < n * group; i += kCombineThreads) {
      const int p = i / group, g = i - p * group;
      const float* src = a.partials + ((size_t)pieces[base + p] * group + g) * S;
      pm[i] = __ldcg(src + D);
      pl[i] = __ldcg(src + D + 1);
    }
    __syncthreads();
    for (int g = warp; g < group; g += NW) {
      float M = first ? -INFINITY : rowM[g];
      for (int i = lane; i < n; i += 32) M = fmaxf(M, pm[i * group + g]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
      float ls = 0.f;
      for (int i = lane; i < n; i += 32) {
        const float mi = pm[i * group + g];
        const float wi = mi == -INFINITY ? 0.f : exp2f(mi - M);
        pm[i * group + g] = wi;  // the weight replaces m
        ls = fmaf(wi, pl[i * group + g], ls);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
      if (lane == 0) {
        const float r = first || rowM[g] == -INFINITY ? 0.f : exp2f(rowM[g] - M);
        rowR[g] = r;
        rowL[g] = (first ? 0.f : rowL[g] * r) + ls;
        rowM[g] = M;
      }
    }
    __syncthreads();
    // Output float4s [o_begin, o_end): kpar threads (lanes of one warp) per
    // output, each summing every kpar-th piece, then a shuffle reduction, so
    // a small slice over many pieces is not one long chain of loads.
    const int nout = o_end - o_begin;
    int kpar = 1;
    while (kpar < 32 && 2 * kpar * nout <= kCombineThreads) kpar *= 2;
    const int sub = tid & (kpar - 1);
    // every lane runs the same number of rounds (the shuffles below are
    // warp-wide); lanes past the slice carry zeros and store nothing
    for (int o0 = o_begin; o0 < o_end; o0 += kCombineThreads / kpar) {
      const int o = o0 + tid / kpar;
      const bool live = o < o_end;
      const int g = live ? o / (D / 4) : 0, d4 = live ? o - g * (D / 4) : 0;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      if (live && !first && sub == 0) {
        const float r = rowR[g];
        const float4 v = reinterpret_cast<const float4*>(run + g * S)[d4];
        acc = make_float4(v.x * r, v.y * r, v.z * r, v.w * r);
      }
#pragma unroll 4
      for (int i = sub; live && i < n; i += kpar) {
        const float w = pm[i * group + g];
        const float4 v = __ldcg(reinterpret_cast<const float4*>(a.partials + ((size_t)pieces[base + i] * group + g) * S) + d4);
        acc.x = fmaf(w, v.x, acc.x);
        acc.y = fmaf(w, v.y, acc.y);
        acc.z = fmaf(w, v.z, acc.z);
        acc.w = fmaf(w, v.w, acc.w);
      }
      for (int off = kpar / 2; off > 0; off >>= 1) {
        acc.x += __shfl_xor_sync(0xffffffffu, acc.x, off, kpar);
        acc.y += __shfl_xor_sync(0xffffffffu, acc.y, off, kpar);
        acc.z += __shfl_xor_sync(0xffffffffu, acc.z, off, kpar);
        acc.w += __shfl_xor_sync(0xffffffffu, acc.w, off, kpar);
      }
      if (!live || sub != 0) continue;
      if (last) {
        const float inv = 1.f / rowL[g];
        float* dst = a.out + ((size_t)b * Hq + (size_t)h * group + g) * D + 4 * d4;
        dst[0] = acc.x * inv;
        dst[1] = acc.y * inv;
        dst[2] = acc.z * inv;
        dst[3] = acc.w * inv;
      } else {
        reinterpret_cast<float4*>(run + g * S)[d4] = acc;
      }
    }
    __syncthreads();
  }
}

template <int D>
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const DecodeArgs a) {
  constexpr int S = state_stride(D);
  __shared__ float pm[kCombinePass * 8];
  __shared__ float pl[kCombinePass * 8];
  __shared__ __align__(16) float run[8 * S];  // running merged state between passes
  __shared__ float rowv[24];
  __shared__ int pieces[kCombineMaxPieces];
  __shared__ int s_np;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if constexpr (kTrace) {
    if (a.trace && threadIdx.x == 0) atomicMin(a.trace + 2, gtime());
  }
  // The decode grid has finished: publish this call's check flags and clear
  // the accumulating word for the next call (whose decode waits for this
  // grid before it raises anything).
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *a.err_last = *a.err;
    *a.err = 0;
  }
  const long long W = *a.total;
  const long long P = a.num_ctas;
  const int alpha = a.seg_cost;
  const int n_out = a.group * (D / 4);  // float4 outputs of a segment
  for (int c = 1 + blockIdx.x; c < P; c += gridDim.x) {
    const int4 d = a.desc[c];
    // empty range, or the boundary does not fall inside the segment's blocks
    if (d.x < 0 || d.z <= alpha) continue;
    // segment (d.x, d.y) starts at stream position S0 and is d.w positions
    // long; its pieces belong to CTAs c_first .. c_last
    const long long S0 = range_begin(c, W, P) - d.z;
    const long long c_first = cta_of(S0 + alpha, W, P);
    const long long c_last = cta_of(S0 + d.w - 1, W, P);
    int helper = 0, helpers = 1, np;
    if (W >= P) {
      // no empty ranges: every boundary inside the segment has a combine
      // CTA, and they share the segment's outputs
      helper = (int)(c - c_first - 1);
      helpers = (int)(c_last - c_first);
      np = (int)(c_last - c_first + 1);
      const int slot_first = range_begin(c_first, W, P) < S0 ? 1 : 0;
      for (int i = threadIdx.x; i < np && i < kCombineMaxPieces; i += kCombineThreads)
        pieces[i] = (int)((c_first + i) * 2 + (i == 0 ? slot_first : 0));
      np = min(np, kCombineMaxPieces);
    } else {
      // less work than CTAs (empty ranges hold no piece): the first boundary
      // inside merges alone
      if (cta_of(range_begin(c, W, P) - 1, W, P) != c_first) continue;
      if (threadIdx.x == 0) {
        int n = 0;
        for (long long k = c_first; k <= c_last && n < kCombineMaxPieces; ++k) {
          if (range_begin(k, W, P) == range_begin(k + 1, W, P)) continue;
          pieces[n++] = (int)(k * 2 + ((k == c_first && range_begin(k, W, P) < S0) ? 1 : 0));
        }
        s_np = n;
      }
      __syncthreads();
      np = s_np;
    }
    __syncthreads();
    const int o_begin = (int)((long long)helper * n_out / helpers);
    const int o_end = (int)((long long)(helper + 1) * n_out / helpers);
    combine_segment<D>(a, d.x, d.y, pieces, np, pm, pl, run, rowv, o_begin, o_end);
  }
  if constexpr (kTrace) {
    if (a.trace && threadIdx.x == 0) atomicMax(a.trace + 3, gtime());
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
constexpr int kNCW = 4;          // consumer warps of the CUDA-core kernel
constexpr int kRingTarget = 96 * 1024;

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Stream positions charged per segment for the fixed cost of starting a
// piece (query load, the consumer warps' state hand-off and merge): 40 KB
// worth of blocks (one position = the K and V [block_size, head_dim] tiles of
// one head).  Measured by sweeping it: the best steps came at 40-48 KB on
// c3 (8 KB blocks, alpha 5) and c5 (16 KB blocks, alpha 3).
// CLOVE_SEG_COST overrides it (for measurement sweeps).
static int segment_cost(const clove_pool& pool) {
  static const int env = [] {
    const char* v = std::getenv("CLOVE_SEG_COST");
    return v ? std::max(0, std::atoi(v)) : -1;
  }();
  if (env >= 0) return env;
  const int block_bytes = 2 * pool.block_size * pool.head_dim * pool.elem_bytes;
  return std::max(1, (40 * 1024 + block_bytes - 1) / block_bytes);
}

DecodeLayout decode_layout(const clove_pool& pool, int batch, int num_q_heads, int max_ctx) {
  (void)batch;
  (void)max_ctx;
  DecodeLayout L;
  const int group = num_q_heads / pool.num_kv_heads;
  L.max_ctas = pool.num_sms * kMaxCtasPerSm;
  size_t off = 0;
  L.off_err = off;  // [0] flags of this call, [1] flags of the last call, [4..5] W
  off += 256;
  L.off_desc = off;
  off = align256(off + sizeof(int4) * (size_t)L.max_ctas);
  L.off_partials = off;
  off = align256(off + sizeof(float) * (size_t)L.max_ctas * 2 * group * state_stride(pool.head_dim));
  L.total = off;
  return L;
}

// Launch configuration of one decode kernel instance for one pool shape,
// worked out once (function attributes and the occupancy query are not free
// on the host).
struct KernelCfg {
  int ok = 0;
  int nstage = 0, ncw = 0, smem = 0, ctas = 0;
};

template <typename T, int D, int G>
static KernelCfg simt_cfg(const clove_pool& pool, int group) {
  static std::mutex mu;
  static std::unordered_map<long long, KernelCfg> cache;
  const long long key = ((long long)pool.device << 32) | ((long long)pool.block_size << 8) | group;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  KernelCfg c;
  auto kern = paged_decode_simt_kernel<T, D, G, kNCW>;
  const int bs = pool.block_size;
  const int sb = bs >= 16 ? 1 : 16 / bs;
  const int scratch = kNCW * group * state_stride(D) * 4;
  const int qb = group * D * (int)sizeof(T);
  SmemPlan sp = smem_plan(bs, D, sizeof(T), sb, 1, scratch, qb, 2);
  // nstage: a multiple of the number of consumer warps that take stages (see
  // the kernel); large tiles use fewer of them.
  int ncw = kNCW;
  int nstage = (kRingTarget / sp.stage_bytes) / ncw * ncw;
  if (nstage < ncw) nstage = ncw;
  if (nstage > 4 * ncw) nstage = 4 * ncw;
  sp = smem_plan(bs, D, sizeof(T), sb, nstage, scratch, qb, 2);
  while (sp.total > 200 * 1024 && nstage > 1) {
    if (nstage > ncw) {
      nstage -= ncw;
    } else {
      ncw = --nstage;
    }
    sp = smem_plan(bs, D, sizeof(T), sb, nstage, scratch, qb, 2);
  }
  if (sp.total > 227 * 1024) {
    set_last_error("paged_decode: block_size %d x head_dim %d tile does not fit shared memory", bs, D);
    return c;  // not cached: the error text is set on every call
  }
  // The attribute belongs to the kernel, not to this block size: only raise
  // it, so configurations cached for other block sizes stay launchable.
  static int attr_smem = 0;
  if (sp.total > attr_smem) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sp.total) != cudaSuccess) {
      set_last_error("cudaFuncSetAttribute: %s", cudaGetErrorString(cudaGetLastError()));
      return c;
    }
    attr_smem = sp.total;
  }
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, (kNCW + 1) * 32, sp.total) != cudaSuccess ||
      occ < 1) {
    cudaGetLastError();
    occ = 1;
  }
  c.ok = 1;
  c.nstage = nstage;
  c.ncw = ncw;
  c.smem = sp.total;
  c.ctas = pool.num_sms * std::min(occ, kMaxCtasPerSm);
  cache[key] = c;
  return c;
}

template <typename T, int D, int G>
static int run_simt(const clove_pool& pool, DecodeArgs& a, cudaStream_t stream) {
  const KernelCfg c = simt_cfg<T, D, G>(pool, a.group);
  if (!c.ok) return CLOVE_ERR_UNSUPPORTED;
  const int bs = pool.block_size;
  a.stage_blocks = bs >= 16 ? 1 : 16 / bs;
  a.nscr = 2;
  a.nstage = c.nstage;
  a.ncw = c.ncw;
  a.num_ctas = c.ctas;
  cudaError_t e = launch_dependent(paged_decode_simt_kernel<T, D, G, kNCW>, (unsigned)c.ctas, (kNCW + 1) * 32,
                                   c.smem, stream, pool.tm_k, pool.tm_v, a);
  if (e != cudaSuccess) {
    set_last_error("paged_decode launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(1);
  return CLOVE_OK;
}

template <typename T, int D>
static int dispatch_group(const clove_pool& pool, DecodeArgs& a, cudaStream_t stream) {
  const int g = a.group;
  const int variant = decode_variant();
  if constexpr (!std::is_same<T, float>::value) {
    if constexpr (mma_supported<D>()) {
      const bool ok = g <= 8 && pool.has_swizzled && pool.block_size >= 8;
      if (ok && (variant == 2 || (variant == 0 && g >= 4))) return run_mma<T, D>(pool, a, stream);
    }
  }
  if (variant == 2) {
    set_last_error("paged_decode: tensor-core variant needs bf16/f16, head_dim 64/128, block_size >= 8, group <= 8 (group %d)", g);
    return CLOVE_ERR_UNSUPPORTED;
  }
  if (g == 1) return run_simt<T, D, 1>(pool, a, stream);
  if (g == 2) return run_simt<T, D, 2>(pool, a, stream);
  if (g <= 4) return run_simt<T, D, 4>(pool, a, stream);
  if (g <= 8) return run_simt<T, D, 8>(pool, a, stream);
  set_last_error("paged_decode: group size %d > 8 not built", g);
  return CLOVE_ERR_UNSUPPORTED;
}

template <typename T>
static int dispatch_dim(const clove_pool& pool, DecodeArgs& a, cudaStream_t stream) {
  switch (pool.head_dim) {
    case 64: return dispatch_group<T, 64>(pool, a, stream);
    case 128: return dispatch_group<T, 128>(pool, a, stream);
    case 256: return dispatch_group<T, 256>(pool, a, stream);
    default:
      set_last_error("paged_decode: head_dim %d not built (64, 128, 256)", pool.head_dim);
      return CLOVE_ERR_UNSUPPORTED;
  }
}

// Phase timing (measurement hook): CUDA events around the plan, decode and
// combine launches of the most recent call.  The events sit between the
// launches, so while timing is on the programmatic overlap of consecutive
// launches is lost; the phases are then serialised, as in a profiler's
// launch list.
static std::atomic<int> g_phase_timing{0};
static std::mutex g_phase_mu;
static cudaEvent_t g_phase_ev[4] = {nullptr, nullptr, nullptr, nullptr};
static int g_phase_dev = -1;
static bool g_phase_recorded = false;

static void phase_mark(int i, cudaStream_t stream) {
  if (!g_phase_timing.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lk(g_phase_mu);
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != g_phase_dev) {
    for (auto& e : g_phase_ev)
      if (e) {
        cudaEventDestroy(e);
        e = nullptr;
      }
    g_phase_dev = dev;
  }
  if (!g_phase_ev[i] && cudaEventCreate(&g_phase_ev[i]) != cudaSuccess) return;
  cudaEventRecord(g_phase_ev[i], stream);
  if (i == 3) g_phase_recorded = true;
}

void set_phase_timing(int on) { g_phase_timing.store(on ? 1 : 0); }

static std::atomic<unsigned long long*> g_trace{nullptr};
void set_trace_buffer(void* buf) { g_trace.store(static_cast<unsigned long long*>(buf)); }
unsigned long long* trace_buffer() { return g_trace.load(); }

int read_phase_ms(float* plan_ms, float* decode_ms, float* combine_ms) {
  std::lock_guard<std::mutex> lk(g_phase_mu);
  if (!g_phase_recorded) {
    set_last_error("debug_phase_ms: no decode was timed (enable with clove_cuda_debug_phase_timing)");
    return CLOVE_ERR_INVALID_ARG;
  }
  cudaError_t e = cudaEventSynchronize(g_phase_ev[3]);
  float t[3] = {0.f, 0.f, 0.f};
  for (int i = 0; i < 3 && e == cudaSuccess; ++i) e = cudaEventElapsedTime(&t[i], g_phase_ev[i], g_phase_ev[i + 1]);
  if (e != cudaSuccess) {
    set_last_error("debug_phase_ms: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  if (plan_ms) *plan_ms = t[0];
  if (decode_ms) *decode_ms = t[1];
  if (combine_ms) *combine_ms = t[2];
  return CLOVE_OK;
}

int launch_decode(const clove_pool& pool, const DecodeCall& call, cudaStream_t stream) {
  const DecodeLayout L = decode_layout(pool, call.batch, call.num_q_heads, call.max_ctx);
  if (call.workspace_bytes < L.total) {
    set_last_error("paged_decode: workspace %zu bytes < required %zu", call.workspace_bytes, L.total);
    return CLOVE_ERR_WORKSPACE;
  }
  unsigned char* ws = static_cast<unsigned char*>(call.workspace);
  const int append = call.k_new != nullptr ? 1 : 0;

  DecodeArgs a;
  a.q = call.q;
  a.k_new = call.k_new;
  a.v_new = call.v_new;
  a.k_cache = pool.k_cache;
  a.v_cache = pool.v_cache;
  a.block_tables = call.block_tables;
  a.context_lens = call.context_lens;
  a.out = call.out;
  a.partials = reinterpret_cast<float*>(ws + L.off_partials);
  a.desc = reinterpret_cast<int4*>(ws + L.off_desc);
  a.err = reinterpret_cast<int32_t*>(ws + L.off_err);
  a.err_last = a.err + 1;
  a.total = reinterpret_cast<long long*>(ws + L.off_err + 16);
  a.bt_stride = call.bt_stride;
  a.batch = call.batch;
  a.num_kv_heads = pool.num_kv_heads;
  a.num_blocks = pool.num_blocks;
  a.block_size = pool.block_size;
  a.num_ctas = 1;
  a.seg_cost = segment_cost(pool);
  a.max_ctx = call.max_ctx;
  a.group = call.num_q_heads / pool.num_kv_heads;
  a.append = append;
  a.nstage = 2;
  a.ncw = 1;
  a.stage_blocks = 1;
  a.nscr = 2;
  a.wait_limit = debug_wait_limit();
  a.inject_stall = debug_inject_stall();
  a.qscale = call.scale * kLog2e;
  a.trace = kTrace ? g_trace.load() : nullptr;

  phase_mark(0, stream);
  phase_mark(1, stream);  // no planning launch: the plan phase is empty
  int rc;
  switch (pool.dtype) {
    case CLOVE_DTYPE_F32: rc = dispatch_dim<float>(pool, a, stream); break;
    case CLOVE_DTYPE_BF16: rc = dispatch_dim<__nv_bfloat16>(pool, a, stream); break;
    case CLOVE_DTYPE_F16: rc = dispatch_dim<__half>(pool, a, stream); break;
    default:
      set_last_error("paged_decode: dtype %d", pool.dtype);
      return CLOVE_ERR_UNSUPPORTED;
  }
  if (rc != CLOVE_OK) return rc;
  if (a.num_ctas > L.max_ctas || a.num_ctas > kCombineMaxPieces) {
    // cannot happen with the occupancy cap; guards the workspace bound
    set_last_error("paged_decode: %d CTAs exceed the workspace bound %d", a.num_ctas, L.max_ctas);
    return CLOVE_ERR_UNSUPPORTED;
  }
  phase_mark(2, stream);
  // Combine (always: it also publishes the call's check flags).
  {
    cudaLaunchConfig_t cfg = {};
    // one CTA per boundary between decode CTAs; most find no segment to merge
    cfg.gridDim = dim3((unsigned)std::max(1, std::min(a.num_ctas - 1, kCombineMaxPieces)));
    cfg.blockDim = dim3(kCombineThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    switch (pool.head_dim) {
      case 64: e = cudaLaunchKernelEx(&cfg, combine_kernel<64>, a); break;
      case 128: e = cudaLaunchKernelEx(&cfg, combine_kernel<128>, a); break;
      default: e = cudaLaunchKernelEx(&cfg, combine_kernel<256>, a); break;
    }
    if (e != cudaSuccess) {
      set_last_error("combine launch: %s", cudaGetErrorString(e));
      return CLOVE_ERR_CUDA;
    }
    count_launches(1);
  }
  phase_mark(3, stream);
  return CLOVE_OK;
}

}  // namespace clove
