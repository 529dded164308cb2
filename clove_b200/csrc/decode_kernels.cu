// PagedAttention decode for sm_100a.
//
// Work decomposition.  A work unit is (sequence b, context chunk c, KV head
// h): `chunk_blocks` consecutive logical blocks of one sequence, for all the
// query heads that share KV head h (the GQA group).  K/V of a unit are read
// from HBM exactly once; every query head of the group consumes them from
// shared memory.
//
// Two launches per call:
//   plan_kernel     1 CTA: per-sequence chunk counts, a compact list of
//                   (b, c) items, counter reset, zero rows for empty
//                   sequences, context-length checks.
//   decode kernel   persistent: gridDim = SMs x resident CTAs, each CTA walks
//                   units u = blockIdx.x + k*gridDim.x.  One producer warp
//                   streams K/V tiles (one block of one head = a
//                   [block_size, head_dim] box) into a shared-memory ring with
//                   3-D bulk tensor copies (TMA) and mbarriers; consumer warps
//                   compute QK^T, an fp32 online softmax and P.V.  A sequence
//                   split into several chunks writes per-chunk partials
//                   (m, l, acc); the CTA that finishes the last chunk of
//                   (b, h) — detected with an atomic counter, no waiting —
//                   merges them with a log-sum-exp combine and writes the
//                   output.  No inter-CTA spin-waits exist.
//
// With append (fused reshape-and-cache), the CTA that owns the last chunk of
// (b, h) writes the new token's K/V row of head h into its slot before it
// issues the tile copies of that chunk (ordered with a proxy fence), so the
// tile it then reads already holds the new token.
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
// plan
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;

constexpr int kPlanBins = 256;

// Block-wide exclusive scan of one int per thread; *total gets the sum.
__device__ __forceinline__ int block_excl_scan(int n, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = n;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_tot[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const int excl = x - n + (warp > 0 ? warp_tot[warp - 1] : 0);
  *total = warp_tot[31];
  __syncthreads();
  return excl;
}

// Work list, longest first: every sequence of nbl blocks yields nbl / cb
// full chunks (listed first, all the same size) and, if nbl % cb != 0, one
// partial chunk; the partial chunks follow in descending size order (counting
// sort over kPlanBins size bins).  The decode kernel's CTAs claim units from
// the front with an atomic counter, so the big units start first and the
// small ones fill the tail.
__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const PlanArgs p) {
  __shared__ int warp_tot[32];
  __shared__ int hist[kPlanBins];
  __shared__ int binbase[kPlanBins];
  __shared__ long long s_blocks;
  __shared__ int s_full;
  const int tid = threadIdx.x, lane = tid & 31;
  // Let the decode kernel launch now: it sets up its barriers and then waits
  // (griddepcontrol.wait) for this grid's results.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // Context lengths of this thread's first sequence stay in registers; only
  // batches beyond kPlanThreads sequences re-read the rest.
  const int b0 = tid;
  const int L0 = b0 < p.batch ? clamp_ctx(p.context_lens, b0, p.max_ctx, p.append) : 0;
  if (tid == 0) {
    s_blocks = 0;
    s_full = 0;
    *p.err = 0;            // flags report the most recent call only
    *p.unit_counter = 0;   // the decode kernel's work-claim counter
    *p.n_multi = 0;
  }
  for (int i = tid; i < kPlanBins; i += kPlanThreads) hist[i] = 0;
  __syncthreads();
  auto len_of = [&](int b) { return b == b0 ? L0 : clamp_ctx(p.context_lens, b, p.max_ctx, p.append); };
  // Chunk size from the actual work: total (block, KV head) pairs spread
  // over ~target_units work items, capped at max_chunk_blocks, never below
  // min_chunk_blocks.
  {
    long long mine = 0;
    for (int b = tid; b < p.batch; b += kPlanThreads) mine += (len_of(b) + p.block_size - 1) / p.block_size;
    for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
    if (lane == 0 && mine) atomicAdd(reinterpret_cast<unsigned long long*>(&s_blocks), (unsigned long long)mine);
  }
  __syncthreads();
  const long long want = (s_blocks * p.num_kv_heads + p.target_units - 1) / p.target_units;
  const int cb = (int)max((long long)p.min_chunk_blocks, min((long long)p.max_chunk_blocks, want));
  if (tid == 0) *p.chunk_blocks = cb;

  // pass 1: per-sequence bookkeeping, full chunks, partial-size histogram
  for (int base = 0; base < p.batch; base += kPlanThreads) {
    const int b = base + tid;
    int nfull = 0;
    if (b < p.batch) {
      const int raw = __ldg(p.context_lens + b);
      const int L = len_of(b);
      if (raw != L - p.append) atomicOr(p.err, CLOVE_FLAG_CTX_RANGE);
      const int nbl = (L + p.block_size - 1) / p.block_size;
      nfull = nbl / cb;
      const int rem = nbl - nfull * cb;
      p.seq_chunks[b] = nfull + (rem > 0);
      if (nfull + (rem > 0) > 1) p.multi[atomicAdd(p.n_multi, 1)] = b;
      if (rem > 0) atomicAdd(&hist[(rem - 1) * kPlanBins / cb], 1);
      if (L == 0) {
        float* row = p.out + (size_t)b * p.row_floats;
        for (int i = 0; i < p.row_floats; ++i) row[i] = 0.f;
      }
    }
    int tot;
    const int excl = block_excl_scan(nfull, warp_tot, &tot);
    for (int c = 0; c < nfull; ++c) p.items[s_full + excl + c] = make_int2(b, c);
    __syncthreads();
    if (tid == 0) s_full += tot;
    __syncthreads();
  }
  // partial chunks: bases per size bin, largest bin first (parallel scan over
  // the bins in descending order)
  {
    const int bin = kPlanBins - 1 - tid;
    const int cnt = tid < kPlanBins ? hist[bin] : 0;
    int tot;
    const int excl = block_excl_scan(cnt, warp_tot, &tot);
    if (tid < kPlanBins) {
      binbase[bin] = s_full + excl;
      hist[bin] = 0;  // reused as the per-bin cursor
    }
    if (tid == 0) *p.n_items = s_full + tot;
  }
  __syncthreads();
  for (int b = tid; b < p.batch; b += kPlanThreads) {
    const int L = len_of(b);
    const int nbl = (L + p.block_size - 1) / p.block_size;
    const int nfull = nbl / cb;
    const int rem = nbl - nfull * cb;
    if (rem > 0) {
      const int bin = (rem - 1) * kPlanBins / cb;
      p.items[binbase[bin] + atomicAdd(&hist[bin], 1)] = make_int2(b, nfull);
    }
  }
}

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
  constexpr int NCT = NCW * 32;
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
                                NCW * G * (D + 2) * (int)sizeof(float), G * D * (int)sizeof(T));
  const SmemPtrs sm = smem_ptrs(smem, sp, a.nstage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  init_barriers(sm, a.nstage, NCW);
  const int n_units = *a.n_items * a.num_kv_heads;

  if (warp == 0) {
    produce<T, D, 1>(a, &tm_k, &tm_v, sm, sp, sb, n_units);
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
      const int ntok = min(TT, x.L - (x.blk0 + j * sb) * bs);
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

    // ---- publish this warp's state (double-buffered scratch), hand off ----
    const int sbuf = n_done & 1;
    if (!wait_or_abort(a, sm, &sm.scr_empty[sbuf], ((uint32_t)(n_done >> 1) & 1u) ^ 1u)) return;
    float* my_scr = sm.scratch + sbuf * sm.scratch_floats + (size_t)cw * G * (D + 2);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float lsum = warp_sum(l[g]);
#pragma unroll
      for (int e = 0; e < E; ++e) my_scr[g * (D + 2) + lane * E + e] = acc[g][e];
      if (lane == 0) {
        my_scr[g * (D + 2) + D] = m[g];
        my_scr[g * (D + 2) + D + 1] = lsum;
      }
    }
    hand_off<D, G, NCW>(a, sm, us, sbuf, uk, lane);
    ++n_done;
    if (++uk == kUnitRing) {
      uk = 0;
      uphase ^= 1;
    }
  }
}

// ---------------------------------------------------------------------------
// split-K combine
// ---------------------------------------------------------------------------
// One CTA per (sequence, query head): for a sequence the decode split into
// several chunks, merge the chunk states (m, l, acc) of the partials with a
// log-sum-exp combine and write the output row.  Sequences in one chunk were
// finished by the decode kernel; their CTAs exit at once.  Launched as a
// programmatic dependent of the decode kernel.
constexpr int kCombineThreads = 128;
constexpr int kCombineMaxChunks = 2048;  // chunk weights staged in shared memory

// Merge the chunks of (sequence b, query head hq): M = max m_c,
// w_c = 2^(m_c - M), out = sum_c w_c acc_c / sum_c w_c l_c.  All threads of
// the CTA take part; ends with a CTA barrier so the shared arrays can be
// reused.
__device__ void combine_one(const DecodeArgs& a, int D, int b, int hq, float* w, float* red, float* bcast) {
  const int group = a.group;
  const int Hq = a.num_kv_heads * group;
  const int h = hq / group, g = hq - h * group;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t cstride = (size_t)group * (D + 2);  // floats between consecutive chunks
  const float* base = a.partials + (((size_t)b * a.num_kv_heads + h) * a.max_chunks * group + g) * (D + 2);
  const int nc = min(a.seq_chunks[b], kCombineMaxChunks);  // decode_layout keeps it within bounds
  float mx = -INFINITY;
  for (int c = tid; c < nc; c += kCombineThreads) mx = fmaxf(mx, base[c * cstride + D]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  if (tid == 0) {
    float m = red[0];
    for (int i = 1; i < kCombineThreads / 32; ++i) m = fmaxf(m, red[i]);
    *bcast = m;
  }
  __syncthreads();
  const float M = *bcast;
  float ls = 0.f;
  for (int c = tid; c < nc; c += kCombineThreads) {
    const float wc = exp2f(base[c * cstride + D] - M);
    w[c] = wc;
    ls = fmaf(wc, base[c * cstride + D + 1], ls);
  }
  for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
  __syncthreads();
  if (lane == 0) red[warp] = ls;
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    for (int i = 0; i < kCombineThreads / 32; ++i) t += red[i];
    *bcast = 1.f / t;
  }
  __syncthreads();
  const float inv = *bcast;
  // loads coalesced over d, independent over c
  for (int d = tid; d < D; d += kCombineThreads) {
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
    int c = 0;
    for (; c + 4 <= nc; c += 4) {
      o0 = fmaf(w[c], base[c * cstride + d], o0);
      o1 = fmaf(w[c + 1], base[(c + 1) * cstride + d], o1);
      o2 = fmaf(w[c + 2], base[(c + 2) * cstride + d], o2);
      o3 = fmaf(w[c + 3], base[(c + 3) * cstride + d], o3);
    }
    for (; c < nc; ++c) o0 = fmaf(w[c], base[c * cstride + d], o0);
    a.out[((size_t)b * Hq + hq) * D + d] = ((o0 + o1) + (o2 + o3)) * inv;
  }
  __syncthreads();
}

// Split-K combine: CTAs stride over the (sequence, query head) pairs of the
// sequences the plan split into several chunks (the others were finished by
// the decode kernel).  Launched as a programmatic dependent of the decode.
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const DecodeArgs a, int head_dim) {
  __shared__ float w[kCombineMaxChunks];
  __shared__ float red[kCombineThreads / 32];
  __shared__ float bcast;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int Hq = a.num_kv_heads * a.group;
  const int n_items = *a.n_multi * Hq;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x)
    combine_one(a, head_dim, a.multi[item / Hq], item - (item / Hq) * Hq, w, red, &bcast);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
constexpr int kNCW = 4;          // consumer warps of the CUDA-core kernel
constexpr int kRingTarget = 96 * 1024;

// Smallest work item: 256 tokens (a chunk shorter than that spends more on
// its epilogue than on streaming).  The plan kernel picks the actual chunk
// size per call from the total work; this bound sizes the workspace.
static int min_chunk_blocks(int block_size) { return (256 + block_size - 1) / block_size; }

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

DecodeLayout decode_layout(const clove_pool& pool, int batch, int num_q_heads, int max_ctx) {
  DecodeLayout L;
  const int hkv = pool.num_kv_heads;
  const int group = num_q_heads / hkv;
  const int max_blocks = (max_ctx + pool.block_size - 1) / pool.block_size;
  // Smallest chunk: 256 tokens, and few enough chunks per sequence for the
  // combine kernel's shared-memory weights.
  L.chunk_blocks = max(min_chunk_blocks(pool.block_size), (max_blocks + kCombineMaxChunks - 1) / kCombineMaxChunks);
  L.max_chunks = max_blocks <= 0 ? 1 : (max_blocks + L.chunk_blocks - 1) / L.chunk_blocks;
  size_t off = 0;
  L.off_err = off;
  off += 256;
  L.off_nitems = off;
  off += 256;
  L.off_items = off;
  off = align256(off + sizeof(int2) * (size_t)batch * L.max_chunks);
  L.off_seq_chunks = off;
  off = align256(off + sizeof(int32_t) * (size_t)batch);
  L.off_multi = off;
  off = align256(off + sizeof(int32_t) * (size_t)batch);
  L.off_partials = off;
  // Partials are only written when a sequence spans more than one chunk.
  if (L.max_chunks > 1)
    off = align256(off + sizeof(float) * (size_t)batch * hkv * L.max_chunks * group * (pool.head_dim + 2));
  L.total = off;
  return L;
}

template <typename T, int D, int G>
static int run_simt(const clove_pool& pool, DecodeArgs& a, cudaStream_t stream) {
  auto kern = paged_decode_simt_kernel<T, D, G, kNCW>;
  const int bs = pool.block_size;
  const int sb = bs >= 16 ? 1 : 16 / bs;
  a.stage_blocks = sb;
  const int scratch = kNCW * G * (D + 2) * 4;
  const int qb = G * D * (int)sizeof(T);
  SmemPlan sp = smem_plan(bs, D, sizeof(T), sb, 1, scratch, qb);
  // nstage: a multiple of the number of consumer warps that take stages (see
  // the kernel); large tiles use fewer of them.
  int ncw = kNCW;
  int nstage = (kRingTarget / sp.stage_bytes) / ncw * ncw;
  if (nstage < ncw) nstage = ncw;
  if (nstage > 4 * ncw) nstage = 4 * ncw;
  sp = smem_plan(bs, D, sizeof(T), sb, nstage, scratch, qb);
  while (sp.total > 200 * 1024 && nstage > 1) {
    if (nstage > ncw) {
      nstage -= ncw;
    } else {
      ncw = --nstage;
    }
    sp = smem_plan(bs, D, sizeof(T), sb, nstage, scratch, qb);
  }
  a.ncw = ncw;
  if (sp.total > 227 * 1024) {
    set_last_error("paged_decode: block_size %d x head_dim %d tile does not fit shared memory", bs, D);
    return CLOVE_ERR_UNSUPPORTED;
  }
  a.nstage = nstage;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sp.total);
  if (e != cudaSuccess) {
    set_last_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  int occ = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, (kNCW + 1) * 32, sp.total);
  if (e != cudaSuccess || occ < 1) occ = 1;
  long long units_max = (long long)a.batch * a.max_chunks * a.num_kv_heads;
  long long grid = (long long)pool.num_sms * occ;
  if (grid > units_max) grid = units_max;
  if (grid < 1) grid = 1;
  e = launch_dependent(kern, (unsigned)grid, (kNCW + 1) * 32, sp.total, stream, pool.tm_k, pool.tm_v, a);
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

  PlanArgs p;
  p.context_lens = call.context_lens;
  p.items = reinterpret_cast<int2*>(ws + L.off_items);
  p.n_items = reinterpret_cast<int32_t*>(ws + L.off_nitems);
  p.seq_chunks = reinterpret_cast<int32_t*>(ws + L.off_seq_chunks);
  p.out = call.out;
  p.err = reinterpret_cast<int32_t*>(ws + L.off_err);
  p.batch = call.batch;
  p.num_kv_heads = pool.num_kv_heads;
  p.row_floats = call.num_q_heads * pool.head_dim;
  p.block_size = pool.block_size;
  p.min_chunk_blocks = L.chunk_blocks;
  // ~2 units per resident CTA, and no unit above ~2 MiB of K/V, so the tail
  // (the last units still streaming) stays short (measured on c2-c5).
  p.target_units = (long long)pool.num_sms * 4;
  p.max_chunk_blocks = (int)((2u << 20) / (2u * pool.block_size * pool.head_dim * pool.elem_bytes));
  p.chunk_blocks = reinterpret_cast<int32_t*>(ws + L.off_nitems) + 1;
  p.unit_counter = reinterpret_cast<int32_t*>(ws + L.off_nitems) + 2;
  p.n_multi = reinterpret_cast<int32_t*>(ws + L.off_nitems) + 3;
  p.multi = reinterpret_cast<int32_t*>(ws + L.off_multi);
  p.max_ctx = call.max_ctx;
  p.append = append;
  phase_mark(0, stream);
  plan_kernel<<<1, kPlanThreads, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("plan launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(1);
  phase_mark(1, stream);

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
  a.items = p.items;
  a.n_items = p.n_items;
  a.seq_chunks = p.seq_chunks;
  a.err = p.err;
  a.bt_stride = call.bt_stride;
  a.batch = call.batch;
  a.num_kv_heads = pool.num_kv_heads;
  a.num_blocks = pool.num_blocks;
  a.block_size = pool.block_size;
  a.chunk_blocks = p.chunk_blocks;
  a.unit_counter = p.unit_counter;
  a.multi = p.multi;
  a.n_multi = p.n_multi;
  a.max_chunks = L.max_chunks;
  a.max_ctx = call.max_ctx;
  a.group = call.num_q_heads / pool.num_kv_heads;
  a.append = append;
  a.nstage = 2;
  a.ncw = 1;
  a.wait_limit = debug_wait_limit();
  a.inject_stall = debug_inject_stall();
  a.qscale = call.scale * kLog2e;

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
  phase_mark(2, stream);
  if (L.max_chunks <= 1) {
    phase_mark(3, stream);
    return rc;
  }
  // Split-K combine for the sequences the plan split into several chunks.
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min<long long>((long long)call.batch * call.num_q_heads,
                                                     (long long)pool.num_sms * 8));
    cfg.blockDim = dim3(kCombineThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, combine_kernel, a, pool.head_dim);
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
