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
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "host.h"
#include "mma_decode.cuh"

namespace clove {

__device__ __forceinline__ int clamp_ctx(const int32_t* ctx_lens, int b, int max_ctx, int append) {
  int c = __ldg(ctx_lens + b);
  c = max(0, min(c, max_ctx - append));
  return c + append;
}

// ---------------------------------------------------------------------------
// plan
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const PlanArgs p) {
  __shared__ int warp_tot[32];
  __shared__ int s_base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    s_base = 0;
    *p.err = 0;  // flags report the most recent call only
  }
  __syncthreads();
  for (int base = 0; base < p.batch; base += kPlanThreads) {
    const int b = base + tid;
    int n = 0;
    if (b < p.batch) {
      int raw = p.context_lens[b];
      int L = clamp_ctx(p.context_lens, b, p.max_ctx, p.append);
      if (raw != L - p.append) atomicOr(p.err, CLOVE_FLAG_CTX_RANGE);
      n = (L + p.chunk_tokens - 1) / p.chunk_tokens;
      p.seq_chunks[b] = n;
      for (int h = 0; h < p.num_kv_heads; ++h) p.counters[(size_t)b * p.num_kv_heads + h] = 0;
      if (L == 0) {
        float* row = p.out + (size_t)b * p.row_floats;
        for (int i = 0; i < p.row_floats; ++i) row[i] = 0.f;
      }
    }
    // block-wide exclusive scan of n
    int x = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = warp_tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_tot[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    int excl = x - n + (warp > 0 ? warp_tot[warp - 1] : 0);
    int off = s_base + excl;
    for (int c = 0; c < n; ++c) p.items[off + c] = make_int2(b, c);
    __syncthreads();
    if (tid == 0) s_base += warp_tot[31];
    __syncthreads();
  }
  if (tid == 0) *p.n_items = s_base;
}

// ---------------------------------------------------------------------------
// shared-memory carve-up of the decode kernels
// ---------------------------------------------------------------------------
struct SmemPlan {
  int tile_stride;  // bytes of one [block_size, head_dim] tile, 128-aligned
  int ring_bytes;   // nstage * 2 tiles
  int bar_bytes;    // 2 * nstage mbarriers + misc ints
  int scratch_bytes;
  int total;        // + 128 alignment slack
};

__host__ __device__ inline SmemPlan smem_plan(int block_size, int head_dim, int elem_bytes, int nstage,
                                             int scratch_bytes) {
  SmemPlan s;
  s.tile_stride = (block_size * head_dim * elem_bytes + 127) & ~127;
  s.ring_bytes = 2 * s.tile_stride * nstage;
  s.bar_bytes = ((2 * nstage * 8 + 64) + 127) & ~127;
  s.scratch_bytes = (scratch_bytes + 127) & ~127;
  s.total = s.ring_bytes + s.bar_bytes + s.scratch_bytes + 128;
  return s;
}

// ---------------------------------------------------------------------------
// the CUDA-core decode kernel
// ---------------------------------------------------------------------------
// T: KV/Q element type.  D: head_dim.  G: max query heads per KV head
// (runtime a.group <= G).  NCW: consumer warps.  Each consumer warp owns
// every NCW-th token of a tile, keeps a private (m, l, acc) state per query
// head, and the warps are merged at the end of the unit.  Within a warp the
// head_dim is split across lanes (E = D/32 elements each), so a score is a
// lane-partial dot product plus a 5-step butterfly sum.
template <typename T, int D, int G, int NCW>
__global__ void __launch_bounds__((NCW + 1) * 32)
    paged_decode_simt_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                             const DecodeArgs a) {
  constexpr int E = D / 32;
  constexpr int TPW = 8;  // tokens per warp per sub-round
  constexpr int NCT = NCW * 32;
  const int bs = a.block_size;
  const int Hkv = a.num_kv_heads;
  const int group = a.group;
  const int Hq = Hkv * group;
  const int tile_bytes = bs * D * (int)sizeof(T);

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const SmemPlan sp = smem_plan(bs, D, (int)sizeof(T), a.nstage, NCW * G * (D + 2) * 4);
  unsigned char* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + sp.ring_bytes);
  uint64_t* empty = full + a.nstage;
  volatile int* s_misc = reinterpret_cast<volatile int*>(empty + a.nstage);  // [0] abort, [1] last flag
  float* scratch = reinterpret_cast<float*>(smem + sp.ring_bytes + sp.bar_bytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.nstage; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    s_misc[0] = 0;
    s_misc[1] = 0;
    fence_barrier_init();
  }
  __syncthreads();

  const int n_units = *a.n_items * Hkv;

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    const uint64_t pol = policy_evict_first();
    int stage = 0;
    uint32_t phase = 0;
    bool aborted = false;
    for (int u = blockIdx.x; u < n_units && !aborted; u += gridDim.x) {
      const int2 it = a.items[u / Hkv];
      const int h = u - (u / Hkv) * Hkv;
      const int b = it.x, c = it.y;
      const int L = clamp_ctx(a.context_lens, b, a.max_ctx, a.append);
      const int blk0 = c * a.chunk_blocks;
      const int nblk = min(a.chunk_blocks, (L + bs - 1) / bs - blk0);
      const int32_t* bt = a.block_tables + (size_t)b * a.bt_stride;
      if (a.append && c == a.seq_chunks[b] - 1) {
        // fused reshape-and-cache of the new token, head h
        const int pos = L - 1;
        int phys = __ldg(bt + pos / bs);
        if (phys < 0 || phys >= a.num_blocks) {
          if (lane == 0) atomicOr(a.err, CLOVE_FLAG_BLOCK_OOB);
        } else {
          const size_t row = (((size_t)phys * bs + (pos % bs)) * Hkv + h) * D;
          const size_t src = ((size_t)b * Hkv + h) * D;
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
      for (int j0 = 0; j0 < nblk && !aborted; j0 += 32) {
        int my = 0;
        if (j0 + lane < nblk) {
          my = __ldg(bt + blk0 + j0 + lane);
          if (my < 0 || my >= a.num_blocks) {
            atomicOr(a.err, CLOVE_FLAG_BLOCK_OOB);
            my = 0;
          }
        }
        const int cnt = min(32, nblk - j0);
        for (int jj = 0; jj < cnt; ++jj) {
          const int phys = __shfl_sync(0xffffffffu, my, jj);
          int ok = 1;
          if (lane == 0) {
            if (s_misc[0] || !mbar_wait_bounded(&empty[stage], phase ^ 1, a.err)) {
              ok = 0;
              s_misc[0] = 1;
            } else {
              mbar_arrive_expect_tx(&full[stage], 2 * tile_bytes);
              unsigned char* kt = ring + (size_t)stage * 2 * sp.tile_stride;
              tma_load_3d(kt, &tm_k, &full[stage], 0, h, phys * bs, pol);
              tma_load_3d(kt + sp.tile_stride, &tm_v, &full[stage], 0, h, phys * bs, pol);
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) {
            aborted = true;
            break;
          }
          if (++stage == a.nstage) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    if (aborted && lane == 0) {
      // Drain: wait (bounded) for the copies of the last nstage issues to
      // land before the CTA's shared memory goes away.  Walk back from the
      // next (stage, phase) slot; issues before those have been waited on by
      // the consumers already.
      int s = stage;
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
    return;
  }

  // ------------------------------ consumers -------------------------------
  const int cw = warp - 1;
  const int ct = threadIdx.x - 32;
  int stage = 0;
  uint32_t phase = 0;
  float* my_scr = scratch + (size_t)cw * G * (D + 2);

  for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
    const int2 it = a.items[u / Hkv];
    const int h = u - (u / Hkv) * Hkv;
    const int b = it.x, c = it.y;
    const int L = clamp_ctx(a.context_lens, b, a.max_ctx, a.append);
    const int blk0 = c * a.chunk_blocks;
    const int nblk = min(a.chunk_blocks, (L + bs - 1) / bs - blk0);
    const int nchunks = a.seq_chunks[b];

    float qr[G][E];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (g < group) {
        const T* qp = static_cast<const T*>(a.q) + ((size_t)b * Hq + (size_t)h * group + g) * D + lane * E;
        load_vec_f32<T, E>(qp, qr[g]);
#pragma unroll
        for (int e = 0; e < E; ++e) qr[g][e] *= a.qscale;
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) qr[g][e] = 0.f;
      }
    }
    float m[G], l[G], acc[G][E];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m[g] = -INFINITY;
      l[g] = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[g][e] = 0.f;
    }

    bool aborted = false;
    for (int j = 0; j < nblk; ++j) {
      if (s_misc[0] || !mbar_wait_bounded(&full[stage], phase, a.err)) {
        s_misc[0] = 1;
        aborted = true;
        break;
      }
      const T* kt = reinterpret_cast<const T*>(ring + (size_t)stage * 2 * sp.tile_stride);
      const T* vt = reinterpret_cast<const T*>(ring + (size_t)stage * 2 * sp.tile_stride + sp.tile_stride);
      const int ntok = min(bs, L - (blk0 + j) * bs);
      for (int t0 = 0; t0 < ntok; t0 += NCW * TPW) {
        float sc[TPW][G];
        float mloc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) mloc[g] = -INFINITY;
#pragma unroll
        for (int i = 0; i < TPW; ++i) {
          const int t = t0 + cw + i * NCW;
          if (t < ntok) {
            float kv[E];
            load_vec_f32<T, E>(kt + t * D + lane * E, kv);
#pragma unroll
            for (int g = 0; g < G; ++g) {
              float part = 0.f;
#pragma unroll
              for (int e = 0; e < E; ++e) part = fmaf(qr[g][e], kv[e], part);
              sc[i][g] = warp_sum(part);
              mloc[g] = fmaxf(mloc[g], sc[i][g]);
            }
          } else {
#pragma unroll
            for (int g = 0; g < G; ++g) sc[i][g] = -INFINITY;
          }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float mn = fmaxf(m[g], mloc[g]);
          if (mn != -INFINITY) {
            const float corr = exp2f(m[g] - mn);  // m = -inf -> 0
            l[g] *= corr;
#pragma unroll
            for (int e = 0; e < E; ++e) acc[g][e] *= corr;
            m[g] = mn;
          }
        }
#pragma unroll
        for (int i = 0; i < TPW; ++i) {
          const int t = t0 + cw + i * NCW;
          if (t < ntok) {
            float vv[E];
            load_vec_f32<T, E>(vt + t * D + lane * E, vv);
#pragma unroll
            for (int g = 0; g < G; ++g) {
              const float p = exp2f(sc[i][g] - m[g]);
              l[g] += p;
#pragma unroll
              for (int e = 0; e < E; ++e) acc[g][e] = fmaf(p, vv[e], acc[g][e]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == a.nstage) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (aborted) return;

    // ---- merge the NCW warp states ----
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int e = 0; e < E; ++e) my_scr[g * (D + 2) + lane * E + e] = acc[g][e];
      if (lane == 0) {
        my_scr[g * (D + 2) + D] = m[g];
        my_scr[g * (D + 2) + D + 1] = l[g];
      }
    }
    named_bar_sync(1, NCT);
    float* part_base = a.partials + (((size_t)b * Hkv + h) * a.max_chunks) * G * (D + 2);
    for (int idx = ct; idx < group * D; idx += NCT) {
      const int g = idx / D, d = idx - (idx / D) * D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < NCW; ++w) M = fmaxf(M, scratch[(w * G + g) * (D + 2) + D]);
      float Ls = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < NCW; ++w) {
        const float mw = scratch[(w * G + g) * (D + 2) + D];
        if (mw != -INFINITY) {
          const float f = exp2f(mw - M);
          Ls = fmaf(scratch[(w * G + g) * (D + 2) + D + 1], f, Ls);
          O = fmaf(scratch[(w * G + g) * (D + 2) + d], f, O);
        }
      }
      if (nchunks == 1) {
        a.out[((size_t)b * Hq + (size_t)h * group + g) * D + d] = O / Ls;
      } else {
        float* P = part_base + ((size_t)c * G + g) * (D + 2);
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
        const int prev = atomicAdd(a.counters + (size_t)b * Hkv + h, 1);
        s_misc[1] = (prev == nchunks - 1);
      }
      named_bar_sync(1, NCT);
      if (s_misc[1]) {
        __threadfence();
        for (int idx = ct; idx < group * D; idx += NCT) {
          const int g = idx / D, d = idx - (idx / D) * D;
          float M = -INFINITY;
          for (int cc = 0; cc < nchunks; ++cc) M = fmaxf(M, __ldcg(part_base + ((size_t)cc * G + g) * (D + 2) + D));
          float Ls = 0.f, O = 0.f;
          for (int cc = 0; cc < nchunks; ++cc) {
            const float* P = part_base + ((size_t)cc * G + g) * (D + 2);
            const float f = exp2f(__ldcg(P + D) - M);
            Ls = fmaf(__ldcg(P + D + 1), f, Ls);
            O = fmaf(__ldcg(P + d), f, O);
          }
          a.out[((size_t)b * Hq + (size_t)h * group + g) * D + d] = O / Ls;
        }
        if (ct == 0) a.counters[(size_t)b * Hkv + h] = 0;
      }
    }
    named_bar_sync(1, NCT);  // scratch and s_misc[1] are reused by the next unit
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
constexpr int kNCW = 4;          // consumer warps of the CUDA-core kernel
constexpr int kRingTarget = 96 * 1024;

static int chunk_blocks_for(int batch, int hkv, int max_ctx, int block_size, int sms) {
  const int max_blocks = (max_ctx + block_size - 1) / block_size;
  if (max_blocks <= 0) return 1;
  const long long units1 = (long long)batch * hkv;
  const long long target = (long long)sms * 8;  // ~4 waves of 2 resident CTAs per SM
  if (units1 >= target) return max_blocks;
  long long nchunks = (target + units1 - 1) / units1;
  int cb = (int)((max_blocks + nchunks - 1) / nchunks);
  const int min_blocks = (256 + block_size - 1) / block_size;  // >= 256 tokens per chunk
  if (cb < min_blocks) cb = min_blocks;
  if (cb > max_blocks) cb = max_blocks;
  return cb;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

DecodeLayout decode_layout(const clove_pool& pool, int batch, int num_q_heads, int max_ctx) {
  DecodeLayout L;
  const int hkv = pool.num_kv_heads;
  const int group = num_q_heads / hkv;
  L.chunk_blocks = chunk_blocks_for(batch, hkv, max_ctx, pool.block_size, pool.num_sms);
  const int max_blocks = (max_ctx + pool.block_size - 1) / pool.block_size;
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
  L.off_counters = off;
  off = align256(off + sizeof(int32_t) * (size_t)batch * hkv);
  L.off_partials = off;
  // Partials are only written when a sequence spans more than one chunk.
  const size_t gpad = group <= 1 ? 1 : group <= 2 ? 2 : group <= 4 ? 4 : group <= 8 ? 8 : 16;
  if (L.max_chunks > 1) off = align256(off + sizeof(float) * (size_t)batch * hkv * L.max_chunks * gpad * (pool.head_dim + 2));
  L.total = off;
  return L;
}

template <typename T, int D, int G>
static int run_simt(const clove_pool& pool, DecodeArgs& a, cudaStream_t stream) {
  auto kern = paged_decode_simt_kernel<T, D, G, kNCW>;
  const int scratch = kNCW * G * (D + 2) * 4;
  const int tile = (pool.block_size * D * (int)sizeof(T) + 127) & ~127;
  int nstage = kRingTarget / (2 * tile);
  if (nstage < 2) nstage = 2;
  if (nstage > 16) nstage = 16;
  SmemPlan sp = smem_plan(pool.block_size, D, sizeof(T), nstage, scratch);
  while (sp.total > 200 * 1024 && nstage > 2) {
    --nstage;
    sp = smem_plan(pool.block_size, D, sizeof(T), nstage, scratch);
  }
  if (sp.total > 227 * 1024) {
    set_last_error("paged_decode: block_size %d x head_dim %d tile does not fit shared memory", pool.block_size, D);
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
  kern<<<(unsigned)grid, (kNCW + 1) * 32, sp.total, stream>>>(pool.tm_k, pool.tm_v, a);
  e = cudaGetLastError();
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
    if ((variant == 2 || (variant == 0 && g >= 4)) && g <= 8 && mma_supported<D>()) {
      return run_mma<T, D>(pool, a, stream);
    }
  }
  if (variant == 2) {
    set_last_error("paged_decode: tensor-core variant needs bf16/f16 and 4 <= group <= 8 (group %d)", g);
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
  p.counters = reinterpret_cast<int32_t*>(ws + L.off_counters);
  p.out = call.out;
  p.err = reinterpret_cast<int32_t*>(ws + L.off_err);
  p.batch = call.batch;
  p.num_kv_heads = pool.num_kv_heads;
  p.row_floats = call.num_q_heads * pool.head_dim;
  p.chunk_tokens = L.chunk_blocks * pool.block_size;
  p.max_ctx = call.max_ctx;
  p.append = append;
  plan_kernel<<<1, kPlanThreads, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("plan launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(1);

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
  a.counters = p.counters;
  a.items = p.items;
  a.n_items = p.n_items;
  a.seq_chunks = p.seq_chunks;
  a.err = p.err;
  a.bt_stride = call.bt_stride;
  a.batch = call.batch;
  a.num_kv_heads = pool.num_kv_heads;
  a.num_blocks = pool.num_blocks;
  a.block_size = pool.block_size;
  a.chunk_blocks = L.chunk_blocks;
  a.max_chunks = L.max_chunks;
  a.max_ctx = call.max_ctx;
  a.group = call.num_q_heads / pool.num_kv_heads;
  a.append = append;
  a.nstage = 2;
  a.qscale = call.scale * kLog2e;

  switch (pool.dtype) {
    case CLOVE_DTYPE_F32: return dispatch_dim<float>(pool, a, stream);
    case CLOVE_DTYPE_BF16: return dispatch_dim<__nv_bfloat16>(pool, a, stream);
    case CLOVE_DTYPE_F16: return dispatch_dim<__half>(pool, a, stream);
    default:
      set_last_error("paged_decode: dtype %d", pool.dtype);
      return CLOVE_ERR_UNSUPPORTED;
  }
}

}  // namespace clove
