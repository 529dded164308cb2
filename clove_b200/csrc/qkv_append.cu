// Fused Q/K/V projection + KV append for one decode step, on the 5th-generation
// tensor cores (tcgen05, accumulator in tensor memory).
//
// The reference computes q = x Wq + bq, k = x Wk + bk, v = x Wv + bv with its
// Linear layer (src/nn.rs:102-123, called from PagedAttention::forward at
// src/nn.rs:538-540) and then hands k, v to the paged-attention op, which
// must write them into the cache slot of each sequence's new token.  Here one
// kernel does both: the GEMM epilogue adds the bias, optionally rotates q and
// k (RoPE, the pairing of src/lazy.rs:4834-4842), writes q for the decode
// and stores k, v straight into their cache slots, so K/V never make a round
// trip through global memory.
//
// Shape of the work.  At decode the batch is small and the weights W
// [hidden, (Hq + 2 Hkv) D] are large: the kernel streams the weights once,
// so HBM bandwidth bounds it.  Every tcgen05.mma costs about the same issue
// time whatever its shape, so the weights ride in the MMA's N operand: a
// tile is 256 output features (N = 256, 8 KB of weights per K = 16 step)
// against up to 128 batch rows (M = 128; x rows past the batch tile only
// feed accumulator rows that are never stored).  With the weights in M (4 KB
// per instruction) the tensor pipe, not HBM, set the streaming rate.  The
// accumulator holds batch row b in tensor-memory lane b and feature f in
// column f, so an epilogue thread writes 16 consecutive features (32 bytes)
// of a q row or cache slot at a time.
//
// Weight layout.  W^T is packed once (clove_cuda_qkv_pack_weights) into
// 128-feature x 64-element chunks, each a contiguous 16 KB block already in
// the 128-byte-swizzled K-major order the tensor cores read; a stage takes
// two of them (the tile's two halves at one K block) with plain bulk copies.
// x, small and L2-resident, comes through a 2-D tensor map with the same
// swizzle.
//
// Two schedules:
//  - cluster (qkv_cluster_n_kernel), the usual one: grid (feature tiles) x
//    (K splits) x (128-row batch tiles), the K splits of a tile forming one
//    thread-block cluster sized so that every cluster is resident and the
//    CTAs cover the SMs.  After the main loops the split-K partial sums meet
//    in distributed shared memory, each CTA of the cluster adding and
//    storing its slice of the batch rows.
//  - stream-K (qkv_stream_kernel), for batches up to 32 rows when the
//    clusters would leave over 40 % of the SMs idle: (feature tile) x
//    (64-wide K block) units split evenly and contiguously over one CTA per
//    SM.  A CTA's range covers pieces ("segments") of one or more tiles; a
//    whole-tile segment goes straight to the epilogue, otherwise its f32
//    partial goes to a workspace slot and the CTA that completes the tile's
//    last piece (a per-tile arrival counter, reset by that CTA) sums the
//    slots in order and runs the epilogue.
// Both are programmatic dependents of the previous kernel on the stream: the
// barrier set-up, tensor-memory allocation and the first ring of weight
// copies run before griddepcontrol.wait.  The epilogue adds the bias,
// rotates (RoPE), rounds and stores q and the K/V slot rows.  Every wait is
// bounded; a wait that runs out sets CLOVE_FLAG_TIMEOUT in the pool's flag
// word and the CTA finishes without hanging.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <type_traits>

#include "../../include/clove_cuda.h"
#include "common.cuh"
#include "host.h"
#include "tc_common.cuh"

namespace clove {

namespace {

constexpr int kQkvThreads = 192;      // stream-K: warp 0 copies, warp 1 MMAs, warps 2-5 epilogue
constexpr int kEpiThreads = 128;
constexpr int kClusterThreads = 256;  // cluster schedule: warp 0 copies, warp 1 MMAs, all 8 in the epilogue
constexpr int kStreamMaxBatch = 32;   // stream-K only up to this batch (its partials grow with the batch)
constexpr int kStreamM = 128;         // batch rows per tile (MMA M)
constexpr int kStreamN = 256;         // output features per tile (MMA N: two packed 128-feature chunks)
constexpr int kMaxHeadDim = 256;
constexpr int kTileN = 128;           // features per packed weight chunk
constexpr int kTileK = 64;            // hidden elements per stage (one 128-byte swizzle row)
constexpr size_t kSmemBudget = 224 * 1024;  // stage ring + padding

struct QkvArgs {
  const void* w_packed;         // [ntiles_n][kb_total][128][64] pre-swizzled
  const float* bias;            // [N] or null
  const int32_t* block_tables;  // [M, bt_stride]
  const int32_t* context_lens;  // [M] tokens cached before this one
  int32_t* lens_out;            // [M] context_lens + 1, or null
  void* q_out;                  // [M, Hq, D]
  void* k_cache;
  void* v_cache;
  int32_t* flags;
  float* partials;              // stream-K: [tiles][max_contrib][16 chunks][4][batch_tile] float4
  int32_t* counters;            // [tiles], zero between calls
  int M, hidden, hq, hkv, D, bs, bt_stride, num_blocks;
  int n_out;        // (hq + 2 hkv) * D
  int kb_total;     // K blocks per tile
  int ntiles_n;     // packed 128-feature chunks
  int batch_tile;   // batch rows per tile, a multiple of 16 (cluster schedule: the MMA N)
  int nstage;
  int max_contrib;  // partial slots per tile
  int splits;       // cluster schedule: K splits (cluster size)
  long long units;  // stream-K: 256-feature tiles * kb_total
  float rope_theta;
  uint32_t wait_limit;
  int inject_stall;  // test hook: the first stage of the first CTA is never filled
  unsigned long long* trace;  // timeline buffer (trace builds only; null otherwise)
};

// Instruction descriptor, kind::f16: f32 accumulate (bits 4-5 = 1), A and B
// both bf16 (1) or both f16 (0) at bits 7-9 / 10-12, both K-major, N >> 3 at
// bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ inline uint32_t qkv_idesc(bool bf16, int m, int n) {
  const uint32_t f = bf16 ? 1u : 0u;
  return (1u << 4) | (f << 7) | (f << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of `p` (this CTA's shared memory) in the shared window of cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_peer(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}

__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float x, float y, float z, float w) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(x), "f"(y), "f"(z), "f"(w)
               : "memory");
}

template <typename T>
__device__ __forceinline__ T to_elem(float x);
template <> __device__ __forceinline__ __nv_bfloat16 to_elem<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half to_elem<__half>(float x) { return __float2half_rn(x); }

// First CTA whose unit range [g*U/G, (g+1)*U/G) contains unit x.
__device__ __forceinline__ int first_cta(long long x, long long units, int grid) {
  return (int)(((x + 1) * grid - 1) / units);
}

// Piece of a tile inside one CTA's unit range.
struct Segment {
  int tile, kb0, kb1;
};

__device__ __forceinline__ Segment segment_at(long long u, long long u_end, int kb_total) {
  Segment s;
  s.tile = (int)(u / kb_total);
  s.kb0 = (int)(u - (long long)s.tile * kb_total);
  s.kb1 = (int)min((long long)kb_total, (long long)s.kb0 + (u_end - u));
  return s;
}

// Epilogue state of the kernels that carry the weights in N: RoPE factors,
// the current tile's bias, and each batch row's position and cache slot.
struct RowState {
  float inv_freq[kMaxHeadDim / 2];  // RoPE: theta^(-2i/D)
  float bias[kStreamN];             // the current 256-feature tile's bias
  int pos[kStreamM];                // context length of each batch row
  int slot[kStreamM];               // its cache slot (-1: none)
};

// Threads tid = 0, stride, 2 stride .. fill the RoPE factors and the
// positions and slots of batch rows m0 .. m0 + batch_tile - 1 (rs index r =
// row - m0); `report` (one CTA per batch tile) also flags bad positions /
// blocks and writes the new lengths.  Reads context lengths and
// tables: call after griddepcontrol.wait.
__device__ __forceinline__ void init_rows(const QkvArgs& a, RowState& rs, int m0, int tid, int stride, bool report) {
  if (a.rope_theta > 0.f)
    for (int i = tid; i < a.D / 2; i += stride) rs.inv_freq[i] = powf(a.rope_theta, -2.f * (float)i / (float)a.D);
  for (int r = tid; r < a.batch_tile; r += stride) {
    const int b = m0 + r;
    int slot = -1, pos = 0;
    if (b < a.M) {
      pos = __ldg(a.context_lens + b);
      if (pos >= 0 && pos / a.bs < a.bt_stride) {
        const int phys = __ldg(a.block_tables + (size_t)b * a.bt_stride + pos / a.bs);
        if (phys >= 0 && phys < a.num_blocks) slot = phys * a.bs + pos % a.bs;
        else if (report) atomicOr(a.flags, CLOVE_FLAG_BLOCK_OOB);
      } else if (report) {
        atomicOr(a.flags, CLOVE_FLAG_CTX_RANGE);
      }
      if (report && a.lens_out) a.lens_out[b] = pos + 1;
    }
    rs.pos[r] = pos;
    rs.slot[r] = slot;
  }
}

// Bias, RoPE, round and store features [f0, f0 + 16) of batch row m0 + r
// (n0: the tile's first feature, whose bias rs.bias holds).  The q | k | v
// boundaries are multiples of 64 features, so a chunk never straddles one.
template <typename T>
__device__ __forceinline__ void emit_chunk(const QkvArgs& a, const RowState& rs, int m0, int r, int f0, int n0,
                                           float (&v)[16]) {
  const int qd = a.hq * a.D, kd = a.hkv * a.D;
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] += rs.bias[f0 - n0 + i];
  if (a.rope_theta > 0.f && f0 < qd + kd) {
    const int d0 = f0 % a.D;
    const float pos = (float)rs.pos[r];
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      float sn, cs;
      sincosf(pos * rs.inv_freq[(d0 + i) >> 1], &sn, &cs);
      const float x0 = v[i], x1 = v[i + 1];
      v[i] = x0 * cs - x1 * sn;
      v[i + 1] = x1 * cs + x0 * sn;
    }
  }
  T* dst;
  if (f0 < qd) {
    dst = static_cast<T*>(a.q_out) + (size_t)(m0 + r) * qd + f0;
  } else {
    const int slot = rs.slot[r];
    if (slot < 0) return;
    const bool is_k = f0 < qd + kd;
    dst = static_cast<T*>(is_k ? a.k_cache : a.v_cache) + (size_t)slot * kd + (f0 - (is_k ? qd : qd + kd));
  }
  uint4 out[2];
  T* o = reinterpret_cast<T*>(out);
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i] = to_elem<T>(v[i]);
  __stcs(reinterpret_cast<uint4*>(dst), out[0]);
  __stcs(reinterpret_cast<uint4*>(dst) + 1, out[1]);
}

// Load the bias of features [n0, n0 + 256) into rs.bias (zeros past ncols).
__device__ __forceinline__ void load_tile_bias(const QkvArgs& a, RowState& rs, int n0, int ncols, int tid, int stride) {
  for (int i = tid; i < kStreamN; i += stride) rs.bias[i] = (a.bias && i < ncols) ? __ldg(a.bias + n0 + i) : 0.f;
}

// Stream-K schedule for batches up to 128 (qkv_stream_kernel).  The weights
// are the MMA's B operand: a tile is 256 output features (two packed
// 128-feature chunks at the same K block, side by side in shared memory, so
// one tcgen05.mma of N = 256, K = 16 consumes 8 KB of weights) against the
// batch as M = 128 rows (x rows beyond the batch tile are never stored).
// Every tcgen05.mma costs about the same issue time whatever its N, so
// carrying the weights in N rather than M halves the instructions per
// weight byte; with the weights in M (4 KB per instruction) the tensor pipe,
// not HBM, set the streaming rate.
//
// The accumulator holds row b of the batch in tensor-memory lane b and
// feature f in column f, so an epilogue thread owns one sequence and writes
// 16 consecutive features (32 bytes) of its q row or cache slot per chunk.
template <typename T>
__global__ void __launch_bounds__(kQkvThreads, 1)
    qkv_stream_kernel(const __grid_constant__ CUtensorMap tm_x, const QkvArgs a) {
  __shared__ __align__(8) uint64_t full_bar[16];
  __shared__ __align__(8) uint64_t empty_bar[16];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ uint32_t tmem_base_slot;
  __shared__ int last_flag;
  __shared__ RowState rs;
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte aligned (the swizzle atom), by offsetting the shared array
  // itself so the compiler keeps the shared address space
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BT = a.batch_tile;                        // x rows copied per stage (16..128)
  constexpr uint32_t w_half = kTileN * 128;           // one packed 128-feature chunk: 16 KB
  const uint32_t x_bytes = (uint32_t)BT * 128;
  const uint32_t stage_bytes = 2 * w_half + x_bytes;  // weights [256][64], then x [BT][64]
  const int G = gridDim.x;
  const long long u_begin = (long long)blockIdx.x * a.units / G;
  const long long u_end = (long long)(blockIdx.x + 1) * a.units / G;
  if constexpr (kTrace) {
    if (a.trace && threadIdx.x == 0 && blockIdx.x < kTraceMaxCta) a.trace[kTraceCta + 8 * blockIdx.x] = gtime();
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.nstage; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiThreads);
    }
    fence_barrier_init();
  }
  __syncwarp();
  if (warp == 0) {
    // two accumulators of 256 columns: a segment drains while the next accumulates
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_slot)),
                 "r"(2 * kStreamN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_slot;
  // the next kernel on the stream may be scheduled now (it waits for this
  // grid before reading anything)
  griddep_launch_dependents();

  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  if (warp == 0) {
    if (lane == 0) {
      // producer.  Stage i holds unit u_begin + i: tile u / kb_total, K
      // block u % kb_total.  The packed weights are never written by the
      // kernel this one may overlap (clove_cuda_qkv_pack_weights ends with a
      // full dependency), so the first ring's worth of weight chunks is
      // requested before griddepcontrol.wait; x, which the previous kernel
      // may write, only after it.
      const bool stall = a.inject_stall && blockIdx.x == 0;
      prefetch_tensor_map(&tm_x);  // x is copied right after griddepcontrol.wait
      const int n = (int)(u_end - u_begin);
      const int pre = min(n, a.nstage);
      auto load_w = [&](int i) {
        const long long u = u_begin + i;
        const int tile = (int)(u / a.kb_total), kb = (int)(u % a.kb_total);
        const int s = i % a.nstage;
        unsigned char* st = smem + (size_t)s * stage_bytes;
        // the second chunk is absent when the packed chunk count is odd: its
        // features lie beyond n_out and are never stored
        const bool two = 2 * tile + 1 < a.ntiles_n;
        mbar_arrive_expect_tx(&full_bar[s], (two ? 2 : 1) * w_half + x_bytes);
        const unsigned char* w = static_cast<const unsigned char*>(a.w_packed);
        bulk_load(st, w + ((size_t)(2 * tile) * a.kb_total + kb) * w_half, w_half, &full_bar[s]);
        if (two) bulk_load(st + w_half, w + ((size_t)(2 * tile + 1) * a.kb_total + kb) * w_half, w_half, &full_bar[s]);
      };
      auto load_x = [&](int i) {
        const int k0 = (int)((u_begin + i) % a.kb_total) * kTileK;  // 64 elements = 128 bytes: the 16-byte rule
        const int s = i % a.nstage;
        tma_load_2d(smem + (size_t)s * stage_bytes + 2 * w_half, &tm_x, &full_bar[s], k0, 0);
      };
      for (int i = (stall ? 1 : 0); i < pre; ++i) load_w(i);  // fresh ring: no empty wait
      griddep_wait();
      if constexpr (kTrace) {
        if (a.trace && blockIdx.x < kTraceMaxCta) a.trace[kTraceCta + 8 * blockIdx.x + 1] = gtime();
      }
      for (int i = (stall ? 1 : 0); i < pre; ++i) load_x(i);  // test hook: stage 0 never filled
      int i = pre;
      for (; i < n; ++i) {
        const int s = i % a.nstage;
        const uint32_t ph = (uint32_t)(i / a.nstage) & 1u;
        if (!mbar_wait_bounded(&empty_bar[s], ph ^ 1u, a.flags, a.wait_limit)) break;
        load_w(i);
        load_x(i);
      }
      // drain: the last copies must land before the CTA exits
      for (int t = max(stall ? 1 : 0, i - a.nstage); t < i; ++t)
        mbar_wait_bounded(&full_bar[t % a.nstage], (uint32_t)(t / a.nstage) & 1u, a.flags, a.wait_limit);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer: segment j accumulates in tensor-memory buffer j % 2
      const uint32_t idesc = qkv_idesc(bf16, kStreamM, kStreamN);
      int i = 0, j = 0;
      bool ok = true;
      for (long long u = u_begin; u < u_end && ok; ++j) {
        const Segment sg = segment_at(u, u_end, a.kb_total);
        u += sg.kb1 - sg.kb0;
        const int buf = j & 1;
        const uint32_t use = (uint32_t)(j >> 1);
        // the epilogue has drained this buffer's previous segment
        ok = mbar_wait_bounded(&acc_empty[buf], (use & 1u) ^ 1u, a.flags, a.wait_limit);
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(buf * kStreamN);
        for (int kb = sg.kb0; kb < sg.kb1 && ok; ++kb, ++i) {
          const int s = i % a.nstage;
          const uint32_t ph = (uint32_t)(i / a.nstage) & 1u;
          if (!mbar_wait_bounded(&full_bar[s], ph, a.flags, a.wait_limit)) {
            ok = false;
            break;
          }
          if constexpr (kTrace) {
            if (a.trace && i == 0 && blockIdx.x < kTraceMaxCta) a.trace[kTraceCta + 8 * blockIdx.x + 2] = gtime();
          }
          tc_fence_after();
          const uint32_t sw = smem_u32(smem + (size_t)s * stage_bytes);
          // A = x rows (M 128; rows past the copied BT read the next stage's
          // bytes and only feed accumulator rows that are never stored),
          // B = the 256 weight rows
          const uint64_t da = sw128_kmajor_desc(sw + 2 * w_half), db = sw128_kmajor_desc(sw);
#pragma unroll
          for (int k = 0; k < kTileK / 16; ++k)  // 16 elements = 32 bytes = 2 descriptor units
            umma_f16(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb > sg.kb0 || k > 0) ? 1u : 0u);
          umma_commit(&empty_bar[s]);
        }
        umma_commit(&acc_full[buf]);  // arrives once the segment's MMAs complete
      }
      if constexpr (kTrace) {
        if (a.trace && blockIdx.x < kTraceMaxCta) a.trace[kTraceCta + 8 * blockIdx.x + 3] = gtime();
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue warps 2-5.  They read context lengths, tables and the
    // workspace, and write q and the cache: all after the previous kernel has
    // finished.  Draining tensor memory, thread e owns batch row b (its
    // tensor-memory lane: warp w reads lanes 32 (w % 4) ..).
    griddep_wait();
    const int e = threadIdx.x - 64;
    const int b = (warp & 3) * 32 + lane;
    const bool live = b < a.M;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    init_rows(a, rs, 0, e, kEpiThreads, blockIdx.x == 0);  // visible after the first barrier below
    auto emit = [&](int r, int f0, int n0, float (&v)[16]) { emit_chunk<T>(a, rs, 0, r, f0, n0, v); };
    int j = 0;
    bool aborted = false;
    for (long long u = u_begin; u < u_end; ++j) {
      const Segment sg = segment_at(u, u_end, a.kb_total);
      u += sg.kb1 - sg.kb0;
      const bool whole = sg.kb0 == 0 && sg.kb1 == a.kb_total;
      const long long t0 = (long long)sg.tile * a.kb_total;
      const int g_first = first_cta(t0, a.units, G);
      const int n_contrib = first_cta(t0 + a.kb_total - 1, a.units, G) - g_first + 1;
      const int n0 = sg.tile * kStreamN;
      const int ncols = min(kStreamN, a.n_out - n0);  // a multiple of 64
      // this tile's bias, once every thread is done with the previous one's
      named_bar_sync(1, kEpiThreads);
      load_tile_bias(a, rs, n0, ncols, e, kEpiThreads);
      if (!aborted) {
        const bool ok = mbar_wait_bounded(&acc_full[(j & 1)], (uint32_t)(j >> 1) & 1u, a.flags, a.wait_limit);
        aborted = named_bar_or(1, kEpiThreads, !ok);  // every epilogue warp decides together
      }
      if constexpr (kTrace) {
        if (a.trace && e == 0 && blockIdx.x < kTraceMaxCta) a.trace[kTraceCta + 8 * blockIdx.x + 5] = gtime();
      }
      if (aborted) {
        // the flag is set; still count this CTA's pieces so that every tile's
        // arrival counter returns to zero and the workspace stays usable
        if (!whole && e == 0 && atomicAdd(a.counters + sg.tile, 1) == n_contrib - 1) a.counters[sg.tile] = 0;
        continue;
      }
      const int buf = j & 1;
      tc_fence_after();
      const uint32_t acc = tmem + lane_off + (uint32_t)(buf * kStreamN);
      if (whole) {
        for (int c0 = 0; c0 < ncols; c0 += 16) {
          float v[16];
          tmem_ld16(acc + (uint32_t)c0, v);
          if (live) emit(b, n0 + c0, n0, v);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);
        continue;
      }
      // A piece: publish its partial.  Partials are float4s laid out
      // [slot][16-feature chunk][quarter][row], so the 32 lanes of a warp (32
      // consecutive rows) move 512 contiguous bytes per access.
      const size_t slot_stride = (size_t)(kStreamN / 16) * 4 * BT;  // float4s per slot
      float4* part4 = reinterpret_cast<float4*>(a.partials) + (size_t)sg.tile * a.max_contrib * slot_stride;
      {
        float4* mine = part4 + (size_t)(blockIdx.x - g_first) * slot_stride + b;
        for (int c0 = 0; c0 < ncols; c0 += 16) {
          float v[16];
          tmem_ld16(acc + (uint32_t)c0, v);
          if (live) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              __stcg(mine + (size_t)(c0 / 16 * 4 + i) * BT, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      __threadfence();  // the partial is visible before this CTA's arrival is counted
      named_bar_sync(1, kEpiThreads);
      if (e == 0) last_flag = atomicAdd(a.counters + sg.tile, 1) == n_contrib - 1;
      named_bar_sync(1, kEpiThreads);
      if (!last_flag) continue;
      // the tile's last piece: sum the slots in order and run the epilogue,
      // spread over (row, chunk) items with the row fastest (coalesced
      // loads), up to eight slots' loads in flight per item
      __threadfence();
      if (e == 0) a.counters[sg.tile] = 0;  // zero again for the next call
      if constexpr (kTrace) {
        if (a.trace && e == 0 && blockIdx.x < kTraceMaxCta) a.trace[kTraceCta + 8 * blockIdx.x + 6] = gtime();
      }
      const int M = min(a.M, BT);
      const int items = M * (ncols / 16);
      for (int it = e; it < items; it += kEpiThreads) {
        const int r = it % M, c = it / M;
        const float4* src = part4 + (size_t)c * 4 * BT + r;
        float sum[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) sum[i] = 0.f;
        for (int p0 = 0; p0 < n_contrib; p0 += 8) {
          float4 t[8][4];
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (p0 + q < n_contrib) {
#pragma unroll
              for (int i = 0; i < 4; ++i) t[q][i] = __ldcg(src + (size_t)(p0 + q) * slot_stride + (size_t)i * BT);
            }
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (p0 + q < n_contrib) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                sum[4 * i] += t[q][i].x;
                sum[4 * i + 1] += t[q][i].y;
                sum[4 * i + 2] += t[q][i].z;
                sum[4 * i + 3] += t[q][i].w;
              }
            }
        }
        emit(r, n0 + c * 16, n0, sum);
      }
    }
    if constexpr (kTrace) {
      if (a.trace && e == 0 && blockIdx.x < kTraceMaxCta) a.trace[kTraceCta + 8 * blockIdx.x + 4] = gtime();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kStreamN) : "memory");
  }
}

// Cluster schedule with the weights in N (qkv_cluster_n_kernel), when the
// 256-feature tiles times the 128-row batch tiles times a cluster's K splits
// cover the SMs: grid (feature tiles) x (splits) x (batch tiles), the splits
// of a tile forming one thread-block cluster, each CTA accumulating its K range as in the
// stream-K kernel (M = 128 batch rows, N = 256 features, one accumulator).
// The split-K reduction runs through distributed shared memory: CTA j of the
// cluster owns batch rows [j rs, (j + 1) rs); after the main loops every CTA
// pushes its sums of each owner's rows into that owner's receive buffer
// (overlaying the now idle stage ring), and each owner adds the S partial
// sums in rank order and runs the epilogue for its rows — no global
// workspace, no atomics, and the reduction spread over the cluster.
// 256 threads: warp 0 copies, warp 1 MMAs, warps 2-7 look up the rows; all 8
// drain tensor memory (warp w: lanes 32 (w % 4) .., alternating 16-column
// chunks by w / 4) and run the epilogue.
template <typename T>
__global__ void __launch_bounds__(kClusterThreads, 1)
    qkv_cluster_n_kernel(const __grid_constant__ CUtensorMap tm_x, const QkvArgs a) {
  __shared__ __align__(8) uint64_t full_bar[16];
  __shared__ __align__(8) uint64_t empty_bar[16];
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_base_slot;
  __shared__ RowState rs;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, m0 = blockIdx.z * kStreamM;
  const int n0 = tile * kStreamN;
  const int M = min(a.M - m0, kStreamM);  // rows of this batch tile
  const int ncols = min(kStreamN, a.n_out - n0);  // a multiple of 64
  const int BT = a.batch_tile;
  constexpr uint32_t w_half = kTileN * 128;
  const uint32_t x_bytes = (uint32_t)BT * 128;
  const uint32_t stage_bytes = 2 * w_half + x_bytes;
  // this split's range of 64-wide K blocks
  const int kb_per = a.kb_total / a.splits, kb_rem = a.kb_total % a.splits;
  const int kb0 = split * kb_per + min(split, kb_rem);
  const int nkb = kb_per + (split < kb_rem ? 1 : 0);
  const bool two = 2 * tile + 1 < a.ntiles_n;  // the tile's second 128-feature chunk exists
  const int cta_lin = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;  // trace slot
  if constexpr (kTrace) {
    if (a.trace && threadIdx.x == 0 && cta_lin < kTraceMaxCta) a.trace[kTraceCta + 8 * cta_lin + 0] = gtime();
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.nstage; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&done_bar, 1);
    fence_barrier_init();
  }
  __syncwarp();
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_slot)),
                 "r"(kStreamN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_slot;
  griddep_launch_dependents();  // the next kernel waits for this grid before reading anything

  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  if (warp == 0) {
    if (lane == 0) {
      // producer: the first ring's worth of weight chunks before
      // griddepcontrol.wait (the packed weights are never written by the
      // kernel this one may overlap), x only after it
      const bool stall = a.inject_stall && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
      prefetch_tensor_map(&tm_x);  // x is copied right after griddepcontrol.wait
      const int pre = min(nkb, a.nstage);
      const unsigned char* w = static_cast<const unsigned char*>(a.w_packed);
      auto load_w = [&](int i) {
        const int s = i % a.nstage;
        unsigned char* st = smem + (size_t)s * stage_bytes;
        mbar_arrive_expect_tx(&full_bar[s], (two ? 2 : 1) * w_half + x_bytes);
        bulk_load(st, w + ((size_t)(2 * tile) * a.kb_total + kb0 + i) * w_half, w_half, &full_bar[s]);
        if (two) bulk_load(st + w_half, w + ((size_t)(2 * tile + 1) * a.kb_total + kb0 + i) * w_half, w_half, &full_bar[s]);
      };
      auto load_x = [&](int i) {
        const int s = i % a.nstage;
        // 64 elements = 128 bytes: meets the 16-byte rule
        tma_load_2d(smem + (size_t)s * stage_bytes + 2 * w_half, &tm_x, &full_bar[s], (kb0 + i) * kTileK, m0);
      };
      for (int i = (stall ? 1 : 0); i < pre; ++i) load_w(i);  // fresh ring: no empty wait
      griddep_wait();
      if constexpr (kTrace) {
        if (a.trace && true && cta_lin < kTraceMaxCta) a.trace[kTraceCta + 8 * cta_lin + 1] = gtime();
      }
      for (int i = (stall ? 1 : 0); i < pre; ++i) load_x(i);  // test hook: stage 0 never filled
      int issued = pre;
      for (int i = pre; i < nkb; ++i) {
        const uint32_t ph = (uint32_t)(i / a.nstage) & 1u;
        if (!mbar_wait_bounded(&empty_bar[i % a.nstage], ph ^ 1u, a.flags, a.wait_limit)) break;
        load_w(i);
        load_x(i);
        ++issued;
      }
      // drain: the copies issued last must have landed before shared memory is reused
      for (int i = max(stall ? 1 : 0, issued - a.nstage); i < issued; ++i)
        mbar_wait_bounded(&full_bar[i % a.nstage], (uint32_t)(i / a.nstage) & 1u, a.flags, a.wait_limit);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer: A = x rows (rows past the copied batch tile only feed
      // accumulator rows that are never stored), B = the 256 weight rows
      const uint32_t idesc = qkv_idesc(bf16, kStreamM, kStreamN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % a.nstage;
        const uint32_t ph = (uint32_t)(i / a.nstage) & 1u;
        if (!mbar_wait_bounded(&full_bar[s], ph, a.flags, a.wait_limit)) break;
        if constexpr (kTrace) {
          if (a.trace && i == 0 && cta_lin < kTraceMaxCta) a.trace[kTraceCta + 8 * cta_lin + 2] = gtime();
        }
        tc_fence_after();
        const uint32_t sw = smem_u32(smem + (size_t)s * stage_bytes);
        const uint64_t da = sw128_kmajor_desc(sw + 2 * w_half), db = sw128_kmajor_desc(sw);
#pragma unroll
        for (int k = 0; k < kTileK / 16; ++k)  // 16 elements = 32 bytes = 2 descriptor units
          umma_f16(tmem, da + 2 * k, db + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
        umma_commit(&empty_bar[s]);
      }
      umma_commit(&done_bar);
      if constexpr (kTrace) {
        if (a.trace && true && cta_lin < kTraceMaxCta) a.trace[kTraceCta + 8 * cta_lin + 3] = gtime();
      }
    }
    __syncwarp();
  } else {
    // warps 2-7, idle during the main loop: rows, RoPE factors, this tile's
    // bias (all read after the barrier below)
    griddep_wait();
    init_rows(a, rs, m0, threadIdx.x - 64, kClusterThreads - 64, blockIdx.x == 0 && blockIdx.y == 0);
    load_tile_bias(a, rs, n0, ncols, threadIdx.x - 64, kClusterThreads - 64);
  }
  griddep_wait();  // warps 0-1 (the others have waited already): outputs
  __syncthreads();
  mbar_wait_bounded(&done_bar, 0, a.flags, a.wait_limit);
  tc_fence_after();

  const int g = warp & 3, half = warp >> 2;
  const int r = g * 32 + lane;  // this thread's batch row while draining
  const uint32_t t_lane = tmem + ((uint32_t)(g * 32) << 16);
  const int S = a.splits;
  const int nchunks = ncols / 16;
  if (S == 1) {
    for (int c = half; c < nchunks; c += 2) {
      float v[16];
      tmem_ld16(t_lane + (uint32_t)(c * 16), v);
      if (r < M) emit_chunk<T>(a, rs, m0, r, n0 + c * 16, n0, v);
    }
  } else {
    // rows per owner and the receive buffer, float4s laid out
    // recv[src][16-feature chunk][quarter][row - lo]: the lanes of a warp
    // (consecutive rows) write consecutive 16-byte words of a peer's buffer
    const uint32_t rank = cluster_rank();
    const int rows_per = (BT + S - 1) / S;
    float4* recv = reinterpret_cast<float4*>(smem);
    // every CTA of the cluster has finished its main loop before anyone
    // writes into another's ring
    cluster_sync();
    if constexpr (kTrace) {
      if (a.trace && threadIdx.x == 0 && cta_lin < kTraceMaxCta) a.trace[kTraceCta + 8 * cta_lin + 5] = gtime();
    }
    for (int c = half; c < nchunks; c += 2) {
      float v[16];
      tmem_ld16(t_lane + (uint32_t)(c * 16), v);
      if (r < M) {
        const int owner = r / rows_per;
        float4* dst = recv + ((size_t)(rank * (kStreamN / 16) + c) * 4) * rows_per + (r - owner * rows_per);
        const uint32_t da = map_peer(dst, (uint32_t)owner);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          st_cluster_v4(da + 16u * (uint32_t)(i * rows_per), v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
    }
    tc_fence_before();
    cluster_sync();  // pushes visible; no shared memory is touched remotely after this
    if constexpr (kTrace) {
      if (a.trace && threadIdx.x == 0 && cta_lin < kTraceMaxCta) a.trace[kTraceCta + 8 * cta_lin + 6] = gtime();
    }
    const int lo = (int)rank * rows_per;
    const int n_rows = max(0, min(rows_per, M - lo));
    const int items = n_rows * nchunks;
    for (int it = threadIdx.x; it < items; it += kClusterThreads) {
      const int rr = it % n_rows, c = it / n_rows;
      float sum[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) sum[i] = 0.f;
      for (int p = 0; p < S; ++p) {
        const float4* src = recv + ((size_t)(p * (kStreamN / 16) + c) * 4) * rows_per + rr;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 x4 = src[(size_t)i * rows_per];
          sum[4 * i] += x4.x;
          sum[4 * i + 1] += x4.y;
          sum[4 * i + 2] += x4.z;
          sum[4 * i + 3] += x4.w;
        }
      }
      emit_chunk<T>(a, rs, m0, lo + rr, n0 + c * 16, n0, sum);
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (kTrace) {
    if (a.trace && threadIdx.x == 0 && cta_lin < kTraceMaxCta) a.trace[kTraceCta + 8 * cta_lin + 4] = gtime();
  }
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kStreamN) : "memory");
  }
}

}  // namespace

}  // namespace clove

using namespace clove;

// Clusters of `splits` CTAs of this kernel that fit on the GPU at once,
// cached per (device, kernel kind, splits, shared memory); kind tells the
// kernels and their element types apart.
template <typename Kern>
static int resident_clusters(Kern kern, const cudaLaunchConfig_t& cfg, int device, int kind, int splits,
                             size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, size_t>, int> cache;
  const auto key = std::make_tuple(device, kind, splits, smem);
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> g(mu);
  cache[key] = n;
  return n;
}

// Encode a 2-D K-major operand map {hidden, rows} with a 64 x box_rows box and
// the 128-byte swizzle.
static int encode_operand_map(CUtensorMap* map, const void* base, int dtype, int hidden, int rows, int box_rows) {
  auto fn = tensor_map_encoder();
  if (!fn) return CLOVE_ERR_CUDA;
  const CUtensorMapDataType dt =
      dtype == CLOVE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {(cuuint64_t)hidden, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)hidden * 2};
  cuuint32_t box[2] = {(cuuint32_t)kTileK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CLOVE_OK : CLOVE_ERR_INVALID_ARG;
}

// One thread per 16-byte chunk of the packed layout: chunk (tile t, K block
// kb, row r, position p) holds the 8 elements of W^T row t*128 + r, columns
// kb*64 + 8 (p ^ (r % 8)) .. +7 — the 128-byte swizzle that the bulk-tensor
// copies would apply — with zeros past n_out / hidden.
__global__ void stream_fence_kernel() {}

template <typename T>
__global__ void pack_weights_kernel(const T* __restrict__ w_t, T* __restrict__ out, int n_out, int hidden,
                                    int kb_total, long long chunks) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < chunks;
       i += (long long)gridDim.x * blockDim.x) {
    const int p = (int)(i & 7);
    const int r = (int)((i >> 3) & 127);
    const long long tk = i >> 10;  // t * kb_total + kb
    const int kb = (int)(tk % kb_total), t = (int)(tk / kb_total);
    const int row = t * kTileN + r, col0 = kb * kTileK + 8 * (p ^ (r & 7));
    T v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int col = col0 + e;
      v[e] = (row < n_out && col < hidden) ? w_t[(size_t)row * hidden + col] : T(0.f);
    }
    *reinterpret_cast<uint4*>(out + i * 8) = *reinterpret_cast<const uint4*>(v);
  }
}

static size_t packed_bytes(int n_out, int hidden) {
  return (size_t)((n_out + kTileN - 1) / kTileN) * ((hidden + kTileK - 1) / kTileK) * kTileN * kTileK * 2;
}

// Schedule and workspace of one call.
struct QkvPlan {
  bool stream_k;   // the stream-K schedule
  bool cluster_n;  // the cluster schedule (exactly one of the two is set)
  int batch_tile, ntiles_n, n_btiles, kb_total, grid, max_contrib, nstage;
  long long units;
  size_t smem, off_partials, ws_bytes;
};

// Stage-ring bytes per CTA: the built-in budget, or CLOVE_QKV_RING_KB (a
// tuning override, read once) when that is smaller.
static size_t ring_budget(size_t builtin) {
  static const size_t env = [] {
    const char* v = std::getenv("CLOVE_QKV_RING_KB");
    return v ? (size_t)std::max(0L, std::atol(v)) * 1024 : (size_t)0;
  }();
  return env ? std::min(env, builtin) : builtin;
}

static QkvPlan plan_qkv(const clove_pool& pool, int batch, int hidden, int num_q_heads) {
  QkvPlan P;
  const int n_out = (num_q_heads + 2 * pool.num_kv_heads) * pool.head_dim;
  P.ntiles_n = (n_out + kTileN - 1) / kTileN;
  P.kb_total = (hidden + kTileK - 1) / kTileK;
  // The cluster schedule when its CTAs (256-feature tiles x 128-row batch
  // tiles x K splits, at most 8) cover 60 % of the SMs or the batch is above
  // 32 rows; stream-K (one CTA per SM whatever the tile count) otherwise.
  {
    const int tiles = (P.ntiles_n + 1) / 2, mt = (batch + kStreamM - 1) / kStreamM;
    const int s_fit = std::max(1, std::min({pool.num_sms / (tiles * mt), 8, std::max(1, P.kb_total / 2)}));
    const bool covers = 10 * tiles * mt * s_fit >= 6 * pool.num_sms;
    P.cluster_n = batch > kStreamMaxBatch || covers;
    // CLOVE_QKV_SCHEDULE = stream | cluster forces a schedule (a tuning
    // override, read once; stream-K only up to 128 batch rows)
    static const int forced = [] {
      const char* v = std::getenv("CLOVE_QKV_SCHEDULE");
      if (!v) return 0;
      const std::string t(v);
      return t == "stream" ? 1 : t == "cluster" ? 2 : 0;
    }();
    if (forced) P.cluster_n = forced == 2 || batch > kStreamM;
    P.stream_k = !P.cluster_n;
  }
  if (P.cluster_n) {
    P.n_btiles = (batch + kStreamM - 1) / kStreamM;
    P.batch_tile = P.n_btiles > 1 ? kStreamM : ((batch + 15) / 16) * 16;
    P.units = (long long)((P.ntiles_n + 1) / 2) * P.kb_total;
    const size_t stage = 2 * (size_t)kTileN * 128 + (size_t)P.batch_tile * 128;
    const size_t pad = (size_t)(kStreamM - P.batch_tile) * 128;
    P.nstage = (int)std::max<size_t>(2, std::min<size_t>(16, ring_budget(kSmemBudget - pad) / stage));
    P.smem = stage * P.nstage + pad + 1024;
    P.grid = 0;  // splits chosen at launch (cluster occupancy)
    P.max_contrib = 0;
    P.off_partials = 0;
    P.ws_bytes = 256;  // no workspace
  } else if (P.stream_k) {
    // (256-feature tile) x (64-wide K block) units, split evenly and
    // contiguously over one CTA per SM, at least two K blocks each
    P.n_btiles = 1;
    P.batch_tile = ((batch + 15) / 16) * 16;
    const long long tiles = (P.ntiles_n + 1) / 2;
    P.units = tiles * P.kb_total;
    P.grid = (int)std::max(1LL, std::min((long long)pool.num_sms, P.units / 2));
    const long long per_cta = P.units / P.grid;  // shortest range
    P.max_contrib = (int)std::min((long long)P.grid, (P.kb_total + per_cta - 1) / per_cta + 1);
    // stage: two weight chunks + x [batch_tile][64]; the MMA reads 128 x
    // rows, so the last stage is followed by padding up to 128 rows
    const size_t stage = 2 * (size_t)kTileN * 128 + (size_t)P.batch_tile * 128;
    const size_t pad = (size_t)(kStreamM - P.batch_tile) * 128;
    P.nstage = (int)std::max<size_t>(2, std::min<size_t>(16, ring_budget(kSmemBudget - pad) / stage));
    P.smem = stage * P.nstage + pad + 1024;
    P.off_partials = ((size_t)tiles * 4 + 255) & ~size_t(255);
    P.ws_bytes = P.off_partials + (size_t)tiles * P.max_contrib * P.batch_tile * kStreamN * 4;
  }
  return P;
}

extern "C" {

size_t clove_cuda_qkv_packed_bytes(int n_out, int hidden) {
  if (n_out <= 0 || hidden <= 0) return 0;
  return packed_bytes(n_out, hidden);
}

int clove_cuda_qkv_pack_weights(int dtype, const void* w_t, int n_out, int hidden, void* packed, void* stream) {
  if ((dtype != CLOVE_DTYPE_BF16 && dtype != CLOVE_DTYPE_F16) || !w_t || !packed || n_out <= 0 || hidden <= 0 ||
      (reinterpret_cast<uintptr_t>(packed) & 15u)) {
    set_last_error("qkv_pack_weights: bf16/f16 weights, non-null pointers, packed 16-byte aligned");
    return CLOVE_ERR_INVALID_ARG;
  }
  const int kb_total = (hidden + kTileK - 1) / kTileK;
  const long long chunks = (long long)packed_bytes(n_out, hidden) / 16;
  const int blocks = (int)std::min<long long>((chunks + 255) / 256, 65535);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == CLOVE_DTYPE_BF16)
    pack_weights_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(w_t),
                                                              static_cast<__nv_bfloat16*>(packed), n_out, hidden,
                                                              kb_total, chunks);
  else
    pack_weights_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(w_t), static_cast<__half*>(packed),
                                                       n_out, hidden, kb_total, chunks);
  // An empty kernel with an ordinary (full) dependency on the packing: the
  // projection kernel, a programmatic dependent of whatever precedes it,
  // reads weights before its griddepcontrol.wait, so the kernel right before
  // it must not be the one that wrote them.
  stream_fence_kernel<<<1, 32, 0, s>>>();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("qkv_pack_weights launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(2);
  return CLOVE_OK;
}

size_t clove_cuda_qkv_workspace_size(clove_pool_t pool, int batch, int hidden, int num_q_heads) {
  if (!pool || batch <= 0 || hidden <= 0 || num_q_heads <= 0) return 0;
  return plan_qkv(*pool, batch, hidden, num_q_heads).ws_bytes;
}

int clove_cuda_qkv_append(clove_pool_t pool, const void* x, const void* w_packed, const float* bias, int batch,
                          int hidden, int num_q_heads, const int32_t* block_tables, int bt_stride,
                          const int32_t* context_lens, float rope_theta, void* q_out, int32_t* context_lens_out,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (!pool || batch < 0 || hidden <= 0 || num_q_heads <= 0 || bt_stride <= 0 || rope_theta < 0.f) {
    set_last_error("qkv_append: bad arguments");
    return CLOVE_ERR_INVALID_ARG;
  }
  if (batch == 0) return CLOVE_OK;
  if (!x || !w_packed || !block_tables || !context_lens || !q_out || !workspace ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u)) {
    set_last_error("qkv_append: null pointer or workspace not 256-byte aligned");
    return CLOVE_ERR_INVALID_ARG;
  }
  if (pool->dtype == CLOVE_DTYPE_F32) {
    set_last_error("qkv_append: the tensor-core projection takes bf16/f16 pools");
    return CLOVE_ERR_UNSUPPORTED;
  }
  if (num_q_heads % pool->num_kv_heads || hidden % 8 ||
      (reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(w_packed) & 15u) ||
      (reinterpret_cast<uintptr_t>(q_out) & 15u)) {
    set_last_error("qkv_append: num_q_heads must be a multiple of num_kv_heads, hidden of 8, x/w_packed/q_out 16-byte aligned");
    return CLOVE_ERR_INVALID_ARG;
  }
  const QkvPlan P = plan_qkv(*pool, batch, hidden, num_q_heads);
  if (workspace_bytes < P.ws_bytes) {
    set_last_error("qkv_append: workspace %zu bytes < required %zu", workspace_bytes, P.ws_bytes);
    return CLOVE_ERR_WORKSPACE;
  }
  QkvArgs a = {};
  a.w_packed = w_packed;
  a.bias = bias;
  a.block_tables = block_tables;
  a.context_lens = context_lens;
  a.lens_out = context_lens_out;
  a.q_out = q_out;
  a.k_cache = pool->k_cache;
  a.v_cache = pool->v_cache;
  a.flags = pool->flags;
  a.counters = static_cast<int32_t*>(workspace);
  a.partials = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + P.off_partials);
  a.M = batch;
  a.hidden = hidden;
  a.hq = num_q_heads;
  a.hkv = pool->num_kv_heads;
  a.D = pool->head_dim;
  a.bs = pool->block_size;
  a.bt_stride = bt_stride;
  a.num_blocks = pool->num_blocks;
  a.n_out = (num_q_heads + 2 * pool->num_kv_heads) * pool->head_dim;
  a.kb_total = P.kb_total;
  a.ntiles_n = P.ntiles_n;
  a.batch_tile = P.batch_tile;
  a.nstage = P.nstage;
  a.max_contrib = P.max_contrib;
  a.units = P.units;
  a.rope_theta = rope_theta;
  a.inject_stall = debug_inject_stall();
  a.trace = kTrace ? trace_buffer() : nullptr;
  const uint32_t lim = debug_wait_limit();
  a.wait_limit = lim ? lim : kWaitLimit;

  CUtensorMap tm_x;
  if (encode_operand_map(&tm_x, x, pool->dtype, hidden, batch, P.batch_tile) != CLOVE_OK) {
    set_last_error("qkv_append: cuTensorMapEncodeTiled failed (hidden %d, batch %d)", hidden, batch);
    return CLOVE_ERR_INVALID_ARG;
  }
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != pool->device) cudaSetDevice(pool->device);
  cudaError_t e = cudaSuccess;
  if (P.stream_k) {
    auto kern = pool->dtype == CLOVE_DTYPE_BF16 ? qkv_stream_kernel<__nv_bfloat16> : qkv_stream_kernel<__half>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P.smem);
    if (e == cudaSuccess) {
      // a programmatic dependent of the previous kernel on the stream: its
      // set-up and first weight copies overlap that kernel's tail
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(P.grid);
      cfg.blockDim = dim3(kQkvThreads);
      cfg.dynamicSmemBytes = P.smem;
      cfg.stream = static_cast<cudaStream_t>(stream);
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      e = cudaLaunchKernelEx(&cfg, kern, tm_x, a);
    }
  } else if (P.cluster_n) {
    auto kern = pool->dtype == CLOVE_DTYPE_BF16 ? qkv_cluster_n_kernel<__nv_bfloat16> : qkv_cluster_n_kernel<__half>;
    const int tiles = (P.ntiles_n + 1) / 2;
    const size_t stage = 2 * (size_t)kTileN * 128 + (size_t)P.batch_tile * 128;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kClusterThreads);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cfg.dynamicSmemBytes = P.smem;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;  // the occupancy query sees the cluster shape only
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P.smem);
    // K splits: enough CTAs to cover the SMs, at most 8 (portable cluster),
    // at least 2 K blocks each, a receive buffer of splits x (rows per CTA) x
    // 256 f32 that fits in the ring, and all clusters resident at once
    const int mt = P.n_btiles;
    int splits = std::max(1, std::min({pool->num_sms / (tiles * mt), 8, std::max(1, P.kb_total / 2)}));
    for (; e == cudaSuccess && splits > 1; --splits) {
      const size_t rows_per = ((size_t)P.batch_tile + splits - 1) / splits;
      if ((size_t)splits * rows_per * kStreamN * 4 > stage * P.nstage) continue;
      cfg.gridDim = dim3(tiles, splits, mt);
      attr[0].val.clusterDim.y = splits;
      if (resident_clusters(kern, cfg, pool->device, 16 + (int)pool->dtype, splits, P.smem) >= tiles * mt) break;
    }
    a.splits = splits;
    if (e == cudaSuccess) {
      cfg.gridDim = dim3(tiles, splits, mt);
      attr[0].val.clusterDim.y = splits;
      cfg.numAttrs = 2;
      e = cudaLaunchKernelEx(&cfg, kern, tm_x, a);
    }
  }
  if (prev >= 0 && prev != pool->device) cudaSetDevice(prev);
  if (e != cudaSuccess) {
    set_last_error("qkv_append launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(1);
  return CLOVE_OK;
}

}  // extern "C"
