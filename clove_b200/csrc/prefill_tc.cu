// Prefill attention over the paged cache on the 5th-generation tensor cores
// (tcgen05): bf16 / f16, head_dim 128, 1..16 query heads per KV head (a
// divisor of 128), block sizes dividing 128.
//
// Semantics: the reference's FlashAttention step (src/lazy.rs:4821-4923),
// causal, on RoPE-rotated q and k (the prep kernel in prefill.cu rotates them
// and writes the prompt's K/V into the cache), scale 1/sqrt(head_dim): every
// prompt token attends over its sequence's cache up to its own position.
//
// Work unit: (sequence b, tile j of TQ = 128 / G prompt tokens, KV head h):
// 128 query rows = (token, query head of the group) pairs, the M of the
// tensor-core tile.  Units are claimed longest-first (prefill_plan_kernel's
// list) by a persistent grid of one CTA per SM.
//
// Per 128-key step of a unit:
//   S = Q K^T   tcgen05.mma, M 128 rows x N 128 keys x K 128 dims, both
//               operands K-major in shared memory (128-byte swizzle), the f32
//               result in one of two 128-column tensor-memory buffers;
//   softmax     one thread per row reads its 128 scores from tensor memory,
//               applies the causal mask and scale, updates its reference
//               max and sum, and writes P (16-bit) to shared memory as a
//               K-major operand; only when its max rose by more than 2^8 does
//               it move the reference and rescale its O row in tensor memory
//               (after the previous P.V finished);
//   O += P V    tcgen05.mma, M 128 x N 128 dims x K 128 keys, P K-major and V
//               MN-major (the cache rows are dim-contiguous), O in tensor
//               memory for the whole unit.
// Roles (320 threads): warp 0 issues the bulk tensor copies (Q once per unit;
// K and V of each step as [block_size, 64] boxes per 64-dim half), warp 1
// issues the MMAs and owns the tensor-memory allocation, warps 2-9 run the
// softmax and the epilogue (two warpgroups: row r = tensor-memory lane r,
// each warpgroup on 64 of the row's key columns and of O's dims).  S
// of step s+1 is computed while the softmax of step s runs and P.V of step s
// waits for its P.  Every wait is bounded; a wait that runs out sets
// CLOVE_FLAG_TIMEOUT and the CTA winds down without hanging.
//
// Shared memory (1024-byte aligned): Q [2 halves][128 rows][128 B] = 32 KB,
// 2 K/V stages of [K | V][2 halves][128 keys][128 B] = 64 KB each, 2 P
// buffers [2 key chunks][128 rows][128 B] = 32 KB each: 224 KB.
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "host.h"
#include "prefill_common.cuh"
#include "tc_common.cuh"

namespace clove {

namespace {

constexpr int kTcThreads = 320;  // TMA warp, MMA warp, 8 softmax warps
constexpr int kSoftThreads = 256;  // two warpgroups, each on 64 of a row's 128 key columns
constexpr int kTcRows = 128;                            // query rows per unit (MMA M)
constexpr int kTcKeys = 128;                            // keys per step
constexpr int kTcD = 128;                               // head_dim
constexpr uint32_t kQBytes = kTcRows * kTcD * 2;        // 32 KB
constexpr uint32_t kHalfBytes = kTcKeys * 128;          // 16 KB: 128 keys x 64 dims
constexpr uint32_t kKVBytes = 2 * kHalfBytes;           // K (or V) of one step
constexpr uint32_t kStageBytes = 2 * kKVBytes;          // K + V
constexpr int kStages = 2;
constexpr uint32_t kPBytes = kTcRows * kTcKeys * 2;     // 32 KB
constexpr uint32_t kSmemBytes = kQBytes + kStages * kStageBytes + 2 * kPBytes + 1024;
constexpr uint32_t kTmemCols = 512;                     // S buffers at columns 0 and 128, O at 256
constexpr uint32_t kTmemO = 256;
constexpr uint32_t kTmemX = 384;                        // row max / sum exchange between the two softmax halves

struct TcUnit {
  int b, j, h, nkeys, nsteps, valid;
};

// 16 consecutive columns of this thread's tensor-memory lane, no wait.
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// One 32-bit column of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_st1(uint32_t taddr, float v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(__float_as_uint(v)) : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
  tmem_ld_wait();
  return __uint_as_float(r);
}

// 2^x with the tensor-core path's accuracy needs (P is rounded to 16 bits
// next): the special-function unit's approximation, -inf -> +0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void fence_proxy_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  const __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const PrefillArgs a) {
  __shared__ __align__(8) uint64_t q_full, q_empty, o_empty, drain;
  // K and V of a stage are filled and released separately: K is free again
  // once that step's S MMAs finish, V once its P.V finishes
  __shared__ __align__(8) uint64_t k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
  __shared__ __align__(8) uint64_t s_full[2], s_empty[2], p_full[2];
  // P.V of P index i completes phase i / 2 of pv_done[i % 2]: a waiter is never more than one phase
  // behind (the next completion on that barrier needs a P the waiter has not produced yet)
  __shared__ __align__(8) uint64_t pv_done[2];
  __shared__ __align__(8) uint64_t ufull[2], uempty[2];
  __shared__ __align__(8) uint64_t pair_bar[4];  // the two softmax warps on one lane quarter
  __shared__ TcUnit slots[2];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  unsigned char* sQ = smem;
  unsigned char* sKV = smem + kQBytes;
  unsigned char* sP = sKV + kStages * kStageBytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.group, TQ = a.tq;
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&q_empty, 1);
    mbar_init(&o_empty, kSoftThreads);
    mbar_init(&drain, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&pair_bar[i], 64);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kSoftThreads);
      mbar_init(&p_full[i], kSoftThreads);
      mbar_init(&pv_done[i], 1);
      mbar_init(&ufull[i], 1);
      mbar_init(&uempty[i], 1 + kSoftThreads / 32);  // the MMA thread + one arrival per softmax warp
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the plan kernel's list
  const int n_units = *a.n_items * a.hkv;

  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (abort_flag) return false;
    if (!mbar_wait_bounded(bar, parity, a.err, a.wait_limit)) {
      abort_flag = 1;
      return false;
    }
    return true;
  };
  auto unit_of = [&](int u) {
    TcUnit x;
    x.valid = u < n_units;
    x.b = x.j = x.h = x.nkeys = x.nsteps = 0;
    if (x.valid) {
      const int2 it = a.items[u / a.hkv];
      x.b = it.x;
      x.j = it.y;
      x.h = u - (u / a.hkv) * a.hkv;
      const int len = __ldg(a.cu_seqlens + x.b + 1) - __ldg(a.cu_seqlens + x.b);
      x.nkeys = __ldg(a.context_lens + x.b) + min((x.j + 1) * TQ, len);
      x.nsteps = (x.nkeys + kTcKeys - 1) / kTcKeys;
    }
    return x;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol = policy_evict_first();
    const int bs = a.bs, bps = kTcKeys / bs;  // blocks per step
    int ui = 0, g = 0, stalled_g = -1;
    bool ok = true;
    while (ok) {
      int u = 0;
      if (lane == 0) u = atomicAdd(a.unit_counter, 1);
      u = __shfl_sync(0xffffffffu, u, 0);
      const TcUnit x = unit_of(u);
      const int uk = ui & 1;
      if (lane == 0) {
        if (wait(&uempty[uk], ((uint32_t)(ui >> 1) & 1u) ^ 1u)) {
          slots[uk] = x;
          mbar_arrive(&ufull[uk]);
        } else {
          ok = false;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok || !x.valid) break;
      const int seq0 = __ldg(a.cu_seqlens + x.b);
      if (lane == 0) {
        if (wait(&q_empty, ((uint32_t)ui & 1u) ^ 1u)) {
          mbar_arrive_expect_tx(&q_full, kQBytes);
          tma_load_3d(sQ, &tm_q, &q_full, 0, x.h * G, seq0 + x.j * TQ, pol);
          tma_load_3d(sQ + kQBytes / 2, &tm_q, &q_full, 64, x.h * G, seq0 + x.j * TQ, pol);
        } else {
          ok = false;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      const int32_t* bt = a.block_tables + (size_t)x.b * a.bt_stride;
      const int nblk = (x.nkeys + bs - 1) / bs;
      // block-table entries of a step, one per lane (bps <= 16), loaded a step ahead
      auto table = [&](int s) {
        const int kb = s * bps + lane;
        int v = 0;
        if (lane < bps && kb < nblk) {
          v = __ldg(bt + kb);
          if (v < 0 || v >= a.num_blocks) {
            atomicOr(a.err, CLOVE_FLAG_BLOCK_OOB);
            v = 0;
          }
        }
        return v;
      };
      int cur = table(0);
      for (int s = 0; s < x.nsteps && ok; ++s, ++g) {
        const int nxt = s + 1 < x.nsteps ? table(s + 1) : 0;
        const int st = g % kStages;
        if (a.inject_stall && u == 0 && s == 0) stalled_g = g;
        const int nb = min(bps, nblk - s * bps);
        int phys[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) phys[i] = __shfl_sync(0xffffffffu, cur, i);
        if (lane == 0) {
          const uint32_t par = ((uint32_t)(g / kStages) & 1u) ^ 1u;
          const uint32_t bytes = (uint32_t)nb * (uint32_t)bs * 128u * 2u;  // two 64-dim halves
          unsigned char* kst = sKV + (size_t)st * kStageBytes;
          unsigned char* vst = kst + kKVBytes;
          if (!wait(&k_empty[st], par)) {
            ok = false;
          } else if (a.inject_stall && u == 0 && s == 0) {
            // test hook: this step's K is never filled, so the MMA warp's wait runs out
          } else {
            {
              mbar_arrive_expect_tx(&k_full[st], bytes);
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                if (i < nb) {
                  const uint32_t row = (uint32_t)(i * bs) * 128u;
                  tma_load_3d(kst + row, &tm_k, &k_full[st], 0, x.h, phys[i] * bs, pol);
                  tma_load_3d(kst + kHalfBytes + row, &tm_k, &k_full[st], 64, x.h, phys[i] * bs, pol);
                }
              }
            }
          }
          if (ok && !wait(&v_empty[st], par)) {
            ok = false;
          } else if (ok) {
            {
              mbar_arrive_expect_tx(&v_full[st], bytes);
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                if (i < nb) {
                  const uint32_t row = (uint32_t)(i * bs) * 128u;
                  tma_load_3d(vst + row, &tm_v, &v_full[st], 0, x.h, phys[i] * bs, pol);
                  tma_load_3d(vst + kHalfBytes + row, &tm_v, &v_full[st], 64, x.h, phys[i] * bs, pol);
                }
              }
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        cur = nxt;
      }
      ++ui;
    }
    if (lane == 0) {
      // drain: copies in flight must land before the CTA exits
      for (int t = max(0, g - kStages); t < g; ++t) {
        for (uint32_t i = 0; i < a.wait_limit; ++i)
          if (mbar_try_wait(&v_full[t % kStages], (uint32_t)(t / kStages) & 1u)) break;
        if (a.inject_stall && t == stalled_g) continue;
        for (uint32_t i = 0; i < a.wait_limit; ++i)
          if (mbar_try_wait(&k_full[t % kStages], (uint32_t)(t / kStages) & 1u)) break;
      }
      if (ui > 0)
        for (uint32_t i = 0; i < a.wait_limit; ++i)
          if (mbar_try_wait(&q_full, (uint32_t)(ui - 1) & 1u)) break;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = f16_idesc(bf16, kTcRows, kTcKeys, 0);
      const uint32_t idesc_pv = f16_idesc(bf16, kTcRows, kTcD, 1);
      int ui = 0, g = 0, sc = 0, pc = 0;
      bool ok = true;
      while (ok) {
        const int uk = ui & 1;
        if (!wait(&ufull[uk], (uint32_t)(ui >> 1) & 1u)) break;
        const TcUnit x = slots[uk];
        mbar_arrive(&uempty[uk]);
        if (!x.valid) break;
        if (!wait(&q_full, (uint32_t)ui & 1u)) break;
        for (int s = 0; s <= x.nsteps && ok; ++s) {
          if (s < x.nsteps) {
            const int st = (g + s) % kStages;
            const int sb = sc & 1;
            if (!wait(&k_full[st], (uint32_t)((g + s) / kStages) & 1u) ||
                !wait(&s_empty[sb], ((uint32_t)(sc >> 1) & 1u) ^ 1u)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t qa = smem_u32(sQ), ka = smem_u32(sKV + (size_t)st * kStageBytes);
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma_f16(tmem + (uint32_t)(sb * kTcKeys), sw128_kmajor_desc(qa + c * (kQBytes / 2)) + 2 * k,
                         sw128_kmajor_desc(ka + c * kHalfBytes) + 2 * k, idesc_s, (c | k) ? 1u : 0u);
            umma_commit(&s_full[sb]);
            umma_commit(&k_empty[st]);  // K of this stage is free once S completes
            ++sc;
            if (s == x.nsteps - 1) umma_commit(&q_empty);  // Q is free once these complete
          }
          if (s >= 1) {
            const int t = s - 1;
            const int st = (g + t) % kStages;
            const int pb = pc & 1;
            if (!wait(&p_full[pb], (uint32_t)(pc >> 1) & 1u) || !wait(&v_full[st], (uint32_t)((g + t) / kStages) & 1u) ||
                (t == 0 && !wait(&o_empty, ((uint32_t)ui & 1u) ^ 1u))) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t pa = smem_u32(sP + (size_t)pb * kPBytes);
            const uint32_t va = smem_u32(sKV + (size_t)st * kStageBytes + kKVBytes);
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma_f16(tmem + kTmemO, sw128_kmajor_desc(pa + c * (kPBytes / 2)) + 2 * k,
                         sw128_mnmajor_desc(va + (uint32_t)(64 * c + 16 * k) * 128u, kHalfBytes, 1024), idesc_pv,
                         (t == 0 && c == 0 && k == 0) ? 0u : 1u);
            umma_commit(&v_empty[st]);
            umma_commit(&pv_done[pb]);
            ++pc;
          }
        }
        g += x.nsteps;
        ++ui;
      }
      // every MMA issued has completed before the tensor memory is released
      umma_commit(&drain);
      for (uint32_t i = 0; i < a.wait_limit; ++i)
        if (mbar_try_wait(&drain, 0)) break;
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    // Warps 2-9: warp w reads tensor-memory lanes 32 (w % 4) .. (its rows);
    // warps w and w + 4 share those rows, warp 2-5 taking key columns 0-63
    // and dims 0-63 of O, warps 6-9 columns 64-127 and dims 64-127.  The two
    // halves of a row exchange their maxima each step (a pairwise named
    // barrier) and their sums once per unit.
    const int r = (warp & 3) * 32 + lane;  // this thread's row = tensor-memory lane
    const int half = (warp - 2) >> 2;      // 0: columns 0-63, 1: columns 64-127
    const int col0 = 64 * half;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    uint64_t* pbar = &pair_bar[warp & 3];  // the pair of warps on these rows
    uint32_t pphase = 0;
    const int t_in = r / G, gq = r - (r / G) * G;
    // exchange columns: kTmemX + 2 parity + half (maxima, by step parity), kTmemX + 4 + half (sums)
    const uint32_t xcol = tmem + lane_off + kTmemX;
    int ui = 0, g = 0, sc = 0, pc = 0, st_par = 0;
    // Waits here are warp-uniform: the tensor-memory loads and stores that
    // follow are warp-collective (.sync.aligned), so no lane may leave early.
    auto wait_w = [&](uint64_t* bar, uint32_t parity) -> bool {
      const bool r = wait(bar, parity);
      return __all_sync(0xffffffffu, r ? 1 : 0) != 0;
    };
    // wait until P.V of P index i has completed (i < 0: nothing to wait for)
    auto pv_wait = [&](int i) -> bool {
      return i < 0 || wait_w(&pv_done[i & 1], (uint32_t)(i >> 1) & 1u);
    };
    // The two warps of a row pair meet (bounded, like every wait here: a
    // partner that left on an abort makes this return false, never hang).
    auto pair_sync = [&]() -> bool {
      tc_fence_before();
      mbar_arrive(pbar);
      const bool r = wait_w(pbar, pphase);
      pphase ^= 1u;
      tc_fence_after();
      return r;
    };
    bool ok = true;
    while (ok) {
      const int uk = ui & 1;
      if (!wait_w(&ufull[uk], (uint32_t)(ui >> 1) & 1u)) break;
      const TcUnit x = slots[uk];
      __syncwarp();
      if (lane == 0) mbar_arrive(&uempty[uk]);
      if (!x.valid) break;
      const int seq0 = __ldg(a.cu_seqlens + x.b);
      const int len = __ldg(a.cu_seqlens + x.b + 1) - seq0;
      const int ntq = min(TQ, len - x.j * TQ);
      const bool row_ok = t_in < ntq;
      const int pos = row_ok ? __ldg(a.context_lens + x.b) + x.j * TQ + t_in : -1;
      float m = -INFINITY, l = 0.f;
      for (int s = 0; s < x.nsteps && ok; ++s) {
        const int sb = sc & 1;
        if (!wait_w(&s_full[sb], (uint32_t)(sc >> 1) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float v[64];
        {
          uint32_t rr[4][16];
#pragma unroll
          for (int i = 0; i < 4; ++i) tmem_ld16_async(tmem + lane_off + (uint32_t)(sb * kTcKeys + col0 + 16 * i), rr[i]);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int k = 0; k < 16; ++k) v[16 * i + k] = __uint_as_float(rr[i][k]);
        }
        tc_fence_before();
        mbar_arrive(&s_empty[sb]);
        ++sc;
        const int key0 = s * kTcKeys + col0;
        // this half's max of the raw scores (the scale is positive); the
        // causal mask only on steps that reach past this row's position
        float mx = -INFINITY;
        if (key0 + 63 <= pos) {
#pragma unroll
          for (int k = 0; k < 64; ++k) mx = fmaxf(mx, v[k]);
        } else {
#pragma unroll
          for (int k = 0; k < 64; ++k) {
            v[k] = key0 + k <= pos ? v[k] : -INFINITY;
            mx = fmaxf(mx, v[k]);
          }
        }
        tmem_st1(xcol + 2 * st_par + half, mx);
        if (!pair_sync()) {
          ok = false;
          break;
        }
        mx = fmaxf(mx, tmem_ld1(xcol + 2 * st_par + (half ^ 1))) * a.qscale;  // the row's max, log2 domain
        st_par ^= 1;
        // P is taken relative to a reference m that moves only when the row's
        // max rises by more than 8 (log2 units): P <= 2^8 stays exact enough
        // in 16 bits and the sums in f32, and O is rescaled (a wait on the
        // previous P.V) only on those rare jumps.  Both halves of a row see
        // the same maxima, so they take the same decisions.
        const bool move = mx > m + 8.f;  // also true on the first visible key (m = -inf)
        const float m_new = move ? mx : m;
        const float ref = m_new == -INFINITY ? 0.f : m_new;
        const float corr = move ? exp2f(m - ref) : 1.f;  // 0 when m was -inf
        float rs = 0.f;
#pragma unroll
        for (int k = 0; k < 64; ++k) {
          v[k] = ex2_approx(fmaf(v[k], a.qscale, -ref));
          rs += v[k];
        }
        l = l * corr + rs;
        const bool rescale = move && s > 0 && m != -INFINITY;
        m = m_new;
        // P buffer pc & 1 was last read by the P.V of P index pc - 2
        if (!pv_wait(pc - 2)) {
          ok = false;
          break;
        }
        {
          unsigned char* prow = sP + (size_t)(pc & 1) * kPBytes + (size_t)half * (kPBytes / 2) + (size_t)r * 128;
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            uint4 q4;
            q4.x = pack2<T>(v[8 * w + 0], v[8 * w + 1]);
            q4.y = pack2<T>(v[8 * w + 2], v[8 * w + 3]);
            q4.z = pack2<T>(v[8 * w + 4], v[8 * w + 5]);
            q4.w = pack2<T>(v[8 * w + 6], v[8 * w + 7]);
            *reinterpret_cast<uint4*>(prow + ((w ^ (r & 7)) << 4)) = q4;
          }
        }
        if (__any_sync(0xffffffffu, rescale ? 1 : 0)) {
          // the previous P.V must have finished writing O; the whole warp
          // takes part (rows whose max did not rise scale by 1)
          if (!pv_wait(pc - 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float f = rescale ? corr : 1.f;
#pragma unroll 1
          for (int i = 0; i < 4; ++i) {
            float t16[16];
            tmem_ld16(tmem + lane_off + kTmemO + col0 + 16 * i, t16);
#pragma unroll
            for (int k = 0; k < 16; ++k) t16[k] *= f;
            tmem_st16(tmem + lane_off + kTmemO + col0 + 16 * i, t16);
          }
        }
        if (s == x.nsteps - 1 && s * kTcKeys + kTcKeys > x.nkeys) {
          // V rows past the last key may hold any bits (P is 0 there, but
          // 0 * NaN is NaN inside the MMA): zero them once the copies landed;
          // thread (row r, half) clears key row r's dims of its half
          const int st = (g + s) % kStages;
          if (!wait_w(&v_full[st], (uint32_t)((g + s) / kStages) & 1u)) {
            ok = false;
            break;
          }
          if (s * kTcKeys + r >= x.nkeys) {
            unsigned char* vst = sKV + (size_t)st * kStageBytes + kKVBytes + (size_t)half * kHalfBytes + (size_t)r * 128;
#pragma unroll
            for (int u = 0; u < 8; ++u) *reinterpret_cast<uint4*>(vst + u * 16) = make_uint4(0, 0, 0, 0);
          }
        }
        fence_proxy_async_shared();  // P (and zeroed V rows) visible to the tensor cores
        tc_fence_before();
        mbar_arrive(&p_full[pc & 1]);
        ++pc;
      }
      if (!ok) break;
      // ---- epilogue: O / l for valid rows, this half's 64 dims ----
      tmem_st1(xcol + 4 + half, l);
      if (!pair_sync()) break;
      const float lt = l + tmem_ld1(xcol + 4 + (half ^ 1));
      if (!pv_wait(pc - 1)) break;
      tc_fence_after();
      {
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
        float* dst = a.out + ((size_t)(seq0 + x.j * TQ + t_in) * a.hq + (size_t)x.h * G + gq) * kTcD + col0;
#pragma unroll 1
        for (int i = 0; i < 4; ++i) {
          float o[16];
          tmem_ld16(tmem + lane_off + kTmemO + col0 + 16 * i, o);
          if (row_ok) {
#pragma unroll
            for (int k = 0; k < 16; k += 4)
              *reinterpret_cast<float4*>(dst + 16 * i + k) =
                  make_float4(o[k] * inv, o[k + 1] * inv, o[k + 2] * inv, o[k + 3] * inv);
          }
        }
        tc_fence_before();
        mbar_arrive(&o_empty);
      }
      g += x.nsteps;
      ++ui;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// 3-D map {64-dim half, rows, tokens} with the 128-byte swizzle over a
// [tokens, rows, 128] 16-bit array; box {64, box_rows, box_tokens}.
static int encode_half_map(CUtensorMap* map, const void* base, int dtype, long long tokens, int rows, int box_rows,
                           int box_tokens) {
  auto fn = tensor_map_encoder();
  if (!fn) {
    set_last_error("cuTensorMapEncodeTiled unavailable from the driver");
    return CLOVE_ERR_CUDA;
  }
  const CUtensorMapDataType dt =
      dtype == CLOVE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {(cuuint64_t)kTcD, (cuuint64_t)rows, (cuuint64_t)tokens};
  cuuint64_t strides[2] = {(cuuint64_t)kTcD * 2, (cuuint64_t)rows * kTcD * 2};
  cuuint32_t box[3] = {64u, (cuuint32_t)box_rows, (cuuint32_t)box_tokens};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("paged_prefill: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return CLOVE_ERR_INVALID_ARG;
  }
  return CLOVE_OK;
}

}  // namespace

bool prefill_tc_supported(const clove_pool& pool, int num_q_heads) {
  const int group = num_q_heads / pool.num_kv_heads;
  return pool.elem_bytes == 2 && pool.head_dim == kTcD && group >= 1 && group <= 16 && kTcRows % group == 0 &&
         pool.block_size >= 8 && kTcKeys % pool.block_size == 0;
}

// Plan (the longest-first list over tiles of 128 / group tokens) + the
// tensor-core kernel.  q_rot: rotated queries [num_tokens, num_q_heads, 128]
// (256-byte aligned); ws: prefill_mma_scratch_bytes(num_tokens) bytes.
int launch_prefill_tc(const clove_pool& pool, const void* q_rot, float* out, const int32_t* cu_seqlens,
                      const int32_t* context_lens, const int32_t* block_tables, int bt_stride, int batch,
                      int num_tokens, int num_q_heads, float scale, int max_ctx, void* ws, cudaStream_t stream) {
  const int group = num_q_heads / pool.num_kv_heads;
  CUtensorMap tm_q, tm_k, tm_v;
  const long long slots = (long long)pool.num_blocks * pool.block_size;
  int rc = encode_half_map(&tm_q, q_rot, pool.dtype, num_tokens, num_q_heads, group, kTcRows / group);
  if (!rc) rc = encode_half_map(&tm_k, pool.k_cache, pool.dtype, slots, pool.num_kv_heads, 1, pool.block_size);
  if (!rc) rc = encode_half_map(&tm_v, pool.v_cache, pool.dtype, slots, pool.num_kv_heads, 1, pool.block_size);
  if (rc) return rc;
  unsigned char* w = static_cast<unsigned char*>(ws);
  PrefillArgs a;
  a.q = q_rot;
  a.out = out;
  a.cu_seqlens = cu_seqlens;
  a.context_lens = context_lens;
  a.block_tables = block_tables;
  a.items = reinterpret_cast<int2*>(w + 512);  // tiles <= num_tokens
  a.n_items = reinterpret_cast<int32_t*>(w + 256);
  a.unit_counter = reinterpret_cast<int32_t*>(w + 256) + 2;
  a.err = pool.flags;
  a.bt_stride = bt_stride;
  a.batch = batch;
  a.hq = num_q_heads;
  a.hkv = pool.num_kv_heads;
  a.group = group;
  a.bs = pool.block_size;
  a.num_blocks = pool.num_blocks;
  a.tq = kTcRows / group;
  a.sb = 1;
  a.nstage = kStages;
  a.max_ctx = max_ctx;
  a.wait_limit = debug_wait_limit();
  a.inject_stall = debug_inject_stall();
  a.qscale = scale * kLog2e;
  prefill_plan_kernel<<<1, 1024, 0, stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("prefill plan launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(1);
  const bool bf16 = pool.dtype == CLOVE_DTYPE_BF16;
  auto kern = bf16 ? prefill_tc_kernel<__nv_bfloat16> : prefill_tc_kernel<__half>;
  static std::once_flag attr_once[2];
  static cudaError_t attr_err[2];
  std::call_once(attr_once[bf16 ? 1 : 0], [&] {
    attr_err[bf16 ? 1 : 0] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  });
  if (attr_err[bf16 ? 1 : 0] != cudaSuccess) {
    set_last_error("cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err[bf16 ? 1 : 0]));
    return CLOVE_ERR_CUDA;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pool.num_sms);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, tm_q, tm_k, tm_v, a);
  if (e != cudaSuccess) {
    set_last_error("paged_prefill (tcgen05) launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(1);
  return CLOVE_OK;
}

}  // namespace clove
