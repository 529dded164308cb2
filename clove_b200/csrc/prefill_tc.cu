// Prefill attention over the paged cache on the 5th-generation tensor cores
// with two query tiles in flight per CTA ("ping-pong"): bf16 / f16, head_dim
// 128, 1..16 query heads per KV head (a divisor of 128), block sizes
// dividing 128.
//
// Semantics: the reference's FlashAttention step (src/lazy.rs:4821-4923),
// causal, on RoPE-rotated q and k (the prep kernel in prefill.cu rotates them
// and writes the prompt's K/V into the cache), scale 1/sqrt(head_dim): every
// prompt token attends over its sequence's cache up to its own position.
//
// Work unit: (sequence b, pair of consecutive tiles of TQ = 128 / G prompt
// tokens, KV head h).  Tile A holds the first TQ tokens of the pair, tile B
// the next TQ (absent past the prompt's end); each is 128 query rows =
// (token, query head of the group) pairs, the M of the tensor-core tile.  The
// two tiles read the same keys (B's range extends A's by TQ), so K and V of
// a step are loaded once for both.  Units are claimed longest-first
// (prefill_plan_kernel's list over tile pairs) by a persistent grid of one
// CTA per SM.
//
// Tensor memory (512 columns): S_A at 0, S_B at 128, O_A at 256, O_B at 384.
// Per 128-key step s the MMA warp issues, in this order,
//   S_A(s) = Q_A K^T,  P_B(s-1) V -> O_B,  S_B(s) = Q_B K^T,  P_A(s) V -> O_A
// so the softmax of one tile (S -> P) runs while the tensor cores work on the
// other's.  The softmax writes P (16-bit, packed in pairs) over the first 64
// columns of its S buffer and the P.V MMA reads A from tensor memory; the
// next S of that tile is issued after that P.V, and the tensor pipe executes
// one thread's MMAs in issue order.
// Roles (320 threads): warp 0 issues the bulk tensor copies (Q of both tiles
// once per unit; K and V of each step as [block_size, 64] boxes per 64-dim
// half), warp 1 issues the MMAs and owns the tensor-memory allocation, warps
// 2-5 run tile A's softmax and epilogue, warps 6-9 tile B's (row r = tensor
// memory lane r; warp w reads lanes 32 (w % 4) ..).  Only when a row's max
// rises by more than 2^8 does its softmax move the reference and rescale its
// O row (after the previous P.V of that tile finished).  Every wait is
// bounded; a wait that runs out sets CLOVE_FLAG_TIMEOUT and the CTA winds
// down without hanging.
//
// Shared memory (1024-byte aligned): Q [2 tiles][2 halves][128 rows][128 B]
// = 64 KB, 2 K/V stages of [K | V][2 halves][128 keys][128 B] = 64 KB each:
// 192 KB.
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "host.h"
#include "prefill_common.cuh"
#include "tc_common.cuh"

namespace clove {

namespace {

constexpr int kThreads = 320;          // TMA warp, MMA warp, 2 x 4 softmax warps
constexpr int kTileThreads = 128;      // softmax threads of one tile
constexpr int kRows = 128;             // query rows per tile (MMA M)
constexpr int kKeys = 128;             // keys per step
constexpr int kD = 128;                // head_dim
constexpr uint32_t kQTile = kRows * kD * 2;     // 32 KB
constexpr uint32_t kHalf = kKeys * 128;         // 16 KB: 128 keys x 64 dims
constexpr uint32_t kKV = 2 * kHalf;             // K (or V) of one step
constexpr uint32_t kStage = 2 * kKV;            // K + V
constexpr int kStages = 2;
constexpr uint32_t kSmem = 2 * kQTile + kStages * kStage + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;    // + 128 tile: S (f32), then P (16-bit pairs) in its first 64 columns
constexpr uint32_t kTmemO = 256;  // + 128 tile

struct PairUnit {
  int b, jp, h, valid;
  int nk[2];  // keys of tile A / B (0: tile absent)
  int ns[2];  // 128-key steps of tile A / B
};

// 16 consecutive 32-bit columns of this thread's tensor-memory lane, no wait.
__device__ __forceinline__ void tmem_ld16f_nowait(uint32_t taddr, float* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7]),
        "=f"(v[8]), "=f"(v[9]), "=f"(v[10]), "=f"(v[11]), "=f"(v[12]), "=f"(v[13]), "=f"(v[14]), "=f"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 16 consecutive 32-bit columns of this thread's lane, no wait.
__device__ __forceinline__ void tmem_st16_nowait(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// tcgen05.mma with A read from tensor memory (M x K, a row per lane, two
// 16-bit K elements per 32-bit column).
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack_pair<__nv_bfloat16>(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack_pair<__half>(float lo, float hi) {
  const __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const PrefillArgs a) {
  __shared__ __align__(8) uint64_t q_full, q_empty, drain;
  __shared__ __align__(8) uint64_t k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
  // per tile: S ready, P ready (its 128 softmax threads), P.V done, O free (epilogue read it)
  __shared__ __align__(8) uint64_t s_full[2], p_full[2], pv_done[2], o_empty[2];
  __shared__ __align__(8) uint64_t ufull[2], uempty[2];
  __shared__ PairUnit slots[2];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  unsigned char* sQ = smem;              // [tile][2 halves][128][128 B]
  unsigned char* sKV = smem + 2 * kQTile;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.group, TQ = a.tq / 2;  // the plan's items are tile pairs of 2 TQ tokens
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&q_empty, 1);
    mbar_init(&drain, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kTileThreads);
      mbar_init(&pv_done[i], 1);
      mbar_init(&o_empty[i], kTileThreads);
      mbar_init(&ufull[i], 1);
      mbar_init(&uempty[i], 1 + 8);  // the MMA thread + one arrival per softmax warp
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
  // the previous kernel (the prep kernel, which itself waited for the plan
  // kernel) has finished: the cache rows, rotated q and the work list are in place
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if constexpr (kTrace) {
    if (a.trace && threadIdx.x == 0) a.trace[16 + 16 * 32 * 16 + 2 * blockIdx.x] = gtime();
  }
  const int n_units = *a.n_items * a.hkv;

  // trace builds: CTA 0's first 16 units, 32 steps each, 16 events per step:
  // 0-2 softmax A (S landed, S read, P ready), 3-5 softmax B, 6-9 MMA issue
  // of S_A, P_B.V, S_B, P_A.V; then each CTA's start (past the plan) and end
  auto mark = [&](int ui, int s, int k) {
    if constexpr (kTrace) {
      if (a.trace && blockIdx.x == 0 && ui < 16 && s < 32) a.trace[16 + (ui * 32 + s) * 16 + k] = gtime();
    }
  };
  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (abort_flag) return false;
    if (!mbar_wait_bounded(bar, parity, a.err, a.wait_limit)) {
      abort_flag = 1;
      return false;
    }
    return true;
  };
  auto unit_of = [&](int u) {
    PairUnit x;
    x.valid = u < n_units;
    x.b = x.jp = x.h = 0;
    x.nk[0] = x.nk[1] = x.ns[0] = x.ns[1] = 0;
    if (x.valid) {
      const int2 it = a.items[u / a.hkv];
      x.b = it.x;
      x.jp = it.y;
      x.h = u - (u / a.hkv) * a.hkv;
      const int len = __ldg(a.cu_seqlens + x.b + 1) - __ldg(a.cu_seqlens + x.b);
      const int ctx = __ldg(a.context_lens + x.b);
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int tok0 = (2 * x.jp + t) * TQ;
        if (tok0 < len) {
          x.nk[t] = ctx + min(tok0 + TQ, len);
          x.ns[t] = (x.nk[t] + kKeys - 1) / kKeys;
        }
      }
    }
    return x;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol = policy_evict_first();
    if (lane == 0) {
      prefetch_tensor_map(&tm_q);
      prefetch_tensor_map(&tm_k);
      prefetch_tensor_map(&tm_v);
    }
    const int bs = a.bs, bps = kKeys / bs;  // blocks per step
    int ui = 0, g = 0, stalled_g = -1;
    bool ok = true;
    while (ok) {
      int u = 0;
      if (lane == 0) u = atomicAdd(a.unit_counter, 1);
      u = __shfl_sync(0xffffffffu, u, 0);
      const PairUnit x = unit_of(u);
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
      const int tiles = x.ns[1] > 0 ? 2 : 1;
      const int nsteps = max(x.ns[0], x.ns[1]);
      const int nkeys = max(x.nk[0], x.nk[1]);
      if (lane == 0) {
        if (wait(&q_empty, ((uint32_t)ui & 1u) ^ 1u)) {
          mbar_arrive_expect_tx(&q_full, (uint32_t)tiles * kQTile);
          for (int t = 0; t < tiles; ++t) {
            const int tok = seq0 + (2 * x.jp + t) * TQ;
            tma_load_3d(sQ + t * kQTile, &tm_q, &q_full, 0, x.h * G, tok, pol);
            tma_load_3d(sQ + t * kQTile + kQTile / 2, &tm_q, &q_full, 64, x.h * G, tok, pol);
          }
        } else {
          ok = false;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      const int32_t* bt = a.block_tables + (size_t)x.b * a.bt_stride;
      const int nblk = (nkeys + bs - 1) / bs;
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
      for (int s = 0; s < nsteps && ok; ++s, ++g) {
        const int nxt = s + 1 < nsteps ? table(s + 1) : 0;
        const int st = g % kStages;
        if (a.inject_stall && u == 0 && s == 0) stalled_g = g;
        const int nb = min(bps, nblk - s * bps);
        int phys[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) phys[i] = __shfl_sync(0xffffffffu, cur, i);
        if (lane == 0) {
          const uint32_t par = ((uint32_t)(g / kStages) & 1u) ^ 1u;
          const uint32_t bytes = (uint32_t)nb * (uint32_t)bs * 128u * 2u;  // two 64-dim halves
          unsigned char* kst = sKV + (size_t)st * kStage;
          unsigned char* vst = kst + kKV;
          if (!wait(&k_empty[st], par)) {
            ok = false;
          } else if (a.inject_stall && u == 0 && s == 0) {
            // test hook: this step's K is never filled, so the MMA warp's wait runs out
          } else {
            mbar_arrive_expect_tx(&k_full[st], bytes);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              if (i < nb) {
                const uint32_t row = (uint32_t)(i * bs) * 128u;
                tma_load_3d(kst + row, &tm_k, &k_full[st], 0, x.h, phys[i] * bs, pol);
                tma_load_3d(kst + kHalf + row, &tm_k, &k_full[st], 64, x.h, phys[i] * bs, pol);
              }
            }
          }
          if (ok && !wait(&v_empty[st], par)) {
            ok = false;
          } else if (ok) {
            mbar_arrive_expect_tx(&v_full[st], bytes);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              if (i < nb) {
                const uint32_t row = (uint32_t)(i * bs) * 128u;
                tma_load_3d(vst + row, &tm_v, &v_full[st], 0, x.h, phys[i] * bs, pol);
                tma_load_3d(vst + kHalf + row, &tm_v, &v_full[st], 64, x.h, phys[i] * bs, pol);
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
      const uint32_t idesc_s = f16_idesc(bf16, kRows, kKeys, 0);
      const uint32_t idesc_pv = f16_idesc(bf16, kRows, kD, 1);
      int ui = 0, g = 0;
      int sc[2] = {0, 0}, pc[2] = {0, 0}, uc[2] = {0, 0};  // per tile: S issued, P.V issued, units
      bool ok = true;
      // S_t(s): Q_t K(s)^T into S_t
      auto issue_s = [&](int t, int s) -> bool {
        const int st = (g + s) % kStages;
        if (t == 0 && !wait(&k_full[st], (uint32_t)((g + s) / kStages) & 1u)) return false;
        tc_fence_after();
        mark(ui, s, 6 + 2 * t);
        const uint32_t qa = smem_u32(sQ + t * kQTile), ka = smem_u32(sKV + (size_t)st * kStage);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem + kTmemS + 128u * t, sw128_kmajor_desc(qa + c * (kQTile / 2)) + 2 * k,
                     sw128_kmajor_desc(ka + c * kHalf) + 2 * k, idesc_s, (c | k) ? 1u : 0u);
        umma_commit(&s_full[t]);
        ++sc[t];
        return true;
      };
      // O_t += P_t(s) V(s), P from tensor memory
      auto issue_pv = [&](int t, int s) -> bool {
        const int st = (g + s) % kStages;
        if (!wait(&p_full[t], (uint32_t)pc[t] & 1u)) return false;
        if (!wait(&v_full[st], (uint32_t)((g + s) / kStages) & 1u)) return false;
        if (s == 0 && !wait(&o_empty[t], ((uint32_t)uc[t] & 1u) ^ 1u)) return false;
        tc_fence_after();
        mark(ui, s, t == 0 ? 9 : 7);
        const uint32_t va = smem_u32(sKV + (size_t)st * kStage + kKV);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16_ts(tmem + kTmemO + 128u * t, tmem + kTmemS + 128u * t + (uint32_t)(32 * c + 8 * k),
                        sw128_mnmajor_desc(va + (uint32_t)(64 * c + 16 * k) * 128u, kHalf, 1024), idesc_pv,
                        (s == 0 && c == 0 && k == 0) ? 0u : 1u);
        umma_commit(&pv_done[t]);
        ++pc[t];
        return true;
      };
      while (ok) {
        const int uk = ui & 1;
        if (!wait(&ufull[uk], (uint32_t)(ui >> 1) & 1u)) break;
        const PairUnit x = slots[uk];
        mbar_arrive(&uempty[uk]);
        if (!x.valid) break;
        if (!wait(&q_full, (uint32_t)ui & 1u)) break;
        const int nA = x.ns[0], nB = x.ns[1];
        const int ns = max(nA, nB);
        for (int s = 0; s <= ns && ok; ++s) {
          const int st = (g + s) % kStages;
          if (s < nA) ok = issue_s(0, s);
          if (ok && s >= 1 && s - 1 < nB) {
            ok = issue_pv(1, s - 1);
            if (ok) umma_commit(&v_empty[(g + s - 1) % kStages]);  // V(s-1): B's P.V is its last reader
          }
          if (ok && s < nB) {
            if (s >= nA && !wait(&k_full[st], (uint32_t)((g + s) / kStages) & 1u)) ok = false;  // not waited by S_A
            if (ok) ok = issue_s(1, s);
          }
          if (ok && s < ns) {
            umma_commit(&k_empty[st]);  // K(s) is free once the S MMAs above complete
            if (s == ns - 1) umma_commit(&q_empty);  // and Q once the unit's last S completes
          }
          if (ok && s < nA) {
            ok = issue_pv(0, s);
            if (ok && s >= nB) umma_commit(&v_empty[st]);  // V(s) not read by tile B
          }
        }
        if (nA > 0) ++uc[0];
        if (nB > 0) ++uc[1];
        g += ns;
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
    const int t = (warp - 2) >> 2;         // 0: tile A (warps 2-5), 1: tile B (warps 6-9)
    const int r = (warp & 3) * 32 + lane;  // this thread's row = tensor-memory lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t sreg = tmem + lane_off + kTmemS + 128u * t;
    const uint32_t oreg = tmem + lane_off + kTmemO + 128u * t;
    const int t_in = r / G, gq = r - (r / G) * G;
    int ui = 0, g = 0, sc = 0, pc = 0;
    // Waits here are warp-uniform: the tensor-memory loads and stores that
    // follow are warp-collective (.sync.aligned), so no lane may leave early.
    auto wait_w = [&](uint64_t* bar, uint32_t parity) -> bool {
      const bool r = wait(bar, parity);
      return __all_sync(0xffffffffu, r ? 1 : 0) != 0;
    };
    // wait until this tile's P.V number i has completed (i < 0: nothing to wait for)
    auto pv_wait = [&](int i) -> bool { return i < 0 || wait_w(&pv_done[t], (uint32_t)i & 1u); };
    bool ok = true;
    while (ok) {
      const int uk = ui & 1;
      if (!wait_w(&ufull[uk], (uint32_t)(ui >> 1) & 1u)) break;
      const PairUnit x = slots[uk];
      __syncwarp();
      if (lane == 0) mbar_arrive(&uempty[uk]);
      if (!x.valid) break;
      const int ns_all = max(x.ns[0], x.ns[1]);
      const int nk_all = max(x.nk[0], x.nk[1]);
      const int nsteps = x.ns[t];
      if (nsteps == 0) {  // tile B past the prompt's end
        g += ns_all;
        ++ui;
        continue;
      }
      const int seq0 = __ldg(a.cu_seqlens + x.b);
      const int len = __ldg(a.cu_seqlens + x.b + 1) - seq0;
      const int tok0 = (2 * x.jp + t) * TQ;
      const int ntq = min(TQ, len - tok0);
      const bool row_ok = t_in < ntq;
      const int pos = row_ok ? __ldg(a.context_lens + x.b) + tok0 + t_in : -1;
      float m = -INFINITY, l = 0.f;
      for (int s = 0; s < nsteps && ok; ++s) {
        if (!wait_w(&s_full[t], (uint32_t)sc & 1u)) {
          ok = false;
          break;
        }
        ++sc;
        tc_fence_after();
        if ((warp & 3) == 0 && lane == 0) mark(ui, s, 3 * t);
        float v[128];
#pragma unroll
        for (int i = 0; i < 8; ++i) tmem_ld16f_nowait(sreg + 16u * i, v + 16 * i);
        tmem_wait_ld();
        if ((warp & 3) == 0 && lane == 0) mark(ui, s, 3 * t + 1);
        const int key0 = s * kKeys;
        if (key0 + kKeys - 1 > pos) {  // the causal mask, only on steps that reach past the row's position
#pragma unroll
          for (int k = 0; k < 128; ++k) v[k] = key0 + k <= pos ? v[k] : -INFINITY;
        }
        float mx = row_max128(v);
        mx *= a.qscale;  // the row's max, log2 domain (the scale is positive)
        // P is taken relative to a reference m that moves only when the
        // row's max rises by more than 8 (log2 units): P <= 2^8 stays exact
        // enough in 16 bits and the sums in f32, and O is rescaled (a wait on
        // the previous P.V) only on those rare jumps.
        const bool move = mx > m + 8.f;  // also true on the first visible key (m = -inf)
        const float m_new = move ? mx : m;
        const float ref = m_new == -INFINITY ? 0.f : m_new;
        const float corr = move ? exp2f(m - ref) : 1.f;  // 0 when m was -inf
        const float rs = row_exp2_sum128(v, a.qscale, ref);
        l = l * corr + rs;
        const bool rescale = move && s > 0 && m != -INFINITY;
        m = m_new;
        // P over the first 64 columns of this tile's S buffer (S is read)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t pk[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) pk[k] = pack_pair<T>(v[32 * i + 2 * k], v[32 * i + 2 * k + 1]);
          tmem_st16_nowait(sreg + 16u * i, pk);
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
          for (int i = 0; i < 8; ++i) {
            float t16[16];
            tmem_ld16(oreg + 16u * i, t16);
#pragma unroll
            for (int k = 0; k < 16; ++k) t16[k] *= f;
            tmem_st16(oreg + 16u * i, t16);
          }
        }
        tmem_wait_st();
        if (s == ns_all - 1 && s * kKeys + kKeys > nk_all) {
          // V rows past the pair's last key may hold any bits (P is 0 there,
          // but 0 * NaN is NaN inside the MMA): zero them once the copies
          // landed (both tiles' softmaxes do, whichever P.V comes first);
          // thread r clears key row r
          const int st = (g + s) % kStages;
          if (!wait_w(&v_full[st], (uint32_t)((g + s) / kStages) & 1u)) {
            ok = false;
            break;
          }
          if (s * kKeys + r >= nk_all) {
            unsigned char* vst = sKV + (size_t)st * kStage + kKV + (size_t)r * 128;
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              *reinterpret_cast<uint4*>(vst + u * 16) = make_uint4(0, 0, 0, 0);
              *reinterpret_cast<uint4*>(vst + kHalf + u * 16) = make_uint4(0, 0, 0, 0);
            }
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor cores
        }
        tc_fence_before();
        if ((warp & 3) == 0 && lane == 0) mark(ui, s, 3 * t + 2);
        mbar_arrive(&p_full[t]);
        ++pc;
      }
      if (!ok) break;
      // ---- epilogue: O / l for valid rows ----
      if (!pv_wait(pc - 1)) break;
      tc_fence_after();
      {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        float* dst = a.out + ((size_t)(seq0 + tok0 + t_in) * a.hq + (size_t)x.h * G + gq) * kD;
#pragma unroll 1
        for (int i = 0; i < 8; ++i) {
          float o[16];
          tmem_ld16(oreg + 16u * i, o);
          if (row_ok) {
#pragma unroll
            for (int k = 0; k < 16; k += 4)
              *reinterpret_cast<float4*>(dst + 16 * i + k) =
                  make_float4(o[k] * inv, o[k + 1] * inv, o[k + 2] * inv, o[k + 3] * inv);
          }
        }
        tc_fence_before();
        mbar_arrive(&o_empty[t]);
      }
      g += ns_all;
      ++ui;
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (kTrace) {
    if (a.trace && threadIdx.x == 0) a.trace[16 + 16 * 32 * 16 + 2 * blockIdx.x + 1] = gtime();
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// 3-D map {64-dim half, rows, tokens} with the 128-byte swizzle over a
// [tokens, rows, 128] 16-bit array; box {64, box_rows, box_tokens}.
static int encode_map(CUtensorMap* map, const void* base, int dtype, long long tokens, int rows, int box_rows,
                      int box_tokens) {
  auto fn = tensor_map_encoder();
  if (!fn) {
    set_last_error("cuTensorMapEncodeTiled unavailable from the driver");
    return CLOVE_ERR_CUDA;
  }
  const CUtensorMapDataType dt =
      dtype == CLOVE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)rows, (cuuint64_t)tokens};
  cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)rows * kD * 2};
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
  return pool.elem_bytes == 2 && pool.head_dim == kD && group >= 1 && group <= 16 && kRows % group == 0 &&
         pool.block_size >= 8 && kKeys % pool.block_size == 0;
}

// Plan (the longest-first list over pairs of tiles of 128 / group tokens) +
// the paired tensor-core kernel.  q_rot: rotated queries [num_tokens,
// num_q_heads, 128] (256-byte aligned); ws: prefill_mma_scratch_bytes(num_tokens) bytes.
int launch_prefill_tc(const clove_pool& pool, const void* q_rot, float* out, const int32_t* cu_seqlens,
                      const int32_t* context_lens, const int32_t* block_tables, int bt_stride, int batch,
                      int num_tokens, int num_q_heads, float scale, int max_ctx, void* ws, cudaStream_t stream, int phase) {
  const int group = num_q_heads / pool.num_kv_heads;
  const int tq = kRows / group;
  CUtensorMap tm_q, tm_k, tm_v;
  const long long slots = (long long)pool.num_blocks * pool.block_size;
  int rc = encode_map(&tm_q, q_rot, pool.dtype, num_tokens, num_q_heads, group, tq);
  if (!rc) rc = encode_map(&tm_k, pool.k_cache, pool.dtype, slots, pool.num_kv_heads, 1, pool.block_size);
  if (!rc) rc = encode_map(&tm_v, pool.v_cache, pool.dtype, slots, pool.num_kv_heads, 1, pool.block_size);
  if (rc) return rc;
  unsigned char* w = static_cast<unsigned char*>(ws);
  PrefillArgs a{};
  a.q = q_rot;
  a.out = out;
  a.cu_seqlens = cu_seqlens;
  a.context_lens = context_lens;
  a.block_tables = block_tables;
  a.items = reinterpret_cast<int2*>(w + 512);  // pairs <= num_tokens
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
  a.tq = 2 * tq;  // the plan lists pairs of tiles
  a.sb = 1;
  a.nstage = kStages;
  a.max_ctx = max_ctx;
  a.wait_limit = debug_wait_limit();
  a.inject_stall = debug_inject_stall();
  a.qscale = scale * kLog2e;
  a.trace = kTrace ? trace_buffer() : nullptr;
  cudaError_t e = cudaSuccess;
  if (phase & kPrefillPlanOnly) {
    prefill_plan_kernel<<<1, 1024, 0, stream>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
      set_last_error("prefill plan launch: %s", cudaGetErrorString(e));
      return CLOVE_ERR_CUDA;
    }
    count_launches(1);
  }
  if (!(phase & kPrefillKernelOnly)) return CLOVE_OK;
  const bool bf16 = pool.dtype == CLOVE_DTYPE_BF16;
  auto kern = bf16 ? prefill_tc_kernel<__nv_bfloat16> : prefill_tc_kernel<__half>;
  static std::once_flag attr_once[2];
  static cudaError_t attr_err[2];
  std::call_once(attr_once[bf16 ? 1 : 0], [&] {
    attr_err[bf16 ? 1 : 0] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  });
  if (attr_err[bf16 ? 1 : 0] != cudaSuccess) {
    set_last_error("cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err[bf16 ? 1 : 0]));
    return CLOVE_ERR_CUDA;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pool.num_sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, tm_q, tm_k, tm_v, a);
  if (e != cudaSuccess) {
    set_last_error("paged_prefill (tcgen05, paired tiles) launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(1);
  return CLOVE_OK;
}

}  // namespace clove
