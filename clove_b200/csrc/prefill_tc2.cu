// Prefill attention over the paged cache with 2-CTA tensor-core MMAs
// (tcgen05 .cta_group::2): a cluster of two CTAs on an SM pair computes S and
// P.V for 256 query rows per instruction (128 in each CTA), so each SM issues
// half the MMA instructions per FLOP of the one-CTA kernel.  bf16 / f16,
// head_dim 128, 1..16 query heads per KV head (a divisor of 128), block sizes
// dividing 128.
//
// Semantics: the reference's FlashAttention step (src/lazy.rs:4821-4923),
// causal, on RoPE-rotated q and k (rotated by the prep kernel in prefill.cu,
// which also writes the prompt's K/V into the cache), scale 1/sqrt(head_dim).
//
// Work unit (per cluster): (sequence b, quad of consecutive tiles of TQ = 128
// / G prompt tokens, KV head h).  CTA r of the pair holds tiles 4 jq + r
// ("tile A") and 4 jq + 2 + r ("tile B"); the MMA "tile A" is the 256 rows of
// both CTAs' tile A, likewise B.  Each CTA keeps the ping-pong of the one-CTA
// kernel (S_A, P_B.V, S_B, P_A.V per 128-key step, P over S in tensor
// memory).  The B operands are split between the pair: CTA r loads keys
// [64 r, 64 r + 64) of K and dims [64 r, 64 r + 64) of V for each step, so
// each SM also loads half of the K/V bytes.
//
// Only the leader (rank 0) issues MMAs.  Barriers the MMA warp waits on live
// in the leader: both CTAs' copies complete their transaction bytes there
// (bulk tensor copies with .cta_group::2), the peer's softmax and epilogue
// threads arrive there remotely.  The MMA commits multicast to both CTAs
// (S ready, P.V done, K/V stage and Q free).  Units are claimed by the
// leader's producer and written into both CTAs' slots.  Every wait is
// bounded; a wait that runs out sets CLOVE_FLAG_TIMEOUT and both CTAs wind
// down (each of their waits is bounded too).
//
// Shared memory per CTA (1024-byte aligned, identical layout in both CTAs,
// which the MMA descriptors rely on): Q [tile A | tile B][2 halves][128
// rows][128 B] = 64 KB, 4 stages of K [2 dim halves][64 keys][128 B] + V
// [128 keys][128 B] = 32 KB each: 192 KB.
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "host.h"
#include "prefill_common.cuh"
#include "tc_common.cuh"

namespace clove {

namespace {

constexpr int kThreads = 320;                   // TMA warp, MMA warp, 2 x 4 softmax warps
constexpr int kTileThreads = 128;
constexpr int kRows = 128;                      // query rows per tile per CTA
constexpr int kKeys = 128;                      // keys per step
constexpr int kD = 128;                         // head_dim
constexpr uint32_t kQTile = kRows * kD * 2;     // 32 KB
constexpr uint32_t kKHalf = 64 * 128;           // 8 KB: 64 keys x 64 dims
constexpr uint32_t kKBytes = 2 * kKHalf;        // this CTA's K: 64 keys x 128 dims
constexpr uint32_t kVBytes = kKeys * 128;       // this CTA's V: 128 keys x 64 dims
constexpr uint32_t kStage = kKBytes + kVBytes;  // 32 KB
constexpr int kStages = 4;
constexpr uint32_t kSmem = 2 * kQTile + kStages * kStage + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;    // + 128 tile
constexpr uint32_t kTmemO = 256;  // + 128 tile
constexpr int kRemoteArrivals = 2 * kTileThreads / 32;  // one per softmax warp of a tile, both CTAs

struct QuadUnit {
  int u, b, jq, h, valid;  // u: the claimed unit index
  int nk[2];  // keys of MMA tile A / B (the longer of the pair's two CTA tiles; 0: absent)
  int ns[2];  // 128-key steps
};

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of this CTA's shared variable `p` in the window of cluster CTA `rank`.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}
__device__ __forceinline__ void arrive_remote(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void arrive_expect_tx_remote(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void st_remote_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
// Phase wait that also acquires at cluster scope (the arrivals may come from
// the other CTA); bounded like every wait here.
__device__ __forceinline__ bool try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// 3-D bulk tensor copy into this CTA's shared memory whose transaction bytes
// complete on the leader's barrier (`bar`: a shared::cluster address).
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                                 int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void umma_pair_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_pair_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrive on `bar` (same offset) in both CTAs once every MMA issued so far completes.
__device__ __forceinline__ void commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void commit_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16f(uint32_t taddr, float* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7]),
        "=f"(v[8]), "=f"(v[9]), "=f"(v[10]), "=f"(v[11]), "=f"(v[12]), "=f"(v[13]), "=f"(v[14]), "=f"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

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
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    prefill_tc2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const PrefillArgs a) {
  // waited by the leader's MMA thread (the peer's instances stay unused)
  __shared__ __align__(8) uint64_t q_full, k_full[kStages], v_full[kStages], p_full[2], o_empty[2], uempty[2], drain;
  // completed by the leader's multicast commits, waited in each CTA
  __shared__ __align__(8) uint64_t q_empty, k_empty[kStages], v_empty[kStages], s_full[2], pv_done[2];
  __shared__ __align__(8) uint64_t ufull[2];
  // peer only: the leader saw this stage's copies land (before zeroing V rows past the last key)
  __shared__ __align__(8) uint64_t v_landed[kStages];
  __shared__ QuadUnit slots[2];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  unsigned char* sQ = smem;  // [tile A | tile B]
  unsigned char* sKV = smem + 2 * kQTile;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cta_rank();
  const bool leader = rank == 0;
  const int G = a.group, TQ = a.tq / 4;  // the plan's items are quads of tiles
  const int kSub = min(a.bs, 64);        // tokens per K/V copy box
  const int nsub = kKeys / kSub;         // boxes per 128-key step
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 2);
    mbar_init(&q_empty, 1);
    mbar_init(&drain, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&k_full[i], 2);
      mbar_init(&v_full[i], 2);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&v_landed[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&pv_done[i], 1);
      mbar_init(&p_full[i], kRemoteArrivals);
      mbar_init(&o_empty[i], kRemoteArrivals);
      mbar_init(&ufull[i], 1);
      // the leader's MMA thread + both CTAs' 8 softmax warps + the peer's producer
      mbar_init(&uempty[i], 1 + 16 + 1);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before anyone arrives remotely
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  // the previous kernel (the prep kernel, which itself waited for the plan
  // kernel) has finished: the cache rows, rotated q and the work list are in place
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if constexpr (kTrace) {
    if (a.trace && threadIdx.x == 0) a.trace[16 + 16 * 32 * 16 + 2 * blockIdx.x] = gtime();
  }
  const int n_units = *a.n_items * a.hkv;

  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (abort_flag) return false;
    for (uint32_t i = 0; i < a.wait_limit; ++i)
      if (try_wait_cluster(bar, parity)) return true;
    atomicOr(a.err, CLOVE_FLAG_TIMEOUT);
    if constexpr (kTrace) {
      // trace builds: the first wait of this CTA that ran out (barrier, parity, warp)
      if (a.trace && blockIdx.x < 256 && atomicCAS(reinterpret_cast<unsigned long long*>(a.trace) + 16 + 4 * blockIdx.x, 0ull, 1ull) == 0ull) {
        a.trace[12000 + 4 * blockIdx.x + 1] = smem_u32(bar);
        a.trace[12000 + 4 * blockIdx.x + 2] = parity;
        a.trace[12000 + 4 * blockIdx.x + 3] = (unsigned long long)(threadIdx.x) | ((unsigned long long)rank << 32);
      }
    }
    abort_flag = 1;
    return false;
  };
  if constexpr (kTrace) {
    if (a.trace && blockIdx.x == 0 && threadIdx.x == 0) {
      const void* names[12] = {&q_full, &k_full[0], &v_full[0], &p_full[0], &o_empty[0], &uempty[0],
                               &q_empty, &k_empty[0], &v_empty[0], &s_full[0], &pv_done[0], &ufull[0]};
      for (int i = 0; i < 12; ++i) a.trace[13200 + i] = smem_u32(names[i]);
    }
  }
  // trace builds: CTA 0's first 16 units, 32 steps each, 16 events per step
  // (0-2 softmax A: S landed, S read, P ready; 3-5 softmax B; 6-9 MMA issue
  // of S_A, P_B.V, S_B, P_A.V; 10-15 the peer's softmax events); then each
  // CTA's start and end
  auto mark = [&](int ui, int s, int k) {
    if constexpr (kTrace) {
      if (a.trace && blockIdx.x < 2 && ui < 16 && s < 32 && (blockIdx.x == 0 || k < 6))
        a.trace[16 + (ui * 32 + s) * 16 + k + (blockIdx.x == 1 ? 10 : 0)] = gtime();
    }
  };
  auto unit_of = [&](int u) {
    QuadUnit x;
    x.u = u;
    x.valid = u < n_units;
    x.b = x.jq = x.h = 0;
    x.nk[0] = x.nk[1] = x.ns[0] = x.ns[1] = 0;
    if (x.valid) {
      const int2 it = a.items[u / a.hkv];
      x.b = it.x;
      x.jq = it.y;
      x.h = u - (u / a.hkv) * a.hkv;
      const int len = __ldg(a.cu_seqlens + x.b + 1) - __ldg(a.cu_seqlens + x.b);
      const int ctx = __ldg(a.context_lens + x.b);
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        // the pair's tiles 4 jq + 2 t + {0, 1}: keys of the later one present
        const int tok0 = (4 * x.jq + 2 * t) * TQ;
        if (tok0 < len) {
          x.nk[t] = ctx + min(tok0 + 2 * TQ, len);
          x.ns[t] = (x.nk[t] + kKeys - 1) / kKeys;
        }
      }
    }
    return x;
  };
  const uint32_t lead_q_full = peer_addr(&q_full, 0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    const uint64_t pol = policy_evict_first();
    if (lane == 0) {
      prefetch_tensor_map(&tm_q);
      prefetch_tensor_map(&tm_k);
      prefetch_tensor_map(&tm_v);
    }
    const int bs = a.bs, bps = kKeys / bs;
    int ui = 0, g = 0;
    bool ok = true;
    while (ok) {
      const int uk = ui & 1;
      QuadUnit x;
      if (leader) {
        int u = 0;
        if (lane == 0) u = atomicAdd(a.unit_counter, 1);
        u = __shfl_sync(0xffffffffu, u, 0);
        x = unit_of(u);
        if (lane == 0) {
          if (wait(&uempty[uk], ((uint32_t)(ui >> 1) & 1u) ^ 1u)) {
            slots[uk] = x;
            const uint32_t base = peer_addr(&slots[uk], 1);
            const uint32_t* src = reinterpret_cast<const uint32_t*>(&x);
            for (int i = 0; i < (int)(sizeof(QuadUnit) / 4); ++i) st_remote_u32(base + 4u * i, src[i]);
            mbar_arrive(&ufull[uk]);
            arrive_remote(peer_addr(&ufull[uk], 1));  // release: the slot stores above first
          } else {
            ok = false;
          }
        }
      } else {
        // every lane waits (acquire) before reading the slot the leader wrote
        ok = __all_sync(0xffffffffu, wait(&ufull[uk], (uint32_t)(ui >> 1) & 1u) ? 1 : 0) != 0;
        if (!ok) break;
        x = slots[uk];
        __syncwarp();
        if (lane == 0) arrive_remote(peer_addr(&uempty[uk], 0));
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok || !x.valid) break;
      const int seq0 = __ldg(a.cu_seqlens + x.b);
      const int nsteps = max(x.ns[0], x.ns[1]);
      const int nkeys = max(x.nk[0], x.nk[1]);
      if (lane == 0) {
        // this CTA's two Q tiles (rows of absent or partial tiles are never
        // stored; past the last token the copy fills zeros)
        if (wait(&q_empty, ((uint32_t)ui & 1u) ^ 1u)) {
          arrive_expect_tx_remote(lead_q_full, 2 * kQTile);
          for (int t = 0; t < 2; ++t) {
            const int tok = seq0 + (4 * x.jq + 2 * t + (int)rank) * TQ;
            tma_load_3d_pair(sQ + t * kQTile, &tm_q, lead_q_full, 0, x.h * G, tok, pol);
            tma_load_3d_pair(sQ + t * kQTile + kQTile / 2, &tm_q, lead_q_full, 64, x.h * G, tok, pol);
          }
        } else {
          ok = false;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      const int32_t* bt = a.block_tables + (size_t)x.b * a.bt_stride;
      const int nblk = (nkeys + bs - 1) / bs;
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
        int phys[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) phys[i] = __shfl_sync(0xffffffffu, cur, i);
        if (lane == 0) {
          const uint32_t par = ((uint32_t)(g / kStages) & 1u) ^ 1u;
          unsigned char* kst = sKV + (size_t)st * kStage;
          unsigned char* vst = kst + kKBytes;
          // boxes of kSub keys present in this step
          const int nvalid = min(nsub, (nkeys - s * kKeys + kSub - 1) / kSub);
          auto box_token = [&](int j) {  // first cache slot of box j of the step
            const int key = j * kSub;
            return phys[key / bs] * bs + key % bs;
          };
          if (!wait(&k_empty[st], par)) {
            ok = false;
          } else if (a.inject_stall && x.u == 0 && s == 0 && leader) {
            // test hook: the leader's first K half is never filled, so the MMA warp's wait runs out
          } else {
            // K: this CTA's 64 keys [64 rank, 64 rank + 64), both dim halves
            const int j0 = (int)rank * (nsub / 2), j1 = min(j0 + nsub / 2, nvalid);
            const uint32_t bytes = (uint32_t)max(0, j1 - j0) * (uint32_t)kSub * 128u * 2u;
            arrive_expect_tx_remote(peer_addr(&k_full[st], 0), bytes);
            for (int j = j0; j < j1; ++j) {
              const uint32_t row = (uint32_t)((j - j0) * kSub) * 128u;
              tma_load_3d_pair(kst + row, &tm_k, peer_addr(&k_full[st], 0), 0, x.h, box_token(j), pol);
              tma_load_3d_pair(kst + kKHalf + row, &tm_k, peer_addr(&k_full[st], 0), 64, x.h, box_token(j), pol);
            }
          }
          if (ok && !wait(&v_empty[st], par)) {
            ok = false;
          } else if (ok) {
            // V: dims [64 rank, 64 rank + 64) of all the step's keys
            const uint32_t bytes = (uint32_t)nvalid * (uint32_t)kSub * 128u;
            arrive_expect_tx_remote(peer_addr(&v_full[st], 0), bytes);
            for (int j = 0; j < nvalid; ++j)
              tma_load_3d_pair(vst + (uint32_t)(j * kSub) * 128u, &tm_v, peer_addr(&v_full[st], 0), 64 * (int)rank,
                               x.h, box_token(j), pol);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        cur = nxt;
      }
      ++ui;
    }
    // Both CTAs' copies complete on the leader's barriers: on a normal run
    // the MMA thread has waited for all of them; after an abort the leader
    // waits here (bounded) for the last ring of steps and the last Q, so no
    // copy lands after the pair leaves (the peer leaves with the leader).
    if (leader && lane == 0) {
      for (int t = max(0, g - kStages); t < g; ++t) {
        for (uint32_t i = 0; i < a.wait_limit; ++i)
          if (try_wait_cluster(&k_full[t % kStages], (uint32_t)(t / kStages) & 1u)) break;
        for (uint32_t i = 0; i < a.wait_limit; ++i)
          if (try_wait_cluster(&v_full[t % kStages], (uint32_t)(t / kStages) & 1u)) break;
      }
      if (ui > 0)
        for (uint32_t i = 0; i < a.wait_limit; ++i)
          if (try_wait_cluster(&q_full, (uint32_t)(ui - 1) & 1u)) break;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (leader && lane == 0) {
      const uint32_t idesc_s = f16_idesc(bf16, 2 * kRows, kKeys, 0);
      const uint32_t idesc_pv = f16_idesc(bf16, 2 * kRows, kD, 1);
      int ui = 0, g = 0;
      int pc[2] = {0, 0}, uc[2] = {0, 0};
      bool ok = true;
      auto issue_s = [&](int t, int s) -> bool {
        const int st = (g + s) % kStages;
        if (!wait(&k_full[st], (uint32_t)((g + s) / kStages) & 1u)) return false;
        tc_fence_after();
        mark(ui, s, 6);
        const uint32_t qa = smem_u32(sQ + t * kQTile), ka = smem_u32(sKV + (size_t)st * kStage);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_pair_ss(tmem + kTmemS + 128u * t, sw128_kmajor_desc(qa + c * (kQTile / 2)) + 2 * k,
                         sw128_kmajor_desc(ka + c * kKHalf) + 2 * k, idesc_s, (c | k) ? 1u : 0u);
        commit_both(&s_full[t]);
        return true;
      };
      auto issue_pv = [&](int t, int s) -> bool {
        const int st = (g + s) % kStages;
        if (!wait(&p_full[t], (uint32_t)pc[t] & 1u)) return false;
        if (!wait(&v_full[st], (uint32_t)((g + s) / kStages) & 1u)) return false;
        if (s == 0 && !wait(&o_empty[t], ((uint32_t)uc[t] & 1u) ^ 1u)) return false;
        tc_fence_after();
        mark(ui, s, t == 0 ? 9 : 7);
        const uint32_t va = smem_u32(sKV + (size_t)st * kStage + kKBytes);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_pair_ts(tmem + kTmemO + 128u * t, tmem + kTmemS + 128u * t + (uint32_t)(8 * k),
                       sw128_mnmajor_desc(va + (uint32_t)(16 * k) * 128u, kVBytes, 1024), idesc_pv,
                       (s == 0 && k == 0) ? 0u : 1u);
        commit_both(&pv_done[t]);
        ++pc[t];
        return true;
      };
      while (ok) {
        const int uk = ui & 1;
        if (!wait(&ufull[uk], (uint32_t)(ui >> 1) & 1u)) break;
        const QuadUnit x = slots[uk];
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
            if (ok) commit_both(&v_empty[(g + s - 1) % kStages]);  // V(s-1): B's P.V is its last reader
          }
          if (ok && s < nB) {
            if (s >= nA && !wait(&k_full[st], (uint32_t)((g + s) / kStages) & 1u)) ok = false;
            if (ok) {
              tc_fence_after();
              mark(ui, s, 8);
              const uint32_t qa = smem_u32(sQ + kQTile), ka = smem_u32(sKV + (size_t)st * kStage);
#pragma unroll
              for (int c = 0; c < 2; ++c)
#pragma unroll
                for (int k = 0; k < 4; ++k)
                  umma_pair_ss(tmem + kTmemS + 128u, sw128_kmajor_desc(qa + c * (kQTile / 2)) + 2 * k,
                               sw128_kmajor_desc(ka + c * kKHalf) + 2 * k, idesc_s, (c | k) ? 1u : 0u);
              commit_both(&s_full[1]);
            }
          }
          if (ok && s < ns) {
            commit_both(&k_empty[st]);  // K(s) is free once the S MMAs above complete
            if (s == ns - 1) commit_both(&q_empty);
          }
          if (ok && s < nA) {
            ok = issue_pv(0, s);
            if (ok && s >= nB) commit_both(&v_empty[st]);
          }
        }
        if (nA > 0) ++uc[0];
        if (nB > 0) ++uc[1];
        g += ns;
        ++ui;
      }
      // every MMA issued has completed before the tensor memory is released
      commit_local(&drain);
      for (uint32_t i = 0; i < a.wait_limit; ++i)
        if (mbar_try_wait(&drain, 0)) break;
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax + epilogue (both CTAs)
    const int t = (warp - 2) >> 2;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t sreg = tmem + lane_off + kTmemS + 128u * t;
    const uint32_t oreg = tmem + lane_off + kTmemO + 128u * t;
    const int t_in = r / G, gq = r - (r / G) * G;
    const uint32_t lead_p_full = peer_addr(&p_full[t], 0), lead_o_empty = peer_addr(&o_empty[t], 0);
    int ui = 0, g = 0, sc = 0, pc = 0;
    uint32_t zpar = 0;  // per stage: parity of the next v_landed phase (zeroing steps seen)
    auto wait_w = [&](uint64_t* bar, uint32_t parity) -> bool {
      const bool r = wait(bar, parity);
      return __all_sync(0xffffffffu, r ? 1 : 0) != 0;
    };
    auto pv_wait = [&](int i) -> bool { return i < 0 || wait_w(&pv_done[t], (uint32_t)i & 1u); };
    bool ok = true;
    while (ok) {
      const int uk = ui & 1;
      if (!wait_w(&ufull[uk], (uint32_t)(ui >> 1) & 1u)) break;
      const QuadUnit x = slots[uk];
      __syncwarp();
      if (lane == 0) arrive_remote(peer_addr(&uempty[uk], 0));
      if (!x.valid) break;
      const int ns_all = max(x.ns[0], x.ns[1]);
      const int nk_all = max(x.nk[0], x.nk[1]);
      const int nsteps = x.ns[t];
      // a unit whose last step holds keys past nk_all completes one v_landed
      // phase on that step's stage: every thread counts it, whichever tiles run
      const int zst = (g + ns_all - 1) % kStages;
      const uint32_t zp = (zpar >> zst) & 1u;
      if (ns_all * kKeys > nk_all) zpar ^= 1u << zst;
      if (nsteps == 0) {
        g += ns_all;
        ++ui;
        continue;
      }
      const int seq0 = __ldg(a.cu_seqlens + x.b);
      const int len = __ldg(a.cu_seqlens + x.b + 1) - seq0;
      const int tok0 = (4 * x.jq + 2 * t + (int)rank) * TQ;
      const int ntq = min(TQ, len - tok0);  // may be <= 0: this CTA's tile is empty, its rows are never stored
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
        for (int i = 0; i < 8; ++i) tmem_ld16f(sreg + 16u * i, v + 16 * i);
        tmem_wait_ld();
        if ((warp & 3) == 0 && lane == 0) mark(ui, s, 3 * t + 1);
        const int key0 = s * kKeys;
        if (key0 + kKeys - 1 > pos) {  // the causal mask, only on steps that reach past the row's position
#pragma unroll
          for (int k = 0; k < 128; ++k) v[k] = key0 + k <= pos ? v[k] : -INFINITY;
        }
        float mx = row_max128(v);
        mx *= a.qscale;
        const bool move = mx > m + 8.f;
        const float m_new = move ? mx : m;
        const float ref = m_new == -INFINITY ? 0.f : m_new;
        const float corr = move ? exp2f(m - ref) : 1.f;
        const float rs = row_exp2_sum128(v, a.qscale, ref);
        l = l * corr + rs;
        const bool rescale = move && s > 0 && m != -INFINITY;
        m = m_new;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t pk[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) pk[k] = pack_pair<T>(v[32 * i + 2 * k], v[32 * i + 2 * k + 1]);
          tmem_st16u(sreg + 16u * i, pk);
        }
        if (__any_sync(0xffffffffu, rescale ? 1 : 0)) {
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
          // V rows past the unit's last key may hold any bits: zero this
          // CTA's half of them once the copies landed (thread r: key row r)
          // The copies complete on the leader's v_full: the leader waits for
          // them and tells the peer through v_landed (one arrival, from the
          // first of the pair's tiles that reaches this last step).
          const int st = (g + s) % kStages;
          bool landed;
          if (leader) {
            landed = wait_w(&v_full[st], (uint32_t)((g + s) / kStages) & 1u);
            const int signal_tile = x.ns[0] == ns_all ? 0 : 1;
            if (landed && t == signal_tile && r == 0) arrive_remote(peer_addr(&v_landed[st], 1));
          } else {
            landed = wait_w(&v_landed[st], zp);
          }
          if (!landed) {
            ok = false;
            break;
          }
          if (s * kKeys + r >= nk_all) {
            unsigned char* vst = sKV + (size_t)st * kStage + kKBytes + (size_t)r * 128;
#pragma unroll
            for (int u = 0; u < 8; ++u) *reinterpret_cast<uint4*>(vst + u * 16) = make_uint4(0, 0, 0, 0);
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        tc_fence_before();
        if ((warp & 3) == 0 && lane == 0) mark(ui, s, 3 * t + 2);
        // each lane's P stores (and V zeroing) are fenced above; the warp
        // meets, then one lane arrives for it
        __syncwarp();
        if (lane == 0) arrive_remote(lead_p_full);
        ++pc;
      }
      if (!ok) break;
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
        __syncwarp();
        if (lane == 0) arrive_remote(lead_o_empty);
      }
      g += ns_all;
      ++ui;
    }
  }
  // Both CTAs leave together: the leader's MMAs (which read the peer's shared
  // and tensor memory) have drained, and no remote arrival is in flight.
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if constexpr (kTrace) {
    if (a.trace && threadIdx.x == 0) a.trace[16 + 16 * 32 * 16 + 2 * blockIdx.x + 1] = gtime();
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

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

// Plan (longest-first list over quads of tiles) + the 2-CTA kernel; same
// arguments and shape coverage as launch_prefill_tc.
int launch_prefill_tc2(const clove_pool& pool, const void* q_rot, float* out, const int32_t* cu_seqlens,
                       const int32_t* context_lens, const int32_t* block_tables, int bt_stride, int batch,
                       int num_tokens, int num_q_heads, float scale, int max_ctx, void* ws, cudaStream_t stream, int phase) {
  const int group = num_q_heads / pool.num_kv_heads;
  const int tq = kRows / group;
  CUtensorMap tm_q, tm_k, tm_v;
  const long long slots = (long long)pool.num_blocks * pool.block_size;
  const int sub = std::min(pool.block_size, 64);
  int rc = encode_map(&tm_q, q_rot, pool.dtype, num_tokens, num_q_heads, group, tq);
  if (!rc) rc = encode_map(&tm_k, pool.k_cache, pool.dtype, slots, pool.num_kv_heads, 1, sub);
  if (!rc) rc = encode_map(&tm_v, pool.v_cache, pool.dtype, slots, pool.num_kv_heads, 1, sub);
  if (rc) return rc;
  unsigned char* w = static_cast<unsigned char*>(ws);
  PrefillArgs a{};
  a.q = q_rot;
  a.out = out;
  a.cu_seqlens = cu_seqlens;
  a.context_lens = context_lens;
  a.block_tables = block_tables;
  a.items = reinterpret_cast<int2*>(w + 512);
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
  a.tq = 4 * tq;  // the plan lists quads of tiles
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
  auto kern = bf16 ? prefill_tc2_kernel<__nv_bfloat16> : prefill_tc2_kernel<__half>;
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
  cfg.gridDim = dim3((unsigned)(pool.num_sms & ~1));
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
    set_last_error("paged_prefill (tcgen05, 2-CTA) launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(1);
  return CLOVE_OK;
}

}  // namespace clove
