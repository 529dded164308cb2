// Tensor-core prefill attention over the paged cache (bf16 / f16, head_dim
// 64 or 128, up to 16 query heads per KV head).
//
// FlashAttention-2 structure on the paged layout.  A work unit is (sequence
// b, tile of TQ prompt tokens, KV head h): 64 query rows = (token, query
// head) pairs of that KV head, TQ = 64 / group tokens.  A producer warp
// streams the sequence's K/V tiles for keys 0 .. (last position of the tile)
// into a shared-memory ring (one 4-D 128-byte-swizzled bulk copy per block
// and plane); each of the 4 consumer warps owns 16 query rows and consumes
// every stage: S = Q K^T with m16n8k16 MMAs (all 16 rows real), the causal
// mask key <= position(row), an fp32 online softmax per row, O += P V.  Rows
// are finished by their own warp, so there is no cross-warp merge.  Units
// are claimed longest-first (key count) with an atomic counter.
//
// Semantics: the reference's FlashAttention step (src/lazy.rs:4821-4923),
// causal, on RoPE-rotated q and k (the prep kernel in prefill.cu rotates
// them and writes K/V into the cache), scale 1/sqrt(head_dim), exact
// exponential.
#include "common.cuh"
#include "decode_common.cuh"
#include "host.h"
#include "mma_common.cuh"
#include "prefill_common.cuh"

namespace clove {

constexpr int kPfNCW = 4;      // consumer warps, 16 query rows each
constexpr int kPfRows = 64;    // query rows per unit

// Work list: every (sequence, token tile), ordered by key count (context +
// tile end) descending through a counting sort over kPfBins bins.
__global__ void __launch_bounds__(1024) prefill_plan_kernel(PrefillArgs p) {
  __shared__ int hist[kPfBins];
  __shared__ int base[kPfBins];
  __shared__ int s_maxk;
  const int tid = threadIdx.x;
  for (int i = tid; i < kPfBins; i += blockDim.x) hist[i] = 0;
  if (tid == 0) {
    s_maxk = 1;
    *p.unit_counter = 0;
  }
  __syncthreads();
  auto keys_of = [&](int b, int j, int len, int ctx) { return ctx + min((j + 1) * p.tq, len); };
  for (int b = tid; b < p.batch; b += blockDim.x) {
    const int len = p.cu_seqlens[b + 1] - p.cu_seqlens[b];
    if (len > 0) atomicMax(&s_maxk, p.context_lens[b] + len);
  }
  __syncthreads();
  const int maxk = s_maxk;
  // a sequence's tiles are spread over all threads (few long prompts are
  // the common prefill batch)
  for (int b = 0; b < p.batch; ++b) {
    const int len = __ldg(p.cu_seqlens + b + 1) - __ldg(p.cu_seqlens + b), ctx = __ldg(p.context_lens + b);
    for (int j = tid; j * p.tq < len; j += blockDim.x)
      atomicAdd(&hist[(int)((long long)(keys_of(b, j, len, ctx) - 1) * kPfBins / maxk)], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int bin = kPfBins - 1; bin >= 0; --bin) {
      base[bin] = acc;
      acc += hist[bin];
      hist[bin] = 0;
    }
    *p.n_items = acc;
  }
  __syncthreads();
  for (int b = 0; b < p.batch; ++b) {
    const int len = __ldg(p.cu_seqlens + b + 1) - __ldg(p.cu_seqlens + b), ctx = __ldg(p.context_lens + b);
    for (int j = tid; j * p.tq < len; j += blockDim.x) {
      const int bin = (int)((long long)(keys_of(b, j, len, ctx) - 1) * kPfBins / maxk);
      p.items[base[bin] + atomicAdd(&hist[bin], 1)] = make_int2(b, j);
    }
  }
}

struct PfUnit {
  int b, j, h, nkeys, valid;
};

struct PfSmem {
  unsigned char* ring;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* ufull;
  uint64_t* uempty;
  volatile int* abort;
  PfUnit* slots;
};

__host__ __device__ inline int pf_tile_stride(int bs, int D, int eb) { return (bs * D * eb + 1023) & ~1023; }
__host__ __device__ inline int pf_stage_bytes(int bs, int D, int eb, int sb) { return 2 * sb * pf_tile_stride(bs, D, eb); }
__host__ __device__ inline int pf_smem_bytes(int bs, int D, int eb, int sb, int nstage) {
  return pf_stage_bytes(bs, D, eb, sb) * nstage + 1024 /* barriers, slots */ + 1024 /* alignment */;
}

__device__ __forceinline__ PfSmem pf_smem(unsigned char* base, int stage_bytes, int nstage) {
  PfSmem s;
  s.ring = base;
  s.full = reinterpret_cast<uint64_t*>(base + (size_t)stage_bytes * nstage);
  s.empty = s.full + nstage;
  s.ufull = s.empty + nstage;
  s.uempty = s.ufull + 2;
  s.abort = reinterpret_cast<volatile int*>(s.uempty + 2);
  s.slots = reinterpret_cast<PfUnit*>(s.uempty + 4);
  return s;
}

__device__ __forceinline__ bool pf_wait(const PrefillArgs& a, const PfSmem& sm, uint64_t* bar, uint32_t parity) {
  if (*sm.abort || !mbar_wait_bounded(bar, parity, a.err, a.wait_limit)) {
    *sm.abort = 1;
    return false;
  }
  return true;
}

// Producer warp: claim units, post them, stream their K/V tiles.
template <typename T, int D>
__device__ void pf_produce(const PrefillArgs& a, const CUtensorMap* tm_k, const CUtensorMap* tm_v, const PfSmem& sm,
                           int stage_bytes, int tile_stride, int n_units) {
  const int lane = threadIdx.x & 31;
  const int bs = a.bs, sb = a.sb;
  const uint32_t tile_bytes = (uint32_t)(bs * D * (int)sizeof(T));
  const uint64_t pol = policy_evict_first();
  int slot = 0, uk = 0;
  uint32_t phase = 0, uphase = 0;
  bool aborted = false;
  while (!aborted) {
    int u = 0;
    if (lane == 0) u = atomicAdd(a.unit_counter, 1);
    u = __shfl_sync(0xffffffffu, u, 0);
    PfUnit x;
    x.valid = u < n_units;
    if (x.valid) {
      const int2 it = a.items[u / a.hkv];
      x.b = it.x;
      x.j = it.y;
      x.h = u - (u / a.hkv) * a.hkv;
      const int len = __ldg(a.cu_seqlens + x.b + 1) - __ldg(a.cu_seqlens + x.b);
      x.nkeys = __ldg(a.context_lens + x.b) + min((x.j + 1) * a.tq, len);
    }
    int ok = 1;
    if (lane == 0) {
      if (!pf_wait(a, sm, &sm.uempty[uk], uphase ^ 1)) {
        ok = 0;
      } else {
        sm.slots[uk] = x;
        mbar_arrive(&sm.ufull[uk]);
      }
    }
    if (!__shfl_sync(0xffffffffu, ok, 0)) {
      aborted = true;
      break;
    }
    if (++uk == 2) {
      uk = 0;
      uphase ^= 1;
    }
    if (!x.valid) break;
    const int nblk = (x.nkeys + bs - 1) / bs;
    const int nst = (nblk + sb - 1) / sb;
    const int32_t* bt = a.block_tables + (size_t)x.b * a.bt_stride;
    int my = 0;
    for (int s = 0; s < nst && !aborted; ++s) {
      const int j0 = s * sb;
      if ((j0 & 31) == 0) {
        const bool in = j0 + lane < nblk;
        my = in ? __ldg(bt + j0 + lane) : 0;
        if (in && (my < 0 || my >= a.num_blocks)) {
          atomicOr(a.err, CLOVE_FLAG_BLOCK_OOB);
          my = 0;
        }
      }
      const int nb = min(sb, nblk - j0);
      int phys[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) phys[i] = __shfl_sync(0xffffffffu, my, (j0 + i) & 31);
      ok = 1;
      if (lane == 0) {
        if (!pf_wait(a, sm, &sm.empty[slot], phase ^ 1)) {
          ok = 0;
        } else {
          mbar_arrive_expect_tx(&sm.full[slot], 2u * tile_bytes * (uint32_t)nb);
          unsigned char* st = sm.ring + (size_t)slot * stage_bytes;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (i < nb) {
              tma_load_4d(st + i * tile_stride, tm_k, &sm.full[slot], 0, 0, x.h, phys[i] * bs, pol);
              tma_load_4d(st + (sb + i) * tile_stride, tm_v, &sm.full[slot], 0, 0, x.h, phys[i] * bs, pol);
            }
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) aborted = true;
      if (++slot == a.nstage) {
        slot = 0;
        phase ^= 1;
      }
    }
  }
  if (aborted && lane == 0) {  // drain the copies of the last nstage issues
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
  }
}

// The kernel: warp 0 produces, warps 1..4 each own 16 query rows of a unit.
template <typename T, int D>
__global__ void __launch_bounds__((kPfNCW + 1) * 32, 2)
    prefill_mma_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                       const PrefillArgs a) {
  constexpr int KS = D / 16;  // k-steps of QK^T
  constexpr int NT = D / 8;   // n-tiles of P.V
  constexpr int NH = D / 64;  // 128-byte rows per token in a swizzled tile
  const int bs = a.bs, sb = a.sb;
  const int TT = sb * bs;     // keys per stage (a multiple of 32)
  const int tile_stride = pf_tile_stride(bs, D, (int)sizeof(T));
  const int stage_bytes = pf_stage_bytes(bs, D, (int)sizeof(T), sb);

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const PfSmem sm = pf_smem(smem, stage_bytes, a.nstage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.nstage; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kPfNCW);
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(&sm.ufull[k], 1);
      mbar_init(&sm.uempty[k], kPfNCW);
    }
    *sm.abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the plan kernel's list
  const int n_units = *a.n_items * a.hkv;
  if (warp == 0) {
    pf_produce<T, D>(a, &tm_k, &tm_v, sm, stage_bytes, tile_stride, n_units);
    return;
  }

  const int cw = warp - 1;
  const int gq = lane >> 2, tq = lane & 3;  // fragment row / column pair
  const int mi = lane >> 3, mr = lane & 7;  // ldmatrix matrix / row
  const int G = a.group;
  // this lane's two rows of the warp's 16: r_lo = 16 cw + gq, r_hi = r_lo + 8
  const int r_lo = 16 * cw + gq, r_hi = r_lo + 8;
  const int ti_lo = r_lo / G, gi_lo = r_lo - ti_lo * G;
  const int ti_hi = r_hi / G, gi_hi = r_hi - ti_hi * G;
  const int warp_last_tok = (16 * cw + 15) / G;
  int uk = 0, gs = 0;
  uint32_t uphase = 0;

  while (true) {
    if (!pf_wait(a, sm, &sm.ufull[uk], uphase)) return;
    const PfUnit x = sm.slots[uk];
    if (!x.valid) return;
    const int seq0 = __ldg(a.cu_seqlens + x.b);
    const int len = __ldg(a.cu_seqlens + x.b + 1) - seq0;
    const int ntq = min(a.tq, len - x.j * a.tq);             // tokens in this tile
    const int pos0 = __ldg(a.context_lens + x.b) + x.j * a.tq;  // position of its first token
    const bool v_lo = ti_lo < ntq && r_lo < a.tq * G, v_hi = ti_hi < ntq && r_hi < a.tq * G;
    const int p_lo = v_lo ? pos0 + ti_lo : -1, p_hi = v_hi ? pos0 + ti_hi : -1;
    const int kmax = min(ntq - 1, warp_last_tok) + pos0;  // last key any row of this warp needs
    const bool warp_live = 16 * cw < ntq * G;
    // Q fragments (full 16-row A operand), unscaled
    uint32_t qa[KS][4];
    {
      const T* q_lo = static_cast<const T*>(a.q) + ((size_t)(seq0 + x.j * a.tq + ti_lo) * a.hq + x.h * G + gi_lo) * D;
      const T* q_hi = static_cast<const T*>(a.q) + ((size_t)(seq0 + x.j * a.tq + ti_hi) * a.hq + x.h * G + gi_hi) * D;
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        qa[k][0] = v_lo ? *reinterpret_cast<const uint32_t*>(q_lo + k * 16 + 2 * tq) : 0u;
        qa[k][1] = v_hi ? *reinterpret_cast<const uint32_t*>(q_hi + k * 16 + 2 * tq) : 0u;
        qa[k][2] = v_lo ? *reinterpret_cast<const uint32_t*>(q_lo + k * 16 + 8 + 2 * tq) : 0u;
        qa[k][3] = v_hi ? *reinterpret_cast<const uint32_t*>(q_hi + k * 16 + 8 + 2 * tq) : 0u;
      }
    }
    float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

    const int nblk = (x.nkeys + bs - 1) / bs;
    const int nst = (nblk + sb - 1) / sb;
    for (int s = 0; s < nst; ++s, ++gs) {
      const int slot = gs % a.nstage;
      if (!pf_wait(a, sm, &sm.full[slot], (uint32_t)(gs / a.nstage) & 1u)) return;
      const int k0 = s * TT;  // key index of the stage's first token
      if (warp_live && k0 <= kmax) {
        const uint32_t kbase = smem_u32(sm.ring + (size_t)slot * stage_bytes);
        const uint32_t vbase = kbase + (uint32_t)(sb * tile_stride);
        for (int p0 = 0; p0 < TT && k0 + p0 <= kmax; p0 += 32) {
          uint32_t krow[2], vrow[2];
          int kr[2], vr[2];
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int tk_k = p0 + 16 * h2 + (mi >> 1) * 8 + mr, tk_v = p0 + 16 * h2 + (mi & 1) * 8 + mr;
            const int bk = tk_k / bs, rk = tk_k - bk * bs, bv = tk_v / bs, rv = tk_v - bv * bs;
            kr[h2] = rk * NH;
            vr[h2] = rv * NH;
            krow[h2] = kbase + (uint32_t)(bk * tile_stride + kr[h2] * 128);
            vrow[h2] = vbase + (uint32_t)(bv * tile_stride + vr[h2] * 128);
          }
          const uint32_t kc = (uint32_t)(mi & 1), vc = (uint32_t)(mi >> 1);
          // ---- S = Q K^T over 32 keys: 4 n-tiles ----
          float sacc[4][4];
#pragma unroll
          for (int jn = 0; jn < 4; ++jn) sacc[jn][0] = sacc[jn][1] = sacc[jn][2] = sacc[jn][3] = 0.f;
#pragma unroll
          for (int k = 0; k < KS; ++k) {
            const int hb = k >> 2;
            uint32_t b0[4], b1[4];
            ldsm_x4(krow[0] + hb * 128 + (((((uint32_t)(2 * k) & 7u) + kc) ^ (uint32_t)((kr[0] + hb) & 7)) << 4), b0);
            ldsm_x4(krow[1] + hb * 128 + (((((uint32_t)(2 * k) & 7u) + kc) ^ (uint32_t)((kr[1] + hb) & 7)) << 4), b1);
            mma16816_full<T>(sacc[0], qa[k][0], qa[k][1], qa[k][2], qa[k][3], b0[0], b0[1]);
            mma16816_full<T>(sacc[1], qa[k][0], qa[k][1], qa[k][2], qa[k][3], b0[2], b0[3]);
            mma16816_full<T>(sacc[2], qa[k][0], qa[k][1], qa[k][2], qa[k][3], b1[0], b1[1]);
            mma16816_full<T>(sacc[3], qa[k][0], qa[k][1], qa[k][2], qa[k][3], b1[2], b1[3]);
          }
          // ---- causal mask + online softmax, rows lo (values 0,1) and hi (values 2,3) ----
          float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
          for (int jn = 0; jn < 4; ++jn) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int key = k0 + p0 + 8 * jn + 2 * tq + e;
              sacc[jn][e] = key <= p_lo ? sacc[jn][e] * a.qscale : -INFINITY;
              sacc[jn][2 + e] = key <= p_hi ? sacc[jn][2 + e] * a.qscale : -INFINITY;
              mx_lo = fmaxf(mx_lo, sacc[jn][e]);
              mx_hi = fmaxf(mx_hi, sacc[jn][2 + e]);
            }
          }
          mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
          mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
          mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
          mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
          const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
          // rows with no visible key yet keep m = -inf: use 0 as the reference
          const float rf_lo = mn_lo == -INFINITY ? 0.f : mn_lo, rf_hi = mn_hi == -INFINITY ? 0.f : mn_hi;
          const float c_lo = exp2f(m_lo - rf_lo), c_hi = exp2f(m_hi - rf_hi);
          m_lo = mn_lo;
          m_hi = mn_hi;
          float s_lo = 0.f, s_hi = 0.f;
#pragma unroll
          for (int jn = 0; jn < 4; ++jn) {
            sacc[jn][0] = exp2f(sacc[jn][0] - rf_lo);
            sacc[jn][1] = exp2f(sacc[jn][1] - rf_lo);
            sacc[jn][2] = exp2f(sacc[jn][2] - rf_hi);
            sacc[jn][3] = exp2f(sacc[jn][3] - rf_hi);
            s_lo += sacc[jn][0] + sacc[jn][1];
            s_hi += sacc[jn][2] + sacc[jn][3];
          }
          l_lo = l_lo * c_lo + s_lo;
          l_hi = l_hi * c_hi + s_hi;
#pragma unroll
          for (int n = 0; n < NT; ++n) {
            o[n][0] *= c_lo;
            o[n][1] *= c_lo;
            o[n][2] *= c_hi;
            o[n][3] *= c_hi;
          }
          // A operands of P.V: k-tile 0 = keys p0 .. p0+15 (n-tiles 0, 1), k-tile 1 = n-tiles 2, 3
          uint32_t pa[2][4];
#pragma unroll
          for (int kt = 0; kt < 2; ++kt) {
            pa[kt][0] = MmaType<T>::pack(sacc[2 * kt][0], sacc[2 * kt][1]);
            pa[kt][1] = MmaType<T>::pack(sacc[2 * kt][2], sacc[2 * kt][3]);
            pa[kt][2] = MmaType<T>::pack(sacc[2 * kt + 1][0], sacc[2 * kt + 1][1]);
            pa[kt][3] = MmaType<T>::pack(sacc[2 * kt + 1][2], sacc[2 * kt + 1][3]);
          }
          // V rows at or past nkeys may hold any bits: P is 0 there, but 0 * NaN
          // is NaN inside the MMA, so zero those halves of the B fragments.
          const bool tail = k0 + p0 + 32 > x.nkeys;
#pragma unroll
          for (int n = 0; n < NT; n += 2) {
            const int hb = n >> 3;
            uint32_t b[2][4];
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              ldsm_x4_trans(vrow[h2] + hb * 128 + (((((uint32_t)n & 7u) + vc) ^ (uint32_t)((vr[h2] + hb) & 7)) << 4),
                            b[h2]);
              if (tail) {
                // register i: keys p0 + 16*h2 + (i & 1) * 8 + 2*tq + {0, 1}
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const int key = k0 + p0 + 16 * h2 + (i & 1) * 8 + 2 * tq;
                  if (key >= x.nkeys) b[h2][i] &= 0xffff0000u;
                  if (key + 1 >= x.nkeys) b[h2][i] &= 0x0000ffffu;
                }
              }
            }
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              mma16816_full<T>(o[n], pa[h2][0], pa[h2][1], pa[h2][2], pa[h2][3], b[h2][0], b[h2][1]);
              mma16816_full<T>(o[n + 1], pa[h2][0], pa[h2][1], pa[h2][2], pa[h2][3], b[h2][2], b[h2][3]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[slot]);
    }
    // ---- finish this warp's rows ----
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
    const float inv_lo = 1.f / l_lo, inv_hi = 1.f / l_hi;
    float* out_lo = a.out + ((size_t)(seq0 + x.j * a.tq + ti_lo) * a.hq + x.h * G + gi_lo) * D;
    float* out_hi = a.out + ((size_t)(seq0 + x.j * a.tq + ti_hi) * a.hq + x.h * G + gi_hi) * D;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      if (v_lo) *reinterpret_cast<float2*>(out_lo + n * 8 + 2 * tq) = make_float2(o[n][0] * inv_lo, o[n][1] * inv_lo);
      if (v_hi) *reinterpret_cast<float2*>(out_hi + n * 8 + 2 * tq) = make_float2(o[n][2] * inv_hi, o[n][3] * inv_hi);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.uempty[uk]);
    if (++uk == 2) {
      uk = 0;
      uphase ^= 1;
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
constexpr int kPfRingTarget = 96 * 1024;

template <typename T, int D>
static int run_prefill(const clove_pool& pool, PrefillArgs& a, cudaStream_t stream) {
  auto kern = prefill_mma_kernel<T, D>;
  const int eb = (int)sizeof(T);
  int nstage = kPfRingTarget / pf_stage_bytes(a.bs, D, eb, a.sb);
  if (nstage < 2) nstage = 2;
  a.nstage = nstage;
  const int smem = pf_smem_bytes(a.bs, D, eb, a.sb, nstage);
  if (smem > 227 * 1024) {
    set_last_error("paged_prefill: tile does not fit shared memory");
    return CLOVE_ERR_UNSUPPORTED;
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    set_last_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, (kPfNCW + 1) * 32, smem) != cudaSuccess || occ < 1)
    occ = 1;
  e = launch_dependent(kern, (unsigned)(pool.num_sms * occ), (kPfNCW + 1) * 32, smem, stream, pool.tm_k_sw,
                       pool.tm_v_sw, a);
  if (e != cudaSuccess) {
    set_last_error("paged_prefill launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(1);
  return CLOVE_OK;
}

size_t prefill_mma_scratch_bytes(int num_tokens) { return 512 + sizeof(int2) * (size_t)num_tokens; }

// Tensor-core prefill of already rotated queries (q_rot) over a cache that
// already holds the prompt's K/V.  ws: scratch of at least
// prefill_mma_scratch_bytes(num_tokens) bytes.  Returns CLOVE_ERR_UNSUPPORTED
// (nothing launched) when the shape is not covered.
int launch_prefill_mma(const clove_pool& pool, const void* q_rot, float* out, const int32_t* cu_seqlens,
                       const int32_t* context_lens, const int32_t* block_tables, int bt_stride, int batch,
                       int num_tokens, int num_q_heads, float scale, int max_ctx, void* ws, cudaStream_t stream) {
  const int group = num_q_heads / pool.num_kv_heads;
  if (pool.elem_bytes != 2 || !pool.has_swizzled || pool.block_size < 8 || group > 16 ||
      (pool.head_dim != 64 && pool.head_dim != 128))
    return CLOVE_ERR_UNSUPPORTED;
  unsigned char* w = static_cast<unsigned char*>(ws);
  PrefillArgs a{};
  a.q = q_rot;
  a.out = out;
  a.cu_seqlens = cu_seqlens;
  a.context_lens = context_lens;
  a.block_tables = block_tables;
  a.items = reinterpret_cast<int2*>(w + 512);  // tiles <= num_tokens
  a.n_items = reinterpret_cast<int32_t*>(w + 256);
  a.unit_counter = reinterpret_cast<int32_t*>(w + 256) + 2;
  a.err = reinterpret_cast<int32_t*>(w);
  a.bt_stride = bt_stride;
  a.batch = batch;
  a.hq = num_q_heads;
  a.hkv = pool.num_kv_heads;
  a.group = group;
  a.bs = pool.block_size;
  a.num_blocks = pool.num_blocks;
  a.tq = kPfRows / group;
  a.sb = pool.block_size >= 32 ? 1 : 32 / pool.block_size;
  a.max_ctx = max_ctx;
  a.wait_limit = debug_wait_limit();
  a.qscale = scale * kLog2e;
  a.nstage = 2;
  cudaMemsetAsync(a.err, 0, sizeof(int32_t), stream);
  prefill_plan_kernel<<<1, 1024, 0, stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("prefill plan launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(1);
  const bool bf16 = pool.dtype == CLOVE_DTYPE_BF16;
  if (pool.head_dim == 64)
    return bf16 ? run_prefill<__nv_bfloat16, 64>(pool, a, stream) : run_prefill<__half, 64>(pool, a, stream);
  return bf16 ? run_prefill<__nv_bfloat16, 128>(pool, a, stream) : run_prefill<__half, 128>(pool, a, stream);
}

}  // namespace clove
