// Tensor-core decode consumer for 16-bit KV (bf16 / f16) and GQA groups of
// 4..8 query heads per KV head, head_dim 64 or 128.
//
// Why tensor cores here: with a group of G query heads every K/V element
// feeds G multiply-adds in QK^T and again in P.V, 2G flop per byte for
// 16-bit data; at HBM speed (~6.5 TB/s) a group of 8 needs ~100 TFLOP/s,
// beyond what the CUDA cores sustain next to the softmax.  The query rows of
// one KV head form a real (if short) dense tile, so a warp-level
// m16n8k16 MMA handles them: M = 16 query rows (G real, the rest zero),
// N = 8 tokens (QK^T) or 8 dims (P.V), K = 16 dims (QK^T) or 16 tokens (P.V).
// The score fragment of QK^T is, register for register, the A operand of
// P.V, so probabilities never leave registers.
//
// Shared memory: each [block_size, head_dim] tile arrives as head_dim/64
// sub-tiles of [block_size, 64] elements (128-byte rows) written by the bulk
// tensor copy with the 128-byte swizzle: 16-byte chunk c of row r sits at
// chunk c ^ (r & 7).  ldmatrix reads (8 rows x 16 bytes per matrix) are then
// conflict-free.
//
// Pipeline, work units, ring-slot ownership and the epilogue are those of
// the CUDA-core kernel (decode_common.cuh).
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "decode_common.cuh"
#include "host.h"
#include "mma_common.cuh"
#include "mma_decode.cuh"

namespace clove {

// Byte offset, inside a stage's K (or V) region, of 16-byte chunk `ch`
// (head_dim / 8 chunks per token) of token `tok` (0 .. sb*block_size-1).
__device__ __forceinline__ uint32_t swz_off(int tok, int ch, int bs, int tile_stride, int nh) {
  const int blk = tok / bs, r = tok - blk * bs;
  const int row = r * nh + (ch >> 3);  // 128-byte row (token, 64-dim half) within the tile
  return (uint32_t)(blk * tile_stride + row * 128 + (((ch & 7) ^ (row & 7)) << 4));
}

// NCW consumer warps; D = 64 or 128.  Each consumer warp owns whole stages;
// per pass of 16 tokens: S = Q K^T (2 n-tiles x D/16 k-steps), online
// softmax on the score fragment, O += P V (D/8 n-tiles).
template <typename T, int D, int NCW>
__global__ void __launch_bounds__((NCW + 1) * 32)
    paged_decode_mma_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                            const DecodeArgs a) {
  constexpr int G = 8;              // rows of the per-KV-head query tile that can be real
  constexpr int KS = D / 16;        // k-steps of QK^T
  constexpr int NT = D / 8;         // n-tiles of P.V
  const int bs = a.block_size;
  const int sb = a.stage_blocks;
  const int TT = sb * bs;
  const int group = a.group;

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SmemPlan sp = smem_plan(bs, D, (int)sizeof(T), sb, a.nstage, NCW * group * state_stride(D) * (int)sizeof(float),
                                group * D * (int)sizeof(T), a.nscr);
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
    produce<T, D, 2>(a, &tm_k, &tm_v, sm, sp, sb, walk);
    return;
  }

  const int cw = warp - 1;
  const int g = lane >> 2;      // query row of this lane's fragment values
  const int tq = lane & 3;      // column pair within an 8-wide n-tile
  const int mi = lane >> 3;     // ldmatrix: which 8x8 matrix this lane addresses
  const int mr = lane & 7;      // ldmatrix: which row of it
  const float sl2 = a.qscale;   // scale * log2(e), applied to the f32 scores
  int gbase = 0;
  int uk = 0, n_done = 0;
  uint32_t uphase = 0;
  UnitSlot us;

  while (wait_unit(a, sm, uk, uphase, us)) {
    const Unit x = us.x;
    // Q fragments (A operand rows = query heads of this KV head), unscaled,
    // from the unit's query buffer.
    uint32_t qa[KS][2];
    {
      const T* qrow = reinterpret_cast<const T*>(sm.qbuf + uk * sp.q_stride) + g * D;
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        if (g < group) {
          qa[k][0] = *reinterpret_cast<const uint32_t*>(qrow + k * 16 + 2 * tq);
          qa[k][1] = *reinterpret_cast<const uint32_t*>(qrow + k * 16 + 8 + 2 * tq);
        } else {
          qa[k][0] = 0u;
          qa[k][1] = 0u;
        }
      }
    }
    float m = -INFINITY, l = 0.f;
    float o[NT][2];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = 0.f;

    bool aborted = false;
    const int ncw = a.ncw;
    // Stage ownership as in the CUDA-core kernel: stage gs -> warp gs % ncw.
    for (int j = cw < ncw ? ((cw - gbase) % ncw + ncw) % ncw : x.nstages; j < x.nstages; j += ncw) {
      const int gs = gbase + j;
      const int slot = gs % a.nstage;
      const uint32_t par = (uint32_t)(gs / a.nstage) & 1u;
      if (sm.misc[0] || !mbar_wait_bounded(&sm.full[slot], par, a.err, a.wait_limit)) {
        sm.misc[0] = 1;
        aborted = true;
        break;
      }
      unsigned char* kst = sm.ring + (size_t)slot * sp.stage_bytes;
      unsigned char* vst = kst + sb * sp.tile_stride;
      // tokens of this stage: up to the piece's end (a piece may end inside
      // a stage of sb blocks, before its sequence does) and the sequence's
      const int ntok = min(TT, min((x.blk0 + x.nblk) * bs, x.L) - (x.blk0 + j * sb) * bs);
      if (ntok < TT) {
        // Rows past the context may hold any bits (even NaN patterns); P is
        // zero there but 0 * NaN is NaN inside the MMA, so clear those V rows.
        for (int i = lane; i < (TT - ntok) * (D / 8); i += 32) {
          const int tok = ntok + i / (D / 8), ch = i % (D / 8);
          *reinterpret_cast<uint4*>(vst + swz_off(tok, ch, bs, sp.tile_stride, D / 64)) = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      const uint32_t kbase = smem_u32(kst), vbase = smem_u32(vst);
      constexpr int NH = D / 64;  // 128-byte rows per token
      for (int p0 = 0; p0 < ntok; p0 += 32) {
        // 32 tokens per pass, as two 16-token halves h = 0, 1.  Per-pass
        // ldmatrix row addresses: chunk ch of token tok lives at
        // tile_off(tok) + row * 128 + (((ch & 7) ^ (row & 7)) << 4), with
        // row = token_in_block * NH + (ch >> 3) (the layout of the 4-D box).
        uint32_t krow[2], vrow[2];
        int kr[2], vr[2];
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int tk_k = p0 + 16 * h2 + (mi >> 1) * 8 + mr, tk_v = p0 + 16 * h2 + (mi & 1) * 8 + mr;
          const int bk = tk_k / bs, rk = tk_k - bk * bs;
          const int bv = tk_v / bs, rv = tk_v - bv * bs;
          kr[h2] = rk * NH;
          vr[h2] = rv * NH;
          krow[h2] = kbase + (uint32_t)(bk * sp.tile_stride + kr[h2] * 128);
          vrow[h2] = vbase + (uint32_t)(bv * sp.tile_stride + vr[h2] * 128);
        }
        const uint32_t kc = (uint32_t)(mi & 1), vc = (uint32_t)(mi >> 1);
        // ---- S = Q K^T: 4 n-tiles of 8 tokens, 4 independent MMA chains ----
        float sacc[4][2];
#pragma unroll
        for (int j = 0; j < 4; ++j) sacc[j][0] = sacc[j][1] = 0.f;
#pragma unroll
        for (int k = 0; k < KS; ++k) {
          const int hb = k >> 2;  // which 64-dim half
          const uint32_t off = (uint32_t)(hb * 128);
          // matrices: (tok 0-7, d 0-7), (tok 0-7, d 8-15), (tok 8-15, d 0-7), (tok 8-15, d 8-15)
          uint32_t b0[4], b1[4];
          ldsm_x4(krow[0] + off + (((((uint32_t)(2 * k) & 7u) + kc) ^ (uint32_t)((kr[0] + hb) & 7)) << 4), b0);
          ldsm_x4(krow[1] + off + (((((uint32_t)(2 * k) & 7u) + kc) ^ (uint32_t)((kr[1] + hb) & 7)) << 4), b1);
          mma16816<T>(sacc[0], qa[k][0], qa[k][1], b0[0], b0[1]);
          mma16816<T>(sacc[1], qa[k][0], qa[k][1], b0[2], b0[3]);
          mma16816<T>(sacc[2], qa[k][0], qa[k][1], b1[0], b1[1]);
          mma16816<T>(sacc[3], qa[k][0], qa[k][1], b1[2], b1[3]);
        }
        // ---- online softmax on row g: values c0, c1 of each n-tile ----
        float sv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int tok = p0 + (e >> 1) * 8 + 2 * tq + (e & 1);
          sv[e] = tok < ntok ? sacc[e >> 1][e & 1] * sl2 : -INFINITY;
        }
        float mx = sv[0];
#pragma unroll
        for (int e = 1; e < 8; ++e) mx = fmaxf(mx, sv[e]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m, mx);
        const float corr = exp2f(m - mn);
        m = mn;
        float pr[8];
        float ps = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          pr[e] = exp2f(sv[e] - mn);
          ps += pr[e];
        }
        l = l * corr + ps;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          o[n][0] *= corr;
          o[n][1] *= corr;
        }
        // A operands of P.V: k-tile h2 covers tokens 16*h2 .. 16*h2+15
        const uint32_t pa0 = MmaType<T>::pack(pr[0], pr[1]);  // P[g][2tq, 2tq+1]
        const uint32_t pa2 = MmaType<T>::pack(pr[2], pr[3]);  // P[g][8+2tq, +1]
        const uint32_t pb0 = MmaType<T>::pack(pr[4], pr[5]);  // P[g][16+2tq, +1]
        const uint32_t pb2 = MmaType<T>::pack(pr[6], pr[7]);  // P[g][24+2tq, +1]
        // ---- O += P V ----
#pragma unroll
        for (int n = 0; n < NT; n += 2) {
          const int hb = n >> 3;
          const uint32_t off = (uint32_t)(hb * 128);
          // matrices: (tok 0-7, d n*8..), (tok 8-15, d n*8..), (tok 0-7, d n*8+8..), (tok 8-15, d n*8+8..)
          uint32_t b0[4], b1[4];
          ldsm_x4_trans(vrow[0] + off + (((((uint32_t)n & 7u) + vc) ^ (uint32_t)((vr[0] + hb) & 7)) << 4), b0);
          ldsm_x4_trans(vrow[1] + off + (((((uint32_t)n & 7u) + vc) ^ (uint32_t)((vr[1] + hb) & 7)) << 4), b1);
          mma16816<T>(o[n], pa0, pa2, b0[0], b0[1]);
          mma16816<T>(o[n + 1], pa0, pa2, b0[2], b0[3]);
          mma16816<T>(o[n], pb0, pb2, b1[0], b1[1]);
          mma16816<T>(o[n + 1], pb0, pb2, b1[2], b1[3]);
        }
      }
      if (ntok < TT) fence_proxy_async_smem();  // order the zero-fill before the slot's next bulk copy
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[slot]);
    }
    if (aborted) return;  // the abort flag is up; every other warp leaves at its next wait
    gbase += x.nstages;

    // ---- publish (acc, m, l) of rows g < group (double-buffered scratch), hand off ----
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int sbuf = n_done % a.nscr;
    if (!wait_or_abort(a, sm, &sm.scr_empty[sbuf], ((uint32_t)(n_done / a.nscr) & 1u) ^ 1u)) return;
    float* my_scr = sm.scratch + sbuf * sm.scratch_floats + (size_t)cw * group * state_stride(D);
    if (g < group) {
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        my_scr[g * state_stride(D) + n * 8 + 2 * tq] = o[n][0];
        my_scr[g * state_stride(D) + n * 8 + 2 * tq + 1] = o[n][1];
      }
      if (tq == 0) {
        my_scr[g * state_stride(D) + D] = m;
        my_scr[g * state_stride(D) + D + 1] = l;
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

// Two configurations, both at 2 CTAs per SM.  Groups of up to 4 query heads:
// 3 consumer warps, a 6-stage ring (96 KB of K/V in flight per CTA) and one
// merge scratch buffer.  Larger groups need twice the scratch and take 4
// consumer warps over a 4-stage ring (64 KB) with two scratch buffers.
template <typename T, int D, int NCW>
static int run_mma_cfg(const clove_pool& pool, DecodeArgs& a, cudaStream_t stream, int ring_target, int nscr) {
  auto kern = paged_decode_mma_kernel<T, D, NCW>;
  const int bs = pool.block_size;
  // Stages of >= 32 tokens: fixed per-stage costs (barrier round trips, copy
  // issue) halve against 16-token stages.
  const int sb = bs >= 32 ? 1 : 32 / bs;  // stages hold a multiple of 32 tokens
  a.stage_blocks = sb;
  a.nscr = nscr;
  // launch configuration, worked out once per (device, block size, group)
  struct Cfg {
    int ok = 0, nstage = 0, ncw = 0, smem = 0, ctas = 0;
  };
  static std::mutex mu;
  static std::unordered_map<long long, Cfg> cache;
  static int attr_smem = 0;
  Cfg c;
  {
    const long long key = ((long long)pool.device << 32) | ((long long)bs << 8) | a.group;
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      c = it->second;
    } else {
      const int scratch = NCW * a.group * state_stride(D) * 4;
      const int qb = a.group * D * (int)sizeof(T);
      SmemPlan sp = smem_plan(bs, D, sizeof(T), sb, 1, scratch, qb, nscr);
      int ncw = NCW;
      int nstage = (ring_target / sp.stage_bytes) / ncw * ncw;
      if (nstage < ncw) nstage = ncw;
      sp = smem_plan(bs, D, sizeof(T), sb, nstage, scratch, qb, nscr);
      while (sp.total + 1024 > 200 * 1024 && nstage > 1) {
        if (nstage > ncw) {
          nstage -= ncw;
        } else {
          ncw = --nstage;
        }
        sp = smem_plan(bs, D, sizeof(T), sb, nstage, scratch, qb, nscr);
      }
      const int smem = sp.total + 1024;  // 1024-byte alignment slack for the swizzled ring
      if (smem > 227 * 1024) {
        set_last_error("paged_decode: block_size %d x head_dim %d tile does not fit shared memory", bs, D);
        return CLOVE_ERR_UNSUPPORTED;
      }
      // (the attribute belongs to the kernel: only raise it, so configurations
      // cached for other block sizes stay launchable)
      if (smem > attr_smem) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
          set_last_error("cudaFuncSetAttribute: %s", cudaGetErrorString(cudaGetLastError()));
          return CLOVE_ERR_CUDA;
        }
        attr_smem = smem;
      }
      int occ = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, (NCW + 1) * 32, smem) != cudaSuccess ||
          occ < 1) {
        cudaGetLastError();
        occ = 1;
      }
      c.ok = 1;
      c.nstage = nstage;
      c.ncw = ncw;
      c.smem = smem;
      c.ctas = pool.num_sms * std::min(occ, kMaxCtasPerSm);
      cache[key] = c;
    }
  }
  a.nstage = c.nstage;
  a.ncw = c.ncw;
  a.num_ctas = c.ctas;
  cudaError_t e = launch_dependent(kern, (unsigned)c.ctas, (NCW + 1) * 32, c.smem, stream, pool.tm_k_sw,
                                   pool.tm_v_sw, a);
  if (e != cudaSuccess) {
    set_last_error("paged_decode (mma) launch: %s", cudaGetErrorString(e));
    return CLOVE_ERR_CUDA;
  }
  count_launches(1);
  return CLOVE_OK;
}

template <typename T, int D>
int run_mma(const clove_pool& pool, DecodeArgs& a, cudaStream_t stream) {
  if (!pool.has_swizzled || pool.block_size < 8 || a.group > 8) {
    set_last_error("paged_decode: tensor-core kernel needs a 16-bit pool, block_size >= 8, group <= 8");
    return CLOVE_ERR_UNSUPPORTED;
  }
  // CLOVE_DECODE_RING_KB overrides the ring target (a tuning override, read once)
  static const int ring_kb = [] {
    const char* v = std::getenv("CLOVE_DECODE_RING_KB");
    return v ? std::atoi(v) : 0;
  }();
  if (a.group <= 4) return run_mma_cfg<T, D, 3>(pool, a, stream, (ring_kb > 0 ? ring_kb : 96) * 1024, 1);
  return run_mma_cfg<T, D, 4>(pool, a, stream, (ring_kb > 0 ? ring_kb : 64) * 1024, 2);
}

template int run_mma<__nv_bfloat16, 64>(const clove_pool&, DecodeArgs&, cudaStream_t);
template int run_mma<__nv_bfloat16, 128>(const clove_pool&, DecodeArgs&, cudaStream_t);
template int run_mma<__half, 64>(const clove_pool&, DecodeArgs&, cudaStream_t);
template int run_mma<__half, 128>(const clove_pool&, DecodeArgs&, cudaStream_t);

}  // namespace clove
