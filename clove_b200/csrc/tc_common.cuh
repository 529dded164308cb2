// 5th-generation tensor-core helpers (tcgen05, sm_100a) shared by the fused
// Q/K/V projection and the prefill kernel: shared-memory matrix descriptors,
// the MMA issue / commit, tensor-memory loads and stores, and a 2-D tensor
// copy.
#pragma once

#include "common.cuh"

namespace clove {

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor for a K-major tile with the 128-byte
// swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte
// offset), leading byte offset unused by this layout (encoded 1), descriptor
// version 1 (bits 46-47), layout type 2 = 128-byte swizzle (bits 61-63).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  return (uint64_t)((smem_addr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive accumulator columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive 32-bit columns of this thread's tensor-memory lane, stored.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for an MN-major operand with the 128-byte
// swizzle: 128-byte rows of 64 MN-elements, one row per K index, 8-row groups
// `sbo` bytes apart along K, 64-element MN blocks `lbo` bytes apart.
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((smem_addr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16 with f32 accumulate: M x N tile, A and B
// both bf16 or both f16, A K-major, B K-major (b_mn = 0) or MN-major (1).
__host__ __device__ inline uint32_t f16_idesc(bool bf16, int m, int n, int b_mn) {
  const uint32_t f = bf16 ? 1u : 0u;
  return (1u << 4) | (f << 7) | (f << 10) | ((uint32_t)b_mn << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

// ---- softmax row helpers (one 128-score row per thread) ----

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack_f32x2(uint64_t x, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(x));
}

// Max of 128 values: three-input max in 8 independent chains.
__device__ __forceinline__ float row_max128(const float (&v)[128]) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = max3f(v[i], v[8 + i], v[16 + i]);
#pragma unroll
  for (int k = 24; k < 120; k += 16)
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = max3f(m[i], v[k + i], v[k + 8 + i]);
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmaxf(m[i], v[120 + i]);
  return max3f(max3f(m[0], m[1], m[2]), max3f(m[3], m[4], m[5]), fmaxf(m[6], m[7]));
}

// v[k] <- 2^(v[k] * scale - ref) (the special-function unit's 2^x, -inf ->
// +0); returns the sum.  Scale-and-shift and the sum run as packed f32x2
// operations, two elements per instruction.
__device__ __forceinline__ float row_exp2_sum128(float (&v)[128], float scale, float ref) {
  const uint64_t sc = pack_f32x2(scale, scale), nr = pack_f32x2(-ref, -ref);
  uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
  for (int k = 0; k < 128; k += 2) {
    uint64_t x = pack_f32x2(v[k], v[k + 1]);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(x) : "l"(x), "l"(sc), "l"(nr));
    float x0, x1;
    unpack_f32x2(x, x0, x1);
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(v[k]) : "f"(x0));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(v[k + 1]) : "f"(x1));
    const uint64_t y = pack_f32x2(v[k], v[k + 1]);
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(acc[(k >> 1) & 3]) : "l"(acc[(k >> 1) & 3]), "l"(y));
  }
  float s[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) unpack_f32x2(acc[i], s[2 * i], s[2 * i + 1]);
  return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

}  // namespace clove
