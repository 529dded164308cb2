// Tensor-core decode path (bf16 / f16, GQA group >= 4).  Declared here,
// defined in mma_decode.cu.
#pragma once
#include "common.cuh"
#include "host.h"

namespace clove {

template <int D>
constexpr bool mma_supported() {
  return D == 64 || D == 128;
}

template <typename T, int D>
int run_mma(const clove_pool& pool, DecodeArgs& a, cudaStream_t stream);

}  // namespace clove
