// Instantiations of the tcgen05 GEMM with the fused tensor-parallel all-reduce
// epilogue (decode order only: at most 128 tokens per call).
#include "gemm_bf16_impl.cuh"

namespace sil {
namespace gemm_detail {

template <>
void dispatch_swap<kEpiAllReduce>(int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                                  const GemmArgs& a, cudaStream_t st) {
  switch (bn) {
    case 16: launch<16, 11, kEpiAllReduce, true>(ta, tb, a, st); break;
    case 32: launch<32, 10, kEpiAllReduce, true>(ta, tb, a, st); break;
    case 64: launch<64, 8, kEpiAllReduce, true>(ta, tb, a, st); break;
    default: launch<128, 6, kEpiAllReduce, true>(ta, tb, a, st); break;
  }
}

}  // namespace gemm_detail
}  // namespace sil
