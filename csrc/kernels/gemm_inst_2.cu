// Instantiations of the tcgen05 GEMM for epilogue kEpiSwiGLU (one file per epilogue so
// the kernel library compiles in parallel).
#include "gemm_bf16_impl.cuh"

namespace sil {
namespace gemm_detail {

template <>
void dispatch_swap<kEpiSwiGLU>(int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                          const GemmArgs& a, cudaStream_t st) {
  switch (bn) {
    case 16: launch<16, 6, kEpiSwiGLU, true>(ta, tb, a, st); break;
    case 32: launch<32, 6, kEpiSwiGLU, true>(ta, tb, a, st); break;
    case 64: launch<64, 5, kEpiSwiGLU, true>(ta, tb, a, st); break;
    default: launch<128, 4, kEpiSwiGLU, true>(ta, tb, a, st); break;
  }
}

template <>
void dispatch_normal<kEpiSwiGLU>(int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                            const GemmArgs& a, cudaStream_t st) {
  if (bn == 256) launch<256, 4, kEpiSwiGLU, false>(ta, tb, a, st);
  else launch<128, 6, kEpiSwiGLU, false>(ta, tb, a, st);
}

}  // namespace gemm_detail
}  // namespace sil
