// Instantiations of the tcgen05 GEMM for epilogue kEpiF32 (one file per epilogue so
// the kernel library compiles in parallel).
#include "gemm_bf16_impl.cuh"

namespace sil {
namespace gemm_detail {

template <>
void dispatch_swap<kEpiF32>(int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                          const GemmArgs& a, cudaStream_t st) {
  switch (bn) {
    case 16: launch<16, 11, kEpiF32, true>(ta, tb, a, st); break;
    case 32: launch<32, 10, kEpiF32, true>(ta, tb, a, st); break;
    case 64: launch<64, 8, kEpiF32, true>(ta, tb, a, st); break;
    default: launch<128, 6, kEpiF32, true>(ta, tb, a, st); break;
  }
}

template <>
void dispatch_normal<kEpiF32>(int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                            const GemmArgs& a, cudaStream_t st) {
  if (bn == 256) launch<256, 4, kEpiF32, false>(ta, tb, a, st);
  else launch<128, 6, kEpiF32, false>(ta, tb, a, st);
}

}  // namespace gemm_detail
}  // namespace sil
