// Instantiations of the tcgen05 GEMM for epilogue kEpiBf16 (one file per epilogue so
// the kernel library compiles in parallel).
#include "gemm_bf16_impl.cuh"

namespace sil {
namespace gemm_detail {

template <>
void dispatch_swap<kEpiBf16>(int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                          const GemmArgs& a, cudaStream_t st) {
  switch (bn) {
    case 16: launch<16, 11, kEpiBf16, true>(ta, tb, a, st); break;
    case 32: launch<32, 10, kEpiBf16, true>(ta, tb, a, st); break;
    case 64: launch<64, 8, kEpiBf16, true>(ta, tb, a, st); break;
    default: launch<128, 6, kEpiBf16, true>(ta, tb, a, st); break;
  }
}

template <>
void dispatch_normal<kEpiBf16>(int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                            const GemmArgs& a, cudaStream_t st) {
  if (bn == 256) launch<256, 4, kEpiBf16, false>(ta, tb, a, st);
  else launch<128, 6, kEpiBf16, false>(ta, tb, a, st);
}

}  // namespace gemm_detail
}  // namespace sil
