// Instantiations of the tcgen05 GEMM for epilogue kEpiResAdd (split per file so the
// kernel library compiles in parallel).
#include "gemm_bf16_impl.cuh"

namespace sil {
namespace gemm_detail {

template <>
void dispatch_swap<kEpiResAdd>(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                   int mt, int nt, cudaStream_t st) {
  switch (bn) {
    case 16: launch<16, 6, kEpiResAdd, true>(ta, tb, a, mt, nt, st); break;
    case 32: launch<32, 5, kEpiResAdd, true>(ta, tb, a, mt, nt, st); break;
    case 64: launch<64, 4, kEpiResAdd, true>(ta, tb, a, mt, nt, st); break;
    default: launch<128, 3, kEpiResAdd, true>(ta, tb, a, mt, nt, st); break;
  }
}

template <>
void dispatch_normal<kEpiResAdd>(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                     int mt, int nt, cudaStream_t st) {
  if (bn == 256) launch<256, 4, kEpiResAdd, false>(ta, tb, a, mt, nt, st);
  else launch<128, 6, kEpiResAdd, false>(ta, tb, a, mt, nt, st);
}


}  // namespace gemm_detail
}  // namespace sil
