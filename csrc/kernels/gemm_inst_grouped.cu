// Instantiations of the grouped (MoE expert) tcgen05 GEMM: plain bf16 output
// (expert down projection) and SwiGLU (expert gate/up projection), in both
// operand orders.
#include "gemm_bf16_impl.cuh"

namespace sil {
namespace gemm_detail {

template <int EPI, int S16, int S32, int S64, int S128>
static void grouped_impl(bool swap, int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                         const GemmArgs& a, cudaStream_t st) {
  if (swap) {
    switch (bn) {
      case 16: launch<16, S16, EPI, true, true>(ta, tb, a, st); break;
      case 32: launch<32, S32, EPI, true, true>(ta, tb, a, st); break;
      case 64: launch<64, S64, EPI, true, true>(ta, tb, a, st); break;
      default: launch<128, S128, EPI, true, true>(ta, tb, a, st); break;
    }
  } else {
    launch<256, 4, EPI, false, true>(ta, tb, a, st);
  }
}

template <>
void dispatch_grouped<kEpiBf16>(bool swap, int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                                const GemmArgs& a, cudaStream_t st) {
  grouped_impl<kEpiBf16, 11, 10, 8, 6>(swap, bn, ta, tb, a, st);
}

template <>
void dispatch_grouped<kEpiSwiGLU>(bool swap, int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                                  const GemmArgs& a, cudaStream_t st) {
  grouped_impl<kEpiSwiGLU, 6, 6, 5, 4>(swap, bn, ta, tb, a, st);
}

}  // namespace gemm_detail
}  // namespace sil
