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

int max_active_clusters(int s) {
  static int cache[64][kMaxClusterSplit + 1];
  static bool init[64][kMaxClusterSplit + 1];
  if (s < 2 || s > kMaxClusterSplit) return 0;
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64) return 0;
  if (!init[dev][s]) {
    using C = Cfg<32, 10, kEpiBf16, true>;
    auto kern = gemm_bf16_kernel<32, 10, kEpiBf16, true, false>;
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) ==
        cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(s * 64, 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = C::SMEM_BYTES;
      cudaLaunchAttribute at;
      at.id = cudaLaunchAttributeClusterDimension;
      at.val.clusterDim.x = s;
      at.val.clusterDim.y = 1;
      at.val.clusterDim.z = 1;
      cfg.attrs = &at;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();  // a refused query leaves no sticky error behind
    cache[dev][s] = n;
    init[dev][s] = true;
  }
  return cache[dev][s];
}

}  // namespace gemm_detail
}  // namespace sil
