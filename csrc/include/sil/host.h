// Host-side helpers shared by the CUDA extension: TMA tensor-map encoding via
// the driver entry point (no link-time libcuda dependency), launch checks and
// the SM count of the current device.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <set>
#include <utility>
#include <stdexcept>
#include <string>

namespace sil {

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
  }
}

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    check_cuda(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                                cudaEnableDefault, &q),
               "cudaGetDriverEntryPointByVersion(cuTensorMapEncodeTiled)");
    if (q != cudaDriverEntryPointSuccess || p == nullptr) {
      throw std::runtime_error("cuTensorMapEncodeTiled entry point not found");
    }
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D row-major tensor [rows, cols] (cols contiguous) of `elem_bytes`-byte
// elements with a row pitch of `row_stride_elems`.  Box = [box_rows, box_cols].
// The innermost box extent times the element size must be a multiple of 16 B
// and the base address / row pitch must be 16-byte aligned.
inline CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                                uint64_t rows, uint64_t cols, uint64_t row_stride_elems,
                                uint32_t box_rows, uint32_t box_cols,
                                CUtensorMapSwizzle swizzle) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) {
    throw std::invalid_argument("TMA base address must be 16-byte aligned");
  }
  if ((row_stride_elems * elem_bytes) % 16 != 0) {
    throw std::invalid_argument("TMA row pitch must be a multiple of 16 bytes");
  }
  if ((box_cols * elem_bytes) % 16 != 0) {
    throw std::invalid_argument("TMA inner box extent must be a multiple of 16 bytes");
  }
  CUtensorMap map;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * static_cast<cuuint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&map, dtype, 2, const_cast<void*>(base), dims, strides, box,
                                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    throw std::runtime_error("cuTensorMapEncodeTiled failed with code " + std::to_string(r));
  }
  return map;
}

// Raises a kernel's dynamic shared-memory limit to `bytes` on the current device.
// The attribute is per device, so it is set once per (kernel, device) pair.
inline void set_smem_limit(const void* kern, int bytes, const char* what) {
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kern, dev})) return;
  check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what);
  done.insert({kern, dev});
}

inline int device_sm_count() {
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  static int cached[64] = {0};
  if (dev < 64 && cached[dev] > 0) return cached[dev];
  int n = 0;
  check_cuda(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev),
             "cudaDeviceGetAttribute(SM count)");
  if (dev < 64) cached[dev] = n;
  return n;
}

// Programmatic dependent launch is on unless SIL_PDL=0 (or set_pdl_enabled(false)).
inline int& pdl_state() {
  static int v = -1;
  return v;
}

inline bool pdl_enabled() {
  int& v = pdl_state();
  if (v < 0) {
    const char* e = std::getenv("SIL_PDL");
    v = (e == nullptr || e[0] != '0') ? 1 : 0;
  }
  return v == 1;
}

// Affects launches issued afterwards (CUDA graphs keep the attributes they were captured with).
inline void set_pdl_enabled(bool on) { pdl_state() = on ? 1 : 0; }

// Launch `kern` with the programmatic-stream-serialization attribute so its
// pre-`griddepcontrol.wait` prologue may overlap the previous kernel's tail.
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  check_cuda(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...), what);
}

}  // namespace sil
