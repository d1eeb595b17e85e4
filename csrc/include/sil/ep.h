// Layout of the expert-parallel symmetric buffer shared by the dispatch / combine
// kernels (csrc/kernels/ep.cu) and the scatter epilogue of the grouped fp8 GEMM
// (csrc/kernels/gemm_fp8.cu).  Offsets are bytes from the start of each rank's buffer;
// peers[r] is rank r's buffer mapped into this process (peers[rank] is the local one).
#pragma once
#include <stdint.h>

namespace sil {

struct EpLayout {
  long long peers[8];
  int rank, world, T, k, H, KB, e0, el;
  long long dflag_off, cflag_off, rows_off, scales_off, ids_off, wts_off, slots_off;
  int* status;
};

// state words at offset 0 of every buffer
constexpr int kEpEpoch = 0;        // layers completed
constexpr int kEpCtrDispatch = 1;  // arrival counters of grid-wide "last CTA" elections
constexpr int kEpCtrCombine = 2;
constexpr int kEpCtrGemm = 3;

}  // namespace sil
