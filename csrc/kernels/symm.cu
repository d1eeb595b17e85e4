// Symmetric peer memory for the fused tensor-parallel kernels.
//
// Each rank allocates one buffer of the same size with cudaMalloc and
// exports a CUDA IPC handle; every rank opens the others' handles, so a
// kernel can store directly into a peer's buffer over NVLink (P2P stores,
// no library kernel on a peer's memory, no multicast loads).  The handle
// exchange itself is host plumbing done over torch.distributed.
//
// Buffer layout (identical on every rank), see parallel/fused_tp.py:
//   [0, 256)               state words (epoch, finished-CTA counter), local use only
//   [256, 256 + FLAGS)     flags[2][8][max_tiles] uint32 (written by peers)
//   [.., ..)               slots[2][8][max_tokens][max_hidden] bf16 (written by peers)
#include <torch/extension.h>

#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "sil/host.h"

namespace sil {

int64_t symm_alloc(int64_t bytes, int64_t device) {
  check_cuda(cudaSetDevice(static_cast<int>(device)), "cudaSetDevice");
  void* p = nullptr;
  check_cuda(cudaMalloc(&p, static_cast<size_t>(bytes)), "cudaMalloc(symmetric buffer)");
  check_cuda(cudaMemset(p, 0, static_cast<size_t>(bytes)), "cudaMemset(symmetric buffer)");
  check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  return reinterpret_cast<int64_t>(p);
}

void symm_free(int64_t ptr) {
  if (ptr != 0) check_cuda(cudaFree(reinterpret_cast<void*>(ptr)), "cudaFree(symmetric buffer)");
}

// Raw bytes of the IPC handle of an allocation made by symm_alloc.
std::string ipc_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  check_cuda(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)), "cudaIpcGetMemHandle");
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

int64_t ipc_open(const std::string& handle, int64_t device) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "ipc_open: bad handle size");
  check_cuda(cudaSetDevice(static_cast<int>(device)), "cudaSetDevice");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) {
  if (ptr != 0) check_cuda(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)), "cudaIpcCloseMemHandle");
}

bool can_access_peer(int64_t dev, int64_t peer) {
  int ok = 0;
  check_cuda(cudaDeviceCanAccessPeer(&ok, static_cast<int>(dev), static_cast<int>(peer)),
             "cudaDeviceCanAccessPeer");
  return ok != 0;
}

}  // namespace sil
