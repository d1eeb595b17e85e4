// One-shot all-reduce over NVLink peer memory for decode-sized tensor-parallel sums.
//
// Every rank of the group owns a symmetric buffer (CUDA IPC, mapped by every peer):
//
//   [0, 256)             state: epoch, arrival counter (local use)
//   start[8][kMaxCtas]   u32, written by peers: "my partial for this epoch is complete"
//   end[8][kMaxCtas]     u32, written by peers: "I have finished reading your slice"
//   partial[T][H]        bf16, this rank's row-parallel GEMM output (the GEMM writes it
//                        there directly, so no copy precedes the reduction)
//
// CTA c of every rank handles the same slice of the T*H elements:
//   1. raise start[rank][c] on every rank (the partial was written by the previous kernel,
//      complete before this one starts), wait until every rank raised start[*][c];
//   2. pull the slice from every rank's partial with 16-byte loads, sum in rank order in
//      fp32 (the same order on every rank, so all ranks get bit-identical sums), add the
//      residual and store into h;
//   3. raise end[rank][c] everywhere and wait for end[*][c], so no rank overwrites its
//      partial (next GEMM) while a peer still reads it.
// Each CTA synchronises only with its counterparts on the other GPUs (no block of one
// launch waits for another block of the same launch).  Flags carry the epoch; every wait
// is bounded and reports through the sticky status word.  The last CTA advances the epoch.
//
// Reference semantics: the rank-ordered deterministic all-reduce of row-parallel
// projections, si/microsharding/dense.py:600-708.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "sil/host.h"
#include "sil/ptx.cuh"

namespace sil {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 256;
constexpr int kThreadsAR = 256;

struct OneShotArgs {
  long long peers[kMaxRanks];
  int rank, world;
  long long start_off, end_off, partial_off;
  __nv_bfloat16* h;      // [T, H] contiguous: h += sum of partials
  long long n;           // T * H
  int* status;
};

__device__ __forceinline__ uint32_t ld_acq(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_rel(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Threads 0..world-1: raise flag[rank][c] on peer `tid`, then wait for flag[tid][c] here.
__device__ __forceinline__ bool cross_rank_barrier(const OneShotArgs& a, long long off, uint32_t epoch) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  const int p = threadIdx.x;
  if (p < a.world) {
    uint32_t* remote = reinterpret_cast<uint32_t*>(a.peers[p] + off) + a.rank * kMaxCtas + blockIdx.x;
    st_rel(remote, epoch);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(a.peers[a.rank] + off) + p * kMaxCtas + blockIdx.x;
    const uint64_t t0 = globaltimer_ns();
    uint32_t it = 0;
    while (ld_acq(mine) != epoch) {
      if ((++it & 255u) == 0) {
        if (load_status(a.status) != 0 || globaltimer_ns() - t0 > SIL_WAIT_TIMEOUT_NS) {
          raise_status(a.status, kStatusTimeoutPeer);
          ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

__global__ void __launch_bounds__(kThreadsAR)
    oneshot_allreduce_kernel(const OneShotArgs a) {
  pdl_trigger();
  pdl_wait();  // the partial comes from the previous kernel (the row-parallel GEMM)
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(a.peers[a.rank]) + 1u;
  bool ok = cross_rank_barrier(a, a.start_off, epoch);
  const long long units = a.n / 8;  // 16-byte units of bf16
  const long long per = (units + gridDim.x - 1) / gridDim.x;
  const long long u0 = blockIdx.x * per, u1 = min(units, u0 + per);
  if (ok) {
    for (long long u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
      float acc[8];
      const uint4 r = reinterpret_cast<const uint4*>(a.h)[u];
      acc[0] = bf16_lo(r.x); acc[1] = bf16_hi(r.x); acc[2] = bf16_lo(r.y); acc[3] = bf16_hi(r.y);
      acc[4] = bf16_lo(r.z); acc[5] = bf16_hi(r.z); acc[6] = bf16_lo(r.w); acc[7] = bf16_hi(r.w);
      uint4 v[kMaxRanks];
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < a.world)
          v[p] = __ldcv(reinterpret_cast<const uint4*>(a.peers[p] + a.partial_off) + u);
      float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < a.world) {
          s[0] += bf16_lo(v[p].x); s[1] += bf16_hi(v[p].x); s[2] += bf16_lo(v[p].y); s[3] += bf16_hi(v[p].y);
          s[4] += bf16_lo(v[p].z); s[5] += bf16_hi(v[p].z); s[6] += bf16_lo(v[p].w); s[7] += bf16_hi(v[p].w);
        }
      uint4 o;
      o.x = pack_bf16x2(acc[0] + s[0], acc[1] + s[1]);
      o.y = pack_bf16x2(acc[2] + s[2], acc[3] + s[3]);
      o.z = pack_bf16x2(acc[4] + s[4], acc[5] + s[5]);
      o.w = pack_bf16x2(acc[6] + s[6], acc[7] + s[7]);
      reinterpret_cast<uint4*>(a.h)[u] = o;
    }
  }
  __syncthreads();
  ok = cross_rank_barrier(a, a.end_off, epoch) && ok;
  if (threadIdx.x == 0) {
    uint32_t* st = reinterpret_cast<uint32_t*>(a.peers[a.rank]);
    if (atomicAdd(st + 1, 1u) == gridDim.x - 1) {
      st[1] = 0u;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(st) = epoch;
    }
  }
}

// Row-sliced variant fused with the next RMSNorm: CTA t owns token row t, so after the
// rank-ordered sum it holds the whole row and can also write x = rmsnorm(h) * w.
__global__ void __launch_bounds__(kThreadsAR)
    oneshot_allreduce_norm_kernel(const OneShotArgs a, int H, const __nv_bfloat16* __restrict__ nw,
                                  float eps, __nv_bfloat16* __restrict__ x_out) {
  extern __shared__ float row[];  // H fp32 values of h after the sum
  __shared__ float red[32];
  pdl_trigger();
  pdl_wait();
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(a.peers[a.rank]) + 1u;
  bool ok = cross_rank_barrier(a, a.start_off, epoch);
  const int t = blockIdx.x;
  const long long base = (long long)t * H / 8;  // first 16-byte unit of this row
  float ss = 0.f;
  if (ok) {
    for (int u = threadIdx.x; u < H / 8; u += blockDim.x) {
      const uint4 r = reinterpret_cast<const uint4*>(a.h)[base + u];
      float v[8] = {bf16_lo(r.x), bf16_hi(r.x), bf16_lo(r.y), bf16_hi(r.y),
                    bf16_lo(r.z), bf16_hi(r.z), bf16_lo(r.w), bf16_hi(r.w)};
      uint4 pv[kMaxRanks];
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < a.world) pv[p] = __ldcv(reinterpret_cast<const uint4*>(a.peers[p] + a.partial_off) + base + u);
      float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < a.world) {
          s[0] += bf16_lo(pv[p].x); s[1] += bf16_hi(pv[p].x); s[2] += bf16_lo(pv[p].y); s[3] += bf16_hi(pv[p].y);
          s[4] += bf16_lo(pv[p].z); s[5] += bf16_hi(pv[p].z); s[6] += bf16_lo(pv[p].w); s[7] += bf16_hi(pv[p].w);
        }
      uint4 o;
      o.x = pack_bf16x2(v[0] + s[0], v[1] + s[1]);
      o.y = pack_bf16x2(v[2] + s[2], v[3] + s[3]);
      o.z = pack_bf16x2(v[4] + s[4], v[5] + s[5]);
      o.w = pack_bf16x2(v[6] + s[6], v[7] + s[7]);
      reinterpret_cast<uint4*>(a.h)[base + u] = o;
      // The norm sees the bf16-rounded residual stream, as the unfused RMSNorm would.
      const float hv[8] = {bf16_lo(o.x), bf16_hi(o.x), bf16_lo(o.y), bf16_hi(o.y),
                           bf16_lo(o.z), bf16_hi(o.z), bf16_lo(o.w), bf16_hi(o.w)};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        row[u * 8 + j] = hv[j];
        ss += hv[j] * hv[j];
      }
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rstd = rsqrtf(red[0] / H + eps);
  if (ok) {
    for (int u = threadIdx.x; u < H / 8; u += blockDim.x) {
      const uint4 wq = reinterpret_cast<const uint4*>(nw)[u];
      const float wv[8] = {bf16_lo(wq.x), bf16_hi(wq.x), bf16_lo(wq.y), bf16_hi(wq.y),
                           bf16_lo(wq.z), bf16_hi(wq.z), bf16_lo(wq.w), bf16_hi(wq.w)};
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        o[j] = wv[j] * __bfloat162float(__float2bfloat16_rn(row[u * 8 + j] * rstd));
      uint4 q;
      q.x = pack_bf16x2(o[0], o[1]); q.y = pack_bf16x2(o[2], o[3]);
      q.z = pack_bf16x2(o[4], o[5]); q.w = pack_bf16x2(o[6], o[7]);
      reinterpret_cast<uint4*>(x_out)[base + u] = q;
    }
  }
  __syncthreads();
  ok = cross_rank_barrier(a, a.end_off, epoch) && ok;
  if (threadIdx.x == 0) {
    uint32_t* st = reinterpret_cast<uint32_t*>(a.peers[a.rank]);
    if (atomicAdd(st + 1, 1u) == gridDim.x - 1) {
      st[1] = 0u;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(st) = epoch;
    }
  }
}

}  // namespace

// h [T, H] += sum of the ranks' partials, then x_out = rmsnorm(h) * w (one CTA per token).
void oneshot_allreduce_norm(at::Tensor& h, const std::vector<int64_t>& peers, int64_t rank,
                            int64_t start_off, int64_t end_off, int64_t partial_off, int64_t max_elems,
                            const at::Tensor& norm_w, double eps, at::Tensor& x_out,
                            const at::Tensor& status) {
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous() && h.dim() == 2,
              "oneshot_allreduce_norm: h [T, H] bf16 contiguous");
  TORCH_CHECK(x_out.is_contiguous() && x_out.sizes() == h.sizes() && x_out.scalar_type() == at::kBFloat16,
              "oneshot_allreduce_norm: x_out like h");
  const int world = static_cast<int>(peers.size());
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world, "oneshot_allreduce_norm: group");
  const int T = h.size(0), H = h.size(1);
  TORCH_CHECK(H % 8 == 0 && (long long)T * H <= max_elems && T <= kMaxCtas && norm_w.numel() == H &&
                  norm_w.scalar_type() == at::kBFloat16,
              "oneshot_allreduce_norm: shapes");
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(h.device());
  OneShotArgs a{};
  for (int i = 0; i < world; ++i) a.peers[i] = peers[i];
  a.rank = static_cast<int>(rank);
  a.world = world;
  a.start_off = start_off;
  a.end_off = end_off;
  a.partial_off = partial_off;
  a.h = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  a.n = (long long)T * H;
  a.status = status.data_ptr<int>();
  launch_pdl(oneshot_allreduce_norm_kernel, dim3(T), dim3(kThreadsAR), H * sizeof(float),
             at::cuda::getCurrentCUDAStream(), "oneshot_allreduce_norm launch", a, H,
             reinterpret_cast<const __nv_bfloat16*>(norm_w.data_ptr()), static_cast<float>(eps),
             reinterpret_cast<__nv_bfloat16*>(x_out.data_ptr()));
}

// h [T, H] bf16 contiguous += sum over ranks of each rank's partial (same shape) stored at
// byte offset `partial_off` of its symmetric buffer.
void oneshot_allreduce(at::Tensor& h, const std::vector<int64_t>& peers, int64_t rank,
                       int64_t start_off, int64_t end_off, int64_t partial_off, int64_t max_elems,
                       const at::Tensor& status) {
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous(), "oneshot_allreduce: h bf16 contiguous");
  const int world = static_cast<int>(peers.size());
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world, "oneshot_allreduce: group");
  const long long n = h.numel();
  TORCH_CHECK(n % 8 == 0 && n <= max_elems, "oneshot_allreduce: size exceeds the buffer or not 16-byte units");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(h.data_ptr()) & 15) == 0 && partial_off % 16 == 0,
              "oneshot_allreduce: 16-byte alignment");
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(h.device());
  OneShotArgs a{};
  for (int i = 0; i < world; ++i) a.peers[i] = peers[i];
  a.rank = static_cast<int>(rank);
  a.world = world;
  a.start_off = start_off;
  a.end_off = end_off;
  a.partial_off = partial_off;
  a.h = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  a.n = n;
  a.status = status.data_ptr<int>();
  const long long units = n / 8;
  // Two 16-byte units per thread: 32 CTAs pull 2 MB (32 tokens x 4096 x 8 ranks) in parallel.
  const int grid = static_cast<int>(std::max<long long>(
      1, std::min<long long>(kMaxCtas, (units + 2 * kThreadsAR - 1) / (2 * kThreadsAR))));
  launch_pdl(oneshot_allreduce_kernel, dim3(grid), dim3(kThreadsAR), 0,
             at::cuda::getCurrentCUDAStream(), "oneshot_allreduce launch", a);
}

// A bf16 [rows, cols] tensor over bytes [offset, ...) of a symmetric buffer (no ownership).
at::Tensor symm_tensor(int64_t ptr, int64_t offset, int64_t rows, int64_t cols, int64_t device) {
  auto opts = at::TensorOptions().dtype(at::kBFloat16).device(at::kCUDA, device);
  return torch::from_blob(reinterpret_cast<void*>(ptr + offset), {rows, cols}, opts);
}

}  // namespace sil
