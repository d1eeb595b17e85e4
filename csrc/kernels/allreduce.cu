// One-shot all-reduce over NVLink peer memory for decode-sized tensor-parallel sums.
//
// Every rank of the group owns a symmetric buffer (CUDA IPC, mapped by every peer):
//
//   [0, 256)                state: epoch, arrival counter (local use)
//   flags[8][kMaxCtas]      u32, written by peers: "slice c of my partial has landed here"
//   partial[T][H]           bf16, this rank's row-parallel GEMM output (the GEMM writes it
//                           there directly)
//   recv[2][8][T][H]        bf16, the peers' partials pushed here (alternating by epoch parity)
//
// CTA c of every rank owns the same slice of the T*H elements:
//   1. push its slice of the local partial into recv[parity][rank] of every peer with
//      16-byte stores, then (after a barrier, one system fence) raise flags[rank][c] on
//      every peer;
//   2. wait until every peer's flags[*][c] reached this epoch, sum the slice in rank order (the
//      local partial for this rank's term; the same order on every rank, so all ranks get
//      bit-identical sums), add the residual and store into h.
// Data crosses NVLink once, as fire-and-forget stores.  A peer can only push epoch e+2 into
// the parity this CTA reads at epoch e after it has seen this rank's flag for epoch e+1,
// which this rank raises after finishing epoch e, so no second barrier is needed.  Each CTA
// synchronises only with its counterparts on the other GPUs (no block of one launch waits
// for another block of the same launch).  Every wait is bounded and reports through the
// sticky status word.  The last CTA advances the epoch.
//
// Reference semantics: the rank-ordered deterministic all-reduce of row-parallel
// projections, si/microsharding/dense.py:600-708.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>
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
  long long flags_off, partial_off, recv_off;
  long long max_elems;
  __nv_bfloat16* h;      // [T, H] contiguous: h += sum of partials
  long long n;           // T * H
  int* status;
  int late_trigger;      // 1: let the next kernel launch only after this one's exchange
};

// SIL_AR_LATE_TRIGGER=1 moves the programmatic-launch trigger of the one-shot kernels from
// their first instruction to after the exchange, so the next GEMM's CTAs (and their weight
// prefetch) do not start while this kernel is still waiting on its peers.
inline int ar_late_trigger() {
  static const char* v = std::getenv("SIL_AR_LATE_TRIGGER");
  return v != nullptr && v[0] == '1' ? 1 : 0;
}

__device__ __forceinline__ uint32_t ld_acq(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_rel(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ __nv_bfloat16* recv_slot(const OneShotArgs& a, int owner, int par, int src) {
  return reinterpret_cast<__nv_bfloat16*>(a.peers[owner] + a.recv_off) +
         ((long long)par * kMaxRanks + src) * a.max_elems;
}

// Push units [u0, u1) of the local partial to every peer, then raise flags[rank][c] there.
__device__ __forceinline__ void push_slice(const OneShotArgs& a, int par, uint32_t epoch,
                                           long long u0, long long u1) {
  const uint4* src = reinterpret_cast<const uint4*>(a.peers[a.rank] + a.partial_off);
  for (long long u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
    const uint4 v = src[u];
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p)
      if (p < a.world && p != a.rank) reinterpret_cast<uint4*>(recv_slot(a, p, par, a.rank))[u] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) __threadfence_system();  // cumulative over the CTA's pushes
  __syncthreads();
  const int p = threadIdx.x;
  if (p < a.world && p != a.rank)
    st_rel(reinterpret_cast<uint32_t*>(a.peers[p] + a.flags_off) + a.rank * kMaxCtas + blockIdx.x, epoch);
}

// Threads 0..world-1 wait for flags[p][c] >= epoch (p != rank).
__device__ __forceinline__ bool wait_slice(const OneShotArgs& a, uint32_t epoch) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  const int p = threadIdx.x;
  if (p < a.world && p != a.rank) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(a.peers[a.rank] + a.flags_off) + p * kMaxCtas + blockIdx.x;
    const uint64_t t0 = globaltimer_ns();
    uint32_t it = 0;
    // >= rather than ==: a fast peer may already have raised the next epoch's flag (it only
    // needs this rank's flag for the current epoch to go on), and epochs only grow.
    while (static_cast<int>(ld_acq(f) - epoch) < 0) {
      if ((++it & 255u) == 0) {
        if (load_status(a.status) != 0 || globaltimer_ns() - t0 > wait_limit_ns(a.status)) {
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

// Rank-ordered fp32 sum of unit u over all ranks (local partial for this rank's term).
__device__ __forceinline__ void sum_unit(const OneShotArgs& a, int par, long long u, float (&s)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = 0.f;
  uint4 v[kMaxRanks];
#pragma unroll
  for (int p = 0; p < kMaxRanks; ++p)
    if (p < a.world)
      v[p] = p == a.rank ? reinterpret_cast<const uint4*>(a.peers[a.rank] + a.partial_off)[u]
                         : __ldcv(reinterpret_cast<const uint4*>(recv_slot(a, a.rank, par, p)) + u);
#pragma unroll
  for (int p = 0; p < kMaxRanks; ++p)
    if (p < a.world) {
      s[0] += bf16_lo(v[p].x); s[1] += bf16_hi(v[p].x); s[2] += bf16_lo(v[p].y); s[3] += bf16_hi(v[p].y);
      s[4] += bf16_lo(v[p].z); s[5] += bf16_hi(v[p].z); s[6] += bf16_lo(v[p].w); s[7] += bf16_hi(v[p].w);
    }
}

__device__ __forceinline__ void bump_epoch(const OneShotArgs& a, uint32_t epoch) {
  if (threadIdx.x == 0) {
    uint32_t* st = reinterpret_cast<uint32_t*>(a.peers[a.rank]);
    if (atomicAdd(st + 1, 1u) == gridDim.x - 1) {
      st[1] = 0u;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(st) = epoch;
    }
  }
}

__global__ void __launch_bounds__(kThreadsAR)
    oneshot_allreduce_kernel(const OneShotArgs a) {
  if (!a.late_trigger) pdl_trigger();
  pdl_wait();  // the partial comes from the previous kernel (the row-parallel GEMM)
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(a.peers[a.rank]) + 1u;
  const int par = epoch & 1;
  const long long units = a.n / 8;  // 16-byte units of bf16
  const long long per = (units + gridDim.x - 1) / gridDim.x;
  const long long u0 = blockIdx.x * per, u1 = min(units, u0 + per);
  push_slice(a, par, epoch, u0, u1);
  if (wait_slice(a, epoch)) {
    for (long long u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
      float s[8];
      sum_unit(a, par, u, s);
      const uint4 r = reinterpret_cast<const uint4*>(a.h)[u];
      uint4 o;
      o.x = pack_bf16x2(bf16_lo(r.x) + s[0], bf16_hi(r.x) + s[1]);
      o.y = pack_bf16x2(bf16_lo(r.y) + s[2], bf16_hi(r.y) + s[3]);
      o.z = pack_bf16x2(bf16_lo(r.z) + s[4], bf16_hi(r.z) + s[5]);
      o.w = pack_bf16x2(bf16_lo(r.w) + s[6], bf16_hi(r.w) + s[7]);
      reinterpret_cast<uint4*>(a.h)[u] = o;
    }
  }
  if (a.late_trigger) pdl_trigger();
  bump_epoch(a, epoch);
}

// Row-sliced variant fused with the next RMSNorm: CTA t owns token row t, so after the
// rank-ordered sum it holds the whole row and can also write x = rmsnorm(h) * w.
__global__ void __launch_bounds__(kThreadsAR)
    oneshot_allreduce_norm_kernel(const OneShotArgs a, int H, const __nv_bfloat16* __restrict__ nw,
                                  float eps, __nv_bfloat16* __restrict__ x_out) {
  extern __shared__ float row[];  // H fp32 values of h after the sum
  __shared__ float red[32];
  if (!a.late_trigger) pdl_trigger();
  pdl_wait();
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(a.peers[a.rank]) + 1u;
  const int par = epoch & 1;
  const int t = blockIdx.x;
  const long long base = (long long)t * H / 8;  // first 16-byte unit of this row
  push_slice(a, par, epoch, base, base + H / 8);
  const bool ok = wait_slice(a, epoch);
  float ss = 0.f;
  if (ok) {
    for (int u = threadIdx.x; u < H / 8; u += blockDim.x) {
      float s[8];
      sum_unit(a, par, base + u, s);
      const uint4 r = reinterpret_cast<const uint4*>(a.h)[base + u];
      uint4 o;
      o.x = pack_bf16x2(bf16_lo(r.x) + s[0], bf16_hi(r.x) + s[1]);
      o.y = pack_bf16x2(bf16_lo(r.y) + s[2], bf16_hi(r.y) + s[3]);
      o.z = pack_bf16x2(bf16_lo(r.z) + s[4], bf16_hi(r.z) + s[5]);
      o.w = pack_bf16x2(bf16_lo(r.w) + s[6], bf16_hi(r.w) + s[7]);
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
  if (a.late_trigger) pdl_trigger();
  bump_epoch(a, epoch);
}

}  // namespace

// h [T, H] += sum of the ranks' partials, then x_out = rmsnorm(h) * w (one CTA per token).
void oneshot_allreduce_norm(at::Tensor& h, const std::vector<int64_t>& peers, int64_t rank,
                            int64_t flags_off, int64_t recv_off, int64_t partial_off, int64_t max_elems,
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
  a.flags_off = flags_off;
  a.recv_off = recv_off;
  a.max_elems = max_elems;
  a.partial_off = partial_off;
  a.h = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  a.n = (long long)T * H;
  a.status = status.data_ptr<int>();
  a.late_trigger = ar_late_trigger();
  launch_pdl(oneshot_allreduce_norm_kernel, dim3(T), dim3(kThreadsAR), H * sizeof(float),
             at::cuda::getCurrentCUDAStream(), "oneshot_allreduce_norm launch", a, H,
             reinterpret_cast<const __nv_bfloat16*>(norm_w.data_ptr()), static_cast<float>(eps),
             reinterpret_cast<__nv_bfloat16*>(x_out.data_ptr()));
}

// h [T, H] bf16 contiguous += sum over ranks of each rank's partial (same shape) stored at
// byte offset `partial_off` of its symmetric buffer.
void oneshot_allreduce(at::Tensor& h, const std::vector<int64_t>& peers, int64_t rank,
                       int64_t flags_off, int64_t recv_off, int64_t partial_off, int64_t max_elems,
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
  a.flags_off = flags_off;
  a.recv_off = recv_off;
  a.max_elems = max_elems;
  a.partial_off = partial_off;
  a.h = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  a.n = n;
  a.status = status.data_ptr<int>();
  a.late_trigger = ar_late_trigger();
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
