// Two-shot all-reduce through NVSwitch multicast (NVLS) for decode-sized tensor-parallel
// sums, optionally fused with the next RMSNorm.
//
// Every rank owns the same symmetric buffer (allocated and bound to one multicast object by
// torch's symmetric-memory rendezvous); `mc` is the multicast address of that buffer and
// `peers[r]` the unicast address of rank r's copy:
//
//   [0, 256)             state: epoch, CTA arrival counter (local use)
//   flags1[256][8]       u32: "rank src has its partial ready"       (written by peers)
//   flags2[256][8]       u32: "rank src has broadcast its slice"     (written by peers)
//   partial[T][H]        bf16: this rank's row-parallel GEMM output (the GEMM writes it)
//   sum[T][H]            bf16: the all-reduced rows, written by every rank through `mc`
//
// CTA t owns token row t on every rank.  Rank r reduces the column slice
// [r*H/N, (r+1)*H/N) of row t: one `multimem.ld_reduce` per 16 bytes makes the switch read
// that slice from all N partials and return their sum (fp32 accumulation, one bf16 rounding),
// and one `multimem.st` writes the result into every rank's `sum`.  Two flag exchanges
// (per CTA, unicast release stores to each peer) order the steps: before the reduce every
// partial is complete; before `sum` is read every slice has landed.  Then the CTA adds its
// row to the residual stream h and, when a norm weight is given, writes the next block's
// input x = rmsnorm(h) * w.  Each rank sends H*2/N bytes per row and receives H*2 bytes:
// the NVLink traffic of a reduce-scatter plus an all-gather, with the reduction in the
// switch.  Every rank reads the same sums, so all ranks hold bit-identical h.
//
// Buffers need no double-buffering: a rank writes its next partial only after it passed
// this call's second exchange, i.e. after every peer finished reading its partial, and a
// peer writes the next sums only after this rank raised the next first-exchange flag,
// i.e. after it finished reading this call's sums.  Flags carry a monotonically growing
// epoch and waits compare with >=, so early flags of the next call are harmless.  Every
// wait is bounded and reports through the sticky status word.
//
// Reference semantics: the row-parallel all-reduce of the logical tensor-parallel model,
// si/microsharding/dense.py:600-708, and the RMSNorm that follows it (:146-166).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "sil/host.h"
#include "sil/ptx.cuh"

namespace sil {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxRows = 256;
constexpr int kThreadsNvls = 128;

struct NvlsArgs {
  long long peers[kMaxRanks];  // unicast base of every rank's buffer
  long long mc;                // multicast base of the buffer
  int rank, world;
  long long flags1_off, flags2_off, partial_off, sum_off;
  __nv_bfloat16* h;            // [T, H] contiguous residual stream
  int T, H;
  const __nv_bfloat16* nw;     // RMSNorm weight [H] or nullptr (no norm)
  float eps;
  __nv_bfloat16* x_out;        // [T, H] when nw != nullptr
  int* status;
};

__device__ __forceinline__ uint32_t ld_acq_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_rel_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Sum over all ranks of 8 bf16 at multicast address p (fp32 accumulation in the switch).
__device__ __forceinline__ uint4 mc_ld_reduce_bf16x8(long long p) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p)
               : "memory");
  return r;
}

// Store 16 bytes into every rank's copy of multicast address p.
__device__ __forceinline__ void mc_st_16(long long p, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Flag exchange of CTA blockIdx.x with its counterparts on every peer: raise flags[cta][rank]
// on each peer after this CTA's prior writes are visible system-wide, then wait until every
// peer raised flags[cta][p] here.  Returns false (status raised) when a peer never arrives.
__device__ __forceinline__ bool exchange(const NvlsArgs& a, long long flags_off, uint32_t epoch) {
  __shared__ int ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    ok = 1;
    __threadfence_system();  // cumulative over the CTA's writes ordered before it by the barrier
  }
  __syncthreads();
  const int p = threadIdx.x;
  if (p < a.world && p != a.rank)
    st_rel_sys(reinterpret_cast<uint32_t*>(a.peers[p] + flags_off) + blockIdx.x * kMaxRanks + a.rank,
               epoch);
  if (p < a.world && p != a.rank) {
    const uint32_t* f =
        reinterpret_cast<const uint32_t*>(a.peers[a.rank] + flags_off) + blockIdx.x * kMaxRanks + p;
    const uint64_t t0 = globaltimer_ns();
    uint32_t it = 0;
    while (static_cast<int>(ld_acq_sys(f) - epoch) < 0) {
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

__global__ void __launch_bounds__(kThreadsNvls) nvls_allreduce_kernel(const NvlsArgs a) {
  extern __shared__ float row[];  // H fp32 values of the updated h row (norm only)
  __shared__ float red[32];
  pdl_trigger();
  pdl_wait();  // the partial comes from the previous kernel (the row-parallel GEMM)
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(a.peers[a.rank]) + 1u;
  const int t = blockIdx.x;
  const long long row_off = (long long)t * a.H * 2;  // bytes
  bool ok = exchange(a, a.flags1_off, epoch);
  if (ok) {
    const int cols = a.H / a.world;
    const long long slice = row_off + (long long)a.rank * cols * 2;
    for (int u = threadIdx.x; u < cols / 8; u += blockDim.x) {
      const uint4 s = mc_ld_reduce_bf16x8(a.mc + a.partial_off + slice + u * 16);
      mc_st_16(a.mc + a.sum_off + slice + u * 16, s);
    }
  }
  ok = exchange(a, a.flags2_off, epoch) && ok;
  asm volatile("fence.proxy.alias;" ::: "memory");  // sums arrived through the multicast alias
  float ss = 0.f;
  const uint4* sum = reinterpret_cast<const uint4*>(a.peers[a.rank] + a.sum_off + row_off);
  uint4* h = reinterpret_cast<uint4*>(a.h + (long long)t * a.H);
  if (ok) {
    for (int u = threadIdx.x; u < a.H / 8; u += blockDim.x) {
      const uint4 s = __ldcv(sum + u);
      const uint4 r = h[u];
      uint4 o;
      o.x = pack_bf16x2(bf16_lo(r.x) + bf16_lo(s.x), bf16_hi(r.x) + bf16_hi(s.x));
      o.y = pack_bf16x2(bf16_lo(r.y) + bf16_lo(s.y), bf16_hi(r.y) + bf16_hi(s.y));
      o.z = pack_bf16x2(bf16_lo(r.z) + bf16_lo(s.z), bf16_hi(r.z) + bf16_hi(s.z));
      o.w = pack_bf16x2(bf16_lo(r.w) + bf16_lo(s.w), bf16_hi(r.w) + bf16_hi(s.w));
      h[u] = o;
      if (a.nw != nullptr) {
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
  }
  if (a.nw != nullptr) {
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
      v = warp_sum(v);
      if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float rstd = rsqrtf(red[0] / a.H + a.eps);
    if (ok) {
      uint4* xo = reinterpret_cast<uint4*>(a.x_out + (long long)t * a.H);
      for (int u = threadIdx.x; u < a.H / 8; u += blockDim.x) {
        const uint4 wq = reinterpret_cast<const uint4*>(a.nw)[u];
        const float wv[8] = {bf16_lo(wq.x), bf16_hi(wq.x), bf16_lo(wq.y), bf16_hi(wq.y),
                             bf16_lo(wq.z), bf16_hi(wq.z), bf16_lo(wq.w), bf16_hi(wq.w)};
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = wv[j] * __bfloat162float(__float2bfloat16_rn(row[u * 8 + j] * rstd));
        uint4 q;
        q.x = pack_bf16x2(o[0], o[1]); q.y = pack_bf16x2(o[2], o[3]);
        q.z = pack_bf16x2(o[4], o[5]); q.w = pack_bf16x2(o[6], o[7]);
        xo[u] = q;
      }
    }
  }
  // The last CTA of the launch advances this rank's epoch.
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

// h [T, H] += all-reduce over the group of each rank's partial (bf16 [T, H] at byte offset
// partial_off of its symmetric buffer); with norm_w, x_out = rmsnorm(h) * norm_w as well.
void nvls_allreduce(at::Tensor& h, const std::vector<int64_t>& peers, int64_t mc, int64_t rank,
                    int64_t flags1_off, int64_t flags2_off, int64_t partial_off, int64_t sum_off,
                    int64_t max_elems, const c10::optional<at::Tensor>& norm_w, double eps,
                    const c10::optional<at::Tensor>& x_out, const at::Tensor& status) {
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous() && h.dim() == 2,
              "nvls_allreduce: h [T, H] bf16 contiguous");
  const int world = static_cast<int>(peers.size());
  TORCH_CHECK(world >= 2 && world <= kMaxRanks && rank >= 0 && rank < world && mc != 0,
              "nvls_allreduce: group of 2..8 ranks with a multicast address");
  const int T = h.size(0), H = h.size(1);
  TORCH_CHECK(T <= kMaxRows && (long long)T * H <= max_elems && H % (8 * world) == 0,
              "nvls_allreduce: at most 256 rows, H a multiple of 8 x ranks, within the buffer");
  TORCH_CHECK(partial_off % 16 == 0 && sum_off % 16 == 0, "nvls_allreduce: 16-byte offsets");
  const bool norm = norm_w.has_value();
  if (norm) {
    TORCH_CHECK(x_out.has_value() && x_out->is_contiguous() && x_out->sizes() == h.sizes() &&
                    x_out->scalar_type() == at::kBFloat16 && norm_w->numel() == H &&
                    norm_w->scalar_type() == at::kBFloat16,
                "nvls_allreduce: x_out like h and a bf16 norm weight of H");
  }
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(h.device());
  NvlsArgs a{};
  for (int i = 0; i < world; ++i) a.peers[i] = peers[i];
  a.mc = mc;
  a.rank = static_cast<int>(rank);
  a.world = world;
  a.flags1_off = flags1_off;
  a.flags2_off = flags2_off;
  a.partial_off = partial_off;
  a.sum_off = sum_off;
  a.h = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  a.T = T;
  a.H = H;
  a.nw = norm ? reinterpret_cast<const __nv_bfloat16*>(norm_w->data_ptr()) : nullptr;
  a.eps = static_cast<float>(eps);
  a.x_out = norm ? reinterpret_cast<__nv_bfloat16*>(x_out->data_ptr()) : nullptr;
  a.status = status.data_ptr<int>();
  const size_t smem = norm ? static_cast<size_t>(H) * sizeof(float) : 0;
  if (smem > 48 * 1024) {
    check_cuda(cudaFuncSetAttribute(nvls_allreduce_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)),
               "cudaFuncSetAttribute(nvls_allreduce)");
  }
  launch_pdl(nvls_allreduce_kernel, dim3(T), dim3(kThreadsNvls), smem, at::cuda::getCurrentCUDAStream(),
             "nvls_allreduce launch", a);
}

}  // namespace sil
