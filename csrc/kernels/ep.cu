// Expert-parallel token dispatch and combine over NVLink peer memory (decode).
//
// Every rank of an EP group owns a symmetric buffer (same layout on every GPU,
// mapped by every peer through CUDA IPC):
//
//   state   u32[4]            epoch, arrival counters of the dispatch / combine / GEMM grids
//   dflag   u32[2][8]         dispatch flag [parity][source rank]
//   cflag   u32[2][8]         combine flag  [parity][expert-owner rank]
//   rows    u8 [2][W][T][H]   e4m3 token rows received from each source rank
//   scales  f32[2][W][T][H/128]
//   ids     i32[2][W][T][k]   global expert ids chosen for the received tokens
//   wts     f32[2][W][T][k]   their routing weights
//   slots   bf16[2][T][k][H]  weighted expert outputs of this rank's tokens, slot j of token t
//                             written by the rank owning the token's j-th expert
//
// One MoE layer (T tokens per rank, the same on every rank):
//   ep_dispatch  (source)  quantise each local row to e4m3 / 1x128 scales and store row,
//                          scales, expert ids and weights into every rank's buffer; the
//                          grid's last CTA raises dflag[par][rank] on every rank.
//   ep_recv_map  (owner)   wait for every source's dflag, map expert ids to local groups
//                          (remote experts -> a trailing group).
//   moe_permute            (existing kernel) group offsets and each assignment's sorted position.
//   ep_gather    (owner)   copy the e4m3 rows / scales of local assignments into expert order
//                          and record sorted position -> assignment for the epilogue.
//   grouped fp8 GEMMs      gate/up (SwiGLU) then down; the down GEMM's epilogue multiplies
//                          by the routing weight and stores bf16 straight into the source
//                          rank's slot (gemm_fp8.cu, kScatter), and its last CTA raises
//                          cflag[par][rank] on every rank.
//   ep_combine   (source)  wait for every owner's cflag, h[t] += sum_j slots[t][j] in slot
//                          order (deterministic), advance the epoch.
// Buffers alternate by epoch parity; a rank can only reach layer l+2's writes after every
// peer has passed layer l+1's waits, so a parity is never overwritten while it is read.
// Every wait is bounded (deadline + sticky status word).
//
// Reference: the expert dispatch / return plans of si/microsharding/moe.py:258-548 (host-side
// packing with a Python loop); here the packing is a device scatter over peer memory.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp8.h>
#include <torch/extension.h>

#include <vector>

#include "sil/ep.h"
#include "sil/host.h"
#include "sil/ptx.cuh"

namespace sil {

namespace {

__device__ __forceinline__ uint32_t ld_acq_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_rel_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t* state_of(const EpLayout& L, int r) {
  return reinterpret_cast<uint32_t*>(L.peers[r]);
}

__device__ __forceinline__ uint32_t read_epoch(const EpLayout& L) {
  return *reinterpret_cast<volatile uint32_t*>(state_of(L, L.rank)) + 1u;
}

// Grid-wide "last CTA" election on a counter in this rank's state words.  With `fence_sys`
// thread 0 issues a system-scope fence after the CTA barrier, before it counts in, which
// orders the CTA's peer stores before whatever the last CTA publishes.
__device__ __forceinline__ bool last_cta(const EpLayout& L, int which, bool fence_sys = false) {
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    if (fence_sys) __threadfence_system();
    uint32_t* ctr = state_of(L, L.rank) + which;
    const uint32_t old = atomicAdd(ctr, 1u);
    s_last = old == gridDim.x - 1;
    if (s_last) *reinterpret_cast<volatile uint32_t*>(ctr) = 0u;
  }
  __syncthreads();
  return s_last != 0;
}

// Wait until flag[par][src] == epoch on this rank for every source rank (thread 0 only).
__device__ __forceinline__ bool wait_flags(const EpLayout& L, long long off, int par, uint32_t epoch) {
  const uint32_t* f = reinterpret_cast<const uint32_t*>(L.peers[L.rank] + off) + par * 8;
  for (int r = 0; r < L.world; ++r) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t it = 0;
    while (ld_acq_sys(f + r) != epoch) {
      if ((++it & 255u) == 0) {
        if (load_status(L.status) != 0) return false;
        if (globaltimer_ns() - t0 > wait_limit_ns(L.status)) {
          raise_status(L.status, kStatusTimeoutPeer);
          return false;
        }
      }
    }
  }
  return true;
}

// One warp per (token, 128-column block): quantise and push to every rank.
__global__ void ep_dispatch_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                   const int* __restrict__ ids, const float* __restrict__ wts,
                                   const EpLayout L) {
  pdl_trigger();
  pdl_wait();
  const uint32_t epoch = read_epoch(L);
  const int par = epoch & 1;
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w < L.T * L.KB && load_status(L.status) == 0) {
    const int t = w / L.KB, kb = w % L.KB;
    const uint2 raw = *reinterpret_cast<const uint2*>(x + t * ldx + kb * 128 + lane * 4);
    float v[4] = {bf16_lo(raw.x), bf16_hi(raw.x), bf16_lo(raw.y), bf16_hi(raw.y)};
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = amax > 0.f ? amax / 448.f : 1.f;
    const float inv = 1.f / sc;
    const __nv_fp8x2_storage_t p0 =
        __nv_cvt_float2_to_fp8x2(make_float2(v[0] * inv, v[1] * inv), __NV_SATFINITE, __NV_E4M3);
    const __nv_fp8x2_storage_t p1 =
        __nv_cvt_float2_to_fp8x2(make_float2(v[2] * inv, v[3] * inv), __NV_SATFINITE, __NV_E4M3);
    const uint32_t packed = static_cast<uint32_t>(p0) | (static_cast<uint32_t>(p1) << 16);
    const long long row = (long long)(par * L.world + L.rank) * L.T + t;
    for (int p = 0; p < L.world; ++p) {
      uint8_t* base = reinterpret_cast<uint8_t*>(L.peers[p]);
      *reinterpret_cast<uint32_t*>(base + L.rows_off + row * L.H + kb * 128 + lane * 4) = packed;
      if (lane == 0) reinterpret_cast<float*>(base + L.scales_off)[row * L.KB + kb] = sc;
      if (kb == 0 && lane < L.k) {
        reinterpret_cast<int*>(base + L.ids_off)[row * L.k + lane] = ids[t * L.k + lane];
        reinterpret_cast<float*>(base + L.wts_off)[row * L.k + lane] = wts[t * L.k + lane];
      }
    }
  }
  if (last_cta(L, kEpCtrDispatch, /*fence_sys=*/true) && threadIdx.x == 0) {
    for (int p = 0; p < L.world; ++p)
      st_rel_sys(reinterpret_cast<uint32_t*>(L.peers[p] + L.dflag_off) + par * 8 + L.rank, epoch);
  }
}

// Wait for every source, then global expert ids -> local group ids ([W*T, k], el = remote).
__global__ void ep_recv_map_kernel(int* __restrict__ local_ids, const EpLayout L) {
  pdl_trigger();
  pdl_wait();
  const uint32_t epoch = read_epoch(L);
  const int par = epoch & 1;
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_flags(L, L.dflag_off, par, epoch);
  __syncthreads();
  const int n = L.world * L.T * L.k;
  const int* src = reinterpret_cast<const int*>(L.peers[L.rank] + L.ids_off) +
                   (long long)par * L.world * L.T * L.k;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int e = ok ? src[i] - L.e0 : -1;
    local_ids[i] = (e >= 0 && e < L.el) ? e : L.el;
  }
}

// One warp per routed assignment a (= (src * T + t) * k + j) whose sorted position
// p = pos[a] falls in a local expert group (p < offsets[el]): copy the token's e4m3 row and
// scales to row p, and record inv[p] = a for the scatter epilogue.
__global__ void ep_gather_kernel(const int* __restrict__ pos, const int* __restrict__ offsets,
                                 uint8_t* __restrict__ xq, float* __restrict__ xs, int* __restrict__ inv,
                                 const EpLayout L) {
  pdl_trigger();
  pdl_wait();
  const uint32_t epoch = read_epoch(L);
  const int par = epoch & 1;
  const int limit = offsets[L.el];
  const int n = L.world * L.T * L.k;
  const int lane = threadIdx.x & 31;
  const uint8_t* rbase = reinterpret_cast<const uint8_t*>(L.peers[L.rank] + L.rows_off);
  const float* sbase = reinterpret_cast<const float*>(L.peers[L.rank] + L.scales_off);
  for (int a = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; a < n;
       a += (gridDim.x * blockDim.x) >> 5) {
    const int p = pos[a];
    if (p >= limit) continue;
    const long long srow = (long long)par * L.world * L.T + a / L.k;  // src * T + t
    const uint4* s = reinterpret_cast<const uint4*>(rbase + srow * L.H);
    uint4* d = reinterpret_cast<uint4*>(xq + (long long)p * L.H);
    for (int u = lane; u < L.H / 16; u += 32) d[u] = s[u];
    for (int u = lane; u < L.KB; u += 32) xs[(long long)p * L.KB + u] = sbase[srow * L.KB + u];
    if (lane == 0) inv[p] = a;
  }
}

// Wait for every expert owner, then h[t] += sum_j slots[par][t][j] (slot order), bump epoch.
__global__ void ep_combine_kernel(__nv_bfloat16* __restrict__ h, long long ldh, const EpLayout L) {
  pdl_trigger();
  pdl_wait();
  const uint32_t epoch = read_epoch(L);
  const int par = epoch & 1;
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_flags(L, L.cflag_off, par, epoch);
  __syncthreads();
  const __nv_bfloat16* slots = reinterpret_cast<const __nv_bfloat16*>(L.peers[L.rank] + L.slots_off) +
                               (long long)par * L.T * L.k * L.H;
  const long long n = (long long)L.T * (L.H / 2);
  if (ok) {
    for (long long i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
      const int t = static_cast<int>(i / (L.H / 2));
      const int m = static_cast<int>(i % (L.H / 2)) * 2;
      uint32_t* hp = reinterpret_cast<uint32_t*>(h + t * ldh + m);
      const uint32_t hv = *hp;
      float a0 = bf16_lo(hv), a1 = bf16_hi(hv);
      for (int j = 0; j < L.k; ++j) {
        const uint32_t sv = __ldcv(reinterpret_cast<const unsigned int*>(
            slots + ((long long)t * L.k + j) * L.H + m));
        a0 += bf16_lo(sv);
        a1 += bf16_hi(sv);
      }
      *hp = pack_bf16x2(a0, a1);
    }
  }
  __threadfence();
  if (last_cta(L, kEpCtrCombine) && threadIdx.x == 0) {
    __threadfence();
    *reinterpret_cast<volatile uint32_t*>(state_of(L, L.rank)) = epoch;
  }
}

EpLayout make_layout(const std::vector<int64_t>& peers, int64_t rank, int64_t T, int64_t k,
                     int64_t H, int64_t e0, int64_t el, const std::vector<int64_t>& offs,
                     const at::Tensor& status) {
  TORCH_CHECK(peers.size() >= 1 && peers.size() <= 8, "ep: 1..8 ranks");
  TORCH_CHECK(offs.size() == 7, "ep: 7 buffer offsets");
  TORCH_CHECK(H % 128 == 0 && k <= 32, "ep: hidden % 128, top-k <= 32");
  EpLayout L{};
  for (size_t i = 0; i < peers.size(); ++i) L.peers[i] = peers[i];
  L.rank = static_cast<int>(rank);
  L.world = static_cast<int>(peers.size());
  L.T = static_cast<int>(T);
  L.k = static_cast<int>(k);
  L.H = static_cast<int>(H);
  L.KB = static_cast<int>(H / 128);
  L.e0 = static_cast<int>(e0);
  L.el = static_cast<int>(el);
  L.dflag_off = offs[0];
  L.cflag_off = offs[1];
  L.rows_off = offs[2];
  L.scales_off = offs[3];
  L.ids_off = offs[4];
  L.wts_off = offs[5];
  L.slots_off = offs[6];
  L.status = status.data_ptr<int>();
  return L;
}

int blocks_for(long long threads_needed) {
  const long long b = (threads_needed + 255) / 256;
  return static_cast<int>(std::max<long long>(1, std::min<long long>(b, 4 * 148)));
}

}  // namespace

EpLayout ep_make_layout(const std::vector<int64_t>& peers, int64_t rank, int64_t T, int64_t k,
                        int64_t H, int64_t e0, int64_t el, const std::vector<int64_t>& offs,
                        const at::Tensor& status) {
  return make_layout(peers, rank, T, k, H, e0, el, offs, status);
}

void ep_dispatch(const at::Tensor& x, const at::Tensor& ids, const at::Tensor& wts,
                 const std::vector<int64_t>& peers, int64_t rank, int64_t e0, int64_t el,
                 const std::vector<int64_t>& offs, const at::Tensor& status) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1 && x.stride(0) % 4 == 0,
              "ep_dispatch: x [T, H] bf16");
  TORCH_CHECK(ids.is_contiguous() && wts.is_contiguous() && ids.scalar_type() == at::kInt &&
                  wts.scalar_type() == at::kFloat,
              "ep_dispatch: ids int32 / wts fp32 [T, k]");
  const int T = x.size(0), H = x.size(1), k = ids.size(1);
  EpLayout L = make_layout(peers, rank, T, k, H, e0, el, offs, status);
  c10::cuda::CUDAGuard guard(x.device());
  launch_pdl(ep_dispatch_kernel, dim3(std::max(1, (T * (H / 128) * 32 + 255) / 256)), dim3(256), 0,
             at::cuda::getCurrentCUDAStream(), "ep_dispatch launch",
             reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (long long)x.stride(0),
             (const int*)ids.data_ptr<int>(), (const float*)wts.data_ptr<float>(), L);
}

void ep_recv_map(at::Tensor& local_ids, const std::vector<int64_t>& peers, int64_t rank, int64_t T,
                 int64_t k, int64_t H, int64_t e0, int64_t el, const std::vector<int64_t>& offs,
                 const at::Tensor& status) {
  EpLayout L = make_layout(peers, rank, T, k, H, e0, el, offs, status);
  TORCH_CHECK(local_ids.numel() == (long long)L.world * T * k && local_ids.is_contiguous(),
              "ep_recv_map: local ids [W*T, k]");
  c10::cuda::CUDAGuard guard(local_ids.device());
  launch_pdl(ep_recv_map_kernel, dim3(blocks_for((long long)L.world * T * k)), dim3(256), 0,
             at::cuda::getCurrentCUDAStream(), "ep_recv_map launch", local_ids.data_ptr<int>(), L);
}

// pos: moe_permute's assignment -> sorted position map; inv receives the inverse for the
// local rows.
void ep_gather(const at::Tensor& pos, const at::Tensor& offsets, at::Tensor& xq, at::Tensor& xs,
               at::Tensor& inv, const std::vector<int64_t>& peers, int64_t rank, int64_t T, int64_t k,
               int64_t H, int64_t e0, int64_t el, const std::vector<int64_t>& offs,
               const at::Tensor& status) {
  EpLayout L = make_layout(peers, rank, T, k, H, e0, el, offs, status);
  const long long n = (long long)L.world * T * k;
  TORCH_CHECK(pos.numel() == n && inv.numel() >= n && pos.scalar_type() == at::kInt &&
                  inv.scalar_type() == at::kInt,
              "ep_gather: pos / inv [W*T*k] int32");
  TORCH_CHECK(xq.size(1) == H && xs.size(1) == H / 128 && xq.size(0) >= n, "ep_gather: output shapes");
  c10::cuda::CUDAGuard guard(xq.device());
  launch_pdl(ep_gather_kernel, dim3(blocks_for(n * 32)), dim3(256), 0,
             at::cuda::getCurrentCUDAStream(), "ep_gather launch", pos.data_ptr<int>(),
             offsets.data_ptr<int>(), xq.data_ptr<uint8_t>(), xs.data_ptr<float>(), inv.data_ptr<int>(),
             L);
}

void ep_combine(at::Tensor& h, const std::vector<int64_t>& peers, int64_t rank, int64_t k,
                int64_t e0, int64_t el, const std::vector<int64_t>& offs, const at::Tensor& status) {
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.stride(1) == 1, "ep_combine: h [T, H] bf16");
  const int T = h.size(0), H = h.size(1);
  EpLayout L = make_layout(peers, rank, T, k, H, e0, el, offs, status);
  c10::cuda::CUDAGuard guard(h.device());
  launch_pdl(ep_combine_kernel, dim3(blocks_for((long long)T * H / 2)), dim3(256), 0,
             at::cuda::getCurrentCUDAStream(), "ep_combine launch",
             reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), (long long)h.stride(0), L);
}

}  // namespace sil
