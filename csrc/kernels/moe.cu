// Mixture-of-experts routing kernels: top-k selection, permutation into
// expert-sorted order, row gather, and the weighted combine.
//
//  * moe_topk: one warp per token over the router logits (fp32).  Softmax
//    routing (Mixtral / Qwen3-MoE: softmax over all experts, top-k, optional
//    renormalisation) or sigmoid routing with a selection bias and
//    group-limited top-k (DeepSeek-V3 / Kimi-K2: group score = sum of the
//    group's two best biased scores, keep topk_group groups, top-k inside
//    them, weights = unbiased sigmoid scores renormalised and multiplied by
//    routed_scaling_factor).  Ties go to the lowest expert id.
//  * moe_permute: per-expert counts, exclusive offsets and each (token, slot)
//    assignment's row in the expert-sorted buffer; the gathered rows feed the
//    grouped tcgen05 GEMM.  Row order inside an expert follows arrival order,
//    which does not affect any result (rows are independent and the combine
//    sums in slot order).
//  * moe_combine: out[t] (+)= sum_s w[t,s] * y[row(t,s)] in slot order (fp32),
//    optionally plus a residual and a shared-expert output, rounded to bf16.
//
// Reference semantics: si/model/qwen3.py:1311-1325 and
// si/microsharding/moe.py:429-488 (softmax top-k, renorm, index_add combine);
// si/backends/colibri/sparse_moe.py:60-143 (sigmoid + bias + group top-k).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sil/host.h"
#include "sil/ptx.cuh"

namespace sil {
namespace {

constexpr int kMaxE = 512;
constexpr int kMaxK = 16;
constexpr int kMaxPerLane = kMaxE / 32;

// Warp-wide argmax with lowest-index tie break.  Invalid lanes pass -inf / big index.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
}

__global__ void moe_topk_kernel(const float* __restrict__ logits, int T, int E, int K,
                                int mode /*0 softmax, 1 sigmoid-group*/, int renorm,
                                const float* __restrict__ bias, int n_group, int topk_group,
                                float scale, int* __restrict__ ids, float* __restrict__ weights) {
  pdl_trigger();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* row = logits + (long long)warp * E;
  float sc[kMaxPerLane];   // probability (softmax) or sigmoid score
  float sel[kMaxPerLane];  // selection key (score + bias for sigmoid routing)
  const int per = (E + 31) / 32;
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kMaxPerLane; ++j) {
    const int e = j * 32 + lane;
    sc[j] = (j < per && e < E) ? row[e] : -INFINITY;
    mx = fmaxf(mx, sc[j]);
  }
  if (mode == 0) {
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
      const float p = sc[j] == -INFINITY ? 0.f : __expf(sc[j] - mx);
      sc[j] = p;
      sum += p;
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
      sc[j] *= inv;
      const int e = j * 32 + lane;
      sel[j] = (j < per && e < E) ? sc[j] : -INFINITY;
    }
  } else {
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
      const int e = j * 32 + lane;
      const bool ok = j < per && e < E;
      const float s = ok ? 1.f / (1.f + __expf(-sc[j])) : 0.f;
      sc[j] = s;
      sel[j] = ok ? s + (bias ? bias[e] : 0.f) : -INFINITY;
    }
    if (n_group > 1) {
      // Group score = sum of the two best selection keys in the group.
      const int gsize = E / n_group;
      __shared__ float gscore_s[8][64];
      float* gscore = gscore_s[(threadIdx.x >> 5) & 7];
      for (int g = 0; g < n_group; ++g) {
        float b1 = -INFINITY, b2 = -INFINITY;
#pragma unroll
        for (int j = 0; j < kMaxPerLane; ++j) {
          const int e = j * 32 + lane;
          if (j < per && e < E && e / gsize == g) {
            const float v = sel[j];
            if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) { b2 = v; }
          }
        }
        // Warp-merge the per-lane top-2 lists.
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float o1 = __shfl_xor_sync(0xffffffffu, b1, o);
          const float o2 = __shfl_xor_sync(0xffffffffu, b2, o);
          float n1 = fmaxf(b1, o1);
          float n2 = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
          b1 = n1; b2 = n2;
        }
        if (lane == 0) gscore[g] = b1 + b2;
      }
      __syncwarp();
      // Keep the topk_group best groups (lowest group id on ties).
      unsigned long long keep = 0ull;
      for (int r = 0; r < topk_group; ++r) {
        float bv = -INFINITY;
        int bi = 1 << 30;
        for (int g = lane; g < n_group; g += 32)
          if (!((keep >> g) & 1ull)) {
            const float v = gscore[g];
            if (v > bv || (v == bv && g < bi)) { bv = v; bi = g; }
          }
        warp_argmax(bv, bi);
        keep |= 1ull << bi;
      }
#pragma unroll
      for (int j = 0; j < kMaxPerLane; ++j) {
        const int e = j * 32 + lane;
        if (j < per && e < E && !((keep >> (e / gsize)) & 1ull)) sel[j] = -INFINITY;
      }
    }
  }
  // k rounds of warp argmax over the selection keys.
  float wsum = 0.f;
  float myw = 0.f;
  int myid = 0;
  for (int r = 0; r < K; ++r) {
    float bv = -INFINITY;
    int bi = 1 << 30;
    int bj = -1;
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
      const int e = j * 32 + lane;
      if (sel[j] > bv || (sel[j] == bv && e < bi)) { bv = sel[j]; bi = e; bj = j; }
    }
    int wi = bi;
    float wv = bv;
    warp_argmax(wv, wi);
    // Owner lane reads the routing weight and retires the expert.
    float w = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j)
      if (j * 32 + lane == wi) { w = sc[j]; sel[j] = -INFINITY; }
    w = warp_sum(w);  // exactly one lane contributed
    (void)bj;
    wsum += w;
    if (lane == r) { myw = w; myid = wi; }
  }
  if (lane < K) {
    float w = myw;
    if (renorm) w = w / wsum;
    weights[(long long)warp * K + lane] = w * scale;
    ids[(long long)warp * K + lane] = myid;
  }
}

// Counts, offsets (exclusive, E+1) and rows.  Single CTA per call for E <= 1024
// (counting in shared memory, then a scan), which also keeps it graph-capturable.
__global__ void moe_permute_kernel(const int* __restrict__ ids, int TK, int E,
                                   int* __restrict__ offsets, int* __restrict__ rows,
                                   int* __restrict__ counts_out) {
  pdl_trigger();
  pdl_wait();
  __shared__ int cnt[1024];
  __shared__ int base[1025];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < TK; i += blockDim.x) atomicAdd(&cnt[ids[i]], 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int e = 0; e < E; ++e) {
      base[e] = s;
      s += cnt[e];
    }
    base[E] = s;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) offsets[e] = base[e];
  if (counts_out)
    for (int e = threadIdx.x; e < E; e += blockDim.x) counts_out[e] = cnt[e];
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < TK; i += blockDim.x) {
    const int e = ids[i];
    rows[i] = base[e] + atomicAdd(&cnt[e], 1);
  }
}

// xp[rows[t*K+s]] = x[t]  (bf16 rows, H % 8 == 0)
__global__ void moe_gather_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                  const int* __restrict__ rows, int K, int H,
                                  __nv_bfloat16* __restrict__ xp) {
  pdl_trigger();
  pdl_wait();
  const int a = blockIdx.x;  // assignment index t*K + s
  const int t = a / K;
  const uint4* src = reinterpret_cast<const uint4*>(x + (long long)t * ldx);
  uint4* dst = reinterpret_cast<uint4*>(xp + (long long)rows[a] * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// out[t] = (res[t]) + (shared[t]) + sum_s w[t,s] * y[rows[t*K+s]]
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ rows,
                                   const float* __restrict__ w, int K, int H,
                                   const int* __restrict__ row_limit,
                                   const __nv_bfloat16* __restrict__ res, long long ldr,
                                   const __nv_bfloat16* __restrict__ shared, long long lds,
                                   __nv_bfloat16* __restrict__ out, long long ldo) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int lim = row_limit ? *row_limit : 0x7fffffff;  // rows >= lim belong to other ranks
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int s = 0; s < K; ++s) {
      if (rows[t * K + s] >= lim) continue;
      const float ws = w[(long long)t * K + s];
      const uint4 q = *reinterpret_cast<const uint4*>(y + (long long)rows[t * K + s] * H + i);
      acc[0] += ws * bf16_lo(q.x); acc[1] += ws * bf16_hi(q.x);
      acc[2] += ws * bf16_lo(q.y); acc[3] += ws * bf16_hi(q.y);
      acc[4] += ws * bf16_lo(q.z); acc[5] += ws * bf16_hi(q.z);
      acc[6] += ws * bf16_lo(q.w); acc[7] += ws * bf16_hi(q.w);
    }
    if (shared) {
      const uint4 q = *reinterpret_cast<const uint4*>(shared + (long long)t * lds + i);
      acc[0] += bf16_lo(q.x); acc[1] += bf16_hi(q.x); acc[2] += bf16_lo(q.y); acc[3] += bf16_hi(q.y);
      acc[4] += bf16_lo(q.z); acc[5] += bf16_hi(q.z); acc[6] += bf16_lo(q.w); acc[7] += bf16_hi(q.w);
    }
    if (res) {
      const uint4 q = *reinterpret_cast<const uint4*>(res + (long long)t * ldr + i);
      acc[0] += bf16_lo(q.x); acc[1] += bf16_hi(q.x); acc[2] += bf16_lo(q.y); acc[3] += bf16_hi(q.y);
      acc[4] += bf16_lo(q.z); acc[5] += bf16_hi(q.z); acc[6] += bf16_lo(q.w); acc[7] += bf16_hi(q.w);
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]); o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]); o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + (long long)t * ldo + i) = o;
  }
}

}  // namespace

void moe_topk(const at::Tensor& logits, int64_t k, int64_t mode, bool renorm,
              const c10::optional<at::Tensor>& bias, int64_t n_group, int64_t topk_group,
              double scale, at::Tensor& ids, at::Tensor& weights) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.is_contiguous(), "moe_topk: fp32 logits");
  const int T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(E <= kMaxE && k <= kMaxK && k <= 32 && k <= E, "moe_topk: E <= 512, k <= 16");
  TORCH_CHECK(n_group <= 64 && (n_group <= 1 || E % n_group == 0), "moe_topk: groups");
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(logits.device());
  const int threads = 256;
  const int blocks = (T * 32 + threads - 1) / threads;
  launch_pdl(moe_topk_kernel, dim3(blocks), dim3(threads), 0, at::cuda::getCurrentCUDAStream(),
             "moe_topk launch", (const float*)logits.data_ptr<float>(), T, E, (int)k, (int)mode,
             (int)renorm, bias.has_value() ? (const float*)bias->data_ptr<float>() : nullptr,
             (int)n_group, (int)topk_group, (float)scale, ids.data_ptr<int>(),
             weights.data_ptr<float>());
}

void moe_permute(const at::Tensor& ids, int64_t E, at::Tensor& offsets, at::Tensor& rows,
                 const c10::optional<at::Tensor>& counts) {
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous(), "moe_permute: int32 ids");
  TORCH_CHECK(E <= 1024, "moe_permute: at most 1024 experts");
  const int TK = ids.numel();
  c10::cuda::CUDAGuard guard(ids.device());
  launch_pdl(moe_permute_kernel, dim3(1), dim3(1024), 0, at::cuda::getCurrentCUDAStream(),
             "moe_permute launch", (const int*)ids.data_ptr<int>(), TK, (int)E,
             offsets.data_ptr<int>(), rows.data_ptr<int>(),
             counts.has_value() ? counts->data_ptr<int>() : nullptr);
}

void moe_gather(const at::Tensor& x, const at::Tensor& rows, int64_t k, at::Tensor& xp) {
  const int TK = rows.numel(), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && x.stride(1) == 1, "moe_gather: H % 8");
  if (TK == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  launch_pdl(moe_gather_kernel, dim3(TK), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
             "moe_gather launch", reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
             (long long)x.stride(0), (const int*)rows.data_ptr<int>(), (int)k, H,
             reinterpret_cast<__nv_bfloat16*>(xp.data_ptr()));
}

void moe_combine(const at::Tensor& y, const at::Tensor& rows, const at::Tensor& w, int64_t k,
                 const c10::optional<at::Tensor>& res, const c10::optional<at::Tensor>& shared,
                 at::Tensor& out, const c10::optional<at::Tensor>& row_limit) {
  const int T = out.size(0), H = out.size(1);
  TORCH_CHECK(H % 8 == 0 && y.size(1) == H, "moe_combine: shapes");
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(out.device());
  launch_pdl(moe_combine_kernel, dim3(T), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
             "moe_combine launch", reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()),
             (const int*)rows.data_ptr<int>(), (const float*)w.data_ptr<float>(), (int)k, H,
             row_limit.has_value() ? (const int*)row_limit->data_ptr<int>() : nullptr,
             res.has_value() ? reinterpret_cast<const __nv_bfloat16*>(res->data_ptr()) : nullptr,
             res.has_value() ? (long long)res->stride(0) : 0LL,
             shared.has_value() ? reinterpret_cast<const __nv_bfloat16*>(shared->data_ptr()) : nullptr,
             shared.has_value() ? (long long)shared->stride(0) : 0LL,
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (long long)out.stride(0));
}

}  // namespace sil
