// Memory-bound per-token kernels of the decoder: embedding gather, RMSNorm
// (optionally fused with a residual add), q/k-norm + RoPE + paged KV-cache
// write, and greedy argmax over logits.
//
// Reference semantics: RMSNorm computes the variance in fp32 and multiplies
// the bf16-rounded normalised value by the weight (HF Llama/Qwen3 RMSNorm as
// used through si/model/qwen3.py:517-546 and si/microsharding/dense.py:146-166);
// RoPE is the rotate-half form with a host-built fp32 cos/sin table
// (si/microsharding/dense.py:169-219); greedy argmax breaks ties toward the
// lowest token id (si/model/qwen3_sampling.py:79-96, si/microsharding/dense.py:825-838).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp8.h>
#include <torch/extension.h>

#include "sil/host.h"
#include "sil/ptx.cuh"

namespace sil {
namespace {

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float s = lane < nw ? red[lane] : 0.f;
  s = warp_sum(s);
  __syncthreads();
  return s;
}

// y = rmsnorm(x (+ r)) * w;  when `res_out` is given, it receives x + r (bf16).
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                               const __nv_bfloat16* __restrict__ r, long long ldr,
                               __nv_bfloat16* __restrict__ res_out, long long ldro,
                               const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y,
                               long long ldy, int H, float eps, uint8_t* __restrict__ yq,
                               float* __restrict__ ys) {
  __shared__ float red[32];
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * ldx;
  extern __shared__ float vals[];  // H floats
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    uint4 q = *reinterpret_cast<const uint4*>(xr + i);
    float v[8] = {bf16_lo(q.x), bf16_hi(q.x), bf16_lo(q.y), bf16_hi(q.y),
                  bf16_lo(q.z), bf16_hi(q.z), bf16_lo(q.w), bf16_hi(q.w)};
    if (r != nullptr) {
      uint4 p = *reinterpret_cast<const uint4*>(r + row * ldr + i);
      float u[8] = {bf16_lo(p.x), bf16_hi(p.x), bf16_lo(p.y), bf16_hi(p.y),
                    bf16_lo(p.z), bf16_hi(p.z), bf16_lo(p.w), bf16_hi(p.w)};
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __bfloat162float(__float2bfloat16_rn(v[j] + u[j]));
      uint4 o;
      o.x = pack_bf16x2(v[0], v[1]); o.y = pack_bf16x2(v[2], v[3]);
      o.z = pack_bf16x2(v[4], v[5]); o.w = pack_bf16x2(v[6], v[7]);
      *reinterpret_cast<uint4*>(res_out + row * ldro + i) = o;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      vals[i + j] = v[j];
      ss += v[j] * v[j];
    }
  }
  const float tot = block_sum(ss, red);
  const float rstd = rsqrtf(tot / H + eps);
  // Every thread runs the same number of iterations so the 16-lane shuffles of the
  // e4m3 path see full warps; out-of-range lanes carry zeros.
  for (int base = 0; base < H; base += blockDim.x * 8) {
    const int i = base + threadIdx.x * 8;
    const bool in = i < H;
    float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (in) {
      uint4 wq = *reinterpret_cast<const uint4*>(w + i);
      float wv[8] = {bf16_lo(wq.x), bf16_hi(wq.x), bf16_lo(wq.y), bf16_hi(wq.y),
                     bf16_lo(wq.z), bf16_hi(wq.z), bf16_lo(wq.w), bf16_hi(wq.w)};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float nrm = __bfloat162float(__float2bfloat16_rn(vals[i + j] * rstd));
        o[j] = __bfloat162float(__float2bfloat16_rn(wv[j] * nrm));
      }
      uint4 q;
      q.x = pack_bf16x2(o[0], o[1]); q.y = pack_bf16x2(o[2], o[3]);
      q.z = pack_bf16x2(o[4], o[5]); q.w = pack_bf16x2(o[6], o[7]);
      *reinterpret_cast<uint4*>(y + row * ldy + i) = q;
    }
    if (yq != nullptr) {
      // e4m3 with one scale per 128 columns (16 lanes x 8 values), like quant_fp8_1x128.
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(o[j]));
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      const float sc = amax > 0.f ? amax / 448.f : 1.f;
      const float inv = 1.f / sc;
      if (in) {
        uint32_t pk[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const __nv_fp8x2_storage_t a = __nv_cvt_float2_to_fp8x2(
              make_float2(o[4 * h] * inv, o[4 * h + 1] * inv), __NV_SATFINITE, __NV_E4M3);
          const __nv_fp8x2_storage_t b = __nv_cvt_float2_to_fp8x2(
              make_float2(o[4 * h + 2] * inv, o[4 * h + 3] * inv), __NV_SATFINITE, __NV_E4M3);
          pk[h] = static_cast<uint32_t>(a) | (static_cast<uint32_t>(b) << 16);
        }
        *reinterpret_cast<uint2*>(yq + (long long)row * H + i) = make_uint2(pk[0], pk[1]);
        if ((threadIdx.x & 15) == 0) ys[(long long)row * (H / 128) + i / 128] = sc;
      }
    }
  }
}

// One warp per (token, head).  qkv: [T, (Hq + 2*Hkv) * 128]; q heads are
// rotated in place; k heads are normalised/rotated and written with v into
// the paged cache at `slots[t]` (= page * 64 + offset; negative = skip).
__global__ void rope_kv_write_kernel(__nv_bfloat16* __restrict__ qkv, long long ld,
                                     const int* __restrict__ positions,
                                     const int* __restrict__ slots,
                                     const float* __restrict__ cos_sin,  // [max_pos, 128]
                                     const __nv_bfloat16* __restrict__ q_norm_w,
                                     const __nv_bfloat16* __restrict__ k_norm_w, float eps,
                                     __nv_bfloat16* __restrict__ k_cache,
                                     __nv_bfloat16* __restrict__ v_cache, int T, int Hq, int Hkv) {
  pdl_trigger();
  pdl_wait();
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = Hq + 2 * Hkv;
  const int tok = warp_global / heads;
  const int hh = warp_global % heads;
  if (tok >= T) return;
  __nv_bfloat16* row = qkv + tok * ld + hh * 128;
  const int d0 = 2 * lane;  // this lane owns dims d0, d0+1, d0+64, d0+65
  uint32_t lo = *reinterpret_cast<const uint32_t*>(row + d0);
  uint32_t hi = *reinterpret_cast<const uint32_t*>(row + d0 + 64);
  float x0 = bf16_lo(lo), x1 = bf16_hi(lo), x2 = bf16_lo(hi), x3 = bf16_hi(hi);
  const int slot = slots[tok];
  if (hh >= Hq + Hkv) {  // value head: copy into the cache
    if (slot >= 0) {
      const int kvh = hh - Hq - Hkv;
      const long long base = ((long long)(slot >> 6) * Hkv + kvh) * 64 * 128 + (slot & 63) * 128;
      *reinterpret_cast<uint32_t*>(v_cache + base + d0) = lo;
      *reinterpret_cast<uint32_t*>(v_cache + base + d0 + 64) = hi;
    }
    return;
  }
  const bool is_q = hh < Hq;
  const __nv_bfloat16* nw = is_q ? q_norm_w : k_norm_w;
  if (nw != nullptr) {
    const float ss = warp_sum(x0 * x0 + x1 * x1 + x2 * x2 + x3 * x3);
    const float rstd = rsqrtf(ss / 128.f + eps);
    x0 = __bfloat162float(nw[d0]) * __bfloat162float(__float2bfloat16_rn(x0 * rstd));
    x1 = __bfloat162float(nw[d0 + 1]) * __bfloat162float(__float2bfloat16_rn(x1 * rstd));
    x2 = __bfloat162float(nw[d0 + 64]) * __bfloat162float(__float2bfloat16_rn(x2 * rstd));
    x3 = __bfloat162float(nw[d0 + 65]) * __bfloat162float(__float2bfloat16_rn(x3 * rstd));
    x0 = __bfloat162float(__float2bfloat16_rn(x0));
    x1 = __bfloat162float(__float2bfloat16_rn(x1));
    x2 = __bfloat162float(__float2bfloat16_rn(x2));
    x3 = __bfloat162float(__float2bfloat16_rn(x3));
  }
  const float* cs = cos_sin + (long long)positions[tok] * 128;
  const float c0 = cs[d0], c1 = cs[d0 + 1], s0 = cs[64 + d0], s1 = cs[64 + d0 + 1];
  const float y0 = x0 * c0 - x2 * s0;
  const float y1 = x1 * c1 - x3 * s1;
  const float y2 = x2 * c0 + x0 * s0;
  const float y3 = x3 * c1 + x1 * s1;
  const uint32_t olo = pack_bf16x2(y0, y1), ohi = pack_bf16x2(y2, y3);
  if (is_q) {
    *reinterpret_cast<uint32_t*>(row + d0) = olo;
    *reinterpret_cast<uint32_t*>(row + d0 + 64) = ohi;
  } else if (slot >= 0) {
    const int kvh = hh - Hq;
    const long long base = ((long long)(slot >> 6) * Hkv + kvh) * 64 * 128 + (slot & 63) * 128;
    *reinterpret_cast<uint32_t*>(k_cache + base + d0) = olo;
    *reinterpret_cast<uint32_t*>(k_cache + base + d0 + 64) = ohi;
  }
}

__global__ void embedding_kernel(const long long* __restrict__ ids,
                                 const __nv_bfloat16* __restrict__ table, int H,
                                 __nv_bfloat16* __restrict__ out, long long ldo, long long vocab) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  long long id = ids[row];
  if (id < 0 || id >= vocab) id = 0;  // out-of-range ids map to token 0 (checked on host in tests)
  const uint4* src = reinterpret_cast<const uint4*>(table + id * H);
  uint4* dst = reinterpret_cast<uint4*>(out + row * ldo);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// Greedy argmax per row of fp32 logits; ties resolve to the lowest index.
__global__ void argmax_kernel(const float* __restrict__ logits, long long ld, int V,
                              long long* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const float* row = logits + blockIdx.x * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const bool vec = (ld % 4 == 0) && (V % 4 == 0);
  if (vec) {
    for (int i = threadIdx.x * 4; i < V; i += blockDim.x * 4) {
      float4 q = *reinterpret_cast<const float4*>(row + i);
      if (q.x > best) { best = q.x; bi = i; }
      if (q.y > best) { best = q.y; bi = i + 1; }
      if (q.z > best) { best = q.z; bi = i + 2; }
      if (q.w > best) { best = q.w; bi = i + 3; }
    }
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float v = row[i];
      if (v > best) { best = v; bi = i; }
    }
  }
  // Reduce (value desc, index asc).
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  }
}

// Greedy argmax of one logits row split over a cluster of kArgmaxParts CTAs: CTA p scans
// its quarter of the vocabulary (a CTA streams ~50 GB/s, so one CTA per 128k-entry row was
// latency-bound), keeps its (value, index) in shared memory, and after a cluster barrier CTA
// 0 combines the parts through distributed shared memory (largest value, lowest index on
// ties, as the single-CTA kernel).  Every thread passes both cluster barriers exactly once.
constexpr int kArgmaxParts = 4;

__global__ void __launch_bounds__(1024)
    argmax_cluster_kernel(const float* __restrict__ logits, long long ld, int V,
                          long long* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ float part_v;
  __shared__ int part_i;
  pdl_trigger();
  pdl_wait();
  uint32_t part;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(part));
  const int row_id = blockIdx.x / kArgmaxParts;
  const float* row = logits + row_id * ld;
  const int chunk = ((V + kArgmaxParts - 1) / kArgmaxParts + 3) & ~3;
  const int lo = static_cast<int>(part) * chunk;
  const int hi = min(V, lo + chunk);
  float best = -INFINITY;
  int bi = 0x7fffffff;
  if ((ld % 4 == 0) && (V % 4 == 0)) {
    for (int i = lo + threadIdx.x * 4; i < hi; i += blockDim.x * 4) {
      const float4 q = *reinterpret_cast<const float4*>(row + i);
      if (q.x > best) { best = q.x; bi = i; }
      if (q.y > best) { best = q.y; bi = i + 1; }
      if (q.z > best) { best = q.z; bi = i + 2; }
      if (q.w > best) { best = q.w; bi = i + 3; }
    }
  } else {
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
      const float v = row[i];
      if (v > best) { best = v; bi = i; }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) { part_v = best; part_i = bi; }
  }
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
  if (part == 0 && threadIdx.x == 0) {
    float b = part_v;
    int i0 = part_i;
    for (uint32_t p = 1; p < kArgmaxParts; ++p) {
      uint32_t av, ai;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(av) : "r"(smem_u32(&part_v)), "r"(p));
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ai) : "r"(smem_u32(&part_i)), "r"(p));
      float ov;
      int oi;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(ov) : "r"(av) : "memory");
      asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(oi) : "r"(ai) : "memory");
      if (ov > b || (ov == b && oi < i0)) { b = ov; i0 = oi; }
    }
    out[row_id] = i0 == 0x7fffffff ? 0 : i0;
  }
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

}  // namespace

void rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual,
             const c10::optional<at::Tensor>& residual_out, const at::Tensor& w, at::Tensor& y,
             double eps, const c10::optional<at::Tensor>& yq, const c10::optional<at::Tensor>& ys) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
              "rmsnorm: x must be 2-D bf16 with contiguous rows");
  const int T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && w.numel() == H, "rmsnorm: H must be a multiple of 8");
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  const __nv_bfloat16* rp = nullptr;
  __nv_bfloat16* rop = nullptr;
  long long ldr = 0, ldro = 0;
  if (residual.has_value()) {
    TORCH_CHECK(residual_out.has_value(), "rmsnorm: residual_out required with residual");
    rp = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    ldr = residual->stride(0);
    rop = reinterpret_cast<__nv_bfloat16*>(residual_out->data_ptr());
    ldro = residual_out->stride(0);
  }
  uint8_t* qp = nullptr;
  float* sp = nullptr;
  if (yq.has_value()) {
    TORCH_CHECK(ys.has_value() && H % 128 == 0 && yq->is_contiguous() && ys->is_contiguous() &&
                    yq->numel() == (long long)T * H && ys->numel() == (long long)T * (H / 128),
                "rmsnorm: e4m3 output [T, H] with scales [T, H/128] (H % 128 == 0)");
    qp = reinterpret_cast<uint8_t*>(yq->data_ptr());
    sp = ys->data_ptr<float>();
  }
  const int threads = std::min(1024, std::max(32, ((H / 8 + 31) / 32) * 32));
  launch_pdl(rmsnorm_kernel, dim3(T), dim3(threads), H * sizeof(float),
             at::cuda::getCurrentCUDAStream(), "rmsnorm launch",
             reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (long long)x.stride(0), rp, ldr,
             rop, ldro, reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
             reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), (long long)y.stride(0), H,
             static_cast<float>(eps), qp, sp);
}

void rope_kv_write(at::Tensor& qkv, const at::Tensor& positions, const at::Tensor& slots,
                   const at::Tensor& cos_sin, const c10::optional<at::Tensor>& q_norm_w,
                   const c10::optional<at::Tensor>& k_norm_w, double eps, at::Tensor& k_cache,
                   at::Tensor& v_cache, int64_t Hq, int64_t Hkv) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1, "rope_kv_write: qkv");
  TORCH_CHECK(qkv.size(1) == (Hq + 2 * Hkv) * 128, "rope_kv_write: head_dim must be 128");
  TORCH_CHECK(positions.scalar_type() == at::kInt && slots.scalar_type() == at::kInt,
              "rope_kv_write: int32 positions/slots");
  const int T = qkv.size(0);
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(qkv.device());
  const long long warps = (long long)T * (Hq + 2 * Hkv);
  const int threads = 256;
  const long long blocks = (warps * 32 + threads - 1) / threads;
  const __nv_bfloat16* qn =
      q_norm_w.has_value() ? reinterpret_cast<const __nv_bfloat16*>(q_norm_w->data_ptr()) : nullptr;
  const __nv_bfloat16* kn =
      k_norm_w.has_value() ? reinterpret_cast<const __nv_bfloat16*>(k_norm_w->data_ptr()) : nullptr;
  launch_pdl(rope_kv_write_kernel, dim3(blocks), dim3(threads), 0,
             at::cuda::getCurrentCUDAStream(), "rope_kv_write launch",
             reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), (long long)qkv.stride(0),
             (const int*)positions.data_ptr<int>(), (const int*)slots.data_ptr<int>(),
             (const float*)cos_sin.data_ptr<float>(), qn, kn, static_cast<float>(eps),
             reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()),
             reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()), T, (int)Hq, (int)Hkv);
}

void embedding(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && table.scalar_type() == at::kBFloat16,
              "embedding: int64 ids, bf16 table");
  const int T = ids.numel(), H = table.size(1);
  TORCH_CHECK(H % 8 == 0, "embedding: H % 8");
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(ids.device());
  launch_pdl(embedding_kernel, dim3(T), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             "embedding launch", reinterpret_cast<const long long*>(ids.data_ptr<int64_t>()),
             reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()), H,
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (long long)out.stride(0),
             (long long)table.size(0));
}

void argmax(const at::Tensor& logits, at::Tensor& out) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1,
              "argmax: fp32 [T, V]");
  TORCH_CHECK(out.scalar_type() == at::kLong, "argmax: int64 output");
  const int T = logits.size(0);
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(logits.device());
  const float* lp = logits.data_ptr<float>();
  const long long ld = logits.stride(0);
  const int V = static_cast<int>(logits.size(1));
  long long* op = reinterpret_cast<long long*>(out.data_ptr<int64_t>());
  if (V < 4096) {  // short rows: one CTA per row
    launch_pdl(argmax_kernel, dim3(T), dim3(1024), 0, at::cuda::getCurrentCUDAStream(),
               "argmax launch", lp, ld, V, op);
    return;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(T * kArgmaxParts, 1, 1);
  cfg.blockDim = dim3(1024, 1, 1);
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = kArgmaxParts;
  attr[na].val.clusterDim.y = 1;
  attr[na].val.clusterDim.z = 1;
  ++na;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  check_cuda(cudaLaunchKernelEx(&cfg, argmax_cluster_kernel, lp, ld, V, op), "argmax launch");
}

}  // namespace sil
