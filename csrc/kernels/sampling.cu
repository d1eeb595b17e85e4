// Stochastic token sampling on the device: repetition penalty, temperature,
// top-k and top-p (nucleus) truncation, then an exact categorical draw.
//
// One CTA per row (1024 threads) over fp32 logits:
//  1. penalty: logits of tokens in the row's history are divided by the
//     penalty when positive and multiplied when negative;
//  2. z = logits / temperature, m = max z;
//  3. top-k threshold: radix select over the order-preserving integer image
//     of z (four 8-bit digit passes, histograms in shared memory) gives the
//     k-th largest value; ties at the threshold are kept;
//  4. top-p threshold: the same radix walk over probability mass
//     exp(z - m) (float histograms), keeping the smallest high-probability
//     set whose mass reaches top_p of the (top-k truncated) total;
//  5. Gumbel-max draw: argmax over survivors of z + g, g = -log(-log(u)),
//     u from cuRAND Philox4x32-10 keyed by (seed, row, offset), which samples
//     exactly from the renormalised truncated distribution.
// Greedy rows (temperature == 0) take the lowest-id argmax.
//
// Reference semantics: si/model/qwen3_sampling.py:10-188 (temperature,
// repetition penalty, top-k threshold, top-p sort/cumsum, per-request generators).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <curand_kernel.h>
#include <torch/extension.h>

#include "sil/host.h"
#include "sil/ptx.cuh"

namespace sil {
namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ uint32_t ordered(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float from_ordered(uint32_t o) {
  const uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
  return __uint_as_float(u);
}

struct SampleArgs {
  float* logits;            // [B, V] (modified in place by the penalty)
  long long ld;
  int V;
  const float* temperature; // [B]
  const int* top_k;         // [B] (0 = off)
  const float* top_p;       // [B] (1 = off)
  const float* penalty;     // [B] (1 = off)
  const long long* history; // [B, Hmax] token ids (or null)
  const int* history_len;   // [B]
  int hmax;
  const long long* seeds;   // [B]
  const long long* offsets; // [B] per-request draw counter
  long long* out;           // [B]
};

__global__ void __launch_bounds__(kThreads) sample_kernel(SampleArgs a) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  float* lg = a.logits + (long long)row * a.ld;
  const int V = a.V;
  __shared__ unsigned int hist[256];
  __shared__ float hmass[256];
  __shared__ float red_f[32];
  __shared__ int red_i[32];
  __shared__ uint32_t s_prefix;
  __shared__ float s_remain;
  __shared__ float s_mass_above;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // 1. repetition penalty
  if (a.history != nullptr && a.penalty[row] != 1.0f) {
    const float pen = a.penalty[row];
    const int hl = a.history_len[row];
    for (int i = tid; i < hl; i += kThreads) {
      const long long t = a.history[(long long)row * a.hmax + i];
      if (t >= 0 && t < V) {
        const float v = lg[t];
        // duplicates in the history write the same value: idempotent
        lg[t] = v > 0.f ? v / pen : v * pen;
      }
    }
    __syncthreads();
  }
  const float temp = a.temperature[row];
  // 2. max (and greedy argmax)
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < V; i += kThreads) {
    const float v = lg[i];
    if (v > best) { best = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  if (lane == 0) { red_f[warp] = best; red_i[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    best = red_f[lane];
    bi = red_i[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) { red_f[0] = best; red_i[0] = bi; }
  }
  __syncthreads();
  const float lmax = red_f[0];
  if (temp <= 0.f) {
    if (tid == 0) a.out[row] = red_i[0];
    return;
  }
  const float inv_t = 1.f / temp;
  const float zmax = lmax * inv_t;
  // 3. top-k threshold on ordered keys (keep key >= thr_k)
  uint32_t thr = 0u;
  const int k = a.top_k[row];
  if (k > 0 && k < V) {
    uint32_t prefix = 0u;
    int remaining = k;
    for (int pass = 3; pass >= 0; --pass) {
      const int shift = pass * 8;
      for (int i = tid; i < 256; i += kThreads) hist[i] = 0u;
      __syncthreads();
      const uint32_t hi_mask = pass == 3 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int i = tid; i < V; i += kThreads) {
        const uint32_t key = ordered(lg[i] * inv_t);
        if ((key & hi_mask) == (prefix & hi_mask)) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        int acc = 0;
        int b = 255;
        for (; b >= 0; --b) {
          if (acc + (int)hist[b] >= remaining) break;
          acc += hist[b];
        }
        b = max(b, 0);
        s_prefix = prefix | ((uint32_t)b << shift);
        red_i[0] = remaining - acc;
      }
      __syncthreads();
      prefix = s_prefix;
      remaining = red_i[0];
      __syncthreads();
    }
    thr = prefix;
  }
  // 4. top-p threshold over the probability mass of keys >= thr
  const float p = a.top_p[row];
  if (p < 1.f) {
    float tot = 0.f;
    for (int i = tid; i < V; i += kThreads) {
      const float z = lg[i] * inv_t;
      if (ordered(z) >= thr) tot += __expf(z - zmax);
    }
    tot = warp_sum(tot);
    if (lane == 0) red_f[warp] = tot;
    __syncthreads();
    if (warp == 0) {
      tot = warp_sum(red_f[lane]);
      if (lane == 0) { s_remain = p * tot; s_mass_above = 0.f; }
    }
    __syncthreads();
    uint32_t prefix = 0u;
    for (int pass = 3; pass >= 0; --pass) {
      const int shift = pass * 8;
      for (int i = tid; i < 256; i += kThreads) hmass[i] = 0.f;
      __syncthreads();
      const uint32_t hi_mask = pass == 3 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int i = tid; i < V; i += kThreads) {
        const float z = lg[i] * inv_t;
        const uint32_t key = ordered(z);
        if (key >= thr && (key & hi_mask) == (prefix & hi_mask))
          atomicAdd(&hmass[(key >> shift) & 255u], __expf(z - zmax));
      }
      __syncthreads();
      if (tid == 0) {
        float acc = 0.f;
        int b = 255;
        for (; b >= 0; --b) {
          if (acc + hmass[b] >= s_remain) break;
          acc += hmass[b];
        }
        b = max(b, 0);
        s_prefix = prefix | ((uint32_t)b << shift);
        s_remain -= acc;
      }
      __syncthreads();
      prefix = s_prefix;
    }
    thr = max(thr, prefix);
  }
  // 5. Gumbel-max over survivors
  curandStatePhilox4_32_10_t st;
  curand_init((unsigned long long)a.seeds[row], (unsigned long long)row * kThreads + tid,
              (unsigned long long)a.offsets[row] * 4ull * ((V + kThreads - 1) / kThreads + 1), &st);
  best = -INFINITY;
  bi = 0x7fffffff;
  for (int i = tid; i < V; i += kThreads) {
    const float z = lg[i] * inv_t;
    const float u = curand_uniform(&st);  // (0, 1]
    if (ordered(z) < thr) continue;
    const float g = -__logf(-__logf(fminf(u, 0.99999994f)));
    const float v = z + g;
    if (v > best || (v == best && i < bi)) { best = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  __syncthreads();
  if (lane == 0) { red_f[warp] = best; red_i[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    best = red_f[lane];
    bi = red_i[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) a.out[row] = bi == 0x7fffffff ? red_i[0] : bi;
  }
}

}  // namespace

void sample_tokens(at::Tensor& logits, const at::Tensor& temperature, const at::Tensor& top_k,
                   const at::Tensor& top_p, const at::Tensor& penalty,
                   const c10::optional<at::Tensor>& history,
                   const c10::optional<at::Tensor>& history_len, const at::Tensor& seeds,
                   const at::Tensor& offsets, at::Tensor& out) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1, "sample: fp32 logits");
  const int B = logits.size(0);
  if (B == 0) return;
  c10::cuda::CUDAGuard guard(logits.device());
  SampleArgs a{};
  a.logits = logits.data_ptr<float>();
  a.ld = logits.stride(0);
  a.V = logits.size(1);
  a.temperature = temperature.data_ptr<float>();
  a.top_k = top_k.data_ptr<int>();
  a.top_p = top_p.data_ptr<float>();
  a.penalty = penalty.data_ptr<float>();
  if (history.has_value()) {
    a.history = reinterpret_cast<const long long*>(history->data_ptr<int64_t>());
    a.history_len = history_len->data_ptr<int>();
    a.hmax = history->size(1);
  }
  a.seeds = reinterpret_cast<const long long*>(seeds.data_ptr<int64_t>());
  a.offsets = reinterpret_cast<const long long*>(offsets.data_ptr<int64_t>());
  a.out = reinterpret_cast<long long*>(out.data_ptr<int64_t>());
  launch_pdl(sample_kernel, dim3(B), dim3(kThreads), 0, at::cuda::getCurrentCUDAStream(),
             "sample launch", a);
}

}  // namespace sil
