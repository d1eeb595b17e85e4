// Paged GQA attention over the persistent KV cache (decode and prefill).
//
// KV cache layout (per layer): K, V = [num_pages, Hkv, 64, D=128] bf16, one
// 16 KB contiguous page per (page, kv-head).  A page is brought into shared
// memory by two TMA tiles of [64 tokens x 64 dims] with the 128-byte swizzle,
// so ldmatrix reads of the tile are bank-conflict free.
//
// Decode: one CTA per (split, kv-head, sequence).  The G query heads that
// share a KV head form the rows of a 16-row MMA tile, each of the 4 warps
// owns 16 tokens of every page and keeps its own online-softmax state; the
// CTA merges its warps, and the last CTA of a (sequence, kv-head) merges the
// splits in split order (deterministic flash-decoding), so one launch yields
// the final output.  The split count adapts on the device to each
// sequence's length, which keeps the launch graph-capturable.
//
// Prefill: one CTA per (64-query tile, query head, sequence) with causal
// masking against absolute positions (chunked prefill and prefix reuse work
// because queries sit at the end of the context).
//
// Replaces HF eager/SDPA/FA2 attention used by the reference
// (si/model/qwen3.py:916-996) and the explicit matmul/softmax path of its
// logical TP model (si/microsharding/dense.py:343-351).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sil/host.h"
#include "sil/mma.cuh"
#include "sil/ptx.cuh"

namespace sil {
namespace {

constexpr int kPage = 64;
constexpr int kD = 128;
constexpr int kStages = 3;
constexpr int kTileBytes = kPage * 64 * 2;      // one [64 x 64] bf16 TMA box
constexpr int kKVBytes = 2 * kTileBytes;        // one page of K (or V) for one head
constexpr int kStageBytes = 2 * kKVBytes;       // K + V

struct AttnArgs {
  const __nv_bfloat16* q;
  long long q_stride;     // elements between consecutive tokens
  __nv_bfloat16* out;
  long long o_stride;
  const int* block_table;
  long long bt_stride;
  const int* seq_lens;    // context length incl. the new tokens
  const int* cu_q;        // prefill: [B+1] offsets of each sequence's queries
  int Hq, Hkv, G;
  int num_pages;          // pages of the cache; a block-table entry outside [0, num_pages)
                          // raises kStatusBadArgument instead of being loaded
  float scale_log2;       // softmax scale * log2(e)
  int num_splits;
  float* ws_o;            // decode split partials
  float* ws_ml;
  int* counters;
  int* status;
};

__device__ __forceinline__ void issue_page(uint8_t* stage, const CUtensorMap* tk,
                                           const CUtensorMap* tv, uint64_t* bar, int row) {
  mbar_arrive_expect_tx(bar, kStageBytes);
  tma_load_2d(stage, tk, bar, 0, row);
  tma_load_2d(stage + kTileBytes, tk, bar, 64, row);
  tma_load_2d(stage + kKVBytes, tv, bar, 0, row);
  tma_load_2d(stage + kKVBytes + kTileBytes, tv, bar, 64, row);
}

// Issues the TMA loads of page `pid` of kv-head h into `stage`, after checking the
// page id against the cache.  A bad id raises kStatusBadArgument and loads nothing;
// the consumer's wait on that stage then gives up on the raised status.
__device__ __forceinline__ bool issue_checked(uint8_t* stage, const CUtensorMap* tk,
                                              const CUtensorMap* tv, uint64_t* bar, int pid,
                                              const AttnArgs& a, int h) {
  if (static_cast<unsigned>(pid) >= static_cast<unsigned>(a.num_pages)) {
    raise_status(a.status, kStatusBadArgument);
    return false;
  }
  issue_page(stage, tk, tv, bar, (pid * a.Hkv + h) * kPage);
  return true;
}

// Error path: lets the loads of pages [consumed, issued) land before the shared
// memory they target is reused or the CTA exits (thread 0, which issued them).
__device__ __forceinline__ void drain_pages(uint64_t* full, int consumed, int issued) {
  for (int j = consumed; j < issued; ++j) mbar_drain(&full[j % kStages], (j / kStages) & 1);
}

// Address of the ldmatrix row for K/V tile rows `r` and 8-dim chunk `c` (0..15).
__device__ __forceinline__ uint32_t tile_addr(uint32_t base, int r, int c) {
  const int box = c >> 3;
  const int cc = c & 7;
  return base + box * kTileBytes + r * 128 + ((cc ^ (r & 7)) << 4);
}

// ------------------------------------------------------------------ decode
__global__ void __launch_bounds__(128)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  int* sflag = reinterpret_cast<int*>(full + kStages);

  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int S = args.num_splits;
  const int len = args.seq_lens[b];
  const int n_pages = (len + kPage - 1) / kPage;
  const int per = (n_pages + S - 1) / S;
  const int p_begin = split * per;
  const int count = max(0, min(n_pages, p_begin + per) - p_begin);
  const int* bt = args.block_table + (long long)b * args.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    sflag[0] = load_status(args.status);
    sflag[1] = 0;
  }
  __syncthreads();
  const bool skip = sflag[0] != 0;
  int issued = 0, consumed = 0;  // pages loaded / waited for (thread 0's view)
  if (!skip && threadIdx.x == 0) {
    for (int i = 0; i < min(count, kStages); ++i) {
      if (!issue_checked(smem + i * kStageBytes, &tmK, &tmV, &full[i], bt[p_begin + i], args, h))
        break;
      issued = i + 1;
    }
  }

  // Q fragments: rows = query heads of this group (g and g+8), K-dim = head dim.
  uint32_t qa[8][4];
  {
    const int hq0 = h * args.G;
    const __nv_bfloat16* qb = args.q + (long long)b * args.q_stride;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int d0 = kk * 16 + 2 * t;
      uint32_t lo0 = 0, lo1 = 0, hi0 = 0, hi1 = 0;
      if (g < args.G) {
        const __nv_bfloat16* qr = qb + (long long)(hq0 + g) * kD;
        lo0 = *reinterpret_cast<const uint32_t*>(qr + d0);
        lo1 = *reinterpret_cast<const uint32_t*>(qr + d0 + 8);
      }
      if (g + 8 < args.G) {
        const __nv_bfloat16* qr = qb + (long long)(hq0 + g + 8) * kD;
        hi0 = *reinterpret_cast<const uint32_t*>(qr + d0);
        hi1 = *reinterpret_cast<const uint32_t*>(qr + d0 + 8);
      }
      qa[kk][0] = lo0; qa[kk][1] = hi0; qa[kk][2] = lo1; qa[kk][3] = hi1;
    }
  }

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  bool alive = !skip;

  for (int i = 0; i < count; ++i) {
    const int s = i % kStages;
    if (alive && !mbar_wait(&full[s], (i / kStages) & 1, args.status, kStatusTimeoutFull))
      alive = false;
    if (alive) consumed = i + 1;
    if (alive) {
      const uint32_t kbase = smem_u32(smem + s * kStageBytes);
      const uint32_t vbase = kbase + kKVBytes;
      float sc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int kk2 = 0; kk2 < 4; ++kk2) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int r = warp * 16 + nt * 8 + (lane & 7);
          const int c = kk2 * 4 + (lane >> 3);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(tile_addr(kbase, r, c), b0, b1, b2, b3);
          mma_bf16_16816(sc[nt], qa[2 * kk2], b0, b1);
          mma_bf16_16816(sc[nt], qa[2 * kk2 + 1], b2, b3);
        }
      }
      const int tok0 = (p_begin + i) * kPage + warp * 16;
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int tok = tok0 + nt * 8 + 2 * t + (j & 1);
          float v = sc[nt][j] * args.scale_log2;
          if (tok >= len) v = -INFINITY;
          sc[nt][j] = v;
          mx[j >> 1] = fmaxf(mx[j >> 1], v);
        }
      float alpha[2];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
        mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
        const float m_new = fmaxf(m_r[rr], mx[rr]);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        alpha[rr] = exp2f(m_r[rr] - m_use);
        m_r[rr] = m_new;
        mx[rr] = m_use;
      }
      float rs[2] = {0.f, 0.f};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float p = exp2f(sc[nt][j] - mx[j >> 1]);
          sc[nt][j] = p;
          rs[j >> 1] += p;
        }
      l_r[0] = l_r[0] * alpha[0] + rs[0];
      l_r[1] = l_r[1] * alpha[1] + rs[1];
#pragma unroll
      for (int nd = 0; nd < 16; ++nd) {
        o[nd][0] *= alpha[0]; o[nd][1] *= alpha[0];
        o[nd][2] *= alpha[1]; o[nd][3] *= alpha[1];
      }
      uint32_t pa[4];
      pa[0] = pack_bf16x2(sc[0][0], sc[0][1]);
      pa[1] = pack_bf16x2(sc[0][2], sc[0][3]);
      pa[2] = pack_bf16x2(sc[1][0], sc[1][1]);
      pa[3] = pack_bf16x2(sc[1][2], sc[1][3]);
#pragma unroll
      for (int nd2 = 0; nd2 < 8; ++nd2) {
        const int r = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int c = nd2 * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(tile_addr(vbase, r, c), b0, b1, b2, b3);
        mma_bf16_16816(o[2 * nd2], pa, b0, b1);
        mma_bf16_16816(o[2 * nd2 + 1], pa, b2, b3);
      }
    }
    __syncthreads();
    if (alive && threadIdx.x == 0 && i + kStages < count && issued == i + kStages &&
        issue_checked(smem + s * kStageBytes, &tmK, &tmV, &full[s], bt[p_begin + i + kStages],
                      args, h))
      issued = i + kStages + 1;
  }
  if (threadIdx.x == 0 && consumed < issued) drain_pages(full, consumed, issued);
  __syncthreads();

  // Full row sums (the 4 threads of a row hold disjoint token subsets).
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 1);
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 2);
  }
  // Merge the 4 warps through shared memory (stage buffers are idle now).
  float* so = reinterpret_cast<float*>(smem);                 // [4][16][128]
  float* sm = so + 4 * 16 * kD;                               // [4][16]
  float* sl = sm + 4 * 16;                                    // [4][16]
#pragma unroll
  for (int nd = 0; nd < 16; ++nd) {
    const int d = nd * 8 + 2 * t;
    so[(warp * 16 + g) * kD + d] = o[nd][0];
    so[(warp * 16 + g) * kD + d + 1] = o[nd][1];
    so[(warp * 16 + g + 8) * kD + d] = o[nd][2];
    so[(warp * 16 + g + 8) * kD + d + 1] = o[nd][3];
  }
  if (t == 0) {
    sm[warp * 16 + g] = m_r[0];
    sm[warp * 16 + g + 8] = m_r[1];
    sl[warp * 16 + g] = l_r[0];
    sl[warp * 16 + g + 8] = l_r[1];
  }
  __syncthreads();
  const long long bh = (long long)b * args.Hkv + h;
  const int G = args.G;
  for (int e = threadIdx.x; e < G * kD; e += 128) {
    const int row = e / kD, d = e % kD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm[w * 16 + row]);
    const float Mu = M == -INFINITY ? 0.f : M;
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = exp2f(sm[w * 16 + row] - Mu);
      L += sl[w * 16 + row] * f;
      acc += so[(w * 16 + row) * kD + d] * f;
    }
    if (S == 1) {
      if (!skip)
        args.out[(long long)b * args.o_stride + (long long)(h * G + row) * kD + d] =
            __float2bfloat16_rn(L > 0.f ? acc / L : 0.f);
    } else {
      args.ws_o[((bh * S + split) * G + row) * kD + d] = acc;
      if (d == 0) {
        args.ws_ml[((bh * S + split) * G + row) * 2 + 0] = M;
        args.ws_ml[((bh * S + split) * G + row) * 2 + 1] = L;
      }
    }
  }
  if (S == 1 || skip) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(&args.counters[bh], 1);
    sflag[1] = old == S - 1;
  }
  __syncthreads();
  if (!sflag[1]) return;
  __threadfence();
  for (int e = threadIdx.x; e < G * kD; e += 128) {
    const int row = e / kD, d = e % kD;
    float M = -INFINITY;
    for (int sp = 0; sp < S; ++sp) M = fmaxf(M, __ldcg(&args.ws_ml[((bh * S + sp) * G + row) * 2]));
    const float Mu = M == -INFINITY ? 0.f : M;
    float L = 0.f, acc = 0.f;
    for (int sp = 0; sp < S; ++sp) {
      const long long base = (bh * S + sp) * G + row;
      const float f = exp2f(__ldcg(&args.ws_ml[base * 2]) - Mu);
      L += __ldcg(&args.ws_ml[base * 2 + 1]) * f;
      acc += __ldcg(&args.ws_o[base * kD + d]) * f;
    }
    args.out[(long long)b * args.o_stride + (long long)(h * G + row) * kD + d] =
        __float2bfloat16_rn(L > 0.f ? acc / L : 0.f);
  }
  if (threadIdx.x == 0) args.counters[bh] = 0;
}

// ------------------------------------------------------------------ prefill
__global__ void __launch_bounds__(128)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  int* sflag = reinterpret_cast<int*>(full + kStages);

  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int hq = blockIdx.y, b = blockIdx.z;
  const int h = hq / args.G;
  const int q_begin = args.cu_q[b];
  const int q_len = args.cu_q[b + 1] - q_begin;
  const int n_qt = (q_len + 63) / 64;
  const int qt = (int)gridDim.x - 1 - (int)blockIdx.x;  // heaviest tiles first
  if (qt >= n_qt || qt < 0) return;
  const int kv_len = args.seq_lens[b];
  const int pos0 = kv_len - q_len;  // absolute position of query 0
  const int q0 = qt * 64;
  const int last_q = min(q0 + 63, q_len - 1);
  const int n_pages = min((pos0 + last_q) / kPage + 1, (kv_len + kPage - 1) / kPage);
  const int* bt = args.block_table + (long long)b * args.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    sflag[0] = load_status(args.status);
  }
  __syncthreads();
  const bool skip = sflag[0] != 0;
  int issued = 0, consumed = 0;  // pages loaded / waited for (thread 0's view)
  if (!skip && threadIdx.x == 0) {
    for (int i = 0; i < min(n_pages, kStages); ++i) {
      if (!issue_checked(smem + i * kStageBytes, &tmK, &tmV, &full[i], bt[i], args, h)) break;
      issued = i + 1;
    }
  }
  // Q fragments for this warp's 16 rows.
  const int row_lo = q0 + warp * 16 + g;
  const int row_hi = row_lo + 8;
  uint32_t qa[8][4];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int d0 = kk * 16 + 2 * t;
    uint32_t lo0 = 0, lo1 = 0, hi0 = 0, hi1 = 0;
    if (row_lo < q_len) {
      const __nv_bfloat16* qr = args.q + (long long)(q_begin + row_lo) * args.q_stride + hq * kD;
      lo0 = *reinterpret_cast<const uint32_t*>(qr + d0);
      lo1 = *reinterpret_cast<const uint32_t*>(qr + d0 + 8);
    }
    if (row_hi < q_len) {
      const __nv_bfloat16* qr = args.q + (long long)(q_begin + row_hi) * args.q_stride + hq * kD;
      hi0 = *reinterpret_cast<const uint32_t*>(qr + d0);
      hi1 = *reinterpret_cast<const uint32_t*>(qr + d0 + 8);
    }
    qa[kk][0] = lo0; qa[kk][1] = hi0; qa[kk][2] = lo1; qa[kk][3] = hi1;
  }
  const int qpos_lo = pos0 + row_lo, qpos_hi = pos0 + row_hi;
  const int warp_last_pos = pos0 + min(q0 + warp * 16 + 15, q_len - 1);

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  bool alive = !skip;

  for (int i = 0; i < n_pages; ++i) {
    const int s = i % kStages;
    if (alive && !mbar_wait(&full[s], (i / kStages) & 1, args.status, kStatusTimeoutFull))
      alive = false;
    if (alive) consumed = i + 1;
    // Warps whose queries all precede this page have nothing to add.
    if (alive && i * kPage <= warp_last_pos) {
      const uint32_t kbase = smem_u32(smem + s * kStageBytes);
      const uint32_t vbase = kbase + kKVBytes;
      float sc[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int kk2 = 0; kk2 < 4; ++kk2) {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int r = nt * 8 + (lane & 7);
          const int c = kk2 * 4 + (lane >> 3);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(tile_addr(kbase, r, c), b0, b1, b2, b3);
          mma_bf16_16816(sc[nt], qa[2 * kk2], b0, b1);
          mma_bf16_16816(sc[nt], qa[2 * kk2 + 1], b2, b3);
        }
      }
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int kp = i * kPage + nt * 8 + 2 * t + (j & 1);
          const int qp = (j < 2) ? qpos_lo : qpos_hi;
          float v = sc[nt][j] * args.scale_log2;
          if (kp > qp || kp >= kv_len) v = -INFINITY;
          sc[nt][j] = v;
          mx[j >> 1] = fmaxf(mx[j >> 1], v);
        }
      float alpha[2];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
        mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
        const float m_new = fmaxf(m_r[rr], mx[rr]);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        alpha[rr] = exp2f(m_r[rr] - m_use);
        m_r[rr] = m_new;
        mx[rr] = m_use;
      }
      float rs[2] = {0.f, 0.f};
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float p = exp2f(sc[nt][j] - mx[j >> 1]);
          sc[nt][j] = p;
          rs[j >> 1] += p;
        }
      l_r[0] = l_r[0] * alpha[0] + rs[0];
      l_r[1] = l_r[1] * alpha[1] + rs[1];
#pragma unroll
      for (int nd = 0; nd < 16; ++nd) {
        o[nd][0] *= alpha[0]; o[nd][1] *= alpha[0];
        o[nd][2] *= alpha[1]; o[nd][3] *= alpha[1];
      }
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t pa[4];
        pa[0] = pack_bf16x2(sc[2 * ks][0], sc[2 * ks][1]);
        pa[1] = pack_bf16x2(sc[2 * ks][2], sc[2 * ks][3]);
        pa[2] = pack_bf16x2(sc[2 * ks + 1][0], sc[2 * ks + 1][1]);
        pa[3] = pack_bf16x2(sc[2 * ks + 1][2], sc[2 * ks + 1][3]);
#pragma unroll
        for (int nd2 = 0; nd2 < 8; ++nd2) {
          const int r = ks * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
          const int c = nd2 * 2 + (lane >> 4);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(tile_addr(vbase, r, c), b0, b1, b2, b3);
          mma_bf16_16816(o[2 * nd2], pa, b0, b1);
          mma_bf16_16816(o[2 * nd2 + 1], pa, b2, b3);
        }
      }
    }
    __syncthreads();
    if (alive && threadIdx.x == 0 && i + kStages < n_pages && issued == i + kStages &&
        issue_checked(smem + s * kStageBytes, &tmK, &tmV, &full[s], bt[i + kStages], args, h))
      issued = i + kStages + 1;
  }
  if (threadIdx.x == 0 && consumed < issued) drain_pages(full, consumed, issued);
  if (skip) return;
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 1);
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 2);
  }
  const float inv_lo = l_r[0] > 0.f ? 1.f / l_r[0] : 0.f;
  const float inv_hi = l_r[1] > 0.f ? 1.f / l_r[1] : 0.f;
#pragma unroll
  for (int nd = 0; nd < 16; ++nd) {
    const int d = nd * 8 + 2 * t;
    if (row_lo < q_len) {
      __nv_bfloat16* orow = args.out + (long long)(q_begin + row_lo) * args.o_stride + hq * kD;
      *reinterpret_cast<uint32_t*>(orow + d) = pack_bf16x2(o[nd][0] * inv_lo, o[nd][1] * inv_lo);
    }
    if (row_hi < q_len) {
      __nv_bfloat16* orow = args.out + (long long)(q_begin + row_hi) * args.o_stride + hq * kD;
      *reinterpret_cast<uint32_t*>(orow + d) = pack_bf16x2(o[nd][2] * inv_hi, o[nd][3] * inv_hi);
    }
  }
}

constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 64;

void check_cache(const at::Tensor& c) {
  TORCH_CHECK(c.is_cuda() && c.scalar_type() == at::kBFloat16 && c.is_contiguous(),
              "KV cache must be contiguous bf16 on CUDA");
  TORCH_CHECK(c.dim() == 4 && c.size(2) == kPage && c.size(3) == kD,
              "KV cache must be [pages, Hkv, 64, 128]");
}

CUtensorMap cache_map(const at::Tensor& c) {
  const uint64_t rows = (uint64_t)c.size(0) * c.size(1) * kPage;
  return make_tmap_2d(c.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, kD, kD, kPage, 64,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

// q: [B, Hq, 128] (token stride q.stride(0)); out: [B, Hq*128].
void paged_decode(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                  const at::Tensor& block_table, const at::Tensor& seq_lens, at::Tensor& out,
                  double scale, int64_t num_splits, const at::Tensor& ws, const at::Tensor& counters,
                  const at::Tensor& status) {
  check_cache(k_cache);
  check_cache(v_cache);
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.size(2) == kD &&
                  q.stride(2) == 1 && q.stride(1) == kD,
              "paged_decode: q must be [B, Hq, 128] with contiguous heads");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt,
              "paged_decode: int32 block table / seq lens");
  const int B = q.size(0), Hq = q.size(1), Hkv = k_cache.size(1);
  TORCH_CHECK(Hq % Hkv == 0 && Hq / Hkv <= 16, "paged_decode: group size must be <= 16");
  if (B == 0) return;
  c10::cuda::CUDAGuard guard(q.device());
  AttnArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.q_stride = q.stride(0);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.o_stride = out.stride(0);
  a.block_table = block_table.data_ptr<int>();
  a.bt_stride = block_table.stride(0);
  a.seq_lens = seq_lens.data_ptr<int>();
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.num_pages = static_cast<int>(k_cache.size(0));
  a.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  int S = std::max<int64_t>(1, num_splits);
  const long long need_o = (long long)B * Hkv * S * a.G * kD;
  const long long need_ml = (long long)B * Hkv * S * a.G * 2;
  while (S > 1 && need_o / 1 > 0 && (long long)B * Hkv * S * a.G * (kD + 2) > ws.numel()) --S;
  TORCH_CHECK(S == 1 || (long long)B * Hkv <= counters.numel(), "paged_decode: counters too small");
  (void)need_o; (void)need_ml;
  a.num_splits = S;
  a.ws_o = ws.data_ptr<float>();
  a.ws_ml = a.ws_o + (long long)B * Hkv * S * a.G * kD;
  a.counters = counters.data_ptr<int>();
  a.status = status.data_ptr<int>();
  CUtensorMap tk = cache_map(k_cache), tv = cache_map(v_cache);
  set_smem_limit(reinterpret_cast<const void*>(paged_decode_kernel), kSmemBytes, "cudaFuncSetAttribute(decode)");
  dim3 grid(S, Hkv, B);
  launch_pdl(paged_decode_kernel, grid, dim3(128), kSmemBytes, at::cuda::getCurrentCUDAStream(),
             "paged_decode launch", tk, tv, a);
}

// q: packed [T, Hq, 128]; cu_q: [B+1]; seq_lens: [B] (context after append); out: [T, Hq*128].
void paged_prefill(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                   const at::Tensor& block_table, const at::Tensor& seq_lens,
                   const at::Tensor& cu_q, at::Tensor& out, double scale, int64_t max_q_len,
                   const at::Tensor& status) {
  check_cache(k_cache);
  check_cache(v_cache);
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.size(2) == kD &&
                  q.stride(2) == 1 && q.stride(1) == kD,
              "paged_prefill: q must be [T, Hq, 128] with contiguous heads");
  const int B = seq_lens.size(0), Hq = q.size(1), Hkv = k_cache.size(1);
  TORCH_CHECK(Hq % Hkv == 0, "paged_prefill: Hq must be a multiple of Hkv");
  if (B == 0 || max_q_len <= 0) return;
  c10::cuda::CUDAGuard guard(q.device());
  AttnArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.q_stride = q.stride(0);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.o_stride = out.stride(0);
  a.block_table = block_table.data_ptr<int>();
  a.bt_stride = block_table.stride(0);
  a.seq_lens = seq_lens.data_ptr<int>();
  a.cu_q = cu_q.data_ptr<int>();
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.num_pages = static_cast<int>(k_cache.size(0));
  a.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  a.status = status.data_ptr<int>();
  CUtensorMap tk = cache_map(k_cache), tv = cache_map(v_cache);
  set_smem_limit(reinterpret_cast<const void*>(paged_prefill_kernel), kSmemBytes, "cudaFuncSetAttribute(prefill)");
  dim3 grid((max_q_len + 63) / 64, Hq, B);
  launch_pdl(paged_prefill_kernel, grid, dim3(128), kSmemBytes, at::cuda::getCurrentCUDAStream(),
             "paged_prefill launch", tk, tv, a);
}

}  // namespace sil

// ---------------------------------------------------------------------------
// Allocation-free entry point (declared and documented in sil/noalloc.h; it has
// no counterpart in the reference).  The split-K scratch lives in the
// file-scope array below instead of caller- or torch-allocated memory.
#include "sil/noalloc.h"

namespace {

constexpr long long kNoAllocFloats = 1LL << 20;  // 4 MiB of fp32 partials
constexpr int kNoAllocCounters = 4096;           // (sequence, kv-head) pairs

struct NoAllocScratch {
  float partial[kNoAllocFloats];
  int counters[kNoAllocCounters];
  int status[64];
};

static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

thread_local std::string g_noalloc_error;
std::mutex g_noalloc_mutex;
NoAllocScratch* g_noalloc_ptr[64] = {};  // device address per device ordinal
bool g_noalloc_smem_set[64] = {};

int noalloc_fail(int code, const std::string& msg) {
  g_noalloc_error = msg;
  return code;
}

// Device address of the scratch array on the current device (looked up once per
// device, with that device current: the host-side name of the array is not a
// device address).  Returns SIL_NOALLOC_OK or an error code.
int noalloc_scratch(NoAllocScratch** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return noalloc_fail(SIL_NOALLOC_ECUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return noalloc_fail(SIL_NOALLOC_EINVAL, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return noalloc_fail(SIL_NOALLOC_ECUDA,
                          std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<NoAllocScratch*>(p);
  }
  if (!g_noalloc_smem_set[dev]) {
    e = cudaFuncSetAttribute(sil::paged_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             sil::kSmemBytes);
    if (e != cudaSuccess)
      return noalloc_fail(SIL_NOALLOC_ECUDA,
                          std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    g_noalloc_smem_set[dev] = true;
  }
  *out = g_noalloc_ptr[dev];
  return SIL_NOALLOC_OK;
}

}  // namespace

extern "C" const char* sil_noalloc_last_error(void) { return g_noalloc_error.c_str(); }
extern "C" long long sil_noalloc_scratch_floats(void) { return kNoAllocFloats; }
extern "C" int sil_noalloc_max_counters(void) { return kNoAllocCounters; }

extern "C" int sil_noalloc_status(int* host_out, cudaStream_t stream) {
  g_noalloc_error.clear();
  if (!host_out) return noalloc_fail(SIL_NOALLOC_EINVAL, "null pointer argument");
  NoAllocScratch* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  cudaError_t e = cudaMemcpyAsync(host_out, scratch->status, sizeof(int), cudaMemcpyDeviceToHost,
                                  stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return noalloc_fail(SIL_NOALLOC_ECUDA, cudaGetErrorString(e));
  return SIL_NOALLOC_OK;
}

extern "C" int sil_noalloc_set_wait_limit_ns(unsigned long long ns, cudaStream_t stream) {
  g_noalloc_error.clear();
  NoAllocScratch* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  // Stream-ordered, from a value that must outlive the copy: copy from a static.
  static thread_local unsigned long long value;
  value = ns;
  cudaError_t e = cudaMemcpyAsync(scratch->status + 2, &value, sizeof(value),
                                  cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return noalloc_fail(SIL_NOALLOC_ECUDA, cudaGetErrorString(e));
  return SIL_NOALLOC_OK;
}

extern "C" int sil_paged_decode_noalloc(const void* q, long long q_stride, const void* k_cache,
                                        const void* v_cache, long long num_pages, int kv_heads,
                                        const int* block_table, long long bt_stride,
                                        const int* seq_lens, void* out, long long out_stride,
                                        int batch, int q_heads, float scale, int num_splits,
                                        cudaStream_t stream) {
  using namespace sil;
  g_noalloc_error.clear();
  if (!q || !k_cache || !v_cache || !block_table || !seq_lens || !out)
    return noalloc_fail(SIL_NOALLOC_EINVAL, "null pointer argument");
  if (batch <= 0 || kv_heads <= 0 || q_heads <= 0 || num_pages <= 0 || num_splits <= 0)
    return noalloc_fail(SIL_NOALLOC_EINVAL, "sizes must be positive");
  if (q_heads % kv_heads != 0 || q_heads / kv_heads > 16)
    return noalloc_fail(SIL_NOALLOC_EINVAL, "q_heads must be a multiple of kv_heads, ratio <= 16");
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15u) || (reinterpret_cast<uintptr_t>(v_cache) & 15u) ||
      (reinterpret_cast<uintptr_t>(q) & 3u) || (reinterpret_cast<uintptr_t>(out) & 1u))
    return noalloc_fail(SIL_NOALLOC_EINVAL,
                        "cache pointers must be 16-byte aligned, q 4-byte aligned, out 2-byte aligned");
  // q is read as 32-bit words, so its row stride must be even; rows must not overlap.
  if (q_stride < (long long)q_heads * kD || (q_stride & 1))
    return noalloc_fail(SIL_NOALLOC_EINVAL, "q_stride must be even and >= q_heads * 128");
  if (out_stride < (long long)q_heads * kD)
    return noalloc_fail(SIL_NOALLOC_EINVAL, "out_stride must be >= q_heads * 128");
  if (bt_stride <= 0) return noalloc_fail(SIL_NOALLOC_EINVAL, "bt_stride must be positive");
  if (num_pages * kv_heads * kPage > (1LL << 31) - 1 || num_pages > (1LL << 31) - 1)
    return noalloc_fail(SIL_NOALLOC_EINVAL, "cache too large for 32-bit page rows");
  const int G = q_heads / kv_heads;
  const long long need = (long long)batch * kv_heads * num_splits * G * (kD + 2);
  if (num_splits > 1 && need > kNoAllocFloats)
    return noalloc_fail(SIL_NOALLOC_ETOOBIG,
                        "request needs " + std::to_string(need) + " fp32 scratch values; the " +
                            "allocation-free entry point holds " + std::to_string(kNoAllocFloats));
  if (num_splits > 1 && (long long)batch * kv_heads > kNoAllocCounters)
    return noalloc_fail(SIL_NOALLOC_ETOOBIG,
                        "batch * kv_heads exceeds the " + std::to_string(kNoAllocCounters) +
                            " split counters of the allocation-free entry point");
  NoAllocScratch* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  // Counters and the status word must start at zero (an earlier call that gave up
  // may have left them set); partials are fully written before they are read.  The
  // status is cleared here, at the start of the next call: read it with
  // sil_noalloc_status() before calling again.
  const size_t nctr = static_cast<size_t>(std::min<long long>((long long)batch * kv_heads,
                                                              kNoAllocCounters));
  cudaError_t e = cudaMemsetAsync(scratch->counters, 0, nctr * sizeof(int), stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(scratch->status, 0, sizeof(int), stream);
  if (e != cudaSuccess) return noalloc_fail(SIL_NOALLOC_ECUDA, cudaGetErrorString(e));
  AttnArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_stride;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.o_stride = out_stride;
  a.block_table = block_table;
  a.bt_stride = bt_stride;
  a.seq_lens = seq_lens;
  a.Hq = q_heads;
  a.Hkv = kv_heads;
  a.G = G;
  a.num_pages = static_cast<int>(num_pages);
  a.scale_log2 = scale * 1.4426950408889634f;
  a.num_splits = num_splits;
  a.ws_o = scratch->partial;
  a.ws_ml = scratch->partial + (long long)batch * kv_heads * num_splits * G * kD;
  a.counters = scratch->counters;
  a.status = scratch->status;
  try {
    const uint64_t rows = (uint64_t)num_pages * kv_heads * kPage;
    CUtensorMap tk = make_tmap_2d(k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, kD, kD, kPage,
                                  64, CU_TENSOR_MAP_SWIZZLE_128B);
    CUtensorMap tv = make_tmap_2d(v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, kD, kD, kPage,
                                  64, CU_TENSOR_MAP_SWIZZLE_128B);
    launch_pdl(paged_decode_kernel, dim3(num_splits, kv_heads, batch), dim3(128), kSmemBytes,
               stream, "paged_decode (allocation-free) launch", tk, tv, a);
  } catch (const std::exception& ex) {
    return noalloc_fail(SIL_NOALLOC_ECUDA, ex.what());
  }
  return SIL_NOALLOC_OK;
}
