// Multi-head latent attention (DeepSeek-V3 / Kimi-K2) over a paged latent cache.
//
// Cache layout (per layer): [num_pages, 64 tokens, 576] bf16 -- the RMS-normed
// compressed KV c_kv (512) followed by the rotated shared rope key k_pe (64).
// A 64-token page is 72 KB contiguous; the kernel streams it as two 32-token
// tiles of nine [32 x 64] TMA boxes with the 128-byte swizzle.
//
// Attention runs in the weight-absorbed form for prefill and decode alike:
//   q_lat[t,h] = W_UK[h]^T q_nope[t,h]          (512, a per-head grouped GEMM)
//   score(t,h,j) = (q_lat . c_kv[j] + q_pe[t,h] . k_pe[j]) * scale
//   o_lat[t,h] = softmax_j(score) . c_kv[j]      (512; W_UV is applied afterwards)
// so every query head reads the same 576-wide key / 512-wide value rows: an
// MQA problem with 64 query heads per token.
//
// One CTA owns 64 query rows (row = token * H + head, heads fastest) of one
// sequence and one split of its context.  Eight warps.  Scores: warp w computes
// rows (w % 4) * 16 .. +16 x keys (w / 4) * 16 .. +16 of each 32-key tile; row
// maxima and sums are exchanged through shared memory and P (bf16) is written
// there.  Output: warp w owns all 64 rows x value columns w * 64 .. +64, so every
// V fragment is read from shared memory once per tile.  The running max / sum
// and the per-tile rescale factors live in shared memory.  With more than one
// split, a second kernel merges the fp32 partials in split order (deterministic).
//
// The reference has no MLA kernel (DeepSeek/Kimi are metadata profiles only:
// si/model/architecture_adapters.py:735-976); the math follows the DeepSeek-V3
// attention definition with absorbed up-projections.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sil/host.h"
#include "sil/mma.cuh"
#include "sil/ptx.cuh"

namespace sil {
namespace {

constexpr int kLat = 512;
constexpr int kRope = 64;
constexpr int kQK = kLat + kRope;          // 576
constexpr int kPage = 64;
constexpr int kTile = 32;                  // keys per pipeline stage
constexpr int kChunks = kQK / 64;          // nine 64-column boxes
constexpr int kBoxBytes = kTile * 128;     // [32 rows x 64 cols] bf16
constexpr int kStageBytes = kChunks * kBoxBytes;  // 36 KB
constexpr int kStages = 3;
constexpr int kRows = 64;                  // query rows per CTA
constexpr int kQChunkBytes = kRows * 128;  // [64 rows x 64 cols]
constexpr int kQBytes = kChunks * kQChunkBytes;    // 72 KB
constexpr int kPStride = 40;               // bf16 elements per P row (80 B: conflict-free)
constexpr int kThreads = 256;
constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kQBytes + kRows * kPStride * 2 +
                           8 * kRows * 4 + 64;

struct MlaArgs {
  const __nv_bfloat16* q_lat;   // [.., 512] rows at token * qt_stride + head * qh_stride
  long long qt_stride, qh_stride;
  const __nv_bfloat16* q_pe;    // [.., 64]
  long long pt_stride, ph_stride;
  __nv_bfloat16* out;           // o_lat rows at token * ot_stride + head * oh_stride
  long long ot_stride, oh_stride;
  const int* block_table;
  long long bt_stride;
  const int* seq_lens;          // context incl. this step's tokens
  const int* cu_q;              // [B+1] query offsets, or null (one query per sequence)
  int H;                        // query heads
  int num_splits;
  float scale_log2;
  float* ws_o;                  // [B, RB, S, 64, 512] partial outputs
  float* ws_ml;                 // [B, RB, S, 64, 2]
  int* status;
};

__device__ __forceinline__ uint32_t q_addr(uint32_t base, int row, int col) {
  const int chunk = col >> 6, cc = (col >> 3) & 7;
  return base + chunk * kQChunkBytes + row * 128 + ((cc ^ (row & 7)) << 4);
}

__device__ __forceinline__ uint32_t kv_addr(uint32_t base, int key, int col) {
  const int chunk = col >> 6, cc = (col >> 3) & 7;
  return base + chunk * kBoxBytes + key * 128 + ((cc ^ (key & 7)) << 4);
}

__device__ __forceinline__ void issue_tile(uint8_t* stage, const CUtensorMap* map, uint64_t* bar,
                                           int row) {
  mbar_arrive_expect_tx(bar, kStageBytes);
#pragma unroll
  for (int c = 0; c < kChunks; ++c) tma_load_2d(stage + c * kBoxBytes, map, bar, c * 64, row);
}

__global__ void __launch_bounds__(kThreads, 1)
    mla_attention_kernel(const __grid_constant__ CUtensorMap tmC, const MlaArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem + kStages * kStageBytes;
  __nv_bfloat16* sP = reinterpret_cast<__nv_bfloat16*>(sQ + kQBytes);
  float* red_max = reinterpret_cast<float*>(sP + kRows * kPStride);  // [2][64]
  float* red_sum = red_max + 2 * kRows;                                // [2][64]
  float* s_m = red_sum + 2 * kRows;                                    // running max [64]
  float* s_l = s_m + kRows;                                            // running sum [64]
  float* s_alpha = s_l + kRows;                                        // this tile's rescale [64]
  float* s_mnew = s_alpha + kRows;                                     // this tile's max [64]
  uint64_t* full = reinterpret_cast<uint64_t*>(s_mnew + kRows);
  int* sflag = reinterpret_cast<int*>(full + kStages);

  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rg = warp & 3, vh = warp >> 2;
  const int split = blockIdx.x, b = blockIdx.z;
  const int RB = gridDim.y;
  const int rb = RB - 1 - (int)blockIdx.y;  // causal prefill: heaviest row blocks first
  const int S = args.num_splits;
  const int H = args.H;
  const int q_begin = args.cu_q ? args.cu_q[b] : b;
  const int q_len = args.cu_q ? args.cu_q[b + 1] - q_begin : 1;
  const int rows_total = q_len * H;
  const int row0 = rb * kRows;
  if (row0 >= rows_total) return;
  const int kv_len = args.seq_lens[b];
  const int pos0 = kv_len - q_len;
  const int last_row = min(row0 + kRows, rows_total) - 1;
  const int key_end = min(kv_len, pos0 + last_row / H + 1);  // keys this row block may see
  const int n_tiles = (key_end + kTile - 1) / kTile;
  const int per = (n_tiles + S - 1) / S;
  const int t_begin = split * per;
  const int count = max(0, min(n_tiles, t_begin + per) - t_begin);
  const int* bt = args.block_table + (long long)b * args.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    sflag[0] = load_status(args.status);
    sflag[1] = 0;
  }
  __syncthreads();
  const bool skip = sflag[0] != 0;
  auto tile_row = [&](int ti) { return bt[ti >> 1] * kPage + (ti & 1) * kTile; };
  if (!skip && threadIdx.x == 0) {
    for (int i = 0; i < min(count, kStages); ++i)
      issue_tile(smem + i * kStageBytes, &tmC, &full[i], tile_row(t_begin + i));
  }

  // Q rows -> shared memory (swizzled like the TMA boxes).
  const uint32_t qbase = smem_u32(sQ);
  for (int u = threadIdx.x; u < kRows * (kQK / 8); u += kThreads) {
    const int r = u / (kQK / 8), j = u % (kQK / 8);
    const int row = row0 + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < rows_total) {
      const int tok = q_begin + row / H, h = row % H;
      const __nv_bfloat16* src =
          j < kLat / 8 ? args.q_lat + tok * args.qt_stride + h * args.qh_stride + j * 8
                       : args.q_pe + tok * args.pt_stride + h * args.ph_stride + (j - kLat / 8) * 8;
      v = *reinterpret_cast<const uint4*>(src);
    }
    const int col = j * 8;
    *reinterpret_cast<uint4*>(sQ + (q_addr(0, r, col))) = v;
  }
  __syncthreads();

  // Scores: warp (rg, vh) owns rows rg*16..+16 and keys vh*16..+16 of each tile.
  int lim[2];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int row = row0 + rg * 16 + g + 8 * rr;
    lim[rr] = row < rows_total ? min(kv_len - 1, pos0 + row / H) : -1;
  }
  if (threadIdx.x < kRows) {
    s_m[threadIdx.x] = -INFINITY;
    s_l[threadIdx.x] = 0.f;
  }
  // Output: warp w owns all 64 rows x value columns w*64..+64 (4 m-tiles x 8 n-tiles).
  float o[4][8][4];
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
  bool alive = !skip;
  __syncthreads();

  for (int i = 0; i < count; ++i) {
    const int s = i % kStages;
    if (alive && !mbar_wait(&full[s], (i / kStages) & 1, args.status, kStatusTimeoutFull))
      alive = false;
    const uint32_t kvb = smem_u32(smem + s * kStageBytes);
    const int key0 = (t_begin + i) * kTile;
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
    if (alive) {
#pragma unroll 4
      for (int ks = 0; ks < kQK / 16; ++ks) {
        uint32_t a[4];
        ldmatrix_x4(q_addr(qbase, rg * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8), a[0], a[1],
                    a[2], a[3]);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(kv_addr(kvb, vh * 16 + (lane & 7) + ((lane >> 4) << 3),
                            ks * 16 + ((lane >> 3) & 1) * 8),
                    b0, b1, b2, b3);
        mma_bf16_16816(sc[0], a, b0, b1);
        mma_bf16_16816(sc[1], a, b2, b3);
      }
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = key0 + vh * 16 + nt * 8 + 2 * t + (j & 1);
        float v = sc[nt][j] * args.scale_log2;
        if (key > lim[j >> 1]) v = -INFINITY;
        sc[nt][j] = v;
        mx[j >> 1] = fmaxf(mx[j >> 1], v);
      }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
      if (t == 0) red_max[vh * kRows + rg * 16 + g + 8 * rr] = mx[rr];
    }
    __syncthreads();
    // Probabilities with the row's new running max; the vh == 0 warp publishes alpha.
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int r = rg * 16 + g + 8 * rr;
      const float m_old = s_m[r];
      const float m_new = fmaxf(m_old, fmaxf(red_max[r], red_max[kRows + r]));
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const float p0 = exp2f(sc[nt][2 * rr] - m_use);
        const float p1 = exp2f(sc[nt][2 * rr + 1] - m_use);
        rs[rr] += p0 + p1;
        *reinterpret_cast<uint32_t*>(sP + r * kPStride + vh * 16 + nt * 8 + 2 * t) =
            pack_bf16x2(p0, p1);
      }
      rs[rr] += __shfl_xor_sync(0xffffffffu, rs[rr], 1);
      rs[rr] += __shfl_xor_sync(0xffffffffu, rs[rr], 2);
      if (t == 0) {
        red_sum[vh * kRows + r] = rs[rr];
        if (vh == 0) {
          s_alpha[r] = exp2f(m_old - m_use);
          s_mnew[r] = m_new;
        }
      }
    }
    __syncthreads();
    if (threadIdx.x < kRows) {
      const int r = threadIdx.x;
      s_l[r] = s_l[r] * s_alpha[r] + red_sum[r] + red_sum[kRows + r];
      s_m[r] = s_mnew[r];
    }
    float al[4][2];
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      al[mt][0] = s_alpha[mt * 16 + g];
      al[mt][1] = s_alpha[mt * 16 + g + 8];
    }
#pragma unroll
    for (int mt = 0; mt < 4; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        o[mt][nt][0] *= al[mt][0]; o[mt][nt][1] *= al[mt][0];
        o[mt][nt][2] *= al[mt][1]; o[mt][nt][3] *= al[mt][1];
      }
    if (alive) {
      const uint32_t pbase = smem_u32(sP);
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk) {
        uint32_t pa[4][4];
#pragma unroll
        for (int mt = 0; mt < 4; ++mt)
          ldmatrix_x4(pbase + ((mt * 16 + (lane & 15)) * kPStride + kk * 16 + (lane >> 4) * 8) * 2,
                      pa[mt][0], pa[mt][1], pa[mt][2], pa[mt][3]);
#pragma unroll
        for (int nd2 = 0; nd2 < 4; ++nd2) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(kv_addr(kvb, kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8,
                                    warp * 64 + nd2 * 16 + (lane >> 4) * 8),
                            b0, b1, b2, b3);
#pragma unroll
          for (int mt = 0; mt < 4; ++mt) {
            mma_bf16_16816(o[mt][2 * nd2], pa[mt], b0, b1);
            mma_bf16_16816(o[mt][2 * nd2 + 1], pa[mt], b2, b3);
          }
        }
      }
    }
    __syncthreads();
    if (alive && threadIdx.x == 0 && i + kStages < count)
      issue_tile(smem + s * kStageBytes, &tmC, &full[s], tile_row(t_begin + i + kStages));
  }

  // Epilogue: final rows (one split) or fp32 partials + (max, sum) for the merge kernel.
  const long long slot = ((long long)b * RB + rb) * S + split;
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int r = mt * 16 + g + 8 * rr;
      const int row = row0 + r;
      if (row >= rows_total || skip) continue;
      if (S == 1) {
        const float L = s_l[r];
        const float inv = L > 0.f ? 1.f / L : 0.f;
        const int tok = q_begin + row / H, h = row % H;
        __nv_bfloat16* dst = args.out + tok * args.ot_stride + h * args.oh_stride + warp * 64 + 2 * t;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
          *reinterpret_cast<uint32_t*>(dst + nt * 8) =
              pack_bf16x2(o[mt][nt][2 * rr] * inv, o[mt][nt][2 * rr + 1] * inv);
      } else {
        float* dst = args.ws_o + (slot * kRows + r) * kLat + warp * 64 + 2 * t;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
          *reinterpret_cast<float2*>(dst + nt * 8) = make_float2(o[mt][nt][2 * rr], o[mt][nt][2 * rr + 1]);
        if (warp == 0 && t == 0) {
          args.ws_ml[(slot * kRows + r) * 2] = s_m[r];
          args.ws_ml[(slot * kRows + r) * 2 + 1] = s_l[r];
        }
      }
    }
}

// Merge the split partials of one (sequence, row block) in split order: 8 rows per CTA.
__global__ void __launch_bounds__(256)
    mla_merge_kernel(const MlaArgs args, int RB) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.z, rb = blockIdx.y, r0 = blockIdx.x * 8;
  const int S = args.num_splits, H = args.H;
  const int q_begin = args.cu_q ? args.cu_q[b] : b;
  const int q_len = args.cu_q ? args.cu_q[b + 1] - q_begin : 1;
  const int rows_total = q_len * H;
  if (load_status(args.status) != 0) return;
  const long long base0 = ((long long)b * RB + rb) * S;
  for (int e = threadIdx.x; e < 8 * (kLat / 4); e += blockDim.x) {
    const int r = r0 + e / (kLat / 4), d = (e % (kLat / 4)) * 4;
    const int row = rb * kRows + r;
    if (row >= rows_total) continue;
    float M = -INFINITY;
    for (int sp = 0; sp < S; ++sp) M = fmaxf(M, args.ws_ml[((base0 + sp) * kRows + r) * 2]);
    const float Mu = M == -INFINITY ? 0.f : M;
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < S; ++sp) {
      const long long sr = (base0 + sp) * kRows + r;
      const float f = exp2f(args.ws_ml[sr * 2] - Mu);
      L += args.ws_ml[sr * 2 + 1] * f;
      const float4 v = *reinterpret_cast<const float4*>(args.ws_o + sr * kLat + d);
      acc.x += v.x * f; acc.y += v.y * f; acc.z += v.z * f; acc.w += v.w * f;
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    const int tok = q_begin + row / H, h = row % H;
    __nv_bfloat16* dst = args.out + tok * args.ot_stride + h * args.oh_stride + d;
    *reinterpret_cast<uint2*>(dst) =
        make_uint2(pack_bf16x2(acc.x * inv, acc.y * inv), pack_bf16x2(acc.z * inv, acc.w * inv));
  }
}

// kv_a row [c(512) | k_pe(64)] -> cache[slot] = [rmsnorm(c) * w | rope_interleaved(k_pe)].
// One warp per token.
__global__ void mla_kv_write_kernel(const __nv_bfloat16* __restrict__ kv, long long ld,
                                    const float* __restrict__ w, float eps,
                                    const int* __restrict__ positions, const int* __restrict__ slots,
                                    const float* __restrict__ cos_sin,  // [max_pos, 64]
                                    __nv_bfloat16* __restrict__ cache, int T) {
  pdl_trigger();
  pdl_wait();
  const int tok = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (tok >= T) return;
  const int slot = slots[tok];
  if (slot < 0) return;
  const __nv_bfloat16* src = kv + tok * ld;
  float v[16];
  const uint4 r0 = *reinterpret_cast<const uint4*>(src + lane * 16);
  const uint4 r1 = *reinterpret_cast<const uint4*>(src + lane * 16 + 8);
  const uint32_t raw[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = bf16_lo(raw[i]);
    v[2 * i + 1] = bf16_hi(raw[i]);
    ss += v[2 * i] * v[2 * i] + v[2 * i + 1] * v[2 * i + 1];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / kLat + eps);
  __nv_bfloat16* dst = cache + (long long)slot * kQK;
  uint32_t packed[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    packed[i] = pack_bf16x2(v[2 * i] * inv * w[lane * 16 + 2 * i],
                            v[2 * i + 1] * inv * w[lane * 16 + 2 * i + 1]);
  *reinterpret_cast<uint4*>(dst + lane * 16) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  *reinterpret_cast<uint4*>(dst + lane * 16 + 8) = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  // Rope pair (2 lane, 2 lane + 1) with frequency `lane`.
  const uint32_t pe = *reinterpret_cast<const uint32_t*>(src + kLat + 2 * lane);
  const float x0 = bf16_lo(pe), x1 = bf16_hi(pe);
  const float* cs = cos_sin + (long long)positions[tok] * kRope;
  const float c = cs[lane], s = cs[32 + lane];
  *reinterpret_cast<uint32_t*>(dst + kLat + 2 * lane) = pack_bf16x2(x0 * c - x1 * s, x1 * c + x0 * s);
}

// q [T, H*192] (nope 128 | pe 64 per head) -> q_nope_t [H, T, 128] (grouped-GEMM input) and
// rotated q_pe [T, H, 64].  One warp per (token, head).
__global__ void mla_q_prep_kernel(const __nv_bfloat16* __restrict__ q, long long ld,
                                  const int* __restrict__ positions,
                                  const float* __restrict__ cos_sin, __nv_bfloat16* __restrict__ q_nope,
                                  __nv_bfloat16* __restrict__ q_pe, int T, int H) {
  pdl_trigger();
  pdl_wait();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= T * H) return;
  const int tok = w / H, h = w % H;
  const __nv_bfloat16* src = q + tok * ld + h * 192;
  *reinterpret_cast<uint2*>(q_nope + ((long long)h * T + tok) * 128 + lane * 4) =
      *reinterpret_cast<const uint2*>(src + lane * 4);
  const uint32_t pe = *reinterpret_cast<const uint32_t*>(src + 128 + 2 * lane);
  const float x0 = bf16_lo(pe), x1 = bf16_hi(pe);
  const float* cs = cos_sin + (long long)positions[tok] * kRope;
  const float c = cs[lane], s = cs[32 + lane];
  *reinterpret_cast<uint32_t*>(q_pe + ((long long)tok * H + h) * kRope + 2 * lane) =
      pack_bf16x2(x0 * c - x1 * s, x1 * c + x0 * s);
}

// [H, T, D] -> [T, H*D] (D = 128), 16 bytes per thread.
__global__ void mla_head_major_to_token_major(const __nv_bfloat16* __restrict__ src,
                                              __nv_bfloat16* __restrict__ dst, long long ldd, int T,
                                              int H) {
  pdl_trigger();
  pdl_wait();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long n = (long long)T * H * 16;
  if (i >= n) return;
  const int u = i % 16;
  const long long th = i / 16;
  const int h = th % H, tok = th / H;
  *reinterpret_cast<uint4*>(dst + tok * ldd + h * 128 + u * 8) =
      *reinterpret_cast<const uint4*>(src + ((long long)h * T + tok) * 128 + u * 8);
}

}  // namespace

// q_lat / q_pe / out: 3-D views [tokens, heads, dim] with arbitrary token/head strides
// (unit stride in dim); cache [pages, 64, 576]; cu_q null for one query per sequence.
void mla_attention(const at::Tensor& q_lat, const at::Tensor& q_pe, const at::Tensor& cache,
                   const at::Tensor& block_table, const at::Tensor& seq_lens,
                   const c10::optional<at::Tensor>& cu_q, at::Tensor& out, double scale,
                   int64_t max_q_len, int64_t num_splits, const at::Tensor& ws,
                   const at::Tensor& counters, const at::Tensor& status) {
  TORCH_CHECK(cache.scalar_type() == at::kBFloat16 && cache.dim() == 3 && cache.size(1) == kPage &&
                  cache.size(2) == kQK && cache.is_contiguous(),
              "mla: cache must be [pages, 64, 576] bf16");
  TORCH_CHECK(q_lat.dim() == 3 && q_lat.size(2) == kLat && q_lat.stride(2) == 1, "mla: q_lat [T, H, 512]");
  TORCH_CHECK(q_pe.dim() == 3 && q_pe.size(2) == kRope && q_pe.stride(2) == 1, "mla: q_pe [T, H, 64]");
  TORCH_CHECK(out.dim() == 3 && out.size(2) == kLat && out.stride(2) == 1, "mla: out [T, H, 512]");
  TORCH_CHECK(q_lat.stride(0) % 8 == 0 && q_lat.stride(1) % 8 == 0 && q_pe.stride(0) % 8 == 0 &&
                  q_pe.stride(1) % 8 == 0,
              "mla: q strides must keep 16-byte rows");
  const int B = seq_lens.size(0);
  const int H = q_lat.size(1);
  if (B == 0 || max_q_len <= 0) return;
  const int S = static_cast<int>(std::max<int64_t>(1, num_splits));
  const int RB = static_cast<int>((max_q_len * H + kRows - 1) / kRows);
  TORCH_CHECK(S == 1 || (long long)B * RB * S * kRows * (kLat + 2) <= ws.numel(),
              "mla: split workspace too small");
  c10::cuda::CUDAGuard guard(q_lat.device());
  MlaArgs a{};
  a.q_lat = reinterpret_cast<const __nv_bfloat16*>(q_lat.data_ptr());
  a.qt_stride = q_lat.stride(0);
  a.qh_stride = q_lat.stride(1);
  a.q_pe = reinterpret_cast<const __nv_bfloat16*>(q_pe.data_ptr());
  a.pt_stride = q_pe.stride(0);
  a.ph_stride = q_pe.stride(1);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ot_stride = out.stride(0);
  a.oh_stride = out.stride(1);
  a.block_table = block_table.data_ptr<int>();
  a.bt_stride = block_table.stride(0);
  a.seq_lens = seq_lens.data_ptr<int>();
  a.cu_q = cu_q.has_value() ? cu_q->data_ptr<int>() : nullptr;
  a.H = H;
  a.num_splits = S;
  a.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  a.ws_o = ws.data_ptr<float>();
  a.ws_ml = a.ws_o + (long long)B * RB * S * kRows * kLat;
  (void)counters;  // split partials are merged by mla_merge_kernel; no arrival counters
  a.status = status.data_ptr<int>();
  const uint64_t rows = (uint64_t)cache.size(0) * kPage;
  CUtensorMap tm = make_tmap_2d(cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, kQK, kQK,
                                kTile, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  set_smem_limit(reinterpret_cast<const void*>(mla_attention_kernel), kSmemBytes, "cudaFuncSetAttribute(mla)");
  dim3 grid(S, RB, B);
  launch_pdl(mla_attention_kernel, grid, dim3(kThreads), kSmemBytes,
             at::cuda::getCurrentCUDAStream(), "mla_attention launch", tm, a);
  if (S > 1)
    launch_pdl(mla_merge_kernel, dim3(kRows / 8, RB, B), dim3(256), 0,
               at::cuda::getCurrentCUDAStream(), "mla_merge launch", a, RB);
}

void mla_kv_write(const at::Tensor& kv, const at::Tensor& norm_w, double eps,
                  const at::Tensor& positions, const at::Tensor& slots, const at::Tensor& cos_sin,
                  at::Tensor& cache) {
  TORCH_CHECK(kv.scalar_type() == at::kBFloat16 && kv.size(1) >= kQK && kv.stride(1) == 1 &&
                  kv.stride(0) % 8 == 0,
              "mla_kv_write: kv [T, >=576] bf16 with 16-byte rows");
  TORCH_CHECK(norm_w.scalar_type() == at::kFloat && norm_w.numel() == kLat, "mla_kv_write: fp32 norm weight [512]");
  TORCH_CHECK(cos_sin.size(1) == kRope, "mla_kv_write: cos/sin table [max_pos, 64]");
  TORCH_CHECK(cache.size(1) == kPage && cache.size(2) == kQK, "mla_kv_write: cache [pages, 64, 576]");
  const int T = kv.size(0);
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(kv.device());
  const int threads = 256;
  launch_pdl(mla_kv_write_kernel, dim3((T * 32 + threads - 1) / threads), dim3(threads), 0,
             at::cuda::getCurrentCUDAStream(), "mla_kv_write launch",
             reinterpret_cast<const __nv_bfloat16*>(kv.data_ptr()), (long long)kv.stride(0),
             (const float*)norm_w.data_ptr<float>(), static_cast<float>(eps),
             (const int*)positions.data_ptr<int>(), (const int*)slots.data_ptr<int>(),
             (const float*)cos_sin.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(cache.data_ptr()),
             T);
}

void mla_q_prep(const at::Tensor& q, const at::Tensor& positions, const at::Tensor& cos_sin,
                at::Tensor& q_nope, at::Tensor& q_pe, int64_t H) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.stride(1) == 1 && q.size(1) == H * 192 &&
                  q.stride(0) % 8 == 0,
              "mla_q_prep: q [T, H*192] bf16");
  const int T = q.size(0);
  TORCH_CHECK(q_nope.numel() == (long long)H * T * 128 && q_nope.is_contiguous(), "mla_q_prep: q_nope [H, T, 128]");
  TORCH_CHECK(q_pe.numel() == (long long)T * H * kRope && q_pe.is_contiguous(), "mla_q_prep: q_pe [T, H, 64]");
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(q.device());
  const int threads = 256;
  const long long warps = (long long)T * H;
  launch_pdl(mla_q_prep_kernel, dim3((warps * 32 + threads - 1) / threads), dim3(threads), 0,
             at::cuda::getCurrentCUDAStream(), "mla_q_prep launch",
             reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), (long long)q.stride(0),
             (const int*)positions.data_ptr<int>(), (const float*)cos_sin.data_ptr<float>(),
             reinterpret_cast<__nv_bfloat16*>(q_nope.data_ptr()),
             reinterpret_cast<__nv_bfloat16*>(q_pe.data_ptr()), T, (int)H);
}

void mla_heads_to_tokens(const at::Tensor& src, at::Tensor& dst, int64_t T, int64_t H) {
  TORCH_CHECK(src.is_contiguous() && src.numel() == T * H * 128, "mla: src [H, T, 128]");
  TORCH_CHECK(dst.stride(1) == 1 && dst.size(1) >= H * 128 && dst.stride(0) % 8 == 0, "mla: dst [T, H*128]");
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(src.device());
  const long long n = T * H * 16;
  launch_pdl(mla_head_major_to_token_major, dim3((n + 255) / 256), dim3(256), 0,
             at::cuda::getCurrentCUDAStream(), "mla_heads_to_tokens launch",
             reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()),
             reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()), (long long)dst.stride(0), (int)T,
             (int)H);
}

}  // namespace sil
