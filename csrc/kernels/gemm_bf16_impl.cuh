#pragma once
// Dense bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM) with
// TMA-fed, mbarrier-pipelined shared-memory stages and fused epilogues.
//
//   y[T, Nout] = epilogue( x[T, K] . W[Nw, K]^T )
//
// Two operand orders share one kernel template:
//  * normal  (prefill, T > 128): A = x (M = tokens), B = W (N = features),
//    BN = 128/256.  The accumulator row is a token, columns are features.
//  * swapped (decode, T <= 128):  A = W (M = features), B = x (N = tokens,
//    padded to 16/32/64/128).  Weight streaming is the bound here, so the
//    kernel splits K across CTAs (split-K) until the grid covers every SM;
//    partial tiles go to an fp32 workspace and the last CTA of a tile sums
//    them in split order (deterministic) before the epilogue.
//
// Epilogues: plain bf16 store, residual add (y = acc + r, in place allowed),
// SwiGLU (y = silu(gate) * up from a fused [gate; up] weight) and fp32 store
// (LM-head logits).  Warp roles: warp 0 issues TMA, warp 1 issues tcgen05.mma
// (single elected thread) and owns the TMEM allocation, warps 2-5 drain TMEM.
//
// Replaces the per-layer F.linear / cuBLAS calls of the reference's decoder
// layers (si/microsharding/dense.py:320-412, HF layers via si/model/qwen3.py:517-546).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sil/host.h"
#include "sil/ptx.cuh"

namespace sil {
namespace gemm_detail {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

enum EpiKind : int { kEpiBf16 = 0, kEpiResAdd = 1, kEpiSwiGLU = 2, kEpiF32 = 3 };

struct GemmArgs {
  int M;       // rows of A that are valid (features in swapped mode, tokens otherwise)
  int N;       // valid output columns of the accumulator space (tokens / features)
  int num_kb;  // number of 64-wide K blocks
  int splits;  // split-K factor (grid.z)
  int inter;   // SwiGLU: row offset of the 'up' half inside the fused weight
  void* out;
  long long ldo;
  const __nv_bfloat16* res;
  long long ldr;
  float* ws;
  int* counters;
  int* status;
};

template <int BN, int STAGES, int EPI, bool SWAP>
struct Cfg {
  static constexpr bool kSwiGLU = EPI == kEpiSwiGLU;
  static constexpr int NUM_A = (kSwiGLU && SWAP) ? 2 : 1;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = NUM_A * A_BYTES + B_BYTES;
  static constexpr int ACC_COLS = NUM_A * BN;
  // Output columns produced per tile (SwiGLU in normal order halves them).
  static constexpr int OUT_COLS = (kSwiGLU && !SWAP) ? BN / 2 : BN;
  static constexpr int TMEM_COLS =
      ACC_COLS <= 32 ? 32 : ACC_COLS <= 64 ? 64 : ACC_COLS <= 128 ? 128 : ACC_COLS <= 256 ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N constraint for M=128");
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");
};

// Store CW consecutive accumulator columns [n0, n0+CW) of accumulator row `m_glob`.
template <int EPI, bool SWAP, int CW>
__device__ __forceinline__ void store_chunk(const GemmArgs& a, int m_glob, int n0,
                                            const float (&v)[CW], const float (&u)[CW]) {
  if (m_glob >= a.M) return;
  if constexpr (SWAP) {
    // Accumulator row = output feature m_glob, column = token n.
#pragma unroll
    for (int j = 0; j < CW; ++j) {
      const int n = n0 + j;
      if (n < a.N) {
        float r = v[j];
        if constexpr (EPI == kEpiSwiGLU) r = silu_f(v[j]) * u[j];
        if constexpr (EPI == kEpiF32) {
          reinterpret_cast<float*>(a.out)[(long long)n * a.ldo + m_glob] = r;
        } else {
          if constexpr (EPI == kEpiResAdd) r += __bfloat162float(a.res[(long long)n * a.ldr + m_glob]);
          reinterpret_cast<__nv_bfloat16*>(a.out)[(long long)n * a.ldo + m_glob] =
              __float2bfloat16_rn(r);
        }
      }
    }
  } else {
    // Accumulator row = token m_glob, columns = output features n0 + j.
    if constexpr (EPI == kEpiF32) {
      float* o = reinterpret_cast<float*>(a.out) + (long long)m_glob * a.ldo;
      if (n0 + CW <= a.N && (a.ldo & 3) == 0) {
#pragma unroll
        for (int j = 0; j < CW; j += 4)
          *reinterpret_cast<float4*>(o + n0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      } else {
        for (int j = 0; j < CW; ++j)
          if (n0 + j < a.N) o[n0 + j] = v[j];
      }
    } else {
      float r[CW];
#pragma unroll
      for (int j = 0; j < CW; ++j) {
        r[j] = v[j];
        if constexpr (EPI == kEpiSwiGLU) r[j] = silu_f(v[j]) * u[j];
      }
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) + (long long)m_glob * a.ldo;
      const bool vec = (n0 + CW <= a.N) && ((a.ldo & 7) == 0) &&
                       (EPI != kEpiResAdd || (a.ldr & 7) == 0);
      if (vec) {
        if constexpr (EPI == kEpiResAdd) {
          const __nv_bfloat16* rr = a.res + (long long)m_glob * a.ldr + n0;
#pragma unroll
          for (int j = 0; j < CW; j += 8) {
            uint4 q = *reinterpret_cast<const uint4*>(rr + j);
            r[j + 0] += bf16_lo(q.x); r[j + 1] += bf16_hi(q.x);
            r[j + 2] += bf16_lo(q.y); r[j + 3] += bf16_hi(q.y);
            r[j + 4] += bf16_lo(q.z); r[j + 5] += bf16_hi(q.z);
            r[j + 6] += bf16_lo(q.w); r[j + 7] += bf16_hi(q.w);
          }
        }
#pragma unroll
        for (int j = 0; j < CW; j += 8) {
          uint4 q;
          q.x = pack_bf16x2(r[j + 0], r[j + 1]);
          q.y = pack_bf16x2(r[j + 2], r[j + 3]);
          q.z = pack_bf16x2(r[j + 4], r[j + 5]);
          q.w = pack_bf16x2(r[j + 6], r[j + 7]);
          *reinterpret_cast<uint4*>(o + n0 + j) = q;
        }
      } else {
        for (int j = 0; j < CW; ++j) {
          const int n = n0 + j;
          if (n < a.N) {
            float x = r[j];
            if constexpr (EPI == kEpiResAdd) x += __bfloat162float(a.res[(long long)m_glob * a.ldr + n]);
            o[n] = __float2bfloat16_rn(x);
          }
        }
      }
    }
  }
}

template <int CW>
__device__ __forceinline__ void tmem_load(uint32_t taddr, uint32_t (&r)[CW]) {
  if constexpr (CW == 32) {
    tmem_ld32_sync(taddr, r);
  } else {
    tmem_ld16(taddr, r);
    tmem_ld_wait();
    // Register dependency: keep uses of r after the wait.
#pragma unroll
    for (int j = 0; j < CW; ++j) asm volatile("" : "+r"(r[j]));
  }
}

template <int BN, int STAGES, int EPI, bool SWAP>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
  using C = Cfg<BN, STAGES, EPI, SWAP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accum_full = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_full + 1);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] skip, [1] last split

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tile = blockIdx.x;
  const int n_tile = blockIdx.y;
  const int split = blockIdx.z;
  const int tile_id = blockIdx.y * gridDim.x + blockIdx.x;
  const int kb_per = args.num_kb / args.splits;
  const int kb_rem = args.num_kb % args.splits;
  const int kb0 = split * kb_per + min(split, kb_rem);
  const int nkb = kb_per + (split < kb_rem ? 1 : 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum_full, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    flags[0] = load_status(args.status) != 0 || nkb <= 0;
    flags[1] = 0;
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const bool skip = flags[0] != 0;

  if (!skip) {
    if (warp == 0) {
      if (lane == 0) {
        // Weights are streamed once per step: evict them first so activations stay in L2.
        const uint64_t pol_w = l2_policy_evict_first();
        const uint64_t pol_x = l2_policy_evict_last();
        const uint64_t pol_a = SWAP ? pol_w : pol_x;
        const uint64_t pol_b = SWAP ? pol_x : pol_w;
        for (int i = 0; i < nkb; ++i) {
          const int s = i % STAGES;
          const uint32_t r = i / STAGES;
          if (!mbar_wait(&empty[s], (r & 1) ^ 1, args.status, kStatusTimeoutEmpty)) break;
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          uint8_t* sb = sa + C::NUM_A * C::A_BYTES;
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          const int kx = (kb0 + i) * BK;
          tma_load_2d_hint(sa, &tmA, &full[s], kx, m_tile * BM, pol_a);
          if constexpr (C::NUM_A == 2)
            tma_load_2d_hint(sa + C::A_BYTES, &tmA, &full[s], kx, m_tile * BM + args.inter, pol_a);
          if constexpr (C::kSwiGLU && !SWAP) {
            tma_load_2d_hint(sb, &tmB, &full[s], kx, n_tile * (BN / 2), pol_b);
            tma_load_2d_hint(sb + (BN / 2) * 128, &tmB, &full[s], kx,
                             n_tile * (BN / 2) + args.inter, pol_b);
          } else {
            tma_load_2d_hint(sb, &tmB, &full[s], kx, n_tile * BN, pol_b);
          }
        }
      }
    } else if (warp == 1) {
      if (lane == 0) {
        constexpr uint32_t idesc = umma_idesc_bf16(BM, BN);
        bool ok = true;
        for (int i = 0; i < nkb; ++i) {
          const int s = i % STAGES;
          const uint32_t r = i / STAGES;
          if (!mbar_wait(&full[s], r & 1, args.status, kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + C::NUM_A * C::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t bd = umma_desc_sw128(b_addr + k * 32);
            umma_f16(tmem_base, umma_desc_sw128(a_addr + k * 32), bd, idesc, (i | k) != 0);
            if constexpr (C::NUM_A == 2)
              umma_f16(tmem_base + BN, umma_desc_sw128(a_addr + C::A_BYTES + k * 32), bd, idesc,
                       (i | k) != 0);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(accum_full);
      }
    } else {
      // Epilogue warps 2..5: warp w may only touch TMEM lanes [32*(w%4), 32*(w%4)+32).
      const int q = warp & 3;
      const int row = q * 32 + lane;
      const int m_glob = m_tile * BM + row;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
      bool ok = mbar_wait(accum_full, 0, args.status, kStatusTimeoutAccum);
      if (ok) tc_fence_after();
      bool do_final = ok;
      constexpr int CW = (C::OUT_COLS >= 32 && BN >= 32) ? 32 : 16;  // columns per TMEM load
      if (ok && args.splits > 1) {
        float* mine = args.ws + ((long long)tile_id * args.splits + split) * C::ACC_COLS * BM;
#pragma unroll 1
        for (int c0 = 0; c0 < C::ACC_COLS; c0 += CW) {
          uint32_t v[CW];
          tmem_load<CW>(taddr + c0, v);
#pragma unroll
          for (int j = 0; j < CW; ++j) __stcg(&mine[(c0 + j) * BM + row], __uint_as_float(v[j]));
        }
        __threadfence();
        named_bar_sync(1, 128);
        if (threadIdx.x == 64) {
          const int old = atomicAdd(&args.counters[tile_id], 1);
          flags[1] = (old == args.splits - 1);
        }
        named_bar_sync(1, 128);
        do_final = flags[1] != 0;
        if (do_final) __threadfence();
      }
      if (do_final) {
        const float* base = args.ws + (long long)tile_id * args.splits * C::ACC_COLS * BM;
        constexpr int UOFF = SWAP ? BN : BN / 2;  // column offset of the SwiGLU 'up' half
#pragma unroll 1
        for (int c0 = 0; c0 < C::OUT_COLS; c0 += CW) {
          float v[CW], u[CW];
          if (args.splits == 1) {
            uint32_t rv[CW];
            tmem_load<CW>(taddr + c0, rv);
#pragma unroll
            for (int j = 0; j < CW; ++j) v[j] = __uint_as_float(rv[j]);
            if constexpr (C::kSwiGLU) {
              tmem_load<CW>(taddr + c0 + UOFF, rv);
#pragma unroll
              for (int j = 0; j < CW; ++j) u[j] = __uint_as_float(rv[j]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < CW; ++j) { v[j] = 0.f; u[j] = 0.f; }
            for (int s = 0; s < args.splits; ++s) {
              const float* p = base + (long long)s * C::ACC_COLS * BM;
#pragma unroll
              for (int j = 0; j < CW; ++j) v[j] += __ldcg(&p[(c0 + j) * BM + row]);
              if constexpr (C::kSwiGLU) {
#pragma unroll
                for (int j = 0; j < CW; ++j) u[j] += __ldcg(&p[(c0 + UOFF + j) * BM + row]);
              }
            }
          }
          const int n0 = n_tile * C::OUT_COLS + c0;
          store_chunk<EPI, SWAP, CW>(args, m_glob, n0, v, u);
        }
        if (args.splits > 1) {
          named_bar_sync(1, 128);
          if (threadIdx.x == 64) args.counters[tile_id] = 0;  // re-arm for the next launch
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <int BN, int STAGES, int EPI, bool SWAP>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, int m_tiles,
            int n_tiles, cudaStream_t stream) {
  using C = Cfg<BN, STAGES, EPI, SWAP>;
  auto kern = gemm_bf16_kernel<BN, STAGES, EPI, SWAP>;
  static bool configured = false;  // per instantiation; attribute is per-function
  if (!configured) {
    check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    C::SMEM_BYTES),
               "cudaFuncSetAttribute(gemm smem)");
    configured = true;
  }
  dim3 grid(m_tiles, n_tiles, args.splits);
  kern<<<grid, kThreads, C::SMEM_BYTES, stream>>>(ta, tb, args);
  check_cuda(cudaGetLastError(), "gemm_bf16_kernel launch");
}

template <int EPI>
void dispatch_swap(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                   int mt, int nt, cudaStream_t st);
template <int EPI>
void dispatch_normal(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                     int mt, int nt, cudaStream_t st);

inline int smem_stage_bytes(int bn, bool swiglu_swap) {
  return (swiglu_swap ? 2 : 1) * BM * BK * 2 + bn * BK * 2;
}

}  // namespace gemm_detail
}  // namespace sil
