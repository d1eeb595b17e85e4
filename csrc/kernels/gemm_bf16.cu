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
namespace {

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

// Store 32 consecutive accumulator columns [c0, c0+32) of accumulator row `row`.
template <int EPI, bool SWAP>
__device__ __forceinline__ void store_chunk(const GemmArgs& a, int m_glob, int n0,
                                            const float (&v)[32], const float (&u)[32]) {
  if (m_glob >= a.M) return;
  if constexpr (SWAP) {
    // Accumulator row = output feature m_glob, column = token n.
#pragma unroll
    for (int j = 0; j < 32; ++j) {
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
      if (n0 + 32 <= a.N && (a.ldo & 3) == 0) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(o + n0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      } else {
        for (int j = 0; j < 32; ++j)
          if (n0 + j < a.N) o[n0 + j] = v[j];
      }
    } else {
      float r[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        r[j] = v[j];
        if constexpr (EPI == kEpiSwiGLU) r[j] = silu_f(v[j]) * u[j];
      }
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) + (long long)m_glob * a.ldo;
      const bool vec = (n0 + 32 <= a.N) && ((a.ldo & 7) == 0) &&
                       (EPI != kEpiResAdd || (a.ldr & 7) == 0);
      if (vec) {
        if constexpr (EPI == kEpiResAdd) {
          const __nv_bfloat16* rr = a.res + (long long)m_glob * a.ldr + n0;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 q = *reinterpret_cast<const uint4*>(rr + j);
            r[j + 0] += bf16_lo(q.x); r[j + 1] += bf16_hi(q.x);
            r[j + 2] += bf16_lo(q.y); r[j + 3] += bf16_hi(q.y);
            r[j + 4] += bf16_lo(q.z); r[j + 5] += bf16_hi(q.z);
            r[j + 6] += bf16_lo(q.w); r[j + 7] += bf16_hi(q.w);
          }
        }
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 q;
          q.x = pack_bf16x2(r[j + 0], r[j + 1]);
          q.y = pack_bf16x2(r[j + 2], r[j + 3]);
          q.z = pack_bf16x2(r[j + 4], r[j + 5]);
          q.w = pack_bf16x2(r[j + 6], r[j + 7]);
          *reinterpret_cast<uint4*>(o + n0 + j) = q;
        }
      } else {
        for (int j = 0; j < 32; ++j) {
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
      if (ok && args.splits > 1) {
        float* mine = args.ws + ((long long)tile_id * args.splits + split) * C::ACC_COLS * BM;
#pragma unroll 1
        for (int c0 = 0; c0 < C::ACC_COLS; c0 += 32) {
          uint32_t v[32];
          tmem_ld32_sync(taddr + c0, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) __stcg(&mine[(c0 + j) * BM + row], __uint_as_float(v[j]));
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
#pragma unroll 1
        for (int c0 = 0; c0 < C::OUT_COLS; c0 += 32) {
          float v[32], u[32];
          if (args.splits == 1) {
            uint32_t rv[32];
            tmem_ld32_sync(taddr + c0, rv);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(rv[j]);
            if constexpr (C::kSwiGLU) {
              const int uc = SWAP ? c0 + BN : c0 + BN / 2;
              tmem_ld32_sync(taddr + uc, rv);
#pragma unroll
              for (int j = 0; j < 32; ++j) u[j] = __uint_as_float(rv[j]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) { v[j] = 0.f; u[j] = 0.f; }
            const int uc = SWAP ? c0 + BN : c0 + BN / 2;
            for (int s = 0; s < args.splits; ++s) {
              const float* p = base + (long long)s * C::ACC_COLS * BM;
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += __ldcg(&p[(c0 + j) * BM + row]);
              if constexpr (C::kSwiGLU) {
#pragma unroll
                for (int j = 0; j < 32; ++j) u[j] += __ldcg(&p[(uc + j) * BM + row]);
              }
            }
          }
          const int n0 = n_tile * C::OUT_COLS + c0;
          store_chunk<EPI, SWAP>(args, m_glob, n0, v, u);
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
                   int mt, int nt, cudaStream_t st) {
  switch (bn) {
    case 16: launch<16, (EPI == kEpiSwiGLU ? 4 : 6), EPI, true>(ta, tb, a, mt, nt, st); break;
    case 32: launch<32, (EPI == kEpiSwiGLU ? 4 : 5), EPI, true>(ta, tb, a, mt, nt, st); break;
    case 64: launch<64, (EPI == kEpiSwiGLU ? 3 : 4), EPI, true>(ta, tb, a, mt, nt, st); break;
    default: launch<128, 3, EPI, true>(ta, tb, a, mt, nt, st); break;
  }
}

template <int EPI>
void dispatch_normal(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                     int mt, int nt, cudaStream_t st) {
  if (bn == 256) launch<256, 4, EPI, false>(ta, tb, a, mt, nt, st);
  else launch<128, 6, EPI, false>(ta, tb, a, mt, nt, st);
}

int smem_stage_bytes(int bn, bool swiglu_swap) { return (swiglu_swap ? 2 : 1) * BM * BK * 2 + bn * BK * 2; }

}  // namespace

// y = epilogue(x . W^T).  x: [T, K] bf16 (row pitch 16-byte aligned), W: [Nw, K] bf16,
// out: [T, Nout] (bf16, or fp32 for epi=3).  For SwiGLU W = [gate; up] with
// Nw = 2*inter and out = [T, inter].  `ws`/`counters`/`status` are the caller's
// split-K workspace (fp32), tile counters (int32, zero-initialised) and status word.
void gemm_bf16(const at::Tensor& x, const at::Tensor& w, at::Tensor& out,
               const c10::optional<at::Tensor>& res, int64_t epi, const at::Tensor& ws,
               const at::Tensor& counters, const at::Tensor& status, int64_t force_mode,
               int64_t force_splits) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "gemm_bf16: CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
              "gemm_bf16: bf16 operands required");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2, "gemm_bf16: 2-D tensors");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1,
              "gemm_bf16: innermost dim must be contiguous");
  const int T = x.size(0);
  const int K = x.size(1);
  TORCH_CHECK(w.size(1) == K, "gemm_bf16: K mismatch");
  TORCH_CHECK(K % 8 == 0, "gemm_bf16: K must be a multiple of 8");
  const bool swiglu = epi == kEpiSwiGLU;
  const int Nw = w.size(0);
  const int inter = swiglu ? Nw / 2 : 0;
  const int Nout = swiglu ? inter : Nw;
  TORCH_CHECK(!swiglu || (Nw % 2 == 0 && inter % 128 == 0),
              "gemm_bf16: SwiGLU needs [gate; up] with inter % 128 == 0");
  TORCH_CHECK(out.size(0) == T && out.size(1) == Nout, "gemm_bf16: bad output shape");
  if (epi == kEpiF32) {
    TORCH_CHECK(out.scalar_type() == at::kFloat, "gemm_bf16: fp32 output");
  } else {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16, "gemm_bf16: bf16 output");
  }
  const __nv_bfloat16* res_ptr = nullptr;
  long long ldr = 0;
  if (epi == kEpiResAdd) {
    TORCH_CHECK(res.has_value(), "gemm_bf16: residual required");
    TORCH_CHECK(res->scalar_type() == at::kBFloat16 && res->stride(1) == 1 &&
                    res->size(0) == T && res->size(1) == Nout,
                "gemm_bf16: bad residual");
    res_ptr = reinterpret_cast<const __nv_bfloat16*>(res->data_ptr());
    ldr = res->stride(0);
  }
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();

  const bool swap = force_mode == 1 ? true : force_mode == 2 ? false : (T <= 128);
  GemmArgs a;
  a.num_kb = (K + BK - 1) / BK;
  a.inter = inter;
  a.out = out.data_ptr();
  a.ldo = out.stride(0);
  a.res = res_ptr;
  a.ldr = ldr;
  a.ws = ws.data_ptr<float>();
  a.counters = counters.data_ptr<int>();
  a.status = status.data_ptr<int>();
  const int sms = device_sm_count();

  if (swap) {
    TORCH_CHECK(T <= 128, "gemm_bf16: swapped mode supports at most 128 tokens");
    const int bn = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : 128;
    a.M = swiglu ? inter : Nw;
    a.N = T;
    const int m_tiles = (a.M + BM - 1) / BM;
    const int n_tiles = 1;
    const int tiles = m_tiles * n_tiles;
    const int stage = smem_stage_bytes(bn, swiglu);
    const int ctas_per_sm = stage * 4 <= 110 * 1024 ? 2 : 1;
    int splits = 1;
    if (force_splits > 0) {
      splits = force_splits;
    } else if (tiles < sms * ctas_per_sm) {
      splits = (sms * ctas_per_sm + tiles - 1) / tiles;
      splits = std::min(splits, std::max(1, a.num_kb / 4));
    }
    const long long acc_cols = (swiglu ? 2 : 1) * bn;
    while (splits > 1 && (long long)tiles * splits * acc_cols * BM > ws.numel()) --splits;
    splits = std::max(1, std::min(splits, a.num_kb));
    TORCH_CHECK(splits == 1 || tiles <= counters.numel(), "gemm_bf16: counter array too small");
    a.splits = splits;
    CUtensorMap ta = make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Nw, K,
                                  w.stride(0), BM, BK, CU_TENSOR_MAP_SWIZZLE_128B);
    CUtensorMap tb = make_tmap_2d(x.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, K,
                                  x.stride(0), bn, BK, CU_TENSOR_MAP_SWIZZLE_128B);
    switch (epi) {
      case kEpiBf16: dispatch_swap<kEpiBf16>(bn, ta, tb, a, m_tiles, n_tiles, stream); break;
      case kEpiResAdd: dispatch_swap<kEpiResAdd>(bn, ta, tb, a, m_tiles, n_tiles, stream); break;
      case kEpiSwiGLU: dispatch_swap<kEpiSwiGLU>(bn, ta, tb, a, m_tiles, n_tiles, stream); break;
      case kEpiF32: dispatch_swap<kEpiF32>(bn, ta, tb, a, m_tiles, n_tiles, stream); break;
      default: TORCH_CHECK(false, "gemm_bf16: unknown epilogue");
    }
  } else {
    const int bn = (Nout >= 2048 || swiglu) ? 256 : 128;
    const int out_cols = swiglu ? bn / 2 : bn;
    a.M = T;
    a.N = Nout;
    const int m_tiles = (T + BM - 1) / BM;
    const int n_tiles = (Nout + out_cols - 1) / out_cols;
    int splits = force_splits > 0 ? (int)force_splits : 1;
    const long long acc_cols = bn;
    while (splits > 1 && (long long)m_tiles * n_tiles * splits * acc_cols * BM > ws.numel()) --splits;
    splits = std::max(1, std::min(splits, a.num_kb));
    TORCH_CHECK(splits == 1 || m_tiles * n_tiles <= counters.numel(),
                "gemm_bf16: counter array too small");
    a.splits = splits;
    CUtensorMap ta = make_tmap_2d(x.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, K,
                                  x.stride(0), BM, BK, CU_TENSOR_MAP_SWIZZLE_128B);
    CUtensorMap tb = make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Nw, K,
                                  w.stride(0), swiglu ? bn / 2 : bn, BK,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    switch (epi) {
      case kEpiBf16: dispatch_normal<kEpiBf16>(bn, ta, tb, a, m_tiles, n_tiles, stream); break;
      case kEpiResAdd: dispatch_normal<kEpiResAdd>(bn, ta, tb, a, m_tiles, n_tiles, stream); break;
      case kEpiSwiGLU: dispatch_normal<kEpiSwiGLU>(bn, ta, tb, a, m_tiles, n_tiles, stream); break;
      case kEpiF32: dispatch_normal<kEpiF32>(bn, ta, tb, a, m_tiles, n_tiles, stream); break;
      default: TORCH_CHECK(false, "gemm_bf16: unknown epilogue");
    }
  }
}

}  // namespace sil
