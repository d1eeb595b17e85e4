// Block-scaled fp8 GEMM on tcgen05 (kind::f8f6f4, e4m3 x e4m3 -> fp32 in TMEM).
//
//   y[T, Nout] = epilogue( sum_kb  sx[t, kb] * sw[n/128, kb] * (xq[t, kb] . wq[n, kb]^T) )
//
// The DeepSeek-V3 / Kimi-K2 format: e4m3 weights with one fp32 scale per
// 128x128 block, activations quantised to e4m3 with one fp32 scale per 1x128
// block (quant_fp8_1x128 below).  The scales are arbitrary fp32 values, so
// each 128-wide K block gets its own MMA product in a TMEM buffer and the
// epilogue warps promote it into fp32 registers with both scales
// (double-buffered TMEM: the MMA of block kb+1 overlaps the promotion of kb).
//
// Operand orders as in the bf16 kernel: swapped (decode, <= 64 tokens: A =
// weights, M = features) and normal (prefill: A = activations).  Work units
// are (tile, K-split) pairs over a persistent grid; a split tile's partials
// are summed in split order by its last contributor (deterministic).  A
// grouped variant serves MoE experts (per-group row offsets from the router).
// Epilogues: bf16, residual add, SwiGLU, fp32.
//
// Oracle: csrc/native/swiglu_oracle.cpp (fp8_block_gemm); format semantics of
// the reference's fp8 block dequantisation, si/backends/colibri/sparse_moe.py:146-218.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "sil/ep.h"
#include "sil/host.h"
#include "sil/ptx.cuh"

namespace sil {
namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // fp8 elements per K block (= one 128-byte swizzled row)
constexpr int kThreads = 192;
constexpr int kMaxGroups = 1024;

// kScatter (grouped, swapped order only): expert-parallel combine -- each output row is
// one (token, slot) assignment; the value times its routing weight goes straight into
// the token owner's combine slot over peer memory (layout in sil/ep.h).
enum Epi : int { kBf16 = 0, kResAdd = 1, kSwiGLU = 2, kF32 = 3, kScatter = 4 };

struct Fp8Args {
  int M, N, KB;
  int m_tiles, n_tiles, splits, grid, inter;
  const float* sA;  // swapped: weight scales [rows/128, KB]; normal: activation scales [T, KB]
  const float* sB;  // swapped: activation scales [T, KB]; normal: weight scales [rows/128, KB]
  void* out;
  long long ldo;
  const __nv_bfloat16* res;
  long long ldr;
  float* ws;
  int* counters;
  int* status;
  const int* grp_offsets;
  int num_groups;
  long long w_group_rows;
  EpLayout ep;           // kScatter only
  const int* sc_rows;    // kScatter: sorted position -> assignment (src * T + t) * k + j
};

template <int BN, int STAGES, bool SWAP, int EPI>
struct Cfg8 {
  static constexpr bool kIsSwiGLU = EPI == static_cast<int>(Epi::kSwiGLU);
  static constexpr int NUM_A = (kIsSwiGLU && SWAP) ? 2 : 1;
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = NUM_A * A_BYTES + B_BYTES;
  static constexpr int ACC_COLS = NUM_A * BN;
  static constexpr int OUT_COLS = (kIsSwiGLU && !SWAP) ? BN / 2 : BN;
  static constexpr int TMEM_COLS = 2 * ACC_COLS <= 32 ? 32 : 2 * ACC_COLS <= 64 ? 64
                                   : 2 * ACC_COLS <= 128 ? 128 : 2 * ACC_COLS <= 256 ? 256 : 512;
  static constexpr int CW = ACC_COLS >= 32 && BN >= 32 ? 32 : 16;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256 + (kMaxGroups + 8) * 4;
  static_assert(ACC_COLS <= 128, "fp8 promotion keeps the tile in registers");
};

template <int CW>
__device__ __forceinline__ void tld(uint32_t taddr, uint32_t (&r)[CW]) {
  if constexpr (CW == 32) {
    tmem_ld32_sync(taddr, r);
  } else {
    tmem_ld16(taddr, r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < CW; ++j) asm volatile("" : "+r"(r[j]));
  }
}

struct Unit {
  int tile, split, kb0, kb1;
};

struct Ctx8 {
  int mt, nt, a_base, b_base, Mv, Nv, roff;
};

template <bool GROUPED, bool SWAP>
__device__ __forceinline__ Ctx8 ctx8(const Fp8Args& a, int tile, const int* s_pref) {
  Ctx8 c;
  if constexpr (!GROUPED) {
    c.mt = tile % a.m_tiles;
    c.nt = tile / a.m_tiles;
    c.a_base = c.b_base = c.roff = 0;
    c.Mv = a.M;
    c.Nv = a.N;
  } else {
    int lo = 0, hi = a.num_groups;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_pref[mid] <= tile) lo = mid; else hi = mid;
    }
    const int g = lo, lt = tile - s_pref[g];
    const int off0 = a.grp_offsets[g], cnt = a.grp_offsets[g + 1] - off0;
    c.roff = off0;
    if constexpr (SWAP) {
      c.mt = lt % a.m_tiles;
      c.nt = lt / a.m_tiles;
      c.a_base = static_cast<int>(g * a.w_group_rows);
      c.b_base = off0;
      c.Mv = a.M;
      c.Nv = cnt;
    } else {
      const int mtg = (cnt + BM - 1) / BM;
      c.mt = lt % mtg;
      c.nt = lt / mtg;
      c.a_base = off0;
      c.b_base = static_cast<int>(g * a.w_group_rows);
      c.Mv = cnt;
      c.Nv = a.N;
    }
  }
  return c;
}

template <int BN, int STAGES, bool SWAP, int EPI, bool GROUPED>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB, const Fp8Args args) {
  using C = Cfg8<BN, STAGES, SWAP, EPI>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2] per K-block product ready
  uint64_t* tempty = tfull + 2;      // [2] product consumed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);
  int* s_pref = flags + 4;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    flags[0] = load_status(args.status) != 0;
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
  pdl_wait();  // scales, activations and group offsets come from earlier kernels
  uint32_t ep_epoch = 0;
  if constexpr (EPI == kScatter)
    ep_epoch = *reinterpret_cast<volatile uint32_t*>(args.ep.peers[args.ep.rank]) + 1u;
  int tiles = args.m_tiles * args.n_tiles;
  if constexpr (GROUPED) {
    for (int g = threadIdx.x; g < args.num_groups; g += kThreads) {
      const int cnt = args.grp_offsets[g + 1] - args.grp_offsets[g];
      s_pref[g + 1] = SWAP ? args.m_tiles * ((cnt + BN - 1) / BN) : ((cnt + BM - 1) / BM) * args.n_tiles;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      s_pref[0] = 0;
      for (int g = 0; g < args.num_groups; ++g) s_pref[g + 1] += s_pref[g];
    }
    __syncthreads();
    tiles = s_pref[args.num_groups];
  }
  const int units = tiles * args.splits;
  constexpr int BROWS = (C::kIsSwiGLU && !SWAP) ? BN / 2 : BN;

  auto unit_of = [&](int u) {
    Unit x;
    x.tile = u / args.splits;
    x.split = u % args.splits;
    const int per = args.KB / args.splits, rem = args.KB % args.splits;
    x.kb0 = x.split * per + min(x.split, rem);
    x.kb1 = x.kb0 + per + (x.split < rem ? 1 : 0);
    return x;
  };

  if (!skip) {
    if (warp == 0) {
      if (lane == 0) {
        const uint64_t pol_w = l2_policy_evict_first();
        const uint64_t pol_x = l2_policy_evict_last();
        int i = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < units; u += args.grid) {
          const Unit un = unit_of(u);
          const Ctx8 c = ctx8<GROUPED, SWAP>(args, un.tile, s_pref);
          for (int kb = un.kb0; kb < un.kb1; ++kb, ++i) {
            const int s = i % STAGES;
            if (!mbar_wait(&empty[s], ((i / STAGES) & 1) ^ 1, args.status, kStatusTimeoutEmpty)) {
              ok = false;
              break;
            }
            uint8_t* sa = smem + s * C::STAGE_BYTES;
            uint8_t* sb = sa + C::NUM_A * C::A_BYTES;
            mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
            const int kx = kb * BK;
            if constexpr (SWAP) {
              tma_load_2d_hint(sa, &tmA, &full[s], kx, c.a_base + c.mt * BM, pol_w);
              if constexpr (C::NUM_A == 2)
                tma_load_2d_hint(sa + C::A_BYTES, &tmA, &full[s], kx, c.a_base + c.mt * BM + args.inter, pol_w);
              tma_load_2d_hint(sb, &tmB, &full[s], kx, c.b_base + c.nt * BN, pol_x);
            } else {
              tma_load_2d_hint(sa, &tmA, &full[s], kx, c.a_base + c.mt * BM, pol_x);
              tma_load_2d_hint(sb, &tmB, &full[s], kx, c.b_base + c.nt * BROWS, pol_w);
              if constexpr (C::kIsSwiGLU)
                tma_load_2d_hint(sb + BROWS * BK, &tmB, &full[s], kx,
                                 c.b_base + c.nt * BROWS + args.inter, pol_w);
            }
          }
        }
      }
    } else if (warp == 1) {
      if (lane == 0) {
        constexpr uint32_t idesc = umma_idesc_e4m3(BM, BN);
        int i = 0, j = 0;  // j counts K blocks through the TMEM double buffer
        bool ok = true;
        for (int u = blockIdx.x; ok && u < units; u += args.grid) {
          const Unit un = unit_of(u);
          for (int kb = un.kb0; kb < un.kb1; ++kb, ++i, ++j) {
            const int s = i % STAGES, b = j & 1;
            if (!mbar_wait(&tempty[b], ((j >> 1) & 1) ^ 1, args.status, kStatusTimeoutAccum) ||
                !mbar_wait(&full[s], (i / STAGES) & 1, args.status, kStatusTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(smem + s * C::STAGE_BYTES);
            const uint32_t b_addr = a_addr + C::NUM_A * C::A_BYTES;
            const uint32_t acc = tmem_base + b * C::ACC_COLS;
#pragma unroll
            for (int k = 0; k < BK / 32; ++k) {
              const uint64_t bd = umma_desc_sw128(b_addr + k * 32);
              umma_f8(acc, umma_desc_sw128(a_addr + k * 32), bd, idesc, k > 0);
              if constexpr (C::NUM_A == 2)
                umma_f8(acc + BN, umma_desc_sw128(a_addr + C::A_BYTES + k * 32), bd, idesc, k > 0);
            }
            umma_commit(&empty[s]);
            umma_commit(&tfull[b]);
          }
        }
      }
    } else {
      constexpr int CW = C::CW;
      const int q = warp & 3;
      const int row = q * 32 + lane;
      const uint32_t tq = static_cast<uint32_t>(q * 32) << 16;
      int j = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += args.grid) {
        const Unit un = unit_of(u);
        const Ctx8 c = ctx8<GROUPED, SWAP>(args, un.tile, s_pref);
        float acc[C::ACC_COLS];
#pragma unroll
        for (int t = 0; t < C::ACC_COLS; ++t) acc[t] = 0.f;
        const int m_loc = c.mt * BM + row;  // accumulator row inside the group's A rows
        for (int kb = un.kb0; kb < un.kb1; ++kb, ++j) {
          const int b = j & 1;
          if (!mbar_wait(&tfull[b], (j >> 1) & 1, args.status, kStatusTimeoutAccum)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // Row scale (per accumulator row) and column scales (per column).
          float srow, srow_up = 0.f;
          if constexpr (SWAP) {
            srow = args.sA[(long long)((c.a_base + c.mt * BM) / BM) * args.KB + kb];
            if constexpr (C::NUM_A == 2)
              srow_up = args.sA[(long long)((c.a_base + c.mt * BM + args.inter) / BM) * args.KB + kb];
          } else {
            const int r = c.a_base + min(m_loc, max(c.Mv - 1, 0));
            srow = args.sA[(long long)r * args.KB + kb];
          }
          // Swapped order: the columns are tokens.  Lane l loads token l's activation scale
          // (and token l + 32 when BN = 64) once per K block; the others get it by shuffle.
          float stok0 = 0.f, stok1 = 0.f;
          if constexpr (SWAP) {
            const int hi = max(c.Nv - 1, 0);
            stok0 = args.sB[(long long)(c.b_base + min(c.nt * BN + (lane & (BN - 1) & 31), hi)) * args.KB + kb];
            if constexpr (BN > 32)
              stok1 = args.sB[(long long)(c.b_base + min(c.nt * BN + 32 + lane, hi)) * args.KB + kb];
          }
#pragma unroll
          for (int c0 = 0; c0 < C::ACC_COLS; c0 += CW) {
            uint32_t rv[CW];
            tld<CW>(tmem_base + b * C::ACC_COLS + tq + c0, rv);
#pragma unroll
            for (int t = 0; t < CW; ++t) {
              const int col = c0 + t;
              float scol;
              if constexpr (SWAP) {
                const int j = col % BN;
                const float st = (BN > 32 && j >= 32) ? __shfl_sync(0xffffffffu, stok1, j - 32)
                                                      : __shfl_sync(0xffffffffu, stok0, j & 31);
                scol = st * ((C::NUM_A == 2 && col >= BN) ? srow_up : srow);
              } else {
                int wrow;
                if constexpr (C::kIsSwiGLU)
                  wrow = col < BN / 2 ? c.b_base + c.nt * BROWS + col
                                      : c.b_base + c.nt * BROWS + args.inter + (col - BN / 2);
                else
                  wrow = c.b_base + c.nt * BN + col;
                scol = args.sB[(long long)(wrow / BM) * args.KB + kb] * srow;
              }
              acc[col] += __uint_as_float(rv[t]) * scol;
            }
          }
          tc_fence_before();
          mbar_arrive(&tempty[b]);
        }
        if (!ok) break;
        // Split-K fix-up: partials in split order by the last contributor.
        bool final_ = true;
        if (args.splits > 1) {
          float* mine = args.ws + ((long long)un.tile * args.splits + un.split) * C::ACC_COLS * BM;
#pragma unroll
          for (int t = 0; t < C::ACC_COLS; ++t) __stcg(&mine[t * BM + row], acc[t]);
          __threadfence();
          named_bar_sync(1, 128);
          if (threadIdx.x == 64) {
            const int old = atomicAdd(&args.counters[un.tile], 1);
            flags[1] = old == args.splits - 1;
          }
          named_bar_sync(1, 128);
          final_ = flags[1] != 0;
          named_bar_sync(1, 128);
          if (final_) {
            __threadfence();
            const float* base = args.ws + (long long)un.tile * args.splits * C::ACC_COLS * BM;
#pragma unroll
            for (int t = 0; t < C::ACC_COLS; ++t) acc[t] = 0.f;
            for (int sp = 0; sp < args.splits; ++sp) {
#pragma unroll
              for (int t = 0; t < C::ACC_COLS; ++t)
                acc[t] += __ldcg(&base[((long long)sp * C::ACC_COLS + t) * BM + row]);
            }
            if (threadIdx.x == 64) args.counters[un.tile] = 0;
          }
        }
        if (!final_) continue;
        // Epilogue store.
        if (m_loc < c.Mv) {
#pragma unroll
          for (int col = 0; col < C::OUT_COLS; ++col) {
            float v = acc[col];
            if constexpr (C::kIsSwiGLU) {
              const float up = SWAP ? acc[col + BN] : acc[col + BN / 2];
              v = silu_f(v) * up;
            }
            int orow, ocol;
            if constexpr (SWAP) {
              const int n = c.nt * BN + col;
              if (n >= c.Nv) continue;
              orow = c.roff + n;
              ocol = m_loc;
            } else {
              const int n = c.nt * C::OUT_COLS + col;
              if (n >= c.Nv) continue;
              orow = c.roff + m_loc;
              ocol = n;
            }
            if constexpr (EPI == kScatter) {
              const EpLayout& L = args.ep;
              const int par = ep_epoch & 1;
              const int asg = args.sc_rows[orow];
              const int tok = asg / L.k, slot = asg % L.k;
              const int src = tok / L.T, t = tok % L.T;
              const float wgt = reinterpret_cast<const float*>(L.peers[L.rank] + L.wts_off)
                  [(((long long)par * L.world + src) * L.T + t) * L.k + slot];
              reinterpret_cast<__nv_bfloat16*>(L.peers[src] + L.slots_off)
                  [(((long long)par * L.T + t) * L.k + slot) * L.H + ocol] = __float2bfloat16_rn(v * wgt);
            } else if constexpr (EPI == kF32) {
              reinterpret_cast<float*>(args.out)[(long long)orow * args.ldo + ocol] = v;
            } else {
              if constexpr (EPI == kResAdd) v += __bfloat162float(args.res[(long long)orow * args.ldr + ocol]);
              reinterpret_cast<__nv_bfloat16*>(args.out)[(long long)orow * args.ldo + ocol] =
                  __float2bfloat16_rn(v);
            }
          }
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
  if constexpr (EPI == kScatter) {
    // The grid's last CTA tells every rank that this rank's expert outputs have landed.
    const EpLayout& L = args.ep;
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();  // cumulative over this CTA's scatter stores (ordered by the barrier)
      uint32_t* ctr = reinterpret_cast<uint32_t*>(L.peers[L.rank]) + kEpCtrGemm;
      if (atomicAdd(ctr, 1u) == gridDim.x - 1) {
        *reinterpret_cast<volatile uint32_t*>(ctr) = 0u;
        for (int p = 0; p < L.world; ++p) {
          uint32_t* f = reinterpret_cast<uint32_t*>(L.peers[p] + L.cflag_off) + (ep_epoch & 1) * 8 + L.rank;
          asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(ep_epoch) : "memory");
        }
      }
    }
  }
}

template <int BN, int STAGES, bool SWAP, int EPI, bool GROUPED>
void launch8(const CUtensorMap& ta, const CUtensorMap& tb, const Fp8Args& a, cudaStream_t st) {
  using C = Cfg8<BN, STAGES, SWAP, EPI>;
  auto kern = gemm_fp8_kernel<BN, STAGES, SWAP, EPI, GROUPED>;
  set_smem_limit(reinterpret_cast<const void*>(kern), C::SMEM_BYTES, "cudaFuncSetAttribute(fp8 gemm)");
  launch_pdl(kern, dim3(a.grid), dim3(kThreads), C::SMEM_BYTES, st, "gemm_fp8 launch", ta, tb, a);
}

template <int EPI, bool GROUPED>
void dispatch8(bool swap, int bn, const CUtensorMap& ta, const CUtensorMap& tb, const Fp8Args& a,
               cudaStream_t st) {
  if (swap) {
    if constexpr (EPI == kSwiGLU) {
      if (bn == 16) launch8<16, 5, true, EPI, GROUPED>(ta, tb, a, st);
      else if (bn == 32) launch8<32, 5, true, EPI, GROUPED>(ta, tb, a, st);
      else launch8<64, 4, true, EPI, GROUPED>(ta, tb, a, st);
    } else {
      if (bn == 16) launch8<16, 10, true, EPI, GROUPED>(ta, tb, a, st);
      else if (bn == 32) launch8<32, 9, true, EPI, GROUPED>(ta, tb, a, st);
      else launch8<64, 8, true, EPI, GROUPED>(ta, tb, a, st);
    }
  } else {
    launch8<128, 6, false, EPI, GROUPED>(ta, tb, a, st);
  }
}

template <bool GROUPED>
void run_fp8(const at::Tensor& xq, const at::Tensor& xs, const at::Tensor& wq, const at::Tensor& wsc,
             at::Tensor& out, const c10::optional<at::Tensor>& res, int64_t epi,
             const c10::optional<at::Tensor>& offsets, int64_t num_groups, int64_t rows_hint,
             const at::Tensor& ws, const at::Tensor& counters, const at::Tensor& status,
             const EpLayout* ep = nullptr, const int* sc_rows = nullptr) {
  TORCH_CHECK(xq.scalar_type() == at::kByte || xq.scalar_type() == at::kFloat8_e4m3fn,
              "fp8 gemm: e4m3 activations (uint8 view)");
  TORCH_CHECK(wq.scalar_type() == at::kByte || wq.scalar_type() == at::kFloat8_e4m3fn,
              "fp8 gemm: e4m3 weights (uint8 view)");
  TORCH_CHECK(xs.scalar_type() == at::kFloat && wsc.scalar_type() == at::kFloat, "fp8 gemm: fp32 scales");
  const int T = xq.size(0), K = xq.size(1);
  TORCH_CHECK(K % BK == 0 && wq.size(1) == K, "fp8 gemm: K must be a multiple of 128");
  TORCH_CHECK(xs.size(0) == T && xs.size(1) == K / BK && xs.is_contiguous(), "fp8 gemm: activation scales");
  const bool swiglu = epi == kSwiGLU;
  const long long groups = GROUPED ? num_groups : 1;
  const long long Wr = wq.size(0) / groups;
  const int inter = swiglu ? static_cast<int>(Wr / 2) : 0;
  const int Nout = swiglu ? inter : static_cast<int>(Wr);
  TORCH_CHECK(Wr % BM == 0 && (!swiglu || inter % BM == 0), "fp8 gemm: weight rows per group % 128");
  TORCH_CHECK(wsc.size(0) == wq.size(0) / BM && wsc.size(1) == K / BK && wsc.is_contiguous(),
              "fp8 gemm: weight scales [rows/128, K/128]");
  TORCH_CHECK(epi == kScatter || (out.size(0) == T && out.size(1) == Nout), "fp8 gemm: output shape");
  TORCH_CHECK(epi != kScatter || (GROUPED && ep != nullptr && ep->H == Nout),
              "fp8 gemm: scatter epilogue needs the grouped EP form");
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(xq.device());
  Fp8Args a{};
  a.KB = K / BK;
  a.inter = inter;
  a.out = out.data_ptr();
  a.ldo = out.stride(0);
  if (res.has_value()) {
    a.res = reinterpret_cast<const __nv_bfloat16*>(res->data_ptr());
    a.ldr = res->stride(0);
  }
  a.ws = ws.data_ptr<float>();
  a.counters = counters.data_ptr<int>();
  a.status = status.data_ptr<int>();
  if (ep != nullptr) {
    a.ep = *ep;
    a.sc_rows = sc_rows;
  }
  const int sms = device_sm_count();
  const bool swap = GROUPED ? rows_hint <= 64 : T <= 64;
  int bn;
  CUtensorMap ta, tb;
  if (swap) {
    const int hint = GROUPED ? (int)rows_hint : T;
    bn = hint <= 16 ? 16 : hint <= 32 ? 32 : 64;
    a.M = Nout;
    a.N = T;
    a.m_tiles = (Nout + BM - 1) / BM;
    a.n_tiles = GROUPED ? 1 : (T + bn - 1) / bn;
    a.sA = wsc.data_ptr<float>();
    a.sB = xs.data_ptr<float>();
    ta = make_tmap_2d(wq.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, wq.size(0), K, K, BM, BK,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    tb = make_tmap_2d(xq.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, T, K, K, bn, BK,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    bn = 128;
    const int out_cols = swiglu ? bn / 2 : bn;
    a.M = T;
    a.N = Nout;
    a.m_tiles = (T + BM - 1) / BM;
    a.n_tiles = (Nout + out_cols - 1) / out_cols;
    a.sA = xs.data_ptr<float>();
    a.sB = wsc.data_ptr<float>();
    ta = make_tmap_2d(xq.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, T, K, K, BM, BK,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    tb = make_tmap_2d(wq.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, wq.size(0), K, K,
                      swiglu ? bn / 2 : bn, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if constexpr (GROUPED) {
    TORCH_CHECK(offsets.has_value() && num_groups <= kMaxGroups, "fp8 grouped: offsets");
    a.grp_offsets = offsets->data_ptr<int>();
    a.num_groups = static_cast<int>(num_groups);
    a.w_group_rows = Wr;
    a.splits = 1;
    a.grid = sms;
  } else {
    const int tiles = a.m_tiles * a.n_tiles;
    int splits = 1;
    if (tiles < sms) splits = std::min(std::max(1, sms / tiles), std::max(1, a.KB / 2));
    const long long acc_cols = (swap && swiglu ? 2 : 1) * bn;
    while (splits > 1 && (long long)tiles * splits * acc_cols * BM > ws.numel()) --splits;
    TORCH_CHECK(splits == 1 || tiles <= counters.numel(), "fp8 gemm: counters");
    a.splits = splits;
    a.grid = std::min(sms, tiles * splits);
  }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  switch (epi) {
    case kBf16: dispatch8<kBf16, GROUPED>(swap, bn, ta, tb, a, st); break;
    case kResAdd: dispatch8<kResAdd, GROUPED>(swap, bn, ta, tb, a, st); break;
    case kSwiGLU: dispatch8<kSwiGLU, GROUPED>(swap, bn, ta, tb, a, st); break;
    case kF32: dispatch8<kF32, GROUPED>(swap, bn, ta, tb, a, st); break;
    case kScatter:
      if constexpr (GROUPED) {
        TORCH_CHECK(swap, "fp8 gemm: the scatter epilogue runs in the swapped (decode) order");
        if (bn == 16) launch8<16, 10, true, kScatter, true>(ta, tb, a, st);
        else if (bn == 32) launch8<32, 9, true, kScatter, true>(ta, tb, a, st);
        else launch8<64, 8, true, kScatter, true>(ta, tb, a, st);
      }
      break;
    default: TORCH_CHECK(false, "fp8 gemm: unknown epilogue");
  }
}

// One warp per (row, 128-column block): absmax, scale = absmax / 448, e4m3 with saturation.
__global__ void quant_fp8_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, int K,
                                 uint8_t* __restrict__ q, float* __restrict__ s, int rows) {
  pdl_trigger();
  pdl_wait();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int KB = K / 128;
  if (w >= rows * KB) return;
  const int r = w / KB, kb = w % KB;
  const __nv_bfloat16* src = x + (long long)r * ldx + kb * 128 + lane * 4;
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  float v[4] = {bf16_lo(raw.x), bf16_hi(raw.x), bf16_lo(raw.y), bf16_hi(raw.y)};
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float sc = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = 1.f / sc;
  const __nv_fp8x2_storage_t p0 = __nv_cvt_float2_to_fp8x2(make_float2(v[0] * inv, v[1] * inv),
                                                           __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t p1 = __nv_cvt_float2_to_fp8x2(make_float2(v[2] * inv, v[3] * inv),
                                                           __NV_SATFINITE, __NV_E4M3);
  uint32_t packed = static_cast<uint32_t>(p0) | (static_cast<uint32_t>(p1) << 16);
  *reinterpret_cast<uint32_t*>(q + (long long)r * K + kb * 128 + lane * 4) = packed;
  if (lane == 0) s[(long long)r * KB + kb] = sc;
}

}  // namespace

void gemm_fp8(const at::Tensor& xq, const at::Tensor& xs, const at::Tensor& wq, const at::Tensor& wsc,
              at::Tensor& out, const c10::optional<at::Tensor>& res, int64_t epi,
              const at::Tensor& ws, const at::Tensor& counters, const at::Tensor& status) {
  run_fp8<false>(xq, xs, wq, wsc, out, res, epi, c10::nullopt, 1, 0, ws, counters, status);
}

void gemm_fp8_grouped(const at::Tensor& xq, const at::Tensor& xs, const at::Tensor& wq,
                      const at::Tensor& wsc, at::Tensor& out, const at::Tensor& offsets,
                      int64_t num_groups, bool swiglu, int64_t rows_hint, const at::Tensor& ws,
                      const at::Tensor& counters, const at::Tensor& status) {
  run_fp8<true>(xq, xs, wq, wsc, out, c10::nullopt, swiglu ? kSwiGLU : kBf16, offsets, num_groups,
                rows_hint, ws, counters, status);
}

void quant_fp8_1x128(const at::Tensor& x, at::Tensor& q, at::Tensor& s) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1, "quant: bf16 rows");
  const int rows = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 128 == 0, "quant: K % 128");
  if (rows == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  const long long warps = (long long)rows * (K / 128);
  launch_pdl(quant_fp8_kernel, dim3((warps * 32 + 255) / 256), dim3(256), 0,
             at::cuda::getCurrentCUDAStream(), "quant_fp8 launch",
             reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (long long)x.stride(0), K,
             reinterpret_cast<uint8_t*>(q.data_ptr()), s.data_ptr<float>(), rows);
}

EpLayout ep_make_layout(const std::vector<int64_t>& peers, int64_t rank, int64_t T, int64_t k,
                        int64_t H, int64_t e0, int64_t el, const std::vector<int64_t>& offs,
                        const at::Tensor& status);

// Down projection of the local experts with the weighted combine fused into the epilogue:
// results go to the token owners' combine slots over peer memory (see sil/ep.h).
void gemm_fp8_grouped_scatter(const at::Tensor& xq, const at::Tensor& xs, const at::Tensor& wq,
                              const at::Tensor& wsc, const at::Tensor& offsets, int64_t num_groups,
                              int64_t rows_hint, const at::Tensor& sorted_rows,
                              const std::vector<int64_t>& peers, int64_t rank, int64_t T, int64_t k,
                              int64_t e0, const std::vector<int64_t>& offs, const at::Tensor& ws,
                              const at::Tensor& counters, const at::Tensor& status) {
  const int64_t H = wq.size(0) / num_groups;
  EpLayout L = ep_make_layout(peers, rank, T, k, H, e0, num_groups, offs, status);
  TORCH_CHECK(sorted_rows.scalar_type() == at::kInt && sorted_rows.numel() >= xq.size(0),
              "fp8 scatter: sorted rows");
  at::Tensor dummy = xq;
  run_fp8<true>(xq, xs, wq, wsc, dummy, c10::nullopt, kScatter, offsets, num_groups,
                std::min<int64_t>(rows_hint, 64), ws, counters, status, &L, sorted_rows.data_ptr<int>());
}

}  // namespace sil
