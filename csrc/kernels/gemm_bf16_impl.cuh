#pragma once
// Persistent stream-K bf16 GEMM on the 5th-generation tensor cores
// (tcgen05 + TMEM), TMA-fed through an mbarrier ring of shared-memory stages.
//
//   y[T, Nout] = epilogue( x[T, K] . W[Nw, K]^T )
//
// Operand orders:
//  * normal  (prefill, T > 128): A = x (M = tokens), B = W (N = features).
//  * swapped (decode, T <= 128):  A = W (M = features), B = x (N = tokens,
//    padded to 16/32/64/128).
//
// Work decomposition (stream-K): the (tile, k-block) units of the problem
// are cut into G equal contiguous ranges, one per persistent CTA (G <= SMs).
// A CTA streams its range without draining the pipeline between tiles; a
// tile covered by one CTA is stored directly, a tile shared by several CTAs
// has each contributor write an fp32 partial and the last contributor to
// arrive sums the partials in contributor order (deterministic) before the
// epilogue.  Two TMEM accumulators let the epilogue of one tile overlap the
// main loop of the next.
//
// Warp roles: warp 0 = TMA producer, warp 1 = MMA issuer (one thread) and
// TMEM owner, warps 2-5 = epilogue (warp w reads TMEM lanes 32*(w%4)...).
//
// Programmatic dependent launch: the producer starts streaming the weight
// operand before `griddepcontrol.wait`, so weight traffic overlaps the tail
// of the previous kernel; activations, residuals and the shared workspace
// are touched only after the wait.
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

enum EpiKind : int { kEpiBf16 = 0, kEpiResAdd = 1, kEpiSwiGLU = 2, kEpiF32 = 3, kEpiAllReduce = 4 };

constexpr int kMaxTP = 8;

struct GemmArgs {
  int M;          // valid rows of A (features when swapped, tokens otherwise)
  int N;          // valid output columns (tokens when swapped, features otherwise)
  int num_kb;     // 64-wide K blocks per tile
  int m_tiles;
  int n_tiles;
  int grid;       // G: persistent CTAs
  long long units;  // m_tiles * n_tiles * num_kb
  int stream_k;   // 1: contiguous (tile, k-block) ranges per CTA; 0: whole tiles, strided
  int group_m;    // tile mode: m-tiles per raster group (L2 reuse of the B operand)
  int inter;      // SwiGLU: row offset of the 'up' half inside the fused weight
  void* out;
  long long ldo;
  const __nv_bfloat16* res;
  long long ldr;
  float* ws;      // [G][2][ACC_COLS][128] partial tiles
  int* counters;  // per tile arrivals
  int* status;
  // kEpiAllReduce: one-shot all-reduce over NVLink peer memory fused into the epilogue.
  int tp_rank, tp_size;
  uint8_t* peers[kMaxTP];   // symmetric buffer base of every rank (own rank included)
  long long flags_off;      // byte offset of flags[2][kMaxTP][max_tiles] (uint32)
  long long slots_off;      // byte offset of slots[2][kMaxTP][max_tokens][max_hidden] (bf16)
  int max_tiles, max_tokens, max_hidden;
  // Grouped (MoE expert) GEMM: group g owns activation/output rows
  // [grp_offsets[g], grp_offsets[g+1]) and weight rows [g*w_group_rows, (g+1)*w_group_rows).
  const int* grp_offsets;
  int num_groups;
  long long w_group_rows;
  // Tile-aligned split-K in clusters (swapped order, non-grouped): grid = tiles * split_s,
  // launched as clusters of split_s CTAs; CTA i of cluster t owns the i-th K range of tile
  // t and the cluster reduces the tile through distributed shared memory.  0: stream-K
  // with last-arriver reduction through global memory.
  int split_s;
};

constexpr int kMaxGroups = 1024;
constexpr int kMaxClusterSplit = 8;  // portable cluster size

// Cluster-wide barrier (every thread of every CTA of the cluster): release this CTA's
// shared-memory writes, acquire the peers'.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_cluster(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t* ar_flag(const GemmArgs& a, int rank_buf, int par, int src,
                                             int tile) {
  return reinterpret_cast<uint32_t*>(a.peers[rank_buf] + a.flags_off) +
         ((long long)(par * kMaxTP + src) * a.max_tiles + tile);
}

__device__ __forceinline__ __nv_bfloat16* ar_slot(const GemmArgs& a, int rank_buf, int par,
                                                  int src) {
  return reinterpret_cast<__nv_bfloat16*>(a.peers[rank_buf] + a.slots_off) +
         (long long)(par * kMaxTP + src) * a.max_tokens * a.max_hidden;
}

// Push CW token columns of feature m (rank-local partial, rounded to bf16) into
// slot [par][tp_rank] of every rank's buffer.
template <int CW>
__device__ __forceinline__ void ar_push(const GemmArgs& a, int par, int m, int n0,
                                        const float (&v)[CW]) {
  if (m >= a.M) return;
  for (int p = 0; p < a.tp_size; ++p) {
    __nv_bfloat16* dst = ar_slot(a, p, par, a.tp_rank);
#pragma unroll
    for (int j = 0; j < CW; ++j) {
      const int n = n0 + j;
      if (n < a.N) dst[(long long)n * a.max_hidden + m] = __float2bfloat16_rn(v[j]);
    }
  }
}

// Publish a finished tile to every rank: the epilogue warps meet, then one thread issues a
// system-scope fence (cumulative over the warps' stores ordered before it by the barrier) and
// raises the tile's flag on every rank.
__device__ __forceinline__ void ar_publish(const GemmArgs& a, int par, uint32_t epoch, int tile) {
  named_bar_sync(1, 128);
  if (threadIdx.x == 64) {
    __threadfence_system();
    for (int p = 0; p < a.tp_size; ++p) st_release_sys(ar_flag(a, p, par, a.tp_rank, tile), epoch);
  }
}

template <int BN, int STAGES, int EPI, bool SWAP>
struct Cfg {
  static constexpr bool kSwiGLU = EPI == kEpiSwiGLU;
  static constexpr int NUM_A = (kSwiGLU && SWAP) ? 2 : 1;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = NUM_A * A_BYTES + B_BYTES;
  static constexpr int ACC_COLS = NUM_A * BN;
  static constexpr int OUT_COLS = (kSwiGLU && !SWAP) ? BN / 2 : BN;
  static constexpr int TMEM_COLS = 2 * ACC_COLS <= 32    ? 32
                                   : 2 * ACC_COLS <= 64  ? 64
                                   : 2 * ACC_COLS <= 128 ? 128
                                   : 2 * ACC_COLS <= 256 ? 256
                                                         : 512;
  static constexpr int CW = (OUT_COLS >= 32 && BN >= 32) ? 32 : 16;  // columns per TMEM load
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N constraint for M=128");
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert(2 * ACC_COLS <= 512, "two accumulators must fit in TMEM");
};

__device__ __forceinline__ long long unit_begin(int c, long long U, int G) {
  return (U * c) / G;
}

// Store CW consecutive accumulator columns [n0, n0+CW) of accumulator row `m_glob`.
template <int EPI, bool SWAP, int CW>
__device__ __forceinline__ void store_chunk(const GemmArgs& a, int m_glob, int n0,
                                            const float (&v)[CW], const float (&u)[CW],
                                            int Mv, int Nv, int roff) {
  if (m_glob >= Mv) return;
  if constexpr (SWAP) {
#pragma unroll
    for (int j = 0; j < CW; ++j) {
      const int n = n0 + j;
      if (n < Nv) {
        float r = v[j];
        if constexpr (EPI == kEpiSwiGLU) r = silu_f(v[j]) * u[j];
        if constexpr (EPI == kEpiF32) {
          reinterpret_cast<float*>(a.out)[(long long)(roff + n) * a.ldo + m_glob] = r;
        } else {
          if constexpr (EPI == kEpiResAdd) r += __bfloat162float(a.res[(long long)(roff + n) * a.ldr + m_glob]);
          reinterpret_cast<__nv_bfloat16*>(a.out)[(long long)(roff + n) * a.ldo + m_glob] =
              __float2bfloat16_rn(r);
        }
      }
    }
  } else {
    if constexpr (EPI == kEpiF32) {
      float* o = reinterpret_cast<float*>(a.out) + (long long)(roff + m_glob) * a.ldo;
      if (n0 + CW <= Nv && (a.ldo & 3) == 0) {
#pragma unroll
        for (int j = 0; j < CW; j += 4)
          *reinterpret_cast<float4*>(o + n0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      } else {
        for (int j = 0; j < CW; ++j)
          if (n0 + j < Nv) o[n0 + j] = v[j];
      }
    } else {
      float r[CW];
#pragma unroll
      for (int j = 0; j < CW; ++j) {
        r[j] = v[j];
        if constexpr (EPI == kEpiSwiGLU) r[j] = silu_f(v[j]) * u[j];
      }
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) + (long long)(roff + m_glob) * a.ldo;
      const bool vec = (n0 + CW <= Nv) && ((a.ldo & 7) == 0) &&
                       (EPI != kEpiResAdd || (a.ldr & 7) == 0);
      if (vec) {
        if constexpr (EPI == kEpiResAdd) {
          const __nv_bfloat16* rr = a.res + (long long)(roff + m_glob) * a.ldr + n0;
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
          if (n < Nv) {
            float x = r[j];
            if constexpr (EPI == kEpiResAdd) x += __bfloat162float(a.res[(long long)(roff + m_glob) * a.ldr + n]);
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
#pragma unroll
    for (int j = 0; j < CW; ++j) asm volatile("" : "+r"(r[j]));
  }
}

// Segment of a CTA's work that lies in one tile.
struct Segment {
  int tile;
  int kb0;
  int kb1;
  bool first;  // first segment of this CTA (stream-K partial slot 0)
};

// Walks the segments of one CTA.  Stream-K: the contiguous unit range
// [U*c/G, U*(c+1)/G).  Tile mode: whole tiles c, c+G, c+2G, ... in grouped
// raster order (group_m m-tiles sweep all n-tiles before the next group).
struct Sched {
  long long u, u_end, u_begin;
  int t, tiles;
  __device__ __forceinline__ Sched(const GemmArgs& a, int cta, int total_tiles = -1) {
    u_begin = (a.units * cta) / a.grid;
    u_end = (a.units * (cta + 1)) / a.grid;
    u = u_begin;
    t = cta;
    tiles = total_tiles >= 0 ? total_tiles : a.m_tiles * a.n_tiles;
  }
  __device__ __forceinline__ bool next(const GemmArgs& a, Segment& s) {
    if (a.stream_k) {
      if (u >= u_end) return false;
      s.tile = static_cast<int>(u / a.num_kb);
      s.kb0 = static_cast<int>(u % a.num_kb);
      const long long want = s.kb0 + (u_end - u);
      s.kb1 = want < a.num_kb ? static_cast<int>(want) : a.num_kb;
      s.first = u == u_begin;
      u += s.kb1 - s.kb0;
      return true;
    }
    if (t >= tiles) return false;
    s.tile = t;
    s.kb0 = 0;
    s.kb1 = a.num_kb;
    s.first = t < a.grid;
    t += a.grid;
    return true;
  }
};

// (m-tile, n-tile) of a tile index.  Stream-K: m fastest.  Tile mode: grouped raster.
__device__ __forceinline__ void tile_coords(const GemmArgs& a, int tile, int& mt, int& nt) {
  if (a.stream_k) {
    mt = tile % a.m_tiles;
    nt = tile / a.m_tiles;
    return;
  }
  const int per_group = a.group_m * a.n_tiles;
  const int g = tile / per_group;
  const int first_m = g * a.group_m;
  const int gm = min(a.m_tiles - first_m, a.group_m);
  const int in = tile % per_group;
  mt = first_m + in % gm;
  nt = in / gm;
}

// Where a tile's operands and outputs live.  Non-grouped: the whole problem.
// Grouped: the expert group that owns the tile (found in the per-CTA prefix of
// tiles per group, s_pref[0..num_groups]).
struct TileCtx {
  int mt, nt;
  int a_base, b_base;  // tensor-map row of the group's first A / B row
  int Mv, Nv;          // valid accumulator rows / columns
  int roff;            // output row offset of the group
};

template <bool GROUPED, bool SWAP>
__device__ __forceinline__ TileCtx make_ctx(const GemmArgs& a, int tile, const int* s_pref) {
  TileCtx c;
  if constexpr (!GROUPED) {
    tile_coords(a, tile, c.mt, c.nt);
    c.a_base = c.b_base = c.roff = 0;
    c.Mv = a.M;
    c.Nv = a.N;
  } else {
    int lo = 0, hi = a.num_groups;  // largest g with s_pref[g] <= tile
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_pref[mid] <= tile) lo = mid; else hi = mid;
    }
    const int g = lo;
    const int lt = tile - s_pref[g];
    const int off0 = a.grp_offsets[g];
    const int cnt = a.grp_offsets[g + 1] - off0;
    const long long wrow = (long long)g * a.w_group_rows;
    c.roff = off0;
    if constexpr (SWAP) {
      c.mt = lt % a.m_tiles;
      c.nt = lt / a.m_tiles;
      c.a_base = static_cast<int>(wrow);
      c.b_base = off0;
      c.Mv = a.M;
      c.Nv = cnt;
    } else {
      const int mtg = (cnt + BM - 1) / BM;
      c.mt = lt % mtg;
      c.nt = lt / mtg;
      c.a_base = off0;
      c.b_base = static_cast<int>(wrow);
      c.Mv = cnt;
      c.Nv = a.N;
    }
  }
  return c;
}


template <int BN, int STAGES, int EPI, bool SWAP, bool GROUPED>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
  using C = Cfg<BN, STAGES, EPI, SWAP>;
  static_assert(!GROUPED || EPI != kEpiAllReduce, "grouped all-reduce is not supported");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] skip, [1] last contributor
  int* s_pref = flags + 4;                              // grouped: tiles before group g

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int nkb = args.num_kb;
  const long long U = args.units;
  const int G = args.grid;

  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    flags[0] = load_status(args.status) != 0;
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
  int total_tiles = -1;
  if constexpr (GROUPED) {
    // Group sizes come from the previous kernel (routing): wait, then build the
    // per-group tile prefix in shared memory.
    pdl_wait();
    for (int g = threadIdx.x; g < args.num_groups; g += kThreads) {
      const int cnt = args.grp_offsets[g + 1] - args.grp_offsets[g];
      s_pref[g + 1] = SWAP ? args.m_tiles * ((cnt + BN - 1) / BN)
                           : ((cnt + BM - 1) / BM) * args.n_tiles;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      s_pref[0] = 0;
      for (int g = 0; g < args.num_groups; ++g) s_pref[g + 1] += s_pref[g];
    }
    __syncthreads();
    total_tiles = s_pref[args.num_groups];
  }

  if (!skip) {
    if (warp == 0) {
      if (lane == 0) {
        const uint64_t pol_w = l2_policy_evict_first();
        const uint64_t pol_x = l2_policy_evict_last();
        // Weight operand: A when swapped, B otherwise.  Issue the weight halves of the
        // first stages before waiting on the previous kernel (not for grouped GEMMs,
        // whose tile -> expert map comes from the previous kernel).
        constexpr int BROWS = (C::kSwiGLU && !SWAP) ? BN / 2 : BN;  // B rows per load
        int i = 0;
        bool waited = GROUPED;
        int npre = 0;
        if constexpr (!GROUPED) {
          Sched pre(args, cta);
          Segment sg;
          while (npre < STAGES && pre.next(args, sg)) {
            const TileCtx tc = make_ctx<GROUPED, SWAP>(args, sg.tile, s_pref);
            for (int kb = sg.kb0; kb < sg.kb1 && npre < STAGES; ++kb, ++npre) {
              uint8_t* sa = smem + npre * C::STAGE_BYTES;
              uint8_t* sb = sa + C::NUM_A * C::A_BYTES;
              mbar_arrive_expect_tx(&full[npre], C::STAGE_BYTES);
              const int kx = kb * BK;
              if constexpr (SWAP) {
                tma_load_2d_hint(sa, &tmA, &full[npre], kx, tc.a_base + tc.mt * BM, pol_w);
                if constexpr (C::NUM_A == 2)
                  tma_load_2d_hint(sa + C::A_BYTES, &tmA, &full[npre], kx,
                                   tc.a_base + tc.mt * BM + args.inter, pol_w);
              } else {
                tma_load_2d_hint(sb, &tmB, &full[npre], kx, tc.b_base + tc.nt * BROWS, pol_w);
                if constexpr (C::kSwiGLU)
                  tma_load_2d_hint(sb + BROWS * 128, &tmB, &full[npre], kx,
                                   tc.b_base + tc.nt * BROWS + args.inter, pol_w);
              }
            }
          }
        }
        Sched sch(args, cta, total_tiles);
        Segment sg;
        while (sch.next(args, sg)) {
          const TileCtx tc = make_ctx<GROUPED, SWAP>(args, sg.tile, s_pref);
          bool ok = true;
          for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++i) {
            const int s = i % STAGES;
            const uint32_t r = i / STAGES;
            uint8_t* sa = smem + s * C::STAGE_BYTES;
            uint8_t* sb = sa + C::NUM_A * C::A_BYTES;
            const int kx = kb * BK;
            if (i < npre) {
              // Weight half already in flight; activations need the previous kernel.
              if (!waited) {
                pdl_wait();
                waited = true;
              }
              if constexpr (SWAP) {
                tma_load_2d_hint(sb, &tmB, &full[s], kx, tc.b_base + tc.nt * BN, pol_x);
              } else {
                tma_load_2d_hint(sa, &tmA, &full[s], kx, tc.a_base + tc.mt * BM, pol_x);
              }
              continue;
            }
            if (!waited) {
              pdl_wait();
              waited = true;
            }
            if (!mbar_wait<!SWAP>(&empty[s], (r & 1) ^ 1, args.status, kStatusTimeoutEmpty)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
            if constexpr (SWAP) {
              tma_load_2d_hint(sa, &tmA, &full[s], kx, tc.a_base + tc.mt * BM, pol_w);
              if constexpr (C::NUM_A == 2)
                tma_load_2d_hint(sa + C::A_BYTES, &tmA, &full[s], kx,
                                 tc.a_base + tc.mt * BM + args.inter, pol_w);
              tma_load_2d_hint(sb, &tmB, &full[s], kx, tc.b_base + tc.nt * BN, pol_x);
            } else {
              tma_load_2d_hint(sa, &tmA, &full[s], kx, tc.a_base + tc.mt * BM, pol_x);
              tma_load_2d_hint(sb, &tmB, &full[s], kx, tc.b_base + tc.nt * BROWS, pol_w);
              if constexpr (C::kSwiGLU)
                tma_load_2d_hint(sb + BROWS * 128, &tmB, &full[s], kx,
                                 tc.b_base + tc.nt * BROWS + args.inter, pol_w);
            }
          }
          if (!ok) break;
        }
      }
    } else if (warp == 1) {
      if (lane == 0) {
        constexpr uint32_t idesc = umma_idesc_bf16(BM, BN);
        int i = 0, j = 0;
        bool ok = true;
        Sched sch(args, cta, total_tiles);
        Segment sg;
        while (ok && sch.next(args, sg)) {
          const int b = j & 1;
          if (!mbar_wait<!SWAP>(&acc_empty[b], ((j >> 1) & 1) ^ 1, args.status, kStatusTimeoutAccum)) break;
          tc_fence_after();
          const uint32_t acc = tmem_base + b * C::ACC_COLS;
          for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++i) {
            const int s = i % STAGES;
            if (!mbar_wait<!SWAP>(&full[s], (i / STAGES) & 1, args.status, kStatusTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(smem + s * C::STAGE_BYTES);
            const uint32_t b_addr = a_addr + C::NUM_A * C::A_BYTES;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint32_t accum = (kb > sg.kb0 || k > 0) ? 1u : 0u;
              const uint64_t bd = umma_desc_sw128(b_addr + k * 32);
              umma_f16(acc, umma_desc_sw128(a_addr + k * 32), bd, idesc, accum);
              if constexpr (C::NUM_A == 2)
                umma_f16(acc + BN, umma_desc_sw128(a_addr + C::A_BYTES + k * 32), bd, idesc, accum);
            }
            umma_commit(&empty[s]);
          }
          if (!ok) break;
          umma_commit(&acc_full[b]);
          ++j;
        }
      }
    } else {
      // Epilogue warps 2..5.
      constexpr int CW = C::CW;
      constexpr int UOFF = SWAP ? BN : BN / 2;
      const int q = warp & 3;
      const int row = q * 32 + lane;
      pdl_wait();  // residual, output and workspace belong to the previous kernel until now
      uint32_t epoch = 0;
      int par = 0;
      if constexpr (EPI == kEpiAllReduce) {
        epoch = *reinterpret_cast<volatile uint32_t*>(args.peers[args.tp_rank]) + 1u;
        par = epoch & 1;
      }
      int j = 0;
      Sched sch(args, cta, total_tiles);
      Segment sg;
      while (sch.next(args, sg)) {
        const int b = j & 1;
        const TileCtx tc = make_ctx<GROUPED, SWAP>(args, sg.tile, s_pref);
        const int nt = tc.nt;
        const int m_glob = tc.mt * BM + row;
        if (!mbar_wait<!SWAP>(&acc_full[b], (j >> 1) & 1, args.status, kStatusTimeoutAccum)) break;
        tc_fence_after();
        const uint32_t taddr = tmem_base + b * C::ACC_COLS + (static_cast<uint32_t>(q * 32) << 16);
        const bool whole = sg.kb0 == 0 && sg.kb1 == nkb;
        if (whole) {
#pragma unroll 1
          for (int c0 = 0; c0 < C::OUT_COLS; c0 += CW) {
            float v[CW], uu[CW];
            uint32_t rv[CW];
            tmem_load<CW>(taddr + c0, rv);
#pragma unroll
            for (int t = 0; t < CW; ++t) v[t] = __uint_as_float(rv[t]);
            if constexpr (C::kSwiGLU) {
              tmem_load<CW>(taddr + c0 + UOFF, rv);
#pragma unroll
              for (int t = 0; t < CW; ++t) uu[t] = __uint_as_float(rv[t]);
            }
            if (c0 + CW >= C::OUT_COLS) {
              tc_fence_before();
              mbar_arrive(&acc_empty[b]);
            }
            if constexpr (EPI == kEpiAllReduce) ar_push<CW>(args, par, m_glob, nt * C::OUT_COLS + c0, v);
            else store_chunk<EPI, SWAP, CW>(args, m_glob, nt * C::OUT_COLS + c0, v, uu, tc.Mv, tc.Nv, tc.roff);
          }
          if constexpr (EPI == kEpiAllReduce) ar_publish(args, par, epoch, sg.tile);
        } else if (SWAP && !GROUPED && EPI != kEpiAllReduce && args.split_s > 1) {
          // Cluster split: keep this K range's fp32 partial in this CTA's shared memory
          // ([ACC_COLS][BM], in the stage buffers, idle now that the only segment's MMAs are
          // done); the cluster reduces the tile after the role loops.
          static_assert(C::ACC_COLS * BM * 4 <= STAGES * C::STAGE_BYTES, "partial must fit the stages");
          float* part = reinterpret_cast<float*>(smem);
#pragma unroll 1
          for (int c0 = 0; c0 < C::ACC_COLS; c0 += CW) {
            uint32_t rv[CW];
            tmem_load<CW>(taddr + c0, rv);
#pragma unroll
            for (int t = 0; t < CW; ++t) part[(c0 + t) * BM + row] = __uint_as_float(rv[t]);
          }
          tc_fence_before();
          mbar_arrive(&acc_empty[b]);
        } else {
          // Partial tile: slot 0 = this CTA's first segment, slot 1 = its last.
          const int slot = sg.first ? 0 : 1;
          float* mine = args.ws + ((long long)cta * 2 + slot) * C::ACC_COLS * BM;
#pragma unroll 1
          for (int c0 = 0; c0 < C::ACC_COLS; c0 += CW) {
            uint32_t rv[CW];
            tmem_load<CW>(taddr + c0, rv);
#pragma unroll
            for (int t = 0; t < CW; ++t) __stcg(&mine[(c0 + t) * BM + row], __uint_as_float(rv[t]));
          }
          tc_fence_before();
          mbar_arrive(&acc_empty[b]);
          // Contributors of this tile: CTAs whose unit ranges intersect it.
          const long long t0 = (long long)sg.tile * nkb;
          const int c_first = static_cast<int>(((t0 + 1) * G - 1) / U);
          const int c_last = min(G - 1, static_cast<int>(((t0 + nkb) * (long long)G - 1) / U));
          __threadfence();
          named_bar_sync(1, 128);
          if (threadIdx.x == 64) {
            const int old = atomicAdd(&args.counters[sg.tile], 1);
            flags[1] = (old == c_last - c_first);
          }
          named_bar_sync(1, 128);
          const bool last = flags[1] != 0;
          named_bar_sync(1, 128);  // flags[1] is reused by the next partial segment
          if (last) {
            __threadfence();
#pragma unroll 1
            for (int c0 = 0; c0 < C::OUT_COLS; c0 += CW) {
              float v[CW], uu[CW];
#pragma unroll
              for (int t = 0; t < CW; ++t) { v[t] = 0.f; uu[t] = 0.f; }
              // Contributors in batches of 4: issue every load of a batch before
              // summing, then add in contributor order (deterministic).
              constexpr int NB = 4;
              for (int cb = c_first; cb <= c_last; cb += NB) {
                float pv[NB][CW];
#pragma unroll
                for (int q2 = 0; q2 < NB; ++q2) {
                  const int c = cb + q2;
                  if (c <= c_last) {
                    const int sl = unit_begin(c, U, G) >= t0 ? 0 : 1;
                    const float* p = args.ws + ((long long)c * 2 + sl) * C::ACC_COLS * BM;
#pragma unroll
                    for (int t = 0; t < CW; ++t) pv[q2][t] = __ldcg(&p[(c0 + t) * BM + row]);
                  }
                }
#pragma unroll
                for (int q2 = 0; q2 < NB; ++q2)
                  if (cb + q2 <= c_last) {
#pragma unroll
                    for (int t = 0; t < CW; ++t) v[t] += pv[q2][t];
                  }
                if constexpr (C::kSwiGLU) {
#pragma unroll
                  for (int q2 = 0; q2 < NB; ++q2) {
                    const int c = cb + q2;
                    if (c <= c_last) {
                      const int sl = unit_begin(c, U, G) >= t0 ? 0 : 1;
                      const float* p = args.ws + ((long long)c * 2 + sl) * C::ACC_COLS * BM;
#pragma unroll
                      for (int t = 0; t < CW; ++t) pv[q2][t] = __ldcg(&p[(c0 + UOFF + t) * BM + row]);
                    }
                  }
#pragma unroll
                  for (int q2 = 0; q2 < NB; ++q2)
                    if (cb + q2 <= c_last) {
#pragma unroll
                      for (int t = 0; t < CW; ++t) uu[t] += pv[q2][t];
                    }
                }
              }
              if constexpr (EPI == kEpiAllReduce) ar_push<CW>(args, par, m_glob, nt * C::OUT_COLS + c0, v);
              else store_chunk<EPI, SWAP, CW>(args, m_glob, nt * C::OUT_COLS + c0, v, uu, tc.Mv, tc.Nv, tc.roff);
            }
            if (threadIdx.x == 64) args.counters[sg.tile] = 0;  // re-arm for the next launch
            if constexpr (EPI == kEpiAllReduce) ar_publish(args, par, epoch, sg.tile);
          }
        }
        ++j;
      }
      if constexpr (EPI == kEpiAllReduce) {
        // Phase 2: (tile, 8-token group) items spread over every CTA; each waits for the
        // tile's flags from all ranks, then sums the bf16 partials in rank order (fp32)
        // plus the residual, in place.  All loads of an item are issued before the sum.
        const int NG = (args.N + 7) / 8;
        const int items = args.m_tiles * NG;
        for (int itm = cta; itm < items; itm += G) {
          const int t = itm / NG, ng = itm % NG;
          if (threadIdx.x == 64) {
            for (int r = 0; r < args.tp_size; ++r) {
              const uint32_t* f = ar_flag(args, args.tp_rank, par, r, t);
              const uint64_t t_start = globaltimer_ns();
              uint32_t it = 0;
              while (ld_acquire_sys(f) != epoch) {
                if ((++it & 255u) == 0 &&
                    (load_status(args.status) != 0 || globaltimer_ns() - t_start > wait_limit_ns(args.status))) {
                  raise_status(args.status, kStatusTimeoutPeer);
                  break;
                }
              }
            }
          }
          named_bar_sync(1, 128);
          const int m = t * BM + row;
          if (m < args.M) {
            float acc[8];
            __nv_bfloat16 pv[kMaxTP][8];
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
              const int n = ng * 8 + jj;
              acc[jj] = n < args.N ? __bfloat162float(args.res[(long long)n * args.ldr + m]) : 0.f;
            }
#pragma unroll
            for (int r = 0; r < kMaxTP; ++r) {
              if (r < args.tp_size) {
                const __nv_bfloat16* src = ar_slot(args, args.tp_rank, par, r);
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                  const int n = ng * 8 + jj;
                  pv[r][jj] = n < args.N ? __ldcg(src + (long long)n * args.max_hidden + m)
                                         : __float2bfloat16_rn(0.f);
                }
              }
            }
            // Rank-ordered sum of the partials, then the residual (same order on every rank).
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
              float sum = 0.f;
#pragma unroll
              for (int r = 0; r < kMaxTP; ++r)
                if (r < args.tp_size) sum += __bfloat162float(pv[r][jj]);
              acc[jj] += sum;
            }
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
              const int n = ng * 8 + jj;
              if (n < args.N)
                reinterpret_cast<__nv_bfloat16*>(args.out)[(long long)n * args.ldo + m] =
                    __float2bfloat16_rn(acc[jj]);
            }
          }
        }
      }
    }
  }
  if constexpr (SWAP && !GROUPED && EPI != kEpiAllReduce) {
    if (args.split_s > 1) {
      // Every thread of every CTA of the cluster passes both barriers exactly once (all
      // waits above are bounded and no thread leaves the kernel early), so the cluster
      // cannot stall here.  Between them each CTA reduces its share of the tile's items
      // (row quarter x column chunk) over the s partials in cluster-rank order, reading
      // the peers' shared memory directly.
      cluster_sync_all();
      if (warp >= 2 && !skip) {
        constexpr int CW = C::CW;
        constexpr int UOFF = SWAP ? BN : BN / 2;
        constexpr int CWR = C::OUT_COLS / 8 > 8 ? C::OUT_COLS / 8 : 8;
        constexpr int NI = 4 * (C::OUT_COLS / CWR);
        constexpr int NBW = 32 / (CWR * (C::kSwiGLU ? 2 : 1));
        constexpr int NB = NBW < 1 ? 1 : NBW;
        (void)CW;
        const int s = args.split_s;
        const uint32_t ci = cluster_ctarank();
        const int tile = cta / s;
        const TileCtx tc = make_ctx<false, SWAP>(args, tile, s_pref);
        const uint32_t part = smem_u32(smem);
        for (int k = static_cast<int>(ci) * 4 + (warp - 2); k < NI; k += 4 * s) {
          const int r = (k & 3) * 32 + lane;
          const int c0 = (k >> 2) * CWR;
          float v[CWR], uu[CWR];
#pragma unroll
          for (int t = 0; t < CWR; ++t) { v[t] = 0.f; uu[t] = 0.f; }
#pragma unroll 1
          for (int cb = 0; cb < s; cb += NB) {
            float pv[NB][CWR], pu[NB][CWR];
#pragma unroll
            for (int q2 = 0; q2 < NB; ++q2)
              if (cb + q2 < s) {
                const uint32_t base = mapa_cluster(part, static_cast<uint32_t>(cb + q2));
#pragma unroll
                for (int t = 0; t < CWR; ++t) {
                  pv[q2][t] = ld_dsmem_f32(base + ((c0 + t) * BM + r) * 4);
                  if constexpr (C::kSwiGLU) pu[q2][t] = ld_dsmem_f32(base + ((c0 + UOFF + t) * BM + r) * 4);
                }
              }
#pragma unroll
            for (int q2 = 0; q2 < NB; ++q2)
              if (cb + q2 < s) {
#pragma unroll
                for (int t = 0; t < CWR; ++t) {
                  v[t] += pv[q2][t];
                  if constexpr (C::kSwiGLU) uu[t] += pu[q2][t];
                }
              }
          }
          store_chunk<EPI, SWAP, CWR>(args, tc.mt * BM + r, tc.nt * C::OUT_COLS + c0, v, uu, tc.Mv,
                                      tc.Nv, tc.roff);
        }
      }
      cluster_sync_all();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if constexpr (EPI == kEpiAllReduce) {
    // Advance this rank's epoch once every CTA of the launch has read it.
    if (threadIdx.x == 0) {
      pdl_wait();
      volatile uint32_t* st = reinterpret_cast<volatile uint32_t*>(args.peers[args.tp_rank]);
      const uint32_t e = st[0] + 1u;
      __threadfence();
      const uint32_t old = atomicAdd(const_cast<uint32_t*>(&st[1]), 1u);
      if (old == static_cast<uint32_t>(G - 1)) {
        st[1] = 0u;
        __threadfence();
        st[0] = e;
      }
    }
  }
}

template <int BN, int STAGES, int EPI, bool SWAP, bool GROUPED = false>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args,
            cudaStream_t stream) {
  using C = Cfg<BN, STAGES, EPI, SWAP>;
  auto kern = gemm_bf16_kernel<BN, STAGES, EPI, SWAP, GROUPED>;
  constexpr int kSmem = C::SMEM_BYTES + (GROUPED ? (kMaxGroups + 8) * 4 : 0);
  set_smem_limit(reinterpret_cast<const void*>(kern), kSmem, "cudaFuncSetAttribute(gemm smem)");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(args.grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (args.split_s > 1) {  // one cluster per tile: its K ranges reduce through shared memory
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = args.split_s;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  check_cuda(cudaLaunchKernelEx(&cfg, kern, ta, tb, args), "gemm_bf16_kernel launch");
}

// Clusters of s split CTAs (one CTA per SM: every swapped-order configuration needs more
// than half of an SM's shared memory) that the current device holds at once; 0 when such a
// cluster cannot be launched.  Cached per device.
int max_active_clusters(int s);

template <int EPI>
void dispatch_swap(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                   cudaStream_t st);
template <int EPI>
void dispatch_normal(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                     cudaStream_t st);
template <int EPI>
void dispatch_grouped(bool swap, int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                      const GemmArgs& a, cudaStream_t st);

}  // namespace gemm_detail
}  // namespace sil
