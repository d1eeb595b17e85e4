// Causal paged prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// One CTA per (pair of 128-query tiles, query head, sequence): queries q0..q0+255 of one head
// as two tiles A (q0..q0+127) and B (q0+128..q0+255) that share every K / V tile the CTA
// loads, so a 64 KB K+V tile feeds 2 x 8.4 MFLOP of MMA (one tile per CTA needed twice the
// shared-memory fill rate per FLOP and left the tensor cores waiting on L2).  Three
// warpgroups (384 threads); warpgroup 0 gives registers to the two softmax warpgroups
// (setmaxnreg: 72 / 216 / 216 registers per thread, launched with 168):
//   warp 0      TMA producer: both Q tiles once, then K and V tiles of 128 tokens (two 64-token
//               pages of the paged cache) into two separate two-stage rings.  K runs one tile
//               ahead of V: a K buffer is free once its QK^T MMAs finished, a V buffer only
//               after its PVs;
//   warp 1      MMA issuer (one elected thread) and TMEM owner.  Per key tile j, for X = A, B:
//                 O_X += P_X(j) V_j              (A = P from TMEM, M=128, N=128 dims, K=128 keys)
//                 S_X  = Q_X K_{j+1}^T           (M=128 queries, N=128 keys, K=128 dims)
//               so the tensor cores work on one tile's MMAs while the other tile's softmax runs
//               (ping-pong).  S_X(j+1) overwrites the TMEM columns that P_X(j) occupies, and
//               MMAs with different accumulators are not ordered by the hardware, so the issuer
//               waits for PV_X(j) to complete before it issues S_X(j+1) (issuing the half of
//               S beside P ahead of that wait, as two N=64 MMAs, measured slower);
//   warps 2, 3  idle (they only complete warpgroup 0 for the register hand-over);
//   warps 4..7  softmax and epilogue of tile A, warps 8..11 of tile B: thread i of a group owns
//               query row i (TMEM lane i).  It reads its S row, applies the scale and the causal
//               mask, keeps the running max m and sum l (exp2 domain), rescales its O row in
//               TMEM only when m grew, writes its P row as packed bf16 over its S row, and after
//               the last tile writes O / l as bf16.
// TMEM (512 columns): S_A 0..127 (P_A in 0..63), S_B 128..255 (P_B), O_A 256..383, O_B 384..511.
//
// Shared-memory layouts (all 128-byte swizzled, 1024-byte aligned):
//   Q  [tile][dim half][128 rows][64 dims]      A operand of QK^T, K-major
//   K  [stage][dim half][128 tokens][64 dims]   B operand of QK^T, K-major
//   V  [stage][dim half][128 tokens][64 dims]   B operand of PV, MN-major (dims contiguous)
// A 64-token page of one KV head is two [64 x 64] TMA boxes; page p of a tile lands at
// rows 64p..64p+63 of both dim halves.  A tile's second page past the end of the sequence is
// replaced by its first page (finite values that the mask zeroes).
//
// Every wait is bounded (the status word); a CTA whose wait gave up lets its own loads in
// flight land, frees its TMEM and returns.
//
// Replaces the reference's SDPA / FlashAttention-2 prefill (si/model/qwen3.py:916-996).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sil/host.h"
#include "sil/ptx.cuh"

namespace sil {
namespace {

constexpr int kPage = 64;
constexpr int kD = 128;
constexpr int kBM = 128;                     // queries per tile
constexpr int kQT = 2;                       // query tiles per CTA
constexpr int kBN = 128;                     // keys per tile
constexpr int kHalf = 128 * 64 * 2;          // one [128 rows x 64] bf16 half-tile: 16 KB
constexpr int kTile = 2 * kHalf;             // 32 KB
constexpr int kBox = 64 * 64 * 2;            // one TMA box: 8 KB
constexpr int kThreads = 128 + kQT * 128;   // warpgroup 0 (producer, MMA) + one per tile
constexpr int kLaunchRegs = 168;             // 65536 / 384, rounded down to 8
constexpr int kRegsWg0 = 72, kRegsSoftmax = 216;
static_assert(128 * kRegsWg0 + kQT * 128 * kRegsSoftmax <= kThreads * kLaunchRegs,
              "register split above the launch allocation");
constexpr int kTmemCols = 512;
constexpr uint32_t kColO = 256;              // O_X at kColO + 128 X; S_X / P_X at 128 X

// smem map (offsets from the 1024-aligned base)
constexpr int kOffQ = 0;                     // kQT tiles
constexpr int kOffK = kOffQ + kQT * kTile;   // 2 stages
constexpr int kOffV = kOffK + 2 * kTile;     // 2 stages
constexpr int kOffBar = kOffV + 2 * kTile;
constexpr int kSmemBytes = kOffBar + 256 + 1024;

struct FmhaArgs {
  __nv_bfloat16* out;
  long long o_stride;      // elements between consecutive tokens of out
  const int* block_table;
  long long bt_stride;
  const int* seq_lens;     // context length incl. the new tokens
  const int* cu_q;         // [B+1]
  int Hq, Hkv, G;
  int num_pages;
  float scale_log2;
  int* status;
};

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// D (TMEM) (+)= A (TMEM) x B (shared memory descriptor), kind::f16.  A is M x K with row i in
// lane i and two 16-bit K elements per 32-bit column (lower K index in the low half).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory descriptor of an MN-major operand with the 128-byte swizzle: 64 MN
// elements (128 bytes) per row, consecutive K rows 128 bytes apart; `mn_stride` bytes from
// MN elements 0..63 to 64..127, 1024 bytes per 8 K rows.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t mn_stride) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((mn_stride >> 4) & 0x3FFFu) << 16;   // LBO: along MN
  d |= static_cast<uint64_t>(1024u >> 4) << 32;                     // SBO: 8 K rows
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// K-major A/B with 128 rows per dim half (1024-byte 8-row atoms stacked along M/N).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kslice) {
  return umma_desc_sw128(base + (kslice >> 2) * kHalf + (kslice & 3) * 32);
}

// 2^x with the hardware approximation (MUFU.EX2; flushes denormals), one instruction.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// A running max may lag the true one by up to 2^8 before O is rescaled: P values stay
// below 256 (fine in bf16) and most tiles skip the TMEM round trip of the rescale.
constexpr float kRescaleThreshold = 8.0f;

template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// Packed fp32 pairs (sm_100 f32x2 instructions: two lanes of work per issue slot).
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add_f2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, int* status) {
  return mbar_wait(bar, parity, status, kStatusTimeoutFull);
}

__global__ void __launch_bounds__(kThreads, 1)
    fmha_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                           const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const FmhaArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;     // [2]
  uint64_t* k_empty = bars + 3;    // [2]
  uint64_t* v_full = bars + 5;     // [2]
  uint64_t* v_empty = bars + 7;    // [2]
  uint64_t* s_full = bars + 9;     // [kQT]: S_X(j) in TMEM
  uint64_t* p_full = bars + 11;    // [kQT]: P_X(j) in TMEM (128 arrivals)
  uint64_t* o_done = bars + 13;    // [kQT]: PV_X(j) finished
  uint64_t* mma_done = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  int* sflag = reinterpret_cast<int*>(bars + 17);  // [2]: K / V tiles issued

  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hq = blockIdx.y, b = blockIdx.z;
  const int h = hq / args.G;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int x = 0; x < kQT; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 128);
      mbar_init(&o_done[x], 1);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_wait();  // q and the KV cache come from earlier kernels
  const int q_begin = args.cu_q[b];
  const int q_len = args.cu_q[b + 1] - q_begin;
  const int n_qp = (q_len + kQT * kBM - 1) / (kQT * kBM);
  const int qp = (int)gridDim.x - 1 - (int)blockIdx.x;  // heaviest pairs first
  const int kv_len = args.seq_lens[b];
  const int pos0 = kv_len - q_len;
  const int q0 = qp * kQT * kBM;
  const bool active_cta = qp < n_qp && load_status(args.status) == 0;
  int n_t[kQT];  // key tiles of query tile X (0 when the tile has no query)
#pragma unroll
  for (int x = 0; x < kQT; ++x) {
    const int qx = q0 + x * kBM;
    const int keys = (active_cta && qx < q_len) ? min(pos0 + min(qx + kBM, q_len), kv_len) : 0;
    n_t[x] = (keys + kBN - 1) / kBN;
  }
  int n_tiles = 0;  // K / V tiles the CTA streams
#pragma unroll
  for (int x = 0; x < kQT; ++x) n_tiles = max(n_tiles, n_t[x]);
  const int n_pages = (kv_len + kPage - 1) / kPage;
  const int* bt = args.block_table + (long long)b * args.bt_stride;
  const uint32_t sbase = smem_u32(smem);

  // Each setmaxnreg sits inside its own role branch: ptxas compiles the code it dominates
  // with that register budget, so no softmax code may be reachable after the decrease.
  if (warp < 4) {
    regs_dec<kRegsWg0>();
  if (warp == 0) {
    if (lane == 0 && n_tiles > 0) {
      // Q: two [128 x 64] boxes per tile of head hq at rows q_begin + q0 + 128 X.  Rows past
      // the end of q are filled with zeros by the TMA unit; rows of the next sequence are
      // finite.  Neither is stored.
      mbar_arrive_expect_tx(q_full, kQT * kTile);
      for (int x = 0; x < kQT; ++x)
        for (int d = 0; d < 2; ++d)
          tma_load_2d(smem + kOffQ + x * kTile + d * kHalf, &tmQ, q_full, hq * kD + d * 64,
                      q_begin + q0 + x * kBM);
      // Page ids of tile j (a second page past the context repeats the first).
      auto tile_pages = [&](int j, int (&pg)[2]) -> bool {
        bool good = true;
        for (int p = 0; p < 2; ++p) {
          const int page = 2 * j + p < n_pages ? 2 * j + p : 2 * j;
          const int pid = bt[page];
          if (static_cast<unsigned>(pid) >= static_cast<unsigned>(args.num_pages)) {
            raise_status(args.status, kStatusBadArgument);
            good = false;
          }
          pg[p] = pid;
        }
        return good;
      };
      // One [128 x 128] tile: two pages x two dim halves, four [64 x 64] boxes.
      auto load_tile = [&](const CUtensorMap* tm, uint8_t* dst, uint64_t* bar, const int (&pg)[2]) {
        mbar_arrive_expect_tx(bar, kTile);
        for (int p = 0; p < 2; ++p) {
          const int row = (pg[p] * args.Hkv + h) * kPage;
          for (int d = 0; d < 2; ++d) tma_load_2d(dst + d * kHalf + p * kBox, tm, bar, d * 64, row);
        }
      };
      int k_issued = 0, v_issued = 0;
      // Order K_0, K_1, V_0, K_2, V_1, ...: K one tile ahead of V.
      for (int i = 0; i <= n_tiles; ++i) {
        if (i < n_tiles) {
          const int s = i & 1;
          if (i >= 2 && !wait_bar(&k_empty[s], ((i >> 1) - 1) & 1, args.status)) break;
          int pg[2];
          if (!tile_pages(i, pg)) break;
          load_tile(&tmK, smem + kOffK + s * kTile, &k_full[s], pg);
          k_issued = i + 1;
        }
        if (i >= 1) {
          const int j = i - 1, s = j & 1;
          if (j >= 2 && !wait_bar(&v_empty[s], ((j >> 1) - 1) & 1, args.status)) break;
          int pg[2];
          if (!tile_pages(j, pg)) break;
          load_tile(&tmV, smem + kOffV + s * kTile, &v_full[s], pg);
          v_issued = j + 1;
        }
      }
      sflag[0] = k_issued;
      sflag[1] = v_issued;
    }
  } else if (warp == 1) {
    if (lane == 0 && n_tiles > 0) {
      const uint32_t idesc_s = umma_idesc_bf16(kBM, kBN);  // one 64-key half of S
      const uint32_t idesc_o = umma_idesc_bf16(kBM, kD) | (1u << 16);  // B (V) MN-major
      // Half `hf` of S_X = Q_X K_j^T: keys 64 hf .. 64 hf + 63 (K rows 64 hf.., 8 KB further
      // into each dim half) into TMEM columns 64 hf ...  P_X occupies columns 0..63 only.
      auto issue_s = [&](int x, int j) {  // S_X = Q_X K_j^T
        const uint32_t qa = sbase + kOffQ + x * kTile;
        const uint32_t kb = sbase + kOffK + (j & 1) * kTile;
#pragma unroll
        for (int k = 0; k < kD / 16; ++k)
          umma_f16(tmem + x * 128, kmajor_desc(qa, k), kmajor_desc(kb, k), idesc_s, k > 0 ? 1u : 0u);
        umma_commit(&s_full[x]);
      };
      auto issue_pv = [&](int x, int j) {  // O_X += P_X V_j, 16 keys (8 TMEM columns) per MMA
        const uint32_t vb = sbase + kOffV + (j & 1) * kTile;
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k)
          umma_f16_ts(tmem + kColO + x * 128, tmem + x * 128 + k * 8,
                      umma_desc_sw128_mn(vb + k * 2048, kHalf), idesc_o, (j > 0 || k > 0) ? 1u : 0u);
        umma_commit(&o_done[x]);
      };
      bool ok = wait_bar(q_full, 0, args.status) && wait_bar(&k_full[0], 0, args.status);
      if (ok) {
        tc_fence_after();
        for (int x = 0; x < kQT; ++x)
          if (n_t[x] > 0) issue_s(x, 0);
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int s = j & 1;
        bool v_ready = false, k_ready = false;
        for (int x = 0; x < kQT && ok; ++x) {
          if (j >= n_t[x]) continue;
          if (!wait_bar(&p_full[x], j & 1, args.status)) { ok = false; break; }
          if (!v_ready && !wait_bar(&v_full[s], (j >> 1) & 1, args.status)) { ok = false; break; }
          v_ready = true;
          tc_fence_after();
          issue_pv(x, j);
          if (j + 1 < n_t[x]) {
            // S_X(j+1) overwrites P_X(j): PV_X(j) must have read it.
            if (!wait_bar(&o_done[x], j & 1, args.status)) { ok = false; break; }
            if (!k_ready && !wait_bar(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, args.status)) {
              ok = false;
              break;
            }
            k_ready = true;
            tc_fence_after();
            issue_s(x, j + 1);
          }
        }
        if (!ok) break;
        umma_commit(&v_empty[s]);                              // V_j's PVs are issued
        if (j + 1 < n_tiles) umma_commit(&k_empty[(j + 1) & 1]);  // K_{j+1}'s QK^Ts are issued
      }
      // Every MMA this thread issued has finished before TMEM is released (also when a wait
      // above gave up): one more commit, waited for regardless of the status word.
      umma_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
  }
  } else {
    regs_inc<kRegsSoftmax>();
    const int x = (warp - 4) >> 2;          // query tile of this warpgroup
    const int q4 = warp & 3;                // TMEM lane quarter this warp may access
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    const int n_x = n_t[x];
    const int qx0 = q0 + x * kBM;
    const int qi = qx0 + row;               // query index within the sequence
    const int qpos = pos0 + qi;             // its absolute position
    const uint32_t tS = tmem + x * 128 + lane_off;
    const uint32_t tO = tmem + kColO + x * 128 + lane_off;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // tcgen05.ld / st are warp-collective (.sync.aligned): every branch around them below
    // is made uniform across the warp (__all_sync / __any_sync).
    for (int j = 0; j < n_x && ok; ++j) {
      ok = __all_sync(0xffffffffu, wait_bar(&s_full[x], j & 1, args.status));
      if (!ok) break;
      tc_fence_after();
      float sv[kBN];
      {
        uint32_t r[kBN];  // one x128 load and one wait: a single TMEM round trip
        tmem_ld128_sync(tS, r);
#pragma unroll
        for (int t = 0; t < kBN; ++t) sv[t] = __uint_as_float(r[t]);
      }
      const int key0 = j * kBN;
      // Masks are needed only on tiles that reach past the tile's first query position
      // (the causal diagonal) or past the end of the context (uniform per warpgroup).
      if (key0 + kBN - 1 > pos0 + qx0 || key0 + kBN > kv_len) {
#pragma unroll
        for (int t = 0; t < kBN; ++t)
          if (key0 + t > qpos || key0 + t >= kv_len) sv[t] = -INFINITY;
      }
      // Eight independent partial maxima (3-input max: two keys per instruction).
      float mxp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mxp[u] = fmaxf(sv[2 * u], sv[2 * u + 1]);
#pragma unroll
      for (int t = 16; t < kBN; t += 16)
#pragma unroll
        for (int u = 0; u < 8; ++u) mxp[u] = max3f(mxp[u], sv[t + 2 * u], sv[t + 2 * u + 1]);
      const float mx = max3f(max3f(mxp[0], mxp[1], mxp[2]), max3f(mxp[3], mxp[4], mxp[5]),
                             fmaxf(mxp[6], mxp[7]));
      // Running max in the scaled exp2 domain; it moves only when the tile's max exceeds it by
      // the threshold (or on the first tile with a finite score).
      const float mx_s = mx * args.scale_log2;
      float alpha = 1.f;
      if (m == -INFINITY || mx_s > m + kRescaleThreshold) {
        const float m_new = fmaxf(m, mx_s);
        alpha = m == -INFINITY ? 0.f : ex2_approx(m - m_new);
        m = m_new;
      }
      const float m_use = m == -INFINITY ? 0.f : m;
      // p = 2^(s * scale - m) for key pairs (one f32x2 FMA), sums in four packed accumulators.
      // P_X(j) goes to TMEM over columns 0..63 of the S row (keys 2c, 2c+1 in column c), the
      // first 64 keys stored while the second half's exponentials are computed.
      const uint64_t sc2 = f2(args.scale_log2, args.scale_log2), nm2 = f2(-m_use, -m_use);
      uint64_t acc[4] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t w[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int t = hh * 64 + 2 * c;
          float x0, x1;
          f2_split(fma_f2(f2(sv[t], sv[t + 1]), sc2, nm2), x0, x1);
          const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
          acc[c & 3] = add_f2(acc[c & 3], f2(p0, p1));
          w[c] = pack_bf16x2(p0, p1);
        }
        tmem_st32(tS + hh * 32, w);
      }
      float rsl[4], rsh[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) f2_split(acc[u], rsl[u], rsh[u]);
      const float rs = ((rsl[0] + rsh[0]) + (rsl[1] + rsh[1])) + ((rsl[2] + rsh[2]) + (rsl[3] + rsh[3]));
      l = l * alpha + rs;
      // Rows whose max did not move multiply by 1; the warp skips only if none moved.  O_X is
      // stable here: S_X(j) was issued after PV_X(j - 1) had completed.
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < kD / 32; ++c) {
          uint32_t r[32];
          tmem_ld32_sync(tO + c * 32, r);
#pragma unroll
          for (int t = 0; t < 32; ++t) r[t] = __float_as_uint(__uint_as_float(r[t]) * alpha);
          tmem_st32(tO + c * 32, r);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[x]);
    }
    const bool done = ok && n_x > 0 && wait_bar(&o_done[x], (n_x - 1) & 1, args.status);
    if (__all_sync(0xffffffffu, done)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool store = qi < q_len;
      __nv_bfloat16* orow = args.out + (long long)(q_begin + qi) * args.o_stride + (long long)hq * kD;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t r[32];
        tmem_ld32_sync(tO + c * 32, r);
        if (store) {
#pragma unroll
          for (int t = 0; t < 32; t += 8) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(r[t + 0]) * inv, __uint_as_float(r[t + 1]) * inv);
            v.y = pack_bf16x2(__uint_as_float(r[t + 2]) * inv, __uint_as_float(r[t + 3]) * inv);
            v.z = pack_bf16x2(__uint_as_float(r[t + 4]) * inv, __uint_as_float(r[t + 5]) * inv);
            v.w = pack_bf16x2(__uint_as_float(r[t + 6]) * inv, __uint_as_float(r[t + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + t) = v;
          }
        }
      }
    }
  }
  // Teardown: a producer that gave up lets its own loads land before the CTA exits.
  __syncthreads();
  if (warp == 0 && lane == 0 && n_tiles > 0 && load_status(args.status) != 0) {
    mbar_drain(q_full, 0);
    for (int kv = 0; kv < 2; ++kv) {
      const int issued = sflag[kv];
      uint64_t* full = kv ? v_full : k_full;
      for (int j = max(0, issued - 2); j < issued; ++j) mbar_drain(&full[j & 1], (j >> 1) & 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();  // tcgen05.dealloc is warp-collective: lane 0 ran the MMA loop alone
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

// q: packed [T, Hq, 128] (token stride q.stride(0)); k/v cache [pages, Hkv, 64, 128];
// cu_q [B+1]; seq_lens [B] (context after append); out [T, Hq*128].
void paged_prefill_tc(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                      const at::Tensor& block_table, const at::Tensor& seq_lens,
                      const at::Tensor& cu_q, at::Tensor& out, double scale, int64_t max_q_len,
                      const at::Tensor& status) {
  for (const at::Tensor* c : {&k_cache, &v_cache})
    TORCH_CHECK(c->is_cuda() && c->scalar_type() == at::kBFloat16 && c->is_contiguous() &&
                    c->dim() == 4 && c->size(2) == kPage && c->size(3) == kD,
                "paged_prefill_tc: KV cache must be contiguous bf16 [pages, Hkv, 64, 128]");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.size(2) == kD &&
                  q.stride(2) == 1 && q.stride(1) == kD && q.stride(0) % 8 == 0,
              "paged_prefill_tc: q must be [T, Hq, 128] with contiguous heads, 16-byte row pitch");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.stride(0) % 8 == 0,
              "paged_prefill_tc: out [T, Hq*128] bf16 with a 16-byte row pitch");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  cu_q.scalar_type() == at::kInt,
              "paged_prefill_tc: int32 block table / seq lens / cu_q");
  TORCH_CHECK(status.numel() >= 4, "paged_prefill_tc: status block");
  const int B = seq_lens.size(0), Hq = q.size(1), Hkv = k_cache.size(1);
  TORCH_CHECK(Hq % Hkv == 0, "paged_prefill_tc: Hq must be a multiple of Hkv");
  if (B == 0 || max_q_len <= 0) return;
  c10::cuda::CUDAGuard guard(q.device());
  FmhaArgs a{};
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
  const uint64_t T = q.size(0);
  CUtensorMap tq = make_tmap_2d(q.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T,
                                (uint64_t)Hq * kD, q.stride(0), kBM, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  const uint64_t rows = (uint64_t)k_cache.size(0) * Hkv * kPage;
  CUtensorMap tk = make_tmap_2d(k_cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, kD,
                                kD, kPage, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tv = make_tmap_2d(v_cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, kD,
                                kD, kPage, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  set_smem_limit(reinterpret_cast<const void*>(fmha_prefill_tc_kernel), kSmemBytes,
                 "cudaFuncSetAttribute(fmha)");
  {
    // setmaxnreg.inc waits for registers that warpgroup 0 hands back; the split adds up to
    // the launch allocation only if the kernel was compiled with kLaunchRegs registers.
    static const int regs = [] {
      cudaFuncAttributes fa{};
      check_cuda(cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(fmha_prefill_tc_kernel)),
                 "cudaFuncGetAttributes(fmha)");
      return fa.numRegs;
    }();
    TORCH_CHECK(regs == kLaunchRegs, "paged_prefill_tc: kernel compiled with ", regs,
                " registers per thread, the register split needs ", kLaunchRegs);
  }
  dim3 grid((max_q_len + kQT * kBM - 1) / (kQT * kBM), Hq, B);
  launch_pdl(fmha_prefill_tc_kernel, grid, dim3(kThreads), kSmemBytes,
             at::cuda::getCurrentCUDAStream(), "paged_prefill_tc launch", tq, tk, tv, a);
}

}  // namespace sil
