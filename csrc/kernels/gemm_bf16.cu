// Host entry of the tcgen05 bf16 GEMM (kernel template: gemm_bf16_impl.cuh).
#include "gemm_bf16_impl.cuh"

namespace sil {
using namespace gemm_detail;

// Persistent grid for a stream-K launch.  Splitting a tile over several CTAs
// costs a fix-up chain (partial store, fence, arrival atomic, ordered
// reduction: a few microseconds of latency); it only pays when the tile's own
// streaming time is longer.  Model: one CTA streams ~kPerSmGBs from HBM, the
// box at most kHbmGBs; choose the number of CTAs per tile minimising
// bytes / bandwidth + fix-up.
// Tile-aligned splits (swapped order) run as one thread-block cluster per tile and reduce
// through distributed shared memory; SIL_SPLIT_REDUCE=last selects the global-memory
// fix-up by the last contributor instead.
inline bool split_reduce_cluster() {
  static const char* mode = std::getenv("SIL_SPLIT_REDUCE");
  return mode == nullptr || mode[0] != 'l';
}

inline long long stream_k_grid(long long tiles, int num_kb, long long bytes_per_kb, int sms,
                               bool cluster = false, bool* use_cluster = nullptr) {
  if (use_cluster != nullptr) *use_cluster = false;
  // Default: tile-aligned splits from a calibrated cost model when there are few tiles,
  // otherwise ("fill") one CTA per SM whenever the problem has >= 4 K blocks per CTA.  The
  // older latency model below is kept behind SIL_STREAMK=latency.
  static const char* mode = std::getenv("SIL_STREAMK");
  if (mode == nullptr || mode[0] != 'l') {
    const long long units = tiles * num_kb;
    if (tiles * 2 <= sms) {
      // Few tiles (decode projections under TP, o_proj, QKV): split every tile into the same
      // number s of K ranges so no CTA straddles two tiles.  Calibrated on B200 (32 tokens,
      // 4096 x {512, 4096} weights, s = 1, 2, 4): ~2.2 us fixed cost, ~48 GB/s streamed per
      // CTA, a split fix-up of ~2.5 us + 0.5 us per split; the box streams at most ~6000 GB/s.
      // A cluster reduces through shared memory with two cluster barriers, far cheaper than
      // the global-memory fix-up; clusters hold at most kMaxClusterSplit CTAs.
      // Measured on B200 (32 tokens; 768 / 1792-SwiGLU / 4096 x {512, 4096}): ~2 us for the
      // cluster fix-up.  A cluster split is only taken when every tile's cluster can be
      // resident at once (clusters live inside one GPC, so fewer fit than SMs / s).
      // Splits whose clusters do not all fit at once are skipped in cluster mode: priced with
      // the global-memory fix-up they can win in isolation (48 tiles x 3 K ranges: 14.3 us
      // against 15.4 us for the 2-CTA clusters that fit) but the decode step got slower with
      // them (4.96 against 4.89 ms at TP1).
      constexpr double kFixedUs = 2.2, kPerCtaGBs = 48.0, kBoxGBs = 6000.0;
      constexpr double kLastFixupUs = 2.5, kLastPerSplitUs = 0.5, kClusterFixupUs = 2.0,
                       kClusterPerSplitUs = 0.05;
      const double tile_bytes = (double)bytes_per_kb * num_kb;
      long long best_s = 1;
      bool best_cluster = false;
      double best_t = 1e30;
      for (long long s = 1; s <= num_kb && tiles * s <= sms; ++s) {
        const double stream = kFixedUs + std::max(tile_bytes / s / (kPerCtaGBs * 1e3),
                                                  tile_bytes * tiles / (kBoxGBs * 1e3));
        const bool fits = cluster && s > 1 && s <= kMaxClusterSplit &&
                          tiles <= max_active_clusters(static_cast<int>(s));
        if (cluster && s > 1 && !fits) continue;
        const double t = s == 1 ? stream
                         : fits ? stream + kClusterFixupUs + kClusterPerSplitUs * s
                                : stream + kLastFixupUs + kLastPerSplitUs * s;
        if (t < best_t - 1e-9) {
          best_t = t;
          best_s = s;
          best_cluster = fits;
        }
      }
      if (use_cluster != nullptr) *use_cluster = best_cluster;
      return tiles * best_s;
    }
    if (cluster && tiles <= sms) {
      // Between half a wave and one wave of tiles (the TP1 SwiGLU gate/up: 112 tiles):
      // whole tiles, one CTA each, need no fix-up, while a stream-K fill of every SM
      // straddles tiles and pays last-arriver fix-ups.  Measured on B200 (32 tokens,
      // 28672 x 4096 SwiGLU): 40.5 us whole against 49.6 us filled.  Streamed per CTA
      // ~60 GB/s, the box ~6400 GB/s, the fill's fix-up ~3 us.
      constexpr double kFixedUs = 2.2, kPerCtaGBs = 60.0, kBoxGBs = 6400.0, kFillFixupUs = 3.0;
      const double tile_bytes = (double)bytes_per_kb * num_kb;
      const double box = tile_bytes * tiles / (kBoxGBs * 1e3);
      const double t_whole = kFixedUs + std::max(tile_bytes / (kPerCtaGBs * 1e3), box);
      const double t_fill = kFixedUs + std::max(tile_bytes * tiles / (sms * kPerCtaGBs * 1e3), box) + kFillFixupUs;
      if (t_whole + 2.0 < t_fill) return tiles;
    }
    return std::max<long long>(1, std::min<long long>(std::min<long long>(sms, units), (units + 3) / 4));
  }
  constexpr double kPerSmGBs = 110.0, kHbmGBs = 6000.0, kFixupUs = 3.0, kLatencyUs = 2.0;
  const double tile_bytes = (double)bytes_per_kb * num_kb;
  long long best_g = std::min<long long>(tiles, sms);
  double best_t = 1e30;
  for (int s = 1; s <= std::max(1, num_kb); ++s) {
    const long long g = std::min<long long>((long long)tiles * s, sms);
    const double per_cta = tile_bytes * tiles / g;
    const double bw_us = std::max(per_cta / (kPerSmGBs * 1e3), tile_bytes * tiles / (kHbmGBs * 1e3));
    const double t = bw_us + kLatencyUs + (g > tiles ? kFixupUs : 0.0);
    if (t < best_t - 1e-9) {
      best_t = t;
      best_g = g;
    }
    if (g >= sms) break;
  }
  return std::max<long long>(1, best_g);
}

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
  GemmArgs a{};
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
  int bn;
  CUtensorMap ta, tb;
  if (swap) {
    TORCH_CHECK(T <= 128, "gemm_bf16: swapped mode supports at most 128 tokens");
    bn = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : 128;
    a.M = swiglu ? inter : Nw;
    a.N = T;
    a.m_tiles = (a.M + BM - 1) / BM;
    a.n_tiles = 1;
    ta = make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Nw, K, w.stride(0), BM,
                      BK, CU_TENSOR_MAP_SWIZZLE_128B);
    tb = make_tmap_2d(x.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, K, x.stride(0), bn,
                      BK, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    bn = (Nout >= 2048 || swiglu) ? 256 : 128;
    const int out_cols = swiglu ? bn / 2 : bn;
    a.M = T;
    a.N = Nout;
    a.m_tiles = (T + BM - 1) / BM;
    a.n_tiles = (Nout + out_cols - 1) / out_cols;
    ta = make_tmap_2d(x.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, K, x.stride(0), BM, BK,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    tb = make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Nw, K, w.stride(0),
                      swiglu ? bn / 2 : bn, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  const long long tiles = (long long)a.m_tiles * a.n_tiles;
  a.units = tiles * a.num_kb;
  // Persistent grid: one CTA per SM, fewer when the problem has little work per CTA.
  // force_splits > 0 caps the grid at tiles * force_splits (tests of the fix-up path).
  // Stream-K when the tiles alone cannot fill the SMs (decode shapes); otherwise whole
  // tiles in grouped raster order, which keeps the concurrently active tiles' operands
  // L2-resident.
  a.stream_k = (swap || tiles < 2LL * sms || force_splits > 0) ? 1 : 0;
  a.group_m = 16;
  long long g;
  if (a.stream_k) {
    const bool cluster = swap && split_reduce_cluster();
    bool use_cluster = false;
    g = stream_k_grid(tiles, a.num_kb, (long long)((swap && swiglu ? 2 : 1) * BM + bn) * BK * 2, sms,
                      cluster, &use_cluster);
    if (force_splits > 0) {
      g = std::max<long long>(1, std::min<long long>(a.units, tiles * force_splits));
      // Forced splits use clusters whenever a cluster of that size can be launched at all.
      use_cluster = cluster && g > tiles && g % tiles == 0 && g / tiles <= kMaxClusterSplit &&
                    max_active_clusters(static_cast<int>(g / tiles)) > 0;
    }
    // Whole tiles split into equal K ranges, one cluster per tile (each CTA owns exactly one
    // K range of one tile).
    if (use_cluster && g > tiles && g % tiles == 0 && g / tiles <= a.num_kb && g / tiles <= kMaxClusterSplit)
      a.split_s = static_cast<int>(g / tiles);
  } else {
    g = std::min<long long>(sms, tiles);
  }
  const long long acc_cols = (swap && swiglu ? 2 : 1) * bn;
  TORCH_CHECK(g * 2 * acc_cols * BM <= ws.numel(), "gemm_bf16: workspace too small");
  TORCH_CHECK(tiles <= counters.numel(), "gemm_bf16: counter array too small");
  a.grid = static_cast<int>(g);
  if (swap) {
    switch (epi) {
      case kEpiBf16: dispatch_swap<kEpiBf16>(bn, ta, tb, a, stream); break;
      case kEpiResAdd: dispatch_swap<kEpiResAdd>(bn, ta, tb, a, stream); break;
      case kEpiSwiGLU: dispatch_swap<kEpiSwiGLU>(bn, ta, tb, a, stream); break;
      case kEpiF32: dispatch_swap<kEpiF32>(bn, ta, tb, a, stream); break;
      default: TORCH_CHECK(false, "gemm_bf16: unknown epilogue");
    }
  } else {
    switch (epi) {
      case kEpiBf16: dispatch_normal<kEpiBf16>(bn, ta, tb, a, stream); break;
      case kEpiResAdd: dispatch_normal<kEpiResAdd>(bn, ta, tb, a, stream); break;
      case kEpiSwiGLU: dispatch_normal<kEpiSwiGLU>(bn, ta, tb, a, stream); break;
      case kEpiF32: dispatch_normal<kEpiF32>(bn, ta, tb, a, stream); break;
      default: TORCH_CHECK(false, "gemm_bf16: unknown epilogue");
    }
  }
}

}  // namespace sil

namespace sil {
using namespace gemm_detail;

// h[T, H] += sum over the tensor-parallel group of (x_r[T, K_r] . W_r[H, K_r]^T).
// One launch per rank: the tcgen05 GEMM computes this rank's partial, pushes it
// tile by tile into every rank's symmetric buffer over NVLink, then reduces the
// tiles it owns in rank order once all ranks have published them.
void gemm_allreduce(const at::Tensor& x, const at::Tensor& w, at::Tensor& h,
                    const std::vector<int64_t>& peers, int64_t rank, int64_t max_tiles,
                    int64_t max_tokens, int64_t max_hidden, int64_t flags_off, int64_t slots_off,
                    const at::Tensor& ws, const at::Tensor& counters, const at::Tensor& status) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  h.scalar_type() == at::kBFloat16,
              "gemm_allreduce: bf16 tensors");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && h.stride(1) == 1, "gemm_allreduce: rows");
  const int T = x.size(0), K = x.size(1), H = w.size(0);
  TORCH_CHECK(w.size(1) == K && h.size(0) == T && h.size(1) == H, "gemm_allreduce: shapes");
  const int size = static_cast<int>(peers.size());
  TORCH_CHECK(size >= 1 && size <= kMaxTP && rank >= 0 && rank < size, "gemm_allreduce: group");
  TORCH_CHECK(T <= max_tokens && T <= 128, "gemm_allreduce: too many tokens for the fused path");
  TORCH_CHECK(H <= max_hidden && (H + BM - 1) / BM <= max_tiles, "gemm_allreduce: hidden too large");
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  GemmArgs a{};
  a.num_kb = (K + BK - 1) / BK;
  a.inter = 0;
  a.out = h.data_ptr();
  a.ldo = h.stride(0);
  a.res = reinterpret_cast<const __nv_bfloat16*>(h.data_ptr());
  a.ldr = h.stride(0);
  a.ws = ws.data_ptr<float>();
  a.counters = counters.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.tp_rank = static_cast<int>(rank);
  a.tp_size = size;
  for (int i = 0; i < size; ++i) a.peers[i] = reinterpret_cast<uint8_t*>(peers[i]);
  a.flags_off = flags_off;
  a.slots_off = slots_off;
  a.max_tiles = static_cast<int>(max_tiles);
  a.max_tokens = static_cast<int>(max_tokens);
  a.max_hidden = static_cast<int>(max_hidden);
  const int bn = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : 128;
  a.M = H;
  a.N = T;
  a.m_tiles = (H + BM - 1) / BM;
  a.n_tiles = 1;
  a.units = (long long)a.m_tiles * a.num_kb;
  a.stream_k = 1;
  a.group_m = 16;
  const int sms = device_sm_count();
  long long g = stream_k_grid(a.m_tiles, a.num_kb, (long long)(BM + bn) * BK * 2, sms);
  TORCH_CHECK(g * 2 * bn * BM <= ws.numel(), "gemm_allreduce: workspace too small");
  TORCH_CHECK(a.m_tiles <= counters.numel(), "gemm_allreduce: counters too small");
  a.grid = static_cast<int>(g);
  CUtensorMap ta = make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, H, K,
                                w.stride(0), BM, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tmap_2d(x.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, T, K,
                                x.stride(0), bn, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  dispatch_swap<kEpiAllReduce>(bn, ta, tb, a, stream);
}

}  // namespace sil

namespace sil {
using namespace gemm_detail;

// Grouped GEMM over experts.  xp: [R, K] expert-sorted activation rows; group g
// owns rows [offsets[g], offsets[g+1]) (device int32, produced by moe_permute).
// w: stacked weights [G * Wr, K] (Wr = 2*inter for SwiGLU).  out: [R, Nout].
// `rows_hint` (expected rows per group) picks the operand order: swapped
// (weights as the MMA M side) for decode-sized groups.
void gemm_grouped(const at::Tensor& xp, const at::Tensor& w, at::Tensor& out,
                  const at::Tensor& offsets, int64_t num_groups, bool swiglu, int64_t rows_hint,
                  const at::Tensor& ws, const at::Tensor& counters, const at::Tensor& status) {
  TORCH_CHECK(xp.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16,
              "gemm_grouped: bf16 tensors");
  TORCH_CHECK(offsets.scalar_type() == at::kInt && offsets.numel() >= num_groups + 1,
              "gemm_grouped: int32 offsets [G+1]");
  TORCH_CHECK(num_groups >= 1 && num_groups <= kMaxGroups, "gemm_grouped: 1..1024 groups");
  const int R = xp.size(0), K = xp.size(1);
  TORCH_CHECK(w.size(1) == K && w.size(0) % num_groups == 0, "gemm_grouped: weight shape");
  const long long Wr = w.size(0) / num_groups;
  const int inter = swiglu ? static_cast<int>(Wr / 2) : 0;
  const int Nout = swiglu ? inter : static_cast<int>(Wr);
  TORCH_CHECK(!swiglu || inter % 128 == 0, "gemm_grouped: SwiGLU inter % 128");
  TORCH_CHECK(out.size(0) == R && out.size(1) == Nout, "gemm_grouped: output shape");
  if (R == 0) return;
  c10::cuda::CUDAGuard guard(xp.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  GemmArgs a{};
  a.num_kb = (K + BK - 1) / BK;
  a.inter = inter;
  a.out = out.data_ptr();
  a.ldo = out.stride(0);
  a.ws = ws.data_ptr<float>();
  a.counters = counters.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.grp_offsets = offsets.data_ptr<int>();
  a.num_groups = static_cast<int>(num_groups);
  a.w_group_rows = Wr;
  a.stream_k = 0;
  a.group_m = 16;
  const bool swap = rows_hint <= 64;
  int bn;
  CUtensorMap ta, tb;
  if (swap) {
    bn = rows_hint <= 16 ? 16 : rows_hint <= 32 ? 32 : 64;
    a.M = Nout;
    a.N = 0;  // per group
    a.m_tiles = (Nout + BM - 1) / BM;
    a.n_tiles = 1;
    ta = make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w.size(0), K, w.stride(0),
                      BM, BK, CU_TENSOR_MAP_SWIZZLE_128B);
    tb = make_tmap_2d(xp.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, R, K, xp.stride(0), bn, BK,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    bn = 256;
    const int out_cols = swiglu ? bn / 2 : bn;
    a.M = 0;  // per group
    a.N = Nout;
    a.m_tiles = 1;
    a.n_tiles = (Nout + out_cols - 1) / out_cols;
    ta = make_tmap_2d(xp.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, R, K, xp.stride(0), BM, BK,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    tb = make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w.size(0), K, w.stride(0),
                      swiglu ? bn / 2 : bn, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  a.units = 0;
  a.grid = device_sm_count();
  if (swiglu) dispatch_grouped<kEpiSwiGLU>(swap, bn, ta, tb, a, stream);
  else dispatch_grouped<kEpiBf16>(swap, bn, ta, tb, a, stream);
}

void set_pdl(bool on) { set_pdl_enabled(on); }

bool get_pdl() { return pdl_enabled(); }

}  // namespace sil
