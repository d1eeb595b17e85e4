// Host entry of the tcgen05 bf16 GEMM (kernel template: gemm_bf16_impl.cuh).
#include "gemm_bf16_impl.cuh"

namespace sil {
using namespace gemm_detail;

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
