// Python bindings of the sm_100a kernel library (module swarm_inference_lab_b200._C).
#include <torch/extension.h>

namespace sil {
void gemm_bf16(const at::Tensor& x, const at::Tensor& w, at::Tensor& out,
               const c10::optional<at::Tensor>& res, int64_t epi, const at::Tensor& ws,
               const at::Tensor& counters, const at::Tensor& status, int64_t force_mode,
               int64_t force_splits);
void paged_decode(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                  const at::Tensor& block_table, const at::Tensor& seq_lens, at::Tensor& out,
                  double scale, int64_t num_splits, const at::Tensor& ws,
                  const at::Tensor& counters, const at::Tensor& status);
void paged_prefill(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                   const at::Tensor& block_table, const at::Tensor& seq_lens,
                   const at::Tensor& cu_q, at::Tensor& out, double scale, int64_t max_q_len,
                   const at::Tensor& status);
void rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual,
             const c10::optional<at::Tensor>& residual_out, const at::Tensor& w, at::Tensor& y,
             double eps);
void rope_kv_write(at::Tensor& qkv, const at::Tensor& positions, const at::Tensor& slots,
                   const at::Tensor& cos_sin, const c10::optional<at::Tensor>& q_norm_w,
                   const c10::optional<at::Tensor>& k_norm_w, double eps, at::Tensor& k_cache,
                   at::Tensor& v_cache, int64_t Hq, int64_t Hkv);
void embedding(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out);
void argmax(const at::Tensor& logits, at::Tensor& out);
}  // namespace sil

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels: tcgen05 GEMM, paged attention, norms, RoPE, sampling";
  m.def("gemm_bf16", &sil::gemm_bf16, "tcgen05 bf16 GEMM with fused epilogue");
  m.def("paged_decode", &sil::paged_decode, "paged GQA decode attention (split-KV)");
  m.def("paged_prefill", &sil::paged_prefill, "paged causal prefill attention");
  m.def("rmsnorm", &sil::rmsnorm, "RMSNorm (+ residual add)");
  m.def("rope_kv_write", &sil::rope_kv_write, "q/k-norm + RoPE + paged KV write");
  m.def("embedding", &sil::embedding, "token embedding gather");
  m.def("argmax", &sil::argmax, "greedy argmax (lowest id on ties)");
}
