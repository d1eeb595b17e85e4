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
             double eps, const c10::optional<at::Tensor>& yq, const c10::optional<at::Tensor>& ys);
void rope_kv_write(at::Tensor& qkv, const at::Tensor& positions, const at::Tensor& slots,
                   const at::Tensor& cos_sin, const c10::optional<at::Tensor>& q_norm_w,
                   const c10::optional<at::Tensor>& k_norm_w, double eps, at::Tensor& k_cache,
                   at::Tensor& v_cache, int64_t Hq, int64_t Hkv);
void embedding(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out);
void gemm_allreduce(const at::Tensor& x, const at::Tensor& w, at::Tensor& h,
                    const std::vector<int64_t>& peers, int64_t rank, int64_t max_tiles,
                    int64_t max_tokens, int64_t max_hidden, int64_t flags_off, int64_t slots_off,
                    const at::Tensor& ws, const at::Tensor& counters, const at::Tensor& status);
int64_t symm_alloc(int64_t bytes, int64_t device);
void gemm_fp8(const at::Tensor& xq, const at::Tensor& xs, const at::Tensor& wq, const at::Tensor& wsc,
              at::Tensor& out, const c10::optional<at::Tensor>& res, int64_t epi,
              const at::Tensor& ws, const at::Tensor& counters, const at::Tensor& status);
void gemm_fp8_grouped(const at::Tensor& xq, const at::Tensor& xs, const at::Tensor& wq,
                      const at::Tensor& wsc, at::Tensor& out, const at::Tensor& offsets,
                      int64_t num_groups, bool swiglu, int64_t rows_hint, const at::Tensor& ws,
                      const at::Tensor& counters, const at::Tensor& status);
void quant_fp8_1x128(const at::Tensor& x, at::Tensor& q, at::Tensor& s);
void sample_tokens(at::Tensor& logits, const at::Tensor& temperature, const at::Tensor& top_k,
                   const at::Tensor& top_p, const at::Tensor& penalty,
                   const c10::optional<at::Tensor>& history,
                   const c10::optional<at::Tensor>& history_len, const at::Tensor& seeds,
                   const at::Tensor& offsets, at::Tensor& out);
void gemm_grouped(const at::Tensor& xp, const at::Tensor& w, at::Tensor& out,
                  const at::Tensor& offsets, int64_t num_groups, bool swiglu, int64_t rows_hint,
                  const at::Tensor& ws, const at::Tensor& counters, const at::Tensor& status);
void moe_topk(const at::Tensor& logits, int64_t k, int64_t mode, bool renorm,
              const c10::optional<at::Tensor>& bias, int64_t n_group, int64_t topk_group,
              double scale, at::Tensor& ids, at::Tensor& weights);
void moe_permute(const at::Tensor& ids, int64_t E, at::Tensor& offsets, at::Tensor& rows,
                 const c10::optional<at::Tensor>& counts);
void moe_gather(const at::Tensor& x, const at::Tensor& rows, int64_t k, at::Tensor& xp);
void moe_combine(const at::Tensor& y, const at::Tensor& rows, const at::Tensor& w, int64_t k,
                 const c10::optional<at::Tensor>& res, const c10::optional<at::Tensor>& shared,
                 at::Tensor& out, const c10::optional<at::Tensor>& row_limit);
void symm_free(int64_t ptr);
std::string ipc_handle(int64_t ptr);
int64_t ipc_open(const std::string& handle, int64_t device);
void ipc_close(int64_t ptr);
bool can_access_peer(int64_t dev, int64_t peer);
void argmax(const at::Tensor& logits, at::Tensor& out);
void mla_attention(const at::Tensor& q_lat, const at::Tensor& q_pe, const at::Tensor& cache,
                   const at::Tensor& block_table, const at::Tensor& seq_lens,
                   const c10::optional<at::Tensor>& cu_q, at::Tensor& out, double scale,
                   int64_t max_q_len, int64_t num_splits, const at::Tensor& ws,
                   const at::Tensor& counters, const at::Tensor& status);
void mla_kv_write(const at::Tensor& kv, const at::Tensor& norm_w, double eps,
                  const at::Tensor& positions, const at::Tensor& slots, const at::Tensor& cos_sin,
                  at::Tensor& cache);
void mla_q_prep(const at::Tensor& q, const at::Tensor& positions, const at::Tensor& cos_sin,
                at::Tensor& q_nope, at::Tensor& q_pe, int64_t H);
void mla_heads_to_tokens(const at::Tensor& src, at::Tensor& dst, int64_t T, int64_t H);
void ep_dispatch(const at::Tensor& x, const at::Tensor& ids, const at::Tensor& wts,
                 const std::vector<int64_t>& peers, int64_t rank, int64_t e0, int64_t el,
                 const std::vector<int64_t>& offs, const at::Tensor& status);
void ep_recv_map(at::Tensor& local_ids, const std::vector<int64_t>& peers, int64_t rank, int64_t T,
                 int64_t k, int64_t H, int64_t e0, int64_t el, const std::vector<int64_t>& offs,
                 const at::Tensor& status);
void ep_gather(const at::Tensor& pos, const at::Tensor& offsets, at::Tensor& xq, at::Tensor& xs,
               at::Tensor& inv, const std::vector<int64_t>& peers, int64_t rank, int64_t T, int64_t k,
               int64_t H, int64_t e0, int64_t el, const std::vector<int64_t>& offs,
               const at::Tensor& status);
void ep_combine(at::Tensor& h, const std::vector<int64_t>& peers, int64_t rank, int64_t k,
                int64_t e0, int64_t el, const std::vector<int64_t>& offs, const at::Tensor& status);
void gemm_fp8_grouped_scatter(const at::Tensor& xq, const at::Tensor& xs, const at::Tensor& wq,
                              const at::Tensor& wsc, const at::Tensor& offsets, int64_t num_groups,
                              int64_t rows_hint, const at::Tensor& sorted_rows,
                              const std::vector<int64_t>& peers, int64_t rank, int64_t T, int64_t k,
                              int64_t e0, const std::vector<int64_t>& offs, const at::Tensor& ws,
                              const at::Tensor& counters, const at::Tensor& status);
void set_pdl(bool on);
bool get_pdl();
void oneshot_allreduce(at::Tensor& h, const std::vector<int64_t>& peers, int64_t rank,
                       int64_t flags_off, int64_t recv_off, int64_t partial_off, int64_t max_elems,
                       const at::Tensor& status);
void oneshot_allreduce_norm(at::Tensor& h, const std::vector<int64_t>& peers, int64_t rank,
                            int64_t flags_off, int64_t recv_off, int64_t partial_off, int64_t max_elems,
                            const at::Tensor& norm_w, double eps, at::Tensor& x_out,
                            const at::Tensor& status);
at::Tensor symm_tensor(int64_t ptr, int64_t offset, int64_t rows, int64_t cols, int64_t device);
void paged_prefill_tc(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                      const at::Tensor& block_table, const at::Tensor& seq_lens,
                      const at::Tensor& cu_q, at::Tensor& out, double scale, int64_t max_q_len,
                      const at::Tensor& status);
void decode_advance(const at::Tensor& tok, at::Tensor& ids, at::Tensor& out, at::Tensor& meta,
                    const at::Tensor& valid, const at::Tensor& block_table,
                    const c10::optional<at::Tensor>& offsets, const c10::optional<at::Tensor>& history,
                    const c10::optional<at::Tensor>& hist_len);
void ll_argmax_exchange(const at::Tensor& logits, const at::Tensor& idx, int64_t vocab_start,
                        const std::vector<int64_t>& peers, int64_t rank, int64_t slot_off,
                        int64_t max_rows, at::Tensor& out, const at::Tensor& status);
void ll_allreduce_norm(at::Tensor& h, const std::vector<int64_t>& peers, int64_t rank,
                       int64_t ll_off, int64_t partial_off, int64_t max_elems,
                       const c10::optional<at::Tensor>& norm_w, double eps,
                       const c10::optional<at::Tensor>& x_out, const at::Tensor& status,
                       bool two_shot);
void nvls_allreduce(at::Tensor& h, const std::vector<int64_t>& peers, int64_t mc, int64_t rank,
                    int64_t flags1_off, int64_t flags2_off, int64_t partial_off, int64_t sum_off,
                    int64_t max_elems, const c10::optional<at::Tensor>& norm_w, double eps,
                    const c10::optional<at::Tensor>& x_out, const at::Tensor& status);
}  // namespace sil

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels: tcgen05 GEMM, paged attention, norms, RoPE, sampling";
  m.def("gemm_bf16", &sil::gemm_bf16, "tcgen05 bf16 GEMM with fused epilogue");
  m.def("paged_decode", &sil::paged_decode, "paged GQA decode attention (split-KV)");
  m.def("paged_prefill", &sil::paged_prefill, "paged causal prefill attention (mma.sync)");
  m.def("paged_prefill_tc", &sil::paged_prefill_tc,
        "paged causal prefill attention on tcgen05 (S and O accumulators in TMEM)");
  m.def("rmsnorm", &sil::rmsnorm, "RMSNorm (+ residual add)");
  m.def("rope_kv_write", &sil::rope_kv_write, "q/k-norm + RoPE + paged KV write");
  m.def("embedding", &sil::embedding, "token embedding gather");
  m.def("argmax", &sil::argmax, "greedy argmax (lowest id on ties)");
  m.def("gemm_allreduce", &sil::gemm_allreduce,
        "tcgen05 GEMM fused with a one-shot all-reduce over NVLink peer memory (+ residual)");
  m.def("gemm_grouped", &sil::gemm_grouped, "grouped (per-expert) tcgen05 GEMM");
  m.def("moe_topk", &sil::moe_topk, "router top-k (softmax or sigmoid+bias+group)");
  m.def("moe_permute", &sil::moe_permute, "expert counts, offsets and sorted rows");
  m.def("moe_gather", &sil::moe_gather, "gather token rows into expert order");
  m.def("moe_combine", &sil::moe_combine, "weighted combine of expert outputs");
  m.def("sample_tokens", &sil::sample_tokens,
        "penalty + temperature + top-k + top-p + Gumbel-max sampling (Philox)");
  m.def("gemm_fp8", &sil::gemm_fp8, "block-scaled e4m3 tcgen05 GEMM (128x128 / 1x128 scales)");
  m.def("gemm_fp8_grouped", &sil::gemm_fp8_grouped, "grouped block-scaled e4m3 GEMM (experts)");
  m.def("quant_fp8_1x128", &sil::quant_fp8_1x128, "bf16 -> e4m3 with 1x128 block scales");
  m.def("symm_alloc", &sil::symm_alloc, "allocate a zeroed buffer for peer (IPC) sharing");
  m.def("symm_free", &sil::symm_free, "free a symmetric buffer");
  m.def("ipc_handle", [](int64_t p) { return pybind11::bytes(sil::ipc_handle(p)); },
        "CUDA IPC handle bytes of a symmetric buffer");
  m.def("ipc_open", &sil::ipc_open, "open a peer's IPC handle; returns a device pointer");
  m.def("ipc_close", &sil::ipc_close, "close a peer mapping");
  m.def("mla_attention", &sil::mla_attention, "MLA paged attention over the latent cache (absorbed form)");
  m.def("mla_kv_write", &sil::mla_kv_write, "MLA latent KV write: RMSNorm(c_kv) + interleaved RoPE(k_pe)");
  m.def("mla_q_prep", &sil::mla_q_prep, "MLA query split: q_nope head-major + RoPE(q_pe)");
  m.def("mla_heads_to_tokens", &sil::mla_heads_to_tokens, "[H, T, 128] -> [T, H*128]");
  m.def("ep_dispatch", &sil::ep_dispatch, "EP dispatch: e4m3 quantise + push rows/routing to every rank");
  m.def("ep_recv_map", &sil::ep_recv_map, "EP: wait for every source, map expert ids to local groups");
  m.def("ep_gather", &sil::ep_gather, "EP: received e4m3 rows into expert order");
  m.def("ep_combine", &sil::ep_combine, "EP: wait for every owner, sum combine slots into h");
  m.def("gemm_fp8_grouped_scatter", &sil::gemm_fp8_grouped_scatter,
        "grouped fp8 GEMM with the weighted EP combine scattered to the token owners");
  m.def("set_pdl", &sil::set_pdl, "enable / disable programmatic dependent launch for later launches");
  m.def("get_pdl", &sil::get_pdl, "whether programmatic dependent launch is enabled");
  m.def("oneshot_allreduce", &sil::oneshot_allreduce,
        "one-shot all-reduce of symmetric-buffer partials into h (NVLink pull, per-CTA barriers)");
  m.def("oneshot_allreduce_norm", &sil::oneshot_allreduce_norm,
        "one-shot all-reduce into h fused with the next RMSNorm (x_out = rmsnorm(h) * w)");
  m.def("nvls_allreduce", &sil::nvls_allreduce,
        "two-shot all-reduce through NVSwitch multicast into h, optionally fused with the next RMSNorm");
  m.def("decode_advance", &sil::decode_advance,
        "advance a captured decode step's static inputs (ids, positions, slots, lengths, "
        "sampling offsets and history) from the step's tokens");
  m.def("ll_argmax_exchange", &sil::ll_argmax_exchange,
        "distributed greedy selection over a vocabulary-parallel LM head (peer-memory words "
        "carrying their epoch; lowest global id on ties)");
  m.def("ll_allreduce_norm", &sil::ll_allreduce_norm,
        "one-shot all-reduce with the flag inside every 8-byte word (no fence, no flag round "
        "trip) into h, optionally fused with the next RMSNorm");
  m.def("symm_tensor", &sil::symm_tensor, "bf16 tensor view over a symmetric buffer (no ownership)");
  m.def("can_access_peer", &sil::can_access_peer, "cudaDeviceCanAccessPeer");
}
