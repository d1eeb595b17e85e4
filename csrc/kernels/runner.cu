// Device-side "advance" of a captured decode step: after the step's token of every row is
// known, make the graph's static inputs describe the next step, so back-to-back replays
// need no host round trip and no ATen elementwise kernels.
//
// For each row b (valid rows only; padding rows keep slot -1):
//   out[b] = ids[b] = tok[b]
//   pos[b] += 1, seq_len[b] += 1
//   slot[b] = block_table[b][pos / 64] * 64 + pos % 64        (the next KV write)
//   sampling rows: philox offset[b] += 1, history[b][hist_len[b]++] = tok[b]
//
// One CTA; a decode batch is at most 128 rows.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sil/host.h"
#include "sil/ptx.cuh"

namespace sil {
namespace {

constexpr int kPage = 64;

struct AdvanceArgs {
  const long long* tok;
  long long* ids;
  long long* out;
  int* pos;
  int* slot;
  int* seq_len;
  const bool* valid;
  const int* block_table;
  int bt_stride, max_pages, bsz;
  long long* offsets;   // null: no sampling state
  long long* history;   // [bsz, hmax] or null
  int* hist_len;
  int hmax;
};

__global__ void decode_advance_kernel(const AdvanceArgs a) {
  pdl_trigger();
  pdl_wait();  // the step's tokens come from the previous kernel
  for (int b = threadIdx.x; b < a.bsz; b += blockDim.x) {
    const long long t = a.tok[b];
    a.out[b] = t;
    a.ids[b] = t;
    if (!a.valid[b]) {
      a.slot[b] = -1;
      continue;
    }
    const int p = a.pos[b] + 1;
    a.pos[b] = p;
    a.seq_len[b] += 1;
    const int pg = min(p / kPage, a.max_pages - 1);
    a.slot[b] = a.block_table[(long long)b * a.bt_stride + pg] * kPage + p % kPage;
    if (a.offsets != nullptr) a.offsets[b] += 1;
    if (a.history != nullptr) {
      const int n = a.hist_len[b];
      if (n < a.hmax) {
        a.history[(long long)b * a.hmax + n] = t;
        a.hist_len[b] = n + 1;
      }
    }
  }
}

}  // namespace

// tok [bsz] int64; ids/out [bsz] int64; meta [3, bsz] int32 (positions, slots, seq lens);
// valid [bsz] bool; block_table [bsz, max_pages] int32; optional sampling state.
void decode_advance(const at::Tensor& tok, at::Tensor& ids, at::Tensor& out, at::Tensor& meta,
                    const at::Tensor& valid, const at::Tensor& block_table,
                    const c10::optional<at::Tensor>& offsets, const c10::optional<at::Tensor>& history,
                    const c10::optional<at::Tensor>& hist_len) {
  const int bsz = static_cast<int>(ids.size(0));
  TORCH_CHECK(tok.scalar_type() == at::kLong && ids.scalar_type() == at::kLong &&
                  out.scalar_type() == at::kLong && tok.numel() >= bsz && out.numel() >= bsz,
              "decode_advance: int64 tokens");
  TORCH_CHECK(meta.scalar_type() == at::kInt && meta.dim() == 2 && meta.size(0) == 3 &&
                  meta.size(1) == bsz && meta.is_contiguous(),
              "decode_advance: meta [3, bsz] int32");
  TORCH_CHECK(valid.scalar_type() == at::kBool && valid.numel() == bsz, "decode_advance: valid [bsz]");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.dim() == 2 &&
                  block_table.size(0) == bsz && block_table.stride(1) == 1,
              "decode_advance: block table [bsz, pages] int32");
  if (bsz == 0) return;
  c10::cuda::CUDAGuard guard(ids.device());
  AdvanceArgs a{};
  a.tok = reinterpret_cast<const long long*>(tok.data_ptr<int64_t>());
  a.ids = reinterpret_cast<long long*>(ids.data_ptr<int64_t>());
  a.out = reinterpret_cast<long long*>(out.data_ptr<int64_t>());
  int* m = meta.data_ptr<int>();
  a.pos = m;
  a.slot = m + bsz;
  a.seq_len = m + 2 * bsz;
  a.valid = valid.data_ptr<bool>();
  a.block_table = block_table.data_ptr<int>();
  a.bt_stride = static_cast<int>(block_table.stride(0));
  a.max_pages = static_cast<int>(block_table.size(1));
  a.bsz = bsz;
  if (offsets.has_value() && offsets->defined()) {
    TORCH_CHECK(offsets->scalar_type() == at::kLong && offsets->numel() >= bsz, "decode_advance: offsets");
    a.offsets = reinterpret_cast<long long*>(offsets->data_ptr<int64_t>());
  }
  if (history.has_value() && history->defined()) {
    TORCH_CHECK(history->scalar_type() == at::kLong && history->dim() == 2 && history->size(0) == bsz &&
                    history->is_contiguous() && hist_len.has_value() &&
                    hist_len->scalar_type() == at::kInt && hist_len->numel() >= bsz,
                "decode_advance: history [bsz, hmax] int64 + int32 lengths");
    a.history = reinterpret_cast<long long*>(history->data_ptr<int64_t>());
    a.hist_len = hist_len->data_ptr<int>();
    a.hmax = static_cast<int>(history->size(1));
  }
  launch_pdl(decode_advance_kernel, dim3(1), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
             "decode_advance launch", a);
}

}  // namespace sil
