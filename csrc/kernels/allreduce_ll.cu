// Low-latency one-shot all-reduce (+ residual add + next RMSNorm) over NVLink peer memory
// for decode-sized tensor-parallel sums.
//
// The flag travels inside the data: every 8-byte word a rank sends is {bf16x2 payload,
// epoch}, written with 16-byte vector stores (two words) straight into the receiver's
// buffer.  An 8-byte aligned word is written as a unit, so a receiver that reads a word
// whose epoch half equals the current epoch also holds that word's payload - no
// system-scope fence, no separate flag store and no flag round trip.  The price is twice
// the bytes of a plain push, which at decode sizes (256 KB per rank at 32 tokens x 4096)
// is far below the latency it saves.
//
// Symmetric buffer of every rank (CUDA IPC, mapped by every peer):
//
//   [0, 256)                       state: epoch (u32), arrival counter (u32); local use
//   ll[2][8][max_elems / 2]        u64 words {bf16x2, epoch}: slot [parity][source rank]
//   partial[T][H]                  bf16, this rank's row-parallel GEMM output (the GEMM
//                                  writes it there directly)
//
// One CTA per token row, one thread per 8 consecutive elements of the row:
//   1. read its 8 elements of the local partial and send them, as two 16-byte words with
//      the epoch, to ll[parity][rank] of every peer;
//   2. for every rank in order, read the words of that rank from its own ll[parity][r]
//      until both epochs match (bounded wait), and add them in rank order (the local
//      partial for its own term; fp32; the same order on every rank, so every rank gets
//      bit-identical sums);
//   3. add the residual row, store it, and (when a norm weight is given) write the next
//      block's input rmsnorm(h) * w.
// Two-shot variant (reduce-scatter + all-gather, for larger groups): the row splits into
// `world` equal slices and rank o owns slice o.  A thread whose 8 elements lie in another
// rank's slice sends them to that owner only (ll[parity][rank] of the owner) and then waits
// for the owner's finished values in ll[parity][owner] of its own buffer; an owning thread
// sums every rank's words for its elements in rank order, adds the residual and sends the
// bf16 result to every peer.  Each rank sends 2 x (world-1)/world of a row per token instead
// of (world-1) rows, at the cost of a second NVLink crossing; the sums are the same fp32
// rank-ordered sums, so both variants give bit-identical results.  The reduce-scatter words
// a rank receives sit in its own slice's positions and the all-gather words in the other
// slices' positions, so the two share the slots without overlap.
// Slots alternate by epoch parity.  A peer can only write epoch e+2 into the parity a
// reader uses at epoch e after it has received the reader's epoch e+1 words, which the
// reader sends after it finished reading epoch e, so no second exchange is needed.  No
// block of a launch waits for another block of the same launch; every wait is bounded and
// reports through the sticky status word.  The last CTA advances the epoch.
//
// Reference semantics: the rank-ordered deterministic all-reduce of row-parallel
// projections, si/microsharding/dense.py:600-708.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "sil/host.h"
#include "sil/ptx.cuh"

namespace sil {
namespace {

constexpr int kLLMaxRanks = 8;

struct LLArgs {
  long long peers[kLLMaxRanks];
  int rank, world;
  long long ll_off, partial_off;
  long long max_elems;
  __nv_bfloat16* h;                // [T, H] residual stream, updated in place
  int H;
  const __nv_bfloat16* norm_w;     // null: no norm
  float eps;
  __nv_bfloat16* x_out;            // [T, H] rmsnorm(h) * norm_w
  int* status;
};

__device__ __forceinline__ void st_vol_v4(uint4* p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 ld_vol_v4(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// 16-byte words of slot [par][src] in rank `owner`'s buffer.
__device__ __forceinline__ uint4* ll_slot(const LLArgs& a, int owner, int par, int src) {
  return reinterpret_cast<uint4*>(a.peers[owner] + a.ll_off) +
         ((long long)par * kLLMaxRanks + src) * (a.max_elems / 4);
}

// Polls the two 16-byte LL words at `src` until both carry `epoch` (bounded by the status
// word's limit); false when the wait gave up.
__device__ __forceinline__ bool ll_recv(const uint4* src, uint32_t epoch, uint64_t limit,
                                        int* status, uint4& v0, uint4& v1) {
  v0 = ld_vol_v4(src);
  v1 = ld_vol_v4(src + 1);
  if (v0.y == epoch && v0.w == epoch && v1.y == epoch && v1.w == epoch) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (v0.y != epoch || v0.w != epoch || v1.y != epoch || v1.w != epoch) {
    if ((++it & 255u) == 0 && (load_status(status) != 0 || globaltimer_ns() - t0 > limit)) {
      raise_status(status, kStatusTimeoutPeer);
      return false;
    }
    v0 = ld_vol_v4(src);
    v1 = ld_vol_v4(src + 1);
  }
  return true;
}

template <bool kTwoShot>
__global__ void __launch_bounds__(1024) ll_allreduce_norm_kernel(const LLArgs a) {
  __shared__ float red[32];
  __shared__ int s_ok;
  pdl_trigger();
  pdl_wait();  // the partial comes from the previous kernel (the row-parallel GEMM)
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(a.peers[a.rank]) + 1u;
  const int par = epoch & 1;
  const int t = blockIdx.x;
  const int units = a.H / 8;
  const int u = threadIdx.x;
  if (threadIdx.x == 0) s_ok = load_status(a.status) == 0;
  __syncthreads();
  const bool active = u < units && s_ok;
  const long long widx = ((long long)t * units + u) * 2;  // first 16-byte LL word
  bool ok = true;
  uint4 o = make_uint4(0, 0, 0, 0);  // this thread's 8 elements of the new residual row
  if (active) {
    const uint4 mine =
        reinterpret_cast<const uint4*>(a.peers[a.rank] + a.partial_off)[(long long)t * units + u];
    const uint4 w0 = make_uint4(mine.x, epoch, mine.y, epoch);
    const uint4 w1 = make_uint4(mine.z, epoch, mine.w, epoch);
    const uint64_t limit = wait_limit_ns(a.status);
    const int owner = kTwoShot ? u / (units / a.world) : a.rank;
    if (kTwoShot && owner != a.rank) {
      uint4* dst = ll_slot(a, owner, par, a.rank) + widx;  // reduce-scatter: to the owner only
      st_vol_v4(dst, w0);
      st_vol_v4(dst + 1, w1);
      uint4 v0, v1;  // all-gather: the owner's finished values
      ok = ll_recv(ll_slot(a, a.rank, par, owner) + widx, epoch, limit,
                   a.status, v0, v1);
      o = make_uint4(v0.x, v0.z, v1.x, v1.z);
    } else {
      if (!kTwoShot) {
#pragma unroll
        for (int p = 0; p < kLLMaxRanks; ++p) {
          if (p < a.world && p != a.rank) {
            uint4* dst = ll_slot(a, p, par, a.rank) + widx;
            st_vol_v4(dst, w0);
            st_vol_v4(dst + 1, w1);
          }
        }
      }
      float s[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j] = 0.f;
#pragma unroll 1
      for (int p = 0; p < a.world && ok; ++p) {
        uint4 v0 = w0, v1 = w1;
        if (p != a.rank) ok = ll_recv(ll_slot(a, a.rank, par, p) + widx, epoch, limit, a.status, v0, v1);
        if (!ok) break;
        s[0] += bf16_lo(v0.x); s[1] += bf16_hi(v0.x);
        s[2] += bf16_lo(v0.z); s[3] += bf16_hi(v0.z);
        s[4] += bf16_lo(v1.x); s[5] += bf16_hi(v1.x);
        s[6] += bf16_lo(v1.z); s[7] += bf16_hi(v1.z);
      }
      if (ok) {
        const uint4 r = reinterpret_cast<const uint4*>(a.h)[(long long)t * units + u];
        o.x = pack_bf16x2(bf16_lo(r.x) + s[0], bf16_hi(r.x) + s[1]);
        o.y = pack_bf16x2(bf16_lo(r.y) + s[2], bf16_hi(r.y) + s[3]);
        o.z = pack_bf16x2(bf16_lo(r.z) + s[4], bf16_hi(r.z) + s[5]);
        o.w = pack_bf16x2(bf16_lo(r.w) + s[6], bf16_hi(r.w) + s[7]);
        if (kTwoShot) {  // all-gather: the finished slice to every peer
          const uint4 g0 = make_uint4(o.x, epoch, o.y, epoch);
          const uint4 g1 = make_uint4(o.z, epoch, o.w, epoch);
#pragma unroll
          for (int p = 0; p < kLLMaxRanks; ++p) {
            if (p < a.world && p != a.rank) {
              uint4* dst = ll_slot(a, p, par, a.rank) + widx;
              st_vol_v4(dst, g0);
              st_vol_v4(dst + 1, g1);
            }
          }
        }
      }
    }
  }
  if (active && !ok) s_ok = 0;
  __syncthreads();
  const bool write = active && s_ok;
  float ss = 0.f;
  float hv[8];
  if (write) {
    reinterpret_cast<uint4*>(a.h)[(long long)t * units + u] = o;
    // The norm sees the bf16-rounded residual stream, as the unfused RMSNorm would.
    hv[0] = bf16_lo(o.x); hv[1] = bf16_hi(o.x); hv[2] = bf16_lo(o.y); hv[3] = bf16_hi(o.y);
    hv[4] = bf16_lo(o.z); hv[5] = bf16_hi(o.z); hv[6] = bf16_lo(o.w); hv[7] = bf16_hi(o.w);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += hv[j] * hv[j];
  }
  if (a.norm_w != nullptr) {
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
      v = warp_sum(v);
      if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float rstd = rsqrtf(red[0] / a.H + a.eps);
    if (write) {
      const uint4 wq = reinterpret_cast<const uint4*>(a.norm_w)[u];
      const float wv[8] = {bf16_lo(wq.x), bf16_hi(wq.x), bf16_lo(wq.y), bf16_hi(wq.y),
                           bf16_lo(wq.z), bf16_hi(wq.z), bf16_lo(wq.w), bf16_hi(wq.w)};
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = wv[j] * __bfloat162float(__float2bfloat16_rn(hv[j] * rstd));
      uint4 q;
      q.x = pack_bf16x2(o[0], o[1]); q.y = pack_bf16x2(o[2], o[3]);
      q.z = pack_bf16x2(o[4], o[5]); q.w = pack_bf16x2(o[6], o[7]);
      reinterpret_cast<uint4*>(a.x_out)[(long long)t * units + u] = q;
    }
  }
  // Advance the epoch once every CTA of this launch has read it.
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* st = reinterpret_cast<uint32_t*>(a.peers[a.rank]);
    if (atomicAdd(st + 1, 1u) == gridDim.x - 1) {
      st[1] = 0u;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(st) = epoch;
    }
  }
}

// Distributed greedy selection over a vocabulary-parallel LM head: every rank holds the
// argmax of its vocabulary shard per row; each rank sends {value, epoch, global id, epoch}
// (one 16-byte word) per row to every peer and picks, per row, the largest value over the
// ranks with the lowest global id on ties -- the same answer on every rank.  Its own epoch
// counter lives at byte 8 of the state block.
__global__ void __launch_bounds__(128) ll_argmax_exchange_kernel(
    const LLArgs a, const float* __restrict__ logits, long long ld, const long long* __restrict__ idx,
    long long vocab_start, int rows, long long slot_off, long long* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  uint32_t* st = reinterpret_cast<uint32_t*>(a.peers[a.rank]) + 2;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(st) + 1u;
  const int par = epoch & 1;
  const uint64_t limit = wait_limit_ns(a.status);
  bool ok = load_status(a.status) == 0;
  for (int r = threadIdx.x; r < rows && ok; r += blockDim.x) {
    const long long li = idx[r];
    const float v = logits[(long long)r * ld + li];
    const uint32_t gid = static_cast<uint32_t>(vocab_start + li);
    const uint4 w = make_uint4(__float_as_uint(v), epoch, gid, epoch);
    for (int p = 0; p < a.world; ++p) {
      if (p == a.rank) continue;
      uint4* dst = reinterpret_cast<uint4*>(a.peers[p] + slot_off) +
                   ((long long)par * kLLMaxRanks + a.rank) * a.max_elems + r;
      st_vol_v4(dst, w);
    }
    float best = v;
    uint32_t best_id = gid;
    for (int p = 0; p < a.world; ++p) {
      if (p == a.rank) continue;
      const uint4* src = reinterpret_cast<const uint4*>(a.peers[a.rank] + slot_off) +
                         ((long long)par * kLLMaxRanks + p) * a.max_elems + r;
      uint4 q = ld_vol_v4(src);
      if (q.y != epoch || q.w != epoch) {
        const uint64_t t0 = globaltimer_ns();
        uint32_t it = 0;
        while (q.y != epoch || q.w != epoch) {
          if ((++it & 255u) == 0 && (load_status(a.status) != 0 || globaltimer_ns() - t0 > limit)) {
            raise_status(a.status, kStatusTimeoutPeer);
            ok = false;
            break;
          }
          q = ld_vol_v4(src);
        }
        if (!ok) break;
      }
      const float qv = __uint_as_float(q.x);
      if (qv > best || (qv == best && q.z < best_id)) {
        best = qv;
        best_id = q.z;
      }
    }
    if (ok) out[r] = best_id;
  }
  __syncthreads();
  if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(st) = epoch;
}

}  // namespace

// out[r] = global id of the largest logit of row r over every rank's vocabulary shard
// (lowest id on ties); idx holds this rank's local argmax per row.
void ll_argmax_exchange(const at::Tensor& logits, const at::Tensor& idx, int64_t vocab_start,
                        const std::vector<int64_t>& peers, int64_t rank, int64_t slot_off,
                        int64_t max_rows, at::Tensor& out, const at::Tensor& status) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1,
              "ll_argmax_exchange: fp32 logits [B, V]");
  TORCH_CHECK(idx.scalar_type() == at::kLong && out.scalar_type() == at::kLong,
              "ll_argmax_exchange: int64 ids");
  const int world = static_cast<int>(peers.size());
  const int B = static_cast<int>(logits.size(0));
  TORCH_CHECK(world >= 1 && world <= kLLMaxRanks && rank >= 0 && rank < world && B <= max_rows &&
                  idx.numel() >= B && out.numel() >= B && slot_off % 16 == 0,
              "ll_argmax_exchange: group / rows");
  if (B == 0) return;
  c10::cuda::CUDAGuard guard(logits.device());
  LLArgs a{};
  for (int i = 0; i < world; ++i) a.peers[i] = peers[i];
  a.rank = static_cast<int>(rank);
  a.world = world;
  a.max_elems = max_rows;  // 16-byte words per (parity, source) slot
  a.status = status.data_ptr<int>();
  launch_pdl(ll_argmax_exchange_kernel, dim3(1), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
             "ll_argmax_exchange launch", a, logits.data_ptr<float>(), (long long)logits.stride(0),
             reinterpret_cast<const long long*>(idx.data_ptr<int64_t>()), (long long)vocab_start, B,
             (long long)slot_off, reinterpret_cast<long long*>(out.data_ptr<int64_t>()));
}

// h [T, H] += sum over ranks of each rank's partial (bf16 at byte offset partial_off of its
// symmetric buffer); with norm_w defined also x_out = rmsnorm(h) * norm_w.  two_shot picks
// the reduce-scatter + all-gather exchange (H / 8 must be a multiple of the group size).
void ll_allreduce_norm(at::Tensor& h, const std::vector<int64_t>& peers, int64_t rank,
                       int64_t ll_off, int64_t partial_off, int64_t max_elems,
                       const c10::optional<at::Tensor>& norm_w, double eps,
                       const c10::optional<at::Tensor>& x_out, const at::Tensor& status,
                       bool two_shot) {
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous() && h.dim() == 2,
              "ll_allreduce_norm: h [T, H] bf16 contiguous");
  const int world = static_cast<int>(peers.size());
  TORCH_CHECK(world >= 1 && world <= kLLMaxRanks && rank >= 0 && rank < world,
              "ll_allreduce_norm: group of 1..8 ranks");
  const int T = h.size(0), H = h.size(1);
  TORCH_CHECK(H % 8 == 0 && H / 8 <= 1024, "ll_allreduce_norm: H must be a multiple of 8, <= 8192");
  TORCH_CHECK(!two_shot || (H / 8) % world == 0,
              "ll_allreduce_norm: two-shot needs H / 8 to be a multiple of the group size");
  TORCH_CHECK((long long)T * H <= max_elems && max_elems % 8 == 0,
              "ll_allreduce_norm: T * H exceeds the buffer");
  TORCH_CHECK(ll_off % 16 == 0 && partial_off % 16 == 0 &&
                  (reinterpret_cast<uintptr_t>(h.data_ptr()) & 15) == 0,
              "ll_allreduce_norm: 16-byte alignment");
  TORCH_CHECK(status.numel() >= 4 && status.scalar_type() == at::kInt, "ll_allreduce_norm: status block");
  const bool with_norm = norm_w.has_value() && norm_w->defined();
  if (with_norm) {
    TORCH_CHECK(norm_w->numel() == H && norm_w->scalar_type() == at::kBFloat16 && norm_w->is_contiguous(),
                "ll_allreduce_norm: norm weight [H] bf16");
    TORCH_CHECK(x_out.has_value() && x_out->defined() && x_out->sizes() == h.sizes() &&
                    x_out->scalar_type() == at::kBFloat16 && x_out->is_contiguous(),
                "ll_allreduce_norm: x_out like h");
  }
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(h.device());
  LLArgs a{};
  for (int i = 0; i < world; ++i) a.peers[i] = peers[i];
  a.rank = static_cast<int>(rank);
  a.world = world;
  a.ll_off = ll_off;
  a.partial_off = partial_off;
  a.max_elems = max_elems;
  a.h = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  a.H = H;
  a.norm_w = with_norm ? reinterpret_cast<const __nv_bfloat16*>(norm_w->data_ptr()) : nullptr;
  a.eps = static_cast<float>(eps);
  a.x_out = with_norm ? reinterpret_cast<__nv_bfloat16*>(x_out->data_ptr()) : nullptr;
  a.status = status.data_ptr<int>();
  const int threads = ((H / 8 + 31) / 32) * 32;
  if (two_shot)
    launch_pdl(ll_allreduce_norm_kernel<true>, dim3(T), dim3(threads), 0,
               at::cuda::getCurrentCUDAStream(), "ll_allreduce_norm launch", a);
  else
    launch_pdl(ll_allreduce_norm_kernel<false>, dim3(T), dim3(threads), 0,
               at::cuda::getCurrentCUDAStream(), "ll_allreduce_norm launch", a);
}

}  // namespace sil
