// Allocation-free C entry point of the paged decode attention kernel.
//
// This entry point has no counterpart in the reference; it exists for callers
// that cannot allocate device memory while they run: code executing inside a
// CUDA-graph capture that forbids allocations, embedders whose allocator is
// owned by someone else (a host engine or runtime that hands out only input and
// output buffers), or real-time loops where a cudaMalloc would stall or fail.
//
// It runs the same split-KV flash-decoding kernel as the PyTorch binding
// (`paged_decode`), but its split-K scratch - the per-split fp32 partial
// outputs, the per-(sequence, kv-head) arrival counters and the device status
// word - lives in one file-scope `static __device__ __align__(256)` array in
// the kernel library.  Every GPU that loads the library holds that array
// (about 4.1 MiB) until the process exits.
//
// Limits: batch * kv_heads * num_splits * (q_heads / kv_heads) * 130 <= 1,048,576
// fp32 values and batch * kv_heads <= 4096; larger requests are rejected with
// SIL_NOALLOC_ETOOBIG and a message from sil_noalloc_last_error().  head_dim is
// 128, the page size 64 tokens, q_heads / kv_heads <= 16.
//
// Sharing: all calls on a device share the one array, which keeps the last
// call's contents.  Each call clears the counters and the status word it uses
// (cudaMemsetAsync on the caller's stream) before the kernel runs.  Calls whose
// kernels overlap on the GPU (different streams without ordering, or several
// host threads) race on the array and produce wrong results; serialise them.
//
// Status: the kernel reports failures in a device status word inside the array
// instead of faulting: 1 when a wait for a TMA page load gave up, 5 when a
// block-table entry lies outside [0, num_pages) (that page is not loaded).  The
// output of such a call is incomplete.  The word is cleared at the start of each
// call, so read it with sil_noalloc_status() after the call and before the next
// one.  Every wait is bounded (2 s by default; sil_noalloc_set_wait_limit_ns
// changes the bound for later calls on the current device).
//
// Set-up: the first call on each device (with that device current) looks up
// the array's device address with cudaGetSymbolAddress and sets the kernel's
// shared-memory attribute; make that first call before any stream capture.
// The entry point itself calls no cudaMalloc, cudaFree or allocating library
// routine.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SIL_NOALLOC_OK 0
#define SIL_NOALLOC_EINVAL -1    // a null, misaligned or inconsistent argument
#define SIL_NOALLOC_ETOOBIG -2   // the request needs more scratch than the array holds
#define SIL_NOALLOC_ECUDA -3     // a CUDA runtime call failed (message available)

// q:        [batch, q_heads, 128] bf16, rows q_stride elements apart (heads contiguous)
// k/v:      [num_pages, kv_heads, 64, 128] bf16, contiguous, 16-byte aligned
// block_table: [batch, bt_stride] int32 page ids; seq_lens: [batch] int32 (context
//           length including the token being decoded)
// out:      [batch, q_heads * 128] bf16, rows out_stride elements apart
// q_stride must be even and >= q_heads * 128, out_stride >= q_heads * 128,
// bt_stride > 0.
// Returns SIL_NOALLOC_OK or a negative error code.
int sil_paged_decode_noalloc(const void* q, long long q_stride, const void* k_cache,
                             const void* v_cache, long long num_pages, int kv_heads,
                             const int* block_table, long long bt_stride, const int* seq_lens,
                             void* out, long long out_stride, int batch, int q_heads, float scale,
                             int num_splits, cudaStream_t stream);

// Copies the device status word of the current device's array into *host_out
// (0 = the last call ran clean) and waits for `stream`.  Order it after the call
// on the same stream.
int sil_noalloc_status(int* host_out, cudaStream_t stream);

// Bounds every wait of later calls on the current device to `ns` nanoseconds
// (0 restores the default of 2 s).  Waits for `stream`.
int sil_noalloc_set_wait_limit_ns(unsigned long long ns, cudaStream_t stream);

// Message of the last error returned on this host thread ("" when none).
const char* sil_noalloc_last_error(void);

// Scratch capacity in fp32 values and in (sequence, kv-head) counters.
long long sil_noalloc_scratch_floats(void);
int sil_noalloc_max_counters(void);

#ifdef __cplusplus
}
#endif
