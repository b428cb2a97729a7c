// Allocation-free entry point for the PrefixLM attention forward.
//
// This entry point has no counterpart in the reference implementation. It is for callers of
// this library that cannot allocate device memory themselves: code running inside a host
// runtime that has already reserved the GPU's memory for its own pool (an inference server,
// another framework's caching allocator), or a latency-critical path that cannot accept the
// implicit device synchronisation of cudaMalloc/cudaFree. Such callers own the input and
// output buffers. The only other memory the forward needs -- its work schedule, the
// schedule's counters and an error word -- lives in a fixed-size static device array inside
// the library: HRM_ATTN_NOALLOC_SCRATCH_BYTES on every GPU that loads the library, held until
// the process exits. The call allocates nothing (no cudaMalloc, no allocating library call).
//
// It runs the same tcgen05 forward kernel as the framework's training path.
//
// Inputs / outputs are exactly those of the regular attention forward:
//   qkv         bf16 [T, >= 4*num_heads*128], row stride ld_qkv elements: gate, q, k, v heads
//               (q and k already rotated); base 16-byte aligned, ld_qkv a multiple of 8
//   cu_seqlens  int32 [n_cu], non-decreasing document boundaries starting at 0, with
//               cu_seqlens[last document] <= T (trailing zero padding allowed)
//   prefix_lens int32 [n_cu - 1], bidirectional prefix length per document
//   out, y      bf16 [T, num_heads*128], row stride ld_out (a multiple of 8), 16-byte aligned:
//               O and sigmoid(gate) * O
//   lse         fp32 [num_heads, T]: log2-domain log-sum-exp per (head, token)
//
// Limits: head_dim 128; ceil(T / 128) + n_cu <= HRM_ATTN_NOALLOC_MAX_TILES (pass the number
// of documents + 1 as n_cu rather than a padded length when T is large).
//
// Set-up: the first call on a device (with that device current) looks up the static array's
// device address and configures the kernel; make that first call before any stream capture.
// Host threads may make first calls concurrently. Every call on a device shares the one
// scratch array, which keeps the last call's contents; each call re-initialises the schedule,
// its counters and the error word before use. Calls whose executions overlap on the GPU --
// e.g. issued on two streams at once -- therefore race: serialise them on one stream.
//
// Returns 0 on success, HRM_ATTN_NOALLOC_TOO_LARGE (-1) when the problem exceeds the scratch
// limit, HRM_ATTN_NOALLOC_BAD_ARG (-2) for an invalid argument (checked before anything is
// launched), HRM_ATTN_NOALLOC_TENSOR_MAP (-3) if the TMA descriptor cannot describe qkv, or a
// positive cudaError_t from set-up or launch. hrm_attn_fwd_noalloc_strerror() describes a code.
//
// Device-side problems are reported in the error word, which hrm_attn_fwd_noalloc_status()
// copies to the host (synchronously; call it after the stream has finished):
//   code4[0] == 0  no problem
//   code4[0] == 2  a bounded wait in the attention kernel gave up (outputs are incomplete)
//   code4[0] == 4  the packing was rejected (a boundary past T or a negative start): no tile
//                  was computed and every output row was written as zero
#pragma once

#include <cuda_runtime.h>

#define HRM_ATTN_NOALLOC_SCRATCH_BYTES (1 << 20)
// 8 header ints + 8 ints per tile, then the 4-int error word
#define HRM_ATTN_NOALLOC_MAX_TILES (((HRM_ATTN_NOALLOC_SCRATCH_BYTES / 4) - 8 - 4) / 8)
#define HRM_ATTN_NOALLOC_TOO_LARGE (-1)
#define HRM_ATTN_NOALLOC_BAD_ARG (-2)
#define HRM_ATTN_NOALLOC_TENSOR_MAP (-3)

#ifdef __cplusplus
extern "C" {
#endif

int hrm_attn_fwd_noalloc(const void* qkv, long long ld_qkv, int T, int num_heads, const int* cu_seqlens, int n_cu,
                         const int* prefix_lens, int causal, void* out, void* y, long long ld_out, float* lse,
                         cudaStream_t stream);

const char* hrm_attn_fwd_noalloc_strerror(int code);

// Copies the current device's error word (4 ints: code, site, block, thread) into code4.
// Returns 0 or a cudaError_t of the copy.
int hrm_attn_fwd_noalloc_status(int* code4);

#ifdef __cplusplus
}
#endif
