// Allocation-free entry point for the PrefixLM attention forward.
//
// This entry point has no counterpart in the reference implementation; it exists for
// callers of this library that cannot allocate device memory themselves: code that runs
// inside a host runtime which has already reserved the GPU's memory for its own pool (an
// inference server, another framework's allocator), or a latency-critical path where the
// implicit device synchronisation of cudaMalloc/cudaFree is not acceptable. Such callers
// own the input and output buffers; the only extra memory the kernel needs -- the work
// schedule and its counters -- lives in a fixed-size static device array inside the
// library (HRM_ATTN_NOALLOC_SCRATCH_BYTES per GPU that loads the library, held until the
// process exits).
//
// Inputs / outputs are exactly those of the regular attention forward:
//   qkv         bf16 [T, >= 4*num_heads*128], row stride ld_qkv elements: gate, q, k, v heads
//               (q and k already rotated)
//   cu_seqlens  int32 [n_cu], document boundaries (trailing zero padding allowed)
//   prefix_lens int32 [n_cu - 1], bidirectional prefix length per document
//   out, y      bf16 [T, num_heads*128], row stride ld_out: O and sigmoid(gate) * O
//   lse         fp32 [num_heads, T]: log2-domain log-sum-exp per (head, token)
//
// Limits: head_dim 128; ceil(T / 128) + n_cu <= HRM_ATTN_NOALLOC_MAX_TILES (pass the number
// of documents + 1 as n_cu rather than a padded length when T is large).
//
// Set-up: the first call on a device (with that device current) looks up the static
// array's device address and configures the kernel; make that first call before any
// stream capture. Every call on a device shares the one scratch array (the schedule kernel
// re-initialises it, counters included, at the start of each call), so calls whose
// executions overlap on the GPU -- e.g. on two streams at once -- race and must not be
// issued; serialise them on one stream.
//
// Returns 0 on success, HRM_ATTN_NOALLOC_TOO_LARGE (-1) when the problem exceeds the
// scratch limit, HRM_ATTN_NOALLOC_BAD_ARG (-2) for an invalid argument, or a positive
// cudaError_t from set-up or launch. hrm_attn_fwd_noalloc_strerror() describes a code.
#pragma once

#include <cuda_runtime.h>

#define HRM_ATTN_NOALLOC_SCRATCH_BYTES (1 << 20)
#define HRM_ATTN_NOALLOC_MAX_TILES (((HRM_ATTN_NOALLOC_SCRATCH_BYTES / 4) - 8) / 8)
#define HRM_ATTN_NOALLOC_TOO_LARGE (-1)
#define HRM_ATTN_NOALLOC_BAD_ARG (-2)

#ifdef __cplusplus
extern "C" {
#endif

int hrm_attn_fwd_noalloc(const void* qkv, long long ld_qkv, int T, int num_heads, const int* cu_seqlens, int n_cu,
                         const int* prefix_lens, int causal, void* out, void* y, long long ld_out, float* lse,
                         cudaStream_t stream);

const char* hrm_attn_fwd_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif
