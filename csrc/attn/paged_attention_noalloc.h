// Allocation-free C entry point for paged GQA attention with split-KV.
//
// This entry point has no counterpart in the reference (vllm-neuron); it is an addition of
// this library for callers that cannot allocate device memory.
//
// Who needs it.  The split-KV path of paged attention needs fp32 scratch for the partial
// outputs and log-sum-exps of every KV split.  The Python op takes that scratch from the
// torch caching allocator.  Some callers cannot allocate at all when they attend: code
// that runs inside a host runtime with its own fixed memory pool and no cudaMalloc rights
// (an inference server's custom allocator, a plugin loaded into another framework), code
// that must not call into torch (a plain C or C++ host), and code that runs where a
// cudaMalloc would synchronise the device or could fail under memory pressure in the
// middle of a step.  This entry point takes the scratch from a fixed-size array in the
// library's own device memory instead, so it calls no cudaMalloc, cudaFree or allocating
// library routine.
//
// Limit.  The scratch array is B200_NOALLOC_SCRATCH_BYTES (16 MiB) of device memory.  With
// CUDA's lazy module loading it is reserved on a device when the library's module is first
// loaded there (at the library's first kernel launch on that device, or at the first call of
// this entry point, whose set-up can itself trigger that load) and stays reserved until the
// process exits.  A call needs
//   4 * num_splits * total_tokens * num_q_heads * (head_dim + 1) bytes
// (plus at most 256 bytes of alignment padding) when num_splits > 1, and none otherwise;
// larger calls are rejected with B200_NOALLOC_ERR_TOO_LARGE and a message.
//
// Sharing.  All calls on one device share the one array, which keeps whatever the last call
// left in it.  Each call overwrites every partial it later reads, so nothing has to be
// cleared between calls.  Calls on the same stream are ordered; calls that overlap on the
// GPU (different streams, or different host threads without ordering) race on the array
// and produce wrong results.
//
// Set-up.  The first call on a device, with that device current, looks up the device
// address of the array (cudaGetSymbolAddress) and caches it; later calls reuse it.  That
// look-up may load the module on the device (see Limit), so make the first call before any
// stream capture starts on the device.
#pragma once

#include <stddef.h>

#define B200_NOALLOC_SCRATCH_BYTES (16u << 20)

#define B200_NOALLOC_OK 0
#define B200_NOALLOC_ERR_INVALID 1    // a pointer, size or shape argument is not supported
#define B200_NOALLOC_ERR_TOO_LARGE 2  // the split partials do not fit the scratch array
#define B200_NOALLOC_ERR_CUDA 3       // a CUDA runtime call failed (set-up or launch)

#ifdef __cplusplus
extern "C" {
#endif

// Paged attention of q [total_tokens, num_q_heads, head_dim] (bf16, heads packed, token
// stride q_stride_t elements) over the K/V caches [num_blocks, num_kv_heads, block_size,
// head_dim] (bf16, block stride kv_block_stride elements), writing out [total_tokens,
// num_q_heads, head_dim] (bf16, token stride o_stride_t).  All pointers are device
// pointers of the current device; `work` is int32 [num_work, 2] (sequence, first packed
// row) as built by vllm_neuron_b200.ops.attention.build_work, and block_tables / seq_lens /
// q_start are int32 as for the Python op.  `sinks` is fp32 [num_q_heads] or NULL; `window`
// is 0 for full attention; head_dim is 64 or 128.  `decode` selects the 16-row decode
// tiling, which assumes one query token per sequence: pass 1 only when every step
// q_start[i + 1] - q_start[i] is 1 (the `decode` flag that build_work returns), else 0 --
// the entry point does not check it, and a multi-token query with decode = 1 gives wrong
// results.  `stream` is a cudaStream_t (NULL for the legacy default stream).  On failure the
// return code is non-zero and, when err is not NULL, a NUL-terminated message of at most
// err_len bytes is written to it.
int b200_paged_attention_noalloc(const void* q, long long q_stride_t, const void* k_cache,
                                 const void* v_cache, long long kv_block_stride,
                                 const int* block_tables, int bt_stride, const int* seq_lens,
                                 const int* q_start, const int* work, int num_work, void* out,
                                 long long o_stride_t, const float* sinks, int total_tokens,
                                 int num_q_heads, int num_kv_heads, int head_dim,
                                 int block_size, int window, float scale, int decode,
                                 int num_splits, void* stream, char* err, size_t err_len);

#ifdef __cplusplus
}
#endif
