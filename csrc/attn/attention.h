// Host interface of the paged attention kernels (paged_attention.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

struct PagedAttnParams {
  const __nv_bfloat16* q;  // [T, Hq, D] (token stride q_stride_t)
  long long q_stride_t;
  const __nv_bfloat16* k_cache;  // [num_blocks, Hkv, block_size, D]
  const __nv_bfloat16* v_cache;
  long long kv_block_stride;     // elements between consecutive blocks
  const int* block_tables;       // [B, bt_stride]
  int bt_stride;
  const int* seq_lens;           // [B] total KV length (cached + this step)
  const int* q_start;            // [B + 1] cumulative query lengths
  const int2* work;              // [num_work] (sequence, first packed row)
  __nv_bfloat16* out;            // [T, Hq, D]
  long long o_stride_t;
  float* part_o;                 // [splits, T, Hq, D] (split-KV only)
  float* part_lse;               // [splits, T, Hq]
  const float* sinks;            // [Hq] or null
  int num_splits;
  int Hq, Hkv, G;
  int block_size;
  int window;                    // 0 = full attention
  float scale_log2;              // softmax scale * log2(e)
  int total_tokens;
  long long kv_rows;             // num_blocks * Hkv * block_size of one cache (0 = unknown)
  uint32_t* status;              // device status word for bounded waits (may be null)
  int* sched;                    // decode unit counters [2], zero between launches (may be null)
  // FP8 KV cache: k_cache / v_cache hold e4m3 bytes in the same [blocks, Hkv, bs, D] layout;
  // true values are byte * k_scale (folded into scale_log2 by the caller) and byte * v_scale
  // (applied to the normalized output here).
  int kv_fp8;
  float v_scale;
  // Decode (TMA kernel and combine): when set, the split factor actually used, read on the
  // device (1 <= *splits_dev <= num_splits).  Lets a captured CUDA graph (whose num_splits is
  // sized for max_model_len) split each step by its real context lengths.
  const int* splits_dev;
  // Decode context parallelism: this rank holds the tokens of every (dcp_size * block_size)
  // token window whose block_size-slice index is dcp_rank; seq_lens are then the local token
  // counts and dcp_seq_lens the whole-sequence lengths (null without DCP), from which each
  // query's causal limit in local key indices is derived.
  const int* dcp_seq_lens;
  int dcp_size, dcp_rank;
  // Write unnormalised split partials (part_o / part_lse) even for one split and leave the
  // merge to the caller (DCP merges the partials of all ranks after exchanging them).
  int partial_out;
  // Packed query rows per prefill work item: 64 (mma.sync kernel) or fmha_prefill_rows() = 256
  // (tcgen05 kernel, fmha_sm100.cu); 0 means 64.  The work list must have been built with the
  // same value.
  int prefill_rows;
};

#ifdef __CUDACC__
// Number of tokens among global positions [0, n) that a DCP rank holds (block_size interleave).
__device__ __forceinline__ int dcp_local_count(int n, int bs, int size, int rank) {
  const int vb = bs * size;
  const int full = n / vb;
  const int rem = n - full * vb;
  return full * bs + min(max(rem - rank * bs, 0), bs);
}

// Last local key index visible to the query at global position g (-1: none on this rank).
__device__ __forceinline__ int dcp_last_visible(int g, int bs, int size, int rank) {
  return dcp_local_count(g + 1, bs, size, rank) - 1;
}
#endif

void paged_attention_launch(const PagedAttnParams& p, int num_work, int head_dim, bool decode,
                            cudaStream_t stream);

// tcgen05 prefill attention (fmha_sm100.cu): head_dim 128, bf16 cache, one split, 128-row work
// items.
int fmha_prefill_rows();  // packed rows per tcgen05 prefill work item
bool fmha_prefill_supported(const PagedAttnParams& p, int head_dim);
void fmha_prefill_launch(const PagedAttnParams& p, int num_work, cudaStream_t stream);

// Persistent TMA-fed decode kernel (paged_decode.cu); used for decode batches when the caches
// are contiguous [num_blocks, Hkv, block_size, D] tensors with block_size % 16 == 0 and a
// unit counter is given.
bool paged_decode_tma_supported(const PagedAttnParams& p, int head_dim);
void paged_decode_tma_launch(const PagedAttnParams& p, int num_work, int head_dim,
                             cudaStream_t stream);
int paged_decode_warps_per_cta(int head_dim);

// Merge split partials part_o [S, T, Hq, D] / part_lse [S, T, Hq] (log2 domain) into bf16 out.
void attn_combine_launch(const float* part_o, const float* part_lse, __nv_bfloat16* out,
                         long long o_stride_t, int total_tokens, int Hq, int num_splits,
                         int head_dim, cudaStream_t stream);

}  // namespace b200
