// Host interface of the gated DeltaNet (linear attention) kernels (deltanet.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

// Batch layout shared by the kernels: sequence b owns tokens [q_start[b], q_start[b + 1]) of
// this step and has seq_lens[b] tokens in total (context before the step = seq_lens - q_len;
// 0 means the recurrent state starts from zero).  slots[b] indexes the per-request state
// cache.
struct LinearAttnBatch {
  const int* q_start;
  const int* seq_lens;
  const int* slots;
  int B;
};

// y[t, c] = silu(sum_j w[c, j] * x[t - (K - 1) + j, c]) over this step's tokens, with the
// previous K - 1 inputs of each channel taken from (and written back to) the conv state
// [slots][C][K - 1].
void causal_conv1d_launch(const __nv_bfloat16* x, long long ldx, int C, const __nv_bfloat16* w,
                          int K, const LinearAttnBatch& b, __nv_bfloat16* state,
                          long long state_slot_stride, __nv_bfloat16* y, long long ldy,
                          cudaStream_t s);

struct GatedDeltaParams {
  const __nv_bfloat16* qkv;   // conv output [T, 2 * Hk * dk + Hv * dv]: q | k | v
  long long ld_qkv;
  const __nv_bfloat16* z;     // output gate [T, Hv * dv]
  const __nv_bfloat16* a;     // decay input [T, Hv]
  const __nv_bfloat16* b;     // beta input [T, Hv]
  long long ld_zab;           // row stride of z, a and b (they live in one projection)
  const float* A_log;         // [Hv]
  const float* dt_bias;       // [Hv]
  const __nv_bfloat16* norm_w;  // gated RMSNorm weight [dv]
  float eps;
  float* state;               // [slots][Hv][dk][dv] fp32
  long long state_slot_stride;
  __nv_bfloat16* out;         // [T, Hv * dv]
  long long ld_out;
  int Hk, Hv, dk, dv;
  float4* gb;                 // scratch [T, Hv]: (g, beta, 1/|q|, 1/|k|) per token and value head
  int T;                      // tokens of this step (rows of out)
};

// Recurrent gated delta rule over this step's tokens (q, k l2-normalised, q scaled by
// dk^-1/2; g = -exp(A_log) * softplus(a + dt_bias); beta = sigmoid(b)), followed by the
// per-head gated RMSNorm out = rmsnorm(o) * w * silu(z).
void gated_delta_rule_launch(const GatedDeltaParams& p, const LinearAttnBatch& b, cudaStream_t s);

// Chunked (WY) form of the same rule for prefill-sized steps: tokens of each sequence are cut
// into chunks of 64; a parallel pass solves the intra-chunk triangular system per (chunk,
// value head) and a sequential pass per (sequence, value head, 32 value columns) carries the
// fp32 state across the chunks.  Scratch (device memory the caller provides):
struct GdnChunkScratch {
  float* W;           // [T, Hv, dk]   (I + A)^-1 diag(beta gamma) K^
  float* U;           // [T, Hv, dv]   (I + A)^-1 diag(beta) V
  float* QKm;         // [max_chunks, Hv, 64, 64]  decay-masked Q^ K^T (s <= t)
  float* lg;          // [T, Hv]       log of the cumulative decay from the chunk start
  int4* chunks;       // [max_chunks]  (first token, length, sequence, -)
  int* seq_chunk0;    // [B + 1]       first chunk of each sequence; [B] = chunk count
  int max_chunks;     // >= T / 64 + B
};
void gated_delta_rule_chunked_launch(const GatedDeltaParams& p, const LinearAttnBatch& b,
                                     const GdnChunkScratch& s, cudaStream_t stream);

// x[t, i] *= sigmoid(gate[t, i]) for i < n.
void sigmoid_gate_mul_launch(__nv_bfloat16* x, long long ldx, const __nv_bfloat16* gate,
                             long long ldg, int T, int n, cudaStream_t s);

}  // namespace b200
