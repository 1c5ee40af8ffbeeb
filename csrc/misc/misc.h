// Host interface of the fused memory-bound kernels (norm_rope.cu, sampling.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

void add_rmsnorm_launch(void* x, bool x_is_f32, long long x_stride, __nv_bfloat16* residual,
                        long long r_stride, const __nv_bfloat16* w, __nv_bfloat16* out,
                        long long o_stride, int rows, int H, float eps, bool clear_x,
                        cudaStream_t stream);

struct RopeKvParams {
  const int* positions;        // [T]
  const int* slot_mapping;     // [T] int32 or null (no cache write); < 0 skips
  const float* cos_sin;        // [max_pos, rot_dim]: cos in [0, rot/2), sin in [rot/2, rot)
  long long qkv_stride;        // row stride of the qkv input (elements)
  __nv_bfloat16* q_out;
  long long q_out_stride;
  __nv_bfloat16* k_cache;      // [num_blocks, Hkv, block_size, D]
  __nv_bfloat16* v_cache;
  long long kv_block_stride;
  const __nv_bfloat16* q_norm_w;  // [D] or null
  const __nv_bfloat16* k_norm_w;  // [D] or null
  float eps;
  int Hq, Hkv, head_dim, rot_dim, block_size;
  bool neox;
  bool clear_input;
  const float* qkv_bias;       // [(Hq + 2 Hkv) * D] fp32 added to the input row, or null
  // Interleaved multimodal RoPE (Qwen3-VL): positions3 [T, 3] (temporal, height, width); rotary
  // frequency j uses the height position when j % 3 == 1 and j < 3 * mrope_h, the width
  // position when j % 3 == 2 and j < 3 * mrope_w, else the temporal one.  null: 1-D positions.
  const int* positions3;
  int mrope_h, mrope_w;
  // q *= 1 + q_pos_beta * log(1 + floor(pos / q_pos_period)) after rotation (0: off)
  float q_pos_beta;
  float q_pos_period;
  // FP8 (e4m3) cache: the caches hold bytes, written as satfinite(k * k_inv_scale) and
  // satfinite(v * v_inv_scale).
  int kv_fp8;
  float k_inv_scale, v_inv_scale;
  // Bounds guard: slots at or beyond num_blocks * block_size are not written and raise kBadIndex
  // in the status word (0: unchecked).
  long long num_blocks;
  uint32_t* status;
};
void rope_kv_write_launch(const RopeKvParams& p, void* qkv, bool qkv_is_f32, int T,
                          cudaStream_t stream);

// FP8 (e4m3) activation quantization (quant.cu).
void quant_fp8_launch(const __nv_bfloat16* x, long long ldx, uint8_t* out, long long ldo, int rows,
                      int cols, float inv_scale, cudaStream_t stream);
// Per-token, per-128-column dynamic quantization (scales [rows][lds], max|x| / 448).
void quant_mx8_launch(const __nv_bfloat16* x, long long ldx, uint8_t* out, long long ldo, uint8_t* sf,
                      int rows, int cols, cudaStream_t stream);
void quant_mx8_tiles_launch(const __nv_bfloat16* x, long long ldx, uint8_t* out, long long ldo, uint8_t* sf,
                            const int* tiles, const int* count, int gmax, int cols, int kvalid,
                            cudaStream_t stream);
void quant_fp8_block_launch(const __nv_bfloat16* x, long long ldx, uint8_t* out, long long ldo,
                            float* scales, int lds, int rows, int cols, cudaStream_t stream);
// row_scales == null: static per-tensor scale; else per-row dynamic scales (max|y| / 448).
void rmsnorm_quant_launch(const __nv_bfloat16* x, long long ldx, const __nv_bfloat16* w, float eps,
                          uint8_t* out, long long ldo, int rows, int H, float inv_scale,
                          float* row_scales, cudaStream_t stream);

void silu_mul_launch(void* in, bool in_is_f32, long long in_stride, __nv_bfloat16* out,
                     long long out_stride, int T, int I, int blk, bool clear_input, int act,
                     float limit, float alpha, cudaStream_t stream);

// ids < 0 are device-resident tokens: id = last_tok[-id - 1] (the token a previous step
// sampled into that request slot; see SampleParams::row_slots).
void embedding_launch(const int* ids, const __nv_bfloat16* table, __nv_bfloat16* out, int T,
                      int H, int vocab_start, int vocab_end, const int* last_tok,
                      cudaStream_t stream);

struct SampleParams {
  const void* logits;          // [B, V] (bf16 or fp32)
  bool logits_f32;
  long long logits_stride;
  int B, V;
  const float* temperature;    // [B]; <= 0 means greedy
  const int* top_k;            // [B]; <= 0 or >= V disables
  const float* top_p;          // [B]; >= 1 disables
  const float* min_p;          // [B]; <= 0 disables (may be null)
  const uint64_t* seeds;       // [B] per-row seeds
  const int* offsets;          // [B] per-row step counters (RNG offset)
  int* out_tokens;             // [B]
  float* out_logprob;          // [B] log-probability of the sampled token (may be null)
  int vocab_offset;            // added to the sampled index (vocab shard start)
  float* out_max;              // [B] optional: row max of the processed logits (sharded merge)
  const int* row_slots;        // [B] optional: request slot of each row ...
  int* last_tok;               // ... whose device-resident last token is updated
};
void sample_launch(const SampleParams& p, cudaStream_t stream);

void apply_token_bitmask_launch(__nv_bfloat16* logits, long long stride, int rows, int V,
                                const int32_t* mask, int words, cudaStream_t stream);

void argmax_launch(const void* logits, bool f32, long long stride, int B, int V, int* out_idx,
                   float* out_val, int vocab_offset, cudaStream_t stream);

}  // namespace b200
