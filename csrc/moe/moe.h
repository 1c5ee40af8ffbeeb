// Host interface of the mixture-of-experts routing kernels (moe.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

enum RouteMode : int {
  ROUTE_TOPK_SOFTMAX = 0,  // top-k of the logits, softmax over the k selected (GPT-OSS)
  ROUTE_SOFTMAX_TOPK = 1,  // softmax over all experts, top-k, optional renormalisation (Qwen)
  ROUTE_SIGMOID_TOPK = 2,  // sigmoid scores, top-k, optional renormalisation
  ROUTE_SIGMOID_BIAS_TOPK = 3,  // top-k of sigmoid + correction bias; weights from the
                                // unbiased sigmoid, optional renormalisation (GLM-4.5 MoE)
};

enum MoeAct : int {
  MOE_ACT_SILU = 0,    // silu(gate) * up
  MOE_ACT_GPTOSS = 1,  // gate = min(gate, limit); up = clamp(up, +-limit);
                       // (up + 1) * gate * sigmoid(alpha * gate)
};

// logits [T, E (+1)]: when shared_gate is given, column E is the shared expert's gate logit
// and shared_gate[t] = sigmoid(logits[t, E]).
// weights are multiplied by `scale` (routed scaling factor) after any renormalisation
void moe_route_launch(const __nv_bfloat16* logits, long long ld, const float* bias, int T, int E,
                      int k, int mode, bool renorm, int* ids, float* weights, float* shared_gate,
                      float scale, cudaStream_t s);

// Groups the T*k assignments by local expert [e_start, e_start + e_local).
// Router GEMV (w [rows, H] bf16, rows = E or E + 1 with the shared-expert gate row) fused with
// the routing of moe_route_launch, one CTA per token (decode batches).  `logits` (optional)
// receives the bf16 logits [T, rows].
void moe_router_topk_launch(const __nv_bfloat16* x, long long ldx, const __nv_bfloat16* w, int rows,
                            int H, const float* bias, int T, int E, int k, int mode, bool renorm,
                            float scale, __nv_bfloat16* logits, long long ldl, int* ids,
                            float* weights, float* shared_gate, cudaStream_t s);

void moe_align_launch(const int* ids, int n_assign, int e_start, int e_local, int* offsets,
                      int* sorted_src, int* row_expert, int* inv_pos, int* gtiles, int* gcount,
                      int gmax, cudaStream_t s);

void moe_gather_launch(const __nv_bfloat16* x, long long ldx, const int* sorted_src, int topk,
                       const int* total, int rows_cap, int H, __nv_bfloat16* out, cudaStream_t s);

void moe_act_launch(const __nv_bfloat16* gu, const __nv_bfloat16* bias, const int* row_expert,
                    const int* total, int rows_cap, int I, int mode, float alpha, float limit,
                    __nv_bfloat16* out, cudaStream_t s);

void moe_combine_launch(const __nv_bfloat16* y, const int* inv_pos, const float* weights,
                        const int* ids, const __nv_bfloat16* bias, int e_start, int T, int k,
                        int H, const __nv_bfloat16* shared, long long ld_shared,
                        const float* shared_gate, __nv_bfloat16* out, long long ldo,
                        cudaStream_t s, long long ldy = 0);

// Y[rows, N] = X[rows, K] @ dequant(W_e)^T for the tile list of moe_align (<= 16 rows per pass),
// W in MXFP4 tiles (moe_mxfp4.cu): wt [E, ceil(N / 256), K / 64, tile_bytes] uint8.
int moe_mxfp4_tile_bytes();
int moe_mxfp4_tile_cols();
void moe_mxfp4_gemm_launch(const __nv_bfloat16* x, long long ldx, const uint8_t* wt,
                           const int* gtiles, const int* gcount, int gmax, int N, int K,
                           __nv_bfloat16* y, long long ldy, uint32_t* status, cudaStream_t s);

}  // namespace b200
