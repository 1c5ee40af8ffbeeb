// Host interface of the device-side expert-parallel exchange (ep_fused.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

constexpr int kMaxEP = 8;

// One symmetric allocation per rank (mapped on every peer), byte offsets from its base:
//   off_ctrl  u32 [1 + 2 * kMaxEP]: row-slot counter, disp_done[src], comb_done[src]
//   off_rows  bf16 [rows_cap][H]    received token rows
//   off_ids   int32 [rows_cap][k]   their expert ids (this rank's experts; -1 otherwise)
//   off_w     fp32 [rows_cap][k]    their routing weights
//   off_src   int32 [rows_cap]      (source rank << 24) | source token
//   off_comb  bf16 [tokens_cap][world][H]  reduced rows returned by each expert owner
// rows_cap = world * tokens_cap (every source may send each of its tokens once).
struct EPExchangeParams {
  void* peers[kMaxEP];
  long long off_ctrl, off_rows, off_ids, off_w, off_src, off_comb;
  int rank, world, H, k, num_experts, e_local;
  int tokens_cap, rows_cap;
  int T;                        // tokens of this rank in this call (<= tokens_cap)
  // token side (dispatch / combine)
  const __nv_bfloat16* x;       // [T, H] hidden rows, row pitch ldx
  long long ldx;
  const int* topk_ids;          // [T, k] global expert ids (negative: none)
  const float* topk_w;          // [T, k]
  __nv_bfloat16* out;           // [T, H] combined rows, row pitch ldo
  long long ldo;
  // expert side (return)
  const __nv_bfloat16* y;       // [rows_cap, H] reduced rows of the received tokens, pitch ldy
  long long ldy;
  // local control
  int* recv_count;              // device scalar: rows received this call
  unsigned int* ctas_done;      // device scalar (zero between kernels)
  unsigned long long* state;    // device: [0] calls completed
  uint32_t* status;
};

void ep_dispatch_launch(const EPExchangeParams& p, cudaStream_t s);
void ep_recv_launch(const EPExchangeParams& p, cudaStream_t s);
void ep_return_launch(const EPExchangeParams& p, cudaStream_t s);
void ep_combine_launch(const EPExchangeParams& p, cudaStream_t s);

}  // namespace b200
