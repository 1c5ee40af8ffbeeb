// Host interface of the symmetric peer-memory helpers and the fused tensor-parallel kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace b200 {

void* symm_alloc(size_t bytes, std::string* handle_out);
void* symm_open(const std::string& handle);
void symm_close(void* peer_ptr);
void symm_free(void* p);

constexpr int kMaxTP = 8;

// Reduce-scatter target of the fused row-parallel GEMM (EPI_TP_RS) and input of
// tp_norm_allgather: rank r owns token rows [r * rpr, (r + 1) * rpr).
struct TPRsParams {
  __nv_bfloat16* slots[kMaxTP];        // per rank: [world][rpr][H] bf16 receive slots
  unsigned long long* arrive[kMaxTP];  // per rank: slot-arrival counter (64-bit, cumulative)
  int* tile_count;                     // local: contributions received per output tile
  int rank, world, rows_per_rank, H;
  int splits;                          // contributions per tile (split-K factor)
};

struct TPNormAGParams {
  const __nv_bfloat16* slots;          // local receive slots [world][rpr][H]
  unsigned long long* slot_arrive;     // local slot-arrival counter
  __nv_bfloat16* x_peers[kMaxTP];      // per rank: all-gathered normalized rows [T][H]
  unsigned long long* x_arrive[kMaxTP];  // per rank: row-arrival counter
  unsigned long long* state;           // local: [0] calls completed, [1] CTAs done this call
  __nv_bfloat16* residual;             // local [T][H] (owned rows are updated)
  const __nv_bfloat16* w;              // RMSNorm weight [H]
  uint32_t* status;
  float eps;
  int rank, world, rows_per_rank, H, T;
  int tiles_per_call;                  // output tiles per rank per GEMM (N / 128)
};

void tp_norm_allgather_launch(const TPNormAGParams& p, cudaStream_t stream);

}  // namespace b200
