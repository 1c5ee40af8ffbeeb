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

// One-shot all-reduce of a row-parallel projection's fp32 partial sums, fused with the
// residual add and the next RMSNorm (tp_fused.cu).  Every rank pushes its bf16 partial rows
// into every peer's receive slots over NVLink, publishes one flag per (row, source) and
// sums the world's partials in rank order, so all ranks hold bitwise-identical results.
struct TPArNormParams {
  float* acc;                           // local [T][H] fp32 partials (cleared by the kernel)
  long long acc_stride;
  __nv_bfloat16* recv_peers[kMaxTP];    // per rank: receive slots [2][world][max_rows][H]
  unsigned int* flag_peers[kMaxTP];     // per rank: flags [2][max_rows][world] (epoch numbers)
  unsigned long long* state;            // local: [0] calls completed, [1] CTAs done this call
  __nv_bfloat16* residual;              // local [T][H], updated in place (all rows)
  long long res_stride;
  const __nv_bfloat16* w;               // RMSNorm weight [H]
  __nv_bfloat16* out;                   // local [T][H] normalized activations
  long long out_stride;
  uint32_t* status;
  float eps;
  int rank, world, max_rows, H, T;
};

void tp_allreduce_norm_launch(const TPArNormParams& p, cudaStream_t stream);
void flag_wait_probe_launch(const unsigned int* flag, unsigned int target, unsigned long long timeout_ns,
                            uint32_t* status, int* result, cudaStream_t stream);

}  // namespace b200
