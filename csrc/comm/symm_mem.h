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
  __nv_bfloat16* recv_peers[kMaxTP];    // per rank: receive slots [3][world][max_rows][H]
                                        // (the flag form uses sets 0 and 1)
  unsigned int* flag_peers[kMaxTP];     // per rank: flags [2][max_rows][world] (flag form)
  unsigned long long* state;            // local: [0] calls completed, [1] CTAs done this call,
                                        // [2] rows of the previous call (sentinel form)
  __nv_bfloat16* residual;              // local [T][H], updated in place (all rows)
  long long res_stride;
  const __nv_bfloat16* w;               // RMSNorm weight [H]
  __nv_bfloat16* out;                   // local [T][H] normalized activations
  long long out_stride;
  uint32_t* status;
  float eps;
  int rank, world, max_rows, H, T;
  int algo;  // 0: sentinel form (data polled, no flags); 1: per-row flags with fences
};

void tp_allreduce_norm_launch(const TPArNormParams& p, cudaStream_t stream);

// Sequence-parallel prefill: the consumer of a reduce-scatter GEMM (EPI_BF16_RS) fused with the
// residual add, RMSNorm and the all-gather push of the normalized rows (sp_fused.cu).  For each
// of this rank's `rows` token rows: wait until every source's counter reaches rs_target, sum
// the sources' bf16 partial rows in rank order, residual += sum, y = rmsnorm(residual) * w, store
// y into every rank's all-gather buffer (x_out[r] + row * H, NVLink stores to peers) and finally
// raise every rank's ag_ctr[r] (that rank's counter for this source) once per CTA.
struct SPNormPushParams {
  const __nv_bfloat16* slots;       // local receive slots of this call: [world][slot_rows][H]
  long long slot_src_stride;        // elements between sources' slots
  int nsrc;                         // 0: nothing to sum (first layer: residual already reduced)
  const unsigned int* rs_ctr;       // local [world] counters raised by the sources' GEMMs
  unsigned int rs_target;
  __nv_bfloat16* residual;          // [rows][H], updated in place
  const __nv_bfloat16* w;           // [H]
  float eps;
  __nv_bfloat16* x_out[kMaxTP];     // per rank: its all-gather buffer at this rank's first row
  unsigned int* ag_ctr[kMaxTP];     // per rank: its counter for this source
  int world, rows, H;
  uint32_t* status;
};
void sp_norm_push_launch(const SPNormPushParams& p, cudaStream_t stream);
struct SPWaitTargets {
  unsigned int v[kMaxTP];
};
// Bounded wait until ctr[r] >= target[r] for r < world (one CTA); orders later kernels after
// the peers' pushes.
void sp_wait_launch(const unsigned int* ctr, const unsigned int* targets_host, int world,
                    uint32_t* status, cudaStream_t stream);
void flag_wait_probe_launch(const unsigned int* flag, unsigned int target, unsigned long long timeout_ns,
                            uint32_t* status, int* result, cudaStream_t stream);

}  // namespace b200
