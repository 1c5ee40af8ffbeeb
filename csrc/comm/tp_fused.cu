// Second half of the fused row-parallel projection for tensor-parallel decode:
//
//   GEMM (EPI_TP_RS)      each rank pushes its partial rows to the rows' owners (NVLink)
//   tp_norm_allgather     owner: sum the world partials + residual, RMSNorm, and store the
//                         normalized row into every rank's activation buffer (NVLink), then
//                         wait until all rows of this call have arrived from every owner.
//
// This replaces "GEMM -> all-reduce -> residual add -> RMSNorm" (reference:
// RowParallelLinear + all-reduce, vllm_neuron/nn/rpl.py:23-154, and the decode all-reduce
// sites in vllm_neuron/model/llama3/model.py:989,1113) with one reduce-scatter fused into the
// GEMM epilogue and one all-gather fused into the norm.  The residual stream of a rank is
// only kept for the rows it owns (sequence-parallel residual).
//
// Synchronization: cumulative 64-bit arrival counters in symmetric memory, release/acquire
// at system scope, and a per-rank call counter kept on the device (CUDA-graph safe).  Every
// wait is bounded by %globaltimer; on expiry the kernel records a status code and returns.
#include <cuda_bf16.h>

#include <stdexcept>

#include "../common.cuh"
#include "symm_mem.h"

namespace b200 {

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Returns false (and records `code`) if the counter did not reach `target` in time.
__device__ __forceinline__ bool wait_counter(const unsigned long long* c, unsigned long long target,
                                             uint32_t* status, uint32_t code) {
  if (ld_acquire_sys(c) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys(c) < target) {
    if (globaltimer_ns() - t0 > B200_WAIT_TIMEOUT_NS) {
      set_status(status, code);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

template <int NV>
__global__ void __launch_bounds__(256) tp_norm_allgather_kernel(const TPNormAGParams p) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  __shared__ unsigned long long epoch_s;
  const int tid = threadIdx.x;
  if (tid == 0) {
    const unsigned long long e = *reinterpret_cast<volatile unsigned long long*>(&p.state[0]);
    epoch_s = e;
    wait_counter(p.slot_arrive, (e + 1) * (unsigned long long)(p.tiles_per_call * p.world),
                 p.status, kTimeoutPeerFlag);
  }
  __syncthreads();
  const unsigned long long e = epoch_s;
  const int lrow = blockIdx.x;
  const int gm = p.rank * p.rows_per_rank + lrow;
  if (lrow < p.rows_per_rank && gm < p.T) {
    float v[NV][8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int idx = (j * blockDim.x + tid) * 8;
      if (idx < p.H) {
        float acc[8];
        const uint4 r = *reinterpret_cast<const uint4*>(p.residual + (long long)gm * p.H + idx);
        const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = unpack_bf16x2(rw[i]);
          acc[2 * i] = f.x;
          acc[2 * i + 1] = f.y;
        }
        for (int w = 0; w < p.world; ++w) {
          const uint4 s = __ldcg(reinterpret_cast<const uint4*>(
              p.slots + ((long long)(w * p.rows_per_rank + lrow)) * p.H + idx));
          const uint32_t sw[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = unpack_bf16x2(sw[i]);
            acc[2 * i] += f.x;
            acc[2 * i + 1] += f.y;
          }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          v[j][k] = __bfloat162float(__float2bfloat16(acc[k]));
          ss += v[j][k] * v[j][k];
        }
        *reinterpret_cast<uint4*>(p.residual + (long long)gm * p.H + idx) =
            make_uint4(pack_bf16x2(v[j][0], v[j][1]), pack_bf16x2(v[j][2], v[j][3]),
                       pack_bf16x2(v[j][4], v[j][5]), pack_bf16x2(v[j][6], v[j][7]));
      }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float t = (tid < (int)(blockDim.x >> 5)) ? red[tid] : 0.f;
    if (tid < 32) {
      t = warp_sum(t);
      if (tid == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] / (float)p.H + p.eps);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int idx = (j * blockDim.x + tid) * 8;
      if (idx < p.H) {
        const uint4 g = *reinterpret_cast<const uint4*>(p.w + idx);
        const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = unpack_bf16x2(gw[i]);
          o[i] = pack_bf16x2(v[j][2 * i] * inv * f.x, v[j][2 * i + 1] * inv * f.y);
        }
        const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
        for (int r = 0; r < p.world; ++r)
          *reinterpret_cast<uint4*>(p.x_peers[r] + (long long)gm * p.H + idx) = ov;
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (tid == 0) {
    for (int r = 0; r < p.world; ++r) atomicAdd_system(p.x_arrive[r], 1ull);
    // all rows of this call, from every owner
    wait_counter(p.x_arrive[p.rank], (e + 1) * (unsigned long long)(p.world * p.rows_per_rank),
                 p.status, kTimeoutPeerFlag);
    __threadfence();
    if (atomicAdd(&p.state[1], 1ull) == (unsigned long long)(gridDim.x - 1)) {
      p.state[1] = 0;
      __threadfence();
      p.state[0] = e + 1;
    }
  }
}

void tp_norm_allgather_launch(const TPNormAGParams& p, cudaStream_t stream) {
  if (p.H % 8 != 0) throw std::invalid_argument("tp_norm_allgather: H must be a multiple of 8");
  const int vecs = p.H / 8;
  const int nv = (vecs + 255) / 256;
  const dim3 grid(p.rows_per_rank > 0 ? p.rows_per_rank : 1);
  if (nv <= 1)
    launch_pdl(tp_norm_allgather_kernel<1>, grid, dim3(256), 0, stream, p);
  else if (nv <= 2)
    launch_pdl(tp_norm_allgather_kernel<2>, grid, dim3(256), 0, stream, p);
  else if (nv <= 4)
    launch_pdl(tp_norm_allgather_kernel<4>, grid, dim3(256), 0, stream, p);
  else
    throw std::invalid_argument("tp_norm_allgather: hidden size too large");
}

}  // namespace b200
