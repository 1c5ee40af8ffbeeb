// Sequence-parallel prefill over NVLink peer memory: the reduce-scatter consumer fused with
// the residual add, RMSNorm and the all-gather of the normalized rows.
//
// Under sequence parallelism each rank owns `rows` consecutive token rows of the residual
// stream.  A row-parallel projection (o_proj / down_proj) runs as one GEMM over all tokens whose
// epilogue (EPI_BF16_RS in gemm_sm100.cu) stores each output row into the owner's receive slot
// for its source rank and raises the owner's per-source counter after each tile.  Then, per
// owned row, sp_norm_push_kernel:
//
//   1. waits (bounded) until every source's counter reached this call's target;
//   2. residual += sum over sources of the bf16 partial rows, in rank order (identical order on
//      every rank), and y = rmsnorm(residual) * w;
//   3. stores y into every rank's all-gather buffer at this rank's rows (NVLink stores), so the
//      next column-parallel GEMM of every rank sees all tokens;
//   4. after a system-scope fence, raises each rank's counter for this source once per CTA.
//
// The next GEMM waits per source counter before loading that source's rows (gemm_sm100.cu), so
// it multiplies the rows that have arrived while the rest are in flight.  Counters are monotonic
// (the host tracks cumulative targets); slots and all-gather buffers alternate two parities by
// call, and a rank can reuse a parity only after every peer consumed it (each all-gather GEMM
// is followed by a reduce-scatter whose consumer waits for all peers).  Reference: SP prefill
// collectives of vllm_neuron/model/llama3/model.py:527-532,813-815,1096-1111.
#include <cuda_bf16.h>

#include <stdexcept>

#include "../common.cuh"
#include "symm_mem.h"

namespace b200 {

namespace {
__device__ __forceinline__ unsigned int ld_acq_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool wait_ctr(const unsigned int* c, unsigned int target, uint32_t* status) {
  if ((int)(ld_acq_sys(c) - target) >= 0) return true;
  if (status != nullptr && *reinterpret_cast<volatile uint32_t*>(status) != 0u) return false;
  const uint64_t t0 = globaltimer_ns();
  while ((int)(ld_acq_sys(c) - target) < 0) {
    if (globaltimer_ns() - t0 > B200_PEER_TIMEOUT_NS) {
      set_status(status, kTimeoutPeerFlag);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}
}  // namespace

// One CTA of 256 threads per owned row; NV vectors of 8 bf16 per thread (H <= NV * 2048).
template <int NV>
__global__ void __launch_bounds__(256) sp_norm_push_kernel(const SPNormPushParams p) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[8];
  const int tid = threadIdx.x;
  const int row = blockIdx.x;
  if (p.nsrc > 0) {
    if (tid < p.nsrc) wait_ctr(p.rs_ctr + tid, p.rs_target, p.status);
    __syncthreads();
  }
  float v[NV][8];
  float ss = 0.f;
  __nv_bfloat16* res = p.residual + (long long)row * p.H;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int idx = (j * 256 + tid) * 8;
    if (idx < p.H) {
      const uint4 r4 = *reinterpret_cast<const uint4*>(res + idx);
      const uint32_t rw[4] = {r4.x, r4.y, r4.z, r4.w};
      float acc[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(rw[i]);
        acc[2 * i] = 0.f;
        acc[2 * i + 1] = 0.f;
        v[j][2 * i] = f.x;
        v[j][2 * i + 1] = f.y;
      }
      for (int sidx = 0; sidx < p.nsrc; ++sidx) {
        const uint4 s4 = __ldcv(reinterpret_cast<const uint4*>(
            p.slots + (long long)sidx * p.slot_src_stride + (long long)row * p.H + idx));
        const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = unpack_bf16x2(sw[i]);
          acc[2 * i] += f.x;
          acc[2 * i + 1] += f.y;
        }
      }
      uint32_t ow[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ow[i] = pack_bf16x2(v[j][2 * i] + acc[2 * i], v[j][2 * i + 1] + acc[2 * i + 1]);
        const float2 f = unpack_bf16x2(ow[i]);  // the residual is kept in bf16
        v[j][2 * i] = f.x;
        v[j][2 * i + 1] = f.y;
        ss += f.x * f.x + f.y * f.y;
      }
      if (p.nsrc > 0) *reinterpret_cast<uint4*>(res + idx) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float rstd = rsqrtf(tot / (float)p.H + p.eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int idx = (j * 256 + tid) * 8;
    if (idx < p.H) {
      const uint4 w4 = *reinterpret_cast<const uint4*>(p.w + idx);
      const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
      uint32_t y[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 wf = unpack_bf16x2(ww[i]);
        const float a = __bfloat162float(__float2bfloat16(v[j][2 * i] * rstd)) * wf.x;
        const float b = __bfloat162float(__float2bfloat16(v[j][2 * i + 1] * rstd)) * wf.y;
        y[i] = pack_bf16x2(a, b);
      }
      const uint4 y4 = make_uint4(y[0], y[1], y[2], y[3]);
      for (int r = 0; r < p.world; ++r)
        *reinterpret_cast<uint4*>(p.x_out[r] + (long long)row * p.H + idx) = y4;
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    for (int r = 0; r < p.world; ++r)
      asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(p.ag_ctr[r]) : "memory");
  }
}

__global__ void sp_wait_kernel(const unsigned int* ctr, SPWaitTargets t, int world, uint32_t* status) {
  pdl_trigger();
  pdl_wait();
  if ((int)threadIdx.x < world) wait_ctr(ctr + threadIdx.x, t.v[threadIdx.x], status);
}

void sp_norm_push_launch(const SPNormPushParams& p, cudaStream_t stream) {
  if (p.rows == 0) return;
  if (p.H % 8 != 0) throw std::invalid_argument("sp_norm_push: H must be a multiple of 8");
  if (p.world < 1 || p.world > kMaxTP) throw std::invalid_argument("sp_norm_push: world");
  const int nv = (p.H / 8 + 255) / 256;
  if (nv == 1)
    launch_pdl(sp_norm_push_kernel<1>, dim3(p.rows), dim3(256), 0, stream, p);
  else if (nv == 2)
    launch_pdl(sp_norm_push_kernel<2>, dim3(p.rows), dim3(256), 0, stream, p);
  else if (nv <= 4)
    launch_pdl(sp_norm_push_kernel<4>, dim3(p.rows), dim3(256), 0, stream, p);
  else
    throw std::invalid_argument("sp_norm_push: H above 8192");
}

void sp_wait_launch(const unsigned int* ctr, const unsigned int* targets_host, int world,
                    uint32_t* status, cudaStream_t stream) {
  SPWaitTargets t{};
  for (int r = 0; r < world && r < kMaxTP; ++r) t.v[r] = targets_host[r];
  launch_pdl(sp_wait_kernel, dim3(1), dim3(32), 0, stream, ctr, t, world, status);
}

}  // namespace b200
