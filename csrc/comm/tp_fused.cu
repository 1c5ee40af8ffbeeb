// Fused tensor-parallel all-reduce + residual add + RMSNorm for decode-sized batches.
//
// Replaces "row-parallel GEMM -> all-reduce -> residual add -> RMSNorm" (reference:
// RowParallelLinear + all-reduce, vllm_neuron/nn/rpl.py:23-154, and the decode all-reduce
// sites of vllm_neuron/model/llama3/model.py:989,1113) after the local split-K GEMM has
// accumulated this rank's fp32 partial sums.  One CTA per token row:
//
//   1. read the fp32 partial row, clear it, round it to bf16 and store it into the receive
//      slot [parity][this rank][row] of every other rank (NVLink stores through CUDA-IPC
//      mapped symmetric memory);
//   2. fence at system scope, then release-store flag [parity][row][this rank] = epoch + 1 on
//      every rank;
//   3. wait (bounded) until every peer's flag for this row has reached epoch + 1;
//   4. residual += sum of the world's bf16 partials in rank order 0..world-1 (identical on
//      every rank), RMSNorm, and store the normalized row locally.
//
// Slots and flags alternate between two parities by call number: a rank can only be one call
// ahead of a peer (it needs that peer's flags to finish a call), so the parity it writes is
// never one the peer is still reading.  The call counter lives on the device (state[0]) so
// captured CUDA graphs replay correctly; the grid's last CTA advances it.  The signal count
// per call does not depend on the batch size, so consecutive calls may differ in T.  Every
// wait is bounded by %globaltimer; on expiry the kernel records a status code and carries on,
// and once the status is set later waits return at once (the host checks the status).
#include <cuda_bf16.h>

#include <stdexcept>

#include "../common.cuh"
#include "symm_mem.h"

namespace b200 {

__device__ __forceinline__ unsigned int ld_acquire_sys_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Returns false (and records `code`) if *f did not reach `target` within `timeout_ns`, or at
// once when an earlier wait already failed (status word set: fail fast, peers out of step).
__device__ __forceinline__ bool wait_flag(const unsigned int* f, unsigned int target,
                                          uint32_t* status, uint32_t code,
                                          uint64_t timeout_ns = B200_PEER_TIMEOUT_NS) {
  if ((int)(ld_acquire_sys_u32(f) - target) >= 0) return true;
  if (status != nullptr && *reinterpret_cast<volatile uint32_t*>(status) != 0u) return false;
  const uint64_t t0 = globaltimer_ns();
  while ((int)(ld_acquire_sys_u32(f) - target) < 0) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      set_status(status, code);
      return false;
    }
    __nanosleep(32);
  }
  return true;
}

template <int NV>
__global__ void __launch_bounds__(256) tp_allreduce_norm_kernel(const TPArNormParams p) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[8];
  __shared__ unsigned int epoch_s;
  const int tid = threadIdx.x;
  const int row = blockIdx.x;
  if (tid == 0) epoch_s = (unsigned int)*reinterpret_cast<volatile unsigned long long*>(&p.state[0]);
  __syncthreads();
  const unsigned int e = epoch_s;
  const int par = (int)(e & 1u);
  const long long slot_rows = (long long)p.world * p.max_rows;
  const long long row_off = ((long long)par * slot_rows + (long long)p.rank * p.max_rows + row) * p.H;

  // 1. partial row: fp32 -> bf16, cleared, pushed to every other rank's slot
  uint4 mine[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int idx = (j * 256 + tid) * 8;
    if (idx < p.H) {
      float4* src = reinterpret_cast<float4*>(p.acc + (long long)row * p.acc_stride + idx);
      const float4 a = src[0], b = src[1];
      src[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      src[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      mine[j] = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y),
                           pack_bf16x2(b.z, b.w));
      for (int r = 0; r < p.world; ++r)
        if (r != p.rank) *reinterpret_cast<uint4*>(p.recv_peers[r] + row_off + idx) = mine[j];
    }
  }
  __threadfence_system();
  __syncthreads();
  // 2. publish, 3. wait for every peer's row
  if (tid < p.world) {
    st_release_sys_u32(p.flag_peers[tid] + ((long long)par * p.max_rows + row) * p.world + p.rank,
                       e + 1u);
  }
  if (tid < p.world && tid != p.rank) {
    const unsigned int* f = p.flag_peers[p.rank] + ((long long)par * p.max_rows + row) * p.world + tid;
    wait_flag(f, e + 1u, p.status, kTimeoutPeerFlag);
  }
  __syncthreads();
  // 4. residual += sum of partials (rank order), RMSNorm
  const __nv_bfloat16* recv = p.recv_peers[p.rank];
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int idx = (j * 256 + tid) * 8;
    if (idx < p.H) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      for (int r = 0; r < p.world; ++r) {
        uint4 s;
        if (r == p.rank) {
          s = mine[j];
        } else {
          s = __ldcv(reinterpret_cast<const uint4*>(
              recv + ((long long)par * slot_rows + (long long)r * p.max_rows + row) * p.H + idx));
        }
        const uint32_t sw[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = unpack_bf16x2(sw[i]);
          acc[2 * i] += f.x;
          acc[2 * i + 1] += f.y;
        }
      }
      __nv_bfloat16* res = p.residual + (long long)row * p.res_stride + idx;
      const uint4 rv = *reinterpret_cast<const uint4*>(res);
      const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(rw[i]);
        // the all-reduced projection is rounded to bf16 before the residual add
        v[j][2 * i] = __bfloat162float(__float2bfloat16(acc[2 * i])) + f.x;
        v[j][2 * i + 1] = __bfloat162float(__float2bfloat16(acc[2 * i + 1])) + f.y;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        v[j][k] = __bfloat162float(__float2bfloat16(v[j][k]));
        ss += v[j][k] * v[j][k];
      }
      *reinterpret_cast<uint4*>(res) =
          make_uint4(pack_bf16x2(v[j][0], v[j][1]), pack_bf16x2(v[j][2], v[j][3]),
                     pack_bf16x2(v[j][4], v[j][5]), pack_bf16x2(v[j][6], v[j][7]));
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += red[w];
  const float inv = rsqrtf(t / (float)p.H + p.eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int idx = (j * 256 + tid) * 8;
    if (idx < p.H) {
      const uint4 g = *reinterpret_cast<const uint4*>(p.w + idx);
      const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(gw[i]);
        o[i] = pack_bf16x2(v[j][2 * i] * inv * f.x, v[j][2 * i + 1] * inv * f.y);
      }
      *reinterpret_cast<uint4*>(p.out + (long long)row * p.out_stride + idx) =
          make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  // the grid's last CTA advances the call counter
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&p.state[1], 1ull) == (unsigned long long)(gridDim.x - 1)) {
      p.state[1] = 0;
      __threadfence();
      p.state[0] = (unsigned long long)e + 1ull;
    }
  }
}

// Sentinel form (default).  The receive slots hold the bf16 pattern 0x8000 (negative zero)
// wherever no data has arrived, so the data is its own flag: a rank stores its partial row
// straight into every rank's slot [call % 3][this rank][row] (bf16, a partial that rounds to
// -0.0 is stored as +0.0), and the reader polls its own slots until no half-word of its 16-byte
// vector is the sentinel -- no memory fence, no flag store, no separate flag round trip.  The
// slots of the previous call are reset to the sentinel during this call (rows [0, T_prev) of
// every source, T_prev kept in state[2]); with three slot sets a writer can never reach a set
// before its reader has reset it (a writer that starts call k + 2 has seen every rank's data
// of call k + 1, which each rank pushes only after finishing call k, whose kernel reset the
// set of call k - 1 = k + 2 mod 3).  One CTA per row; every poll is bounded by %globaltimer.
__device__ __forceinline__ uint4 ld_volatile_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ bool has_sentinel(uint32_t w) {
  return (w & 0xffffu) == 0x8000u || (w >> 16) == 0x8000u;
}
__device__ __forceinline__ uint32_t no_neg_zero(uint32_t w) {
  if ((w & 0xffffu) == 0x8000u) w &= 0xffff0000u;
  if ((w >> 16) == 0x8000u) w &= 0x0000ffffu;
  return w;
}

template <int NV>
__global__ void __launch_bounds__(512) tp_allreduce_norm_lamport_kernel(const TPArNormParams p) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[16];
  __shared__ unsigned long long st_s[2];
  const int tid = threadIdx.x;
  const int row = blockIdx.x;
  if (tid == 0) {
    st_s[0] = *reinterpret_cast<volatile unsigned long long*>(&p.state[0]);
    st_s[1] = *reinterpret_cast<volatile unsigned long long*>(&p.state[2]);
  }
  __syncthreads();
  const unsigned long long e = st_s[0];
  const int T_prev = (int)st_s[1];
  const int ph = (int)(e % 3ull);
  const int ph_prev = (ph + 2) % 3;
  const long long set_elems = (long long)p.world * p.max_rows * p.H;  // one slot set
  const long long src_elems = (long long)p.max_rows * p.H;             // one source's slot
  __nv_bfloat16* own = p.recv_peers[p.rank];

  // 1. push this row's partial into every rank's slot (own included)
  const long long my_off = (long long)ph * set_elems + (long long)p.rank * src_elems + (long long)row * p.H;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int idx = (j * 512 + tid) * 8;
    if (idx < p.H) {
      float4* src = reinterpret_cast<float4*>(p.acc + (long long)row * p.acc_stride + idx);
      const float4 a = src[0], b = src[1];
      src[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      src[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      const uint4 m = make_uint4(no_neg_zero(pack_bf16x2(a.x, a.y)), no_neg_zero(pack_bf16x2(a.z, a.w)),
                                 no_neg_zero(pack_bf16x2(b.x, b.y)), no_neg_zero(pack_bf16x2(b.z, b.w)));
      for (int r = 0; r < p.world; ++r) *reinterpret_cast<uint4*>(p.recv_peers[r] + my_off + idx) = m;
    }
  }
  // 2. reset the previous call's slot set (rows [0, T_prev) of every source, grid-stride)
  const uint4 sent = make_uint4(0x80008000u, 0x80008000u, 0x80008000u, 0x80008000u);
  for (int r = row; r < T_prev; r += gridDim.x) {
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int idx = (j * 512 + tid) * 8;
      if (idx < p.H) {
        for (int s = 0; s < p.world; ++s)
          *reinterpret_cast<uint4*>(own + (long long)ph_prev * set_elems + (long long)s * src_elems +
                                    (long long)r * p.H + idx) = sent;
      }
    }
  }
  // 3. poll every source's vector until it has fully arrived, sum in rank order
  bool failed = *reinterpret_cast<volatile uint32_t*>(p.status) != 0u;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int idx = (j * 512 + tid) * 8;
    if (idx < p.H) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      for (int s = 0; s < p.world; ++s) {
        const __nv_bfloat16* q = own + (long long)ph * set_elems + (long long)s * src_elems +
                                 (long long)row * p.H + idx;
        uint4 x = ld_volatile_v4(q);
        if (has_sentinel(x.x) || has_sentinel(x.y) || has_sentinel(x.z) || has_sentinel(x.w)) {
          const uint64_t t0 = globaltimer_ns();
          uint32_t n = 0;
          while (!failed) {
            x = ld_volatile_v4(q);
            if (!(has_sentinel(x.x) || has_sentinel(x.y) || has_sentinel(x.z) || has_sentinel(x.w))) break;
            if ((++n & 63u) == 0 && globaltimer_ns() - t0 > B200_PEER_TIMEOUT_NS) {
              set_status(p.status, kTimeoutPeerFlag);
              failed = true;
            }
          }
        }
        const uint32_t sw[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = unpack_bf16x2(sw[i]);
          acc[2 * i] += f.x;
          acc[2 * i + 1] += f.y;
        }
      }
      __nv_bfloat16* res = p.residual + (long long)row * p.res_stride + idx;
      const uint4 rv = *reinterpret_cast<const uint4*>(res);
      const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(rw[i]);
        v[j][2 * i] = __bfloat162float(__float2bfloat16(acc[2 * i])) + f.x;
        v[j][2 * i + 1] = __bfloat162float(__float2bfloat16(acc[2 * i + 1])) + f.y;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        v[j][k] = __bfloat162float(__float2bfloat16(v[j][k]));
        ss += v[j][k] * v[j][k];
      }
      *reinterpret_cast<uint4*>(res) =
          make_uint4(pack_bf16x2(v[j][0], v[j][1]), pack_bf16x2(v[j][2], v[j][3]),
                     pack_bf16x2(v[j][4], v[j][5]), pack_bf16x2(v[j][6], v[j][7]));
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < 16; ++w) t += red[w];
  const float inv = rsqrtf(t / (float)p.H + p.eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int idx = (j * 512 + tid) * 8;
    if (idx < p.H) {
      const uint4 g = *reinterpret_cast<const uint4*>(p.w + idx);
      const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(gw[i]);
        o[i] = pack_bf16x2(v[j][2 * i] * inv * f.x, v[j][2 * i + 1] * inv * f.y);
      }
      *reinterpret_cast<uint4*>(p.out + (long long)row * p.out_stride + idx) =
          make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  // the grid's last CTA advances the call counter and records this call's row count
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&p.state[1], 1ull) == (unsigned long long)(gridDim.x - 1)) {
      p.state[1] = 0;
      p.state[2] = (unsigned long long)p.T;
      __threadfence();
      p.state[0] = e + 1ull;
    }
  }
}

// One-thread probe of the fused collectives' bounded peer-flag wait (failure-detection test):
// waits for *flag to reach `target` for at most `timeout_ns`; a flag that no peer sets makes
// the wait expire, record kTimeoutPeerFlag in the status word and return -- the context stays
// usable.  result[0] = 1 if the flag arrived, 0 if the wait gave up.
__global__ void flag_wait_probe_kernel(const unsigned int* flag, unsigned int target,
                                       unsigned long long timeout_ns, uint32_t* status, int* result) {
  if (threadIdx.x == 0 && blockIdx.x == 0)
    *result = wait_flag(flag, target, status, kTimeoutPeerFlag, timeout_ns) ? 1 : 0;
}

void flag_wait_probe_launch(const unsigned int* flag, unsigned int target, unsigned long long timeout_ns,
                            uint32_t* status, int* result, cudaStream_t stream) {
  if (timeout_ns > 5000000000ull) throw std::invalid_argument("flag_wait_probe: timeout above 5 s");
  flag_wait_probe_kernel<<<1, 32, 0, stream>>>(flag, target, timeout_ns, status, result);
}

void tp_allreduce_norm_launch(const TPArNormParams& p, cudaStream_t stream) {
  if (p.H % 8 != 0) throw std::invalid_argument("tp_allreduce_norm: H must be a multiple of 8");
  if (p.T > p.max_rows) throw std::invalid_argument("tp_allreduce_norm: too many rows");
  if (p.world < 2 || p.world > kMaxTP) throw std::invalid_argument("tp_allreduce_norm: bad world");
  if (p.T == 0) return;
  if (p.algo == 0) {
    const int nv = (p.H / 8 + 511) / 512;
    const dim3 grid(p.T);
    if (nv <= 1)
      launch_pdl(tp_allreduce_norm_lamport_kernel<1>, grid, dim3(512), 0, stream, p);
    else if (nv <= 2)
      launch_pdl(tp_allreduce_norm_lamport_kernel<2>, grid, dim3(512), 0, stream, p);
    else if (nv <= 4)
      launch_pdl(tp_allreduce_norm_lamport_kernel<4>, grid, dim3(512), 0, stream, p);
    else
      throw std::invalid_argument("tp_allreduce_norm: hidden size too large");
    return;
  }
  const int nv = (p.H / 8 + 255) / 256;
  const dim3 grid(p.T);
  if (nv <= 1)
    launch_pdl(tp_allreduce_norm_kernel<1>, grid, dim3(256), 0, stream, p);
  else if (nv <= 2)
    launch_pdl(tp_allreduce_norm_kernel<2>, grid, dim3(256), 0, stream, p);
  else if (nv <= 4)
    launch_pdl(tp_allreduce_norm_kernel<4>, grid, dim3(256), 0, stream, p);
  else
    throw std::invalid_argument("tp_allreduce_norm: hidden size too large");
}

}  // namespace b200
