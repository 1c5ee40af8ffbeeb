// Expert-parallel token exchange over NVLink peer memory for MoE layers whose ranks hold
// different tokens (data-parallel attention replicas with experts sharded over the EP group).
//
// Replaces the host-driven all-to-all-v (count exchange, then two NCCL all-to-alls per
// direction; reference: NeuronAll2AllManager, vllm_neuron/parallel/all2all.py:113-517, with
// the reduce-scatter-v combine of functional/collectives/reduce_scatter_v.py:53,243) by four
// kernels that need no host round trip, so the whole exchange can be captured in a CUDA graph:
//
//   dispatch  (token owner, one CTA per token)  the token's destination ranks are the owners
//             of its top-k experts (deduplicated).  For each destination it takes a row slot
//             with one system-scope atomic on the destination's slot counter and stores, in
//             the destination's memory, the hidden row, the token's k expert ids (ids of other
//             ranks' experts replaced by -1), its k routing weights and (source, token).  The
//             last CTA raises disp_done[this rank] = epoch + 1 on every rank.
//   recv      (expert owner) waits for every source's disp_done, reads the row count R and
//             marks rows [R, rows_cap) as having no expert, so the expert pipeline (align,
//             grouped GEMMs, weighted top-k combine) runs on a static row bound.
//   return    (expert owner, after the experts) stores each reduced row into its token
//             owner's combine slot comb[token][this rank] and raises comb_done.
//   combine   (token owner) waits for every rank's comb_done and sums the token's slots of the
//             ranks it was sent to, in rank order (deterministic), into the output row.
//
// One set of buffers suffices.  A source writes a peer's receive rows for call k + 1 only
// after its own combine of call k, which waited for that peer's return kernel of call k, which
// ran after the peer's experts consumed the rows of call k; a peer writes a source's combine
// slots for call k + 1 only after its receive kernel of call k + 1, which waited for that
// source's dispatch of call k + 1, issued after the source's combine of call k.  The slot
// counter is reset by the return kernel (after the count was read, before comb_done is raised,
// so before any source can dispatch again).  Flags hold the call number (epoch + 1); the call
// counter lives on the device (state[0]) so captured CUDA graphs replay correctly, and the
// combine kernel's last CTA advances it.  Every wait is bounded by %globaltimer and records a
// status code.  No TMA load ever reads peer memory here: peers are written with plain stores.
#include <cuda_bf16.h>

#include <stdexcept>

#include "../common.cuh"
#include "ep_fused.h"

namespace b200 {

namespace {

__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until *f == target; returns false (status recorded) on expiry or at once when
// the status word is already set.
__device__ bool wait_eq(const unsigned int* f, unsigned int target, uint32_t* status) {
  if (ld_acquire_u32(f) == target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (*reinterpret_cast<volatile uint32_t*>(status) != 0u) return false;
    if (ld_acquire_u32(f) == target) return true;
    if (globaltimer_ns() - t0 > B200_PEER_TIMEOUT_NS) {
      set_status(status, kTimeoutPeerFlag);
      return false;
    }
    __nanosleep(64);
  }
}

// Per-rank symmetric layout (byte offsets from the allocation base; see ep_fused.h).
struct Lay {
  const EPExchangeParams& p;
  __device__ explicit Lay(const EPExchangeParams& q) : p(q) {}
  __device__ unsigned char* base(int r) const { return reinterpret_cast<unsigned char*>(p.peers[r]); }
  __device__ unsigned int* slot_ctr(int r) const {
    return reinterpret_cast<unsigned int*>(base(r) + p.off_ctrl);
  }
  __device__ unsigned int* disp_done(int r, int src) const {
    return reinterpret_cast<unsigned int*>(base(r) + p.off_ctrl) + 1 + src;
  }
  __device__ unsigned int* comb_done(int r, int src) const {
    return reinterpret_cast<unsigned int*>(base(r) + p.off_ctrl) + 1 + kMaxEP + src;
  }
  __device__ __nv_bfloat16* rows(int r) const {
    return reinterpret_cast<__nv_bfloat16*>(base(r) + p.off_rows);
  }
  __device__ int* ids(int r) const { return reinterpret_cast<int*>(base(r) + p.off_ids); }
  __device__ float* wts(int r) const { return reinterpret_cast<float*>(base(r) + p.off_w); }
  __device__ int* src(int r) const { return reinterpret_cast<int*>(base(r) + p.off_src); }
  __device__ __nv_bfloat16* comb(int r) const {
    return reinterpret_cast<__nv_bfloat16*>(base(r) + p.off_comb);
  }
};

__global__ void __launch_bounds__(256) ep_dispatch_kernel(const EPExchangeParams p) {
  pdl_trigger();
  pdl_wait();
  const Lay L(p);
  __shared__ int s_slot[kMaxEP];
  __shared__ unsigned int s_mask;
  __shared__ unsigned int s_epoch;
  const int tid = threadIdx.x;
  const int t = blockIdx.x;
  if (tid == 0) {
    s_epoch = (unsigned int)*reinterpret_cast<volatile unsigned long long*>(&p.state[0]);
    unsigned int mask = 0;
    if (t < p.T) {
      for (int j = 0; j < p.k; ++j) {
        const int e = p.topk_ids[(long long)t * p.k + j];
        if (e >= 0 && e < p.num_experts) mask |= 1u << (e / p.e_local);
      }
    }
    s_mask = mask;
  }
  if (tid < kMaxEP) s_slot[tid] = p.rows_cap;
  __syncthreads();
  const unsigned int e = s_epoch;
  const unsigned int mask = s_mask;
  if (t < p.T) {
    if (tid < p.world && ((mask >> tid) & 1u)) {
      const int d = tid;
      const int slot = (int)atomicAdd_system(L.slot_ctr(d), 1u);
      if (slot < p.rows_cap) {
        s_slot[d] = slot;
        int* idr = L.ids(d) + (long long)slot * p.k;
        float* wr = L.wts(d) + (long long)slot * p.k;
        for (int j = 0; j < p.k; ++j) {
          const int ex = p.topk_ids[(long long)t * p.k + j];
          const bool mine = ex >= 0 && ex < p.num_experts && ex / p.e_local == d;
          idr[j] = mine ? ex : -1;
          wr[j] = mine ? p.topk_w[(long long)t * p.k + j] : 0.f;
        }
        L.src(d)[slot] = (p.rank << 24) | t;
      } else {
        set_status(p.status, kBadIndex);  // more rows than the receive buffer holds
      }
    }
    __syncthreads();
    const int nvec = p.H >> 3;
    const uint4* xr = reinterpret_cast<const uint4*>(p.x + (long long)t * p.ldx);
    for (int d = 0; d < p.world; ++d) {
      if (!((mask >> d) & 1u) || s_slot[d] >= p.rows_cap) continue;
      uint4* dst = reinterpret_cast<uint4*>(L.rows(d) + (long long)s_slot[d] * p.H);
      for (int v = tid; v < nvec; v += blockDim.x) dst[v] = xr[v];
    }
  }
  __threadfence_system();
  __syncthreads();
  if (tid == 0) {
    if (atomicAdd(p.ctas_done, 1u) == gridDim.x - 1) {
      *p.ctas_done = 0u;
      __threadfence_system();
      for (int d = 0; d < p.world; ++d) st_release_u32(L.disp_done(d, p.rank), e + 1u);
    }
  }
}

__global__ void __launch_bounds__(256) ep_recv_kernel(const EPExchangeParams p) {
  pdl_trigger();
  pdl_wait();
  const Lay L(p);
  __shared__ unsigned int s_r;
  const int tid = threadIdx.x;
  const unsigned int e = (unsigned int)*reinterpret_cast<volatile unsigned long long*>(&p.state[0]);
  if (tid < p.world) wait_eq(L.disp_done(p.rank, tid), e + 1u, p.status);
  __syncthreads();
  if (tid == 0) {
    const unsigned int r = ld_acquire_u32(L.slot_ctr(p.rank));
    s_r = r < (unsigned int)p.rows_cap ? r : (unsigned int)p.rows_cap;
    if (blockIdx.x == 0) *p.recv_count = (int)s_r;
  }
  __syncthreads();
  const long long R = s_r;
  int* ids = L.ids(p.rank);
  const long long n = ((long long)p.rows_cap - R) * p.k;
  for (long long i = (long long)blockIdx.x * blockDim.x + tid; i < n; i += (long long)gridDim.x * blockDim.x)
    ids[R * p.k + i] = -1;
}

__global__ void __launch_bounds__(256) ep_return_kernel(const EPExchangeParams p) {
  pdl_trigger();
  pdl_wait();
  const Lay L(p);
  const int tid = threadIdx.x;
  const unsigned int e = (unsigned int)*reinterpret_cast<volatile unsigned long long*>(&p.state[0]);
  const int R = *p.recv_count;
  const int nvec = p.H >> 3;
  const int* src = L.src(p.rank);
  // the count was read by the receive kernel: reset the slot counter before comb_done lets
  // any source dispatch again
  if (blockIdx.x == 0 && tid == 0) *L.slot_ctr(p.rank) = 0u;
  for (int r = blockIdx.x; r < R; r += gridDim.x) {
    const int sv = src[r];
    const int s = sv >> 24, t = sv & 0xffffff;
    if (s >= p.world || t >= p.tokens_cap) {
      if (tid == 0) set_status(p.status, kBadIndex);
      continue;
    }
    const uint4* y = reinterpret_cast<const uint4*>(p.y + (long long)r * p.ldy);
    uint4* dst = reinterpret_cast<uint4*>(L.comb(s) + ((long long)t * p.world + p.rank) * p.H);
    for (int v = tid; v < nvec; v += blockDim.x) dst[v] = y[v];
  }
  __threadfence_system();
  __syncthreads();
  if (tid == 0) {
    if (atomicAdd(p.ctas_done, 1u) == gridDim.x - 1) {
      *p.ctas_done = 0u;
      __threadfence_system();
      for (int d = 0; d < p.world; ++d) st_release_u32(L.comb_done(d, p.rank), e + 1u);
    }
  }
}

__global__ void __launch_bounds__(256) ep_combine_kernel(const EPExchangeParams p) {
  pdl_trigger();
  pdl_wait();
  const Lay L(p);
  const int tid = threadIdx.x;
  const int t = blockIdx.x;
  const unsigned int e = (unsigned int)*reinterpret_cast<volatile unsigned long long*>(&p.state[0]);
  if (tid < p.world) wait_eq(L.comb_done(p.rank, tid), e + 1u, p.status);
  __syncthreads();
  if (t < p.T) {
    unsigned int mask = 0;
    for (int j = 0; j < p.k; ++j) {
      const int ex = p.topk_ids[(long long)t * p.k + j];
      if (ex >= 0 && ex < p.num_experts) mask |= 1u << (ex / p.e_local);
    }
    const __nv_bfloat16* c = L.comb(p.rank) + (long long)t * p.world * p.H;
    const int nvec = p.H >> 3;
    for (int v = tid; v < nvec; v += blockDim.x) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      for (int d = 0; d < p.world; ++d) {
        if (!((mask >> d) & 1u)) continue;
        const uint4 q = __ldcg(reinterpret_cast<const uint4*>(c + (long long)d * p.H) + v);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = unpack_bf16x2(w[i]);
          acc[2 * i] += f.x;
          acc[2 * i + 1] += f.y;
        }
      }
      reinterpret_cast<uint4*>(p.out + (long long)t * p.ldo)[v] =
          make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                     pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
    }
  }
  // the grid's last CTA advances the call counter
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.ctas_done, 1u) == gridDim.x - 1) {
      *p.ctas_done = 0u;
      __threadfence();
      p.state[0] = (unsigned long long)e + 1ull;
    }
  }
}

void check(const EPExchangeParams& p) {
  if (p.world < 1 || p.world > kMaxEP) throw std::invalid_argument("ep exchange: 1..8 ranks");
  if (p.H % 8 != 0) throw std::invalid_argument("ep exchange: hidden size must be a multiple of 8");
  if (p.T < 0 || p.T > p.tokens_cap)
    throw std::invalid_argument("ep exchange: more tokens than the buffers hold");
  if (p.tokens_cap >= (1 << 24)) throw std::invalid_argument("ep exchange: token capacity too large");
  if (p.e_local < 1 || p.num_experts != p.e_local * p.world)
    throw std::invalid_argument("ep exchange: experts must split evenly over the ranks");
  if (p.rows_cap != p.world * p.tokens_cap)
    throw std::invalid_argument("ep exchange: rows_cap must be world * tokens_cap");
}

}  // namespace

void ep_dispatch_launch(const EPExchangeParams& p, cudaStream_t s) {
  check(p);
  launch_pdl(ep_dispatch_kernel, dim3(p.T > 0 ? p.T : 1), dim3(256), 0, s, p);
}
void ep_recv_launch(const EPExchangeParams& p, cudaStream_t s) {
  check(p);
  int g = (int)(((long long)p.rows_cap * p.k + 255) / 256);
  g = g < 1 ? 1 : (g > 64 ? 64 : g);
  launch_pdl(ep_recv_kernel, dim3(g), dim3(256), 0, s, p);
}
void ep_return_launch(const EPExchangeParams& p, cudaStream_t s) {
  check(p);
  const int g = p.rows_cap < 1 ? 1 : (p.rows_cap > 4 * 148 ? 4 * 148 : p.rows_cap);
  launch_pdl(ep_return_kernel, dim3(g), dim3(256), 0, s, p);
}
void ep_combine_launch(const EPExchangeParams& p, cudaStream_t s) {
  check(p);
  launch_pdl(ep_combine_kernel, dim3(p.T > 0 ? p.T : 1), dim3(256), 0, s, p);
}

}  // namespace b200
