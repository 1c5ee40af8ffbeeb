// Mixture-of-experts routing on sm_100a: router top-k, grouping of the token->expert
// assignments by expert, row gather, expert activation and the weighted combine.  The expert
// matmuls themselves run on the grouped mode of the tcgen05 GEMM (gemm_sm100.cu), whose tile
// list moe_align writes.
//
//   route    one warp per token: scores from the router logits (+ bias), top-k selection by k
//            rounds of warp arg-max, weights by softmax / sigmoid (reference orderings:
//            vllm_neuron/functional/moe/router.py:19-71, GPT-OSS top-k then softmax).
//   align    one CTA: per-expert histogram, exclusive scan, 128-row tile list per expert and
//            the scatter of assignments into expert-contiguous rows (reference semantics:
//            build_blockwise_mapping, vllm_neuron/functional/moe/moe_blockwise.py:27 and
//            permute_routed_tokens, permute_routed_tokens.py:26).
//   gather   copies each assignment's token row into its expert-sorted row.
//   act      SwiGLU of the expert gate/up projection (plain SiLU or GPT-OSS clamped form with
//            alpha), per-expert bias.
//   combine  out[t] = g[t] * shared[t] + sum_j w[t, j] * (y[row(t, j)] + bias[e(t, j)]) in
//            j order (the reference's topk_reduce, vllm_neuron/functional/moe/topk_reduce.py:28;
//            shared is the optional shared expert, g its sigmoid gate from the router).
#include <cuda_bf16.h>

#include <stdexcept>

#include "../common.cuh"
#include "moe.h"

namespace b200 {

namespace {
constexpr int kMaxExpertsPerLane = 16;  // E <= 512
}

__global__ void moe_route_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                 const float* __restrict__ bias, int T, int E, int k, int mode,
                                 int renorm, int* __restrict__ ids, float* __restrict__ weights,
                                 float* __restrict__ shared_gate) {
  pdl_trigger();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const __nv_bfloat16* row = logits + (long long)warp * ld;
  // column E (when present) is the shared expert's gate logit
  if (shared_gate != nullptr && lane == 0)
    shared_gate[warp] = 1.f / (1.f + __expf(-__bfloat162float(row[E])));
  float v[kMaxExpertsPerLane];
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = i * 32 + lane;
    float x = -INFINITY;
    if (e < E) {
      x = __bfloat162float(row[e]);
      if (bias != nullptr) x += bias[e];
    }
    v[i] = x;
  }
  // score transform before selection
  if (mode == ROUTE_SOFTMAX_TOPK) {
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) mx = fmaxf(mx, v[i]);
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
      const float e = (i * 32 + lane < E) ? __expf(v[i] - mx) : 0.f;
      v[i] = (i * 32 + lane < E) ? e : -INFINITY;
      sum += e;
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i)
      if (i * 32 + lane < E) v[i] *= inv;
  } else if (mode == ROUTE_SIGMOID_TOPK) {
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i)
      if (i * 32 + lane < E) v[i] = 1.f / (1.f + __expf(-v[i]));
  }
  // k rounds of arg-max (ties -> lower expert id)
  float sel_v = 0.f;
  int sel_e = 0;
  float tot = 0.f, mx0 = 0.f;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
      const int e = i * 32 + lane;
      if (e < E && (v[i] > bv || (v[i] == bv && e < be))) {
        bv = v[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    // remove the winner
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i)
      if (i * 32 + lane == be) v[i] = -INFINITY;
    if (lane == r) {
      sel_v = bv;
      sel_e = be;
    }
    if (r == 0) mx0 = bv;
  }
  // weights of the k selected (lane r holds selection r)
  float w = 0.f;
  if (mode == ROUTE_TOPK_SOFTMAX) {
    w = lane < k ? __expf(sel_v - mx0) : 0.f;
    tot = warp_sum(w);
    w = w / tot;
  } else {
    w = lane < k ? sel_v : 0.f;
    if (renorm) {
      tot = warp_sum(w);
      w = tot > 0.f ? w / tot : 0.f;
    }
  }
  if (lane < k) {
    ids[(long long)warp * k + lane] = sel_e;
    weights[(long long)warp * k + lane] = w;
  }
}

__global__ void __launch_bounds__(1024) moe_align_kernel(const int* __restrict__ ids,
                                                          int n_assign, int e_start, int e_local,
                                                          int* offsets, int* sorted_src,
                                                          int* row_expert, int* inv_pos,
                                                          int4* gtiles, int* gcount, int gmax) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ int sh[];
  int* cnt = sh;             // [e_local]
  int* cur = sh + e_local;   // [e_local]
  for (int e = threadIdx.x; e < e_local; e += blockDim.x) {
    cnt[e] = 0;
    cur[e] = 0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n_assign; i += blockDim.x) {
    const int e = ids[i] - e_start;
    if (e >= 0 && e < e_local) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0, nt = 0;
    for (int e = 0; e < e_local; ++e) {
      offsets[e] = run;
      const int c = cnt[e];
      for (int r = 0; r < c; r += 128) {
        if (nt < gmax) gtiles[nt] = make_int4(e, run + r, run + c, 0);
        ++nt;
      }
      cur[e] = run;
      run += c;
    }
    offsets[e_local] = run;
    *gcount = nt < gmax ? nt : gmax;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n_assign; i += blockDim.x) {
    const int e = ids[i] - e_start;
    if (e >= 0 && e < e_local) {
      const int pos = atomicAdd(&cur[e], 1);
      sorted_src[pos] = i;
      row_expert[pos] = e;
      inv_pos[i] = pos;
    } else {
      inv_pos[i] = -1;
    }
  }
}

__global__ void moe_gather_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                  const int* __restrict__ sorted_src, int topk,
                                  const int* __restrict__ total, int H,
                                  __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  if (r >= *total) return;
  const int t = sorted_src[r] / topk;
  const uint4* src = reinterpret_cast<const uint4*>(x + (long long)t * ldx);
  uint4* dst = reinterpret_cast<uint4*>(out + (long long)r * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

__global__ void moe_act_kernel(const __nv_bfloat16* __restrict__ gu,
                               const __nv_bfloat16* __restrict__ bias,
                               const int* __restrict__ row_expert, const int* __restrict__ total,
                               int I, int mode, float alpha, float limit,
                               __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  if (r >= *total) return;
  const __nv_bfloat16* g = gu + (long long)r * 2 * I;
  const __nv_bfloat16* u = g + I;
  const __nv_bfloat16* bg = bias != nullptr ? bias + (long long)row_expert[r] * 2 * I : nullptr;
  for (int j = threadIdx.x; j < I; j += blockDim.x) {
    float a = __bfloat162float(g[j]);
    float b = __bfloat162float(u[j]);
    if (bg != nullptr) {
      // the projection (+ bias) is rounded to bf16 like the reference's bf16 linear
      a = __bfloat162float(__float2bfloat16(a + __bfloat162float(bg[j])));
      b = __bfloat162float(__float2bfloat16(b + __bfloat162float(bg[I + j])));
    }
    float y;
    if (mode == MOE_ACT_GPTOSS) {
      a = fminf(a, limit);
      b = fminf(fmaxf(b, -limit), limit);
      y = (b + 1.f) * (a / (1.f + __expf(-alpha * a)));
    } else {
      y = a / (1.f + __expf(-a)) * b;
    }
    out[(long long)r * I + j] = __float2bfloat16(y);
  }
}

__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y,
                                   const int* __restrict__ inv_pos,
                                   const float* __restrict__ weights, const int* __restrict__ ids,
                                   const __nv_bfloat16* __restrict__ bias, int e_start, int k,
                                   int H, const __nv_bfloat16* __restrict__ shared,
                                   long long ld_shared, const float* __restrict__ shared_gate,
                                   __nv_bfloat16* __restrict__ out, long long ldo) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const float sg = shared != nullptr ? (shared_gate != nullptr ? shared_gate[t] : 1.f) : 0.f;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float acc = 0.f;
    if (shared != nullptr) acc = sg * __bfloat162float(shared[(long long)t * ld_shared + c]);
    for (int j = 0; j < k; ++j) {
      const int pos = inv_pos[(long long)t * k + j];
      if (pos < 0) continue;
      float v = __bfloat162float(y[(long long)pos * H + c]);
      if (bias != nullptr) {
        const int e = ids[(long long)t * k + j] - e_start;
        v = __bfloat162float(__float2bfloat16(v + __bfloat162float(bias[(long long)e * H + c])));
      }
      acc += weights[(long long)t * k + j] * v;
    }
    out[(long long)t * ldo + c] = __float2bfloat16(acc);
  }
}

void moe_route_launch(const __nv_bfloat16* logits, long long ld, const float* bias, int T, int E,
                      int k, int mode, bool renorm, int* ids, float* weights, float* shared_gate,
                      cudaStream_t s) {
  if (E > 32 * kMaxExpertsPerLane) throw std::invalid_argument("moe_route: at most 512 experts");
  if (k < 1 || k > 32 || k > E) throw std::invalid_argument("moe_route: 1 <= k <= min(32, E)");
  if (T == 0) return;
  const int warps_per_block = 4;
  launch_pdl(moe_route_kernel, dim3((T + warps_per_block - 1) / warps_per_block),
             dim3(32 * warps_per_block), 0, s, logits, ld, bias, T, E, k, mode, renorm ? 1 : 0, ids,
             weights, shared_gate);
}

void moe_align_launch(const int* ids, int n_assign, int e_start, int e_local, int* offsets,
                      int* sorted_src, int* row_expert, int* inv_pos, int* gtiles, int* gcount,
                      int gmax, cudaStream_t s) {
  if (e_local < 1 || e_local > 4096) throw std::invalid_argument("moe_align: bad expert count");
  launch_pdl(moe_align_kernel, dim3(1), dim3(1024), 2 * e_local * sizeof(int), s, ids, n_assign,
             e_start, e_local, offsets, sorted_src, row_expert, inv_pos,
             reinterpret_cast<int4*>(gtiles), gcount, gmax);
}

void moe_gather_launch(const __nv_bfloat16* x, long long ldx, const int* sorted_src, int topk,
                       const int* total, int rows_cap, int H, __nv_bfloat16* out, cudaStream_t s) {
  if (H % 8 != 0 || ldx % 8 != 0) throw std::invalid_argument("moe_gather: H must be a multiple of 8");
  if (rows_cap == 0) return;
  launch_pdl(moe_gather_kernel, dim3(rows_cap), dim3(128), 0, s, x, ldx, sorted_src, topk, total,
             H, out);
}

void moe_act_launch(const __nv_bfloat16* gu, const __nv_bfloat16* bias, const int* row_expert,
                    const int* total, int rows_cap, int I, int mode, float alpha, float limit,
                    __nv_bfloat16* out, cudaStream_t s) {
  if (rows_cap == 0) return;
  launch_pdl(moe_act_kernel, dim3(rows_cap), dim3(256), 0, s, gu, bias, row_expert, total, I, mode,
             alpha, limit, out);
}

void moe_combine_launch(const __nv_bfloat16* y, const int* inv_pos, const float* weights,
                        const int* ids, const __nv_bfloat16* bias, int e_start, int T, int k,
                        int H, const __nv_bfloat16* shared, long long ld_shared,
                        const float* shared_gate, __nv_bfloat16* out, long long ldo,
                        cudaStream_t s) {
  if (T == 0) return;
  launch_pdl(moe_combine_kernel, dim3(T), dim3(256), 0, s, y, inv_pos, weights, ids, bias, e_start,
             k, H, shared, ld_shared, shared_gate, out, ldo);
}

}  // namespace b200
