// Mixture-of-experts routing on sm_100a: router top-k, grouping of the token->expert
// assignments by expert, row gather, expert activation and the weighted combine.  The expert
// matmuls themselves run on the grouped mode of the tcgen05 GEMM (gemm_sm100.cu), whose tile
// list moe_align writes.
//
//   route    one warp per token: scores from the router logits (+ bias), top-k selection by k
//            rounds of warp arg-max, weights by softmax / sigmoid (reference orderings:
//            vllm_neuron/functional/moe/router.py:19-71, GPT-OSS top-k then softmax); for
//            decode batches fused with the router GEMV (moe_router_topk).
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

#include <atomic>
#include <stdexcept>

#include "../common.cuh"
#include "moe.h"

namespace b200 {

namespace {
constexpr int kMaxExpertsPerLane = 16;  // E <= 512
}

// Routing of one token by one warp.  `logit(e)` returns the router logit of expert e (and of
// the shared expert's gate at e = E); the token's k choices go to ids_row / w_row.
template <typename LogitFn>
__device__ __forceinline__ void route_row(LogitFn logit, const float* __restrict__ bias, int E,
                                          int k, int mode, int renorm, float scale,
                                          int* __restrict__ ids_row, float* __restrict__ w_row,
                                          float* __restrict__ shared_gate_out) {
  const int lane = threadIdx.x & 31;
  // column E (when present) is the shared expert's gate logit
  if (shared_gate_out != nullptr && lane == 0) *shared_gate_out = 1.f / (1.f + __expf(-logit(E)));
  const bool bias_after = mode == ROUTE_SIGMOID_BIAS_TOPK;  // bias only ranks the experts
  float v[kMaxExpertsPerLane], raw[kMaxExpertsPerLane];
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = i * 32 + lane;
    float x = -INFINITY;
    if (e < E) {
      x = logit(e);
      if (bias != nullptr && !bias_after) x += bias[e];
    }
    v[i] = x;
  }
  if (bias_after) {
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
      const int e = i * 32 + lane;
      raw[i] = e < E ? 1.f / (1.f + __expf(-v[i])) : 0.f;
      v[i] = e < E ? raw[i] + (bias != nullptr ? bias[e] : 0.f) : -INFINITY;
    }
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
    float bv = -INFINITY, braw = 0.f;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
      const int e = i * 32 + lane;
      if (e < E && (v[i] > bv || (v[i] == bv && e < be))) {
        bv = v[i];
        be = e;
        if (bias_after) braw = raw[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      const float oraw = __shfl_xor_sync(0xffffffffu, braw, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
        braw = oraw;
      }
    }
    // remove the winner
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i)
      if (i * 32 + lane == be) v[i] = -INFINITY;
    if (lane == r) {
      sel_v = bias_after ? braw : bv;
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
    ids_row[lane] = sel_e;
    w_row[lane] = w * scale;
  }
}

__global__ void moe_route_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                 const float* __restrict__ bias, int T, int E, int k, int mode,
                                 int renorm, int* __restrict__ ids, float* __restrict__ weights,
                                 float* __restrict__ shared_gate, float scale) {
  pdl_trigger();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (warp >= T) return;
  const __nv_bfloat16* row = logits + (long long)warp * ld;
  route_row([&](int e) { return __bfloat162float(row[e]); }, bias, E, k, mode, renorm, scale,
            ids + (long long)warp * k, weights + (long long)warp * k,
            shared_gate != nullptr ? shared_gate + warp : nullptr);
}

// Decode-sized batches: router GEMV and top-k in one kernel.  One CTA per token: the token's
// row sits in shared memory (fp32), each warp computes the logits of every 8th router row
// (uint4 loads of the bf16 weights, warp reduction) rounded to bf16 as the GEMM path stores
// them (written to `logits` too), then warp 0 routes the token.  Counterpart of the
// reference's fused decode router (rmsnorm_router_topk_tkg,
// vllm_neuron/functional/moe/rmsnorm_router_topk_tkg.py:34) minus the norm, which this
// framework already fuses into the preceding all-reduce.
__global__ void __launch_bounds__(256, 1) moe_router_topk_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, const __nv_bfloat16* __restrict__ w,
    int rows, int H, const float* __restrict__ bias, int E, int k, int mode, int renorm,
    float scale, __nv_bfloat16* __restrict__ logits, long long ldl, int* __restrict__ ids,
    float* __restrict__ weights, float* __restrict__ shared_gate) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sm_router[];
  float* xs = sm_router;          // [H]
  float* lg = sm_router + H;      // [rows]
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const __nv_bfloat16* xr = x + (long long)t * ldx;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
    const uint32_t ws_[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf16x2(ws_[q]);
      xs[i + 2 * q] = f.x;
      xs[i + 2 * q + 1] = f.y;
    }
  }
  __syncthreads();
  for (int e = warp; e < rows; e += blockDim.x >> 5) {
    const __nv_bfloat16* wr = w + (long long)e * H;
    float acc = 0.f;
    for (int i = lane * 8; i < H; i += 32 * 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(wr + i);
      const uint32_t ws_[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(ws_[q]);
        acc += f.x * xs[i + 2 * q] + f.y * xs[i + 2 * q + 1];
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      const __nv_bfloat16 r = __float2bfloat16(acc);
      lg[e] = __bfloat162float(r);
      if (logits != nullptr) logits[(long long)t * ldl + e] = r;
    }
  }
  __syncthreads();
  if (warp == 0)
    route_row([&](int e) { return lg[e]; }, bias, E, k, mode, renorm, scale, ids + (long long)t * k,
              weights + (long long)t * k, shared_gate != nullptr ? shared_gate + t : nullptr);
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
  // Exclusive scans of the row counts and of the 128-row tile counts, 32 experts at a time
  // by warp 0 (carry kept in lane registers).
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int row_carry = 0, tile_carry = 0;
    for (int e0 = 0; e0 < e_local; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < e_local ? cnt[e] : 0;
      const int nt = (c + 127) / 128;
      int rs = c, ts = nt;  // inclusive scans
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int r2 = __shfl_up_sync(0xffffffffu, rs, o);
        const int t2 = __shfl_up_sync(0xffffffffu, ts, o);
        if (lane >= o) {
          rs += r2;
          ts += t2;
        }
      }
      const int row0 = row_carry + rs - c;
      const int tile0 = tile_carry + ts - nt;
      if (e < e_local) {
        offsets[e] = row0;
        cur[e] = row0;
        for (int r = 0; r < nt; ++r)
          if (tile0 + r < gmax) gtiles[tile0 + r] = make_int4(e, row0 + 128 * r, row0 + c, 0);
      }
      row_carry += __shfl_sync(0xffffffffu, rs, 31);
      tile_carry += __shfl_sync(0xffffffffu, ts, 31);
    }
    if (lane == 0) {
      offsets[e_local] = row_carry;
      *gcount = tile_carry < gmax ? tile_carry : gmax;
    }
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
  auto act = [&](float a, float b) {
    if (mode == MOE_ACT_GPTOSS) {
      a = fminf(a, limit);
      b = fminf(fmaxf(b, -limit), limit);
      return (b + 1.f) * (a / (1.f + __expf(-alpha * a)));
    }
    return a / (1.f + __expf(-a)) * b;
  };
  const bool vec = (I % 8) == 0;
  for (int j = threadIdx.x * (vec ? 8 : 1); j < I; j += blockDim.x * (vec ? 8 : 1)) {
    const int n = vec ? 8 : 1;
    float a[8], b[8];
    if (vec) {
      const uint4 ga = *reinterpret_cast<const uint4*>(g + j);
      const uint4 ub = *reinterpret_cast<const uint4*>(u + j);
      const uint32_t gw[4] = {ga.x, ga.y, ga.z, ga.w}, uw[4] = {ub.x, ub.y, ub.z, ub.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 fg = unpack_bf16x2(gw[q]), fu = unpack_bf16x2(uw[q]);
        a[2 * q] = fg.x;
        a[2 * q + 1] = fg.y;
        b[2 * q] = fu.x;
        b[2 * q + 1] = fu.y;
      }
    } else {
      a[0] = __bfloat162float(g[j]);
      b[0] = __bfloat162float(u[j]);
    }
    float y[8];
    for (int q = 0; q < n; ++q) {
      float av = a[q], bv = b[q];
      if (bg != nullptr) {
        // the projection (+ bias) is rounded to bf16 like the reference's bf16 linear
        av = __bfloat162float(__float2bfloat16(av + __bfloat162float(bg[j + q])));
        bv = __bfloat162float(__float2bfloat16(bv + __bfloat162float(bg[I + j + q])));
      }
      y[q] = act(av, bv);
    }
    __nv_bfloat16* o = out + (long long)r * I + j;
    if (vec) {
      *reinterpret_cast<uint4*>(o) = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                                                pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
    } else {
      o[0] = __float2bfloat16(y[0]);
    }
  }
}

__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y,
                                   const int* __restrict__ inv_pos,
                                   const float* __restrict__ weights, const int* __restrict__ ids,
                                   const __nv_bfloat16* __restrict__ bias, int e_start, int k,
                                   int H, const __nv_bfloat16* __restrict__ shared,
                                   long long ld_shared, const float* __restrict__ shared_gate,
                                   __nv_bfloat16* __restrict__ out, long long ldo, long long ldy) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const float sg = shared != nullptr ? (shared_gate != nullptr ? shared_gate[t] : 1.f) : 0.f;
  // 8 columns per thread, 16-byte loads (H % 8 == 0)
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8];
    if (shared != nullptr) {
      const uint4 u = *reinterpret_cast<const uint4*>(shared + (long long)t * ld_shared + c);
      const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(w4[q]);
        acc[2 * q] = sg * f.x;
        acc[2 * q + 1] = sg * f.y;
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    }
    for (int j = 0; j < k; ++j) {
      const int pos = inv_pos[(long long)t * k + j];
      if (pos < 0) continue;
      const float wt = weights[(long long)t * k + j];
      const uint4 u = *reinterpret_cast<const uint4*>(y + (long long)pos * ldy + c);
      const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
      float v[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(w4[q]);
        v[2 * q] = f.x;
        v[2 * q + 1] = f.y;
      }
      if (bias != nullptr) {
        const int e = ids[(long long)t * k + j] - e_start;
        const uint4 bu = *reinterpret_cast<const uint4*>(bias + (long long)e * H + c);
        const uint32_t b4[4] = {bu.x, bu.y, bu.z, bu.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(b4[q]);
          v[2 * q] = __bfloat162float(__float2bfloat16(v[2 * q] + f.x));
          v[2 * q + 1] = __bfloat162float(__float2bfloat16(v[2 * q + 1] + f.y));
        }
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += wt * v[q];
    }
    *reinterpret_cast<uint4*>(out + (long long)t * ldo + c) =
        make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                   pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
  }
}

void moe_route_launch(const __nv_bfloat16* logits, long long ld, const float* bias, int T, int E,
                      int k, int mode, bool renorm, int* ids, float* weights, float* shared_gate,
                      float scale, cudaStream_t s) {
  if (E > 32 * kMaxExpertsPerLane) throw std::invalid_argument("moe_route: at most 512 experts");
  if (k < 1 || k > 32 || k > E) throw std::invalid_argument("moe_route: 1 <= k <= min(32, E)");
  if (T == 0) return;
  const int warps_per_block = 4;
  launch_pdl(moe_route_kernel, dim3((T + warps_per_block - 1) / warps_per_block),
             dim3(32 * warps_per_block), 0, s, logits, ld, bias, T, E, k, mode, renorm ? 1 : 0, ids,
             weights, shared_gate, scale);
}

void moe_router_topk_launch(const __nv_bfloat16* x, long long ldx, const __nv_bfloat16* w, int rows,
                            int H, const float* bias, int T, int E, int k, int mode, bool renorm,
                            float scale, __nv_bfloat16* logits, long long ldl, int* ids,
                            float* weights, float* shared_gate, cudaStream_t s) {
  if (E > 32 * kMaxExpertsPerLane) throw std::invalid_argument("moe_router_topk: at most 512 experts");
  if (k < 1 || k > 32 || k > E) throw std::invalid_argument("moe_router_topk: 1 <= k <= min(32, E)");
  if (H % 8 != 0 || ldx % 8 != 0) throw std::invalid_argument("moe_router_topk: H must be a multiple of 8");
  if (rows < E || (shared_gate != nullptr && rows < E + 1))
    throw std::invalid_argument("moe_router_topk: router rows");
  const int smem = (H + rows) * (int)sizeof(float);
  if (smem > 200 * 1024) throw std::invalid_argument("moe_router_topk: hidden size too large");
  if (T == 0) return;
  static std::atomic<uint64_t> configured{0};
  // the shared-memory size depends on H: opt in once to the largest size any call may use
  set_max_dynamic_smem_once(moe_router_topk_kernel, 200 * 1024, configured);
  launch_pdl(moe_router_topk_kernel, dim3(T), dim3(256), smem, s, x, ldx, w, rows, H, bias, E, k,
             mode, renorm ? 1 : 0, scale, logits, ldl, ids, weights, shared_gate);
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
                        cudaStream_t s, long long ldy) {
  if (T == 0) return;
  if (ldy == 0) ldy = H;
  if (H % 8 != 0 || ldo % 8 != 0 || ldy % 8 != 0 || ldy < H || (shared != nullptr && ld_shared % 8 != 0))
    throw std::invalid_argument("moe_combine: hidden size and strides must be multiples of 8");
  launch_pdl(moe_combine_kernel, dim3(T), dim3(256), 0, s, y, inv_pos, weights, ids, bias, e_start,
             k, H, shared, ld_shared, shared_gate, out, ldo, ldy);
}

}  // namespace b200
