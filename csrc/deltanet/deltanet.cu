// Gated DeltaNet (linear attention) kernels for the hybrid Qwen3.5/3.6-style models.
//
// The reference has no linear-attention code; these follow the published gated delta rule
// (Yang, Kautz, Hatamizadeh, "Gated Delta Networks: Improving Mamba2 with Delta Rule", 2024):
//
//   S_t = g_t * S_{t-1} + k_t (beta_t * (v_t - (g_t * S_{t-1})^T k_t))^T,   o_t = S_t^T q_t
//
// with per-head state S [dk, dv], q/k l2-normalised and q scaled by dk^-1/2, the decay
// g = exp(-exp(A_log) * softplus(a + dt_bias)) and beta = sigmoid(b), followed by a gated
// RMSNorm of o_t over dv.  Inputs come from a depthwise causal conv1d (kernel K, SiLU) over the
// q|k|v channels; both the conv window and S persist per request in a state cache, so chunked
// prefill and decode continue where the previous step stopped.
//
//   causal_conv1d      one thread per channel, a sliding window of K - 1 inputs in registers,
//                      loads of the step's tokens unrolled so they are in flight together.
//   gated_delta_rule   one CTA (256 threads) per (sequence, value head); thread (v, half) keeps
//                      column v, rows [64 * half, 64 * half + 64) of S in registers; per token
//                      two k-reductions go through shared memory; the gated RMSNorm over dv is
//                      a CTA reduction.  Tokens are processed in order (the recurrence), with
//                      the next token's inputs prefetched; the work is spread over
//                      sequences x heads.
#include <cuda_bf16.h>

#include <stdexcept>

#include "../common.cuh"
#include "deltanet.h"

namespace b200 {

namespace {

__device__ __forceinline__ float silu_d(float x) { return x / (1.f + __expf(-x)); }
__device__ __forceinline__ float softplus_d(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

}  // namespace

template <int K>
__global__ void __launch_bounds__(128) causal_conv1d_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, int C, const __nv_bfloat16* __restrict__ w,
    LinearAttnBatch bt, __nv_bfloat16* __restrict__ state, long long sss,
    __nv_bfloat16* __restrict__ y, long long ldy) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int t0 = bt.q_start[b];
  const int n = bt.q_start[b + 1] - t0;
  const int ctx = bt.seq_lens[b] - n;
  __nv_bfloat16* st = state + (long long)bt.slots[b] * sss + (long long)c * (K - 1);
  float wv[K], win[K - 1];
#pragma unroll
  for (int j = 0; j < K; ++j) wv[j] = __bfloat162float(w[(long long)c * K + j]);
#pragma unroll
  for (int j = 0; j < K - 1; ++j) win[j] = ctx > 0 ? __bfloat162float(st[j]) : 0.f;
  constexpr int U = 8;
  for (int i0 = 0; i0 < n; i0 += U) {
    float xin[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      xin[u] = i0 + u < n ? __bfloat162float(x[(long long)(t0 + i0 + u) * ldx + c]) : 0.f;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (i0 + u < n) {
        float acc = wv[K - 1] * xin[u];
#pragma unroll
        for (int j = 0; j < K - 1; ++j) acc += wv[j] * win[j];
        y[(long long)(t0 + i0 + u) * ldy + c] = __float2bfloat16(silu_d(acc));
#pragma unroll
        for (int j = 0; j < K - 2; ++j) win[j] = win[j + 1];
        win[K - 2] = xin[u];
      }
    }
  }
#pragma unroll
  for (int j = 0; j < K - 1; ++j) st[j] = __float2bfloat16(win[j]);
}

// dk = dv = 128, 256 threads.  The inputs of token i + 1 are loaded while token i is
// processed (they do not depend on the state), and the shared-memory exchanges use separate
// buffers per phase so one token costs five CTA barriers.
__global__ void __launch_bounds__(256) gated_delta_rule_kernel(const GatedDeltaParams p,
                                                                LinearAttnBatch bt) {
  constexpr int DK = 128, DV = 128, R = 64;  // rows of S per thread
  pdl_trigger();
  pdl_wait();
  __shared__ float qs[DK], ks[DK];
  __shared__ float red_kv[2][DV], red_o[2][DV];
  __shared__ float wsum_qk[8], wsum_o[8];
  const int b = blockIdx.x;
  const int h = blockIdx.y;
  const int tid = threadIdx.x;
  const int v = tid & (DV - 1);
  const int half = tid >> 7;
  const int kh = h / (p.Hv / p.Hk);
  const int t0 = bt.q_start[b];
  const int n = bt.q_start[b + 1] - t0;
  const int ctx = bt.seq_lens[b] - n;
  float* S = p.state + (long long)bt.slots[b] * p.state_slot_stride + (long long)h * DK * DV;
  float s[R];
#pragma unroll
  for (int r = 0; r < R; ++r) s[r] = ctx > 0 ? S[(long long)(half * R + r) * DV + v] : 0.f;
  const float A = -__expf(p.A_log[h]);
  const float dtb = p.dt_bias[h];
  const float nw = __bfloat162float(p.norm_w[v]);
  const float qscale = rsqrtf((float)DK);
  const int warp = tid >> 5, lane = tid & 31;
  const int d = tid & (DK - 1);
  const long long qk_off = (half ? p.Hk * DK : 0) + (long long)kh * DK + d;
  const long long v_off = 2 * p.Hk * DK + (long long)h * DV + v;
  const long long z_off = (long long)h * DV + v;

  // per-token inputs of this thread: its q or k element, v element, z element, a, b
  float n_qk = 0.f, n_v = 0.f, n_z = 0.f, n_a = 0.f, n_b = 0.f;
  auto load = [&](long long t) {
    n_qk = __bfloat162float(p.qkv[t * p.ld_qkv + qk_off]);
    n_v = __bfloat162float(p.qkv[t * p.ld_qkv + v_off]);
    n_z = half == 0 ? __bfloat162float(p.z[t * p.ld_zab + z_off]) : 0.f;
    n_a = __bfloat162float(p.a[t * p.ld_zab + h]);
    n_b = __bfloat162float(p.b[t * p.ld_zab + h]);
  };
  if (n > 0) load(t0);

  for (int i = 0; i < n; ++i) {
    const long long t = t0 + i;
    const float val = n_qk, vt = n_v, zt = n_z, a = n_a, bb = n_b;
    if (i + 1 < n) load(t + 1);
    // q (threads 0..127) and k (threads 128..255), l2-normalised over dk
    const float ss = warp_sum(val * val);
    if (lane == 0) wsum_qk[warp] = ss;
    __syncthreads();  // A
    {
      const float tot = half ? wsum_qk[4] + wsum_qk[5] + wsum_qk[6] + wsum_qk[7]
                             : wsum_qk[0] + wsum_qk[1] + wsum_qk[2] + wsum_qk[3];
      const float inv = rsqrtf(tot + 1e-6f);
      if (half) ks[d] = val * inv;
      else qs[d] = val * inv * qscale;
    }
    const float g = __expf(A * softplus_d(a + dtb));
    const float beta = 1.f / (1.f + __expf(-bb));
    __syncthreads();  // B
    float kv = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      s[r] *= g;
      kv += s[r] * ks[half * R + r];
    }
    red_kv[half][v] = kv;
    __syncthreads();  // C
    const float delta = (vt - (red_kv[0][v] + red_kv[1][v])) * beta;
    float o = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      s[r] += ks[half * R + r] * delta;
      o += s[r] * qs[half * R + r];
    }
    red_o[half][v] = o;
    __syncthreads();  // E
    // the recurrence output is rounded to the activation dtype before the gated RMSNorm
    const float ov = __bfloat162float(__float2bfloat16(red_o[0][v] + red_o[1][v]));
    const float sq = warp_sum(half == 0 ? ov * ov : 0.f);
    if (lane == 0) wsum_o[warp] = sq;
    __syncthreads();  // F
    if (half == 0) {
      const float tot = wsum_o[0] + wsum_o[1] + wsum_o[2] + wsum_o[3];
      const float rstd = rsqrtf(tot / (float)DV + p.eps);
      // reference order: normalise, cast, scale by the weight, then multiply by silu(z)
      const float nrm = __bfloat162float(__float2bfloat16(ov * rstd));
      p.out[t * p.ld_out + (long long)h * DV + v] = __float2bfloat16(nw * nrm * silu_d(zt));
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) S[(long long)(half * R + r) * DV + v] = s[r];
}

__global__ void sigmoid_gate_mul_kernel(__nv_bfloat16* __restrict__ x, long long ldx,
                                        const __nv_bfloat16* __restrict__ gate, long long ldg,
                                        int n) {
  pdl_trigger();
  pdl_wait();
  const long long t = blockIdx.x;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float gv = __bfloat162float(gate[t * ldg + i]);
    const float xv = __bfloat162float(x[t * ldx + i]);
    x[t * ldx + i] = __float2bfloat16(xv / (1.f + __expf(-gv)));
  }
}

void causal_conv1d_launch(const __nv_bfloat16* x, long long ldx, int C, const __nv_bfloat16* w,
                          int K, const LinearAttnBatch& b, __nv_bfloat16* state,
                          long long state_slot_stride, __nv_bfloat16* y, long long ldy,
                          cudaStream_t s) {
  if (b.B == 0) return;
  const dim3 grid(b.B, (C + 127) / 128);
  if (K == 4)
    launch_pdl(causal_conv1d_kernel<4>, grid, dim3(128), 0, s, x, ldx, C, w, b, state,
               state_slot_stride, y, ldy);
  else if (K == 2)
    launch_pdl(causal_conv1d_kernel<2>, grid, dim3(128), 0, s, x, ldx, C, w, b, state,
               state_slot_stride, y, ldy);
  else if (K == 3)
    launch_pdl(causal_conv1d_kernel<3>, grid, dim3(128), 0, s, x, ldx, C, w, b, state,
               state_slot_stride, y, ldy);
  else
    throw std::invalid_argument("causal_conv1d: kernel size must be 2, 3 or 4");
}

void gated_delta_rule_launch(const GatedDeltaParams& p, const LinearAttnBatch& b, cudaStream_t s) {
  if (p.dk != 128 || p.dv != 128)
    throw std::invalid_argument("gated_delta_rule: head dims must be 128");
  if (p.Hv % p.Hk != 0) throw std::invalid_argument("gated_delta_rule: Hv % Hk != 0");
  if (b.B == 0) return;
  launch_pdl(gated_delta_rule_kernel, dim3(b.B, p.Hv), dim3(256), 0, s, p, b);
}

void sigmoid_gate_mul_launch(__nv_bfloat16* x, long long ldx, const __nv_bfloat16* gate,
                             long long ldg, int T, int n, cudaStream_t s) {
  if (T == 0) return;
  launch_pdl(sigmoid_gate_mul_kernel, dim3(T), dim3(256), 0, s, x, ldx, gate, ldg, n);
}

}  // namespace b200
