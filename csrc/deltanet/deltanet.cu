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
//   gated_delta_rule   a per-token pass computes the q / k inverse norms and the gates; then
//                      per (sequence, value head, 32 value columns) one CTA of 4 warps; a warp
//                      keeps 8 columns of S in registers (16 rows x 2 columns per lane) and
//                      reduces over dk with shuffles, so tokens are processed in order (the
//                      recurrence) without CTA barriers, next-token inputs prefetched; the
//                      gated RMSNorm over dv runs afterwards (one warp per token and head).
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

// Per token: the inverse l2 norms of q and k of every key head and the decay / write strength
// of every value head, packed per value head as gb[t, h] = (g, beta, 1/|q|, 1/|k|) with
// g = exp(-exp(A_log) * softplus(a + dt_bias)) and beta = sigmoid(b).  Hoisting these out of
// the recurrence removes the reductions every value column used to repeat; q and k stay
// unmodified (the recurrence applies the fp32 factors).
__global__ void __launch_bounds__(256) gdn_prepare_kernel(const GatedDeltaParams p) {
  pdl_trigger();
  pdl_wait();
  __shared__ float inv_norm[2 * 64];  // q heads then k heads (Hk <= 64)
  const long long t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const __nv_bfloat16* row = p.qkv + t * p.ld_qkv;
  for (int h = warp; h < 2 * p.Hk; h += blockDim.x >> 5) {
    const uint2 u = *reinterpret_cast<const uint2*>(row + (long long)h * 128 + lane * 4);
    const float2 f0 = unpack_bf16x2(u.x), f1 = unpack_bf16x2(u.y);
    float ss = f0.x * f0.x + f0.y * f0.y + f1.x * f1.x + f1.y * f1.y;
    ss = warp_sum(ss);
    if (lane == 0) inv_norm[h] = rsqrtf(ss + 1e-6f);
  }
  __syncthreads();
  const int rep = p.Hv / p.Hk;
  for (int h = threadIdx.x; h < p.Hv; h += blockDim.x) {
    const float a = __bfloat162float(p.a[t * p.ld_zab + h]);
    const float bb = __bfloat162float(p.b[t * p.ld_zab + h]);
    const float g = __expf(-__expf(p.A_log[h]) * softplus_d(a + p.dt_bias[h]));
    const int kh = h / rep;
    p.gb[t * p.Hv + h] = make_float4(g, 1.f / (1.f + __expf(-bb)), inv_norm[kh], inv_norm[p.Hk + kh]);
  }
}

// dk = dv = 128.  The recurrence of value column v only reads column v of S, so columns are
// independent: lane = 8 * c + kg holds rows [16 kg, 16 kg + 16) of the two columns 2c, 2c + 1
// of its warp's 8 (32 state floats), so one unpack of the token's q and k serves two columns.
// Every k-reduction (S^T k and S^T q) is 3 butterfly shuffles inside the warp: a token costs
// no CTA barrier; the next token's inputs are loaded while the current one is processed.
// Output: the un-normalised o (bf16), normalised afterwards by gated_rmsnorm_kernel.
// 4 warps per CTA = 32 columns.
constexpr int kGdnColsPerWarp = 8;
constexpr int kGdnWarps = 4;

__global__ void __launch_bounds__(128) gated_delta_rule_kernel(const GatedDeltaParams p,
                                                                LinearAttnBatch bt) {
  constexpr int DK = 128, DV = 128, R = 16;
  constexpr unsigned FULL = 0xffffffffu;
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kg = lane & 7;
  const int v0 = (blockIdx.z * kGdnWarps + warp) * kGdnColsPerWarp + 2 * (lane >> 3);
  const int kh = h / (p.Hv / p.Hk);
  const int t0 = bt.q_start[b];
  const int n = bt.q_start[b + 1] - t0;
  const int ctx = bt.seq_lens[b] - n;
  float* S = p.state + (long long)bt.slots[b] * p.state_slot_stride + (long long)h * DK * DV;
  float s0[R], s1[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float2 sv = make_float2(0.f, 0.f);
    if (ctx > 0) sv = *reinterpret_cast<const float2*>(S + (long long)(kg * R + r) * DV + v0);
    s0[r] = sv.x;
    s1[r] = sv.y;
  }
  const float qscale = rsqrtf((float)DK);
  const long long q_off = (long long)kh * DK + kg * R;
  const long long k_off = (long long)p.Hk * DK + q_off;
  const long long v_off = 2LL * p.Hk * DK + (long long)h * DV + v0;

  uint4 nq[2], nk[2];
  uint32_t nv = 0;
  float4 ngb = make_float4(0.f, 0.f, 0.f, 0.f);
  auto load = [&](long long t) {
    const uint4* q4 = reinterpret_cast<const uint4*>(p.qkv + t * p.ld_qkv + q_off);
    const uint4* k4 = reinterpret_cast<const uint4*>(p.qkv + t * p.ld_qkv + k_off);
    nq[0] = q4[0];
    nq[1] = q4[1];
    nk[0] = k4[0];
    nk[1] = k4[1];
    nv = *reinterpret_cast<const uint32_t*>(p.qkv + t * p.ld_qkv + v_off);
    ngb = p.gb[t * p.Hv + h];
  };
  if (n > 0) load(t0);
  for (int i = 0; i < n; ++i) {
    const long long t = t0 + i;
    float q[R], k[R];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t qw[4] = {nq[j].x, nq[j].y, nq[j].z, nq[j].w};
      const uint32_t kw[4] = {nk[j].x, nk[j].y, nk[j].z, nk[j].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fq = unpack_bf16x2(qw[e]), fk = unpack_bf16x2(kw[e]);
        q[8 * j + 2 * e] = fq.x;
        q[8 * j + 2 * e + 1] = fq.y;
        k[8 * j + 2 * e] = fk.x;
        k[8 * j + 2 * e + 1] = fk.y;
      }
    }
    const float2 vt = unpack_bf16x2(nv);
    const float g = ngb.x, beta = ngb.y, iq = ngb.z * qscale, ik = ngb.w;
    if (i + 1 < n) load(t + 1);
#pragma unroll
    for (int r = 0; r < R; ++r) k[r] *= ik;
    // kv = (g S)^T k for both columns
    float kv0 = 0.f, kv1 = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      kv0 += s0[r] * k[r];
      kv1 += s1[r] * k[r];
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      kv0 += __shfl_xor_sync(FULL, kv0, o);
      kv1 += __shfl_xor_sync(FULL, kv1, o);
    }
    const float d0 = (vt.x - g * kv0) * beta, d1 = (vt.y - g * kv1) * beta;
    float o0 = 0.f, o1 = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      s0[r] = fmaf(g, s0[r], k[r] * d0);
      s1[r] = fmaf(g, s1[r], k[r] * d1);
      o0 += s0[r] * q[r];
      o1 += s1[r] * q[r];
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      o0 += __shfl_xor_sync(FULL, o0, o);
      o1 += __shfl_xor_sync(FULL, o1, o);
    }
    if (kg == 0)
      *reinterpret_cast<uint32_t*>(p.out + t * p.ld_out + (long long)h * DV + v0) =
          pack_bf16x2(o0 * iq, o1 * iq);
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
    *reinterpret_cast<float2*>(S + (long long)(kg * R + r) * DV + v0) = make_float2(s0[r], s1[r]);
}

// out[t, h, :] = w * rmsnorm(out[t, h, :]) * silu(z[t, h, :]) over dv = 128 (one warp per row;
// the normalised value is rounded to bf16 before the weight, as in the reference order).
__global__ void gated_rmsnorm_kernel(__nv_bfloat16* __restrict__ out, long long ld_out,
                                     const __nv_bfloat16* __restrict__ z, long long ld_z,
                                     const __nv_bfloat16* __restrict__ w, int Hv, int rows, float eps) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const long long t = row / Hv;
  const int h = row - (int)t * Hv;
  __nv_bfloat16* o = out + t * ld_out + (long long)h * 128 + lane * 4;
  const __nv_bfloat16* zz = z + t * ld_z + (long long)h * 128 + lane * 4;
  const uint2 ov = *reinterpret_cast<const uint2*>(o);
  const uint2 zv = *reinterpret_cast<const uint2*>(zz);
  const uint2 wv = *reinterpret_cast<const uint2*>(w + lane * 4);
  const float2 o0 = unpack_bf16x2(ov.x), o1 = unpack_bf16x2(ov.y);
  const float2 z0 = unpack_bf16x2(zv.x), z1 = unpack_bf16x2(zv.y);
  const float2 w0 = unpack_bf16x2(wv.x), w1 = unpack_bf16x2(wv.y);
  const float x[4] = {o0.x, o0.y, o1.x, o1.y}, zf[4] = {z0.x, z0.y, z1.x, z1.y},
              wf[4] = {w0.x, w0.y, w1.x, w1.y};
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / 128.f + eps);
  float y[4];
#pragma unroll
  for (int e = 0; e < 4; ++e)
    y[e] = wf[e] * __bfloat162float(__float2bfloat16(x[e] * rstd)) * silu_d(zf[e]);
  *reinterpret_cast<uint2*>(o) = make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
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
  if (p.ld_qkv % 8 != 0 || p.ld_zab % 4 != 0 || p.ld_out % 4 != 0)
    throw std::invalid_argument("gated_delta_rule: row strides must allow vector loads");
  if (b.B == 0) return;
  if (p.Hk > 64) throw std::invalid_argument("gated_delta_rule: at most 64 key heads per rank");
  if (p.T > 0) launch_pdl(gdn_prepare_kernel, dim3(p.T), dim3(256), 0, s, p);
  constexpr int cols_per_cta = kGdnWarps * kGdnColsPerWarp;
  launch_pdl(gated_delta_rule_kernel, dim3(b.B, p.Hv, 128 / cols_per_cta), dim3(32 * kGdnWarps), 0,
             s, p, b);
  // rows of this step: tokens x value heads (token count from the host-side sizes)
  const int rows = p.T * p.Hv;
  if (rows > 0)
    launch_pdl(gated_rmsnorm_kernel, dim3((rows + 7) / 8), dim3(256), 0, s, p.out, p.ld_out, p.z,
               p.ld_zab, p.norm_w, p.Hv, rows, p.eps);
}

void sigmoid_gate_mul_launch(__nv_bfloat16* x, long long ldx, const __nv_bfloat16* gate,
                             long long ldg, int T, int n, cudaStream_t s) {
  if (T == 0) return;
  launch_pdl(sigmoid_gate_mul_kernel, dim3(T), dim3(256), 0, s, x, ldx, gate, ldg, n);
}

}  // namespace b200
