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
//   chunked form       prefill-sized steps: the WY form over 64-token chunks (below), with
//                      the intra-chunk products on the tensor cores and the state carried in
//                      fp32 across the chunks of a sequence.
#include <cuda_bf16.h>

#include <atomic>
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


// ------------------------------------------------------------------------------------------
// Chunked (WY) gated delta rule.  Within a chunk of L <= 64 tokens with entering state S0,
// lg_t = sum_{s<=t} log g_s (from the chunk start), gamma_t = exp(lg_t), unit-norm k^ and
// q^ (q^ also scaled by dk^-1/2), the per-token writes delta_t of the recurrence satisfy
//
//   (I + A) Delta = diag(beta) V - diag(beta gamma) K^ S0,  A[t,s] = beta_t e^{lg_t-lg_s} k^_t.k^_s (s<t)
//
// so Delta = U - W S0 with W = (I + A)^-1 diag(beta gamma) K^ and U = (I + A)^-1 diag(beta) V.
// Then  o_t = gamma_t S0^T q^_t + sum_{s<=t} e^{lg_t-lg_s} (q^_t.k^_s) delta_s   and
//       S_L = gamma_L S0 + sum_s e^{lg_L-lg_s} k^_s delta_s^T.
// gdn_chunk_prep_kernel computes W, U and the masked Q^K^T of every (chunk, value head) in
// parallel (K^K^T and Q^K^T on the tensor cores, the unit lower-triangular solve by forward
// substitution, one thread per right-hand-side column); gdn_chunk_state_kernel walks the chunks
// of one sequence in order for 32 value columns of one head, in fp32.
// ------------------------------------------------------------------------------------------
namespace {
constexpr int kGC = 64;  // chunk length

__device__ __forceinline__ void gdn_ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void gdn_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, "
      "%7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// [64 rows][128] bf16 tile, 16-byte chunks XOR-swizzled by row (conflict-free ldmatrix)
__device__ __forceinline__ uint32_t gdn_swz(int r, int c) {
  return (uint32_t)(r * 256 + ((c ^ (r & 7)) << 4));
}
}  // namespace

__global__ void gdn_chunk_table_kernel(LinearAttnBatch bt, int4* chunks, int* seq_chunk0) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x != 0) return;
  int c = 0;
  for (int b = 0; b < bt.B; ++b) {
    seq_chunk0[b] = c;
    const int t0 = bt.q_start[b], n = bt.q_start[b + 1] - t0;
    for (int s = 0; s < n; s += kGC) chunks[c++] = make_int4(t0 + s, min(kGC, n - s), b, 0);
  }
  seq_chunk0[bt.B] = c;
}

// grid (max_chunks, Hv), 256 threads; dynamic smem = kGdnPrepSmem.  q^ and k^ are held as
// bf16 pairs hi + lo (hi = bf16(x), lo = bf16(x - hi)); the products keep hi*hi + hi*lo + lo*hi,
// about 16 mantissa bits, so the triangular system sees nearly fp32 dot products.
constexpr int kGdnPrepSmem = 4 * kGC * 128 * 2 + 2 * kGC * 65 * 4 + 2 * kGC * 4;

__global__ void __launch_bounds__(256) gdn_chunk_prep_kernel(const GatedDeltaParams p,
                                                             GdnChunkScratch cs, int B) {
  pdl_trigger();
  pdl_wait();
  const int c = blockIdx.x, h = blockIdx.y;
  if (c >= cs.seq_chunk0[B]) return;
  const int4 ch = cs.chunks[c];
  const int t0 = ch.x, L = ch.y;
  const int kh = h / (p.Hv / p.Hk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  extern __shared__ __align__(128) uint8_t gsm[];
  uint8_t* sq = gsm;                                   // q^ hi [64][128] bf16
  uint8_t* sk = sq + kGC * 256;                        // k^ hi
  uint8_t* sql = sk + kGC * 256;                       // q^ lo
  uint8_t* skl = sql + kGC * 256;                      // k^ lo
  float* sKK = reinterpret_cast<float*>(skl + kGC * 256);  // [64][65]: K^K^T, then A
  float* sQK = sKK + kGC * 65;                          // [64][65]: Q^K^T
  float* slg = sQK + kGC * 65;                          // [64]
  float* sbeta = slg + kGC;                             // [64]

  if (tid < kGC) {
    float lg = 0.f, beta = 0.f;
    if (tid < L) {
      const long long t = t0 + tid;
      const float a = __bfloat162float(p.a[t * p.ld_zab + h]);
      lg = -__expf(p.A_log[h]) * softplus_d(a + p.dt_bias[h]);
      beta = p.gb[t * p.Hv + h].y;
    }
    slg[tid] = lg;
    sbeta[tid] = beta;
  }
  // q^ = q / |q| * dk^-1/2 and k^ = k / |k|, rounded to bf16 for the tensor cores
  const float qscale = rsqrtf(128.f);
  for (int i = tid; i < kGC * 16; i += 256) {
    const int r = i >> 4, cc = i & 15;
    uint4 qo = make_uint4(0u, 0u, 0u, 0u), ko = qo, qlo = qo, klo = qo;
    if (r < L) {
      const long long t = t0 + r;
      const float4 gb = p.gb[t * p.Hv + h];
      const __nv_bfloat16* row = p.qkv + t * p.ld_qkv;
      const uint4 qi = *reinterpret_cast<const uint4*>(row + (long long)kh * 128 + cc * 8);
      const uint4 ki = *reinterpret_cast<const uint4*>(row + (long long)(p.Hk + kh) * 128 + cc * 8);
      const uint32_t qw[4] = {qi.x, qi.y, qi.z, qi.w}, kw[4] = {ki.x, ki.y, ki.z, ki.w};
      uint32_t qn[4], kn[4], ql[4], kl[4];
      const float sq_ = gb.z * qscale;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fq = unpack_bf16x2(qw[e]), fk = unpack_bf16x2(kw[e]);
        const float q0 = fq.x * sq_, q1 = fq.y * sq_, k0 = fk.x * gb.w, k1 = fk.y * gb.w;
        qn[e] = pack_bf16x2(q0, q1);
        kn[e] = pack_bf16x2(k0, k1);
        const float2 qh = unpack_bf16x2(qn[e]), kh2 = unpack_bf16x2(kn[e]);
        ql[e] = pack_bf16x2(q0 - qh.x, q1 - qh.y);
        kl[e] = pack_bf16x2(k0 - kh2.x, k1 - kh2.y);
      }
      qo = make_uint4(qn[0], qn[1], qn[2], qn[3]);
      ko = make_uint4(kn[0], kn[1], kn[2], kn[3]);
      qlo = make_uint4(ql[0], ql[1], ql[2], ql[3]);
      klo = make_uint4(kl[0], kl[1], kl[2], kl[3]);
    }
    *reinterpret_cast<uint4*>(sq + gdn_swz(r, cc)) = qo;
    *reinterpret_cast<uint4*>(sk + gdn_swz(r, cc)) = ko;
    *reinterpret_cast<uint4*>(sql + gdn_swz(r, cc)) = qlo;
    *reinterpret_cast<uint4*>(skl + gdn_swz(r, cc)) = klo;
  }
  __syncthreads();
  if (tid == 0) {  // inclusive prefix sum of the log decays
    float acc = 0.f;
    for (int t = 0; t < kGC; ++t) {
      acc += slg[t];
      slg[t] = acc;
    }
  }
  // K^K^T (warps 0-3) and Q^K^T (warps 4-7): 16 rows x 64 columns per warp, k = 128
  {
    const uint8_t* sa = warp < 4 ? sk : sq;
    const uint8_t* sal = warp < 4 ? skl : sql;
    float* dst = warp < 4 ? sKK : sQK;
    const int wrow = (warp & 3) * 16;
    float acc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll 2
    for (int k = 0; k < 8; ++k) {
      uint32_t af[4], al[4];
      const uint32_t aoff = gdn_swz(wrow + (lane & 15), k * 2 + (lane >> 4));
      gdn_ldsm_x4(smem_u32(sa + aoff), af[0], af[1], af[2], af[3]);
      gdn_ldsm_x4(smem_u32(sal + aoff), al[0], al[1], al[2], al[3]);
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        const int i = lane >> 3;
        const int r = n * 8 + (i >> 1) * 8 + (lane & 7);
        const uint32_t boff = gdn_swz(r, k * 2 + (i & 1));
        uint32_t b0, b1, b2, b3, l0, l1, l2, l3;
        gdn_ldsm_x4(smem_u32(sk + boff), b0, b1, b2, b3);
        gdn_ldsm_x4(smem_u32(skl + boff), l0, l1, l2, l3);
        gdn_mma(acc[n], af, b0, b1);
        gdn_mma(acc[n + 1], af, b2, b3);
        gdn_mma(acc[n], af, l0, l1);
        gdn_mma(acc[n + 1], af, l2, l3);
        gdn_mma(acc[n], al, b0, b1);
        gdn_mma(acc[n + 1], al, b2, b3);
      }
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int r = wrow + (lane >> 2), col = n * 8 + (lane & 3) * 2;
      dst[r * 65 + col] = acc[n][0];
      dst[r * 65 + col + 1] = acc[n][1];
      dst[(r + 8) * 65 + col] = acc[n][2];
      dst[(r + 8) * 65 + col + 1] = acc[n][3];
    }
  }
  __syncthreads();
  // A (strictly lower, in place of K^K^T) and the decay-masked Q^K^T (written out)
  float* qkm = cs.QKm + ((long long)c * p.Hv + h) * (kGC * kGC);
  for (int i = tid; i < kGC * kGC; i += 256) {
    const int t = i >> 6, s2 = i & 63;
    float a = 0.f, q = 0.f;
    if (t < L && s2 <= t) {
      const float dec = __expf(slg[t] - slg[s2]);
      q = dec * sQK[t * 65 + s2];
      if (s2 < t) a = sbeta[t] * dec * sKK[t * 65 + s2];
    }
    sKK[t * 65 + s2] = a;
    qkm[i] = q;
  }
  __syncthreads();
  // Forward substitution (I + A) X = R, one right-hand-side column per thread:
  // columns 0..127 -> W (R = beta gamma k^), 128..255 -> U (R = beta v).
  const int j = tid;
  const bool isw = j < 128;
  const __nv_bfloat16* vcol = p.qkv + (long long)t0 * p.ld_qkv + 2LL * p.Hk * 128 +
                              (long long)h * 128 + (j & 127);
  float x[kGC];
#pragma unroll
  for (int t = 0; t < kGC; ++t) {
    float r = 0.f;
    if (t < L) {
      if (isw) {
        const uint32_t off = gdn_swz(t, j >> 3) + (j & 7) * 2;
        const float kv = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(sk + off)) +
                         __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(skl + off));
        r = sbeta[t] * __expf(slg[t]) * kv;
      } else {
        r = sbeta[t] * __bfloat162float(vcol[(long long)t * p.ld_qkv]);
      }
    }
    // four independent partial sums break the dependent FMA chain
    float r1 = 0.f, r2 = 0.f, r3 = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < t; ++s2) {
      const float m = sKK[t * 65 + s2] * x[s2];
      if ((s2 & 3) == 0) r -= m;
      else if ((s2 & 3) == 1) r1 -= m;
      else if ((s2 & 3) == 2) r2 -= m;
      else r3 -= m;
    }
    x[t] = (r + r1) + (r2 + r3);
  }
  float* dst = (isw ? cs.W : cs.U) + ((long long)t0 * p.Hv + h) * 128 + (j & 127);
#pragma unroll
  for (int t = 0; t < kGC; ++t)
    if (t < L) dst[(long long)t * p.Hv * 128] = x[t];
  if (tid < L) cs.lg[(long long)(t0 + tid) * p.Hv + h] = slg[tid];
}

// grid (B, Hv, 4), 256 threads: 32 value columns of one (sequence, value head), all chunks
// of the sequence in order, the chunk products on the tensor cores (mma m16n8k8 tf32, fp32
// accumulation; the state itself stays fp32 in shared memory).  Per chunk, 8 warps:
// The two products that feed the carried state (W S0 and K^T (f Delta)) use 3xTF32 (operands
// split into a tf32 pair), close to fp32; the two output products use single tf32.
//   Delta[64 x 32] = U - W S0                 warp (m tile w % 4, 16 columns w / 4), k = 128
//   O[64 x 32]     = qf * (Q S0) + QKm Delta  same tiling, k = 128 and k = 64 (lower blocks)
//   S[128 x 32]    = gamma_L S0 + K^T (f * Delta)   warp = 16 state rows x 32 columns, k = 64
constexpr int kGdnCols = 32;
constexpr int kSS = 36;        // fp32 row stride of S / Delta (conflict-free B fragments)
constexpr int kWStride = 132;  // fp32 row stride of W (conflict-free A fragments)
constexpr int kQStride = 136;  // bf16 row stride of q and k
constexpr int kQKStride = 72;  // bf16 row stride of the staged masked Q^K^T block
constexpr int kGdnStateSmem = 128 * kSS * 4 + kGC * kWStride * 4 + 2 * kGC * kQStride * 2 +
                              kGC * kSS * 4 + 4 * kGC * 4 + kGC * kQKStride * 2;

namespace {
__device__ __forceinline__ uint32_t tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ float bf(const __nv_bfloat16* p) { return __bfloat162float(*p); }
// x = big + small, both tf32 (3xTF32: big*big + big*small + small*big is close to fp32)
__device__ __forceinline__ void tf32_split(float x, uint32_t& big, uint32_t& small) {
  big = tf32(x);
  small = tf32(x - __uint_as_float(big));
}
}  // namespace

__global__ void __launch_bounds__(256) gdn_chunk_state_kernel(const GatedDeltaParams p,
                                                              LinearAttnBatch bt,
                                                              GdnChunkScratch cs) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, h = blockIdx.y, cg = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int n = bt.q_start[b + 1] - bt.q_start[b];
  if (n == 0) return;
  const int ctx = bt.seq_lens[b] - n;
  extern __shared__ __align__(16) uint8_t ssm[];
  float* sS = reinterpret_cast<float*>(ssm);                                  // [128][36]
  float* sW = sS + 128 * kSS;                                                  // [64][132]
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(sW + kGC * kWStride);  // [64][136]
  __nv_bfloat16* sK = sQ + kGC * kQStride;                                     // [64][136]
  float* sD = reinterpret_cast<float*>(sK + kGC * kQStride);                   // [64][36]
  float* slg = sD + kGC * kSS;   // [64] cumulative log decay
  float* sqf = slg + kGC;        // [64] gamma_t |q|^-1 dk^-1/2
  float* skf = sqf + kGC;        // [64] |k|^-1 e^{lg_L - lg_t}
  float* sik = skf + kGC;        // [64] |k|^-1
  // decay-masked Q^K^T of the chunk, bf16 (it only feeds the bf16 output, not the state)
  __nv_bfloat16* sQK = reinterpret_cast<__nv_bfloat16*>(sik + kGC);  // [64][72]
  float* S = p.state + (long long)bt.slots[b] * p.state_slot_stride + (long long)h * 128 * 128 +
             cg * kGdnCols;
  for (int i = tid; i < 128 * kGdnCols / 4; i += 256) {
    const int r = i >> 3, c4 = i & 7;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ctx > 0) v = *reinterpret_cast<const float4*>(S + (long long)r * 128 + c4 * 4);
    *reinterpret_cast<float4*>(sS + r * kSS + c4 * 4) = v;
  }
  const int kh = h / (p.Hv / p.Hk);
  const float qscale = rsqrtf(128.f);
  const int mt = warp & 3, nh = warp >> 2;  // chunk-output tiling
  const int c0 = cs.seq_chunk0[b], c1 = cs.seq_chunk0[b + 1];
  for (int c = c0; c < c1; ++c) {
    const int4 ch = cs.chunks[c];
    const int t0 = ch.x, L = ch.y;
    // ---- stage the chunk (rows past L are zero)
    for (int i = tid; i < kGC * 32; i += 256) {
      const int r = i >> 5, c4 = i & 31;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < L) v = *reinterpret_cast<const float4*>(cs.W + ((long long)(t0 + r) * p.Hv + h) * 128 + c4 * 4);
      *reinterpret_cast<float4*>(sW + r * kWStride + c4 * 4) = v;
    }
    for (int i = tid; i < kGC * 16; i += 256) {
      const int r = i >> 4, c8 = i & 15;
      uint4 qv = make_uint4(0u, 0u, 0u, 0u), kv = qv;
      if (r < L) {
        const __nv_bfloat16* row = p.qkv + (long long)(t0 + r) * p.ld_qkv;
        qv = *reinterpret_cast<const uint4*>(row + (long long)kh * 128 + c8 * 8);
        kv = *reinterpret_cast<const uint4*>(row + (long long)(p.Hk + kh) * 128 + c8 * 8);
      }
      *reinterpret_cast<uint4*>(sQ + r * kQStride + c8 * 8) = qv;
      *reinterpret_cast<uint4*>(sK + r * kQStride + c8 * 8) = kv;
    }
    {
      const float* qk = cs.QKm + ((long long)c * p.Hv + h) * (kGC * kGC);
      for (int i = tid; i < kGC * kGC / 4; i += 256) {  // rows past L are zero in QKm
        const int r = i >> 4, c4 = i & 15;
        const float4 v = *reinterpret_cast<const float4*>(qk + r * kGC + c4 * 4);
        *reinterpret_cast<uint2*>(sQK + r * kQKStride + c4 * 4) =
            make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
      }
    }
    if (tid < kGC) {
      float lg = 0.f, qf = 0.f, ik = 0.f;
      if (tid < L) {
        const long long t = t0 + tid;
        lg = cs.lg[t * p.Hv + h];
        const float4 gb = p.gb[t * p.Hv + h];
        qf = __expf(lg) * gb.z * qscale;
        ik = gb.w;
      }
      slg[tid] = lg;
      sqf[tid] = qf;
      sik[tid] = ik;
    }
    __syncthreads();
    const float lgL = slg[L - 1];
    if (tid < kGC) skf[tid] = tid < L ? sik[tid] * __expf(lgL - slg[tid]) : 0.f;
    const int r0 = mt * 16 + g, r1 = r0 + 8;  // chunk rows of this lane's accumulators
    // ---- Delta = U - W S0
    {
      float acc[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
      float2 uu[2][2];  // U loads issued before the product so their latency overlaps it
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int col = nh * 16 + j * 8 + 2 * t4;
        uu[j][0] = uu[j][1] = make_float2(0.f, 0.f);
        if (r0 < L) uu[j][0] = *reinterpret_cast<const float2*>(cs.U + ((long long)(t0 + r0) * p.Hv + h) * 128 + cg * kGdnCols + col);
        if (r1 < L) uu[j][1] = *reinterpret_cast<const float2*>(cs.U + ((long long)(t0 + r1) * p.Hv + h) * 128 + cg * kGdnCols + col);
      }
#pragma unroll 2
      for (int ks = 0; ks < 16; ++ks) {
        const int kc = ks * 8 + t4;
        uint32_t a0, a1, a2, a3, e0, e1, e2, e3;
        tf32_split(sW[r0 * kWStride + kc], a0, e0);
        tf32_split(sW[r1 * kWStride + kc], a1, e1);
        tf32_split(sW[r0 * kWStride + kc + 4], a2, e2);
        tf32_split(sW[r1 * kWStride + kc + 4], a3, e3);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int col = nh * 16 + j * 8 + g;
          uint32_t b0, b1, f0, f1;
          tf32_split(sS[kc * kSS + col], b0, f0);
          tf32_split(sS[(kc + 4) * kSS + col], b1, f1);
          mma_tf32(acc[j], e0, e1, e2, e3, b0, b1);
          mma_tf32(acc[j], a0, a1, a2, a3, f0, f1);
          mma_tf32(acc[j], a0, a1, a2, a3, b0, b1);
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int col = nh * 16 + j * 8 + 2 * t4;
        const float2 u0 = uu[j][0], u1 = uu[j][1];
        *reinterpret_cast<float2*>(sD + r0 * kSS + col) = make_float2(u0.x - acc[j][0], u0.y - acc[j][1]);
        *reinterpret_cast<float2*>(sD + r1 * kSS + col) = make_float2(u1.x - acc[j][2], u1.y - acc[j][3]);
      }
    }
    __syncthreads();
    // ---- O = qf * (Q S0) + QKm Delta
    {
      float acc[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll 4
      for (int ks = 0; ks < 16; ++ks) {
        const int kc = ks * 8 + t4;
        const uint32_t a0 = tf32(bf(sQ + r0 * kQStride + kc)), a1 = tf32(bf(sQ + r1 * kQStride + kc));
        const uint32_t a2 = tf32(bf(sQ + r0 * kQStride + kc + 4)), a3 = tf32(bf(sQ + r1 * kQStride + kc + 4));
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int col = nh * 16 + j * 8 + g;
          mma_tf32(acc[j], a0, a1, a2, a3, tf32(sS[kc * kSS + col]), tf32(sS[(kc + 4) * kSS + col]));
        }
      }
      const float f0 = sqf[r0], f1 = sqf[r1];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        acc[j][0] *= f0; acc[j][1] *= f0; acc[j][2] *= f1; acc[j][3] *= f1;
      }
      // QKm is lower triangular: k steps past this m tile's last row contribute nothing
      for (int ks = 0; ks < 2 * mt + 2; ++ks) {
        const int kc = ks * 8 + t4;
        const uint32_t a0 = tf32(bf(sQK + r0 * kQKStride + kc)), a1 = tf32(bf(sQK + r1 * kQKStride + kc));
        const uint32_t a2 = tf32(bf(sQK + r0 * kQKStride + kc + 4)), a3 = tf32(bf(sQK + r1 * kQKStride + kc + 4));
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int col = nh * 16 + j * 8 + g;
          mma_tf32(acc[j], a0, a1, a2, a3, tf32(sD[kc * kSS + col]), tf32(sD[(kc + 4) * kSS + col]));
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int col = h * 128 + cg * kGdnCols + nh * 16 + j * 8 + 2 * t4;
        if (r0 < L)
          *reinterpret_cast<uint32_t*>(p.out + (long long)(t0 + r0) * p.ld_out + col) = pack_bf16x2(acc[j][0], acc[j][1]);
        if (r1 < L)
          *reinterpret_cast<uint32_t*>(p.out + (long long)(t0 + r1) * p.ld_out + col) = pack_bf16x2(acc[j][2], acc[j][3]);
      }
    }
    __syncthreads();
    // ---- S = gamma_L S0 + K^T (f * Delta): warp owns state rows 16w..16w+15, all 32 columns
    {
      const float gL = __expf(lgL);
      const int s0 = warp * 16 + g, s1 = s0 + 8;
      float acc[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = j * 8 + 2 * t4;
        const float2 x0 = *reinterpret_cast<const float2*>(sS + s0 * kSS + col);
        const float2 x1 = *reinterpret_cast<const float2*>(sS + s1 * kSS + col);
        acc[j][0] = gL * x0.x; acc[j][1] = gL * x0.y; acc[j][2] = gL * x1.x; acc[j][3] = gL * x1.y;
      }
      const int ksteps = (L + 7) >> 3;
      for (int ks = 0; ks < ksteps; ++ks) {
        const int kt = ks * 8 + t4;  // token of a0 / b0
        const uint32_t a0 = tf32(bf(sK + kt * kQStride + s0)), a1 = tf32(bf(sK + kt * kQStride + s1));
        const uint32_t a2 = tf32(bf(sK + (kt + 4) * kQStride + s0)), a3 = tf32(bf(sK + (kt + 4) * kQStride + s1));
        const float fa = skf[kt], fb = skf[kt + 4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int col = j * 8 + g;
          // k is bf16, exact in tf32: splitting the (f * Delta) operand suffices
          uint32_t b0, b1, f0, f1;
          tf32_split(fa * sD[kt * kSS + col], b0, f0);
          tf32_split(fb * sD[(kt + 4) * kSS + col], b1, f1);
          mma_tf32(acc[j], a0, a1, a2, a3, f0, f1);
          mma_tf32(acc[j], a0, a1, a2, a3, b0, b1);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = j * 8 + 2 * t4;
        *reinterpret_cast<float2*>(sS + s0 * kSS + col) = make_float2(acc[j][0], acc[j][1]);
        *reinterpret_cast<float2*>(sS + s1 * kSS + col) = make_float2(acc[j][2], acc[j][3]);
      }
    }
    __syncthreads();
  }
  for (int i = tid; i < 128 * kGdnCols / 4; i += 256) {
    const int r = i >> 3, c4 = i & 7;
    *reinterpret_cast<float4*>(S + (long long)r * 128 + c4 * 4) =
        *reinterpret_cast<const float4*>(sS + r * kSS + c4 * 4);
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

void gated_delta_rule_chunked_launch(const GatedDeltaParams& p, const LinearAttnBatch& b,
                                     const GdnChunkScratch& cs, cudaStream_t s) {
  if (p.dk != 128 || p.dv != 128)
    throw std::invalid_argument("gated_delta_rule: head dims must be 128");
  if (p.Hv % p.Hk != 0) throw std::invalid_argument("gated_delta_rule: Hv % Hk != 0");
  if (p.ld_qkv % 8 != 0 || p.ld_zab % 4 != 0 || p.ld_out % 4 != 0)
    throw std::invalid_argument("gated_delta_rule: row strides must allow vector loads");
  if (p.Hk > 64) throw std::invalid_argument("gated_delta_rule: at most 64 key heads per rank");
  if (b.B == 0 || p.T == 0) return;
  if (cs.max_chunks < p.T / kGC + b.B)
    throw std::invalid_argument("gated_delta_rule: chunk scratch too small");
  launch_pdl(gdn_prepare_kernel, dim3(p.T), dim3(256), 0, s, p);
  launch_pdl(gdn_chunk_table_kernel, dim3(1), dim3(32), 0, s, b, cs.chunks, cs.seq_chunk0);
  {
    static std::atomic<uint64_t> configured{0};
    set_max_dynamic_smem_once(gdn_chunk_prep_kernel, kGdnPrepSmem, configured);
    launch_pdl(gdn_chunk_prep_kernel, dim3(cs.max_chunks, p.Hv), dim3(256), kGdnPrepSmem, s, p, cs,
               b.B);
  }
  {
    static std::atomic<uint64_t> configured{0};
    set_max_dynamic_smem_once(gdn_chunk_state_kernel, kGdnStateSmem, configured);
    launch_pdl(gdn_chunk_state_kernel, dim3(b.B, p.Hv, 128 / kGdnCols), dim3(256), kGdnStateSmem,
               s, p, b, cs);
  }
  const int rows = p.T * p.Hv;
  launch_pdl(gated_rmsnorm_kernel, dim3((rows + 7) / 8), dim3(256), 0, s, p.out, p.ld_out, p.z,
             p.ld_zab, p.norm_w, p.Hv, rows, p.eps);
}

void sigmoid_gate_mul_launch(__nv_bfloat16* x, long long ldx, const __nv_bfloat16* gate,
                             long long ldg, int T, int n, cudaStream_t s) {
  if (T == 0) return;
  launch_pdl(sigmoid_gate_mul_kernel, dim3(T), dim3(256), 0, s, x, ldx, gate, ldg, n);
}

}  // namespace b200
