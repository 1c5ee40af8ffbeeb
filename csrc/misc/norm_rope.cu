// Memory-bound fused kernels around the projections:
//   rmsnorm                 out = x * rsqrt(mean(x^2) + eps) * w
//   add_rmsnorm             residual += x ; out = rmsnorm(residual)       (x bf16 or fp32)
//                           With an fp32 x (the split-K / all-reduce accumulation buffer),
//                           the buffer is cleared after it is read, so the next GEMM can
//                           accumulate into it again without a separate memset launch.
//   rope_kv_write           q/k rotary embedding (neox or interleaved pairs), optional
//                           per-head q/k RMSNorm (Qwen3), k/v scatter into the paged cache
//                           at slot_mapping (negative slot = padding token, skipped).
//   silu_mul                out = silu(gate) * up, gate/up either in halves or interleaved
//                           in blocks of `blk` columns.
//   embedding_lookup        out[t] = table[id[t] - vocab_start] (zero outside the shard)
//
// Reference counterparts: rmsnorm/residual fusion inside the NKI mlp/qkv kernels
// (vllm_neuron/functional/mlp.py:65, attention/qkv.py:672), RoPE + in-kernel cache write
// (attention/qkv.py:311 `_torch_qkv_in_kernel_cache_write_impl`), embedding
// (vllm_neuron/functional/embedding.py:6, nn/embedding.py:23).
#include <cuda_bf16.h>

#include <stdexcept>
#include <string>

#include "../common.cuh"
#include "misc.h"

namespace b200 {

namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = (l < nw) ? red[l] : 0.f;
  t = warp_sum(t);
  return t;
}

}  // namespace

// One CTA per row; each thread keeps its slice of the row in registers (H <= 8 * 8 * 256).
template <typename TX, bool HAS_RES>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(TX* x, long long x_stride,
                                                          __nv_bfloat16* residual,
                                                          long long r_stride,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          __nv_bfloat16* out, long long o_stride,
                                                          int H, float eps, bool clear_x) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  TX* xr = x + row * x_stride;
  __nv_bfloat16* rr = HAS_RES ? residual + row * r_stride : nullptr;
  constexpr int kMaxPer = 32;  // elements per thread
  float v[kMaxPer];
  float ss = 0.f;
  int n = 0;
  for (int i = threadIdx.x; i < H; i += blockDim.x, ++n) {
    float a = to_f(xr[i]);
    if (HAS_RES) {
      a += __bfloat162float(rr[i]);
    }
    v[n] = a;
    ss += a * a;
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)H + eps);
  n = 0;
  for (int i = threadIdx.x; i < H; i += blockDim.x, ++n) {
    const __nv_bfloat16 rb = __float2bfloat16(v[n]);
    if (HAS_RES) rr[i] = rb;
    // Normalize the bf16-rounded residual, as the unfused bf16 model would.
    const float a = HAS_RES ? __bfloat162float(rb) : v[n];
    out[row * o_stride + i] = __float2bfloat16(a * inv * __bfloat162float(w[i]));
    if (clear_x) xr[i] = from_f<TX>(0.f);
  }
}

void add_rmsnorm_launch(void* x, bool x_is_f32, long long x_stride, __nv_bfloat16* residual,
                        long long r_stride, const __nv_bfloat16* w, __nv_bfloat16* out,
                        long long o_stride, int rows, int H, float eps, bool clear_x,
                        cudaStream_t stream) {
  if (rows == 0) return;
  if (H > 256 * 32) throw std::invalid_argument("add_rmsnorm: hidden size too large");
  const int threads = H >= 2048 ? 256 : 128;
  if (H > threads * 32) throw std::invalid_argument("add_rmsnorm: hidden size too large");
  if (x_is_f32) {
    if (residual)
      add_rmsnorm_kernel<float, true><<<rows, threads, 0, stream>>>(
          (float*)x, x_stride, residual, r_stride, w, out, o_stride, H, eps, clear_x);
    else
      add_rmsnorm_kernel<float, false><<<rows, threads, 0, stream>>>(
          (float*)x, x_stride, residual, r_stride, w, out, o_stride, H, eps, clear_x);
  } else {
    if (residual)
      add_rmsnorm_kernel<__nv_bfloat16, true><<<rows, threads, 0, stream>>>(
          (__nv_bfloat16*)x, x_stride, residual, r_stride, w, out, o_stride, H, eps, false);
    else
      add_rmsnorm_kernel<__nv_bfloat16, false><<<rows, threads, 0, stream>>>(
          (__nv_bfloat16*)x, x_stride, residual, r_stride, w, out, o_stride, H, eps, false);
  }
}

// ------------------------------------------------------------------------------------------
// RoPE + optional q/k RMSNorm + paged KV write.  One CTA per token, one warp per head.
// Input row layout: [q heads | k heads | v heads] * D.  The rotated q is written to q_out
// (bf16, may alias the input when the input is bf16).
// ------------------------------------------------------------------------------------------
template <typename TIN>
__global__ void __launch_bounds__(256) rope_kv_write_kernel(const RopeKvParams p, TIN* qkv) {
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = p.head_dim;
  const int half = p.rot_dim / 2;
  const int pos = p.positions[t];
  const long long slot = p.slot_mapping ? (long long)p.slot_mapping[t] : -1;
  const float* cs = p.cos_sin + (long long)pos * p.rot_dim;  // [cos(half) | sin(half)]
  const int nheads = p.Hq + 2 * p.Hkv;
  TIN* row = qkv + t * p.qkv_stride;
  for (int h = warp; h < nheads; h += blockDim.x >> 5) {
    const bool is_q = h < p.Hq;
    const bool is_k = !is_q && h < p.Hq + p.Hkv;
    TIN* src = row + (long long)h * D;
    // Each lane handles up to 8 elements (D <= 256).
    float v[8];
    const int per = D / 32;
    for (int e = 0; e < per; ++e) v[e] = to_f(src[lane + 32 * e]);
    if ((is_q && p.q_norm_w) || (is_k && p.k_norm_w)) {
      float ss = 0.f;
      for (int e = 0; e < per; ++e) ss += v[e] * v[e];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / (float)D + p.eps);
      const __nv_bfloat16* nw = is_q ? p.q_norm_w : p.k_norm_w;
      for (int e = 0; e < per; ++e) {
        // round to bf16 like a standalone norm followed by rope would
        v[e] = __bfloat162float(__float2bfloat16(v[e] * inv * __bfloat162float(nw[lane + 32 * e])));
      }
    }
    if (is_q || is_k) {
      // Rotate pairs.  neox: (i, i + half); interleaved: (2i, 2i + 1).  Gather partners via
      // shared-nothing shuffles: write to a small per-warp smem line instead.
      __shared__ float line[8][256];
      float* L = line[warp & 7];
      for (int e = 0; e < per; ++e) L[lane + 32 * e] = v[e];
      __syncwarp();
      for (int e = 0; e < per; ++e) {
        const int i = lane + 32 * e;
        if (i >= p.rot_dim) continue;
        float out;
        if (p.neox) {
          const int j = i < half ? i : i - half;
          const float c = cs[j], s = cs[half + j];
          out = i < half ? L[i] * c - L[i + half] * s : L[i] * c + L[i - half] * s;
        } else {
          const int j = i >> 1;
          const float c = cs[j], s = cs[half + j];
          out = (i & 1) ? L[i] * c + L[i - 1] * s : L[i] * c - L[i + 1] * s;
        }
        v[e] = out;
      }
      __syncwarp();
    }
    if (is_q) {
      __nv_bfloat16* dst = p.q_out + t * p.q_out_stride + (long long)h * D;
      for (int e = 0; e < per; ++e) dst[lane + 32 * e] = __float2bfloat16(v[e]);
    } else if (slot >= 0) {
      const int kvh = is_k ? h - p.Hq : h - p.Hq - p.Hkv;
      const long long blk = slot / p.block_size, off = slot % p.block_size;
      __nv_bfloat16* cache = is_k ? p.k_cache : p.v_cache;
      __nv_bfloat16* dst =
          cache + blk * p.kv_block_stride + ((long long)kvh * p.block_size + off) * D;
      for (int e = 0; e < per; ++e) dst[lane + 32 * e] = __float2bfloat16(v[e]);
    }
    if (p.clear_input) {
      for (int e = 0; e < per; ++e) src[lane + 32 * e] = from_f<TIN>(0.f);
    }
  }
}

void rope_kv_write_launch(const RopeKvParams& p, void* qkv, bool qkv_is_f32, int T,
                          cudaStream_t stream) {
  if (T == 0) return;
  if (p.head_dim % 32 != 0 || p.head_dim > 256)
    throw std::invalid_argument("rope_kv_write: head_dim must be a multiple of 32, <= 256");
  if (qkv_is_f32)
    rope_kv_write_kernel<float><<<T, 256, 0, stream>>>(p, (float*)qkv);
  else
    rope_kv_write_kernel<__nv_bfloat16><<<T, 256, 0, stream>>>(p, (__nv_bfloat16*)qkv);
}

// ------------------------------------------------------------------------------------------
// SiLU(gate) * up
// ------------------------------------------------------------------------------------------
template <typename TIN>
__global__ void silu_mul_kernel(TIN* in, long long in_stride, __nv_bfloat16* out,
                                long long out_stride, int I, int blk, bool clear_input,
                                float limit, float alpha, int act) {
  const int t = blockIdx.y;
  TIN* r = in + t * in_stride;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < I; j += gridDim.x * blockDim.x) {
    int gi, ui;
    if (blk > 0) {
      const int b = j / blk, w = j % blk;
      gi = b * 2 * blk + w;
      ui = gi + blk;
    } else {
      gi = j;
      ui = j + I;
    }
    float g = to_f(r[gi]), u = to_f(r[ui]);
    float y;
    if (act == 0) {  // SwiGLU
      y = g / (1.f + __expf(-g)) * u;
    } else {  // GPT-OSS clamped SwiGLU: (up + 1) * gate * sigmoid(alpha * gate)
      g = fminf(g, limit);
      u = fminf(fmaxf(u, -limit), limit);
      y = (u + 1.f) * g / (1.f + __expf(-alpha * g));
    }
    out[t * out_stride + j] = __float2bfloat16(y);
    if (clear_input) {
      r[gi] = from_f<TIN>(0.f);
      r[ui] = from_f<TIN>(0.f);
    }
  }
}

void silu_mul_launch(void* in, bool in_is_f32, long long in_stride, __nv_bfloat16* out,
                     long long out_stride, int T, int I, int blk, bool clear_input, int act,
                     float limit, float alpha, cudaStream_t stream) {
  if (T == 0) return;
  dim3 grid((I + 255) / 256, T);
  if (in_is_f32)
    silu_mul_kernel<float><<<grid, 256, 0, stream>>>((float*)in, in_stride, out, out_stride, I,
                                                     blk, clear_input, limit, alpha, act);
  else
    silu_mul_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        (__nv_bfloat16*)in, in_stride, out, out_stride, I, blk, false, limit, alpha, act);
}

// ------------------------------------------------------------------------------------------
// Embedding lookup (vocab-sharded).
// ------------------------------------------------------------------------------------------
__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* out, int H, int vocab_start, int vocab_end) {
  const int t = blockIdx.x;
  const int id = ids[t];
  const bool own = id >= vocab_start && id < vocab_end;
  const uint4* src = reinterpret_cast<const uint4*>(table + (long long)(own ? id - vocab_start : 0) * H);
  uint4* dst = reinterpret_cast<uint4*>(out + (long long)t * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = own ? src[i] : make_uint4(0, 0, 0, 0);
}

void embedding_launch(const int* ids, const __nv_bfloat16* table, __nv_bfloat16* out, int T,
                      int H, int vocab_start, int vocab_end, cudaStream_t stream) {
  if (T == 0) return;
  if (H % 8 != 0) throw std::invalid_argument("embedding: hidden size must be a multiple of 8");
  embedding_kernel<<<T, 128, 0, stream>>>(ids, table, out, H, vocab_start, vocab_end);
}

}  // namespace b200
