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

#include <cuda_fp8.h>

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

// One CTA per row.  Thread t owns 8-element vectors t, t + blockDim, ... (NV of them, a
// compile-time count, so the row slice stays in registers).
template <typename TX>
__device__ __forceinline__ void load8(const TX* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 a = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store8_bf16(__nv_bfloat16* p, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                            pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}
template <typename TX>
__device__ __forceinline__ void zero8(TX* p);
template <>
__device__ __forceinline__ void zero8<float>(float* p) {
  reinterpret_cast<float4*>(p)[0] = make_float4(0.f, 0.f, 0.f, 0.f);
  reinterpret_cast<float4*>(p)[1] = make_float4(0.f, 0.f, 0.f, 0.f);
}
template <>
__device__ __forceinline__ void zero8<__nv_bfloat16>(__nv_bfloat16* p) {
  *reinterpret_cast<uint4*>(p) = make_uint4(0, 0, 0, 0);
}

template <typename TX, bool HAS_RES, int NV>
__global__ void __launch_bounds__(1024) add_rmsnorm_kernel(TX* x, long long x_stride,
                                                          __nv_bfloat16* residual,
                                                          long long r_stride,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          __nv_bfloat16* out, long long o_stride,
                                                          int H, float eps, bool clear_x) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  const long long row = blockIdx.x;
  TX* xr = x + row * x_stride;
  __nv_bfloat16* rr = HAS_RES ? residual + row * r_stride : nullptr;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int idx = (j * blockDim.x + threadIdx.x) * 8;
    if (idx < H) {
      load8<TX>(xr + idx, v[j]);
      if (HAS_RES) {
        float r[8];
        load8<__nv_bfloat16>(rr + idx, r);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          // round the new residual to bf16 (the stored value) before normalising it
          v[j][e] = __bfloat162float(__float2bfloat16(v[j][e] + r[e]));
        }
        store8_bf16(rr + idx, v[j]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[j][e] * v[j][e];
      if (clear_x) zero8<TX>(xr + idx);
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)H + eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int idx = (j * blockDim.x + threadIdx.x) * 8;
    if (idx < H) {
      float g[8], o[8];
      load8<__nv_bfloat16>(w + idx, g);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[j][e] * inv * g[e];
      store8_bf16(out + row * o_stride + idx, o);
    }
  }
}

template <typename TX, bool HAS_RES>
static void launch_norm(TX* x, long long xs, __nv_bfloat16* res, long long rs,
                        const __nv_bfloat16* w, __nv_bfloat16* out, long long os, int rows, int H,
                        float eps, bool clear, cudaStream_t stream) {
  const int vecs = H / 8;
  // one 8-element vector per thread up to 1024 threads: a row's loads spread over many warps
  // (decode batches have few rows, so per-row latency dominates)
  int threads = vecs <= 1024 ? ((vecs + 31) / 32) * 32 : 1024;
  const int nv = (vecs + threads - 1) / threads;
#define B200_NORM(NV_)                                                                   \
  if (nv <= NV_) {                                                                       \
    launch_pdl(add_rmsnorm_kernel<TX, HAS_RES, NV_>, dim3(rows), dim3(threads), 0, stream, \
               x, xs, res, rs, w, out, os, H, eps, clear);                                 \
    return;                                                                              \
  }
  B200_NORM(1)
  B200_NORM(2)
  B200_NORM(4)
  B200_NORM(8)
#undef B200_NORM
  throw std::invalid_argument("add_rmsnorm: hidden size too large");
}

void add_rmsnorm_launch(void* x, bool x_is_f32, long long x_stride, __nv_bfloat16* residual,
                        long long r_stride, const __nv_bfloat16* w, __nv_bfloat16* out,
                        long long o_stride, int rows, int H, float eps, bool clear_x,
                        cudaStream_t stream) {
  if (rows == 0) return;
  if (H % 8 != 0) throw std::invalid_argument("add_rmsnorm: hidden size must be a multiple of 8");
  if (x_is_f32) {
    if (residual)
      launch_norm<float, true>((float*)x, x_stride, residual, r_stride, w, out, o_stride, rows,
                               H, eps, clear_x, stream);
    else
      launch_norm<float, false>((float*)x, x_stride, residual, r_stride, w, out, o_stride, rows,
                                H, eps, clear_x, stream);
  } else {
    if (residual)
      launch_norm<__nv_bfloat16, true>((__nv_bfloat16*)x, x_stride, residual, r_stride, w, out,
                                       o_stride, rows, H, eps, false, stream);
    else
      launch_norm<__nv_bfloat16, false>((__nv_bfloat16*)x, x_stride, residual, r_stride, w, out,
                                        o_stride, rows, H, eps, false, stream);
  }
}

// ------------------------------------------------------------------------------------------
// RoPE + optional q/k RMSNorm + paged KV write.  One warp per (token, head); 8 heads per CTA.
// Input row layout: [q heads | k heads | v heads] * D.  The rotated q is written to q_out
// (bf16, may alias the input when the input is bf16).
// ------------------------------------------------------------------------------------------
template <typename TIN, int D>
__global__ void __launch_bounds__(256) rope_kv_write_kernel(const RopeKvParams p, TIN* qkv) {
  pdl_trigger();
  pdl_wait();
  constexpr int PER = D / 32;  // elements per lane: lane l owns l, l + 32, l + 64, ...
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = p.rot_dim / 2;
  const int pos = p.positions[t];
  const long long slot = p.slot_mapping ? (long long)p.slot_mapping[t] : -1;
  const float* cs = p.cos_sin + (long long)pos * p.rot_dim;  // [cos(half) | sin(half)]
  const int nheads = p.Hq + 2 * p.Hkv;
  TIN* row = qkv + (long long)t * p.qkv_stride;
  // blockIdx.y selects a group of heads (one per warp), so small decode batches still fill
  // the SMs
  const int wpc = blockDim.x >> 5;
  const int h_end = min(nheads, ((int)blockIdx.y + 1) * wpc);
  for (int h = (int)blockIdx.y * wpc + warp; h < h_end; h += wpc) {
    const bool is_q = h < p.Hq;
    const bool is_k = !is_q && h < p.Hq + p.Hkv;
    TIN* src = row + (long long)h * D;
    float v[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) v[e] = to_f(src[lane + 32 * e]);
    if (p.qkv_bias != nullptr) {
#pragma unroll
      for (int e = 0; e < PER; ++e) v[e] += p.qkv_bias[(long long)h * D + lane + 32 * e];
    }
    if ((is_q && p.q_norm_w) || (is_k && p.k_norm_w)) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < PER; ++e) ss += v[e] * v[e];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / (float)D + p.eps);
      const __nv_bfloat16* nw = is_q ? p.q_norm_w : p.k_norm_w;
#pragma unroll
      for (int e = 0; e < PER; ++e)
        v[e] = __bfloat162float(__float2bfloat16(v[e] * inv * __bfloat162float(nw[lane + 32 * e])));
    }
    if (is_q || is_k) {
      if (p.neox && p.rot_dim == D && PER >= 2) {
        // Full-width neox rotation: pair (i, i + D/2) lives in one lane, elements e, e + PER/2.
        constexpr int HP = PER / 2;
        float o[PER];
#pragma unroll
        for (int e = 0; e < HP; ++e) {
          const int i = lane + 32 * e;
          const float* ci = cs;
          if (p.positions3 != nullptr) {
            const int comp = (i % 3 == 1 && i < 3 * p.mrope_h) ? 1 : (i % 3 == 2 && i < 3 * p.mrope_w) ? 2 : 0;
            ci = p.cos_sin + (long long)p.positions3[3 * t + comp] * p.rot_dim;
          }
          const float c = ci[i], s = ci[D / 2 + i];
          o[e] = v[e] * c - v[e + HP] * s;
          o[e + HP] = v[e + HP] * c + v[e] * s;
        }
#pragma unroll
        for (int e = 0; e < PER; ++e) v[e] = o[e];
      } else if (!p.neox) {
        // Interleaved pairs (2j, 2j + 1) sit in neighbouring lanes.
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          const int i = lane + 32 * e;
          const float other = __shfl_xor_sync(0xffffffffu, v[e], 1);
          if (i < p.rot_dim) {
            const int j = i >> 1;
            const float c = cs[j], s = cs[half + j];
            v[e] = (i & 1) ? v[e] * c + other * s : v[e] * c - other * s;
          }
        }
      } else {
        // neox with a rotary width that is not a multiple of 64: exchange through smem.
        __shared__ float line[8][256];
        float* Ls = line[warp & 7];
#pragma unroll
        for (int e = 0; e < PER; ++e) Ls[lane + 32 * e] = v[e];
        __syncwarp();
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          const int i = lane + 32 * e;
          if (i >= p.rot_dim) continue;
          const int j = i < half ? i : i - half;
          const float c = cs[j], s = cs[half + j];
          v[e] = i < half ? Ls[i] * c - Ls[i + half] * s : Ls[i] * c + Ls[i - half] * s;
        }
        __syncwarp();
      }
    }
    if (is_q) {
      __nv_bfloat16* dst = p.q_out + (long long)t * p.q_out_stride + (long long)h * D;
      // position-dependent query temperature (long-context scaling of the Llama-4 / Ministral-3
      // families)
      const float qs = p.q_pos_beta != 0.f
                           ? 1.f + p.q_pos_beta * logf(1.f + floorf((float)pos / p.q_pos_period))
                           : 1.f;
#pragma unroll
      for (int e = 0; e < PER; ++e) dst[lane + 32 * e] = __float2bfloat16(v[e] * qs);
    } else if (slot >= 0 && p.num_blocks > 0 && slot >= p.num_blocks * p.block_size) {
      if (lane == 0) set_status(p.status, kBadIndex);  // slot past the cache: not written
    } else if (slot >= 0) {
      const int kvh = is_k ? h - p.Hq : h - p.Hq - p.Hkv;
      const long long blk = slot / p.block_size, off = slot % p.block_size;
      const long long idx = blk * p.kv_block_stride + ((long long)kvh * p.block_size + off) * D;
      if (p.kv_fp8) {
        uint8_t* dst = reinterpret_cast<uint8_t*>(is_k ? p.k_cache : p.v_cache) + idx;
        const float inv = is_k ? p.k_inv_scale : p.v_inv_scale;
#pragma unroll
        for (int e = 0; e < PER; ++e)
          dst[lane + 32 * e] = (uint8_t)__nv_cvt_float_to_fp8(v[e] * inv, __NV_SATFINITE, __NV_E4M3);
      } else {
        __nv_bfloat16* dst = (is_k ? p.k_cache : p.v_cache) + idx;
#pragma unroll
        for (int e = 0; e < PER; ++e) dst[lane + 32 * e] = __float2bfloat16(v[e]);
      }
    }
    if (p.clear_input) {
#pragma unroll
      for (int e = 0; e < PER; ++e) src[lane + 32 * e] = from_f<TIN>(0.f);
    }
  }
}

// Vectorised form for the common layouts (full-width neox rotation or interleaved pairs, 1-D
// positions): lane l owns the D / 32 contiguous elements [l * PER, l * PER + PER) of a head, so
// every access is one 4- to 32-byte vector; the neox partner (i, i + D / 2) sits in lane l ^ 16.
// Each warp first loads all of its HPW heads, so HPW loads per lane are in flight at once --
// the per-head form above waits one load latency per head, which bounds large prefill steps.
namespace {
template <int BYTES>
__device__ __forceinline__ void ld_words(const void* src, uint32_t (&w)[BYTES / 4]) {
  if constexpr (BYTES >= 16) {
#pragma unroll
    for (int i = 0; i < BYTES / 16; ++i) {
      const uint4 u = reinterpret_cast<const uint4*>(src)[i];
      w[4 * i] = u.x; w[4 * i + 1] = u.y; w[4 * i + 2] = u.z; w[4 * i + 3] = u.w;
    }
  } else if constexpr (BYTES == 8) {
    const uint2 u = *reinterpret_cast<const uint2*>(src);
    w[0] = u.x; w[1] = u.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(src);
  }
}
template <int BYTES>
__device__ __forceinline__ void st_words(void* dst, const uint32_t (&w)[BYTES / 4]) {
  if constexpr (BYTES >= 16) {
#pragma unroll
    for (int i = 0; i < BYTES / 16; ++i)
      reinterpret_cast<uint4*>(dst)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  } else if constexpr (BYTES == 8) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  } else {
    *reinterpret_cast<uint32_t*>(dst) = w[0];
  }
}
template <typename T, int N>
__device__ __forceinline__ void ld_vec(const T* src, float (&v)[N]) {
  if constexpr (sizeof(T) == 4) {
    uint32_t w[N];
    ld_words<4 * N>(src, w);
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = __uint_as_float(w[i]);
  } else {
    uint32_t w[N / 2];
    ld_words<2 * N>(src, w);
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
      const float2 f = unpack_bf16x2(w[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}
template <int N>
__device__ __forceinline__ void st_vec_bf16(__nv_bfloat16* dst, const float (&v)[N], float mul) {
  uint32_t w[N / 2];
#pragma unroll
  for (int i = 0; i < N / 2; ++i) w[i] = pack_bf16x2(v[2 * i] * mul, v[2 * i + 1] * mul);
  st_words<N * 2>(dst, w);
}
template <typename T, int N>
__device__ __forceinline__ void zero_vec(T* dst) {
  uint32_t w[N * sizeof(T) / 4];
#pragma unroll
  for (int i = 0; i < (int)(N * sizeof(T) / 4); ++i) w[i] = 0u;
  st_words<N * sizeof(T)>(dst, w);
}
}  // namespace

constexpr int kRopeHeadsPerWarp = 4;

template <typename TIN, int D>
__global__ void __launch_bounds__(256) rope_kv_write_vec_kernel(const RopeKvParams p, TIN* qkv) {
  pdl_trigger();
  pdl_wait();
  constexpr int PER = D / 32;
  constexpr int HPW = kRopeHeadsPerWarp;
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nheads = p.Hq + 2 * p.Hkv;
  const int h0 = ((int)blockIdx.y * (blockDim.x >> 5) + warp) * HPW;
  if (h0 >= nheads) return;
  const int pos = p.positions[t];
  const long long slot = p.slot_mapping ? (long long)p.slot_mapping[t] : -1;
  TIN* row = qkv + (long long)t * p.qkv_stride;
  const int e0 = lane * PER;  // first element of this lane
  float v[HPW][PER];
#pragma unroll
  for (int hh = 0; hh < HPW; ++hh)
    if (h0 + hh < nheads) ld_vec<TIN, PER>(row + (long long)(h0 + hh) * D + e0, v[hh]);
  // rotary coefficients of this lane's elements
  const float* cs = p.cos_sin + (long long)pos * p.rot_dim;
  float c[PER], sn[PER];
  if (p.neox) {  // full width: element i pairs with i +- D / 2, frequency i mod D / 2
    const int j0 = (lane & 15) * PER;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      c[e] = cs[j0 + e];
      sn[e] = cs[D / 2 + j0 + e];
    }
  } else {  // interleaved pairs (2j, 2j + 1) inside the lane; elements past rot_dim keep c = 1
    const int half = p.rot_dim / 2;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      const int i = e0 + e;
      c[e] = i < p.rot_dim ? cs[i >> 1] : 1.f;
      sn[e] = i < p.rot_dim ? cs[half + (i >> 1)] : 0.f;
    }
  }
  const float qs = p.q_pos_beta != 0.f ? 1.f + p.q_pos_beta * logf(1.f + floorf((float)pos / p.q_pos_period)) : 1.f;
#pragma unroll
  for (int hh = 0; hh < HPW; ++hh) {
    const int h = h0 + hh;
    if (h >= nheads) break;
    const bool is_q = h < p.Hq;
    const bool is_k = !is_q && h < p.Hq + p.Hkv;
    float (&x)[PER] = v[hh];
    if (p.qkv_bias != nullptr) {
      float b[PER];
      ld_vec<float, PER>(p.qkv_bias + (long long)h * D + e0, b);
#pragma unroll
      for (int e = 0; e < PER; ++e) x[e] += b[e];
    }
    if ((is_q && p.q_norm_w) || (is_k && p.k_norm_w)) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < PER; ++e) ss += x[e] * x[e];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / (float)D + p.eps);
      float w[PER];
      ld_vec<__nv_bfloat16, PER>(is_q ? p.q_norm_w + e0 : p.k_norm_w + e0, w);
#pragma unroll
      for (int e = 0; e < PER; ++e) x[e] = __bfloat162float(__float2bfloat16(x[e] * inv * w[e]));
    }
    if (is_q || is_k) {
      if (p.neox) {
        const float sgn = lane < 16 ? -1.f : 1.f;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          const float other = __shfl_xor_sync(0xffffffffu, x[e], 16);
          x[e] = x[e] * c[e] + sgn * other * sn[e];
        }
      } else {
#pragma unroll
        for (int e = 0; e < PER; e += 2) {
          const float a = x[e], b = x[e + 1];
          x[e] = a * c[e] - b * sn[e];
          x[e + 1] = b * c[e + 1] + a * sn[e + 1];
        }
      }
    }
    if (is_q) {
      st_vec_bf16<PER>(p.q_out + (long long)t * p.q_out_stride + (long long)h * D + e0, x, qs);
    } else if (slot >= 0 && p.num_blocks > 0 && slot >= p.num_blocks * p.block_size) {
      if (lane == 0) set_status(p.status, kBadIndex);  // slot past the cache: not written
    } else if (slot >= 0) {
      const int kvh = is_k ? h - p.Hq : h - p.Hq - p.Hkv;
      const long long blk = slot / p.block_size, off = slot % p.block_size;
      const long long idx = blk * p.kv_block_stride + ((long long)kvh * p.block_size + off) * D + e0;
      if (p.kv_fp8) {
        uint8_t* dst = reinterpret_cast<uint8_t*>(is_k ? p.k_cache : p.v_cache) + idx;
        const float inv = is_k ? p.k_inv_scale : p.v_inv_scale;
#pragma unroll
        for (int e = 0; e < PER; ++e)
          dst[e] = (uint8_t)__nv_cvt_float_to_fp8(x[e] * inv, __NV_SATFINITE, __NV_E4M3);
      } else {
        st_vec_bf16<PER>((is_k ? p.k_cache : p.v_cache) + idx, x, 1.f);
      }
    }
    if (p.clear_input) zero_vec<TIN, PER>(row + (long long)h * D + e0);
  }
}

void rope_kv_write_launch(const RopeKvParams& p, void* qkv, bool qkv_is_f32, int T,
                          cudaStream_t stream) {
  if (T == 0) return;
  if (p.positions3 != nullptr && !(p.neox && p.rot_dim == p.head_dim && p.head_dim >= 64))
    throw std::invalid_argument("rope_kv_write: multimodal RoPE needs full-width neox rotation");
  const int esz = qkv_is_f32 ? 4 : 2;
  const bool vec = p.positions3 == nullptr && (!p.neox || p.rot_dim == p.head_dim) && (p.rot_dim % 2) == 0 &&
                   (p.qkv_stride * esz) % 16 == 0 && (p.q_out_stride * 2) % 16 == 0 &&
                   (p.kv_block_stride * (p.kv_fp8 ? 1 : 2)) % 16 == 0;
  if (vec) {
    // 8 warps x kRopeHeadsPerWarp heads per CTA, grid (tokens, head groups)
    const int per_cta = 8 * kRopeHeadsPerWarp;
    const dim3 vgrid(T, (p.Hq + 2 * p.Hkv + per_cta - 1) / per_cta);
#define B200_ROPE_VEC(D_)                                                                   \
    if (p.head_dim == D_) {                                                                 \
      if (qkv_is_f32)                                                                       \
        launch_pdl(rope_kv_write_vec_kernel<float, D_>, vgrid, dim3(256), 0, stream, p,      \
                   (float*)qkv);                                                            \
      else                                                                                  \
        launch_pdl(rope_kv_write_vec_kernel<__nv_bfloat16, D_>, vgrid, dim3(256), 0, stream, \
                   p, (__nv_bfloat16*)qkv);                                                 \
      return;                                                                               \
    }
    B200_ROPE_VEC(64)
    B200_ROPE_VEC(128)
    B200_ROPE_VEC(256)
#undef B200_ROPE_VEC
  }
  // one warp per head: 8 heads per CTA, grid (tokens, head groups)
  const dim3 grid(T, (p.Hq + 2 * p.Hkv + 7) / 8);
#define B200_ROPE(D_)                                                                       \
  if (p.head_dim == D_) {                                                                   \
    if (qkv_is_f32)                                                                         \
      launch_pdl(rope_kv_write_kernel<float, D_>, grid, dim3(256), 0, stream, p,             \
                 (float*)qkv);                                                              \
    else                                                                                    \
      launch_pdl(rope_kv_write_kernel<__nv_bfloat16, D_>, grid, dim3(256), 0, stream, p,     \
                 (__nv_bfloat16*)qkv);                                                      \
    return;                                                                                 \
  }
  B200_ROPE(64)
  B200_ROPE(128)
  B200_ROPE(256)
#undef B200_ROPE
  throw std::invalid_argument("rope_kv_write: head_dim must be 64, 128 or 256");
}

// ------------------------------------------------------------------------------------------
// SiLU(gate) * up
// ------------------------------------------------------------------------------------------
template <typename TIN, int VEC>
__global__ void silu_mul_kernel(TIN* in, long long in_stride, __nv_bfloat16* out,
                                long long out_stride, int I, int blk, bool clear_input,
                                float limit, float alpha, int act) {
  pdl_trigger();
  pdl_wait();
  const long long t = blockIdx.y;
  TIN* r = in + t * in_stride;
  const int j = (blockIdx.x * blockDim.x + threadIdx.x) * VEC;
  if (j >= I) return;
  int gi, ui;
  if (blk > 0) {
    const int b = j / blk, w = j % blk;
    gi = b * 2 * blk + w;
    ui = gi + blk;
  } else {
    gi = j;
    ui = j + I;
  }
  float g[VEC], u[VEC], y[VEC];
  if constexpr (VEC == 8) {
    load8<TIN>(r + gi, g);
    load8<TIN>(r + ui, u);
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      g[e] = to_f(r[gi + e]);
      u[e] = to_f(r[ui + e]);
    }
  }
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
    float gg = g[e], uu = u[e];
    if (act == 0) {  // SwiGLU
      y[e] = gg / (1.f + __expf(-gg)) * uu;
    } else {  // GPT-OSS clamped SwiGLU: (up + 1) * gate * sigmoid(alpha * gate)
      gg = fminf(gg, limit);
      uu = fminf(fmaxf(uu, -limit), limit);
      y[e] = (uu + 1.f) * gg / (1.f + __expf(-alpha * gg));
    }
  }
  if constexpr (VEC == 8) {
    store8_bf16(out + t * out_stride + j, y);
    if (clear_input) {
      zero8<TIN>(r + gi);
      zero8<TIN>(r + ui);
    }
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      out[t * out_stride + j + e] = __float2bfloat16(y[e]);
      if (clear_input) {
        r[gi + e] = from_f<TIN>(0.f);
        r[ui + e] = from_f<TIN>(0.f);
      }
    }
  }
}

void silu_mul_launch(void* in, bool in_is_f32, long long in_stride, __nv_bfloat16* out,
                     long long out_stride, int T, int I, int blk, bool clear_input, int act,
                     float limit, float alpha, cudaStream_t stream) {
  if (T == 0) return;
  const bool vec8 = (I % 8 == 0) && (blk % 8 == 0) && (in_stride % 8 == 0) && (out_stride % 8 == 0);
  if (vec8) {
    dim3 grid((I / 8 + 127) / 128, T);
    if (in_is_f32)
      launch_pdl(silu_mul_kernel<float, 8>, grid, dim3(128), 0, stream, (float*)in, in_stride, out, out_stride, I,
                                                          blk, clear_input, limit, alpha, act);
    else
      launch_pdl(silu_mul_kernel<__nv_bfloat16, 8>, grid, dim3(128), 0, stream, 
          (__nv_bfloat16*)in, in_stride, out, out_stride, I, blk, false, limit, alpha, act);
  } else {
    dim3 grid((I + 255) / 256, T);
    if (in_is_f32)
      launch_pdl(silu_mul_kernel<float, 1>, grid, dim3(256), 0, stream, (float*)in, in_stride, out, out_stride, I,
                                                          blk, clear_input, limit, alpha, act);
    else
      launch_pdl(silu_mul_kernel<__nv_bfloat16, 1>, grid, dim3(256), 0, stream, 
          (__nv_bfloat16*)in, in_stride, out, out_stride, I, blk, false, limit, alpha, act);
  }
}

// ------------------------------------------------------------------------------------------
// Embedding lookup (vocab-sharded).
// ------------------------------------------------------------------------------------------
__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* out, int H, int vocab_start, int vocab_end,
                                 const int* __restrict__ last_tok) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 && last_tok != nullptr) id = last_tok[-id - 1];
  const bool own = id >= vocab_start && id < vocab_end;
  const uint4* src = reinterpret_cast<const uint4*>(table + (long long)(own ? id - vocab_start : 0) * H);
  uint4* dst = reinterpret_cast<uint4*>(out + (long long)t * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = own ? src[i] : make_uint4(0, 0, 0, 0);
}

void embedding_launch(const int* ids, const __nv_bfloat16* table, __nv_bfloat16* out, int T,
                      int H, int vocab_start, int vocab_end, const int* last_tok,
                      cudaStream_t stream) {
  if (T == 0) return;
  if (H % 8 != 0) throw std::invalid_argument("embedding: hidden size must be a multiple of 8");
  launch_pdl(embedding_kernel, dim3(T), dim3(128), 0, stream, ids, table, out, H, vocab_start,
             vocab_end, last_tok);
}

}  // namespace b200
