// On-device sampling: greedy, temperature, top-k, top-p and min-p, one CTA per row.
//
// Method.  With x = logits / T and m = max(x), the kept set is {i : x_i >= tau} where tau is
// the largest of: the k-th largest x (top-k), the smallest value whose upper tail holds
// probability mass >= p (top-p, computed inside the top-k set), and m + log(min_p).  Both
// thresholds come from an MSB-first radix select over order-preserving 32-bit keys of x
// (four 8-bit digit passes; counts for top-k, exp-mass for top-p).  The token is then drawn
// by the Gumbel-max trick, argmax_{x_i >= tau} (x_i - log(-log u_i)), which samples exactly
// from softmax restricted to the kept set.  u_i comes from a counter-based hash
// (SplitMix64 finalizer, Steele, Lea & Flood, OOPSLA 2014) of (seed, step offset, i), so a
// seeded request reproduces its tokens.
//
// Reference semantics: vllm_neuron/functional/sampling.py:21 (per-request temperature /
// top-k / top-p, greedy fast path via argmax), functional/topk.py:124, functional/argmax.py:27.
#include <cuda_bf16.h>

#include "../common.cuh"
#include "misc.h"

namespace b200 {

namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ float load_logit(const void* base, bool f32, long long idx) {
  return f32 ? reinterpret_cast<const float*>(base)[idx]
             : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
}

__device__ __forceinline__ uint32_t f2key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
// Uniform in (0, 1).
__device__ __forceinline__ float uniform01(uint64_t seed, uint32_t offset, uint32_t i) {
  const uint64_t h = mix64(seed ^ mix64(((uint64_t)offset << 32) | i));
  return ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
}

// Calls f(i, x) for every logit of the row owned by this thread (strided over the CTA);
// bf16 rows aligned to 16 bytes are read 8 logits per load.
template <typename F>
__device__ __forceinline__ void for_each_logit(const void* row, bool f32, int V, F&& f) {
  if (!f32 && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    const uint4* r4 = reinterpret_cast<const uint4*>(row);
    const int nv = V / 8;
#pragma unroll 4
    for (int j = threadIdx.x; j < nv; j += blockDim.x) {
      const uint4 u = __ldg(r4 + j);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 v = unpack_bf16x2(w[q]);
        f(8 * j + 2 * q, v.x);
        f(8 * j + 2 * q + 1, v.y);
      }
    }
    for (int i = nv * 8 + threadIdx.x; i < V; i += blockDim.x)
      f(i, __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(row)[i]));
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x) f(i, load_logit(row, f32, i));
  }
}

struct ArgMax {
  float v;
  int i;
};
__device__ __forceinline__ ArgMax amax(ArgMax a, ArgMax b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}
__device__ ArgMax block_argmax(ArgMax a, ArgMax* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax b;
    b.v = __shfl_xor_sync(0xffffffffu, a.v, o);
    b.i = __shfl_xor_sync(0xffffffffu, a.i, o);
    a = amax(a, b);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = a;
  __syncthreads();
  if (w == 0) {
    a = (l < (int)(blockDim.x >> 5)) ? red[l] : ArgMax{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ArgMax b;
      b.v = __shfl_xor_sync(0xffffffffu, a.v, o);
      b.i = __shfl_xor_sync(0xffffffffu, a.i, o);
      a = amax(a, b);
    }
    if (l == 0) red[0] = a;
  }
  __syncthreads();
  return red[0];
}
__device__ float block_reduce(float v, float* red, bool is_max) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float t = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, t) : v + t;
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < (int)(blockDim.x >> 5)) ? red[l] : (is_max ? -INFINITY : 0.f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float t = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, t) : v + t;
    }
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// Radix select over keys of x >= floor_key.  Finds the largest key K such that the
// "weight" of {keys >= K} is >= target, where weight is a count (use_mass = false) or the
// exp-mass exp(x - m) (use_mass = true).  Returns K.
__device__ uint32_t radix_select(const void* row, bool f32, int V, float inv_t, float m,
                                 uint32_t floor_key, float target, bool use_mass,
                                 float* hist /*[256]*/, float* scratch /*[64]*/) {
  uint32_t prefix = 0, mask = 0;
  float remaining = target;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0.f;
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float x = load_logit(row, f32, i) * inv_t;
      const uint32_t k = f2key(x);
      if (k >= floor_key && (k & mask) == prefix) {
        const int d = (k >> shift) & 0xFF;
        atomicAdd(&hist[d], use_mass ? __expf(x - m) : 1.f);
      }
    }
    __syncthreads();
    // Warp 0 scans the bins from the top: lane l owns bins 255-8l .. 248-8l.
    if (threadIdx.x < 32) {
      const int l = threadIdx.x;
      float loc[8], s = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        loc[j] = hist[255 - 8 * l - j];
        s += loc[j];
      }
      float incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float t = __shfl_up_sync(0xffffffffu, incl, o);
        if (l >= o) incl += t;
      }
      const float excl = incl - s;
      const bool crosses = incl >= remaining && excl < remaining;
      const unsigned ball = __ballot_sync(0xffffffffu, crosses);
      // If rounding kept every prefix below the target, fall back to the lowest bin.
      const int owner = ball ? __ffs(ball) - 1 : 31;
      if (l == owner) {
        float c = excl;
        int bin = 255 - 8 * l - 7;
        float before = c;
        for (int j = 0; j < 8; ++j) {
          if (c + loc[j] >= remaining || j == 7) {
            bin = 255 - 8 * l - j;
            before = c;
            break;
          }
          c += loc[j];
        }
        scratch[0] = (float)bin;
        scratch[1] = remaining - before;
      }
    }
    __syncthreads();
    const int bin = (int)scratch[0];
    remaining = scratch[1];
    prefix |= (uint32_t)bin << shift;
    mask |= 0xFFu << shift;
    __syncthreads();
  }
  return prefix;
}

}  // namespace

__global__ void __launch_bounds__(kThreads) sample_kernel(const SampleParams p) {
  pdl_trigger();
  pdl_wait();
  __shared__ ArgMax red_am[32];
  __shared__ float red[32];
  __shared__ float hist[256];
  __shared__ float scratch[64];
  const int b = blockIdx.x;
  const void* row = p.logits_f32
                        ? (const void*)(reinterpret_cast<const float*>(p.logits) + b * p.logits_stride)
                        : (const void*)(reinterpret_cast<const __nv_bfloat16*>(p.logits) +
                                        b * p.logits_stride);
  const float temp = p.temperature ? p.temperature[b] : 0.f;
  const bool greedy = !(temp > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / temp;

  // Row max (and argmax for greedy).
  ArgMax best{-INFINITY, 0x7fffffff};
  for_each_logit(row, p.logits_f32, p.V, [&](int i, float v) { best = amax(best, ArgMax{v * inv_t, i}); });
  best = block_argmax(best, red_am);
  const float m = best.v;

  if (greedy) {
    if (p.out_logprob) {
      float z = 0.f;
      for_each_logit(row, p.logits_f32, p.V, [&](int, float v) { z += __expf(v - m); });
      z = block_reduce(z, red, false);
      if (threadIdx.x == 0) p.out_logprob[b] = -logf(z);
    }
    if (threadIdx.x == 0) {
      p.out_tokens[b] = best.i + p.vocab_offset;
      if (p.row_slots) p.last_tok[p.row_slots[b]] = best.i + p.vocab_offset;
      if (p.out_max) p.out_max[b] = m;
    }
    return;
  }

  uint32_t floor_key = 0;
  const int k = p.top_k ? p.top_k[b] : 0;
  if (k > 0 && k < p.V) {
    floor_key = radix_select(row, p.logits_f32, p.V, inv_t, m, 0u, (float)k, false, hist, scratch);
  }
  const float tp = p.top_p ? p.top_p[b] : 1.f;
  if (tp < 1.f) {
    float z = 0.f;
    for_each_logit(row, p.logits_f32, p.V, [&](int, float v) {
      const float x = v * inv_t;
      if (f2key(x) >= floor_key) z += __expf(x - m);
    });
    z = block_reduce(z, red, false);
    const uint32_t kp = radix_select(row, p.logits_f32, p.V, inv_t, m, floor_key, tp * z, true,
                                     hist, scratch);
    floor_key = max(floor_key, kp);
  }
  const float mp = p.min_p ? p.min_p[b] : 0.f;
  if (mp > 0.f) floor_key = max(floor_key, f2key(m + logf(mp)));

  const uint64_t seed = p.seeds ? p.seeds[b] : 0ull;
  const uint32_t off = p.offsets ? (uint32_t)p.offsets[b] : 0u;
  ArgMax g{-INFINITY, 0x7fffffff};
  float z = 0.f;
  for_each_logit(row, p.logits_f32, p.V, [&](int i, float v) {
    const float x = v * inv_t;
    if (f2key(x) < floor_key) return;
    z += __expf(x - m);
    const float u = uniform01(seed, off, (uint32_t)(i + p.vocab_offset));
    g = amax(g, ArgMax{x - __logf(-__logf(u)), i});
  });
  g = block_argmax(g, red_am);
  if (p.out_logprob) z = block_reduce(z, red, false);
  if (threadIdx.x == 0) {
    const int tok = g.i == 0x7fffffff ? best.i : g.i;
    p.out_tokens[b] = tok + p.vocab_offset;
    if (p.row_slots) p.last_tok[p.row_slots[b]] = tok + p.vocab_offset;
    if (p.out_logprob) p.out_logprob[b] = load_logit(row, p.logits_f32, tok) * inv_t - m - logf(z);
    if (p.out_max) p.out_max[b] = m;
  }
}

void sample_launch(const SampleParams& p, cudaStream_t stream) {
  if (p.B == 0) return;
  launch_pdl(sample_kernel, dim3(p.B), dim3(kThreads), 0, stream, p);
}

__global__ void __launch_bounds__(kThreads)
    argmax_kernel(const void* logits, bool f32, long long stride, int V, int* out_idx,
                  float* out_val, int vocab_offset) {
  pdl_trigger();
  pdl_wait();
  __shared__ ArgMax red_am[32];
  const int b = blockIdx.x;
  const void* row = f32 ? (const void*)(reinterpret_cast<const float*>(logits) + b * stride)
                        : (const void*)(reinterpret_cast<const __nv_bfloat16*>(logits) + b * stride);
  ArgMax best{-INFINITY, 0x7fffffff};
  for (int i = threadIdx.x; i < V; i += blockDim.x)
    best = amax(best, ArgMax{load_logit(row, f32, i), i});
  best = block_argmax(best, red_am);
  if (threadIdx.x == 0) {
    out_idx[b] = best.i + vocab_offset;
    if (out_val) out_val[b] = best.v;
  }
}

void argmax_launch(const void* logits, bool f32, long long stride, int B, int V, int* out_idx,
                   float* out_val, int vocab_offset, cudaStream_t stream) {
  if (B == 0) return;
  launch_pdl(argmax_kernel, dim3(B), dim3(kThreads), 0, stream, logits, f32, stride, V, out_idx,
             out_val, vocab_offset);
}

// Structured outputs: logits[r, i] = -inf where bit i of row r's token bitmask is 0
// (bitmask int32 [rows, ceil(V / 32)], bit i % 32 of word i / 32; reference:
// vllm_neuron/vllm/core/scheduler.py:940-952 attaches the grammar bitmask, applied before
// sampling in nn/sampler.py:13-169).
__global__ void apply_token_bitmask_kernel(__nv_bfloat16* logits, long long stride, int V,
                                           const int32_t* __restrict__ mask, int words) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= V) return;
  const uint32_t w = (uint32_t)mask[(long long)r * words + (i >> 5)];
  if (!((w >> (i & 31)) & 1u)) logits[(long long)r * stride + i] = __float2bfloat16(-INFINITY);
}

void apply_token_bitmask_launch(__nv_bfloat16* logits, long long stride, int rows, int V,
                                const int32_t* mask, int words, cudaStream_t stream) {
  if (rows == 0) return;
  launch_pdl(apply_token_bitmask_kernel, dim3((V + 255) / 256, rows), dim3(256), 0, stream, logits,
             stride, V, mask, words);
}

}  // namespace b200
