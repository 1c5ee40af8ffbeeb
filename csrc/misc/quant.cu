// FP8 (e4m3) activation quantization for W8A8 GEMMs.
//
//   quant_fp8       out = satfinite(x * inv_scale) for bf16 rows (static per-tensor scale)
//   rmsnorm_quant   y = rmsnorm(x) * w, then either the static per-tensor quantization above
//                   (STATIC) or a per-row scale s_row = max|y| / 448 with out = y / s_row and
//                   s_row written to `row_scales` (ROW)
//
// Reference: rmsnorm_quant (vllm_neuron/functional/rmsnorm_quant.py:216; STATIC and ROW modes,
// the reference packs the row scale into 4 extra fp8 bytes, here it is a separate fp32 vector).
// Conversion is the hardware cvt (__nv_cvt_float_to_fp8, satfinite, round to nearest even).
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <stdexcept>

#include "../common.cuh"
#include "misc.h"

namespace b200 {

namespace {
__device__ __forceinline__ uint32_t q4(float a, float b, float c, float d) {
  return (uint32_t)__nv_cvt_float_to_fp8(a, __NV_SATFINITE, __NV_E4M3) |
         ((uint32_t)__nv_cvt_float_to_fp8(b, __NV_SATFINITE, __NV_E4M3) << 8) |
         ((uint32_t)__nv_cvt_float_to_fp8(c, __NV_SATFINITE, __NV_E4M3) << 16) |
         ((uint32_t)__nv_cvt_float_to_fp8(d, __NV_SATFINITE, __NV_E4M3) << 24);
}
}  // namespace

// grid (rows, ceil(cols / 2048)), 256 threads x 8 elements
__global__ void __launch_bounds__(256) quant_fp8_kernel(const __nv_bfloat16* __restrict__ x,
                                                        long long ldx, uint8_t* __restrict__ out,
                                                        long long ldo, int cols, float inv_scale) {
  pdl_trigger();
  pdl_wait();
  const long long r = blockIdx.x;
  const int c = (blockIdx.y * 256 + threadIdx.x) * 8;
  if (c >= cols) return;
  const uint4 v = *reinterpret_cast<const uint4*>(x + r * ldx + c);
  const float2 a = unpack_bf16x2(v.x), b = unpack_bf16x2(v.y), d = unpack_bf16x2(v.z),
               e = unpack_bf16x2(v.w);
  *reinterpret_cast<uint2*>(out + r * ldo + c) =
      make_uint2(q4(a.x * inv_scale, a.y * inv_scale, b.x * inv_scale, b.y * inv_scale),
                 q4(d.x * inv_scale, d.y * inv_scale, e.x * inv_scale, e.y * inv_scale));
}

// One CTA (256 threads) per row, H <= 8192.
template <int NV>
__global__ void __launch_bounds__(256) rmsnorm_quant_kernel(const __nv_bfloat16* __restrict__ x,
                                                            long long ldx,
                                                            const __nv_bfloat16* __restrict__ w,
                                                            float eps, uint8_t* __restrict__ out,
                                                            long long ldo, int H, float inv_scale,
                                                            float* __restrict__ row_scales) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[8];
  __shared__ float redm[8];
  const long long r = blockIdx.x;
  const int tid = threadIdx.x;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int idx = (j * 256 + tid) * 8;
    if (idx < H) {
      const uint4 u = *reinterpret_cast<const uint4*>(x + r * ldx + idx);
      const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(uw[i]);
        v[j][2 * i] = f.x;
        v[j][2 * i + 1] = f.y;
        ss += f.x * f.x + f.y * f.y;
      }
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float rstd = rsqrtf(tot / (float)H + eps);
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int idx = (j * 256 + tid) * 8;
    if (idx < H) {
      const uint4 u = *reinterpret_cast<const uint4*>(w + idx);
      const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(uw[i]);
        // the normalized value is rounded to bf16 before the weight (as the bf16 RMSNorm)
        v[j][2 * i] = __bfloat162float(__float2bfloat16(v[j][2 * i] * rstd)) * f.x;
        v[j][2 * i + 1] = __bfloat162float(__float2bfloat16(v[j][2 * i + 1] * rstd)) * f.y;
        amax = fmaxf(amax, fmaxf(fabsf(v[j][2 * i]), fabsf(v[j][2 * i + 1])));
      }
    }
  }
  float inv = inv_scale;
  if (row_scales != nullptr) {
    amax = warp_max(amax);
    if ((tid & 31) == 0) redm[tid >> 5] = amax;
    __syncthreads();
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, redm[i]);
    const float s = m > 0.f ? m / 448.f : 1.f;
    inv = 1.f / s;
    if (tid == 0) row_scales[r] = s;
  }
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int idx = (j * 256 + tid) * 8;
    if (idx < H)
      *reinterpret_cast<uint2*>(out + r * ldo + idx) =
          make_uint2(q4(v[j][0] * inv, v[j][1] * inv, v[j][2] * inv, v[j][3] * inv),
                     q4(v[j][4] * inv, v[j][5] * inv, v[j][6] * inv, v[j][7] * inv));
  }
}

// Per-token, per-128-column block quantization (the activations of the block-scaled W8A8 GEMM):
// one warp per (row, block): s = max|x| / 448 over the block's 128 values (1 for an all-zero
// block), out = satfinite(x / s), s written to scales[row * lds + block].
__global__ void __launch_bounds__(256) quant_fp8_block_kernel(const __nv_bfloat16* __restrict__ x,
                                                              long long ldx, uint8_t* __restrict__ out,
                                                              long long ldo, float* __restrict__ scales,
                                                              int lds, int nblk) {
  pdl_trigger();
  pdl_wait();
  const long long r = blockIdx.x;
  const int b = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= nblk) return;
  const int c = b * 128 + lane * 4;
  const uint2 v = *reinterpret_cast<const uint2*>(x + r * ldx + c);
  const float2 a = unpack_bf16x2(v.x), d = unpack_bf16x2(v.y);
  float m = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(d.x), fabsf(d.y)));
  m = warp_max(m);
  const float sc = m > 0.f ? m / 448.f : 1.f;
  const float inv = 1.f / sc;
  *reinterpret_cast<uint32_t*>(out + r * ldo + c) = q4(a.x * inv, a.y * inv, d.x * inv, d.y * inv);
  if (lane == 0) scales[r * lds + b] = sc;
}

void quant_fp8_block_launch(const __nv_bfloat16* x, long long ldx, uint8_t* out, long long ldo,
                            float* scales, int lds, int rows, int cols, cudaStream_t stream) {
  if (rows == 0) return;
  if (cols % 128 != 0 || ldx % 4 != 0 || ldo % 4 != 0 || lds < cols / 128)
    throw std::invalid_argument("quant_fp8_block: columns must be a multiple of 128");
  const int nblk = cols / 128;
  launch_pdl(quant_fp8_block_kernel, dim3(rows, (nblk + 7) / 8), dim3(256), 0, stream, x, ldx, out, ldo,
             scales, lds, nblk);
}

// MXFP8 quantization (OCP microscaling, e4m3 elements, e8m0 scale per 32 elements): one warp per
// (row, 128-column block), 8 lanes per 32-element group.  The group's scale is the smallest
// power of two 2^e with max|x| <= 448 * 2^e, so the scaled values never saturate and
// q = rn_e4m3(x * 2^-e) is an exact power-of-two scaling before the rounding.  Scales go into
// the 512-byte atom layout the block-scaled GEMM reads: atom (row / 128, block) holds, for row r,
// its 4 group scales at (r % 32) * 16 + ((r / 32) % 4) * 4.
__global__ void __launch_bounds__(256) quant_mx8_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                        uint8_t* __restrict__ out, long long ldo,
                                                        uint8_t* __restrict__ sf, int nblk) {
  pdl_trigger();
  pdl_wait();
  const long long r = blockIdx.x;
  const int b = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= nblk) return;
  const int c = b * 128 + lane * 4;
  const uint2 v = *reinterpret_cast<const uint2*>(x + r * ldx + c);
  const float2 a = unpack_bf16x2(v.x), d = unpack_bf16x2(v.y);
  float m = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(d.x), fabsf(d.y)));
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  // m = 1.f * 2^(E - 127): m <= 1.75 * 2^(8 + e) <=> e >= E - 135 (+1 when 1.f > 1.75)
  const uint32_t bits = __float_as_uint(m);
  int e = (int)((bits >> 23) & 0xffu) - 135 + ((bits & 0x7fffffu) > 0x600000u ? 1 : 0);
  if (m == 0.f) e = 0;
  e = max(-127, min(127, e));
  const float inv = e >= 127 ? __uint_as_float(0x00400000u) : __uint_as_float((uint32_t)(127 - e) << 23);
  *reinterpret_cast<uint32_t*>(out + r * ldo + c) = q4(a.x * inv, a.y * inv, d.x * inv, d.y * inv);
  if ((lane & 7) == 0) {
    const int ri = (int)(r & 127);
    sf[((r >> 7) * nblk + b) * 512 + (ri & 31) * 16 + (ri >> 5) * 4 + (lane >> 3)] = (uint8_t)(e + 127);
  }
}

// The same for the expert-sorted rows of a grouped GEMM: the scales go into one atom per
// tile-list entry (entry t covers rows [first, min(first + 128, end)) of its expert; row
// first + i is atom row i), the layout the grouped block-scaled GEMM reads for its token operand.
// Columns at or past `kvalid` are quantized as zeros (K padded to a multiple of 128).
// grid (gmax, ceil(nblk / 8)), 8 warps, one 128-column block per warp.
__global__ void __launch_bounds__(256) quant_mx8_tiles_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                              uint8_t* __restrict__ out, long long ldo,
                                                              uint8_t* __restrict__ sf, const int4* __restrict__ tiles,
                                                              const int* __restrict__ count, int nblk, int kvalid) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int b = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= *count || b >= nblk) return;
  const int4 g = tiles[t];
  const int r1 = min(g.y + 128, g.z);
  const int c = b * 128 + lane * 4;
  for (int r = g.y; r < r1; ++r) {
    float2 a = make_float2(0.f, 0.f), d = make_float2(0.f, 0.f);
    if (c < kvalid) {  // kvalid % 4 == 0: a lane's 4 columns are all valid or all padding
      const uint2 v = *reinterpret_cast<const uint2*>(x + (long long)r * ldx + c);
      a = unpack_bf16x2(v.x);
      d = unpack_bf16x2(v.y);
    }
    float m = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(d.x), fabsf(d.y)));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const uint32_t bits = __float_as_uint(m);
    int e = (int)((bits >> 23) & 0xffu) - 135 + ((bits & 0x7fffffu) > 0x600000u ? 1 : 0);
    if (m == 0.f) e = 0;
    e = max(-127, min(127, e));
    const float inv = e >= 127 ? __uint_as_float(0x00400000u) : __uint_as_float((uint32_t)(127 - e) << 23);
    *reinterpret_cast<uint32_t*>(out + (long long)r * ldo + c) = q4(a.x * inv, a.y * inv, d.x * inv, d.y * inv);
    if ((lane & 7) == 0) {
      const int ri = r - g.y;
      sf[((long long)t * nblk + b) * 512 + (ri & 31) * 16 + (ri >> 5) * 4 + (lane >> 3)] = (uint8_t)(e + 127);
    }
  }
}

void quant_mx8_tiles_launch(const __nv_bfloat16* x, long long ldx, uint8_t* out, long long ldo, uint8_t* sf,
                            const int* tiles, const int* count, int gmax, int cols, int kvalid,
                            cudaStream_t stream) {
  if (gmax == 0) return;
  if (cols % 128 != 0 || kvalid % 4 != 0 || kvalid > cols || ldx % 4 != 0 || ldo % 4 != 0)
    throw std::invalid_argument("quant_mx8_tiles: columns must be a multiple of 128, valid columns of 4");
  const int nblk = cols / 128;
  launch_pdl(quant_mx8_tiles_kernel, dim3(gmax, (nblk + 7) / 8), dim3(256), 0, stream, x, ldx, out, ldo, sf,
             reinterpret_cast<const int4*>(tiles), count, nblk, kvalid);
}

void quant_mx8_launch(const __nv_bfloat16* x, long long ldx, uint8_t* out, long long ldo, uint8_t* sf,
                      int rows, int cols, cudaStream_t stream) {
  if (rows == 0) return;
  if (cols % 128 != 0 || ldx % 4 != 0 || ldo % 4 != 0)
    throw std::invalid_argument("quant_mx8: columns must be a multiple of 128");
  const int nblk = cols / 128;
  launch_pdl(quant_mx8_kernel, dim3(rows, (nblk + 7) / 8), dim3(256), 0, stream, x, ldx, out, ldo, sf, nblk);
}

void quant_fp8_launch(const __nv_bfloat16* x, long long ldx, uint8_t* out, long long ldo, int rows,
                      int cols, float inv_scale, cudaStream_t stream) {
  if (rows == 0) return;
  if (cols % 8 != 0 || ldx % 8 != 0 || ldo % 8 != 0)
    throw std::invalid_argument("quant_fp8: columns and row pitches must be multiples of 8");
  launch_pdl(quant_fp8_kernel, dim3(rows, (cols + 2047) / 2048), dim3(256), 0, stream, x, ldx, out,
             ldo, cols, inv_scale);
}

void rmsnorm_quant_launch(const __nv_bfloat16* x, long long ldx, const __nv_bfloat16* w, float eps,
                          uint8_t* out, long long ldo, int rows, int H, float inv_scale,
                          float* row_scales, cudaStream_t stream) {
  if (rows == 0) return;
  if (H % 8 != 0 || ldx % 8 != 0 || ldo % 8 != 0)
    throw std::invalid_argument("rmsnorm_quant: H and row pitches must be multiples of 8");
  const int nv = (H / 8 + 255) / 256;
  if (nv == 1)
    launch_pdl(rmsnorm_quant_kernel<1>, dim3(rows), dim3(256), 0, stream, x, ldx, w, eps, out, ldo,
               H, inv_scale, row_scales);
  else if (nv == 2)
    launch_pdl(rmsnorm_quant_kernel<2>, dim3(rows), dim3(256), 0, stream, x, ldx, w, eps, out, ldo,
               H, inv_scale, row_scales);
  else if (nv <= 4)
    launch_pdl(rmsnorm_quant_kernel<4>, dim3(rows), dim3(256), 0, stream, x, ldx, w, eps, out, ldo,
               H, inv_scale, row_scales);
  else
    throw std::invalid_argument("rmsnorm_quant: H above 8192");
}

}  // namespace b200
