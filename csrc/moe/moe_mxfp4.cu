// Grouped expert matmul with MXFP4 weights for decode-sized expert batches (sm_100a).
//
//   Y[rows of entry, n] = X[rows, K] @ dequant(W_e)[n, K]^T
//
// W_e is stored as e2m1 nibbles (two per byte, the lower k in the low nibble) with one e8m0
// scale per 32 k (the OCP MX format of GPT-OSS experts), 4.25 bits per weight instead of 16:
// decode reads every active expert's weights once per step, so the bytes are the cost.
//
// Layout (repacked at load time): blocks [E, N, K/2] where, inside every 32-byte group (64 k),
// byte 8t + j holds original byte t + 4j.  That is the order in which lane t of an
// mma.m16n8k16 B fragment consumes k = 16s + 2t (+1) and 16s + 2t + 8 (+9) for slices s = 0..3,
// so each lane fetches its weights of a 64-k chunk with one 8-byte load.  Scales: [E, N, K/32].
//
// A CTA (8 warps) owns one entry of the moe_align tile list (<= 16 rows of one expert per
// pass) and 256 output columns; the entry's X rows sit in shared memory for the whole K loop,
// each warp streams the fp4 weights of its 32 columns (next chunk's loads in flight while the
// current chunk is converted) and accumulates with mma.sync m16n8k16 (the rows are tokens; a
// tensor-core tile of tokens x 8 columns).
#include <cuda_bf16.h>

#include <stdexcept>

#include "../common.cuh"
#include "moe.h"

namespace b200 {

namespace {

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, "
      "%7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// e2m1 nibble -> bf16 bits (exact): e = 0 -> {0, 0.5}; e > 0 -> (1 + m/2) 2^(e-1).
__device__ __forceinline__ uint32_t fp4_to_bf16_bits(uint32_t x) {
  const uint32_t sign = (x & 8u) << 12;
  const uint32_t e = (x >> 1) & 3u, m = x & 1u;
  const uint32_t mag = e ? (((e + 126u) << 7) | (m << 6)) : (m ? 0x3F00u : 0u);
  return sign | mag;
}

constexpr int kRows = 16;    // token rows per pass
constexpr int kWarpsMx = 8;  // warps per CTA (32 output columns each)
constexpr int kCols = 32 * kWarpsMx;
constexpr int kPadK = 8;     // X row padding (halves) against ldmatrix bank conflicts

}  // namespace

// Dequantisation: a 256-entry shared-memory table maps one byte (two e2m1 nibbles) to the
// bf16x2 pair of their unscaled values (one shared load per two weights); the e8m0 block
// scale is applied after the tensor-core product of each 32-k block (tmp accumulator, then
// acc += 2^(s-127) * tmp), so no per-weight multiply is needed.
__global__ void __launch_bounds__(32 * kWarpsMx) moe_mxfp4_gemm_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, const uint8_t* __restrict__ wq,
    const uint8_t* __restrict__ ws, const int4* __restrict__ gtiles, const int* __restrict__ gcount,
    int N, int K, __nv_bfloat16* __restrict__ y, long long ldy) {
  pdl_trigger();
  __shared__ uint32_t lut[256];
  extern __shared__ __align__(16) uint8_t smem_x[];
  for (int i = threadIdx.x; i < 256; i += blockDim.x)
    lut[i] = fp4_to_bf16_bits(i & 15u) | (fp4_to_bf16_bits(i >> 4) << 16);
  pdl_wait();
  const int entry = blockIdx.x;
  if (entry >= *gcount) return;
  const int4 g = gtiles[entry];
  const int e = g.x, row0 = g.y, row_end = g.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_base = blockIdx.y * kCols + warp * 32;
  const int ldk = K + kPadK;
  const int KB = K / 2;        // bytes per weight row
  const int KS = K / 32;       // scales per weight row
  const uint8_t* wq_e = wq + (long long)e * N * KB;
  const uint8_t* ws_e = ws + (long long)e * N * KS;
  const int t = lane & 3, grp = lane >> 2;

  for (int r0 = row0; r0 < row_end; r0 += kRows) {
    const int nr = min(kRows, row_end - r0);
    __syncthreads();  // LUT ready / previous pass done with the X tile
    for (int i = threadIdx.x; i < kRows * (K / 8); i += blockDim.x) {
      const int r = i / (K / 8), c = i % (K / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < nr) v = *reinterpret_cast<const uint4*>(x + (long long)(r0 + r) * ldx + c * 8);
      *reinterpret_cast<uint4*>(smem_x + ((long long)r * ldk + c * 8) * 2) = v;
    }
    __syncthreads();

    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    int ncol[4];
    bool nok[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ncol[j] = n_base + 8 * j + grp;
      nok[j] = ncol[j] < N;
    }
    // the scales of the D fragment's columns (2t, 2t + 1 of each n-tile) come from lanes
    // grp' = 2t and 2t + 1 of the same n-tile (they load the scale of column grp')
    const int nchunks = K / 64;
    uint2 wb[4];
    uint32_t sb[4];
    auto load_w = [&](int c) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (nok[j]) {
          wb[j] = *reinterpret_cast<const uint2*>(wq_e + (long long)ncol[j] * KB + c * 32 + t * 8);
          sb[j] = *reinterpret_cast<const uint16_t*>(ws_e + (long long)ncol[j] * KS + c * 2);
        } else {
          wb[j] = make_uint2(0, 0);
          sb[j] = 0;
        }
      }
    };
    load_w(0);
    for (int c = 0; c < nchunks; ++c) {
      uint2 cw[4];
      uint32_t cs[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        cw[j] = wb[j];
        cs[j] = sb[j];
      }
      if (c + 1 < nchunks) load_w(c + 1);
      uint32_t a[4][4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int r = lane & 15;
        const int col = c * 64 + s * 16 + (lane >> 4) * 8;
        ldsm4(smem_u32(smem_x + ((long long)r * ldk + col) * 2), a[s]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // scales of output columns 2t and 2t + 1: held by lanes (2t) * 4 + t' and (2t + 1) * 4
        const uint32_t sc_lo = __shfl_sync(0xffffffffu, cs[j], (2 * t) * 4);
        const uint32_t sc_hi = __shfl_sync(0xffffffffu, cs[j], (2 * t + 1) * 4);
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {  // 32-k block of the chunk
          float tmp[4] = {0.f, 0.f, 0.f, 0.f};
          const uint32_t w = hb ? cw[j].y : cw[j].x;
#pragma unroll
          for (int q = 0; q < 2; ++q) {  // slice s = 2 hb + q: bytes 2q, 2q + 1 of w
            const uint32_t b0 = lut[(w >> (16 * q)) & 0xFFu];
            const uint32_t b1 = lut[(w >> (16 * q + 8)) & 0xFFu];
            mma_bf16(tmp, a[2 * hb + q], b0, b1);
          }
          const float s0 = __uint_as_float(((sc_lo >> (8 * hb)) & 0xFFu) << 23);
          const float s1 = __uint_as_float(((sc_hi >> (8 * hb)) & 0xFFu) << 23);
          acc[j][0] += s0 * tmp[0];
          acc[j][1] += s1 * tmp[1];
          acc[j][2] += s0 * tmp[2];
          acc[j][3] += s1 * tmp[3];
        }
      }
    }
    // D fragment: rows grp and grp + 8, columns 2t, 2t + 1 of each n-tile
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n0 = n_base + 8 * j + 2 * t;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = grp + 8 * h;
        if (r < nr && n0 < N) {
          __nv_bfloat16* dst = y + (long long)(r0 + r) * ldy + n0;
          if (n0 + 1 < N)
            *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(acc[j][2 * h], acc[j][2 * h + 1]);
          else
            dst[0] = __float2bfloat16(acc[j][2 * h]);
        }
      }
    }
  }
}

void moe_mxfp4_gemm_launch(const __nv_bfloat16* x, long long ldx, const uint8_t* wq,
                           const uint8_t* ws, const int* gtiles, const int* gcount, int gmax, int N,
                           int K, __nv_bfloat16* y, long long ldy, cudaStream_t s) {
  if (K % 64 != 0) throw std::invalid_argument("moe_mxfp4_gemm: K must be a multiple of 64");
  if (ldx % 8 != 0 || ldy % 2 != 0) throw std::invalid_argument("moe_mxfp4_gemm: strides");
  const int smem = kRows * (K + kPadK) * 2;
  if (smem > 227 * 1024) throw std::invalid_argument("moe_mxfp4_gemm: K too large for the X tile");
  static std::atomic<uint64_t> configured{0};
  set_max_dynamic_smem_once(moe_mxfp4_gemm_kernel, smem, configured);
  launch_pdl(moe_mxfp4_gemm_kernel, dim3(gmax, (N + kCols - 1) / kCols), dim3(32 * kWarpsMx), smem, s, x, ldx,
             wq, ws, reinterpret_cast<const int4*>(gtiles), gcount, N, K, y, ldy);
}

}  // namespace b200
