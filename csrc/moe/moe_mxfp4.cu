// Grouped expert matmul with MXFP4 weights for decode-sized expert batches (sm_100a).
//
//   Y[rows of entry, n] = X[rows, K] @ dequant(W_e)[n, K]^T
//
// W_e is stored as e2m1 nibbles (two per byte, the lower k in the low nibble) with one e8m0
// scale per 32 k (the OCP MX format of GPT-OSS experts), 4.25 bits per weight instead of 16:
// decode reads every active expert's weights once per step, so the bytes are the cost.
//
// Layout (repacked at load time): inside every 32-byte group (64 k of one column), byte 8t + j
// holds original byte t + 4j -- the order in which lane t of an mma.m16n8k16 B fragment
// consumes k = 16s + 2t (+1) and 16s + 2t + 8 (+9) for slices s = 0..3, so each lane reads its
// weights of a 64-k chunk with one 8-byte shared load.  Groups are tiled [E][N/256][K/64] with
// the tile's 256 x 2 scales appended (see the kernel comment).
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
constexpr int kWarpsMx = 8;  // compute warps per CTA (32 output columns each)
constexpr int kCols = 32 * kWarpsMx;
constexpr int kPadK = 8;     // X row padding (halves) against ldmatrix bank conflicts
constexpr int kTileW = kCols * 32;          // fp4 bytes of one (256 columns x 64 k) tile
constexpr int kTileBytes = kTileW + kCols * 2;  // + 2 e8m0 scales per column
constexpr int kStages = 8;

}  // namespace

// Weights arrive as tiles [E][N/256][K/64] of kTileBytes contiguous bytes (the 256 columns'
// 32 fragment-ordered bytes, then their two scales), so one thread streams a CTA's weights with
// one bulk copy per 64-k chunk into an 8-stage shared-memory ring (mbarrier completion); the
// 8 warps consume the ring.  Dequantisation: a 256-entry shared table maps one byte (two e2m1
// nibbles) to their unscaled bf16x2; the e8m0 scale multiplies the tensor-core product of each
// 32-k block (tmp accumulator), so no per-weight multiply is needed.
__global__ void __launch_bounds__(32 * kWarpsMx, 1) moe_mxfp4_gemm_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, const uint8_t* __restrict__ wt,
    const int4* __restrict__ gtiles, const int* __restrict__ gcount, int N, int K,
    __nv_bfloat16* __restrict__ y, long long ldy, uint32_t* status) {
  pdl_trigger();
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem;
  uint8_t* smem_x = smem + kStages * kTileBytes;
  const int ldk = K + kPadK;
  uint32_t* lut = reinterpret_cast<uint32_t*>(smem_x + kRows * ldk * 2);
  uint64_t* bar = reinterpret_cast<uint64_t*>(lut + 256);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) mbar_init(&bar[i], 1);
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < 256; i += blockDim.x)
    lut[i] = fp4_to_bf16_bits(i & 15u) | (fp4_to_bf16_bits(i >> 4) << 16);
  __syncthreads();
  pdl_wait();
  const int entry = blockIdx.x;
  if (entry >= *gcount) return;
  const int4 g = gtiles[entry];
  const int e = g.x, row0 = g.y, row_end = g.z;
  const int NB = (N + kCols - 1) / kCols;
  const int KC = K / 64;
  const uint8_t* wbase = wt + ((long long)e * NB + blockIdx.y) * KC * kTileBytes;
  const int n_base = blockIdx.y * kCols + warp * 32;
  const int t = lane & 3, grp = lane >> 2;
  const uint64_t policy = policy_evict_first();

  const int passes = (row_end - row0 + kRows - 1) / kRows;
  const int total = passes * KC;  // chunks streamed by this CTA
  auto issue = [&](int i) {
    const int st = i % kStages;
    mbar_arrive_expect_tx(&bar[st], kTileBytes);
    bulk_load_1d(ring + st * kTileBytes, wbase + (long long)(i % KC) * kTileBytes, kTileBytes,
                 &bar[st], policy);
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < kStages && i < total; ++i) issue(i);

  int it = 0;
  bool aborted = false;
  for (int pass = 0; pass < passes && !aborted; ++pass) {
    const int r0 = row0 + pass * kRows;
    const int nr = min(kRows, row_end - r0);
    __syncthreads();  // previous pass done with the X tile
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
    for (int c = 0; c < KC; ++c, ++it) {
      const int st = it % kStages;
      const bool ok = mbar_wait(&bar[st], (uint32_t)(it / kStages) & 1u, kTimeoutTmaFull, status);
      if (__syncthreads_or(!ok)) {
        aborted = true;
        break;
      }
      const uint8_t* tile = ring + st * kTileBytes;
      uint32_t a[4][4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int r = lane & 15;
        const int col = c * 64 + s * 16 + (lane >> 4) * 8;
        ldsm4(smem_u32(smem_x + ((long long)r * ldk + col) * 2), a[s]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int row = warp * 32 + 8 * j + grp;  // column within the CTA's 256
        const uint2 w2 = *reinterpret_cast<const uint2*>(tile + row * 32 + t * 8);
        // scales of the D fragment's columns 2t and 2t + 1 of this n-tile
        const uint32_t sc_lo = *reinterpret_cast<const uint16_t*>(tile + kTileW + (warp * 32 + 8 * j + 2 * t) * 2);
        const uint32_t sc_hi = *reinterpret_cast<const uint16_t*>(tile + kTileW + (warp * 32 + 8 * j + 2 * t + 1) * 2);
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          float tmp[4] = {0.f, 0.f, 0.f, 0.f};
          const uint32_t w = hb ? w2.y : w2.x;
#pragma unroll
          for (int q = 0; q < 2; ++q) {
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
      __syncthreads();  // every warp is done with this stage
      if (threadIdx.x == 0 && it + kStages < total) issue(it + kStages);
    }
    if (aborted) break;
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
  if (aborted && threadIdx.x == 0) {
    for (int i = it; i < total && i < it + kStages; ++i)
      mbar_wait(&bar[i % kStages], (uint32_t)(i / kStages) & 1u, kTimeoutTmaFull, status);
  }
}

int moe_mxfp4_tile_bytes() { return kTileBytes; }
int moe_mxfp4_tile_cols() { return kCols; }

void moe_mxfp4_gemm_launch(const __nv_bfloat16* x, long long ldx, const uint8_t* wt,
                           const int* gtiles, const int* gcount, int gmax, int N, int K,
                           __nv_bfloat16* y, long long ldy, uint32_t* status, cudaStream_t s) {
  if (K % 64 != 0) throw std::invalid_argument("moe_mxfp4_gemm: K must be a multiple of 64");
  if (ldx % 8 != 0 || ldy % 2 != 0) throw std::invalid_argument("moe_mxfp4_gemm: strides");
  const int smem = kStages * kTileBytes + kRows * (K + kPadK) * 2 + 256 * 4 + kStages * 8;
  if (smem > 227 * 1024) throw std::invalid_argument("moe_mxfp4_gemm: K too large for the X tile");
  static std::atomic<uint64_t> configured{0};
  set_max_dynamic_smem_once(moe_mxfp4_gemm_kernel, smem, configured);
  launch_pdl(moe_mxfp4_gemm_kernel, dim3(gmax, (N + kCols - 1) / kCols), dim3(32 * kWarpsMx), smem, s,
             x, ldx, wt, reinterpret_cast<const int4*>(gtiles), gcount, N, K, y, ldy, status);
}

}  // namespace b200
