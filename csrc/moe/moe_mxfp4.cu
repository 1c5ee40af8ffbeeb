// Grouped expert matmul with MXFP4 weights for decode-sized expert batches (sm_100a).
//
//   Y[rows of entry, n] = X[rows, K] @ dequant(W_e)[n, K]^T
//
// W_e is stored as e2m1 nibbles (two per byte, the lower k in the low nibble) with one e8m0
// scale per 32 k (the OCP MX format of GPT-OSS experts), 4.25 bits per weight instead of 16:
// decode reads every active expert's weights once per step, so the bytes are the cost.
//
// Layout (repacked at load time): inside every 32-byte group (64 k of one column), byte 8t + j
// holds original byte t + 4j -- the order in which lane t of an mma.m16n8k16 A fragment
// consumes k = 16s + 2t (+1) and 16s + 2t + 8 (+9) for slices s = 0..3, so each lane reads a
// column's weights of a 64-k chunk with one 8-byte shared load.  Groups are tiled
// [E][N/256][K/64] with the tile's 256 x 2 scales appended (see the kernel comment).
//
// A CTA owns one entry of the moe_align tile list (<= 16 rows of one expert per pass) and 256
// output columns: one producer warp streams the weight tiles, eight consumer warps compute.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <stdexcept>

#include "../common.cuh"
#include "moe.h"

namespace b200 {

namespace {

__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, "
      "%7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Four bytes of e2m1 pairs -> four f16x2 (the low nibble of each byte in the low half), with
// the sm_100a conversion instruction.
__device__ __forceinline__ void fp4x8_to_f16x8(uint32_t w, uint32_t (&o)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
}

__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t u) {
  const __half2 h = __floats2half2_rn(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Barrier over the consumer warps only (named barrier 1), OR-reducing a predicate.
__device__ __forceinline__ bool consumers_sync_or(bool pred, int nthreads) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(nthreads)
      : "memory");
  return r != 0;
}

constexpr int kRows = 16;    // token rows per pass (two n8 tensor-core tiles)
constexpr int kMT = 2;        // m16 tiles (16 weight columns each) per consumer warp
constexpr int kWarpsC = 8;   // consumer warps (16 warps x 1 tile measured no faster)
constexpr int kCols = 16 * kMT * kWarpsC;
constexpr int kPadK = 8;     // X row padding (halves) against ldmatrix bank conflicts
constexpr int kTileW = kCols * 32;              // fp4 bytes of one (256 columns x 64 k) tile
constexpr int kTileBytes = kTileW + kCols * 2;  // + 2 e8m0 scales per column
constexpr int kMaxStages = 16;

}  // namespace

// Weights arrive as tiles [E][N/256][K/64] of kTileBytes contiguous bytes (the 256 columns'
// 32 fragment-ordered bytes, then their two scales).  Warp 8 streams a CTA's tiles with one bulk
// copy per 64-k chunk into a ring of `stages` shared-memory slots (full barrier: copy landed;
// empty barrier: the 8 consumer warps are done with the slot).  The consumers hold the entry's
// <= 16 token rows in shared memory as f16 and run mma.m16n8k16 with the weights as the A
// operand (16 output columns) and the tokens as B (8 per tile, one tile when the pass has <= 8
// rows), so a decode entry of a few tokens costs one tensor-core op per 16 x 16 weights.  The
// e2m1 pairs are widened to f16x2 by the hardware conversion; each 32-k block's e8m0 scale
// multiplies that block's tensor-core product (tmp accumulator).  Activations are rounded to
// f16 (10-bit mantissa; decode inputs are normed or clamped, far inside the f16 range).
__global__ void __launch_bounds__(32 * (kWarpsC + 1), 1) moe_mxfp4_gemm_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, const uint8_t* __restrict__ wt,
    const int4* __restrict__ gtiles, const int* __restrict__ gcount, int N, int K, int stages,
    __nv_bfloat16* __restrict__ y, long long ldy, uint32_t* status) {
  pdl_trigger();
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem;
  uint8_t* smem_x = smem + stages * kTileBytes;
  const int ldk = K + kPadK;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_x + kRows * ldk * 2);
  uint64_t* empty = full + kMaxStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kWarpsC);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();
  const int entry = blockIdx.x;
  if (entry >= *gcount) return;
  const int4 g = gtiles[entry];
  const int e = g.x, row0 = g.y, row_end = g.z;
  const int NB = (N + kCols - 1) / kCols;
  const int KC = K / 64;
  const int passes = (row_end - row0 + kRows - 1) / kRows;
  const int total = passes * KC;  // chunks streamed by this CTA

  if (warp == kWarpsC) {  // ---------------------------------------------------- producer
    if (lane != 0) return;
    const uint8_t* wbase = wt + ((long long)e * NB + blockIdx.y) * KC * kTileBytes;
    const uint64_t policy = policy_evict_first();
    int issued = 0;
    for (; issued < total; ++issued) {
      const int st = issued % stages;
      if (issued >= stages &&
          !mbar_wait(&empty[st], (uint32_t)(issued / stages - 1) & 1u, kTimeoutSmemEmpty, status))
        break;
      mbar_arrive_expect_tx(&full[st], kTileBytes);
      bulk_load_1d(ring + st * kTileBytes, wbase + (long long)(issued % KC) * kTileBytes, kTileBytes,
                   &full[st], policy);
    }
    // Teardown: every copy issued must have landed before the CTA's shared memory is released.
    for (int i = max(0, issued - stages); i < issued; ++i)
      mbar_wait(&full[i % stages], (uint32_t)(i / stages) & 1u, kTimeoutTmaFull, status);
    return;
  }
  // ------------------------------------------------------------------------------ consumers
  constexpr int kThreadsC = 32 * kWarpsC;
  const int t = lane & 3, grp = lane >> 2;
  const int n_base = blockIdx.y * kCols + warp * 16 * kMT;
  int it = 0;
  bool bad = false;
  for (int pass = 0; pass < passes; ++pass) {
    const int r0 = row0 + pass * kRows;
    const int nr = min(kRows, row_end - r0);
    if (consumers_sync_or(bad, kThreadsC)) break;  // also: the previous pass is done with X
    for (int i = threadIdx.x; i < kRows * (K / 8); i += kThreadsC) {
      const int r = i / (K / 8), c = i % (K / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < nr) {
        const uint4 u = *reinterpret_cast<const uint4*>(x + (long long)(r0 + r) * ldx + c * 8);
        v = make_uint4(bf16x2_to_f16x2(u.x), bf16x2_to_f16x2(u.y), bf16x2_to_f16x2(u.z),
                       bf16x2_to_f16x2(u.w));
      }
      *reinterpret_cast<uint4*>(smem_x + ((long long)r * ldk + c * 8) * 2) = v;
    }
    consumers_sync_or(false, kThreadsC);
    const bool two = nr > 8;
    float acc[kMT][2][4];
#pragma unroll
    for (int m = 0; m < kMT; ++m)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) acc[m][nt][0] = acc[m][nt][1] = acc[m][nt][2] = acc[m][nt][3] = 0.f;
    for (int c = 0; c < KC; ++c, ++it) {
      const int st = it % stages;
      if (!mbar_wait(&full[st], (uint32_t)(it / stages) & 1u, kTimeoutTmaFull, status)) {
        bad = true;
        break;
      }
      // B fragments (tokens): b[slice][n-tile][reg]; matrix j of an x4 load covers k 8j..8j+7
      // of a 32-k half of the chunk.
      uint32_t b[4][2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        if (nt == 1 && !two) break;
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          uint32_t r[4];
          const int row = nt * 8 + (lane & 7);
          const int col = c * 64 + 32 * p + (lane >> 3) * 8;
          ldsm4(smem_u32(smem_x + ((long long)row * ldk + col) * 2), r);
          b[2 * p][nt][0] = r[0];
          b[2 * p][nt][1] = r[1];
          b[2 * p + 1][nt][0] = r[2];
          b[2 * p + 1][nt][1] = r[3];
        }
      }
      const uint8_t* tile = ring + st * kTileBytes;
#pragma unroll
      for (int m = 0; m < kMT; ++m) {
        const int ra = warp * 16 * kMT + m * 16 + grp;  // weight column (A row) within the CTA's 256
        const uint2 wl = *reinterpret_cast<const uint2*>(tile + ra * 32 + t * 8);
        const uint2 wh = *reinterpret_cast<const uint2*>(tile + (ra + 8) * 32 + t * 8);
        const uint32_t sl = *reinterpret_cast<const uint16_t*>(tile + kTileW + ra * 2);
        const uint32_t sh = *reinterpret_cast<const uint16_t*>(tile + kTileW + (ra + 8) * 2);
        uint32_t fl[2][4], fh[2][4];
        fp4x8_to_f16x8(wl.x, fl[0]);
        fp4x8_to_f16x8(wl.y, fl[1]);
        fp4x8_to_f16x8(wh.x, fh[0]);
        fp4x8_to_f16x8(wh.y, fh[1]);
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {  // 32-k block (one scale each)
          float tmp[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const uint32_t a[4] = {fl[hb][2 * q], fh[hb][2 * q], fl[hb][2 * q + 1], fh[hb][2 * q + 1]};
            mma_f16(tmp[0], a, b[2 * hb + q][0][0], b[2 * hb + q][0][1]);
            if (two) mma_f16(tmp[1], a, b[2 * hb + q][1][0], b[2 * hb + q][1][1]);
          }
          const float s0 = __uint_as_float(((sl >> (8 * hb)) & 0xFFu) << 23);
          const float s1 = __uint_as_float(((sh >> (8 * hb)) & 0xFFu) << 23);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            acc[m][nt][0] += s0 * tmp[nt][0];
            acc[m][nt][1] += s0 * tmp[nt][1];
            acc[m][nt][2] += s1 * tmp[nt][2];
            acc[m][nt][3] += s1 * tmp[nt][3];
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (bad) continue;
    // D fragment: (weight column grp [+8], token 2t [+1]) of each (m, n-tile).
#pragma unroll
    for (int m = 0; m < kMT; ++m)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int col = n_base + m * 16 + grp + 8 * h;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int tok = nt * 8 + 2 * t + u;
            if (col < N && tok < nr)
              y[(long long)(r0 + tok) * ldy + col] = __float2bfloat16(acc[m][nt][2 * h + u]);
          }
        }
  }
}

int moe_mxfp4_tile_bytes() { return kTileBytes; }
int moe_mxfp4_tile_cols() { return kCols; }

void moe_mxfp4_gemm_launch(const __nv_bfloat16* x, long long ldx, const uint8_t* wt,
                           const int* gtiles, const int* gcount, int gmax, int N, int K,
                           __nv_bfloat16* y, long long ldy, uint32_t* status, cudaStream_t s) {
  if (K % 64 != 0) throw std::invalid_argument("moe_mxfp4_gemm: K must be a multiple of 64");
  if (ldx % 8 != 0) throw std::invalid_argument("moe_mxfp4_gemm: strides");
  const int xbytes = kRows * (K + kPadK) * 2;
  const int bars = 2 * kMaxStages * 8;
  const int stages = std::min(kMaxStages, (227 * 1024 - xbytes - bars) / kTileBytes);
  if (stages < 2) throw std::invalid_argument("moe_mxfp4_gemm: K too large for the X tile");
  const int smem = stages * kTileBytes + xbytes + bars;
  static std::atomic<uint64_t> configured{0};
  // the shared-memory size depends on K: opt in once to the largest size any call may use
  set_max_dynamic_smem_once(moe_mxfp4_gemm_kernel, 227 * 1024, configured);
  launch_pdl(moe_mxfp4_gemm_kernel, dim3(gmax, (N + kCols - 1) / kCols), dim3(32 * (kWarpsC + 1)), smem,
             s, x, ldx, wt, reinterpret_cast<const int4*>(gtiles), gcount, N, K, stages, y, ldy, status);
}

}  // namespace b200
