// Persistent, warp-specialized bf16 GEMM for sm_100a on the 5th-generation tensor cores.
//
//   D[M, N] = A[M, K] * B[N, K]^T     (A and B K-contiguous, fp32 accumulation in TMEM)
//
// Roles (192 threads, one CTA per SM):
//   warp 0      TMA producer: one elected thread streams 128x64 A tiles and BNx64 B tiles
//               (128-byte swizzle) into a STAGES-deep shared-memory ring.
//   warp 1      allocates TMEM (2 accumulator buffers of BN fp32 columns) and one elected
//               thread issues tcgen05.mma (M=128, N=BN, K=16) and tcgen05.commit.
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (one TMEM lane = one output row per
//               thread), conversion and global stores, overlapped with the next tile's MMA.
//
// Epilogues:
//   EPI_BF16      out[m, n]  (row-major, bf16)
//   EPI_BF16_T    out[n, m]  (transposed store, used with swapped operands for skinny
//                 decode batches: A = weight rows, B = tokens)
//   EPI_F32_RED   out[m, n] += D (fp32 reductions; used for split-K)
//   EPI_F32_RED_T out[n, m] += D
//   EPI_SILU_BF16 out[m, j] = silu(D[m, g]) * D[m, u] where the weight rows of each BN tile
//                 are [BN/2 gate rows | BN/2 up rows] (interleaved at load time)
//   EPI_BF16_RS   reduce-scatter epilogue of sequence parallelism: row m is stored (bf16) into
//                 the receive slot of the rank that owns it, in that rank's memory over
//                 NVLink, and each finished tile raises the owners' counters
//
// Sequence-parallel all-gather: with GemmSPArgs::ag_ctr set, the A rows of rank r are pushed
// into this rank's A buffer by rank r; the producer waits (bounded) on rank r's counter before
// its first load of those rows, so the local rows are multiplied while the peers' arrive.
//
// Grouped mode with swapped operands (decode-size MoE experts, GemmArgs::grouped_t): A stacks
// the experts' weights [E * M, K] and B is the expert-sorted token rows; the tile of (entry,
// mb) multiplies weight rows [expert * M + 128 mb, ...) by the entry's token rows (at most BN)
// and stores out[token, 128 mb + r] (EPI_BF16_T).  Few tokens per expert then cost an N = BN
// MMA instead of a 128-row token tile, so a 4-bit weight stream stays memory-bound.
//
// Grouped mode (MoE experts): the A operand is the expert-sorted token rows and B stacks the
// experts' weights [E * N, K].  A device tile list, written by the routing kernels, gives
// per 128-row block (expert, first row, end row); the tile of (entry, nb) multiplies rows
// [first, first + 128) of A by rows [expert * N + nb * BN, ...) of B and stores rows below the
// entry's end row only.  Rows past the end of the block belong to the next expert (or are
// TMA zero fill) and are discarded.
//
// Block-scaled FP8 W8A8 with per-k-block promotion (W8 = 5, FP8 operands, swapped decode
// layout EPI_F32_RED_T): e4m3 weights with one fp32 scale per 128 x 128 block and e4m3
// activations with one fp32 scale per token and 128-wide k block.  Each stage is one 128-wide k
// block; its MMAs go into a fresh TMEM accumulator (two alternate), and the epilogue warps add
// it into fp32 registers scaled by the tile's weight-block scale times each token's activation
// scale, then reduce the tile's sum into the output once.  No weight conversion: the fp8 bytes
// stream from HBM straight into the tensor cores.
//
// FP8 (e4m3 x e4m3, per-tensor scales): tcgen05.mma kind::f8f6f4 on the same byte tiles, 128
// elements per k-block, the accumulator scaled by alpha = scale_a * scale_b in the epilogue
// (static W8A8 checkpoints: the reference's ModelOpt FP8 Llama, model/llama3/quantization.py).
//
// This is the B200 replacement of the dense projections that the reference runs through
// its NKI qkv / mlp / output_projection kernels (vllm_neuron/functional/attention/qkv.py:672,
// vllm_neuron/functional/mlp.py:65, vllm_neuron/functional/attention/o_proj.py:124).
#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>
#include <stdexcept>
#include <string>

#include "../common.cuh"
#include "gemm.h"

namespace b200 {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kATileBytes = kBM * kBK * 2;

struct GemmParams {
  int M, N, K;
  int num_m_blocks, num_n_blocks, num_k_blocks;
  int splits, kb_per_split;
  int streamk;  // 1: each CTA owns an equal contiguous range of (tile, k-block) units
  int group_m;
  void* out;
  long long ldo;
  uint32_t* status;
  // grouped mode: 1 = weights as B (token tiles of 128 rows), 2 = weights as A (swapped)
  int grouped;
  const int4* gtiles;  // [entries] (expert, first row, end row, unused)
  const int* gcount;   // number of valid entries
  GemmSPArgs sp;       // sequence-parallel all-gather wait / reduce-scatter epilogue
  float alpha;         // epilogue scale of FP8 operands (1 for bf16)
  // block-scaled FP8 weight operand (W8 kernels): fp32 scales [wsc_rows][wsc_ld], one per
  // 128 x 128 block of the weight
  const float* wsc;
  int wsc_ld, wsc_rows;
  const uint8_t* wsc8;  // MXFP4: e8m0 scale bytes [wsc_rows][wsc_ld], one per 32 elements
  const float* xsc;     // W8 = 5: activation scales [tokens][xsc_ld], one per 128-wide k block
  int xsc_ld;
  // W8 = 6 (MXFP8): e8m0 scales of A and B in 512-byte atoms, atom (row block, k block) at
  // ((row / 128) * sf_kb + k / 128) * 512; inside an atom, the 4 scales of row r (32 k
  // elements each) are bytes (r % 32) * 16 + ((r / 32) % 4) * 4 + [0, 4)
  const uint8_t* sfa;
  const uint8_t* sfb;
  int sf_kb;
};

// Bounded wait until a monotonic counter (written by a peer with a system-scope release)
// reaches `target`; returns at once once the status word is set (peers out of step).
__device__ __forceinline__ bool gemm_wait_ctr(const unsigned int* c, unsigned int target,
                                              uint32_t* status) {
  auto ld = [](const unsigned int* q) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(q) : "memory");
    return v;
  };
  if ((int)(ld(c) - target) >= 0) return true;
  if (status != nullptr && *reinterpret_cast<volatile uint32_t*>(status) != 0u) return false;
  const uint64_t t0 = globaltimer_ns();
  while ((int)(ld(c) - target) < 0) {
    if (globaltimer_ns() - t0 > B200_PEER_TIMEOUT_NS) {
      set_status(status, kTimeoutPeerFlag);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// Row coordinates of tile `mb` (an m-block index, or a tile-list entry in grouped mode).
struct TileRows {
  int a_row;   // first row of the A tile
  int b_base;  // row offset of the B operand (expert * N in grouped mode)
  int m_lim;   // rows >= m_lim are not stored
};
__device__ __forceinline__ TileRows tile_rows(const GemmParams& p, int mb) {
  TileRows t;
  if (p.grouped) {
    const int4 g = p.gtiles[mb];
    t.a_row = g.y;
    t.b_base = g.x * p.N;
    t.m_lim = g.z;
  } else {
    t.a_row = mb * kBM;
    t.b_base = 0;
    t.m_lim = p.M;
  }
  return t;
}

// Swapped grouped mode: first weight row (A) of tile (entry mb, block nb) and its token rows.
__device__ __forceinline__ int gt_weight_row(const GemmParams& p, int mb, int nb) {
  return p.gtiles[mb].x * p.M + nb * kBM;
}

__device__ __forceinline__ void decode_tile(const GemmParams& p, int tile, int& mb, int& nb,
                                            int& split) {
  const int mn_tiles = p.num_m_blocks * p.num_n_blocks;
  split = tile / mn_tiles;
  const int mn = tile - split * mn_tiles;
  const int group_size = p.group_m * p.num_n_blocks;
  const int g = mn / group_size;
  const int first_m = g * p.group_m;
  const int gm = min(p.num_m_blocks - first_m, p.group_m);
  const int r = mn - g * group_size;
  mb = first_m + r % gm;
  nb = r / gm;
}

// Work segments of one CTA: (tile, k-block range).  All three roles walk the same sequence.
struct SegCursor {
  long long u, u_end;
  int tile;
  __device__ explicit SegCursor(const GemmParams& p) {
    if (p.streamk) {
      const long long U = (long long)p.num_m_blocks * p.num_n_blocks * p.num_k_blocks;
      u = U * blockIdx.x / gridDim.x;
      u_end = U * (blockIdx.x + 1) / gridDim.x;
      tile = 0;
    } else {
      u = u_end = 0;
      tile = blockIdx.x;
    }
  }
  __device__ bool next(const GemmParams& p, int& mb, int& nb, int& k0, int& k1) {
    int split;
    if (p.streamk) {
      if (u >= u_end) return false;
      const int t = (int)(u / p.num_k_blocks);
      k0 = (int)(u - (long long)t * p.num_k_blocks);
      k1 = (int)min((long long)p.num_k_blocks, k0 + (u_end - u));
      u += k1 - k0;
      decode_tile(p, t, mb, nb, split);
      return true;
    }
    if (p.grouped == 2) {  // mb = tile-list entry, nb = 128-row block of the expert's weight
      if (tile >= *p.gcount * p.num_m_blocks) return false;
      mb = tile / p.num_m_blocks;
      nb = tile - mb * p.num_m_blocks;
      k0 = 0;
      k1 = p.num_k_blocks;
      tile += gridDim.x;
      return true;
    }
    if (p.grouped) {
      if (tile >= *p.gcount * p.num_n_blocks) return false;
      mb = tile / p.num_n_blocks;
      nb = tile - mb * p.num_n_blocks;
      k0 = 0;
      k1 = p.num_k_blocks;
      tile += gridDim.x;
      return true;
    }
    if (tile >= p.num_m_blocks * p.num_n_blocks * p.splits) return false;
    decode_tile(p, tile, mb, nb, split);
    k0 = split * p.kb_per_split;
    k1 = min(k0 + p.kb_per_split, p.num_k_blocks);
    tile += gridDim.x;
    return true;
  }
};


__host__ __device__ constexpr uint32_t tmem_cols_pow2(int n) {
  return n <= 32 ? 32u : n <= 64 ? 64u : n <= 128 ? 128u : n <= 256 ? 256u : 512u;
}

template <int BN>
struct TmemCols {
  static constexpr int v = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128
                           : (2 * BN <= 256) ? 256 : 512;
};

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// Four bytes of e2m1 pairs -> four f16x2 (the low nibble of each byte in the low half); every
// e2m1 value is exact in f16.
__device__ __forceinline__ void fp4x8_to_f16x8_gemm(uint32_t w, uint32_t (&o)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
}

// FP8 = true: e4m3 operands (kind::f8f6f4).  A 128-byte swizzle row then holds 128 elements, so
// the shared-memory tiles and the per-instruction descriptor advance (32 bytes) are unchanged;
// only the k-block element count, the MMA kind and the epilogue scale differ.
//
// W8 = 1 / 2: operand A / B is a block-scaled FP8 weight (e4m3 bytes, one fp32 scale per 128 x
// 128 block) multiplied with bf16 activations.  TMA streams the weight tile as bytes (64 per
// row, no swizzle) into a staging buffer; four converter warps (warps 6..9) widen it with the
// tile's block scale, bf16(e4m3 * scale), into the 128-byte-swizzled bf16 operand layout the
// MMA descriptors read, and release the stage to the MMA issuer (conv_bar).  Weight bytes cross
// HBM once at one byte per element; the tensor cores run kind::f16.
// W8 = 3 / 4: the same for an MXFP4 weight on A / B (GPT-OSS experts): 32 packed bytes per row
// per stage (two e2m1 per byte), widened with the hardware e2m1x2 conversion and the e8m0
// scale of each 32-element block -- half a byte per element from HBM.
// W8 = 6 (MXFP8 x MXFP8, FP8 operands): the native block-scaled MMA.  Each stage also carries the
// 512-byte e8m0 scale atoms of its A and B rows (1D bulk copies on the stage's barrier); the MMA
// thread copies them into TMEM (tcgen05.cp 32x128b.warpx4, a fresh 8-column slot per stage)
// and issues kind::mxf8f6f4.block_scale with the scale byte of each 32-element k step, so the
// hardware applies the per-32 scales and the epilogue is the plain fp32 one.
template <int BN, int STAGES, int EPI, bool FP8 = false, int W8 = 0>
__global__ void __launch_bounds__((W8 >= 1 && W8 <= 4) ? 320 : 192, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
  constexpr int kBTileBytes = BN * kBK * 2;
  constexpr bool kConv = W8 >= 1 && W8 <= 4;                 // converter warps widen the weight
  constexpr bool kPromote = W8 == 5;                         // block-scaled FP8, per-k-block sums
  static_assert(!kPromote || (FP8 && ((EPI == EPI_F32_RED_T && BN <= 64) || (EPI == EPI_BF16 && BN == 128))),
                "promotion mode: FP8 operands; swapped decode layout with N tile <= 64, or tokens as A "
                "with a 128-wide weight tile");
  constexpr bool kFP4 = W8 == 3 || W8 == 4;                  // MXFP4 (else block FP8)
  constexpr bool kMX = W8 == 6;                              // MXFP8, hardware block scaling
  static_assert(!kMX || (FP8 && BN <= 128 && EPI != EPI_SILU_BF16 && EPI != EPI_BF16_RS),
                "MXFP8 mode: e4m3 operands, N tile <= 128, plain epilogues");
  constexpr int kSFBytes = kMX ? 1024 : 0;                    // scale atoms of A and B per stage
  constexpr int kWSide = !kConv ? 0 : (W8 == 1 || W8 == 3) ? 1 : 2;  // weight operand: A / B
  constexpr int kW8Rows = kWSide == 1 ? kBM : kWSide == 2 ? BN : 0;  // weight rows per tile
  constexpr int kSRow = kFP4 ? kBK / 2 : kBK;                 // staged bytes per row per stage
  constexpr int kSBytes = kW8Rows * kSRow;                    // staging bytes per stage
  constexpr int kStageBytes = kATileBytes + kBTileBytes + kSBytes + kSFBytes;
  // bytes the TMA delivers per stage (the converted operand is written by the converter)
  constexpr int kStageTx = kWSide == 1   ? kSBytes + kBTileBytes
                           : kWSide == 2 ? kATileBytes + kSBytes
                                         : kATileBytes + kBTileBytes + kSFBytes;
  // accumulator buffers: 2 tiles in flight; the promotion mode keeps 4 k-block accumulators so
  // the MMA issuer runs up to 4 k blocks ahead of the promoting epilogue
  constexpr int kAccBufs = kPromote ? 4 : 2;
  constexpr int kSFCol0 = 2 * BN;  // MXFP8: scale slots (8 columns per stage) after the accumulators
  constexpr uint32_t kTmemCols = kPromote ? TmemCols<2 * BN>::v
                                 : kMX    ? tmem_cols_pow2(kSFCol0 + 8 * STAGES)
                                          : TmemCols<BN>::v;
  static_assert(!kMX || kSFCol0 + 8 * STAGES <= 512, "MXFP8 TMEM budget");
  constexpr uint32_t kIdesc = kMX ? make_idesc_mx8(kBM, BN)
                                  : make_idesc_f16(kBM, BN, !FP8);  // FP8: type fields 0 = E4M3
  constexpr int kKElems = FP8 ? 2 * kBK : kBK;                  // elements per k-block

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * kATileBytes;
  uint8_t* smS = smB + STAGES * kBTileBytes;  // fp8 weight staging (W8)
  uint8_t* smSF = smS + STAGES * kSBytes;     // MXFP8 scale atoms: [A 512 | B 512] per stage
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* conv_bar = empty_bar + STAGES;  // converted operand ready (W8)
  uint64_t* tfull_bar = conv_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + kAccBufs;
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(tempty_bar + kAccBufs);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_smem + 1);
  unsigned int* rs_arrivals = tmem_base_smem + 2;  // epilogue threads done with their RS stores

  const int warp = warp_id();
  const int lane = lane_id();
  // a GEMM whose producer waits for peers' all-gathered rows stalls with them: its pipeline
  // waits get the cross-rank budget
  const uint64_t wait_ns = p.sp.ag_ctr != nullptr ? B200_PEER_TIMEOUT_NS : B200_WAIT_TIMEOUT_NS;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
      mbar_init(&conv_bar[s], 4);
    }
    for (int a = 0; a < kAccBufs; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 4);
    }
    *abort_flag = 0;
    *rs_arrivals = 0u;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_smem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_smem;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (elect_one()) {
      constexpr bool kWeightIsA = (EPI == EPI_BF16_T || EPI == EPI_F32_RED_T);
      const uint64_t hint_a = kWeightIsA ? policy_evict_first()  // A = weights, streamed once
                                         : policy_evict_last();
      const uint64_t hint_b = kWeightIsA ? policy_evict_last()   // B = activations, reused
                                         : policy_evict_first();
      uint32_t ag_ready = 0;  // ranks whose all-gathered A rows are known complete
      auto load_a = [&](int s, int kb, int mb, int nb) {
        const int a_row = p.grouped == 2 ? gt_weight_row(p, mb, nb) : tile_rows(p, mb).a_row;
        if (p.sp.ag_ctr != nullptr) {
          const int r0 = a_row / p.sp.ag_rows;
          const int r1 = min(min(a_row + kBM - 1, p.M - 1) / p.sp.ag_rows, p.sp.ag_world - 1);
          bool waited = false;
          for (int r = r0; r <= r1; ++r) {
            if (ag_ready & (1u << r)) continue;
            gemm_wait_ctr(p.sp.ag_ctr + r, p.sp.ag_target[r], p.status);
            ag_ready |= 1u << r;
            waited = true;
          }
          // peer stores (generic proxy) -> this thread's TMA reads (async proxy)
          if (waited) asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        uint8_t* dst = kWSide == 1 ? smS + s * kSBytes : smA + s * kATileBytes;
        tma_load_2d(&tmA, &full_bar[s], dst, (kFP4 && kWSide == 1) ? kb * kSRow : kb * kKElems, a_row, hint_a);
        if constexpr (kMX) {
          // grouped prefill: A = expert-sorted tokens, one scale atom per tile-list entry
          const long long atom = p.grouped == 1 ? (long long)mb : (long long)(a_row >> 7);
          bulk_load_1d(smSF + s * kSFBytes, p.sfa + (atom * p.sf_kb + kb) * 512, 512, &full_bar[s], hint_a);
        }
      };
      auto load_b = [&](int s, int kb, int nb, int mb) {
        const int row = p.grouped == 2 ? p.gtiles[mb].y : (p.grouped ? tile_rows(p, mb).b_base : 0) + nb * BN;
        uint8_t* dst = kWSide == 2 ? smS + s * kSBytes : smB + s * kBTileBytes;
        tma_load_2d(&tmB, &full_bar[s], dst, (kFP4 && kWSide == 2) ? kb * kSRow : kb * kKElems, row, hint_b);
        if constexpr (kMX) {
          // swapped grouped decode: B = the entry's tokens, one scale atom per entry
          const long long atom = p.grouped == 2 ? (long long)mb : (long long)(row >> 7);
          bulk_load_1d(smSF + s * kSFBytes + 512, p.sfb + (atom * p.sf_kb + kb) * 512, 512, &full_bar[s], hint_b);
        }
      };
      // The grouped tile list is written by the previous kernel.
      if (p.grouped) pdl_wait();
      uint32_t it = 0;
      bool ok = true;
      SegCursor cur(p);
      int mb = 0, nb = 0, k0 = 0, k1 = 0;
      bool have = cur.next(p, mb, nb, k0, k1);
      int kb = k0;
      // Phase 1: the weight operand of the first STAGES k-blocks does not depend on the
      // previous kernel, so it streams in before the dependency wait.
      int pre_mb[STAGES], pre_nb[STAGES], pre_kb[STAGES];
      int npre = 0;
#pragma unroll
      for (int i = 0; i < STAGES; ++i) {
        if (have) {
          mbar_arrive_expect_tx(&full_bar[i], kStageTx);
          if (kWeightIsA) load_a(i, kb, mb, nb); else load_b(i, kb, nb, mb);
          pre_mb[i] = mb;
          pre_nb[i] = nb;
          pre_kb[i] = kb;
          npre = i + 1;
          ++it;
          if (++kb == k1) {
            have = cur.next(p, mb, nb, k0, k1);
            kb = k0;
          }
        }
      }
      pdl_wait();
#pragma unroll
      for (int i = 0; i < STAGES; ++i) {
        if (i < npre) {
          if (kWeightIsA) load_b(i, pre_kb[i], pre_nb[i], pre_mb[i]); else load_a(i, pre_kb[i], pre_mb[i], pre_nb[i]);
        }
      }
      // Phase 2: steady state.
      while (have) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait_abortable(&empty_bar[s], ph ^ 1, kTimeoutSmemEmpty, p.status, abort_flag, wait_ns)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[s], kStageTx);
        load_a(s, kb, mb, nb);
        load_b(s, kb, nb, mb);
        ++it;
        if (++kb == k1) {
          have = cur.next(p, mb, nb, k0, k1);
          kb = k0;
        }
      }
      // The successor may launch once every CTA has issued its last load.
      pdl_trigger();
      if (!ok) {
        // Drain the copies still in flight before the CTA's shared memory is released.
        const uint32_t first = it > (uint32_t)STAGES ? it - STAGES : 0;
        for (uint32_t j = first; j < it; ++j)
          mbar_wait(&full_bar[j % STAGES], (j / STAGES) & 1, kTimeoutTmaFull, p.status);
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (elect_one()) {
      if (p.grouped) pdl_wait();  // the tile list is written by the previous kernel
      uint32_t it = 0;
      int t_local = 0;
      bool ok = true;
      SegCursor cur(p);
      int mb, nb, k0, k1;
      uint32_t u = 0;  // promotion mode: k blocks issued (accumulator = u & 1)
      for (; ok && cur.next(p, mb, nb, k0, k1); ++t_local) {
        const int acc = t_local & 1;
        const uint32_t aph = (t_local >> 1) & 1;
        if (!kPromote &&
            !mbar_wait_abortable(&tempty_bar[acc], aph ^ 1, kTimeoutTmemEmpty, p.status, abort_flag, wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = k0; kb < k1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if constexpr (kPromote) {
            // each k block into its own accumulator, once the epilogue has drained it
            const int pa = u % kAccBufs;
            if (!mbar_wait_abortable(&tempty_bar[pa], ((u / kAccBufs) & 1) ^ 1, kTimeoutTmemEmpty, p.status,
                                     abort_flag, wait_ns)) {
              ok = false;
              break;
            }
            d_tmem = tmem_base + pa * BN;
          }
          if (!mbar_wait_abortable(kConv ? &conv_bar[s] : &full_bar[s], ph, kTimeoutTmaFull, p.status,
                                   abort_flag, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smA + s * kATileBytes);
          const uint32_t b_addr = smem_u32(smB + s * kBTileBytes);
          if constexpr (kMX) {
            // this stage's scale atoms -> its TMEM slot (A: 4 columns, B: 4 columns), then the
            // four 32-element k steps, step k reading byte k of each scale word
            const uint32_t sf_a = tmem_base + kSFCol0 + s * 8;
            const uint32_t sf_b = sf_a + 4;
            const uint32_t sf_src = smem_u32(smSF + s * kSFBytes);
            tmem_cp_32x128b_warpx4(sf_a, make_sdesc_none(sf_src, 128, 128));
            tmem_cp_32x128b_warpx4(sf_b, make_sdesc_none(sf_src + 512, 128, 128));
            // B rows of this tile start (nb * BN) % 128 rows into their atom: 32 rows per column
            // (in the swapped grouped mode nb indexes the weight's 128-row blocks; B starts its atom)
            const uint32_t b_col = p.grouped == 2 ? 0u : (uint32_t)(((nb * BN) & 127) >> 5);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint64_t adesc = make_sdesc_sw128(a_addr + k * 32);
              const uint64_t bdesc = make_sdesc_sw128(b_addr + k * 32);
              const uint32_t accum = (kb > k0 || k > 0) ? 1u : 0u;
              const uint32_t id = (uint32_t)k;
              umma_mx8_ss(d_tmem, adesc, bdesc, kIdesc | (id << 4) | (id << 29), sf_a | (id << 30),
                          (sf_b + b_col) | (id << 30), accum);
            }
            umma_commit(&empty_bar[s]);
            continue;
          }
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t adesc = make_sdesc_sw128(a_addr + k * 32);
            const uint64_t bdesc = make_sdesc_sw128(b_addr + k * 32);
            const uint32_t accum = kPromote ? (k > 0 ? 1u : 0u) : ((kb > k0 || k > 0) ? 1u : 0u);
            if constexpr (FP8)
              umma_f8_ss(d_tmem, adesc, bdesc, kIdesc, accum);
            else
              umma_f16_ss(d_tmem, adesc, bdesc, kIdesc, accum);
          }
          umma_commit(&empty_bar[s]);
          if constexpr (kPromote) {
            umma_commit(&tfull_bar[u % kAccBufs]);
            ++u;
          }
        }
        if (ok && !kPromote) umma_commit(&tfull_bar[acc]);
      }
    }
  } else if (kConv && warp >= 6) {
    // ------------------------------ fp8 -> bf16 weight converter ------------------------------
    // Lane l of converter warp cw reads 16 staged bytes (row r, bytes 16 * (l % 4) ..) and
    // writes them as 16 bf16 = 16-byte chunks 2 (l % 4) and 2 (l % 4) + 1 of the 128-byte
    // operand row r, each at chunk ^ (r % 8) (the 128-byte swizzle on the 1024-byte-aligned
    // tile).  Eight lanes of a phase cover two rows: conflict-free reads and writes.
    if (p.grouped) pdl_wait();  // the tile list is written by the previous kernel
    const int cw = warp - 6;
    uint32_t it = 0;
    bool ok = true;
    SegCursor cur(p);
    int mb, nb, k0, k1;
    while (ok && cur.next(p, mb, nb, k0, k1)) {
      const TileRows tr = tile_rows(p, mb);
      const int wrow0 = kWSide == 1 ? (p.grouped == 2 ? gt_weight_row(p, mb, nb) : tr.a_row)
                                    : tr.b_base + nb * BN;  // first weight row of the tile
      // Scales are read from global memory two k-blocks ahead of their use (two register
      // slots), so their latency overlaps the conversion of the blocks in between.
      constexpr int kScPer = kFP4 ? kW8Rows / 32 : 1;  // scale words per lane per k-block
      auto load_scales = [&](int kbx, uint32_t (&d)[kScPer]) {
        if constexpr (kFP4) {
#pragma unroll
          for (int i = 0; i < kScPer; ++i) {
            const int r = cw * (kW8Rows / 4) + i * 8 + (lane >> 2);
            const int wr = min(wrow0 + r, p.wsc_rows - 1);
            d[i] = kbx < k1 ? __ldg(p.wsc8 + (long long)wr * p.wsc_ld + kbx * 2 + ((lane & 3) >> 1)) : 0u;
          }
        } else {
          // one 128 x 128 block scale per lane (rows of a tile share the 128-row block)
          const int r = cw * (kW8Rows / 4) + (lane >> 2);
          const int srow = min((wrow0 + r) >> 7, p.wsc_rows - 1);
          d[0] = kbx < k1 ? __float_as_uint(__ldg(p.wsc + (kbx >> 1) + (long long)srow * p.wsc_ld)) : 0u;
        }
      };
      uint32_t sc_a[kScPer], sc_b[kScPer];
      load_scales(k0, sc_a);
      load_scales(k0 + 1, sc_b);
      for (int kb = k0; kb < k1; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        const bool odd = ((kb - k0) & 1) != 0;
        uint32_t sc_cur[kScPer];
#pragma unroll
        for (int i = 0; i < kScPer; ++i) sc_cur[i] = odd ? sc_b[i] : sc_a[i];
        if (odd)
          load_scales(kb + 2, sc_b);
        else
          load_scales(kb + 2, sc_a);
        if (!mbar_wait_abortable(&full_bar[s], ph, kTimeoutTmaFull, p.status, abort_flag, wait_ns)) {
          ok = false;
          break;
        }
        const uint8_t* src = smS + s * kSBytes;
        uint8_t* dst = kWSide == 1 ? smA + s * kATileBytes : smB + s * kBTileBytes;
        if constexpr (kFP4) {
          // lane: row r, 8 packed bytes = elements [16 c, 16 c + 16) of this 64-k block, whose
          // e8m0 scale is block kb * 2 + c / 2 of the row
#pragma unroll
          for (int i = 0; i < kW8Rows / 32; ++i) {
            const int r = cw * (kW8Rows / 4) + i * 8 + (lane >> 2);
            const int c = lane & 3;
            const uint2 v = *reinterpret_cast<const uint2*>(src + r * kSRow + c * 8);
            const uint32_t e = sc_cur[i];
            const float sc = __uint_as_float(e ? (e << 23) : 0x00400000u);  // 2^(e - 127)
            uint32_t h[8];
            {
              uint32_t t0[4], t1[4];
              fp4x8_to_f16x8_gemm(v.x, t0);
              fp4x8_to_f16x8_gemm(v.y, t1);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                h[j] = t0[j];
                h[4 + j] = t1[j];
              }
            }
            uint32_t o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[j]));
              o[j] = pack_bf16x2(f.x * sc, f.y * sc);
            }
            uint8_t* drow = dst + r * 128;
            const int sw = r & 7;
            *reinterpret_cast<uint4*>(drow + (((2 * c) ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(drow + (((2 * c + 1) ^ sw) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
          }
        } else {
        const float sc = __uint_as_float(sc_cur[0]);  // the tile's 128 x 128 block scale
#pragma unroll
        for (int i = 0; i < kW8Rows / 32; ++i) {
          const int r = cw * (kW8Rows / 4) + i * 8 + (lane >> 2);
          const int c16 = lane & 3;
          const uint4 v = *reinterpret_cast<const uint4*>(src + r * kBK + c16 * 16);
          const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
          uint32_t o[8];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t lo = e4m3x2_to_f16x2(w4[j]), hi = e4m3x2_to_f16x2(w4[j] >> 16);
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
            o[2 * j] = pack_bf16x2(a.x * sc, a.y * sc);
            o[2 * j + 1] = pack_bf16x2(b.x * sc, b.y * sc);
          }
          uint8_t* drow = dst + r * 128;
          const int sw = r & 7;
          *reinterpret_cast<uint4*>(drow + (((2 * c16) ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(drow + (((2 * c16 + 1) ^ sw) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
        }
        }
        // generic-proxy shared-memory writes -> the tensor cores' (async proxy) operand reads
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv_bar[s]);
      }
    }
  } else {
    // ------------------------------ epilogue ------------------------------
    pdl_wait();  // outputs may still be read (or, for reductions, cleared) by the predecessor
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    int t_local = 0;
    SegCursor cur(p);
    int mb, nb, k0, k1;
    if constexpr (kPromote) {
      // per k block: read its accumulator, scale by the weight block's scale times each token's
      // activation scale, add into registers; reduce the tile's sum into out[n, m] once
      uint32_t u = 0;
      bool ok = true;
      while (ok && cur.next(p, mb, nb, k0, k1)) {
        const TileRows trows = tile_rows(p, mb);
        const int m = trows.a_row + row;  // swapped: weight row = output column; else token row
        const int n_base = nb * BN;       // swapped: first token; else first weight row (column)
        constexpr bool kSwapped = EPI == EPI_F32_RED_T;
        const float* wsc_row =
            p.wsc + (long long)min((kSwapped ? trows.a_row : n_base) >> 7, p.wsc_rows - 1) * p.wsc_ld;
        float racc[BN];
#pragma unroll
        for (int j = 0; j < BN; ++j) racc[j] = 0.f;
        for (int kb = k0; kb < k1; ++kb, ++u) {
          const int pa = u % kAccBufs;
          if (!mbar_wait_abortable(&tfull_bar[pa], (u / kAccBufs) & 1, kTimeoutTmemFull, p.status, abort_flag, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float sw = __ldg(wsc_row + kb);
          const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + pa * BN;
          if constexpr (kSwapped) {
#pragma unroll
            for (int c = 0; c < BN; c += 16) {
              uint32_t r[16];
              tmem_ld_32x32b_x16(t_row + c, r);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int n = n_base + c + j;  // the token's scale per column
                const float sx = n < p.N ? __ldg(p.xsc + (long long)n * p.xsc_ld + kb) : 0.f;
                racc[c + j] = fmaf(__uint_as_float(r[j]), sw * sx, racc[c + j]);
              }
            }
          } else {
            // one factor per row: this token's activation scale times the weight block's
            const float f = sw * (m < p.M ? __ldg(p.xsc + (long long)m * p.xsc_ld + kb) : 0.f);
#pragma unroll
            for (int c = 0; c < BN; c += 32) {
              uint32_t r[32];
              tmem_ld_32x32b_x32(t_row + c, r);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; ++j) racc[c + j] = fmaf(__uint_as_float(r[j]), f, racc[c + j]);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty_bar[pa]);
        }
        if (!ok) break;
        if constexpr (kSwapped) {
          if (m < trows.m_lim) {
            float* o = reinterpret_cast<float*>(p.out) + m;
#pragma unroll
            for (int j = 0; j < BN; ++j)
              if (n_base + j < p.N) atomicAdd(o + (long long)(n_base + j) * p.ldo, racc[j]);
          }
        } else if (m < trows.m_lim) {
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + (long long)m * p.ldo + n_base;
          if (n_base + BN <= p.N && (p.ldo % 8) == 0) {
#pragma unroll
            for (int c = 0; c < BN; c += 8)
              *reinterpret_cast<uint4*>(o + c) =
                  make_uint4(pack_bf16x2(racc[c], racc[c + 1]), pack_bf16x2(racc[c + 2], racc[c + 3]),
                             pack_bf16x2(racc[c + 4], racc[c + 5]), pack_bf16x2(racc[c + 6], racc[c + 7]));
          } else {
#pragma unroll
            for (int j = 0; j < BN; ++j)
              if (n_base + j < p.N) o[j] = __float2bfloat16(racc[j]);
          }
        }
      }
    } else
    for (; cur.next(p, mb, nb, k0, k1); ++t_local) {
      const int acc = t_local & 1;
      const uint32_t aph = (t_local >> 1) & 1;
      if (!mbar_wait_abortable(&tfull_bar[acc], aph, kTimeoutTmemFull, p.status, abort_flag, wait_ns)) break;
      tc_fence_after();
      const TileRows trows = tile_rows(p, mb);
      const int m = trows.a_row + row;
      const int m_lim = trows.m_lim;
      const int n_base = nb * BN;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;

      if constexpr (EPI == EPI_SILU_BF16) {
        // Tile columns [0, BN/2) are gate rows, [BN/2, BN) the matching up rows.
        constexpr int H = BN / 2;
        const int j_base = nb * H;  // output column base
        const int n_out = p.N / 2;
#pragma unroll 1
        for (int c = 0; c < H; c += 16) {
          uint32_t g[16], u[16];
          tmem_ld_32x32b_x16(t_row + c, g);
          tmem_ld_32x32b_x16(t_row + H + c, u);
          tmem_ld_wait();
          if constexpr (FP8) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              g[j] = __float_as_uint(__uint_as_float(g[j]) * p.alpha);
              u[j] = __float_as_uint(__uint_as_float(u[j]) * p.alpha);
            }
          }
          if (m < m_lim) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + (long long)m * p.ldo;
            uint32_t packed[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float g0 = __uint_as_float(g[2 * j]), g1 = __uint_as_float(g[2 * j + 1]);
              const float u0 = __uint_as_float(u[2 * j]), u1 = __uint_as_float(u[2 * j + 1]);
              packed[j] = pack_bf16x2(silu_f(g0) * u0, silu_f(g1) * u1);
            }
            const int j0 = j_base + c;
            if (j0 + 16 <= n_out && (p.ldo % 8) == 0) {
              uint4* dst = reinterpret_cast<uint4*>(o + j0);
              dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
              dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
            } else {
              for (int j = 0; j < 16; ++j) {
                if (j0 + j < n_out) {
                  const float2 f = unpack_bf16x2(packed[j >> 1]);
                  o[j0 + j] = __float2bfloat16((j & 1) ? f.y : f.x);
                }
              }
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c, r);
          tmem_ld_wait();
          if constexpr (FP8) {
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * p.alpha);
          }
          const int n0 = n_base + c;
          if constexpr (EPI == EPI_BF16 || EPI == EPI_BF16_RS) {
            if (m < m_lim) {
              __nv_bfloat16* o;
              if constexpr (EPI == EPI_BF16_RS) {
                const int owner = m / p.sp.rs_rows;
                o = p.sp.rs_out[owner] + (long long)(m - owner * p.sp.rs_rows) * p.ldo + n0;
              } else {
                o = reinterpret_cast<__nv_bfloat16*>(p.out) + (long long)m * p.ldo + n0;
              }
              if (n0 + 32 <= p.N && (p.ldo % 8) == 0) {
                uint4* dst = reinterpret_cast<uint4*>(o);
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                  dst[v] = make_uint4(
                      pack_bf16x2(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1])),
                      pack_bf16x2(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3])),
                      pack_bf16x2(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5])),
                      pack_bf16x2(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7])));
                }
              } else {
                for (int j = 0; j < 32; ++j)
                  if (n0 + j < p.N) o[j] = __float2bfloat16(__uint_as_float(r[j]));
              }
            }
          } else if constexpr (EPI == EPI_BF16_T) {
            if (p.grouped == 2) {
              // weight row 128 nb + row of the entry's expert -> column; token rows of the entry
              const int4 g = p.gtiles[mb];
              const int col = nb * kBM + row;
              if (col < p.M) {
                __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + col;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (g.y + c + j < g.z)
                    o[(long long)(g.y + c + j) * p.ldo] = __float2bfloat16(__uint_as_float(r[j]));
              }
            } else if (m < m_lim) {
              __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + m;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (n0 + j < p.N)
                  o[(long long)(n0 + j) * p.ldo] = __float2bfloat16(__uint_as_float(r[j]));
            }
          } else if constexpr (EPI == EPI_F32_RED) {
            if (m < m_lim) {
              float* o = reinterpret_cast<float*>(p.out) + (long long)m * p.ldo + n0;
              if (n0 + 32 <= p.N && (p.ldo % 4) == 0) {
#pragma unroll
                for (int v = 0; v < 8; ++v)
                  atomicAdd(reinterpret_cast<float4*>(o) + v,
                            make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                        __uint_as_float(r[4 * v + 2]),
                                        __uint_as_float(r[4 * v + 3])));
              } else {
                for (int j = 0; j < 32; ++j)
                  if (n0 + j < p.N) atomicAdd(o + j, __uint_as_float(r[j]));
              }
            }
          } else {  // EPI_F32_RED_T: fp32 reductions into out[n, m]
            if (m < m_lim) {
              float* o = reinterpret_cast<float*>(p.out) + m;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (n0 + j < p.N) atomicAdd(o + (long long)(n0 + j) * p.ldo, __uint_as_float(r[j]));
            }
          }
        }
      }
      if constexpr (EPI == EPI_BF16_RS) {
        // Every epilogue thread fences its own peer stores of this tile and arrives on a
        // shared-memory counter; the 128th arrival raises the owners' counters (no blocking
        // barrier, so a warp that left early on a failed wait cannot stall the others).
        __threadfence_system();
        const unsigned int prev = atomicAdd(rs_arrivals, 1u);
        if (prev == 128u * (unsigned int)(t_local + 1) - 1u) {
          __threadfence_system();
          const int r0 = trows.a_row / p.sp.rs_rows;
          const int r1 = min(trows.a_row + kBM - 1, p.M - 1) / p.sp.rs_rows;
          for (int r = r0; r <= r1; ++r)
            asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(p.sp.rs_ctr[r]) : "memory");
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || ptr == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled is not available from the driver");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2D bf16 tensor [outer, inner] with row pitch `ld` elements; box = [box_outer, box_inner].
CUtensorMap make_tmap_bf16_2d(const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                              uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr),
                               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return m;
}

CUtensorMap make_tmap_u8_2d(const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                            uint32_t box_inner, uint32_t box_outer, int swizzle_bytes) {
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                      : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr),
                               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled (u8) failed with code " +
                             std::to_string((int)r));
  return m;
}

template <int BN, int STAGES, int EPI, bool FP8 = false, int W8 = 0>
static void launch_impl(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
                        int grid, cudaStream_t stream) {
  constexpr int w8_rows = (W8 == 1 || W8 == 3) ? kBM : (W8 == 2 || W8 == 4) ? BN : 0;
  constexpr int srow = (W8 == 3 || W8 == 4) ? kBK / 2 : kBK;
  constexpr int smem = STAGES * (kATileBytes + BN * kBK * 2 + w8_rows * srow + (W8 == 6 ? 1024 : 0)) + 1024 + 512;
  static_assert(smem <= 232448, "shared memory budget");
  auto kern = gemm_bf16_kernel<BN, STAGES, EPI, FP8, W8>;
  static std::atomic<uint64_t> configured{0};  // per instantiation, per device
  set_max_dynamic_smem_once(kern, smem, configured);
  launch_pdl(kern, dim3(grid), dim3((W8 >= 1 && W8 <= 4) ? 320 : 192), smem, stream, ta, tb, p);
}

int num_sms_cached() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

void gemm_bf16_launch(const GemmArgs& a, cudaStream_t stream) {
  const int esz = a.fp8 ? 1 : 2;        // bytes per element
  const int kelems = a.fp8 ? 2 * kBK : kBK;  // elements per 128-byte k-block
  if ((a.K * esz) % 16 != 0) throw std::invalid_argument("gemm: K rows must be multiples of 16 bytes");
  if ((a.lda * esz) % 16 != 0 || (a.ldb * esz) % 16 != 0)
    throw std::invalid_argument("gemm: row pitches must be multiples of 16 bytes");
  if (gemm2sm_eligible(a)) {
    gemm2sm_launch(a, stream);
    return;
  }
  const int bn = a.bn;
  const bool grouped = a.gtiles != nullptr;
  if (grouped && (a.splits > 1 || a.splits < 0 || a.num_groups < 1 || a.gmax < 1))
    throw std::invalid_argument("gemm: grouped mode needs splits == 1, groups and a tile bound");
  if (a.grouped_t && (!grouped || a.epi != EPI_BF16_T || a.w8 == 2 || a.w8 == 4))
    throw std::invalid_argument("gemm: swapped grouped mode needs a tile list, EPI_BF16_T and the weight as A");
  if (a.fp8 && a.sp != nullptr)
    throw std::invalid_argument("gemm: FP8 operands are for the non-SP modes");
  if (a.fp8 && grouped && a.w8 != 6)
    throw std::invalid_argument("gemm: grouped FP8 operands need MXFP8 scales (w8 = 6)");
  const uint64_t b_rows = grouped && !a.grouped_t ? (uint64_t)a.N * a.num_groups : (uint64_t)a.N;
  // A rows: the stacked experts' weights in the swapped grouped mode
  const uint64_t a_rows = a.grouped_t ? (uint64_t)a.M * a.num_groups : (uint64_t)a.M;
  const bool w4 = a.w8 == 3 || a.w8 == 4;
  if (a.w8 == 1 || a.w8 == 2) {
    if (a.fp8 || a.w_scales == nullptr || a.w_scale_rows < 1 || a.w_scale_ld < (a.K + 127) / 128)
      throw std::invalid_argument("gemm: bad block-FP8 weight arguments");
    if (a.K % 16 != 0 || (a.w8 == 1 ? a.lda : a.ldb) % 16 != 0)
      throw std::invalid_argument("gemm: block-FP8 weight rows must be multiples of 16 bytes");
    const uint64_t wrows = a.w8 == 1 ? a_rows : b_rows;
    if ((uint64_t)a.w_scale_rows < (wrows + 127) / 128)
      throw std::invalid_argument("gemm: block-FP8 scale rows do not cover the weight rows");
  } else if (w4) {
    if (a.fp8 || a.w_scales8 == nullptr || a.K % 64 != 0 || a.w_scale_ld < a.K / 32)
      throw std::invalid_argument("gemm: bad MXFP4 weight arguments (K must be a multiple of 64)");
    if ((a.w8 == 3 ? a.lda : a.ldb) % 16 != 0)
      throw std::invalid_argument("gemm: MXFP4 weight rows must be multiples of 16 bytes");
    const uint64_t wrows = a.w8 == 3 ? a_rows : b_rows;
    if ((uint64_t)a.w_scale_rows < wrows)
      throw std::invalid_argument("gemm: MXFP4 scale rows do not cover the weight rows");
  } else if (a.w8 == 5) {
    // swapped decode layout (EPI_F32_RED_T): weights = A, tokens = B; prefill (EPI_BF16): tokens
    // = A, weights = B with a 128-wide N tile
    const bool swapped = a.epi == EPI_F32_RED_T;
    const int wrows = swapped ? a.M : a.N;
    if (!a.fp8 || a.w_scales == nullptr || a.x_scales == nullptr || (!swapped && a.epi != EPI_BF16) ||
        (!swapped && a.bn != 128) || grouped || a.sp != nullptr || a.K % 128 != 0 || wrows % 128 != 0 ||
        a.w_scale_ld < a.K / 128 || a.x_scale_ld < a.K / 128 || a.w_scale_rows < wrows / 128 ||
        (!swapped && a.splits > 1))
      throw std::invalid_argument("gemm: block-scaled FP8 W8A8 needs e4m3 operands, weight and activation "
                                  "block scales, EPI_F32_RED_T (weights as A) or EPI_BF16 with bn 128 "
                                  "(weights as B), K and weight rows in 128s");
  } else if (a.w8 == 6) {
    const bool ok_epi = (a.epi == EPI_BF16 && a.bn == 128) || a.epi == EPI_BF16_T || a.epi == EPI_F32_RED_T ||
                        (a.epi == EPI_F32_RED && a.bn == 128);
    // grouped: the token operand's scales are per tile-list entry (atom = entry), the stacked
    // weight's per 128 rows, so an expert's weight rows must fill whole atoms
    const bool bad_grouped = grouped && (a.grouped_t ? (a.M % 128 != 0 || a.epi != EPI_BF16_T)
                                                     : (a.N % 128 != 0 || a.epi != EPI_BF16));
    if (!a.fp8 || a.sfa == nullptr || a.sfb == nullptr || a.sp != nullptr || a.K % 128 != 0 || bad_grouped ||
        !ok_epi || (a.bn != 16 && a.bn != 32 && a.bn != 64 && a.bn != 128) ||
        (a.bn == 16 && a.N > 16 && !a.grouped_t) || (a.epi == EPI_BF16_T && a.bn == 128))
      throw std::invalid_argument("gemm: MXFP8 needs e4m3 operands with both scale atoms, K in 128s, N tile "
                                  "16 (N <= 16) / 32 / 64 / 128 and EPI_BF16 (bn 128), EPI_BF16_T, "
                                  "EPI_F32_RED_T or EPI_F32_RED; grouped: 128-row experts");
  } else if (a.w8 != 0) {
    throw std::invalid_argument("gemm: w8 must be 0..6");
  }
  // block-FP8 weight operand: bytes, 64 per row per stage, no swizzle (the converter swizzles)
  const CUtensorMap ta = a.w8 == 3 ? make_tmap_u8_2d(a.A, a.K / 2, a_rows, a.lda, kBK / 2, kBM, 0)
                         : a.w8 == 1 ? make_tmap_u8_2d(a.A, a.K, a_rows, a.lda, kBK, kBM, 0)
                         : a.fp8   ? make_tmap_u8_2d(a.A, a.K, a_rows, a.lda, 128, kBM, 128)
                                   : make_tmap_bf16_2d(a.A, a.K, a_rows, a.lda, kBK, kBM, true);
  const CUtensorMap tb = a.w8 == 4 ? make_tmap_u8_2d(a.B, a.K / 2, b_rows, a.ldb, kBK / 2, bn, 0)
                         : a.w8 == 2 ? make_tmap_u8_2d(a.B, a.K, b_rows, a.ldb, kBK, bn, 0)
                         : a.fp8   ? make_tmap_u8_2d(a.B, a.K, b_rows, a.ldb, 128, bn, 128)
                                   : make_tmap_bf16_2d(a.B, a.K, b_rows, a.ldb, kBK, bn, true);
  GemmParams p;
  p.grouped = grouped ? (a.grouped_t ? 2 : 1) : 0;
  p.gtiles = reinterpret_cast<const int4*>(a.gtiles);
  p.gcount = a.gcount;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.num_m_blocks = (a.M + kBM - 1) / kBM;
  p.num_n_blocks = (a.N + bn - 1) / bn;
  if (a.epi == EPI_SILU_BF16) p.num_n_blocks = (a.N + bn - 1) / bn;  // N = 2 * I (interleaved)
  p.num_k_blocks = (a.K + kelems - 1) / kelems;
  p.alpha = a.fp8 ? a.alpha : 1.f;
  p.wsc = a.w_scales;
  p.wsc_ld = a.w_scale_ld;
  p.wsc_rows = a.w_scale_rows;
  p.wsc8 = a.w_scales8;
  p.xsc = a.x_scales;
  p.xsc_ld = a.x_scale_ld;
  p.sfa = a.sfa;
  p.sfb = a.sfb;
  p.sf_kb = a.K / 128;
  p.streamk = a.splits < 0 ? 1 : 0;
  int splits = a.splits < 1 ? 1 : a.splits;
  if (splits > p.num_k_blocks) splits = p.num_k_blocks;
  p.kb_per_split = (p.num_k_blocks + splits - 1) / splits;
  p.splits = (p.num_k_blocks + p.kb_per_split - 1) / p.kb_per_split;  // no empty split
  if ((p.splits > 1 || p.streamk) && (a.epi != EPI_F32_RED && a.epi != EPI_F32_RED_T))
    throw std::invalid_argument("gemm: split-K / stream-K require an fp32 reduction epilogue");
  p.group_m = a.group_m > 0 ? a.group_m : 16;
  p.sp = a.sp != nullptr ? *a.sp : GemmSPArgs{};
  if (a.epi == EPI_BF16_RS && (a.sp == nullptr || a.sp->rs_rows <= 0 || grouped || p.splits > 1 ||
                               p.streamk))
    throw std::invalid_argument("gemm: the reduce-scatter epilogue needs SP args and no split-K");
  if (p.sp.ag_ctr != nullptr && (p.sp.ag_rows <= 0 || p.sp.ag_world < 1 ||
                                 p.sp.ag_world > kGemmMaxRanks ||
                                 (long long)p.sp.ag_rows * p.sp.ag_world < a.M))
    throw std::invalid_argument("gemm: bad all-gather layout");
  if (a.epi == EPI_BF16_RS &&
      ((long long)p.sp.rs_rows * kGemmMaxRanks < a.M || (a.M + p.sp.rs_rows - 1) / p.sp.rs_rows > kGemmMaxRanks))
    throw std::invalid_argument("gemm: bad reduce-scatter layout");
  p.out = a.out;
  p.ldo = a.ldo;
  p.status = a.status;
  if (a.grouped_t) p.num_n_blocks = 1;  // an entry's tokens fit one BN tile
  const long long tiles = a.grouped_t ? (long long)a.gmax * p.num_m_blocks
                          : grouped ? (long long)a.gmax * p.num_n_blocks
                                  : (long long)p.num_m_blocks * p.num_n_blocks * p.splits;
  int grid = num_sms_cached();
  if (a.max_ctas > 0 && a.max_ctas < grid) grid = a.max_ctas;
  if (p.streamk) {
    const long long units = (long long)p.num_m_blocks * p.num_n_blocks * p.num_k_blocks;
    if (units < grid) grid = (int)units;
  } else if (tiles < grid) {
    grid = (int)tiles;
  }

#define B200_GEMM_FP8_CASE(BN_, ST_, EPI_)                                \
  if (bn == BN_ && a.epi == EPI_) {                                       \
    launch_impl<BN_, ST_, EPI_, true>(ta, tb, p, grid, stream);           \
    return;                                                               \
  }
  if (a.fp8 && a.w8 == 6) {
    if (a.epi == EPI_BF16) { launch_impl<128, 6, EPI_BF16, true, 6>(ta, tb, p, grid, stream); return; }
    if (a.epi == EPI_F32_RED) { launch_impl<128, 6, EPI_F32_RED, true, 6>(ta, tb, p, grid, stream); return; }
    if (a.epi == EPI_F32_RED_T) {
      if (bn == 16) { launch_impl<16, 8, EPI_F32_RED_T, true, 6>(ta, tb, p, grid, stream); return; }
      if (bn == 32) { launch_impl<32, 8, EPI_F32_RED_T, true, 6>(ta, tb, p, grid, stream); return; }
      if (bn == 64) { launch_impl<64, 8, EPI_F32_RED_T, true, 6>(ta, tb, p, grid, stream); return; }
      launch_impl<128, 6, EPI_F32_RED_T, true, 6>(ta, tb, p, grid, stream);
      return;
    }
    if (bn == 16) { launch_impl<16, 8, EPI_BF16_T, true, 6>(ta, tb, p, grid, stream); return; }
    if (bn == 32) { launch_impl<32, 8, EPI_BF16_T, true, 6>(ta, tb, p, grid, stream); return; }
    launch_impl<64, 8, EPI_BF16_T, true, 6>(ta, tb, p, grid, stream);
    return;
  }
  if (a.fp8 && a.w8 == 5) {
    if (a.epi == EPI_BF16) { launch_impl<128, 6, EPI_BF16, true, 5>(ta, tb, p, grid, stream); return; }
    if (bn == 16) { launch_impl<16, 8, EPI_F32_RED_T, true, 5>(ta, tb, p, grid, stream); return; }
    if (bn == 32) { launch_impl<32, 8, EPI_F32_RED_T, true, 5>(ta, tb, p, grid, stream); return; }
    if (bn == 64) { launch_impl<64, 8, EPI_F32_RED_T, true, 5>(ta, tb, p, grid, stream); return; }
    throw std::invalid_argument("gemm (block-scaled fp8): N tile must be 16, 32 or 64");
  }
  if (a.fp8) {
    B200_GEMM_FP8_CASE(256, 4, EPI_BF16)
    B200_GEMM_FP8_CASE(128, 6, EPI_BF16)
    B200_GEMM_FP8_CASE(256, 4, EPI_SILU_BF16)
    B200_GEMM_FP8_CASE(128, 6, EPI_F32_RED)
    B200_GEMM_FP8_CASE(16, 8, EPI_F32_RED_T)
    B200_GEMM_FP8_CASE(32, 8, EPI_F32_RED_T)
    B200_GEMM_FP8_CASE(64, 8, EPI_F32_RED_T)
    B200_GEMM_FP8_CASE(128, 6, EPI_F32_RED_T)
    throw std::invalid_argument("gemm (fp8): unsupported (bn, epilogue) combination: bn=" +
                                std::to_string(bn) + " epi=" + std::to_string(a.epi));
  }
#undef B200_GEMM_FP8_CASE
#define B200_GEMM_W8_CASE(W8_, BN_, ST_, EPI_)                           \
  if (a.w8 == W8_ && bn == BN_ && a.epi == EPI_) {                        \
    launch_impl<BN_, ST_, EPI_, false, W8_>(ta, tb, p, grid, stream);     \
    return;                                                               \
  }
  if (a.w8 != 0) {
    // weights as A: decode (swapped operands) -- split-K fp32 reductions
    B200_GEMM_W8_CASE(1, 16, 8, EPI_F32_RED_T)
    B200_GEMM_W8_CASE(1, 32, 8, EPI_F32_RED_T)
    B200_GEMM_W8_CASE(1, 64, 7, EPI_F32_RED_T)
    B200_GEMM_W8_CASE(1, 128, 5, EPI_F32_RED_T)
    B200_GEMM_W8_CASE(1, 16, 8, EPI_BF16_T)
    B200_GEMM_W8_CASE(1, 32, 8, EPI_BF16_T)
    B200_GEMM_W8_CASE(1, 64, 7, EPI_BF16_T)
    B200_GEMM_W8_CASE(1, 128, 5, EPI_BF16_T)
    // weights as B: prefill / grouped experts
    B200_GEMM_W8_CASE(2, 256, 3, EPI_BF16)
    B200_GEMM_W8_CASE(2, 128, 5, EPI_BF16)
    B200_GEMM_W8_CASE(2, 256, 3, EPI_SILU_BF16)
    B200_GEMM_W8_CASE(2, 128, 5, EPI_F32_RED)
    B200_GEMM_W8_CASE(2, 256, 3, EPI_BF16_RS)
    B200_GEMM_W8_CASE(2, 128, 5, EPI_BF16_RS)
    // MXFP4 weights
    B200_GEMM_W8_CASE(3, 16, 8, EPI_F32_RED_T)
    B200_GEMM_W8_CASE(3, 32, 8, EPI_F32_RED_T)
    B200_GEMM_W8_CASE(3, 64, 7, EPI_F32_RED_T)
    B200_GEMM_W8_CASE(3, 128, 5, EPI_F32_RED_T)
    B200_GEMM_W8_CASE(3, 16, 8, EPI_BF16_T)
    B200_GEMM_W8_CASE(3, 32, 8, EPI_BF16_T)
    B200_GEMM_W8_CASE(3, 64, 7, EPI_BF16_T)
    B200_GEMM_W8_CASE(4, 256, 3, EPI_BF16)
    B200_GEMM_W8_CASE(4, 128, 5, EPI_BF16)
    throw std::invalid_argument("gemm (fp8 / fp4 weight): unsupported (operand, bn, epilogue): w8=" +
                                std::to_string(a.w8) + " bn=" + std::to_string(bn) +
                                " epi=" + std::to_string(a.epi));
  }
#undef B200_GEMM_W8_CASE
#define B200_GEMM_CASE(BN_, ST_, EPI_)                                    \
  if (bn == BN_ && a.epi == EPI_) {                                       \
    launch_impl<BN_, ST_, EPI_>(ta, tb, p, grid, stream);                 \
    return;                                                               \
  }
  B200_GEMM_CASE(256, 4, EPI_BF16)
  B200_GEMM_CASE(128, 6, EPI_BF16)
  B200_GEMM_CASE(256, 4, EPI_SILU_BF16)
  B200_GEMM_CASE(256, 4, EPI_BF16_RS)
  B200_GEMM_CASE(128, 6, EPI_BF16_RS)
  B200_GEMM_CASE(128, 6, EPI_F32_RED)
  B200_GEMM_CASE(256, 4, EPI_F32_RED)
  B200_GEMM_CASE(16, 8, EPI_BF16_T)
  B200_GEMM_CASE(32, 8, EPI_BF16_T)
  B200_GEMM_CASE(64, 8, EPI_BF16_T)
  B200_GEMM_CASE(128, 6, EPI_BF16_T)
  B200_GEMM_CASE(16, 8, EPI_F32_RED_T)
  B200_GEMM_CASE(32, 8, EPI_F32_RED_T)
  B200_GEMM_CASE(64, 8, EPI_F32_RED_T)
  B200_GEMM_CASE(128, 6, EPI_F32_RED_T)
#undef B200_GEMM_CASE
  throw std::invalid_argument("gemm: unsupported (bn, epilogue) combination: bn=" +
                              std::to_string(bn) + " epi=" + std::to_string(a.epi));
}

}  // namespace b200
