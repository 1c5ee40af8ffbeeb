// Host interface of the sm_100a tcgen05 GEMM (gemm_sm100.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

enum GemmEpilogue : int {
  EPI_BF16 = 0,       // out[m, n] = D           (bf16)
  EPI_BF16_T = 1,     // out[n, m] = D           (bf16, swapped operands)
  EPI_F32_RED = 2,    // out[m, n] += D          (fp32 reduction, split-K)
  EPI_F32_RED_T = 3,  // out[n, m] += D          (fp32 reduction, swapped operands)
  EPI_SILU_BF16 = 4,  // out[m, j] = silu(gate) * up, gate/up interleaved per BN tile
  EPI_BF16_RS = 5,    // row m -> rank m / rs_rows (bf16 peer store) + per-tile counters
};

constexpr int kGemmMaxRanks = 8;

// Sequence-parallel fusion of a GEMM with the all-gather of its A rows and / or the
// reduce-scatter of its output rows over NVLink peer memory.
struct GemmSPArgs {
  // A rows [r * ag_rows, (r + 1) * ag_rows) are pushed by rank r into this rank's A buffer;
  // they are complete once ag_ctr[r] (this rank's memory, incremented by rank r) reaches
  // ag_target[r].  The TMA producer waits per rank before loading those rows.
  const unsigned int* ag_ctr = nullptr;
  unsigned int ag_target[kGemmMaxRanks] = {};
  int ag_rows = 0;
  int ag_world = 0;
  // EPI_BF16_RS: output row m is stored at rs_out[m / rs_rows] + (m % rs_rows) * ldo (rank
  // m / rs_rows's receive slot for this rank), and after each tile rs_ctr[r] += 1 for every
  // rank r whose rows the tile holds (release, system scope).
  __nv_bfloat16* rs_out[kGemmMaxRanks] = {};
  unsigned int* rs_ctr[kGemmMaxRanks] = {};
  int rs_rows = 0;
};

struct GemmArgs {
  const void* A;  // [M, K] bf16, row pitch lda
  const void* B;  // [N, K] bf16, row pitch ldb
  void* out;
  long long lda, ldb, ldo;
  int M, N, K;
  int bn;         // N tile: 16/32/64/128/256
  int epi;        // GemmEpilogue
  int splits;     // split-K factor (fp32 reduction epilogue when > 1); < 0 = stream-K
  int group_m;    // rasterization group along M (0 = default)
  int max_ctas;   // cap on persistent CTAs (0 = number of SMs)
  uint32_t* status;  // device status word for bounded-wait failures (may be null)
  // Grouped (MoE) mode: B is [num_groups * N, K]; gtiles = int4 (group, first row, end row, -)
  // entries written on the device, *gcount of them, at most gmax.
  const int* gtiles = nullptr;
  const int* gcount = nullptr;
  int gmax = 0;
  int num_groups = 0;
  // Swapped grouped mode (decode-size experts): A = stacked expert weights [num_groups * M, K],
  // B = token rows [N, K], out[token, col] (EPI_BF16_T); each entry's rows fit one BN tile.
  int grouped_t = 0;
  const GemmSPArgs* sp = nullptr;  // sequence-parallel fusion (null: plain GEMM)
  // FP8 (e4m3) operands: A and B hold bytes, K counts elements (multiple of 16), and the
  // accumulator is multiplied by `alpha` (per-tensor scales a * b) in the epilogue.
  int fp8 = 0;
  float alpha = 1.f;
  // Block-scaled FP8 weight (W8A16): w8 = 1 when A, 2 when B is the weight, held as e4m3 bytes
  // with fp32 scales [w_scale_rows][w_scale_ld], one per 128 x 128 block (row block = weight
  // row / 128, column = k / 128); the other operand is bf16.
  int w8 = 0;
  const float* w_scales = nullptr;
  int w_scale_ld = 0;
  int w_scale_rows = 0;
  // MXFP4 weight (w8 = 3 when A, 4 when B is the weight): e2m1 nibbles packed two per byte
  // (lower k in the low nibble), rows of K / 2 bytes (lda / ldb in bytes), with one e8m0 scale
  // byte per 32 elements: w_scales8 [w_scale_rows][w_scale_ld] (one row per weight row).
  const uint8_t* w_scales8 = nullptr;
  // Block-scaled FP8 W8A8 (w8 = 5, fp8 = 1, EPI_F32_RED_T, weights as A): w_scales are the
  // weight's fp32 128 x 128 block scales, x_scales [N tokens][x_scale_ld] the activations' fp32
  // scales per token and 128-wide k block; each k block is summed with its scales applied
  // (per-k-block promotion), so no operand is widened.
  const float* x_scales = nullptr;
  int x_scale_ld = 0;
  // MXFP8 x MXFP8 (w8 = 6, fp8 = 1): e4m3 A and B with e8m0 scales per 32 k elements in the
  // 512-byte atom layout (atom (row / 128, k / 128) at ((row / 128) * K / 128 + k / 128) * 512;
  // row r's 4 scales of the atom at (r % 32) * 16 + ((r / 32) % 4) * 4); K a multiple of 128.
  const uint8_t* sfa = nullptr;
  const uint8_t* sfb = nullptr;
};

void gemm_bf16_launch(const GemmArgs& args, cudaStream_t stream);
// Two-SM (cta_group::2) kernel for the large dense bf16 shapes (gemm_2sm.cu): EPI_BF16 and
// EPI_SILU_BF16, no split-K, M >= 512; gemm_bf16_launch routes eligible calls to it unless
// VLLM_B200_GEMM_2SM=0.
bool gemm2sm_enabled();
void gemm2sm_set(bool on);  // process-wide switch (benchmarks and tests)
int gemm2sm_pairs();        // co-resident CTA pairs the kernel launches
bool gemm2sm_eligible(const GemmArgs& args);
void gemm2sm_launch(const GemmArgs& args, cudaStream_t stream);
CUtensorMap make_tmap_bf16_2d(const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                              uint32_t box_inner, uint32_t box_outer, bool swizzle128);
// Byte-element 2-D map (fp8 data); swizzle_bytes is 0, 64 or 128.
CUtensorMap make_tmap_u8_2d(const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                            uint32_t box_inner, uint32_t box_outer, int swizzle_bytes);
int num_sms_cached();

}  // namespace b200
