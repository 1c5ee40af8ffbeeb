// Paged GQA decode attention: persistent warps streaming TMA-fed K/V pages (sm_100a).
//
// Same semantics as the decode mode of paged_attention.cu (up to 16 packed query rows =
// q_len * G per (sequence, KV head); causal, sliding window, sinks; split-KV partials merged
// by attn_combine_kernel), organised for bandwidth:
//
//   * Work unit = (decode work item, KV head, KV split).  One CTA per SM; each of its WARPS
//     warps claims units from a global counter (atomicAdd) until none are left, so the load
//     balances itself and no CTA pays a launch/prologue per unit.
//   * Each warp owns a private ring of STAGES shared-memory stages.  A stage holds one
//     16-token K tile and V tile of its KV head, written by the Tensor Memory Accelerator:
//     the cache of one layer, K or V [num_blocks, Hkv, block_size, D], is a 2-D tensor of rows
//     (block * Hkv + kv_head) * block_size + slot and D columns, and a 16-token chunk of one
//     page is D / 64 boxes of 16 rows x 64 columns (128-byte rows, 128-byte swizzle).
//     Completion is an mbarrier transaction count per stage.
//   * The warp's lane 0 keeps the ring STAGES tiles ahead of the warp's math, across unit
//     boundaries: while the warp finishes one unit, the first tiles of its next unit are
//     already in flight.  No CTA-wide barrier appears in the loop.
//   * Math per tile: S = Q K^T (two m16n8k16 n-tiles), online softmax in the log2 domain,
//     O += P V (D / 8 n-tiles), fp32 accumulation in registers.
//   * FP8 (e4m3) cache: the same layout in bytes, so a tile is half the bytes and the ring has
//     twice the stages.  ldmatrix reads the byte tiles as b16 matrices and cvt.e4m3x2 widens
//     them to f16 fragments: for S the k order inside each 16-dim step is permuted (the Q
//     fragments are loaded in the same order), for P V the transposed matrices give byte
//     pairs of two neighbouring dims, split by byte permutes into an even-dim and an odd-dim
//     n tile.  Q and P are f16; the K scale is folded into the softmax scale and the V scale
//     into the output normalization.
//
// Chunks past the sequence end read the null block 0 (zeros), which keeps the byte count of
// every stage constant.  Empty splits write a -inf log-sum-exp so the combine skips them.
// Every mbarrier wait is bounded: on expiry the warp records a status code, drains (again
// bounded) the copies it has in flight, and stops.
#include <cuda.h>
#include <cuda_bf16.h>

#include <atomic>
#include <stdexcept>
#include <string>

#include "../common.cuh"
#include "../gemm/gemm.h"
#include "attention.h"

namespace b200 {

namespace {

constexpr int kTok = 16;  // tokens per tile (= rows of one TMA box)
constexpr float kLog2eDec = 1.4426950408889634f;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, "
      "%7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk c of token row r in a 16-token tile written by TMA:
// D/64 boxes of [16 rows][128 B], each with the 128-byte swizzle.
__device__ __forceinline__ uint32_t kv_swz16(int r, int c) {
  return (uint32_t)((c >> 3) * (kTok * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// FP8 tiles: one TMA box per BOXC bytes of the row (BOXC = min(D, 128)), 128-byte swizzle for
// 128-byte rows, 64-byte swizzle for 64-byte rows (D = 64).
template <int BOXC>
__device__ __forceinline__ uint32_t kv_swz8(int r, int c) {
  constexpr int CPB = BOXC / 16;  // 16-byte chunks per box row
  const int box = c / CPB, cc = c % CPB;
  if constexpr (BOXC == 128)
    return (uint32_t)(box * (kTok * 128) + r * 128 + ((cc ^ (r & 7)) << 4));
  else
    return (uint32_t)(box * (kTok * 64) + r * 64 + ((cc ^ ((r >> 1) & 3)) << 4));
}

__device__ __forceinline__ void mma16816_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, "
      "%7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

struct Unit {
  int b, row0, kvh, split;
  int q_begin, kv_len, ctx0, rows_here, p_min, p_max;
  int s_lo, s_hi;  // tile range [s_lo, s_hi) of 16-token tiles
};

// Last visible key (local index) of packed query i of unit x; under decode context
// parallelism the causal limit is taken in global positions and mapped to this rank's tokens.
__device__ __forceinline__ int unit_last_key(const PagedAttnParams& p, const Unit& x, int i) {
  if (p.dcp_seq_lens == nullptr) return x.ctx0 + i;
  const int q_len = p.q_start[x.b + 1] - x.q_begin;
  return dcp_last_visible(p.dcp_seq_lens[x.b] - q_len + i, p.block_size, p.dcp_size, p.dcp_rank);
}

__device__ __forceinline__ Unit unit_info(const PagedAttnParams& p, int u, int ns) {
  Unit x;
  const int per_item = p.Hkv * ns;
  const int item = u / per_item;
  const int rem = u - item * per_item;
  x.kvh = rem / ns;
  x.split = rem - x.kvh * ns;
  const int2 w = p.work[item];
  x.b = w.x;
  x.row0 = w.y;
  x.q_begin = p.q_start[x.b];
  const int q_len = p.q_start[x.b + 1] - x.q_begin;
  x.kv_len = p.seq_lens[x.b];
  x.ctx0 = x.kv_len - q_len;
  x.rows_here = min(16, q_len * p.G - x.row0);
  x.p_min = unit_last_key(p, x, x.row0 / p.G);
  x.p_max = unit_last_key(p, x, (x.row0 + x.rows_here - 1) / p.G);
  int lo = 0;
  if (p.window > 0) lo = max(0, x.p_min - p.window + 1);
  const int hi = min(x.p_max + 1, x.kv_len);
  const int t_lo = lo / kTok;
  const int t_hi = hi > lo ? (hi + kTok - 1) / kTok : t_lo;
  const int per = (t_hi - t_lo + ns - 1) / ns;
  x.s_lo = t_lo + x.split * per;
  x.s_hi = min(x.s_lo + per, t_hi);
  return x;
}

}  // namespace

template <int D, int STAGES, int kWarps, bool FP8>
__global__ void __launch_bounds__(kWarps * 32, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const PagedAttnParams p,
                        int num_units_max) {
  constexpr int BOXC = FP8 ? (D < 128 ? D : 128) : 64;  // columns per TMA box
  constexpr int BOX_BYTES = kTok * (FP8 ? BOXC : 128);
  constexpr int HALVES = D / BOXC;
  constexpr int TILE_BYTES = kTok * D * (FP8 ? 1 : 2);  // K or V of one tile
  constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  constexpr int QN = STAGES + 2;             // claimed units not yet finished
  constexpr unsigned FULL = 0xffffffffu;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint8_t* ring = smem + warp * STAGES * STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kWarps * STAGES * STAGE_BYTES) + warp * STAGES;
  int* uq = reinterpret_cast<int*>(smem + kWarps * STAGES * STAGE_BYTES + kWarps * STAGES * 8) +
            warp * QN;

  pdl_trigger();
  if (lane == 0) {
    if (warp == 0) {
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
    }
#pragma unroll
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  pdl_wait();

  uint32_t* status = p.status;
  int* sched = p.sched;
  // split factor of this step (device value under CUDA graphs, else the launch's)
  const int ns = p.splits_dev != nullptr ? max(1, min(*p.splits_dev, p.num_splits)) : p.num_splits;
  const bool direct = ns == 1 && !p.partial_out;  // bf16 output without a split merge
  const int num_units = num_units_max / p.num_splits * ns;
  uint64_t policy = 0;
  if (lane == 0) policy = policy_evict_first();  // each K/V byte is read once per step

  // ---- producer state (uniform over the warp)
  int prod_n = 0;                     // tiles issued by this warp
  int p_tile = 0, p_end = 0, p_b = 0, p_kvh = 0, p_kvlen = 0;
  bool p_done = false;
  int q_head = 0, q_tail = 0;         // unit queue (smem ring of QN)

  auto issue = [&](int tile, int stage) {
    uint8_t* dk = ring + stage * STAGE_BYTES;
    uint8_t* dv = dk + TILE_BYTES;
    const int tok = tile * kTok;
    int blk = 0, slot0 = 0;
    if (tok < p_kvlen) {
      const int page = tok / p.block_size;
      slot0 = tok - page * p.block_size;
      blk = p.block_tables[(long long)p_b * p.bt_stride + page];
    }
    const int y = (blk * p.Hkv + p_kvh) * p.block_size + slot0;
    mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
#pragma unroll
    for (int h = 0; h < HALVES; ++h) {
      tma_load_2d(&tk, &full[stage], dk + h * BOX_BYTES, h * BOXC, y, policy);
      tma_load_2d(&tv, &full[stage], dv + h * BOX_BYTES, h * BOXC, y, policy);
    }
  };

  // Issue the next tile of the claimed units, claiming new units as needed.
  auto produce = [&]() {
    while (p_tile >= p_end) {
      if (p_done) return;
      int u = 0;
      if (lane == 0) u = atomicAdd(&sched[0], 1);
      u = __shfl_sync(FULL, u, 0);
      if (u >= num_units) {
        p_done = true;
        return;
      }
      const Unit x = unit_info(p, u, ns);
      if (x.s_lo >= x.s_hi) {
        // empty split: its partial carries no weight in the combine
        if (!direct && lane < x.rows_here) {
          const int pr = x.row0 + lane;
          const int tok = x.q_begin + pr / p.G;
          const int head = x.kvh * p.G + pr % p.G;
          p.part_lse[((long long)x.split * p.total_tokens + tok) * p.Hq + head] = -INFINITY;
        }
        continue;
      }
      if (lane == 0) uq[q_tail % QN] = u;
      __syncwarp();
      ++q_tail;
      p_tile = x.s_lo;
      p_end = x.s_hi;
      p_b = x.b;
      p_kvh = x.kvh;
      p_kvlen = x.kv_len;
    }
    if (lane == 0) issue(p_tile, prod_n % STAGES);
    ++prod_n;
    ++p_tile;
  };

  for (int i = 0; i < STAGES; ++i) produce();

  int cons_n = 0;
  bool aborted = false;
  const int g4 = lane >> 2, t4 = lane & 3;
  while (q_head < q_tail && !aborted) {
    const int u = uq[q_head % QN];
    ++q_head;
    const Unit x = unit_info(p, u, ns);

    // Q fragments (m16n8k16 A layout) straight from global memory; rows past the end are 0.
    uint32_t qf[D / 16][4];
    int qrow_tok[2], qrow_head[2];
    bool rvalid[2];
    int qpos[2];
    float m_r[2], l_r[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = g4 + h * 8;
      rvalid[h] = r < x.rows_here;
      const int pr = x.row0 + (rvalid[h] ? r : 0);
      qrow_tok[h] = x.q_begin + pr / p.G;
      qrow_head[h] = x.kvh * p.G + pr % p.G;
      qpos[h] = unit_last_key(p, x, pr / p.G);
      m_r[h] = -INFINITY;
      l_r[h] = 0.f;
      if (p.sinks != nullptr && x.split == 0 && rvalid[h]) {
        m_r[h] = p.sinks[qrow_head[h]] * kLog2eDec;
        l_r[h] = 1.f;
      }
    }
    {
      const __nv_bfloat16* q0 = p.q + (long long)qrow_tok[0] * p.q_stride_t + (long long)qrow_head[0] * D;
      const __nv_bfloat16* q1 = p.q + (long long)qrow_tok[1] * p.q_stride_t + (long long)qrow_head[1] * D;
      if constexpr (FP8) {
        // f16 fragments in the k order of the fp8 K fragments: k slots (2t, 2t+1, 2t+8, 2t+9)
        // of step k hold dims 16k + 4t + (0, 1, 2, 3).
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const int c = k * 16 + t4 * 4;
          const uint2 z = make_uint2(0u, 0u);
          const uint2 v0 = rvalid[0] ? *reinterpret_cast<const uint2*>(q0 + c) : z;
          const uint2 v1 = rvalid[1] ? *reinterpret_cast<const uint2*>(q1 + c) : z;
          qf[k][0] = bf16x2_to_f16x2_sat(v0.x);
          qf[k][1] = bf16x2_to_f16x2_sat(v1.x);
          qf[k][2] = bf16x2_to_f16x2_sat(v0.y);
          qf[k][3] = bf16x2_to_f16x2_sat(v1.y);
        }
      } else {
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const int c = k * 16 + t4 * 2;
          qf[k][0] = rvalid[0] ? *reinterpret_cast<const uint32_t*>(q0 + c) : 0u;
          qf[k][1] = rvalid[1] ? *reinterpret_cast<const uint32_t*>(q1 + c) : 0u;
          qf[k][2] = rvalid[0] ? *reinterpret_cast<const uint32_t*>(q0 + c + 8) : 0u;
          qf[k][3] = rvalid[1] ? *reinterpret_cast<const uint32_t*>(q1 + c + 8) : 0u;
        }
      }
    }
    float o[D / 8][4];
#pragma unroll
    for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

    for (int tile = x.s_lo; tile < x.s_hi; ++tile) {
      const int stage = cons_n % STAGES;
      const uint32_t phase = (uint32_t)(cons_n / STAGES) & 1u;
      const bool ok = __all_sync(FULL, mbar_wait(&full[stage], phase, kTimeoutTmaFull, status));
      if (!ok) {
        aborted = true;
        break;
      }
      const uint8_t* k_s = ring + stage * STAGE_BYTES;
      const uint8_t* v_s = k_s + TILE_BYTES;
      const int tok0 = tile * kTok;
      const bool full_vis = (tok0 + kTok <= x.p_min + 1) && (tok0 + kTok <= x.kv_len) &&
                            (p.window == 0 || tok0 > x.p_max - p.window);

      float s[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
      if constexpr (FP8) {
        // One 8x8 b16 matrix = 8 tokens x 16 fp8 dims; a lane's register holds dims
        // 16c + 4t .. 4t + 3 of token g, i.e. the B fragment of one k step after widening.
#pragma unroll
        for (int k = 0; k < D / 16; k += 2) {
          const int i = lane >> 3;
          const int r = (i & 1) * 8 + (lane & 7);
          const int c = k + (i >> 1);
          uint32_t r0, r1, r2, r3;
          ldsm_x4(smem_u32(k_s + kv_swz8<BOXC>(r, c)), r0, r1, r2, r3);
          mma16816_f16(s[0], qf[k], e4m3x2_to_f16x2(r0), e4m3x2_to_f16x2(r0 >> 16));
          mma16816_f16(s[1], qf[k], e4m3x2_to_f16x2(r1), e4m3x2_to_f16x2(r1 >> 16));
          mma16816_f16(s[0], qf[k + 1], e4m3x2_to_f16x2(r2), e4m3x2_to_f16x2(r2 >> 16));
          mma16816_f16(s[1], qf[k + 1], e4m3x2_to_f16x2(r3), e4m3x2_to_f16x2(r3 >> 16));
        }
      } else {
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const int i = lane >> 3;
          const int r = (i >> 1) * 8 + (lane & 7);
          const int c = k * 2 + (i & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(smem_u32(k_s + kv_swz16(r, c)), b0, b1, b2, b3);
          mma16816(s[0], qf[k], b0, b1);
          mma16816(s[1], qf[k], b2, b3);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float mx = -INFINITY;
#pragma unroll
        for (int n = 0; n < 2; ++n) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float v = s[n][h * 2 + e] * p.scale_log2;
            if (!full_vis) {
              const int j = tok0 + n * 8 + t4 * 2 + e;
              bool vis = rvalid[h] && j <= qpos[h] && j < x.kv_len;
              if (p.window > 0) vis = vis && (j > qpos[h] - p.window);
              v = vis ? v : -INFINITY;
            }
            s[n][h * 2 + e] = v;
            mx = fmaxf(mx, v);
          }
        }
        mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 2));
        const float m_new = fmaxf(m_r[h], mx);
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        const float corr = exp2f(m_r[h] - m_use);
        float rs = 0.f;
#pragma unroll
        for (int n = 0; n < 2; ++n) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float pv = exp2f(s[n][h * 2 + e] - m_use);
            s[n][h * 2 + e] = pv;
            rs += pv;
          }
        }
        rs += __shfl_xor_sync(FULL, rs, 1);
        rs += __shfl_xor_sync(FULL, rs, 2);
        l_r[h] = l_r[h] * corr + rs;
        m_r[h] = m_new;
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          o[n][h * 2 + 0] *= corr;
          o[n][h * 2 + 1] *= corr;
        }
      }
      uint32_t a[4];
      if constexpr (FP8) {
        a[0] = pack_f16x2(s[0][0], s[0][1]);
        a[1] = pack_f16x2(s[0][2], s[0][3]);
        a[2] = pack_f16x2(s[1][0], s[1][1]);
        a[3] = pack_f16x2(s[1][2], s[1][3]);
        // Transposed 8x8 b16 matrices of the fp8 V tile: a lane's register holds bytes
        // (token 2t, dim 2g), (2t, 2g + 1), (2t + 1, 2g), (2t + 1, 2g + 1) of a 16-dim chunk.
        // Even and odd dims of chunk c are the n tiles 2c and 2c + 1.
#pragma unroll
        for (int c = 0; c < D / 16; c += 2) {
          const int i = lane >> 3;
          const int r = (i & 1) * 8 + (lane & 7);
          const int cc = c + (i >> 1);
          uint32_t r0, r1, r2, r3;
          ldsm_x4_t(smem_u32(v_s + kv_swz8<BOXC>(r, cc)), r0, r1, r2, r3);
          mma16816_f16(o[2 * c], a, e4m3x2_to_f16x2(__byte_perm(r0, 0u, 0x0020)),
                       e4m3x2_to_f16x2(__byte_perm(r1, 0u, 0x0020)));
          mma16816_f16(o[2 * c + 1], a, e4m3x2_to_f16x2(__byte_perm(r0, 0u, 0x0031)),
                       e4m3x2_to_f16x2(__byte_perm(r1, 0u, 0x0031)));
          mma16816_f16(o[2 * c + 2], a, e4m3x2_to_f16x2(__byte_perm(r2, 0u, 0x0020)),
                       e4m3x2_to_f16x2(__byte_perm(r3, 0u, 0x0020)));
          mma16816_f16(o[2 * c + 3], a, e4m3x2_to_f16x2(__byte_perm(r2, 0u, 0x0031)),
                       e4m3x2_to_f16x2(__byte_perm(r3, 0u, 0x0031)));
        }
      } else {
        a[0] = pack_bf16x2(s[0][0], s[0][1]);
        a[1] = pack_bf16x2(s[0][2], s[0][3]);
        a[2] = pack_bf16x2(s[1][0], s[1][1]);
        a[3] = pack_bf16x2(s[1][2], s[1][3]);
#pragma unroll
        for (int n = 0; n < D / 8; n += 2) {
          const int i = lane >> 3;
          const int r = (i & 1) * 8 + (lane & 7);
          const int c = n + (i >> 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(smem_u32(v_s + kv_swz16(r, c)), b0, b1, b2, b3);
          mma16816(o[n], a, b0, b1);
          mma16816(o[n + 1], a, b2, b3);
        }
      }
      __syncwarp();  // every lane's reads of this stage are done before it is refilled
      ++cons_n;
      produce();
    }
    if (aborted) break;

    // ---- epilogue of the unit
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (!rvalid[h]) continue;
      const int tok = qrow_tok[h], head = qrow_head[h];
      const float inv = (l_r[h] > 0.f ? 1.f / l_r[h] : 0.f) * (FP8 ? p.v_scale : 1.f);
      if constexpr (FP8) {
        // n tiles 2c / 2c + 1 hold the even / odd dims of chunk c: dims 16c + 4t + (0..3)
        // are o[2c][2h], o[2c + 1][2h], o[2c][2h + 1], o[2c + 1][2h + 1].
        if (direct) {
          __nv_bfloat16* dst = p.out + (long long)tok * p.o_stride_t + (long long)head * D;
#pragma unroll
          for (int c = 0; c < D / 16; ++c)
            *reinterpret_cast<uint2*>(dst + c * 16 + t4 * 4) =
                make_uint2(pack_bf16x2(o[2 * c][h * 2] * inv, o[2 * c + 1][h * 2] * inv),
                           pack_bf16x2(o[2 * c][h * 2 + 1] * inv, o[2 * c + 1][h * 2 + 1] * inv));
        } else {
          const long long rowi = ((long long)x.split * p.total_tokens + tok) * p.Hq + head;
          float* dst = p.part_o + rowi * D;
#pragma unroll
          for (int c = 0; c < D / 16; ++c)
            *reinterpret_cast<float4*>(dst + c * 16 + t4 * 4) =
                make_float4(o[2 * c][h * 2] * inv, o[2 * c + 1][h * 2] * inv,
                            o[2 * c][h * 2 + 1] * inv, o[2 * c + 1][h * 2 + 1] * inv);
          if (t4 == 0) {
            const float mu = m_r[h] == -INFINITY ? 0.f : m_r[h];
            p.part_lse[rowi] = l_r[h] > 0.f ? mu + log2f(l_r[h]) : -INFINITY;
          }
        }
        continue;
      }
      if (direct) {
        __nv_bfloat16* dst = p.out + (long long)tok * p.o_stride_t + (long long)head * D;
#pragma unroll
        for (int n = 0; n < D / 8; ++n)
          *reinterpret_cast<uint32_t*>(dst + n * 8 + t4 * 2) =
              pack_bf16x2(o[n][h * 2] * inv, o[n][h * 2 + 1] * inv);
      } else {
        const long long rowi = ((long long)x.split * p.total_tokens + tok) * p.Hq + head;
        float* dst = p.part_o + rowi * D;
#pragma unroll
        for (int n = 0; n < D / 8; ++n)
          *reinterpret_cast<float2*>(dst + n * 8 + t4 * 2) =
              make_float2(o[n][h * 2] * inv, o[n][h * 2 + 1] * inv);
        if (t4 == 0) {
          const float mu = m_r[h] == -INFINITY ? 0.f : m_r[h];
          p.part_lse[rowi] = l_r[h] > 0.f ? mu + log2f(l_r[h]) : -INFINITY;
        }
      }
    }
  }

  if (aborted && lane == 0) {
    // drain this warp's copies in flight (bounded) before leaving
    for (int i = cons_n; i < prod_n; ++i)
      mbar_wait(&full[i % STAGES], (uint32_t)(i / STAGES) & 1u, kTimeoutTmaFull, status);
  }
  // The last warp to finish resets the unit counter for the next launch.
  if (lane == 0) {
    __threadfence();
    if (atomicAdd(&sched[1], 1) == (int)(gridDim.x * kWarps) - 1) {
      sched[0] = 0;
      sched[1] = 0;
      __threadfence();
    }
  }
}

namespace {
// Per head dim: warps per CTA and ring stages per warp (16-token K+V stages of 64 * D bytes),
// sized so the rings fill ~192 KB of shared memory with one CTA per SM.
// FP8 stages are half the bytes, so an FP8 ring has twice the stages in the same space.
template <int D, bool FP8 = false>
struct DecodeCfg {
  static constexpr int warps = D == 256 ? 4 : 8;
  static constexpr int stages = (D == 64 ? 6 : 3) * (FP8 ? 2 : 1);
  static constexpr int smem = warps * stages * 2 * kTok * D * (FP8 ? 1 : 2) + warps * stages * 8 +
                              warps * (stages + 2) * 4 + 1024;
};
}  // namespace

int paged_decode_warps_per_cta(int head_dim) {
  return head_dim == 256 ? DecodeCfg<256>::warps : DecodeCfg<128>::warps;
}

template <int D, bool FP8>
static void launch_decode(const CUtensorMap& tk, const CUtensorMap& tv, const PagedAttnParams& p,
                          int num_units, cudaStream_t stream) {
  using C = DecodeCfg<D, FP8>;
  static_assert(C::smem <= 227 * 1024, "decode ring exceeds shared memory");
  auto kern = paged_decode_kernel<D, C::stages, C::warps, FP8>;
  static std::atomic<uint64_t> configured{0};
  set_max_dynamic_smem_once(kern, C::smem, configured);
  int grid = num_sms_cached();
  const int need = (num_units + C::warps - 1) / C::warps;
  if (need < grid) grid = need;
  launch_pdl(kern, dim3(grid), dim3(C::warps * 32), C::smem, stream, tk, tv, p, num_units);
}

bool paged_decode_tma_supported(const PagedAttnParams& p, int head_dim) {
  return p.kv_rows > 0 && p.sched != nullptr &&
         (head_dim == 64 || head_dim == 128 || head_dim == 256) &&
         p.block_size % kTok == 0 &&
         p.kv_block_stride == (long long)p.Hkv * p.block_size * head_dim &&
         (reinterpret_cast<uintptr_t>(p.k_cache) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(p.v_cache) & 15) == 0;
}

void paged_decode_tma_launch(const PagedAttnParams& p, int num_work, int head_dim,
                             cudaStream_t stream) {
  const int num_units = num_work * p.Hkv * p.num_splits;
  if (p.kv_fp8) {
    const uint32_t boxc = head_dim < 128 ? (uint32_t)head_dim : 128u;
    const CUtensorMap tk = make_tmap_u8_2d(p.k_cache, head_dim, (uint64_t)p.kv_rows, head_dim,
                                           boxc, kTok, (int)boxc);
    const CUtensorMap tv = make_tmap_u8_2d(p.v_cache, head_dim, (uint64_t)p.kv_rows, head_dim,
                                           boxc, kTok, (int)boxc);
    if (head_dim == 128)
      launch_decode<128, true>(tk, tv, p, num_units, stream);
    else if (head_dim == 256)
      launch_decode<256, true>(tk, tv, p, num_units, stream);
    else
      launch_decode<64, true>(tk, tv, p, num_units, stream);
    return;
  }
  const CUtensorMap tk =
      make_tmap_bf16_2d(p.k_cache, head_dim, (uint64_t)p.kv_rows, head_dim, 64, kTok, true);
  const CUtensorMap tv =
      make_tmap_bf16_2d(p.v_cache, head_dim, (uint64_t)p.kv_rows, head_dim, 64, kTok, true);
  if (head_dim == 128)
    launch_decode<128, false>(tk, tv, p, num_units, stream);
  else if (head_dim == 256)
    launch_decode<256, false>(tk, tv, p, num_units, stream);
  else
    launch_decode<64, false>(tk, tv, p, num_units, stream);
}

}  // namespace b200
