// Paged GQA attention over a block-table KV cache, for prefill chunks, decode and mixed
// batches, with causal masking, sliding windows, learned per-head sinks and split-KV.
//
// Cache layout (per layer): K and V are [num_blocks, num_kv_heads, block_size, head_dim]
// bf16 ("HND" per block, as in the reference's NeuronAttentionBackend,
// vllm_neuron/vllm/attention/attn.py:6-35).  Query token i of sequence b sits at absolute
// position seq_len[b] - q_len[b] + i and sees KV positions j <= pos (and j > pos - window
// when a sliding window is set).  Sinks follow GPT-OSS: an extra per-head logit in the
// softmax denominator that contributes no value (reference semantics in
// vllm_neuron/functional/attention/attention_cte.py:47, attention_decode.py:653).
//
// Work decomposition.  Query rows are "packed": row r of sequence b and KV head h is
// (token r / G, q-head h * G + r % G) for G = q_heads / kv_heads, so the G heads sharing a
// KV head share every K/V tile.  A CTA (4 warps) owns one (work item, kv head, split):
//   prefill mode: 64 packed rows, warp w owns rows 16w..16w+15 and every token of a
//                 64-token K/V tile;
//   decode mode:  16 packed rows (q_len * G <= 16), warp w owns tokens 16w..16w+15 of each
//                 K/V tile; the four partial softmax states are merged at the end.
// K/V tiles are gathered from the block table with cp.async into XOR-swizzled shared
// memory (double buffered) and multiplied on the tensor cores (bf16 mma, fp32 accum).
// An FP8 (e4m3) cache keeps the same layout; its tiles are loaded into registers, widened to
// bf16 (exact) and stored to the same tiles, with the per-tensor K scale folded into the
// softmax scale and the V scale applied to the normalized output (the reference's FP8 KV
// cache: vllm_neuron/utils/dtype_utils.py, functional/attention/attention_decode.py:527-651).
// With more than one split, each split writes an fp32 partial output and its log-sum-exp
// and attn_combine_kernel merges them.
#include <cuda_bf16.h>

#include <stdexcept>
#include <string>

#include "../common.cuh"
#include "attention.h"

namespace b200 {

namespace {

constexpr int kKvTile = 64;
constexpr float kLog2e = 1.4426950408889634f;

// A block id at or beyond the cache's block count (kv_rows / (Hkv * block_size), when known)
// is replaced by the null block 0 and reported as kBadIndex in the status word, so a corrupt
// block table cannot make the kernel read outside the cache.
__device__ __forceinline__ int checked_block(const PagedAttnParams& p, int blk) {
  if (p.kv_rows > 0 && (blk < 0 || (long long)(blk + 1) * p.Hkv * p.block_size > p.kv_rows)) {
    set_status(p.status, kBadIndex);
    return 0;
  }
  return blk;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, "
      "%7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `c` of row `r` in a swizzled [rows][D] bf16 tile.
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * D * 2 + ((c ^ (r & 7)) << 4));
}

}  // namespace

// Four e4m3 bytes -> four bf16 (two words), exact.
__device__ __forceinline__ void e4m3x4_to_bf16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t a = e4m3x2_to_f16x2(w), b = e4m3x2_to_f16x2(w >> 16);
  const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&a));
  const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&b));
  lo = pack_bf16x2(fa.x, fa.y);
  hi = pack_bf16x2(fb.x, fb.y);
}

template <int D, bool DECODE, bool FP8>
__global__ void __launch_bounds__(128)
    paged_attention_kernel(const PagedAttnParams p) {
  pdl_trigger();
  pdl_wait();
  constexpr int BM = DECODE ? 16 : 64;        // packed rows per CTA
  constexpr int KVW = DECODE ? 16 : kKvTile;  // tokens per warp per tile
  constexpr int CH = D / 8;                   // 16-byte chunks per row
  constexpr int TILE_BYTES = kKvTile * D * 2;

  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK = smem + BM * D * 2;
  uint8_t* sV = sK + 2 * TILE_BYTES;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int2 w = p.work[blockIdx.x];
  const int b = w.x;
  const int row0 = w.y;
  const int kvh = blockIdx.y;
  const int split = blockIdx.z;
  const int G = p.G;

  const int q_begin = p.q_start[b];
  const int q_len = p.q_start[b + 1] - q_begin;
  const int kv_len = p.seq_lens[b];
  const int ctx0 = kv_len - q_len;
  const int rows_total = q_len * G;
  const int rows_here = min(BM, rows_total - row0);
  // Last visible key (local index) of query i of this sequence: causal in global positions,
  // mapped onto this rank's tokens under decode context parallelism.
  const int ctx0g = p.dcp_seq_lens != nullptr ? p.dcp_seq_lens[b] - q_len : 0;
  auto last_key = [&](int i) -> int {
    return p.dcp_seq_lens != nullptr
               ? dcp_last_visible(ctx0g + i, p.block_size, p.dcp_size, p.dcp_rank)
               : ctx0 + i;
  };

  // Visible KV range of the whole tile.
  const int p_min = last_key(row0 / G);
  const int p_max = last_key((row0 + rows_here - 1) / G);
  int lo = 0;
  if (p.window > 0) lo = max(0, p_min - p.window + 1);
  const int hi = min(p_max + 1, kv_len);
  const int t_lo = lo / kKvTile;
  const int t_hi = (hi + kKvTile - 1) / kKvTile;
  const int per = (t_hi - t_lo + p.num_splits - 1) / p.num_splits;
  const int s_lo = t_lo + split * per;
  const int s_hi = min(s_lo + per, t_hi);

  // ---- load Q (packed rows) into shared memory
  for (int i = threadIdx.x; i < BM * CH; i += blockDim.x) {
    const int r = i / CH, c = i % CH;
    const int pr = row0 + r;
    const bool valid = r < rows_here;
    const int tok = q_begin + (valid ? pr / G : 0);
    const int head = kvh * G + (valid ? pr % G : 0);
    const __nv_bfloat16* src = p.q + (long long)tok * p.q_stride_t + (long long)head * D + c * 8;
    cp_async16(sQ + swz<D>(r, c), src, valid);
  }
  cp_async_commit();

  auto load_kv_tile = [&](int tile, int stage) {
    const int tok0 = tile * kKvTile;
    if constexpr (FP8) {
      // e4m3 cache: 16-byte loads widened to bf16 in registers and stored to the same
      // swizzled bf16 tiles (the scales are applied to the scores and the output).
      const uint8_t* k8 = reinterpret_cast<const uint8_t*>(p.k_cache);
      const uint8_t* v8 = reinterpret_cast<const uint8_t*>(p.v_cache);
      for (int i = threadIdx.x; i < kKvTile * (D / 16); i += blockDim.x) {
        const int r = i / (D / 16), c = i % (D / 16);
        const int tok = tok0 + r;
        const bool valid = tok < kv_len;
        const int page = valid ? tok / p.block_size : 0;
        const int slot = tok - page * p.block_size;
        const int blk = valid ? checked_block(p, p.block_tables[(long long)b * p.bt_stride + page]) : 0;
        const long long off = (long long)blk * p.kv_block_stride +
                              ((long long)kvh * p.block_size + slot) * D + c * 16;
        uint4 kr = make_uint4(0u, 0u, 0u, 0u), vr = kr;
        if (valid) {
          kr = __ldg(reinterpret_cast<const uint4*>(k8 + off));
          vr = __ldg(reinterpret_cast<const uint4*>(v8 + off));
        }
        uint4 k0, k1, v0, v1;
        e4m3x4_to_bf16x4(kr.x, k0.x, k0.y);
        e4m3x4_to_bf16x4(kr.y, k0.z, k0.w);
        e4m3x4_to_bf16x4(kr.z, k1.x, k1.y);
        e4m3x4_to_bf16x4(kr.w, k1.z, k1.w);
        e4m3x4_to_bf16x4(vr.x, v0.x, v0.y);
        e4m3x4_to_bf16x4(vr.y, v0.z, v0.w);
        e4m3x4_to_bf16x4(vr.z, v1.x, v1.y);
        e4m3x4_to_bf16x4(vr.w, v1.z, v1.w);
        *reinterpret_cast<uint4*>(sK + stage * TILE_BYTES + swz<D>(r, 2 * c)) = k0;
        *reinterpret_cast<uint4*>(sK + stage * TILE_BYTES + swz<D>(r, 2 * c + 1)) = k1;
        *reinterpret_cast<uint4*>(sV + stage * TILE_BYTES + swz<D>(r, 2 * c)) = v0;
        *reinterpret_cast<uint4*>(sV + stage * TILE_BYTES + swz<D>(r, 2 * c + 1)) = v1;
      }
    } else {
    for (int i = threadIdx.x; i < kKvTile * CH; i += blockDim.x) {
      const int r = i / CH, c = i % CH;
      const int tok = tok0 + r;
      const bool valid = tok < kv_len;
      const int page = valid ? tok / p.block_size : 0;
      const int slot = tok - page * p.block_size;
      const int blk = valid ? checked_block(p, p.block_tables[(long long)b * p.bt_stride + page]) : 0;
      const long long off = (long long)blk * p.kv_block_stride +
                            ((long long)kvh * p.block_size + slot) * D + c * 8;
      cp_async16(sK + stage * TILE_BYTES + swz<D>(r, c), p.k_cache + off, valid);
      cp_async16(sV + stage * TILE_BYTES + swz<D>(r, c), p.v_cache + off, valid);
    }
    }
  };

  if (s_lo < s_hi) load_kv_tile(s_lo, 0);
  cp_async_commit();

  // ---- per-thread softmax state for rows (lane/4) and (lane/4 + 8) of the warp's 16 rows
  const int wrow = DECODE ? 0 : warp * 16;  // first tile row of this warp
  float m_r[2], l_r[2];
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  int qpos[2];
  bool rvalid[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = wrow + (lane >> 2) + h * 8;
    rvalid[h] = r < rows_here;
    const int pr = row0 + r;
    qpos[h] = last_key(pr / G);
    m_r[h] = -INFINITY;
    l_r[h] = 0.f;
    // The sink joins the softmax once, in split 0 (and in decode mode in warp 0 only).
    if (p.sinks != nullptr && split == 0 && (!DECODE || warp == 0) && rvalid[h]) {
      const int head = kvh * G + pr % G;
      m_r[h] = p.sinks[head] * kLog2e;
      l_r[h] = 1.f;
    }
  }

  cp_async_wait<1>();  // Q landed
  __syncthreads();
  uint32_t qf[D / 16][4];
#pragma unroll
  for (int k = 0; k < D / 16; ++k) {
    const int r = wrow + (lane & 15);
    const int c = k * 2 + (lane >> 4);
    ldmatrix_x4(smem_u32(sQ + swz<D>(r, c)), qf[k][0], qf[k][1], qf[k][2], qf[k][3]);
  }

  for (int tile = s_lo; tile < s_hi; ++tile) {
    const int stage = (tile - s_lo) & 1;
    if (tile + 1 < s_hi) load_kv_tile(tile + 1, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    const uint8_t* k_s = sK + stage * TILE_BYTES;
    const uint8_t* v_s = sV + stage * TILE_BYTES;
    const int kv_off = DECODE ? warp * 16 : 0;  // first tile token of this warp
    const int tok_base = tile * kKvTile + kv_off;

    // S = Q K^T over this warp's KVW tokens
    float s[KVW / 8][4];
#pragma unroll
    for (int n = 0; n < KVW / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int k = 0; k < D / 16; ++k) {
#pragma unroll
      for (int n = 0; n < KVW / 8; n += 2) {
        const int i = lane >> 3;
        const int r = kv_off + n * 8 + (i >> 1) * 8 + (lane & 7);
        const int c = k * 2 + (i & 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(smem_u32(k_s + swz<D>(r, c)), b0, b1, b2, b3);
        mma_bf16_16816(s[n], qf[k], b0, b1);
        mma_bf16_16816(s[n + 1], qf[k], b2, b3);
      }
    }

    // scale, mask, online softmax (log2 domain)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < KVW / 8; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int j = tok_base + n * 8 + (lane & 3) * 2 + e;
          bool vis = rvalid[h] && j <= qpos[h] && j < kv_len;
          if (p.window > 0) vis = vis && (j > qpos[h] - p.window);
          float v = s[n][h * 2 + e] * p.scale_log2;
          v = vis ? v : -INFINITY;
          s[n][h * 2 + e] = v;
          mx = fmaxf(mx, v);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_r[h], mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float corr = exp2f(m_r[h] - m_use);
      float rs = 0.f;
#pragma unroll
      for (int n = 0; n < KVW / 8; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pv = exp2f(s[n][h * 2 + e] - m_use);
          s[n][h * 2 + e] = pv;
          rs += pv;
        }
      }
      rs += __shfl_xor_sync(0xffffffffu, rs, 1);
      rs += __shfl_xor_sync(0xffffffffu, rs, 2);
      l_r[h] = l_r[h] * corr + rs;
      m_r[h] = m_new;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        o[n][h * 2 + 0] *= corr;
        o[n][h * 2 + 1] *= corr;
      }
    }

    // O += P V
#pragma unroll
    for (int kk = 0; kk < KVW / 16; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int n = 0; n < D / 8; n += 2) {
        const int i = lane >> 3;
        const int r = kv_off + kk * 16 + (i & 1) * 8 + (lane & 7);
        const int c = n + (i >> 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(smem_u32(v_s + swz<D>(r, c)), b0, b1, b2, b3);
        mma_bf16_16816(o[n], a, b0, b1);
        mma_bf16_16816(o[n + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  if constexpr (DECODE) {
    // Merge the four warps' partial states (same 16 rows, disjoint tokens) via smem.
    __syncthreads();
    float* sm_m = reinterpret_cast<float*>(sK);      // [4][16]
    float* sm_l = sm_m + 4 * 16;                     // [4][16]
    float* sm_o = sm_l + 4 * 16;                     // [4][16][D]  (fits in 2 K tiles)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = (lane >> 2) + h * 8;
      if ((lane & 3) == 0) {
        sm_m[warp * 16 + r] = m_r[h];
        sm_l[warp * 16 + r] = l_r[h];
      }
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        const int c = n * 8 + (lane & 3) * 2;
        sm_o[(warp * 16 + r) * D + c] = o[n][h * 2];
        sm_o[(warp * 16 + r) * D + c + 1] = o[n][h * 2 + 1];
      }
    }
    __syncthreads();
    // 128 threads: each thread finalizes (row, 16-column slice) pairs.
    for (int idx = threadIdx.x; idx < 16 * (D / 16); idx += blockDim.x) {
      const int r = idx / (D / 16);
      const int c0 = (idx % (D / 16)) * 16;
      if (r >= rows_here) continue;
      float mm = -INFINITY;
      for (int ww = 0; ww < 4; ++ww) mm = fmaxf(mm, sm_m[ww * 16 + r]);
      const float mu = (mm == -INFINITY) ? 0.f : mm;
      float ll = 0.f, f[4];
      for (int ww = 0; ww < 4; ++ww) {
        f[ww] = exp2f(sm_m[ww * 16 + r] - mu);
        ll += sm_l[ww * 16 + r] * f[ww];
      }
      const int pr = row0 + r;
      const int tok = q_begin + pr / G;
      const int head = kvh * G + pr % G;
      const float inv = (ll > 0.f ? 1.f / ll : 0.f) * (FP8 ? p.v_scale : 1.f);
      float acc[16];
      for (int c = 0; c < 16; ++c) {
        float v = 0.f;
        for (int ww = 0; ww < 4; ++ww) v += sm_o[(ww * 16 + r) * D + c0 + c] * f[ww];
        acc[c] = v * inv;
      }
      if (p.num_splits == 1 && !p.partial_out) {
        __nv_bfloat16* dst = p.out + (long long)tok * p.o_stride_t + (long long)head * D + c0;
        uint4 v0 = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                              pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
        uint4 v1 = make_uint4(pack_bf16x2(acc[8], acc[9]), pack_bf16x2(acc[10], acc[11]),
                              pack_bf16x2(acc[12], acc[13]), pack_bf16x2(acc[14], acc[15]));
        reinterpret_cast<uint4*>(dst)[0] = v0;
        reinterpret_cast<uint4*>(dst)[1] = v1;
      } else {
        float* dst = p.part_o + (((long long)split * p.total_tokens + tok) * p.Hq + head) * D + c0;
        for (int c = 0; c < 16; ++c) dst[c] = acc[c];
        if (c0 == 0)
          p.part_lse[((long long)split * p.total_tokens + tok) * p.Hq + head] =
              (ll > 0.f) ? mu + log2f(ll) : -INFINITY;
      }
    }
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (!rvalid[h]) continue;
      const int r = wrow + (lane >> 2) + h * 8;
      const int pr = row0 + r;
      const int tok = q_begin + pr / G;
      const int head = kvh * G + pr % G;
      const float inv = (l_r[h] > 0.f ? 1.f / l_r[h] : 0.f) * (FP8 ? p.v_scale : 1.f);
      if (p.num_splits == 1 && !p.partial_out) {
        __nv_bfloat16* dst = p.out + (long long)tok * p.o_stride_t + (long long)head * D;
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          const int c = n * 8 + (lane & 3) * 2;
          *reinterpret_cast<uint32_t*>(dst + c) =
              pack_bf16x2(o[n][h * 2] * inv, o[n][h * 2 + 1] * inv);
        }
      } else {
        float* dst = p.part_o + (((long long)split * p.total_tokens + tok) * p.Hq + head) * D;
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          const int c = n * 8 + (lane & 3) * 2;
          dst[c] = o[n][h * 2] * inv;
          dst[c + 1] = o[n][h * 2 + 1] * inv;
        }
        if ((lane & 3) == 0) {
          const float mu = m_r[h] == -INFINITY ? 0.f : m_r[h];
          p.part_lse[((long long)split * p.total_tokens + tok) * p.Hq + head] =
              (l_r[h] > 0.f) ? mu + log2f(l_r[h]) : -INFINITY;
        }
      }
    }
  }
}

// Merge split-KV partials: out = sum_s 2^(lse_s - M) O_s / sum_s 2^(lse_s - M).
template <int D>
__global__ void attn_combine_kernel(const float* __restrict__ part_o,
                                    const float* __restrict__ part_lse, __nv_bfloat16* out,
                                    long long o_stride_t, int total_tokens, int Hq,
                                    int num_splits) {
  pdl_trigger();
  pdl_wait();
  const int tok = blockIdx.x;
  const int head = blockIdx.y;
  float mx = -INFINITY;
  for (int s = 0; s < num_splits; ++s)
    mx = fmaxf(mx, part_lse[((long long)s * total_tokens + tok) * Hq + head]);
  const float mu = mx == -INFINITY ? 0.f : mx;
  float den = 0.f;
  for (int s = 0; s < num_splits; ++s)
    den += exp2f(part_lse[((long long)s * total_tokens + tok) * Hq + head] - mu);
  const float inv = den > 0.f ? 1.f / den : 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < num_splits; ++s) {
      const float wgt = exp2f(part_lse[((long long)s * total_tokens + tok) * Hq + head] - mu);
      if (wgt > 0.f) acc += wgt * part_o[(((long long)s * total_tokens + tok) * Hq + head) * D + d];
    }
    out[(long long)tok * o_stride_t + (long long)head * D + d] = __float2bfloat16(acc * inv);
  }
}

// Same merge, one warp per (token, head) for up to 32 splits: lane s holds split s's
// log-sum-exp, the weights come from two warp reductions, and each lane accumulates D / 32
// contiguous dims of every split with vector loads.
template <int D>
__global__ void __launch_bounds__(256) attn_combine_warp_kernel(
    const float* __restrict__ part_o, const float* __restrict__ part_lse, __nv_bfloat16* out,
    long long o_stride_t, int total_tokens, int Hq, int num_splits, const int* splits_dev) {
  pdl_trigger();
  pdl_wait();
  if (splits_dev != nullptr) {
    num_splits = max(1, min(*splits_dev, num_splits));
    if (num_splits == 1) return;  // the decode kernel wrote the output directly
  }
  constexpr int PER = D / 32;
  const int wid = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wid >= total_tokens * Hq) return;
  const int tok = wid / Hq, head = wid - tok * Hq;
  const long long row = (long long)tok * Hq + head;
  const long long split_stride = (long long)total_tokens * Hq;
  const float my = lane < num_splits ? part_lse[lane * split_stride + row] : -INFINITY;
  const float mx = warp_max(my);
  const float mu = mx == -INFINITY ? 0.f : mx;
  const float wl = lane < num_splits ? exp2f(my - mu) : 0.f;
  const float den = warp_sum(wl);
  const float inv = den > 0.f ? 1.f / den : 0.f;
  float acc[PER];
#pragma unroll
  for (int e = 0; e < PER; ++e) acc[e] = 0.f;
  // four splits per iteration: their loads are in flight together (empty splits, weight 0,
  // are not read: their partials were never written)
  for (int s0 = 0; s0 < num_splits; s0 += 4) {
    float wg[4];
    float2 v[4][PER / 2];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int sp = s0 + q;
      wg[q] = __shfl_sync(0xffffffffu, wl, sp < num_splits ? sp : 0);
      if (sp >= num_splits) wg[q] = 0.f;
      const float* src = part_o + ((long long)(sp < num_splits ? sp : 0) * split_stride + row) * D + lane * PER;
#pragma unroll
      for (int e = 0; e < PER / 2; ++e)
        v[q][e] = wg[q] != 0.f ? *reinterpret_cast<const float2*>(src + 2 * e) : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
      for (int e = 0; e < PER / 2; ++e) {
        acc[2 * e] += wg[q] * v[q][e].x;
        acc[2 * e + 1] += wg[q] * v[q][e].y;
      }
    }
  }
  __nv_bfloat16* dst = out + (long long)tok * o_stride_t + (long long)head * D + lane * PER;
#pragma unroll
  for (int e = 0; e < PER; e += 2)
    *reinterpret_cast<uint32_t*>(dst + e) = pack_bf16x2(acc[e] * inv, acc[e + 1] * inv);
}

template <int D, bool DECODE, bool FP8>
static void launch_attn_t(const PagedAttnParams& p, int num_work, cudaStream_t stream) {
  constexpr int BM = DECODE ? 16 : 64;
  constexpr int smem = BM * D * 2 + 4 * kKvTile * D * 2;
  static_assert(!DECODE || (2 * 4 * 16 + 4 * 16 * D) * 4 <= 4 * kKvTile * D * 2,
                "decode merge scratch must fit in the K/V tiles");
  auto kern = paged_attention_kernel<D, DECODE, FP8>;
  static std::atomic<uint64_t> configured{0};
  set_max_dynamic_smem_once(kern, smem, configured);
  dim3 grid(num_work, p.Hkv, p.num_splits);
  launch_pdl(kern, grid, dim3(128), smem, stream, p);
}

template <int D, bool DECODE>
static void launch_attn(const PagedAttnParams& p, int num_work, cudaStream_t stream) {
  if (p.kv_fp8)
    launch_attn_t<D, DECODE, true>(p, num_work, stream);
  else
    launch_attn_t<D, DECODE, false>(p, num_work, stream);
}

static void combine_splits(const float* po, const float* pl, __nv_bfloat16* out,
                           long long o_stride_t, int total_tokens, int Hq, int num_splits,
                           int head_dim, const int* splits_dev, cudaStream_t stream) {
  if (num_splits <= 32) {
    const dim3 grid((unsigned)((total_tokens * Hq + 7) / 8));
    if (head_dim == 128)
      launch_pdl(attn_combine_warp_kernel<128>, grid, dim3(256), 0, stream, po, pl, out,
                 o_stride_t, total_tokens, Hq, num_splits, splits_dev);
    else if (head_dim == 256)
      launch_pdl(attn_combine_warp_kernel<256>, grid, dim3(256), 0, stream, po, pl, out,
                 o_stride_t, total_tokens, Hq, num_splits, splits_dev);
    else
      launch_pdl(attn_combine_warp_kernel<64>, grid, dim3(256), 0, stream, po, pl, out,
                 o_stride_t, total_tokens, Hq, num_splits, splits_dev);
  } else {
    dim3 grid(total_tokens, Hq);
    if (head_dim == 128)
      launch_pdl(attn_combine_kernel<128>, grid, dim3(128), 0, stream, po, pl, out, o_stride_t,
                 total_tokens, Hq, num_splits);
    else if (head_dim == 256)
      launch_pdl(attn_combine_kernel<256>, grid, dim3(256), 0, stream, po, pl, out, o_stride_t,
                 total_tokens, Hq, num_splits);
    else
      launch_pdl(attn_combine_kernel<64>, grid, dim3(64), 0, stream, po, pl, out, o_stride_t,
                 total_tokens, Hq, num_splits);
  }
}

void paged_attention_launch(const PagedAttnParams& p_in, int num_work, int head_dim, bool decode,
                            cudaStream_t stream) {
  if (num_work == 0) return;
  PagedAttnParams p = p_in;
  const bool tma = decode && paged_decode_tma_supported(p, head_dim);
  // device split factors are a feature of the TMA decode path with the warp combine (<= 32)
  if (!tma || p.num_splits > 32 || p.partial_out) p.splits_dev = nullptr;
  if (!decode && p.prefill_rows == fmha_prefill_rows()) {
    if (!fmha_prefill_supported(p, head_dim))
      throw std::invalid_argument("paged_attention: tcgen05 prefill work items need head_dim 128, a bf16 "
                                  "cache, one split, no DCP and a block size dividing 128");
    fmha_prefill_launch(p, num_work, stream);
    return;
  }
  if (!decode && p.prefill_rows != 0 && p.prefill_rows != 64)
    throw std::invalid_argument("paged_attention: prefill work items must hold 64 rows (mma.sync "
                                "kernel) or " + std::to_string(fmha_prefill_rows()) + " (tcgen05 kernel)");
  if (tma) {
    paged_decode_tma_launch(p, num_work, head_dim, stream);
  } else if (head_dim == 128) {
    decode ? launch_attn<128, true>(p, num_work, stream)
           : launch_attn<128, false>(p, num_work, stream);
  } else if (head_dim == 64) {
    decode ? launch_attn<64, true>(p, num_work, stream)
           : launch_attn<64, false>(p, num_work, stream);
  } else if (head_dim == 256 && !decode) {
    launch_attn<256, false>(p, num_work, stream);
  } else {
    throw std::invalid_argument("paged_attention: unsupported head_dim " +
                                std::to_string(head_dim));
  }
  if (p.num_splits > 1 && !p.partial_out)
    combine_splits(p.part_o, p.part_lse, p.out, p.o_stride_t, p.total_tokens, p.Hq,
                   p.num_splits, head_dim, p.splits_dev, stream);
}

void attn_combine_launch(const float* part_o, const float* part_lse, __nv_bfloat16* out,
                         long long o_stride_t, int total_tokens, int Hq, int num_splits,
                         int head_dim, cudaStream_t stream) {
  if (total_tokens == 0) return;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    throw std::invalid_argument("attn_combine: unsupported head_dim " + std::to_string(head_dim));
  combine_splits(part_o, part_lse, out, o_stride_t, total_tokens, Hq, num_splits, head_dim,
                 nullptr, stream);
}

}  // namespace b200
