// Paged GQA prefill attention on the 5th-generation tensor cores (head_dim 128, bf16 KV).
//
// One CTA owns one work item: 256 packed query rows of one sequence and one KV head, held as
// two 128-row Q tiles A and B (packed row r is token r / G and query head h * G + r % G,
// G = q heads per KV head, so the G heads sharing a KV head share every K/V tile).  The two
// tiles share each 128-token K/V tile and their softmax runs ping-pong against the other
// tile's MMAs, so the tensor cores and the exponential units work at the same time.
//
//   warp 0      TMA producer: both Q tiles once (a 4-D tensor map over [T, Hkv, G, D] delivers
//               the packed rows directly), then 128-token K and V tiles page by page from the
//               block table (2-D maps over the cache rows, 128-byte swizzle) into 2-stage
//               rings.  Pages past the sequence read the null block 0.
//   warp 1      allocates TMEM (512 columns: S_A, S_B, O_A, O_B, 128 each) and one elected
//               thread issues tcgen05.mma:
//                 S_X  = Q_X K_j^T          (M 128, N 128, K 128; both operands K-major)
//                 O_X += P_X V_j            (M 128, N 128, K 128; P from TMEM, V read MN-major
//                                            straight from the token-major V tile)
//               in the order S_A(0) S_B(0) | PV_A(j) S_A(j+1) PV_B(j) S_B(j+1) | ...
//   warps 2, 3  idle
//   warps 4..7  softmax of tile A, warps 8..11 softmax of tile B: one thread per query row (its
//               TMEM lane).  tcgen05.ld of the 128 scores, causal / sliding-window mask only on
//               the tiles that cross a boundary, online softmax in the log2 domain, P (bf16)
//               stored back into the first 64 columns of the row's S (tcgen05.st), where the
//               PV MMA reads it.  The running maximum is only raised when a tile's maximum
//               exceeds it by more than 8 (a factor 256), so the O rows in TMEM are rescaled
//               rarely (the conditional rescaling of FlashAttention-4); P stays below 256 and
//               the final O / l is unchanged.
//
// P aliases S: tcgen05.mma operations of one issuing thread execute in order, so S_X(j + 1)
// overwrites P_X(j) only after PV_X(j) has read it, and the commit that reports S_X(j + 1)
// also reports PV_X(j) -- the softmax of tile j + 1 may then rescale O_X.
//
// Registers: 168 per thread (3 warps per SM sub-partition); a softmax row keeps its 128 scores
// in registers and writes P in 16-token pieces so that the peak stays below that.
//
// Shared memory: Q 2 x 32 KB, K 2 x 32 KB, V 2 x 32 KB (each [128 tokens][128 B] per
// 64-element half of d, 128-byte swizzle).  Every mbarrier wait is bounded; on expiry a role
// records a status code, raises the CTA's abort flag and leaves its loop, the producer drains
// its copies in flight, and TMEM is freed.
// Reference semantics: the context-encoding attention of vllm_neuron/functional/attention/
// attention_cte.py:189 (causal prefill with sliding window and sinks over the block table) and
// the chunked-prefill path attention_segmented_cte.py:657.
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <stdexcept>
#include <string>

#include "../common.cuh"
#include "../gemm/gemm.h"
#include "attention.h"

namespace b200 {

namespace {

constexpr int kRows = 128;                    // rows per Q tile (MMA M)
constexpr int kItemRows = 2 * kRows;          // packed rows per work item
constexpr int kTok = 128;                     // tokens per KV tile
constexpr int kHD = 128;                      // head dim
constexpr int kStages = 2;
constexpr int kQBytes = kRows * kHD * 2;      // 32 KB: 2 halves of [128][128 B]
constexpr int kKVBytes = kTok * kHD * 2;      // 32 KB: 2 halves of [128 tokens][128 B]
constexpr int kHalfBytes = kTok * 128;        // one 64-element half of d
constexpr int kSmem = 2 * kQBytes + 2 * kStages * kKVBytes;
constexpr uint32_t kTmemCols = 512;           // S_A 0, S_B 128, O_A 256, O_B 384
constexpr float kLog2eF = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;           // raise the running max only past 2^8

struct FmhaParams {
  PagedAttnParams a;
  int G;
};

__device__ __forceinline__ void tma_load_4d(const void* desc, uint64_t* bar, void* dst, int32_t c0,
                                            int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(desc), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d_nohint(const void* desc, uint64_t* bar, void* dst,
                                                   int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(desc), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_x8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
// 2^x on the multi-function unit (x <= 0 here; -inf gives +0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Shared-memory descriptor of an MN-major operand with 128-byte swizzle: rows of 128 bytes
// (64 elements along MN) for consecutive K indices, 8-row groups `sbo` bytes apart along K and
// 64-element MN blocks `lbo` bytes apart.
__device__ __forceinline__ uint64_t make_sdesc_sw128_mn(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// The KV range a work item sees: [lo, hi) in tokens, lo aligned down to the tile.
struct ItemRange {
  int b, r0, q_len, seq_len, lo, hi, ntiles, q_tok0;
  bool has_b;  // rows of tile B hold query tokens of this sequence
};
__device__ __forceinline__ ItemRange item_range(const PagedAttnParams& p, int G, int item) {
  ItemRange it;
  const int2 w = p.work[item];
  it.b = w.x;
  it.r0 = w.y;
  const int qs = p.q_start[it.b];
  it.q_len = p.q_start[it.b + 1] - qs;
  it.seq_len = p.seq_lens[it.b];
  it.q_tok0 = qs + it.r0 / G;
  it.has_b = (it.r0 + kRows) / G < it.q_len;
  const int first_tok = it.r0 / G;
  const int last_tok = min(it.q_len, (it.r0 + kItemRows + G - 1) / G) - 1;
  const int ctx = it.seq_len - it.q_len;
  const int max_pos = ctx + last_tok;
  const int min_pos = ctx + first_tok;
  int lo = 0;
  if (p.window > 0) lo = max(0, min_pos - p.window + 1);
  lo = lo / kTok * kTok;
  it.hi = min(it.seq_len, max_pos + 1);
  it.lo = lo;
  it.ntiles = it.hi > lo ? (it.hi - lo + kTok - 1) / kTok : 0;
  return it;
}

__global__ void __launch_bounds__(384, 1)
    fmha_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const FmhaParams fp) {
  const PagedAttnParams& p = fp.a;
  const int G = fp.G;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                            // [tile] 32 KB
  uint8_t* sK = sQ + 2 * kQBytes;                // [stage] 32 KB
  uint8_t* sV = sK + kStages * kKVBytes;         // [stage] 32 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kStages * kKVBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;                   // [kStages]
  uint64_t* k_empty = k_full + kStages;          // [kStages]: MMA commit after both S
  uint64_t* v_full = k_empty + kStages;          // [kStages]
  uint64_t* v_empty = v_full + kStages;          // [kStages]: MMA commit after both PV
  uint64_t* s_full = v_empty + kStages;          // [tile]: MMA commit after S_X(j)
  uint64_t* p_full = s_full + 2;                 // [tile]: 4 softmax warps
  uint64_t* o_done = p_full + 2;                 // [tile]: MMA commit after the last PV_X
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(o_done + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_s + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int h = blockIdx.y;
  const ItemRange it = item_range(p, G, blockIdx.x);

  pdl_wait();     // q and the caches are written by the previous kernels
  pdl_trigger();  // dependents launch once every CTA of this grid has started
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 4);
      mbar_init(&o_done[x], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_s, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;
  const int n = it.ntiles;
  const bool hb = it.has_b;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (elect_one()) {
      int issued = 0;
      bool ok = true;
      mbar_arrive_expect_tx(q_full, hb ? 2 * kQBytes : kQBytes);
      for (int x = 0; x < (hb ? 2 : 1); ++x)
        for (int half = 0; half < 2; ++half)
          tma_load_4d(&tmQ, q_full, sQ + x * kQBytes + half * (kRows * 128), half * 64, 0, h,
                      it.q_tok0 + x * (kRows / G));
      const int bs = p.block_size;
      const int pages = kTok / bs;
      const int* bt = p.block_tables + (long long)it.b * p.bt_stride;
      const int max_page = (it.seq_len + bs - 1) / bs;
      for (int j = 0; j < n && ok; ++j) {
        const int s = j % kStages;
        const uint32_t ph = ((j / kStages) & 1) ^ 1;
        const int page0 = (it.lo + j * kTok) / bs;
        for (int kv = 0; kv < 2; ++kv) {  // K then V of tile j
          uint64_t* empty = kv ? &v_empty[s] : &k_empty[s];
          uint64_t* full = kv ? &v_full[s] : &k_full[s];
          if (!mbar_wait_abortable(empty, ph, kTimeoutSmemEmpty, p.status, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full, kKVBytes);
          uint8_t* dst0 = (kv ? sV : sK) + s * kKVBytes;
          for (int pg = 0; pg < pages; ++pg) {
            const int page = page0 + pg;
            int blk = page < max_page ? bt[page] : 0;
            if (p.kv_rows > 0 && ((long long)blk + 1) * p.Hkv * bs > p.kv_rows) {
              set_status(p.status, kBadIndex);  // block id beyond the cache: read the null block
              blk = 0;
            }
            const int row = (blk * p.Hkv + h) * bs;
            for (int half = 0; half < 2; ++half)
              tma_load_2d_nohint(kv ? &tmV : &tmK, full, dst0 + half * kHalfBytes + pg * bs * 128, half * 64, row);
          }
          ++issued;
        }
      }
      if (!ok) {  // drain the copies in flight before shared memory is released
        mbar_wait(q_full, 0, kTimeoutTmaFull, p.status);
        const int first = issued > 2 * kStages ? issued - 2 * kStages : 0;
        for (int u = first; u < issued; ++u) {
          const int j = u >> 1;
          mbar_wait((u & 1) ? &v_full[j % kStages] : &k_full[j % kStages], (j / kStages) & 1, kTimeoutTmaFull,
                    p.status);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (elect_one()) {
      constexpr uint32_t idS = make_idesc_f16(kRows, kTok);
      constexpr uint32_t idO = make_idesc_f16(kRows, kHD) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait_abortable(q_full, 0, kTimeoutTmaFull, p.status, abort_flag);
      auto issue_s = [&](int x, int j) {
        const int s = j % kStages;
        const uint32_t d = tmem + x * kTok;
#pragma unroll
        for (int k = 0; k < kHD / 16; ++k) {
          const int half = k >> 2, kk = k & 3;
          const uint64_t ad = make_sdesc_sw128(smem_u32(sQ + x * kQBytes + half * (kRows * 128)) + kk * 32);
          const uint64_t bd = make_sdesc_sw128(smem_u32(sK + s * kKVBytes + half * kHalfBytes) + kk * 32);
          umma_f16_ss(d, ad, bd, idS, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[x]);
      };
      auto issue_pv = [&](int x, int j) {
        const int s = j % kStages;
        const uint32_t d = tmem + 2 * kTok + x * kHD;
        const uint32_t vbase = smem_u32(sV + s * kKVBytes);
#pragma unroll
        for (int k = 0; k < kTok / 16; ++k) {
          // 16 tokens = two 8-row groups; the two d halves are kHalfBytes apart
          const uint64_t bd = make_sdesc_sw128_mn(vbase + k * 2048, kHalfBytes, 1024);
          umma_f16_ts(d, tmem + x * kTok + k * 8, bd, idO, (j > 0 || k > 0) ? 1u : 0u);
        }
      };
      auto wait_k = [&](int j) {
        return mbar_wait_abortable(&k_full[j % kStages], (j / kStages) & 1, kTimeoutTmaFull, p.status, abort_flag);
      };
      if (ok && n > 0) {
        ok = wait_k(0);
        if (ok) {
          tc_fence_after();
          issue_s(0, 0);
          if (hb) issue_s(1, 0);
          umma_commit(&k_empty[0]);
        }
      }
      for (int j = 0; ok && j < n; ++j) {
        const int s = j % kStages;
        for (int x = 0; x < (hb ? 2 : 1) && ok; ++x) {
          if (!mbar_wait_abortable(&p_full[x], j & 1, kTimeoutTmemFull, p.status, abort_flag) ||
              (x == 0 && !mbar_wait_abortable(&v_full[s], (j / kStages) & 1, kTimeoutTmaFull, p.status, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(x, j);
          if (j + 1 < n) {
            if (x == 0 && !wait_k(j + 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(x, j + 1);
          } else {
            umma_commit(&o_done[x]);
          }
        }
        if (!ok) break;
        if (j + 1 < n) umma_commit(&k_empty[(j + 1) % kStages]);
        umma_commit(&v_empty[s]);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------ softmax (tile A: warps 4..7, B: 8..11) ------------------------------
    const int x = warp < 8 ? 0 : 1;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t tS = tmem + lane_base + x * kTok;
    const uint32_t tO = tmem + lane_base + 2 * kTok + x * kHD;
    const int rloc = it.r0 + x * kRows + row;  // packed row within the sequence
    const int tok_local = rloc / G;
    const bool valid = tok_local < it.q_len;
    const int pos = it.seq_len - it.q_len + tok_local;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    if (x == 0 || hb) {
      for (int j = 0; j < n; ++j) {
        if (!mbar_wait_abortable(&s_full[x], j & 1, kTimeoutTmemFull, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[kTok / 32][32];
#pragma unroll
        for (int c = 0; c < kTok / 32; ++c) tmem_ld_32x32b_x32(tS + c * 32, sr[c]);
        tmem_ld_wait();
#define SV(c) sr[(c) >> 5][(c) & 31]
        // visible keys of this row in tile-local indices: [v_lo, v_hi)
        const int kv0 = it.lo + j * kTok;
        int v_hi = valid ? min(pos, it.seq_len - 1) - kv0 + 1 : 0;
        int v_lo = p.window > 0 ? pos - p.window + 1 - kv0 : 0;
        v_hi = min(max(v_hi, 0), kTok);
        v_lo = min(max(v_lo, 0), v_hi);
        if (!__all_sync(0xffffffffu, v_lo == 0 && v_hi == kTok)) {
#pragma unroll
          for (int c = 0; c < kTok; ++c)
            if (c < v_lo || c >= v_hi) SV(c) = __float_as_uint(-INFINITY);
        }
        float mx = __uint_as_float(SV(0));
#pragma unroll
        for (int c = 1; c < kTok; ++c) mx = fmaxf(mx, __uint_as_float(SV(c)));
        const float mxs = mx * sl2;  // -inf stays -inf (sl2 > 0)
        const bool raise = mxs > m + kRescaleLog2;
        const float m_new = raise ? mxs : m;
        const float alpha = (raise && m != -INFINITY) ? ex2(m - m_new) : 1.f;
        l *= alpha;
        m = m_new;
        const float mb = (m == -INFINITY) ? 0.f : m;  // fully masked so far: every p is 0
        // P in 16-token pieces (8 TMEM columns of bf16 pairs) over the S columns already read
        float sum = 0.f;
#pragma unroll
        for (int cc = 0; cc < kTok / 16; ++cc) {
          uint32_t pk[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int c = cc * 16 + 2 * i;
            const float p0 = ex2(fmaf(__uint_as_float(SV(c)), sl2, -mb));
            const float p1 = ex2(fmaf(__uint_as_float(SV(c + 1)), sl2, -mb));
            sum += p0 + p1;
            pk[i] = pack_bf16x2(p0, p1);
          }
          tmem_st_x8(tS + cc * 8, pk);
        }
#undef SV
        l += sum;
        // O_X holds PV_X(0 .. j-1), complete: the commit of S_X(j) follows them.  Rescaled
        // after P is out of registers, before PV_X(j) is released.
        if (j > 0 && __any_sync(0xffffffffu, alpha < 1.f)) {
#pragma unroll 1
          for (int c = 0; c < kHD; c += 16) {
            uint32_t o[16];
            tmem_ld_32x32b_x16(tO + c, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st_x16(tO + c, o);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[x]);
      }
      if (ok && n > 0 && mbar_wait_abortable(&o_done[x], 0, kTimeoutTmemFull, p.status, abort_flag)) {
        tc_fence_after();
        const int head = h * G + rloc % G;
        if (p.sinks != nullptr && valid) {
          const float s2 = p.sinks[head] * kLog2eF;
          if (m == -INFINITY) {
            l += 1.f;  // no visible key: the sink takes all the weight, the output is zero
            m = s2;
          } else {
            l += ex2(s2 - m);
          }
        }
        const float inv = l > 0.f ? p.v_scale / l : 0.f;
        __nv_bfloat16* orow = p.out + (long long)(it.q_tok0 - it.r0 / G + tok_local) * p.o_stride_t + (long long)head * kHD;
#pragma unroll 1
        for (int c = 0; c < kHD; c += 32) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tO + c, o);
          tmem_ld_wait();
          if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              dst[v] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * v]) * inv, __uint_as_float(o[8 * v + 1]) * inv),
                                  pack_bf16x2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv),
                                  pack_bf16x2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv),
                                  pack_bf16x2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv));
          }
        }
      } else if (n == 0 && valid) {
        // nothing visible (a query past the sequence): zero rows
        const int head = h * G + rloc % G;
        __nv_bfloat16* orow = p.out + (long long)(it.q_tok0 - it.r0 / G + tok_local) * p.o_stride_t + (long long)head * kHD;
        for (int v = 0; v < kHD / 8; ++v) reinterpret_cast<uint4*>(orow)[v] = make_uint4(0, 0, 0, 0);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || ptr == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled is not available from the driver");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

}  // namespace

int fmha_prefill_rows() { return kItemRows; }

bool fmha_prefill_supported(const PagedAttnParams& p, int head_dim) {
  return head_dim == kHD && !p.kv_fp8 && p.num_splits == 1 && !p.partial_out && p.dcp_size <= 1 &&
         p.kv_block_stride == (long long)p.Hkv * p.block_size * kHD &&
         p.block_size > 0 && kTok % p.block_size == 0 && p.block_size % 8 == 0 && p.G > 0 &&
         kRows % p.G == 0 && p.kv_rows > 0 && (p.q_stride_t % 8) == 0 && (p.o_stride_t % 8) == 0 &&
         (reinterpret_cast<uintptr_t>(p.q) & 15) == 0 && (reinterpret_cast<uintptr_t>(p.k_cache) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(p.v_cache) & 15) == 0;
}

// Q [T, Hq = Hkv * G, D] with token stride q_stride_t; K/V [kv_rows, D] rows of the caches.
void fmha_prefill_launch(const PagedAttnParams& p, int num_work, cudaStream_t stream) {
  if (num_work == 0) return;
  const int G = p.G;
  CUtensorMap tq, tk, tv;
  {
    cuuint64_t dims[4] = {(cuuint64_t)kHD, (cuuint64_t)G, (cuuint64_t)p.Hkv, (cuuint64_t)p.total_tokens};
    cuuint64_t strides[3] = {(cuuint64_t)kHD * 2, (cuuint64_t)G * kHD * 2, (cuuint64_t)p.q_stride_t * 2};
    cuuint32_t box[4] = {64, (cuuint32_t)G, 1, (cuuint32_t)(kRows / G)};
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = encode_fn()(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<__nv_bfloat16*>(p.q), dims,
                             strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("fmha: Q tensor map failed (" + std::to_string((int)r) + ")");
  }
  tk = make_tmap_bf16_2d(p.k_cache, kHD, (uint64_t)p.kv_rows, kHD, 64, (uint32_t)p.block_size, true);
  tv = make_tmap_bf16_2d(p.v_cache, kHD, (uint64_t)p.kv_rows, kHD, 64, (uint32_t)p.block_size, true);
  FmhaParams fp;
  fp.a = p;
  fp.G = G;
  constexpr int smem = kSmem + 1024 + 256;
  static std::atomic<uint64_t> configured{0};
  set_max_dynamic_smem_once(fmha_prefill_kernel, smem, configured);
  const dim3 grid(num_work, p.Hkv);
  launch_pdl(fmha_prefill_kernel, grid, dim3(384), smem, stream, tq, tk, tv, fp);
}

}  // namespace b200
