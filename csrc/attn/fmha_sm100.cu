// Paged GQA prefill attention on the 5th-generation tensor cores (head_dim 128, bf16 KV).
//
// One CTA owns one work item: 128 packed query rows of one sequence and one KV head (row r is
// token r / G and query head h * G + r % G, G = q heads per KV head, so the G heads sharing a KV
// head share every K/V tile).  Roles (320 threads):
//
//   warp 0      TMA producer: the Q tile once (a 4-D tensor map over [T, Hkv, G, D] delivers
//               the packed rows directly), then 64-token K and V tiles page by page from the
//               block table (2-D maps over the cache rows, 128-byte swizzle) into a 2-stage
//               ring.  Pages past the sequence read the null block 0.
//   warp 1      allocates TMEM (S double buffer: 2 x 64 fp32 columns, O: 128 columns) and one
//               elected thread issues tcgen05.mma: S_j = Q K_j^T (M 128, N 64, K 128) into
//               S[j % 2], one tile ahead of O += P_j V_j (M 128, N 128, K 64).
//   warps 2..5  softmax, one thread per query row (its TMEM lane): tcgen05.ld of the S row,
//               causal / sliding-window mask, online softmax in the log2 domain, P (bf16) into
//               shared memory as the A operand of the second MMA; when a row's running maximum
//               grows, the warp rescales its O rows in TMEM (tcgen05.ld / st) before P_j is
//               released.  At the end O / l (sinks add to l) goes to the output rows.
//   warps 6..9  V transposer: the tensor cores read both operands K-major, and V arrives
//               token-major, so each 8x8 block of the V tile is moved by ldmatrix.trans +
//               stmatrix into V^T (d rows, tokens contiguous, 128-byte swizzle).
//
// Shared memory: Q 32 KB, K 2 x 16 KB, V 2 x 16 KB, V^T 2 x 16 KB, P 16 KB.  Every mbarrier
// wait is bounded; on expiry a role records a status code, raises the CTA's abort flag and
// leaves its loop, the producer drains its copies in flight, and TMEM is freed.
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

constexpr int kRows = 128;     // packed query rows per CTA (MMA M)
constexpr int kTok = 64;       // tokens per KV tile
constexpr int kHD = 128;       // head dim
constexpr int kStages = 2;
constexpr int kQBytes = kRows * kHD * 2;      // 32 KB: 2 halves of [128][128 B]
constexpr int kKVBytes = kTok * kHD * 2;      // 16 KB: 2 halves of [64][128 B]
constexpr int kVTBytes = kHD * kTok * 2;      // 16 KB: [128 d][128 B = 64 tokens]
constexpr int kPBytes = kRows * kTok * 2;     // 16 KB: [128 rows][128 B]
constexpr int kSmem = kQBytes + 2 * kStages * kKVBytes + 2 * kVTBytes + kPBytes;
constexpr uint32_t kTmemCols = 256;           // S0 [0, 64), S1 [64, 128), O [128, 256)
constexpr float kLog2eF = 1.4426950408889634f;

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
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void stsm_x4(uint32_t addr, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}
__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// byte offset of 16-byte chunk c of row r in a 128-byte-swizzled tile (1024-byte aligned)
__device__ __forceinline__ uint32_t swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// The KV range a work item sees: [lo, hi) in tokens, lo aligned down to the tile.
struct ItemRange {
  int b, r0, q_len, seq_len, lo, hi, ntiles, q_tok0;
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
  const int first_tok = it.r0 / G;
  const int last_tok = min(it.q_len, (it.r0 + kRows + G - 1) / G) - 1;
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

__global__ void __launch_bounds__(320, 1)
    fmha_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const FmhaParams fp) {
  const PagedAttnParams& p = fp.a;
  const int G = fp.G;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kQBytes;                    // [stage] 16 KB
  uint8_t* sV = sK + kStages * kKVBytes;         // [stage] 16 KB
  uint8_t* sVT = sV + kStages * kKVBytes;        // [2] 16 KB
  uint8_t* sP = sVT + 2 * kVTBytes;              // 16 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kPBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                  // [kStages]
  uint64_t* kv_empty = kv_full + kStages;        // [kStages]: S MMA commit + 4 transposer warps
  uint64_t* vt_full = kv_empty + kStages;        // [2]: 4 transposer warps
  uint64_t* vt_empty = vt_full + 2;              // [2]: PV MMA commit
  uint64_t* s_full = vt_empty + 2;               // [2]: S MMA commit
  uint64_t* s_empty = s_full + 2;                // [2]: 4 softmax warps
  uint64_t* p_full = s_empty + 2;                // 4 softmax warps
  uint64_t* o_done = p_full + 1;                 // PV MMA commit
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(o_done + 1);
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
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 5);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&vt_full[i], 4);
      mbar_init(&vt_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
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

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (elect_one()) {
      int issued = 0;
      bool ok = true;
      mbar_arrive_expect_tx(q_full, kQBytes);
      for (int half = 0; half < 2; ++half)
        tma_load_4d(&tmQ, q_full, sQ + half * (kRows * 128), half * 64, 0, h, it.q_tok0);
      const int bs = p.block_size;
      const int pages = kTok / bs;
      const int* bt = p.block_tables + (long long)it.b * p.bt_stride;
      const int max_page = (it.seq_len + bs - 1) / bs;
      for (int j = 0; j < n && ok; ++j) {
        const int s = j % kStages;
        if (!mbar_wait_abortable(&kv_empty[s], ((j / kStages) & 1) ^ 1, kTimeoutSmemEmpty, p.status,
                                 abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[s], 2 * kKVBytes);
        const int page0 = (it.lo + j * kTok) / bs;
        for (int pg = 0; pg < pages; ++pg) {
          const int page = page0 + pg;
          int blk = page < max_page ? bt[page] : 0;
          if (p.kv_rows > 0 && ((long long)blk + 1) * p.Hkv * bs > p.kv_rows) {
            set_status(p.status, kBadIndex);  // block id beyond the cache: read the null block
            blk = 0;
          }
          const int row = (blk * p.Hkv + h) * bs;
          for (int half = 0; half < 2; ++half) {
            uint8_t* kd = sK + s * kKVBytes + half * (kTok * 128) + pg * bs * 128;
            uint8_t* vd = sV + s * kKVBytes + half * (kTok * 128) + pg * bs * 128;
            tma_load_2d_nohint(&tmK, &kv_full[s], kd, half * 64, row);
            tma_load_2d_nohint(&tmV, &kv_full[s], vd, half * 64, row);
          }
        }
        ++issued;
      }
      if (!ok) {  // drain the copies in flight before shared memory is released
        mbar_wait(q_full, 0, kTimeoutTmaFull, p.status);
        const int first = issued > kStages ? issued - kStages : 0;
        for (int j = first; j < issued; ++j) mbar_wait(&kv_full[j % kStages], (j / kStages) & 1, kTimeoutTmaFull, p.status);
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (elect_one()) {
      constexpr uint32_t idS = make_idesc_f16(kRows, kTok);
      constexpr uint32_t idO = make_idesc_f16(kRows, kHD);
      bool ok = mbar_wait_abortable(q_full, 0, kTimeoutTmaFull, p.status, abort_flag);
      auto issue_s = [&](int j) -> bool {
        const int s = j % kStages;
        if (!mbar_wait_abortable(&kv_full[s], (j / kStages) & 1, kTimeoutTmaFull, p.status, abort_flag)) return false;
        if (!mbar_wait_abortable(&s_empty[j & 1], ((j >> 1) & 1) ^ 1, kTimeoutTmemEmpty, p.status, abort_flag))
          return false;
        tc_fence_after();
        const uint32_t d = tmem + (j & 1) * kTok;
#pragma unroll
        for (int k = 0; k < kHD / 16; ++k) {
          const int half = k >> 2, kk = k & 3;
          const uint64_t ad = make_sdesc_sw128(smem_u32(sQ + half * (kRows * 128)) + kk * 32);
          const uint64_t bd = make_sdesc_sw128(smem_u32(sK + s * kKVBytes + half * (kTok * 128)) + kk * 32);
          umma_f16_ss(d, ad, bd, idS, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[j & 1]);
        umma_commit(&kv_empty[s]);
        return true;
      };
      if (ok && n > 0) ok = issue_s(0);
      for (int j = 0; ok && j < n; ++j) {
        if (j + 1 < n && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait_abortable(p_full, j & 1, kTimeoutTmemFull, p.status, abort_flag) ||
            !mbar_wait_abortable(&vt_full[j & 1], (j >> 1) & 1, kTimeoutTmaFull, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kTok / 16; ++k) {
          const uint64_t ad = make_sdesc_sw128(smem_u32(sP) + k * 32);
          const uint64_t bd = make_sdesc_sw128(smem_u32(sVT + (j & 1) * kVTBytes) + k * 32);
          umma_f16_ss(tmem + 2 * kTok, ad, bd, idO, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(o_done);
        umma_commit(&vt_empty[j & 1]);
      }
    }
  } else if (warp < 6) {
    // ------------------------------ softmax ------------------------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int tok_local = (it.r0 + row) / G;
    const bool valid = tok_local < it.q_len;
    const int pos = it.seq_len - it.q_len + tok_local;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!mbar_wait_abortable(&s_full[j & 1], (j >> 1) & 1, kTimeoutTmemFull, p.status, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[2][32];
      tmem_ld_32x32b_x32(tmem + lane_base + (j & 1) * kTok, sr[0]);
      tmem_ld_32x32b_x32(tmem + lane_base + (j & 1) * kTok + 32, sr[1]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[j & 1]);
      const int kv0 = it.lo + j * kTok;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kTok; ++c) {
        const int kv = kv0 + c;
        float v = __uint_as_float(sr[c >> 5][c & 31]) * sl2;
        const bool vis = valid && kv <= pos && kv < it.seq_len && (p.window <= 0 || kv > pos - p.window);
        v = vis ? v : -INFINITY;
        sr[c >> 5][c & 31] = __float_as_uint(v);
        mx = fmaxf(mx, v);
      }
      const float m_new = fmaxf(m, mx);
      const float alpha = (m_new == -INFINITY) ? 1.f : exp2f(m - m_new);
      float sum = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < kTok; c += 2) {
        const float v0 = __uint_as_float(sr[c >> 5][c & 31]), v1 = __uint_as_float(sr[(c + 1) >> 5][(c + 1) & 31]);
        const float p0 = (v0 == -INFINITY) ? 0.f : exp2f(v0 - m_new);
        const float p1 = (v1 == -INFINITY) ? 0.f : exp2f(v1 - m_new);
        const uint32_t u = pack_bf16x2(p0, p1);
        const float2 r = unpack_bf16x2(u);  // the denominator sums what the MMA multiplies
        sum += r.x + r.y;
        pk[c >> 1] = u;
      }
      l = l * alpha + sum;
      m = m_new;
      // O and the P buffer are free once PV_{j-1} has completed
      if (j > 0) {
        if (!mbar_wait_abortable(o_done, (j - 1) & 1, kTimeoutTmemFull, p.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha < 1.f)) {
#pragma unroll 1
          for (int c = 0; c < kHD; c += 32) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(tmem + lane_base + 2 * kTok + c, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st_x32(tmem + lane_base + 2 * kTok + c, o);
          }
          tmem_st_wait();
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(sP + swz(row, c)) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && n > 0 && mbar_wait_abortable(o_done, (n - 1) & 1, kTimeoutTmemFull, p.status, abort_flag)) {
      tc_fence_after();
      const int head = h * G + (it.r0 + row) % G;
      if (p.sinks != nullptr && valid) {
        const float s2 = p.sinks[head] * kLog2eF;
        if (m == -INFINITY) {
          l += 1.f;  // no visible key: the sink takes all the weight, the output is zero
          m = s2;
        } else {
          l += exp2f(s2 - m);
        }
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const float vs = p.v_scale;
      __nv_bfloat16* orow = p.out + (long long)(it.q_tok0 - it.r0 / G + tok_local) * p.o_stride_t + (long long)head * kHD;
#pragma unroll 1
      for (int c = 0; c < kHD; c += 32) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tmem + lane_base + 2 * kTok + c, o);
        tmem_ld_wait();
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[v] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * v]) * inv * vs, __uint_as_float(o[8 * v + 1]) * inv * vs),
                                pack_bf16x2(__uint_as_float(o[8 * v + 2]) * inv * vs, __uint_as_float(o[8 * v + 3]) * inv * vs),
                                pack_bf16x2(__uint_as_float(o[8 * v + 4]) * inv * vs, __uint_as_float(o[8 * v + 5]) * inv * vs),
                                pack_bf16x2(__uint_as_float(o[8 * v + 6]) * inv * vs, __uint_as_float(o[8 * v + 7]) * inv * vs));
        }
      }
    } else if (n == 0) {
      // nothing visible (a query past the sequence): zero rows are written for valid tokens
      const int head = h * G + (it.r0 + row) % G;
      if (valid) {
        __nv_bfloat16* orow = p.out + (long long)(it.q_tok0 - it.r0 / G + tok_local) * p.o_stride_t + (long long)head * kHD;
        for (int v = 0; v < kHD / 8; ++v) reinterpret_cast<uint4*>(orow)[v] = make_uint4(0, 0, 0, 0);
      }
    }
  } else {
    // ------------------------------ V transposer ------------------------------
    // V tile: 2 d-halves of [64 tokens][128 B] (swizzled); V^T: [128 d][128 B = 64 tokens]
    // (swizzled).  Warp tw moves the 8x8 blocks of d rows [32 tw, 32 tw + 32): per ldmatrix.x4
    // four token blocks of one 8-d column.
    const int tw = warp - 6;
    for (int j = 0; j < n; ++j) {
      const int s = j % kStages;
      if (!mbar_wait_abortable(&kv_full[s], (j / kStages) & 1, kTimeoutTmaFull, p.status, abort_flag)) break;
      if (!mbar_wait_abortable(&vt_empty[j & 1], ((j >> 1) & 1) ^ 1, kTimeoutSmemEmpty, p.status, abort_flag))
        break;
      const uint8_t* v = sV + s * kKVBytes;
      uint8_t* vt = sVT + (j & 1) * kVTBytes;
      const int mi = lane >> 3, ri = lane & 7;
#pragma unroll
      for (int db = 0; db < 4; ++db) {          // 8-d blocks of this warp
        const int d0 = tw * 32 + db * 8;
        const int half = d0 >> 6, dc = (d0 & 63) >> 3;
#pragma unroll
        for (int tb = 0; tb < kTok / 32; ++tb) {  // 4 token blocks per ldmatrix.x4
          const int t = tb * 32 + mi * 8 + ri;    // this lane's source row (token)
          uint32_t r[4];
          ldsm_x4_t(smem_u32(v + half * (kTok * 128) + swz(t, dc)), r);
          // matrix mi = tokens [tb * 32 + 8 mi, +8): destination chunk tb * 4 + mi of d row d0 + ri
          stsm_x4(smem_u32(vt + swz(d0 + ri, tb * 4 + mi)), r);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&vt_full[j & 1]);
        mbar_arrive(&kv_empty[s]);
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
  launch_pdl(fmha_prefill_kernel, grid, dim3(320), smem, stream, tq, tk, tv, fp);
}

}  // namespace b200
