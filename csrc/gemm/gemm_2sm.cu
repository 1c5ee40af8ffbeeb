// Two-SM (CTA pair) bf16 GEMM for the prefill projections on sm_100a.
//
//   D[M, N] = A[M, K] * B[N, K]^T   with 256 x 256 output tiles
//
// A thread-block cluster of two CTAs (one per SM of a TPC) owns each tile: CTA r loads rows
// [128 r, 128 r + 128) of the tile's A rows and of its B rows, and the even CTA issues
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16), which reads the A halves of both CTAs
// and the B halves of both CTAs.  Each CTA's TMEM receives its 128 rows x 256 columns of the
// accumulator.  Per k-block an SM therefore loads 32 KB (16 KB A + 16 KB B) for 256 x 128 x
// 64 MACs, two thirds of the 48 KB a single-SM 128 x 256 tile needs: the L2 -> SM operand
// traffic, which bounds the single-SM kernel on the large prefill shapes, drops by a third.
//
// Roles (192 threads per CTA, one CTA per SM):
//   warp 0      TMA producer (both CTAs): its A and B halves into a 6-stage ring of its own
//               shared memory.  The loads use the .cta_group::2 form, whose completion is
//               counted on the even CTA's full barrier (the even CTA's producer arms it for
//               the bytes of both halves), so one barrier tells the MMA issuer that both
//               halves of a stage have landed.  No load is multicast.
//   warp 1      allocates TMEM with the peer (2 x 256 fp32 columns, cta_group::2); in the
//               even CTA one elected thread issues the MMAs, and tcgen05.commit multicasts
//               the stage release and the accumulator-ready signal to both CTAs' barriers.
//   warps 2..5  epilogue (both CTAs): tcgen05.ld of the CTA's 128 accumulator rows, bf16
//               conversion (or SiLU(gate) * up) and global stores, overlapped with the next
//               tile's MMAs; they release the accumulator buffer on the even CTA's barrier.
//
// Epilogues: EPI_BF16 and EPI_SILU_BF16 (tile columns [0, 128) gate rows, [128, 256) the
// matching up rows, the interleave of the single-SM kernel's 256-column tile).
//
// Every wait is bounded (status word + abort flag).  A pair that gives up leaves through a
// cluster barrier after the even CTA has drained the stages it armed and its MMAs have
// retired; the copies a CTA issued land within microseconds, long before any bounded wait
// of the pair expires, so no copy outlives the CTA whose shared memory it writes.  Each CTA
// reads only its own rows from global memory.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "../common.cuh"
#include "gemm.h"

namespace b200 {

namespace {

constexpr int kTile = 256;       // output tile rows and columns (per CTA pair)
constexpr int kHalf = 128;       // rows per CTA
constexpr int kBK2 = 64;         // k elements per stage (128 bytes, one swizzle row)
constexpr int kStages2 = 6;
constexpr int kHalfBytes = kHalf * kBK2 * 2;          // 16 KB
constexpr int kStageBytes2 = 2 * kHalfBytes;          // A half + B half
constexpr int kSmem2 = kStages2 * kStageBytes2 + 1024 + 256;

struct Gemm2Params {
  int M, N, K;
  int tiles_m, tiles_n, num_k_blocks, group_m;
  void* out;
  long long ldo;
  uint32_t* status;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_rank(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
// Arrive on a barrier of another CTA of the cluster (default release semantics: the caller
// has retired its TMEM reads and fenced them with tcgen05.fence::before_thread_sync).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_2sm(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_2sm() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_2sm(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_f16_ss_2sm(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at this offset in both CTAs of the pair once the pair's MMAs issued
// so far have completed.
__device__ __forceinline__ void umma_commit_2sm_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((unsigned short)3)
      : "memory");
}
__device__ __forceinline__ void umma_commit_2sm_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 2-D tile load into this CTA's shared memory whose completion is counted on the mbarrier at
// shared::cluster address `bar` (this CTA's or the even peer's).
__device__ __forceinline__ void tma_load_2d_pair(const void* desc, uint32_t bar, void* dst, int32_t x,
                                                 int32_t y, uint64_t hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(desc), "r"(bar), "r"(x), "r"(y), "l"(hint)
      : "memory");
}

__device__ __forceinline__ void decode_tile2(const Gemm2Params& p, int t, int& tm, int& tn) {
  const int group = p.group_m * p.tiles_n;
  const int g = t / group;
  const int first = g * p.group_m;
  const int gm = min(p.tiles_m - first, p.group_m);
  const int r = t - g * group;
  tm = first + r % gm;
  tn = r / gm;
}

__device__ __forceinline__ float silu2(float x) { return x / (1.0f + __expf(-x)); }

template <int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const Gemm2Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;                                  // [stage] 16 KB
  uint8_t* smB = smem + kStages2 * kHalfBytes;          // [stage] 16 KB
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kStages2 * kStageBytes2);
  uint64_t* empty_bar = full_bar + kStages2;  // MMA commit (multicast)
  uint64_t* tfull_bar = empty_bar + kStages2; // [2] MMA commit (multicast)
  uint64_t* tempty_bar = tfull_bar + 2;       // [2] even CTA: 4 local + 4 remote epilogue warps
  uint64_t* mma_done = tempty_bar + 2;
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_smem + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_rank();
  const int cid = blockIdx.x >> 1;
  const int ncl = gridDim.x >> 1;
  const int num_tiles = p.tiles_m * p.tiles_n;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 8);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_2sm(tmem_base_smem, 512);
    tmem_relinquish_2sm();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_smem;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (elect_one()) {
      const uint64_t hint_a = policy_evict_last();   // activations: reused across N tiles
      const uint64_t hint_b = policy_evict_first();  // weights: streamed
      uint32_t it = 0;
      bool ok = true;
      bool waited = false;
      for (int t = cid; t < num_tiles && ok; t += ncl) {
        int tm, tn;
        decode_tile2(p, t, tm, tn);
        const int arow = tm * kTile + (int)rank * kHalf;
        const int brow = tn * kTile + (int)rank * kHalf;
        for (int kb = 0; kb < p.num_k_blocks; ++kb, ++it) {
          const int s = it % kStages2;
          const uint32_t ph = (it / kStages2) & 1;
          if (!mbar_wait_abortable(&empty_bar[s], ph ^ 1, kTimeoutSmemEmpty, p.status, abort_flag)) {
            ok = false;
            break;
          }
          // the even CTA's full barrier counts both CTAs' halves
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[s], 2 * kStageBytes2);
          const uint32_t fb = mapa_rank(&full_bar[s], 0);
          // the weight tile does not depend on the previous kernel: it streams in first
          tma_load_2d_pair(&tmB, fb, smB + s * kHalfBytes, kb * kBK2, brow, hint_b);
          if (!waited) {
            pdl_wait();
            waited = true;
          }
          tma_load_2d_pair(&tmA, fb, smA + s * kHalfBytes, kb * kBK2, arow, hint_a);
        }
      }
      if (!waited) pdl_wait();
      if (!ok && rank == 0) {
        const uint32_t first = it > (uint32_t)kStages2 ? it - kStages2 : 0;
        for (uint32_t j = first; j < it; ++j)
          mbar_wait(&full_bar[j % kStages2], (j / kStages2) & 1, kTimeoutTmaFull, p.status);
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // ------------------------------ MMA issuer (even CTA) ------------------------------
      if (elect_one()) {
        constexpr uint32_t kIdesc = make_idesc_f16(kTile, kTile);
        uint32_t it = 0;
        int tl = 0;
        bool ok = true;
        bool issued = false;
        for (int t = cid; t < num_tiles && ok; t += ncl, ++tl) {
          const int acc = tl & 1;
          const uint32_t aph = (tl >> 1) & 1;
          if (!mbar_wait_abortable(&tempty_bar[acc], aph ^ 1, kTimeoutTmemEmpty, p.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + acc * kTile;
          for (int kb = 0; kb < p.num_k_blocks; ++kb, ++it) {
            const int s = it % kStages2;
            const uint32_t ph = (it / kStages2) & 1;
            // both CTAs' halves of the stage have landed
            if (!mbar_wait_abortable(&full_bar[s], ph, kTimeoutTmaFull, p.status, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(smA + s * kHalfBytes);
            const uint32_t b_addr = smem_u32(smB + s * kHalfBytes);
#pragma unroll
            for (int k = 0; k < kBK2 / 16; ++k)
              umma_f16_ss_2sm(d, make_sdesc_sw128(a_addr + k * 32), make_sdesc_sw128(b_addr + k * 32), kIdesc,
                              (kb > 0 || k > 0) ? 1u : 0u);
            umma_commit_2sm_both(&empty_bar[s]);
            issued = true;
          }
          if (ok) umma_commit_2sm_both(&tfull_bar[acc]);
        }
        // no MMA may still read either CTA's shared memory when the pair leaves
        if (issued) {
          umma_commit_2sm_local(mma_done);
          mbar_wait(mma_done, 0, kTimeoutTmemFull, p.status);
        }
      }
    }
  } else {
    // ------------------------------ epilogue ------------------------------
    pdl_wait();
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t tempty_remote0 = mapa_rank(&tempty_bar[0], 0);
    const uint32_t tempty_remote1 = mapa_rank(&tempty_bar[1], 0);
    int tl = 0;
    for (int t = cid; t < num_tiles; t += ncl, ++tl) {
      const int acc = tl & 1;
      const uint32_t aph = (tl >> 1) & 1;
      if (!mbar_wait_abortable(&tfull_bar[acc], aph, kTimeoutTmemFull, p.status, abort_flag)) break;
      tc_fence_after();
      int tm, tn;
      decode_tile2(p, t, tm, tn);
      const int m = tm * kTile + (int)rank * kHalf + row;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * kTile;
      if constexpr (EPI == EPI_SILU_BF16) {
        constexpr int H = kTile / 2;
        const int n_out = p.N / 2;
        const int j_base = tn * H;
#pragma unroll 1
        for (int c = 0; c < H; c += 16) {
          uint32_t g[16], u[16];
          tmem_ld_32x32b_x16(t_row + c, g);
          tmem_ld_32x32b_x16(t_row + H + c, u);
          tmem_ld_wait();
          if (m < p.M) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + (long long)m * p.ldo;
            uint32_t pk[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
              pk[j] = pack_bf16x2(silu2(__uint_as_float(g[2 * j])) * __uint_as_float(u[2 * j]),
                                  silu2(__uint_as_float(g[2 * j + 1])) * __uint_as_float(u[2 * j + 1]));
            const int j0 = j_base + c;
            if (j0 + 16 <= n_out && (p.ldo % 8) == 0) {
              uint4* dst = reinterpret_cast<uint4*>(o + j0);
              dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
            } else {
              for (int j = 0; j < 16; ++j)
                if (j0 + j < n_out) {
                  const float2 f = unpack_bf16x2(pk[j >> 1]);
                  o[j0 + j] = __float2bfloat16((j & 1) ? f.y : f.x);
                }
            }
          }
        }
      } else {
        const int n_base = tn * kTile;
#pragma unroll 1
        for (int c = 0; c < kTile; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c, r);
          tmem_ld_wait();
          const int n0 = n_base + c;
          if (m < p.M) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + (long long)m * p.ldo + n0;
            if (n0 + 32 <= p.N && (p.ldo % 8) == 0) {
              uint4* dst = reinterpret_cast<uint4*>(o);
#pragma unroll
              for (int v = 0; v < 4; ++v)
                dst[v] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1])),
                                    pack_bf16x2(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3])),
                                    pack_bf16x2(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5])),
                                    pack_bf16x2(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7])));
            } else {
              for (int j = 0; j < 32; ++j)
                if (n0 + j < p.N) o[j] = __float2bfloat16(__uint_as_float(r[j]));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(&tempty_bar[acc]);
        else
          mbar_arrive_remote(acc ? tempty_remote1 : tempty_remote0);
      }
    }
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // no remote arrive, MMA operand read or TMEM read is outstanding
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_2sm(tmem_base, 512);
  }
}

template <int EPI>
void launch2(const CUtensorMap& ta, const CUtensorMap& tb, const Gemm2Params& p, int clusters,
             cudaStream_t stream) {
  auto kern = gemm2sm_kernel<EPI>;
  static std::atomic<uint64_t> configured{0};
  set_max_dynamic_smem_once(kern, kSmem2, configured);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = kSmem2;
  cfg.stream = stream;
  // Plain stream order (no programmatic dependent launch): with the pair kernel launched early,
  // the hybrid model's prefill (DeltaNet / MoE kernels between its CTA-pair GEMMs) stopped
  // making progress on the GPU in 4 of 4 serving runs, and ran to completion with either the
  // pair kernel or programmatic launch switched off.  The kernel does not trigger its
  // successors either, so it never overlaps a neighbouring kernel.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, p);
  if (e != cudaSuccess) throw std::runtime_error(std::string("gemm2sm launch: ") + cudaGetErrorString(e));
}

// Co-resident CTA pairs for the 2-SM kernel (per device, queried once).
int max_pairs() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] > 0) return cached[dev];
  auto kern = gemm2sm_kernel<EPI_BF16>;
  static std::atomic<uint64_t> configured{0};
  set_max_dynamic_smem_once(kern, kSmem2, configured);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 128);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = kSmem2;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = num_sms_cached() / 2;
  }
  cached[dev] = n;
  return n;
}

}  // namespace

namespace {
// -1: not read yet; 0 / 1: off / on (VLLM_B200_GEMM_2SM, or gemm2sm_set)
std::atomic<int> g_2sm_on{-1};
}  // namespace

bool gemm2sm_enabled() {
  int v = g_2sm_on.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* e = std::getenv("VLLM_B200_GEMM_2SM");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
    g_2sm_on.store(v, std::memory_order_relaxed);
  }
  return v != 0;
}

void gemm2sm_set(bool on) { g_2sm_on.store(on ? 1 : 0, std::memory_order_relaxed); }

int gemm2sm_pairs() { return max_pairs(); }

bool gemm2sm_eligible(const GemmArgs& a) {
  if (!(gemm2sm_enabled() && a.fp8 == 0 && a.w8 == 0 && a.gtiles == nullptr && a.sp == nullptr &&
        (a.epi == EPI_BF16 || (a.epi == EPI_SILU_BF16 && a.N % kTile == 0)) && a.splits <= 1 &&
        a.splits >= 0 && a.M >= 2 * kTile && a.K % 8 == 0 && a.lda % 8 == 0 && a.ldb % 8 == 0))
    return false;
  // Wave quantization: the pair kernel is ~1.15x faster per tile-wave on the large shapes, but
  // its 256 x 256 tiles come in fewer, coarser waves (a TP-sharded qkv of 768 columns has 96
  // tiles for 74 pairs).  Keep the single-SM kernel (128 x bn tiles) when its waves are fuller
  // by more than that margin.
  const int sms = num_sms_cached();
  const int pairs = max(1, sms / 2);
  const int bn1 = a.bn > 0 ? a.bn : 256;
  const long long t2 = (long long)((a.M + kTile - 1) / kTile) * ((a.N + kTile - 1) / kTile);
  const long long t1 = (long long)((a.M + 127) / 128) * ((a.N + bn1 - 1) / bn1);
  const double eff2 = (double)t2 / (double)(((t2 + pairs - 1) / pairs) * pairs);
  const double eff1 = (double)t1 / (double)(((t1 + sms - 1) / sms) * sms);
  return eff2 * 1.15 >= eff1;
}

void gemm2sm_launch(const GemmArgs& a, cudaStream_t stream) {
  if (!gemm2sm_eligible(a)) throw std::invalid_argument("gemm2sm: unsupported arguments");
  const CUtensorMap ta = make_tmap_bf16_2d(a.A, a.K, a.M, a.lda, kBK2, kHalf, true);
  const CUtensorMap tb = make_tmap_bf16_2d(a.B, a.K, a.N, a.ldb, kBK2, kHalf, true);
  Gemm2Params p;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.tiles_m = (a.M + kTile - 1) / kTile;
  p.tiles_n = (a.N + kTile - 1) / kTile;
  p.num_k_blocks = (a.K + kBK2 - 1) / kBK2;
  p.group_m = a.group_m > 0 ? a.group_m : 16;
  p.out = a.out;
  p.ldo = a.ldo;
  p.status = a.status;
  int clusters = max_pairs();
  if (a.max_ctas > 0 && a.max_ctas / 2 < clusters) clusters = a.max_ctas / 2;
  const int tiles = p.tiles_m * p.tiles_n;
  if (tiles < clusters) clusters = tiles;
  if (clusters < 1) clusters = 1;
  if (a.epi == EPI_SILU_BF16)
    launch2<EPI_SILU_BF16>(ta, tb, p, clusters, stream);
  else
    launch2<EPI_BF16>(ta, tb, p, clusters, stream);
}

}  // namespace b200
