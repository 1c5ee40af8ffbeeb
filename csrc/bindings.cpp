// Python bindings of the sm_100a kernels.  Every op launches on the caller's current CUDA
// stream and allocates nothing (outputs and scratch are passed in), so the calls can be
// recorded into CUDA graphs.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <atomic>
#include <mutex>
#include <unordered_map>

#include "attn/attention.h"
#include "comm/ep_fused.h"
#include "comm/symm_mem.h"
#include "gemm/gemm.h"
#include "misc/misc.h"
#include "moe/moe.h"
#include "deltanet/deltanet.h"

namespace {

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bfloat16")

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// One status word per device; kernels record bounded-wait failures into it.
uint32_t* status_word() {
  static std::mutex mu;
  static std::unordered_map<int, uint32_t*> words;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  auto it = words.find(dev);
  if (it != words.end()) return it->second;
  uint32_t* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, sizeof(uint32_t)) == cudaSuccess, "status word allocation failed");
  TORCH_CHECK(cudaMemset(p, 0, sizeof(uint32_t)) == cudaSuccess, "status word init failed");
  words[dev] = p;
  return p;
}

// Unit counters of the persistent decode attention kernel, one pair per device (zeroed once;
// each launch's last warp resets them).
int* decode_sched_words() {
  static std::mutex mu;
  static std::unordered_map<int, int*> words;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  auto it = words.find(dev);
  if (it != words.end()) return it->second;
  int* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, 2 * sizeof(int)) == cudaSuccess, "decode counter allocation failed");
  TORCH_CHECK(cudaMemset(p, 0, 2 * sizeof(int)) == cudaSuccess, "decode counter init failed");
  words[dev] = p;
  return p;
}

int64_t read_status() {
  uint32_t v = 0;
  TORCH_CHECK(cudaMemcpy(&v, status_word(), sizeof(v), cudaMemcpyDeviceToHost) == cudaSuccess);
  return v;
}
void reset_status() { TORCH_CHECK(cudaMemset(status_word(), 0, sizeof(uint32_t)) == cudaSuccess); }
// Asynchronous read of the status word into a pinned host int32 (ordered on the current
// stream): lets a serving loop watch for expired device waits without a device sync.
void status_copy_async(at::Tensor dst) {
  TORCH_CHECK(!dst.is_cuda() && dst.is_pinned() && dst.scalar_type() == at::kInt && dst.numel() >= 1,
              "dst must be a pinned host int32 tensor");
  TORCH_CHECK(cudaMemcpyAsync(dst.data_ptr(), status_word(), sizeof(uint32_t), cudaMemcpyDeviceToHost,
                              cur_stream()) == cudaSuccess);
}

// Number of kernels this library has launched (or recorded into a CUDA graph) in this
// process; the benchmark reports it for its timed region.
std::atomic<int64_t> g_launches{0};

void check_launch(const char* what, int kernels = 1) {
  g_launches.fetch_add(kernels, std::memory_order_relaxed);
  const cudaError_t e = cudaGetLastError();
  TORCH_CHECK(e == cudaSuccess, what, " launch failed: ", cudaGetErrorString(e));
}

// out = A @ B^T with the given epilogue.  A [M, K], B [N, K], both K-contiguous bf16.
void gemm(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, int64_t epi, int64_t bn,
          int64_t splits, int64_t group_m, int64_t max_ctas) {
  CHECK_CUDA(a);
  CHECK_CUDA(b);
  CHECK_CUDA(out);
  CHECK_BF16(a);
  CHECK_BF16(b);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1), "gemm: bad shapes");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(-1) == 1,
              "gemm: inner dims must be contiguous");
  const bool f32_out = (epi == b200::EPI_F32_RED || epi == b200::EPI_F32_RED_T);
  TORCH_CHECK(out.scalar_type() == (f32_out ? at::kFloat : at::kBFloat16), "gemm: out dtype");
  const c10::cuda::CUDAGuard guard(a.device());
  b200::GemmArgs g{};
  g.A = a.data_ptr();
  g.B = b.data_ptr();
  g.out = out.data_ptr();
  g.lda = a.stride(0);
  g.ldb = b.stride(0);
  g.ldo = out.stride(0);
  g.M = (int)a.size(0);
  g.N = (int)b.size(0);
  g.K = (int)a.size(1);
  g.bn = (int)bn;
  g.epi = (int)epi;
  g.splits = (int)splits;
  g.group_m = (int)group_m;
  g.max_ctas = (int)max_ctas;
  g.status = status_word();
  if (g.M == 0 || g.N == 0) return;
  b200::gemm_bf16_launch(g, cur_stream());
  check_launch("gemm");
}

static void fill_ptrs(const std::vector<int64_t>& v, void** dst, const char* what);

// Block-scaled FP8 weight GEMM (W8A16): out = a @ b^T where the weight operand (a when w8 == 1,
// b when w8 == 2) is float8_e4m3fn with fp32 scales [ceil(rows / 128), ceil(K / 128)] and the
// other operand is bf16; the kernel widens weight tiles in shared memory (gemm_sm100.cu).
// gtiles / gcount select the grouped (MoE) mode with w8 == 2.
void gemm_w8(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, int64_t epi, int64_t bn,
             int64_t splits, const at::Tensor& scales, int64_t w8, c10::optional<at::Tensor> gtiles,
             c10::optional<at::Tensor> gcount) {
  CHECK_CUDA(a);
  CHECK_CUDA(b);
  TORCH_CHECK(w8 >= 1 && w8 <= 4, "gemm_w8: w8 must be 1 / 2 (block FP8 weight as A / B) or 3 / 4 (MXFP4)");
  const bool fp4 = w8 >= 3;
  const at::Tensor& wt = (w8 == 1 || w8 == 3) ? a : b;
  const at::Tensor& act = (w8 == 1 || w8 == 3) ? b : a;
  if (fp4) {
    TORCH_CHECK(wt.scalar_type() == at::kByte, "gemm_w8: MXFP4 weight must be uint8 (packed e2m1)");
    TORCH_CHECK(scales.scalar_type() == at::kByte && scales.stride(-1) == 1,
                "gemm_w8: MXFP4 scales must be uint8 e8m0 [rows, K / 32]");
  } else {
    TORCH_CHECK(wt.scalar_type() == at::kFloat8_e4m3fn, "gemm_w8: weight must be float8_e4m3fn");
    TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.dim() == 2 && scales.stride(1) == 1,
                "gemm_w8: scales must be fp32 [row blocks, k blocks]");
  }
  CHECK_BF16(act);
  const bool grouped = gtiles.has_value();
  // grouped with the weight as A (w8 == 3): the swapped mode for decode-size expert batches
  TORCH_CHECK(!grouped || w8 == 2 || w8 == 3 || w8 == 4, "gemm_w8: grouped mode takes block-FP8 weights as B");
  const bool grouped_t = grouped && w8 == 3;
  TORCH_CHECK(a.stride(-1) == 1 && b.stride(-1) == 1 && out.stride(-1) == 1,
              "gemm_w8: inner dims must be contiguous");
  const bool f32_out = (epi == b200::EPI_F32_RED || epi == b200::EPI_F32_RED_T);
  TORCH_CHECK(out.scalar_type() == (f32_out ? at::kFloat : at::kBFloat16), "gemm_w8: out dtype");
  const c10::cuda::CUDAGuard guard(a.device());
  b200::GemmArgs g{};
  g.A = a.data_ptr();
  g.B = b.data_ptr();
  g.out = out.data_ptr();
  g.lda = a.stride(-2);
  g.ldb = b.stride(-2);
  g.ldo = out.stride(0);
  g.M = (int)a.size(0);
  g.K = (int)act.size(-1);  // logical elements (an MXFP4 row holds K / 2 bytes)
  TORCH_CHECK(wt.size(-1) * (fp4 ? 2 : 1) == g.K, "gemm_w8: weight and activation K differ");
  if (grouped_t) {
    TORCH_CHECK(a.dim() == 3 && a.is_contiguous() && b.dim() == 2, "gemm_w8: swapped grouped a [E, rows, K/2], b [R, K]");
    TORCH_CHECK(epi == b200::EPI_BF16_T, "gemm_w8: swapped grouped mode stores out[token, col] (EPI_BF16_T)");
    TORCH_CHECK(out.dim() == 2 && out.size(0) >= b.size(0) && out.size(1) >= a.size(1), "gemm_w8: grouped out");
    g.M = (int)a.size(1);
    g.N = (int)b.size(0);
    g.gtiles = gtiles->data_ptr<int>();
    g.gcount = gcount.value().data_ptr<int>();
    g.gmax = (int)gtiles->size(0);
    g.num_groups = (int)a.size(0);
    g.grouped_t = 1;
  } else if (grouped) {
    TORCH_CHECK(b.dim() == 3 && b.is_contiguous(), "gemm_w8: grouped b");
    TORCH_CHECK(fp4 || b.size(1) % 128 == 0, "gemm_w8: grouped block-FP8 expert rows must be multiples of 128");
    g.N = (int)b.size(1);
    g.gtiles = gtiles->data_ptr<int>();
    g.gcount = gcount.value().data_ptr<int>();
    g.gmax = (int)gtiles->size(0);
    g.num_groups = (int)b.size(0);
  } else {
    TORCH_CHECK(a.dim() == 2 && b.dim() == 2, "gemm_w8: bad shapes");
    g.N = (int)b.size(0);
  }
  g.bn = (int)bn;
  g.epi = (int)epi;
  g.splits = (int)splits;
  g.status = status_word();
  g.w8 = (int)w8;
  if (fp4) {
    g.w_scales8 = scales.data_ptr<uint8_t>();
    g.w_scale_ld = (int)scales.size(-1);
    g.w_scale_rows = (int)(scales.numel() / scales.size(-1));
    TORCH_CHECK(scales.is_contiguous(), "gemm_w8: MXFP4 scales must be contiguous");
  } else {
    g.w_scales = scales.data_ptr<float>();
    g.w_scale_ld = (int)scales.stride(0);
    g.w_scale_rows = (int)scales.size(0);
  }
  if (g.M == 0 || g.N == 0) return;
  b200::gemm_bf16_launch(g, cur_stream());
  check_launch("gemm_w8");
}

// Per-token, per-128-column FP8 quantization: out (e4m3) and scales [rows, cols / 128] fp32.
void quant_fp8_block(const at::Tensor& x, at::Tensor& out, at::Tensor& scales) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  TORCH_CHECK(out.scalar_type() == at::kFloat8_e4m3fn && scales.scalar_type() == at::kFloat,
              "quant_fp8_block: out e4m3, scales fp32");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && out.stride(1) == 1 && scales.stride(1) == 1,
              "quant_fp8_block: contiguous rows");
  TORCH_CHECK(out.size(0) >= x.size(0) && scales.size(0) >= x.size(0) && scales.size(1) >= x.size(1) / 128,
              "quant_fp8_block: output shapes");
  const c10::cuda::CUDAGuard guard(x.device());
  b200::quant_fp8_block_launch(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
                               reinterpret_cast<uint8_t*>(out.data_ptr()), out.stride(0),
                               scales.data_ptr<float>(), (int)scales.stride(0), (int)x.size(0),
                               (int)x.size(1), cur_stream());
  check_launch("quant_fp8_block");
}

// Block-scaled FP8 W8A8 decode GEMM: out[n, m] += sum_k w[m, k] xq[n, k] * ws[m / 128, k / 128] *
// xs[n, k / 128] (fp32 reductions, weights as the 128-row operand; per-k-block promotion).
void gemm_fp8_block(const at::Tensor& w, const at::Tensor& xq, at::Tensor& out, int64_t bn, int64_t splits,
                    const at::Tensor& w_scales, const at::Tensor& x_scales) {
  CHECK_CUDA(w);
  CHECK_CUDA(xq);
  TORCH_CHECK(w.scalar_type() == at::kFloat8_e4m3fn && xq.scalar_type() == at::kFloat8_e4m3fn,
              "gemm_fp8_block: operands must be float8_e4m3fn");
  TORCH_CHECK(w.dim() == 2 && xq.dim() == 2 && w.size(1) == xq.size(1), "gemm_fp8_block: bad shapes");
  TORCH_CHECK(w.stride(1) == 1 && xq.stride(1) == 1 && out.stride(1) == 1, "gemm_fp8_block: inner dims");
  TORCH_CHECK(out.scalar_type() == at::kFloat, "gemm_fp8_block: out must be fp32 (reductions)");
  TORCH_CHECK(w_scales.scalar_type() == at::kFloat && x_scales.scalar_type() == at::kFloat &&
                  w_scales.stride(1) == 1 && x_scales.stride(1) == 1,
              "gemm_fp8_block: scales must be fp32 with contiguous rows");
  const c10::cuda::CUDAGuard guard(w.device());
  b200::GemmArgs g{};
  g.A = w.data_ptr();
  g.B = xq.data_ptr();
  g.out = out.data_ptr();
  g.lda = w.stride(0);
  g.ldb = xq.stride(0);
  g.ldo = out.stride(0);
  g.M = (int)w.size(0);
  g.N = (int)xq.size(0);
  g.K = (int)w.size(1);
  g.bn = (int)bn;
  g.epi = b200::EPI_F32_RED_T;
  g.splits = (int)splits;
  g.status = status_word();
  g.fp8 = 1;
  g.w8 = 5;
  g.w_scales = w_scales.data_ptr<float>();
  g.w_scale_ld = (int)w_scales.stride(0);
  g.w_scale_rows = (int)w_scales.size(0);
  g.x_scales = x_scales.data_ptr<float>();
  g.x_scale_ld = (int)x_scales.stride(0);
  if (g.M == 0 || g.N == 0) return;
  b200::gemm_bf16_launch(g, cur_stream());
  check_launch("gemm_fp8_block");
}

// MXFP8 activations: x bf16 [M, K] -> q e4m3 [M, K] and e8m0 scales in 512-byte atoms
// [ceil(M / 128), K / 128, 512] (rows >= M of the last atom are left as they are).
void quant_mx8(const at::Tensor& x, at::Tensor& q, at::Tensor& sf) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  TORCH_CHECK(q.scalar_type() == at::kFloat8_e4m3fn && sf.scalar_type() == at::kByte, "quant_mx8: q e4m3, sf uint8");
  TORCH_CHECK(x.dim() == 2 && q.dim() == 2 && x.stride(1) == 1 && q.stride(1) == 1 && sf.is_contiguous(),
              "quant_mx8: contiguous rows");
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(q.size(0) >= M && q.size(1) == K && sf.numel() >= ((M + 127) / 128) * (K / 128) * 512,
              "quant_mx8: output shapes");
  const c10::cuda::CUDAGuard guard(x.device());
  b200::quant_mx8_launch(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
                         reinterpret_cast<uint8_t*>(q.data_ptr()), q.stride(0), sf.data_ptr<uint8_t>(), (int)M,
                         (int)K, cur_stream());
  check_launch("quant_mx8");
}

// MXFP8 of expert-sorted rows x [R, kvalid] (bf16) into q [R, K] (K >= kvalid, a multiple of 128;
// columns past kvalid are zeros) and per-entry scale atoms sf [gmax, K / 128, 512].
void quant_mx8_tiles(const at::Tensor& x, at::Tensor& q, at::Tensor& sf, const at::Tensor& gtiles,
                     const at::Tensor& gcount) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  TORCH_CHECK(q.scalar_type() == at::kFloat8_e4m3fn && sf.scalar_type() == at::kByte, "quant_mx8_tiles: q e4m3, sf uint8");
  TORCH_CHECK(x.dim() == 2 && q.dim() == 2 && x.stride(1) == 1 && q.stride(1) == 1 && sf.is_contiguous() &&
                  gtiles.is_contiguous() && gtiles.size(-1) == 4, "quant_mx8_tiles: layouts");
  const int64_t K = q.size(1), gmax = gtiles.size(0);
  TORCH_CHECK(q.size(0) >= x.size(0) && x.size(1) <= K && sf.numel() >= gmax * (K / 128) * 512,
              "quant_mx8_tiles: output shapes");
  const c10::cuda::CUDAGuard guard(x.device());
  b200::quant_mx8_tiles_launch(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
                               reinterpret_cast<uint8_t*>(q.data_ptr()), q.stride(0), sf.data_ptr<uint8_t>(),
                               gtiles.data_ptr<int>(), gcount.data_ptr<int>(), (int)gmax, (int)K, (int)x.size(1),
                               cur_stream());
  check_launch("quant_mx8_tiles");
}

// Grouped MXFP8 expert GEMM.  grouped_t = 0 (prefill): a = expert-sorted token rows [R, K] with
// per-entry atoms sfa, b = stacked expert weights [E, N, K] (N a multiple of 128) with atoms sfb
// over the stacked rows, EPI_BF16 out[R, N], bn 128.  grouped_t = 1 (decode): a = stacked weights
// [E, M, K] (M a multiple of 128), b = token rows [R, K] with per-entry atoms, EPI_BF16_T
// out[R, M] with bn >= the tokens of any expert.
void gemm_mx8_grouped(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, int64_t epi, int64_t bn,
                      const at::Tensor& sfa, const at::Tensor& sfb, const at::Tensor& gtiles,
                      const at::Tensor& gcount, int64_t grouped_t) {
  CHECK_CUDA(a);
  CHECK_CUDA(b);
  CHECK_BF16(out);
  TORCH_CHECK(a.scalar_type() == at::kFloat8_e4m3fn && b.scalar_type() == at::kFloat8_e4m3fn,
              "gemm_mx8_grouped: operands must be float8_e4m3fn");
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous() && out.stride(1) == 1 && sfa.is_contiguous() &&
                  sfb.is_contiguous() && sfa.scalar_type() == at::kByte && sfb.scalar_type() == at::kByte,
              "gemm_mx8_grouped: layouts");
  const c10::cuda::CUDAGuard guard(a.device());
  b200::GemmArgs g{};
  g.A = a.data_ptr();
  g.B = b.data_ptr();
  g.out = out.data_ptr();
  g.lda = a.size(-1);
  g.ldb = b.size(-1);
  g.ldo = out.stride(0);
  g.K = (int)a.size(-1);
  TORCH_CHECK(b.size(-1) == g.K && g.K % 128 == 0, "gemm_mx8_grouped: K");
  if (grouped_t) {
    TORCH_CHECK(a.dim() == 3 && b.dim() == 2 && epi == b200::EPI_BF16_T, "gemm_mx8_grouped: a [E, M, K], b [R, K]");
    TORCH_CHECK(out.size(0) >= b.size(0) && out.size(1) >= a.size(1), "gemm_mx8_grouped: out");
    g.M = (int)a.size(1);
    g.N = (int)b.size(0);
    g.num_groups = (int)a.size(0);
    g.grouped_t = 1;
    TORCH_CHECK(sfa.numel() >= a.size(0) * a.size(1) / 128 * (g.K / 128) * 512 &&
                    sfb.numel() >= gtiles.size(0) * (g.K / 128) * 512, "gemm_mx8_grouped: scale atoms");
  } else {
    TORCH_CHECK(a.dim() == 2 && b.dim() == 3 && epi == b200::EPI_BF16, "gemm_mx8_grouped: a [R, K], b [E, N, K]");
    TORCH_CHECK(out.size(0) >= a.size(0) && out.size(1) >= b.size(1), "gemm_mx8_grouped: out");
    g.M = (int)a.size(0);
    g.N = (int)b.size(1);
    g.num_groups = (int)b.size(0);
    TORCH_CHECK(sfb.numel() >= b.size(0) * b.size(1) / 128 * (g.K / 128) * 512 &&
                    sfa.numel() >= gtiles.size(0) * (g.K / 128) * 512, "gemm_mx8_grouped: scale atoms");
  }
  g.gtiles = gtiles.data_ptr<int>();
  g.gcount = gcount.data_ptr<int>();
  g.gmax = (int)gtiles.size(0);
  g.bn = (int)bn;
  g.epi = (int)epi;
  g.splits = 1;
  g.status = status_word();
  g.fp8 = 1;
  g.w8 = 6;
  g.sfa = sfa.data_ptr<uint8_t>();
  g.sfb = sfb.data_ptr<uint8_t>();
  if (g.M == 0 || g.N == 0) return;
  b200::gemm_bf16_launch(g, cur_stream());
  check_launch("gemm_mx8_grouped");
}

// MXFP8 x MXFP8 GEMM on the block-scaled tensor cores: out = a @ b^T with a [M, K], b [N, K] e4m3
// and their scale atoms (see quant_mx8).  epi: EPI_BF16 (bn 128, bf16 out[M, N]), EPI_BF16_T
// (bf16 out[N, M]), EPI_F32_RED_T (fp32 out[N, M] +=, split-K) or EPI_F32_RED (fp32 out[M, N] +=).
void gemm_mx8(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, int64_t epi, int64_t bn,
              int64_t splits, const at::Tensor& sfa, const at::Tensor& sfb) {
  CHECK_CUDA(a);
  CHECK_CUDA(b);
  TORCH_CHECK(a.scalar_type() == at::kFloat8_e4m3fn && b.scalar_type() == at::kFloat8_e4m3fn,
              "gemm_mx8: operands must be float8_e4m3fn");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1), "gemm_mx8: bad shapes");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(1) == 1, "gemm_mx8: inner dims");
  TORCH_CHECK(sfa.scalar_type() == at::kByte && sfb.scalar_type() == at::kByte && sfa.is_contiguous() &&
                  sfb.is_contiguous(), "gemm_mx8: scale atoms must be contiguous uint8");
  const int64_t M = a.size(0), N = b.size(0), K = a.size(1);
  TORCH_CHECK(K % 128 == 0 && sfa.numel() >= ((M + 127) / 128) * (K / 128) * 512 &&
                  sfb.numel() >= ((N + 127) / 128) * (K / 128) * 512, "gemm_mx8: scale atoms do not cover the operands");
  const bool f32 = epi == b200::EPI_F32_RED_T || epi == b200::EPI_F32_RED;
  TORCH_CHECK(out.scalar_type() == (f32 ? at::kFloat : at::kBFloat16), "gemm_mx8: output dtype");
  const bool tr = epi == b200::EPI_F32_RED_T || epi == b200::EPI_BF16_T;
  TORCH_CHECK(out.size(0) >= (tr ? N : M) && out.size(1) == (tr ? M : N), "gemm_mx8: output shape");
  const c10::cuda::CUDAGuard guard(a.device());
  b200::GemmArgs g{};
  g.A = a.data_ptr();
  g.B = b.data_ptr();
  g.out = out.data_ptr();
  g.lda = a.stride(0);
  g.ldb = b.stride(0);
  g.ldo = out.stride(0);
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.bn = (int)bn;
  g.epi = (int)epi;
  g.splits = (int)splits;
  g.status = status_word();
  g.fp8 = 1;
  g.w8 = 6;
  g.sfa = sfa.data_ptr<uint8_t>();
  g.sfb = sfb.data_ptr<uint8_t>();
  if (M == 0 || N == 0) return;
  b200::gemm_bf16_launch(g, cur_stream());
  check_launch("gemm_mx8");
}

// Block-scaled FP8 W8A8 prefill GEMM: out[m, n] = sum_k xq[m, k] w[n, k] * xs[m, k / 128] *
// ws[n / 128, k / 128] (bf16 store; tokens as the 128-row operand, 128-wide weight tiles).
void gemm_fp8_block_prefill(const at::Tensor& xq, const at::Tensor& w, at::Tensor& out,
                            const at::Tensor& w_scales, const at::Tensor& x_scales) {
  CHECK_CUDA(w);
  CHECK_CUDA(xq);
  CHECK_BF16(out);
  TORCH_CHECK(w.scalar_type() == at::kFloat8_e4m3fn && xq.scalar_type() == at::kFloat8_e4m3fn,
              "gemm_fp8_block_prefill: operands must be float8_e4m3fn");
  TORCH_CHECK(w.dim() == 2 && xq.dim() == 2 && w.size(1) == xq.size(1), "gemm_fp8_block_prefill: bad shapes");
  TORCH_CHECK(w.stride(1) == 1 && xq.stride(1) == 1 && out.stride(1) == 1, "gemm_fp8_block_prefill: inner dims");
  TORCH_CHECK(w_scales.scalar_type() == at::kFloat && x_scales.scalar_type() == at::kFloat &&
                  w_scales.stride(1) == 1 && x_scales.stride(1) == 1,
              "gemm_fp8_block_prefill: scales must be fp32 with contiguous rows");
  const c10::cuda::CUDAGuard guard(w.device());
  b200::GemmArgs g{};
  g.A = xq.data_ptr();
  g.B = w.data_ptr();
  g.out = out.data_ptr();
  g.lda = xq.stride(0);
  g.ldb = w.stride(0);
  g.ldo = out.stride(0);
  g.M = (int)xq.size(0);
  g.N = (int)w.size(0);
  g.K = (int)w.size(1);
  g.bn = 128;
  g.epi = b200::EPI_BF16;
  g.splits = 1;
  g.status = status_word();
  g.fp8 = 1;
  g.w8 = 5;
  g.w_scales = w_scales.data_ptr<float>();
  g.w_scale_ld = (int)w_scales.stride(0);
  g.w_scale_rows = (int)w_scales.size(0);
  g.x_scales = x_scales.data_ptr<float>();
  g.x_scale_ld = (int)x_scales.stride(0);
  if (g.M == 0 || g.N == 0) return;
  b200::gemm_bf16_launch(g, cur_stream());
  check_launch("gemm_fp8_block_prefill");
}

// FP8 (e4m3) GEMM with per-tensor scales: out = alpha * (a @ b^T) (epilogue as in `gemm`).
void gemm_fp8(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, int64_t epi, int64_t bn,
              int64_t splits, double alpha) {
  CHECK_CUDA(a);
  CHECK_CUDA(b);
  TORCH_CHECK(a.scalar_type() == at::kFloat8_e4m3fn && b.scalar_type() == at::kFloat8_e4m3fn,
              "gemm_fp8: operands must be float8_e4m3fn");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1), "gemm_fp8: bad shapes");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(-1) == 1,
              "gemm_fp8: inner dims must be contiguous");
  const bool f32_out = (epi == b200::EPI_F32_RED || epi == b200::EPI_F32_RED_T);
  TORCH_CHECK(out.scalar_type() == (f32_out ? at::kFloat : at::kBFloat16), "gemm_fp8: out dtype");
  const c10::cuda::CUDAGuard guard(a.device());
  b200::GemmArgs g{};
  g.A = a.data_ptr();
  g.B = b.data_ptr();
  g.out = out.data_ptr();
  g.lda = a.stride(0);
  g.ldb = b.stride(0);
  g.ldo = out.stride(0);
  g.M = (int)a.size(0);
  g.N = (int)b.size(0);
  g.K = (int)a.size(1);
  g.bn = (int)bn;
  g.epi = (int)epi;
  g.splits = (int)splits;
  g.status = status_word();
  g.fp8 = 1;
  g.alpha = (float)alpha;
  if (g.M == 0 || g.N == 0) return;
  b200::gemm_bf16_launch(g, cur_stream());
  check_launch("gemm_fp8");
}

void quant_fp8(const at::Tensor& x, at::Tensor& out, double inv_scale) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  TORCH_CHECK(out.scalar_type() == at::kFloat8_e4m3fn && x.dim() == 2 && out.sizes() == x.sizes() &&
                  x.stride(1) == 1 && out.stride(1) == 1, "quant_fp8: layouts");
  const c10::cuda::CUDAGuard guard(x.device());
  b200::quant_fp8_launch(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
                         reinterpret_cast<uint8_t*>(out.data_ptr()), out.stride(0), (int)x.size(0),
                         (int)x.size(1), (float)inv_scale, cur_stream());
  check_launch("quant_fp8", x.size(0) > 0 ? 1 : 0);
}

void rmsnorm_quant(const at::Tensor& x, const at::Tensor& w, double eps, at::Tensor& out,
                   double inv_scale, c10::optional<at::Tensor> row_scales) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  TORCH_CHECK(out.scalar_type() == at::kFloat8_e4m3fn && x.dim() == 2 && out.sizes() == x.sizes() &&
                  x.stride(1) == 1 && out.stride(1) == 1, "rmsnorm_quant: layouts");
  float* rs = nullptr;
  if (row_scales.has_value()) {
    TORCH_CHECK(row_scales->scalar_type() == at::kFloat && row_scales->numel() >= x.size(0),
                "rmsnorm_quant: row_scales must be fp32 [rows]");
    rs = row_scales->data_ptr<float>();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  b200::rmsnorm_quant_launch(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
                             reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), (float)eps,
                             reinterpret_cast<uint8_t*>(out.data_ptr()), out.stride(0), (int)x.size(0),
                             (int)x.size(1), (float)inv_scale, rs, cur_stream());
  check_launch("rmsnorm_quant", x.size(0) > 0 ? 1 : 0);
}

// Sequence-parallel GEMM: optional all-gather wait on the A rows (ag_ctr != 0: local counter
// array address, ag_targets per source rank, ag_rows rows per rank) and / or the reduce-scatter
// epilogue (epi == EPI_BF16_RS: rs_out / rs_ctr peer addresses per owner rank, rs_rows rows per
// owner; `out` is then only a shape / stride carrier).
void gemm_sp(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, int64_t epi, int64_t bn,
             int64_t ag_ctr, const std::vector<int64_t>& ag_targets, int64_t ag_rows,
             const std::vector<int64_t>& rs_out, const std::vector<int64_t>& rs_ctr, int64_t rs_rows,
             c10::optional<at::Tensor> b_scales) {
  CHECK_CUDA(a);
  CHECK_CUDA(b);
  CHECK_BF16(a);
  // b: bf16 weight, or a block-scaled FP8 weight with its fp32 128 x 128 block scales
  if (b_scales.has_value()) {
    TORCH_CHECK(b.scalar_type() == at::kFloat8_e4m3fn, "gemm_sp: block-FP8 weight must be e4m3");
    TORCH_CHECK(b_scales->scalar_type() == at::kFloat && b_scales->dim() == 2 &&
                    b_scales->stride(1) == 1, "gemm_sp: scales must be fp32 [row blocks, k blocks]");
  } else {
    CHECK_BF16(b);
  }
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1), "gemm_sp: bad shapes");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(-1) == 1,
              "gemm_sp: inner dims must be contiguous");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16, "gemm_sp: bf16 output");
  TORCH_CHECK(ag_targets.size() <= (size_t)b200::kGemmMaxRanks && rs_out.size() == rs_ctr.size() &&
                  rs_out.size() <= (size_t)b200::kGemmMaxRanks, "gemm_sp: too many ranks");
  const c10::cuda::CUDAGuard guard(a.device());
  b200::GemmSPArgs sp{};
  sp.ag_ctr = reinterpret_cast<const unsigned int*>(ag_ctr);
  for (size_t r = 0; r < ag_targets.size(); ++r) sp.ag_target[r] = (unsigned int)ag_targets[r];
  sp.ag_rows = (int)ag_rows;
  sp.ag_world = (int)ag_targets.size();
  for (size_t r = 0; r < rs_out.size(); ++r) {
    sp.rs_out[r] = reinterpret_cast<__nv_bfloat16*>(rs_out[r]);
    sp.rs_ctr[r] = reinterpret_cast<unsigned int*>(rs_ctr[r]);
  }
  sp.rs_rows = (int)rs_rows;
  b200::GemmArgs g{};
  g.A = a.data_ptr();
  g.B = b.data_ptr();
  g.out = out.data_ptr();
  g.lda = a.stride(0);
  g.ldb = b.stride(0);
  g.ldo = out.stride(0);
  g.M = (int)a.size(0);
  g.N = (int)b.size(0);
  g.K = (int)a.size(1);
  g.bn = (int)bn;
  g.epi = (int)epi;
  g.splits = 1;
  g.status = status_word();
  g.sp = &sp;
  if (b_scales.has_value()) {
    g.w8 = 2;
    g.w_scales = b_scales->data_ptr<float>();
    g.w_scale_ld = (int)b_scales->stride(0);
    g.w_scale_rows = (int)b_scales->size(0);
  }
  if (g.M == 0 || g.N == 0) return;
  b200::gemm_bf16_launch(g, cur_stream());
  check_launch("gemm_sp");
}

void sp_norm_push(int64_t slots, int64_t slot_src_stride, int64_t nsrc, int64_t rs_ctr,
                  int64_t rs_target, at::Tensor& residual, const at::Tensor& w, double eps,
                  const std::vector<int64_t>& x_out, const std::vector<int64_t>& ag_ctr) {
  CHECK_CUDA(residual);
  CHECK_BF16(residual);
  CHECK_BF16(w);
  TORCH_CHECK(residual.is_contiguous(), "sp_norm_push: residual rows must be contiguous");
  TORCH_CHECK(x_out.size() == ag_ctr.size() && !x_out.empty() && x_out.size() <= (size_t)b200::kMaxTP,
              "sp_norm_push: rank lists");
  const c10::cuda::CUDAGuard guard(residual.device());
  b200::SPNormPushParams p{};
  p.slots = reinterpret_cast<const __nv_bfloat16*>(slots);
  p.slot_src_stride = slot_src_stride;
  p.nsrc = (int)nsrc;
  p.rs_ctr = reinterpret_cast<const unsigned int*>(rs_ctr);
  p.rs_target = (unsigned int)rs_target;
  p.residual = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  p.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  p.eps = (float)eps;
  fill_ptrs(x_out, (void**)p.x_out, "x_out");
  fill_ptrs(ag_ctr, (void**)p.ag_ctr, "ag_ctr");
  p.world = (int)x_out.size();
  p.rows = (int)residual.size(0);
  p.H = (int)residual.size(1);
  p.status = status_word();
  b200::sp_norm_push_launch(p, cur_stream());
  check_launch("sp_norm_push", p.rows > 0 ? 1 : 0);
}

void sp_wait(int64_t ctr, const std::vector<int64_t>& targets) {
  TORCH_CHECK(!targets.empty() && targets.size() <= (size_t)b200::kMaxTP, "sp_wait: targets");
  unsigned int t[b200::kMaxTP] = {};
  for (size_t r = 0; r < targets.size(); ++r) t[r] = (unsigned int)targets[r];
  b200::sp_wait_launch(reinterpret_cast<const unsigned int*>(ctr), t, (int)targets.size(),
                       status_word(), cur_stream());
  check_launch("sp_wait");
}

void paged_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                     const at::Tensor& block_tables, const at::Tensor& seq_lens,
                     const at::Tensor& q_start, const at::Tensor& work, at::Tensor& out,
                     c10::optional<at::Tensor> part_o, c10::optional<at::Tensor> part_lse,
                     c10::optional<at::Tensor> sinks, int64_t num_splits, int64_t num_kv_heads,
                     int64_t window, double scale, bool decode, double k_scale, double v_scale,
                     c10::optional<at::Tensor> splits_dev, c10::optional<at::Tensor> dcp_seq_lens,
                     int64_t dcp_size, int64_t dcp_rank, bool partial_out, int64_t prefill_rows) {
  CHECK_CUDA(q);
  CHECK_BF16(q);
  const bool fp8 = k_cache.scalar_type() == at::kFloat8_e4m3fn;
  TORCH_CHECK(fp8 || k_cache.scalar_type() == at::kBFloat16,
              "k_cache must be bfloat16 or float8_e4m3fn");
  TORCH_CHECK(v_cache.scalar_type() == k_cache.scalar_type(), "k/v cache dtypes differ");
  TORCH_CHECK(q.dim() == 3, "q must be [T, Hq, D]");
  TORCH_CHECK(k_cache.dim() == 4, "k_cache must be [num_blocks, Hkv, block_size, D]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  q_start.scalar_type() == at::kInt && work.scalar_type() == at::kInt,
              "metadata must be int32");
  TORCH_CHECK(q.stride(2) == 1 && q.stride(1) == q.size(2), "q heads must be packed");
  TORCH_CHECK(out.stride(2) == 1 && out.stride(1) == out.size(2), "out heads must be packed");
  const c10::cuda::CUDAGuard guard(q.device());
  b200::PagedAttnParams p{};
  const int D = (int)q.size(2);
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.q_stride_t = q.stride(0);
  p.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  p.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  p.kv_block_stride = k_cache.stride(0);
  TORCH_CHECK(v_cache.stride(0) == k_cache.stride(0), "k/v cache strides differ");
  p.block_tables = block_tables.data_ptr<int>();
  p.bt_stride = (int)block_tables.stride(0);
  p.seq_lens = seq_lens.data_ptr<int>();
  p.q_start = q_start.data_ptr<int>();
  p.work = reinterpret_cast<const int2*>(work.data_ptr<int>());
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.o_stride_t = out.stride(0);
  p.num_splits = (int)num_splits;
  p.partial_out = partial_out ? 1 : 0;
  p.prefill_rows = (int)prefill_rows;
  if (num_splits > 1 || partial_out) {
    TORCH_CHECK(part_o.has_value() && part_lse.has_value(), "split-KV needs partial buffers");
    TORCH_CHECK(part_o->scalar_type() == at::kFloat && part_lse->scalar_type() == at::kFloat,
                "partials must be float32");
    TORCH_CHECK(part_lse->numel() >= num_splits * q.size(0) * q.size(1), "part_lse too small");
    TORCH_CHECK(part_o->numel() >= num_splits * q.size(0) * q.size(1) * D, "part_o too small");
    p.part_o = part_o->data_ptr<float>();
    p.part_lse = part_lse->data_ptr<float>();
  }
  p.sinks = sinks.has_value() ? sinks->data_ptr<float>() : nullptr;
  p.Hq = (int)q.size(1);
  p.Hkv = (int)num_kv_heads;
  p.G = p.Hq / p.Hkv;
  p.block_size = (int)k_cache.size(2);
  p.window = (int)window;
  p.scale_log2 = (float)(scale * 1.4426950408889634 * (fp8 ? k_scale : 1.0));
  p.kv_fp8 = fp8 ? 1 : 0;
  p.v_scale = fp8 ? (float)v_scale : 1.f;
  if (splits_dev.has_value()) {
    TORCH_CHECK(splits_dev->scalar_type() == at::kInt && splits_dev->is_cuda(), "splits_dev must be int32 CUDA");
    p.splits_dev = splits_dev->data_ptr<int>();
  }
  if (dcp_seq_lens.has_value()) {
    TORCH_CHECK(dcp_seq_lens->scalar_type() == at::kInt && dcp_seq_lens->is_cuda(),
                "dcp_seq_lens must be int32 CUDA");
    TORCH_CHECK(dcp_size >= 1 && dcp_rank >= 0 && dcp_rank < dcp_size, "bad DCP rank / size");
    TORCH_CHECK(window == 0 && !sinks.has_value(),
                "decode context parallelism supports neither sliding windows nor sinks");
    p.dcp_seq_lens = dcp_seq_lens->data_ptr<int>();
    p.dcp_size = (int)dcp_size;
    p.dcp_rank = (int)dcp_rank;
  }
  p.total_tokens = (int)q.size(0);
  p.status = status_word();
  if (k_cache.is_contiguous() && v_cache.is_contiguous()) {
    // rows of the caches: the TMA maps' extent and the kernels' block-id bound
    p.kv_rows = k_cache.size(0) * k_cache.size(1) * k_cache.size(2);
    p.sched = decode_sched_words();
  }
  const int num_work = (int)work.size(0);
  b200::paged_attention_launch(p, num_work, D, decode, cur_stream());
  check_launch("paged_attention", num_work == 0 ? 0 : (num_splits > 1 && !partial_out ? 2 : 1));
}

// Merge split partials part_o [S, T, Hq, D] / part_lse [S, T, Hq] into out [T, Hq, D] bf16.
void attn_combine(const at::Tensor& part_o, const at::Tensor& part_lse, at::Tensor& out) {
  CHECK_CUDA(part_o);
  CHECK_BF16(out);
  TORCH_CHECK(part_o.scalar_type() == at::kFloat && part_lse.scalar_type() == at::kFloat,
              "partials must be float32");
  TORCH_CHECK(part_o.dim() == 4 && part_o.is_contiguous() && part_lse.is_contiguous(),
              "part_o must be a contiguous [S, T, Hq, D] tensor");
  TORCH_CHECK(out.dim() == 3 && out.stride(2) == 1 && out.stride(1) == out.size(2),
              "out heads must be packed");
  const int S = (int)part_o.size(0), T = (int)part_o.size(1), Hq = (int)part_o.size(2),
            D = (int)part_o.size(3);
  TORCH_CHECK(out.size(0) == T && out.size(1) == Hq && out.size(2) == D, "out shape mismatch");
  TORCH_CHECK(part_lse.numel() == (int64_t)S * T * Hq, "part_lse shape mismatch");
  const c10::cuda::CUDAGuard guard(part_o.device());
  b200::attn_combine_launch(part_o.data_ptr<float>(), part_lse.data_ptr<float>(),
                            reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), T, Hq,
                            S, D, cur_stream());
  check_launch("attn_combine");
}

void add_rmsnorm(at::Tensor& x, c10::optional<at::Tensor> residual, const at::Tensor& w,
                 at::Tensor& out, double eps, bool clear_x) {
  CHECK_CUDA(x);
  const c10::cuda::CUDAGuard guard(x.device());
  const int rows = (int)x.size(0), H = (int)x.size(1);
  TORCH_CHECK(x.stride(1) == 1 && out.stride(1) == 1, "rows must be contiguous");
  __nv_bfloat16* res = nullptr;
  long long rs = 0;
  if (residual.has_value()) {
    CHECK_BF16(*residual);
    res = reinterpret_cast<__nv_bfloat16*>(residual->data_ptr());
    rs = residual->stride(0);
  }
  b200::add_rmsnorm_launch(x.data_ptr(), x.scalar_type() == at::kFloat, x.stride(0), res, rs,
                           reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                           reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), rows,
                           H, (float)eps, clear_x, cur_stream());
  check_launch("add_rmsnorm");
}

void rope_kv_write(at::Tensor& qkv, const at::Tensor& positions,
                   c10::optional<at::Tensor> slot_mapping, const at::Tensor& cos_sin,
                   at::Tensor& q_out, c10::optional<at::Tensor> k_cache,
                   c10::optional<at::Tensor> v_cache, c10::optional<at::Tensor> q_norm_w,
                   c10::optional<at::Tensor> k_norm_w, double eps, int64_t num_q_heads,
                   int64_t num_kv_heads, int64_t head_dim, int64_t rot_dim, bool neox,
                   bool clear_input, double q_pos_beta, double q_pos_period,
                   c10::optional<at::Tensor> qkv_bias, c10::optional<at::Tensor> positions3,
                   int64_t mrope_h, int64_t mrope_w, double k_scale, double v_scale) {
  CHECK_CUDA(qkv);
  TORCH_CHECK(q_pos_beta == 0.0 || q_pos_period > 0.0, "rope_kv_write: q_pos_period must be positive");
  const c10::cuda::CUDAGuard guard(qkv.device());
  b200::RopeKvParams p{};
  p.positions = positions.data_ptr<int>();
  if (slot_mapping.has_value())
    TORCH_CHECK(slot_mapping->scalar_type() == at::kInt, "slot_mapping must be int32");
  p.slot_mapping = slot_mapping.has_value() ? slot_mapping->data_ptr<int>() : nullptr;
  p.cos_sin = cos_sin.data_ptr<float>();
  p.qkv_stride = qkv.stride(0);
  p.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  p.q_out_stride = q_out.stride(0);
  if (k_cache.has_value()) {
    p.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache->data_ptr());
    p.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache->data_ptr());
    p.kv_block_stride = k_cache->stride(0);
    p.block_size = (int)k_cache->size(2);
    p.num_blocks = k_cache->size(0);
    p.status = status_word();
    const bool fp8 = k_cache->scalar_type() == at::kFloat8_e4m3fn;
    TORCH_CHECK(fp8 || k_cache->scalar_type() == at::kBFloat16,
                "rope_kv_write: cache must be bfloat16 or float8_e4m3fn");
    TORCH_CHECK(v_cache->scalar_type() == k_cache->scalar_type(), "k/v cache dtypes differ");
    TORCH_CHECK(!fp8 || (k_scale > 0.0 && v_scale > 0.0), "fp8 KV scales must be positive");
    p.kv_fp8 = fp8 ? 1 : 0;
    p.k_inv_scale = fp8 ? (float)(1.0 / k_scale) : 1.f;
    p.v_inv_scale = fp8 ? (float)(1.0 / v_scale) : 1.f;
  } else {
    p.slot_mapping = nullptr;
    p.block_size = 1;
  }
  p.q_norm_w = q_norm_w.has_value() ? reinterpret_cast<const __nv_bfloat16*>(q_norm_w->data_ptr()) : nullptr;
  p.k_norm_w = k_norm_w.has_value() ? reinterpret_cast<const __nv_bfloat16*>(k_norm_w->data_ptr()) : nullptr;
  p.eps = (float)eps;
  p.Hq = (int)num_q_heads;
  p.Hkv = (int)num_kv_heads;
  p.head_dim = (int)head_dim;
  p.rot_dim = (int)rot_dim;
  p.neox = neox;
  p.clear_input = clear_input;
  if (qkv_bias.has_value()) {
    TORCH_CHECK(qkv_bias->scalar_type() == at::kFloat && qkv_bias->is_contiguous() &&
                    qkv_bias->numel() == (num_q_heads + 2 * num_kv_heads) * head_dim,
                "rope_kv_write: qkv_bias must be fp32 [(Hq + 2 Hkv) * D]");
    p.qkv_bias = qkv_bias->data_ptr<float>();
  }
  if (positions3.has_value()) {
    TORCH_CHECK(positions3->scalar_type() == at::kInt && positions3->is_contiguous() &&
                    positions3->dim() == 2 && positions3->size(1) == 3,
                "rope_kv_write: positions3 must be int32 [T, 3]");
    p.positions3 = positions3->data_ptr<int>();
    p.mrope_h = (int)mrope_h;
    p.mrope_w = (int)mrope_w;
  }
  p.q_pos_beta = (float)q_pos_beta;
  p.q_pos_period = (float)(q_pos_period > 0.0 ? q_pos_period : 1.0);
  b200::rope_kv_write_launch(p, qkv.data_ptr(), qkv.scalar_type() == at::kFloat,
                             (int)qkv.size(0), cur_stream());
  check_launch("rope_kv_write");
}

void silu_mul(at::Tensor& inp, at::Tensor& out, int64_t blk, bool clear_input, int64_t act,
              double limit, double alpha) {
  CHECK_CUDA(inp);
  const c10::cuda::CUDAGuard guard(inp.device());
  const int T = (int)inp.size(0), I = (int)out.size(1);
  TORCH_CHECK(inp.size(1) == 2 * I, "silu_mul: input must have 2 * I columns");
  b200::silu_mul_launch(inp.data_ptr(), inp.scalar_type() == at::kFloat, inp.stride(0),
                        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), T, I,
                        (int)blk, clear_input, (int)act, (float)limit, (float)alpha,
                        cur_stream());
  check_launch("silu_mul");
}

void embedding(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out,
               int64_t vocab_start, int64_t vocab_end, c10::optional<at::Tensor> last_tok) {
  CHECK_CUDA(ids);
  TORCH_CHECK(ids.scalar_type() == at::kInt, "ids must be int32");
  const c10::cuda::CUDAGuard guard(ids.device());
  b200::embedding_launch(ids.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
                         reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (int)ids.size(0),
                         (int)table.size(1), (int)vocab_start, (int)vocab_end,
                         last_tok.has_value() ? last_tok->data_ptr<int>() : nullptr, cur_stream());
  check_launch("embedding");
}

void sample(const at::Tensor& logits, const at::Tensor& temperature, const at::Tensor& top_k,
            const at::Tensor& top_p, c10::optional<at::Tensor> min_p, const at::Tensor& seeds,
            const at::Tensor& offsets, at::Tensor& out_tokens,
            c10::optional<at::Tensor> out_logprob, int64_t vocab_offset,
            c10::optional<at::Tensor> row_slots, c10::optional<at::Tensor> last_tok) {
  CHECK_CUDA(logits);
  const c10::cuda::CUDAGuard guard(logits.device());
  b200::SampleParams p{};
  p.logits = logits.data_ptr();
  p.logits_f32 = logits.scalar_type() == at::kFloat;
  p.logits_stride = logits.stride(0);
  p.B = (int)logits.size(0);
  p.V = (int)logits.size(1);
  p.temperature = temperature.data_ptr<float>();
  p.top_k = top_k.data_ptr<int>();
  p.top_p = top_p.data_ptr<float>();
  p.min_p = min_p.has_value() ? min_p->data_ptr<float>() : nullptr;
  p.seeds = reinterpret_cast<const uint64_t*>(seeds.data_ptr<int64_t>());
  p.offsets = offsets.data_ptr<int>();
  p.out_tokens = out_tokens.data_ptr<int>();
  p.out_logprob = out_logprob.has_value() ? out_logprob->data_ptr<float>() : nullptr;
  p.vocab_offset = (int)vocab_offset;
  if (row_slots.has_value()) {
    TORCH_CHECK(last_tok.has_value(), "row_slots needs last_tok");
    p.row_slots = row_slots->data_ptr<int>();
    p.last_tok = last_tok->data_ptr<int>();
  }
  b200::sample_launch(p, cur_stream());
  check_launch("sample");
}

void argmax(const at::Tensor& logits, at::Tensor& out_idx, c10::optional<at::Tensor> out_val,
            int64_t vocab_offset) {
  CHECK_CUDA(logits);
  const c10::cuda::CUDAGuard guard(logits.device());
  b200::argmax_launch(logits.data_ptr(), logits.scalar_type() == at::kFloat, logits.stride(0),
                      (int)logits.size(0), (int)logits.size(1), out_idx.data_ptr<int>(),
                      out_val.has_value() ? out_val->data_ptr<float>() : nullptr,
                      (int)vocab_offset, cur_stream());
  check_launch("argmax");
}

// ---------------------------------------------------------------- symmetric memory / TP
py::tuple symm_alloc(int64_t nbytes) {
  std::string h;
  void* p = b200::symm_alloc((size_t)nbytes, &h);
  return py::make_tuple((int64_t)p, py::bytes(h));
}
int64_t symm_open(py::bytes handle) { return (int64_t)b200::symm_open(std::string(handle)); }
void symm_close(int64_t p) { b200::symm_close((void*)p); }
void symm_free(int64_t p) { b200::symm_free((void*)p); }

// Non-owning tensor over device memory (e.g. a mapped peer buffer).
at::Tensor tensor_from_ptr(int64_t ptr, std::vector<int64_t> shape, at::ScalarType dtype,
                           int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, device);
  return at::from_blob((void*)ptr, shape, [](void*) {}, opts);
}

static void fill_ptrs(const std::vector<int64_t>& v, void** dst, const char* what) {
  TORCH_CHECK((int)v.size() <= b200::kMaxTP, what, ": at most 8 ranks");
  for (size_t i = 0; i < v.size(); ++i) dst[i] = (void*)v[i];
}

// residual += all_reduce(acc) over the TP group (one-shot push through symmetric peer
// memory), out = rmsnorm(residual) * w; acc is cleared.
void tp_allreduce_norm(at::Tensor& acc, const std::vector<int64_t>& recv_ptrs,
                       const std::vector<int64_t>& flag_ptrs, at::Tensor& state, at::Tensor& residual,
                       const at::Tensor& w, at::Tensor& out, double eps, int64_t rank,
                       int64_t max_rows, int64_t algo) {
  CHECK_CUDA(acc);
  TORCH_CHECK(acc.scalar_type() == at::kFloat, "acc must be fp32");
  CHECK_BF16(residual);
  CHECK_BF16(out);
  TORCH_CHECK(recv_ptrs.size() == flag_ptrs.size(), "recv/flag pointer lists differ");
  TORCH_CHECK(acc.stride(1) == 1 && residual.stride(1) == 1 && out.stride(1) == 1,
              "rows must be contiguous");
  TORCH_CHECK(acc.stride(0) % 4 == 0, "acc row stride must be a multiple of 4");
  const c10::cuda::CUDAGuard guard(acc.device());
  b200::TPArNormParams p{};
  p.acc = acc.data_ptr<float>();
  p.acc_stride = acc.stride(0);
  fill_ptrs(recv_ptrs, (void**)p.recv_peers, "recv");
  fill_ptrs(flag_ptrs, (void**)p.flag_peers, "flags");
  TORCH_CHECK(state.scalar_type() == at::kLong && state.numel() >= 4, "state must be int64[4]");
  p.state = (unsigned long long*)state.data_ptr<int64_t>();
  p.residual = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  p.res_stride = residual.stride(0);
  p.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.out_stride = out.stride(0);
  p.status = status_word();
  p.eps = (float)eps;
  p.rank = (int)rank;
  p.world = (int)recv_ptrs.size();
  p.max_rows = (int)max_rows;
  p.H = (int)acc.size(1);
  p.T = (int)acc.size(0);
  TORCH_CHECK(algo == 0 || algo == 1, "tp_allreduce_norm: algo 0 (sentinel) or 1 (flags)");
  p.algo = (int)algo;
  b200::tp_allreduce_norm_launch(p, cur_stream());
  check_launch("tp_allreduce_norm", p.T > 0 ? 1 : 0);
}

// ------------------------------------------------------------------------- EP exchange
// One stage of the device-side expert-parallel exchange (ep_fused.cu): 0 dispatch, 1 receive,
// 2 return, 3 combine.  `offs` = byte offsets (ctrl, rows, ids, w, src, comb) of the symmetric
// layout, `dims` = (rank, world, H, k, num_experts, e_local, tokens_cap, rows_cap, T).
void ep_exchange(int64_t stage, const std::vector<int64_t>& peers, const std::vector<int64_t>& offs,
                 const std::vector<int64_t>& dims, c10::optional<at::Tensor> x,
                 c10::optional<at::Tensor> topk_ids, c10::optional<at::Tensor> topk_w,
                 c10::optional<at::Tensor> out, c10::optional<at::Tensor> y, at::Tensor& recv_count,
                 at::Tensor& ctas_done, at::Tensor& state) {
  TORCH_CHECK(offs.size() == 6 && dims.size() == 9, "ep_exchange: bad layout arguments");
  TORCH_CHECK(peers.size() == (size_t)dims[1] && dims[1] <= b200::kMaxEP, "ep_exchange: peers");
  CHECK_CUDA(recv_count);
  TORCH_CHECK(recv_count.scalar_type() == at::kInt && ctas_done.scalar_type() == at::kInt &&
                  state.scalar_type() == at::kLong, "ep_exchange: control tensor dtypes");
  const c10::cuda::CUDAGuard guard(recv_count.device());
  b200::EPExchangeParams p{};
  for (size_t r = 0; r < peers.size(); ++r) p.peers[r] = (void*)peers[r];
  p.off_ctrl = offs[0];
  p.off_rows = offs[1];
  p.off_ids = offs[2];
  p.off_w = offs[3];
  p.off_src = offs[4];
  p.off_comb = offs[5];
  p.rank = (int)dims[0];
  p.world = (int)dims[1];
  p.H = (int)dims[2];
  p.k = (int)dims[3];
  p.num_experts = (int)dims[4];
  p.e_local = (int)dims[5];
  p.tokens_cap = (int)dims[6];
  p.rows_cap = (int)dims[7];
  p.T = (int)dims[8];
  p.recv_count = recv_count.data_ptr<int>();
  p.ctas_done = reinterpret_cast<unsigned int*>(ctas_done.data_ptr<int>());
  p.state = (unsigned long long*)state.data_ptr<int64_t>();
  p.status = status_word();
  if (stage == 0 || stage == 3) {
    TORCH_CHECK(topk_ids.has_value() && topk_ids->scalar_type() == at::kInt && topk_ids->is_contiguous() &&
                    topk_ids->size(-1) == p.k && topk_ids->size(0) >= p.T,
                "ep_exchange: topk_ids int32 [T, k]");
    p.topk_ids = topk_ids->data_ptr<int>();
  }
  if (stage == 0) {
    TORCH_CHECK(x.has_value() && topk_w.has_value(), "ep_exchange: dispatch needs x and weights");
    CHECK_BF16(x.value());
    TORCH_CHECK(x->stride(1) == 1 && x->stride(0) % 8 == 0 && x->size(1) == p.H && x->size(0) >= p.T,
                "ep_exchange: x [T, H]");
    TORCH_CHECK(topk_w->scalar_type() == at::kFloat && topk_w->is_contiguous(), "ep_exchange: weights");
    p.x = reinterpret_cast<const __nv_bfloat16*>(x->data_ptr());
    p.ldx = x->stride(0);
    p.topk_w = topk_w->data_ptr<float>();
    b200::ep_dispatch_launch(p, cur_stream());
  } else if (stage == 1) {
    b200::ep_recv_launch(p, cur_stream());
  } else if (stage == 2) {
    TORCH_CHECK(y.has_value(), "ep_exchange: return needs y");
    CHECK_BF16(y.value());
    TORCH_CHECK(y->stride(1) == 1 && y->stride(0) % 8 == 0 && y->size(1) == p.H && y->size(0) >= p.rows_cap,
                "ep_exchange: y [rows_cap, H]");
    p.y = reinterpret_cast<const __nv_bfloat16*>(y->data_ptr());
    p.ldy = y->stride(0);
    b200::ep_return_launch(p, cur_stream());
  } else if (stage == 3) {
    TORCH_CHECK(out.has_value(), "ep_exchange: combine needs out");
    CHECK_BF16(out.value());
    TORCH_CHECK(out->stride(1) == 1 && out->stride(0) % 8 == 0 && out->size(1) == p.H && out->size(0) >= p.T,
                "ep_exchange: out [T, H]");
    p.out = reinterpret_cast<__nv_bfloat16*>(out->data_ptr());
    p.ldo = out->stride(0);
    b200::ep_combine_launch(p, cur_stream());
  } else {
    TORCH_CHECK(false, "ep_exchange: stage 0..3");
  }
  check_launch("ep_exchange");
}

// ------------------------------------------------------------------------------ MoE
// out[rows of expert e] = x_perm[rows] @ w[e]^T for the tile list written by moe_align.
// x_perm [R, K] bf16 (expert-sorted rows), w [E_local, N, K] bf16, out [R, N] (bf16) with the
// EPI_BF16 or EPI_SILU_BF16 epilogue.
void gemm_grouped(const at::Tensor& x_perm, const at::Tensor& w, at::Tensor& out,
                  const at::Tensor& gtiles, const at::Tensor& gcount, int64_t epi, int64_t bn) {
  CHECK_CUDA(x_perm);
  CHECK_BF16(x_perm);
  CHECK_BF16(w);
  CHECK_BF16(out);
  TORCH_CHECK(w.dim() == 3 && w.is_contiguous() && w.size(2) == x_perm.size(1), "gemm_grouped: w");
  TORCH_CHECK(x_perm.stride(1) == 1 && out.stride(1) == 1, "gemm_grouped: inner dims");
  TORCH_CHECK(gtiles.scalar_type() == at::kInt && gtiles.is_contiguous() && gtiles.size(-1) == 4,
              "gemm_grouped: gtiles must be int32 [n, 4]");
  TORCH_CHECK(epi == b200::EPI_BF16 || epi == b200::EPI_SILU_BF16, "gemm_grouped: epilogue");
  const c10::cuda::CUDAGuard guard(x_perm.device());
  b200::GemmArgs g{};
  g.A = x_perm.data_ptr();
  g.B = w.data_ptr();
  g.out = out.data_ptr();
  g.lda = x_perm.stride(0);
  g.ldb = w.stride(1);
  g.ldo = out.stride(0);
  g.M = (int)x_perm.size(0);
  g.N = (int)w.size(1);
  g.K = (int)w.size(2);
  g.bn = (int)bn;
  g.epi = (int)epi;
  g.splits = 1;
  g.status = status_word();
  g.gtiles = gtiles.data_ptr<int>();
  g.gcount = gcount.data_ptr<int>();
  g.gmax = (int)gtiles.size(0);
  g.num_groups = (int)w.size(0);
  b200::gemm_bf16_launch(g, cur_stream());
  check_launch("gemm_grouped");
}

void moe_route(const at::Tensor& logits, c10::optional<at::Tensor> bias, int64_t num_experts,
               int64_t k, int64_t mode, bool renorm, at::Tensor& ids, at::Tensor& weights,
               c10::optional<at::Tensor> shared_gate, double scale) {
  CHECK_CUDA(logits);
  CHECK_BF16(logits);
  TORCH_CHECK(logits.stride(1) == 1, "moe_route: logits rows must be contiguous");
  TORCH_CHECK(ids.scalar_type() == at::kInt && weights.scalar_type() == at::kFloat, "moe_route: out dtypes");
  const c10::cuda::CUDAGuard guard(logits.device());
  const float* b = nullptr;
  if (bias.has_value()) {
    TORCH_CHECK(bias->scalar_type() == at::kFloat, "moe_route: bias must be fp32");
    b = bias->data_ptr<float>();
  }
  b200::moe_route_launch(reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
                         b, (int)logits.size(0), (int)num_experts, (int)k, (int)mode, renorm,
                         ids.data_ptr<int>(), weights.data_ptr<float>(),
                         shared_gate.has_value() ? shared_gate->data_ptr<float>() : nullptr,
                         (float)scale, cur_stream());
  check_launch("moe_route", logits.size(0) > 0 ? 1 : 0);
}

// Fused router GEMV + top-k for decode batches: x [T, H], w [rows, H] (rows = E, or E + 1 with
// the shared-expert gate row), logits [T, >= rows] bf16 output.
void moe_router_topk(const at::Tensor& x, const at::Tensor& w, c10::optional<at::Tensor> bias,
                     int64_t num_experts, int64_t k, int64_t mode, bool renorm, double scale,
                     at::Tensor& logits, at::Tensor& ids, at::Tensor& weights,
                     c10::optional<at::Tensor> shared_gate) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  CHECK_BF16(logits);
  TORCH_CHECK(x.stride(1) == 1 && w.is_contiguous() && logits.stride(1) == 1, "moe_router_topk: layouts");
  TORCH_CHECK(ids.scalar_type() == at::kInt && weights.scalar_type() == at::kFloat, "moe_router_topk: out dtypes");
  const c10::cuda::CUDAGuard guard(x.device());
  const float* b = nullptr;
  if (bias.has_value()) {
    TORCH_CHECK(bias->scalar_type() == at::kFloat, "moe_router_topk: bias must be fp32");
    b = bias->data_ptr<float>();
  }
  b200::moe_router_topk_launch(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
                               reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), (int)w.size(0),
                               (int)x.size(1), b, (int)x.size(0), (int)num_experts, (int)k, (int)mode,
                               renorm, (float)scale, reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()),
                               logits.stride(0), ids.data_ptr<int>(), weights.data_ptr<float>(),
                               shared_gate.has_value() ? shared_gate->data_ptr<float>() : nullptr,
                               cur_stream());
  check_launch("moe_router_topk", x.size(0) > 0 ? 1 : 0);
}

void moe_align(const at::Tensor& ids, int64_t e_start, int64_t e_local, at::Tensor& offsets,
               at::Tensor& sorted_src, at::Tensor& row_expert, at::Tensor& inv_pos,
               at::Tensor& gtiles, at::Tensor& gcount) {
  CHECK_CUDA(ids);
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous(), "moe_align: ids int32");
  const c10::cuda::CUDAGuard guard(ids.device());
  b200::moe_align_launch(ids.data_ptr<int>(), (int)ids.numel(), (int)e_start, (int)e_local,
                         offsets.data_ptr<int>(), sorted_src.data_ptr<int>(),
                         row_expert.data_ptr<int>(), inv_pos.data_ptr<int>(), gtiles.data_ptr<int>(),
                         gcount.data_ptr<int>(), (int)gtiles.size(0), cur_stream());
  check_launch("moe_align");
}

void moe_gather(const at::Tensor& x, const at::Tensor& sorted_src, int64_t topk,
                const at::Tensor& offsets, at::Tensor& out) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  TORCH_CHECK(x.stride(1) == 1 && out.is_contiguous(), "moe_gather: layouts");
  const c10::cuda::CUDAGuard guard(x.device());
  const int e_local = (int)offsets.numel() - 1;
  b200::moe_gather_launch(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
                          sorted_src.data_ptr<int>(), (int)topk, offsets.data_ptr<int>() + e_local,
                          (int)out.size(0), (int)x.size(1),
                          reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), cur_stream());
  check_launch("moe_gather", out.size(0) > 0 ? 1 : 0);
}

void moe_act(const at::Tensor& gu, c10::optional<at::Tensor> bias, const at::Tensor& row_expert,
             const at::Tensor& offsets, int64_t mode, double alpha, double limit, at::Tensor& out) {
  CHECK_CUDA(gu);
  CHECK_BF16(gu);
  TORCH_CHECK(gu.is_contiguous() && out.is_contiguous(), "moe_act: layouts");
  const c10::cuda::CUDAGuard guard(gu.device());
  const __nv_bfloat16* b = nullptr;
  if (bias.has_value()) {
    CHECK_BF16(*bias);
    b = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  const int e_local = (int)offsets.numel() - 1;
  b200::moe_act_launch(reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), b,
                       row_expert.data_ptr<int>(), offsets.data_ptr<int>() + e_local,
                       (int)out.size(0), (int)out.size(1), (int)mode, (float)alpha, (float)limit,
                       reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), cur_stream());
  check_launch("moe_act", out.size(0) > 0 ? 1 : 0);
}

void moe_combine(const at::Tensor& y, const at::Tensor& inv_pos, const at::Tensor& weights,
                 const at::Tensor& ids, c10::optional<at::Tensor> bias, int64_t e_start,
                 c10::optional<at::Tensor> shared, c10::optional<at::Tensor> shared_gate,
                 at::Tensor& out) {
  CHECK_CUDA(y);
  CHECK_BF16(y);
  CHECK_BF16(out);
  TORCH_CHECK(y.stride(1) == 1 && y.stride(0) >= out.size(1) && out.stride(1) == 1, "moe_combine: layouts");
  const c10::cuda::CUDAGuard guard(y.device());
  const __nv_bfloat16* b = nullptr;
  if (bias.has_value()) {
    CHECK_BF16(*bias);
    b = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  const int T = (int)out.size(0);
  b200::moe_combine_launch(reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), inv_pos.data_ptr<int>(),
                           weights.data_ptr<float>(), ids.data_ptr<int>(), b, (int)e_start, T,
                           (int)ids.size(1), (int)out.size(1),
                           shared.has_value() ? reinterpret_cast<const __nv_bfloat16*>(shared->data_ptr()) : nullptr,
                           shared.has_value() ? shared->stride(0) : 0,
                           shared_gate.has_value() ? shared_gate->data_ptr<float>() : nullptr,
                           reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0),
                           cur_stream(), y.stride(0));
  check_launch("moe_combine", T > 0 ? 1 : 0);
}

// ------------------------------------------------------------------------- DeltaNet
static b200::LinearAttnBatch linear_batch(const at::Tensor& q_start, const at::Tensor& seq_lens,
                                          const at::Tensor& slots) {
  TORCH_CHECK(q_start.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  slots.scalar_type() == at::kInt,
              "batch metadata must be int32");
  b200::LinearAttnBatch b{};
  b.q_start = q_start.data_ptr<int>();
  b.seq_lens = seq_lens.data_ptr<int>();
  b.slots = slots.data_ptr<int>();
  b.B = (int)seq_lens.size(0);
  return b;
}

void causal_conv1d(const at::Tensor& x, const at::Tensor& w, const at::Tensor& q_start,
                   const at::Tensor& seq_lens, const at::Tensor& slots, at::Tensor& state,
                   at::Tensor& y) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  CHECK_BF16(state);
  CHECK_BF16(y);
  TORCH_CHECK(x.stride(1) == 1 && y.stride(1) == 1 && w.is_contiguous(), "causal_conv1d: layouts");
  TORCH_CHECK(state.dim() == 3 && state.size(1) == x.size(1) && state.size(2) == w.size(1) - 1 &&
                  state.stride(2) == 1 && state.stride(1) == state.size(2),
              "causal_conv1d: state must be [slots, C, K - 1]");
  const c10::cuda::CUDAGuard guard(x.device());
  b200::causal_conv1d_launch(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
                             (int)x.size(1), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                             (int)w.size(1), linear_batch(q_start, seq_lens, slots),
                             reinterpret_cast<__nv_bfloat16*>(state.data_ptr()), state.stride(0),
                             reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), y.stride(0), cur_stream());
  check_launch("causal_conv1d", seq_lens.size(0) > 0 ? 1 : 0);
}

void gated_delta_rule(const at::Tensor& qkv, const at::Tensor& z, const at::Tensor& a,
                      const at::Tensor& b, const at::Tensor& A_log, const at::Tensor& dt_bias,
                      const at::Tensor& norm_w, double eps, const at::Tensor& q_start,
                      const at::Tensor& seq_lens, const at::Tensor& slots, at::Tensor& state,
                      at::Tensor& out, int64_t Hk, int64_t Hv, int64_t mode) {
  CHECK_CUDA(qkv);
  CHECK_BF16(qkv);
  CHECK_BF16(z);
  CHECK_BF16(out);
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.dim() == 4 && state.is_contiguous(),
              "gated_delta_rule: state must be fp32 [slots, Hv, dk, dv]");
  TORCH_CHECK(z.stride(0) == a.stride(0) && z.stride(0) == b.stride(0), "z, a, b must share a row stride");
  const c10::cuda::CUDAGuard guard(qkv.device());
  b200::GatedDeltaParams p{};
  p.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  p.ld_qkv = qkv.stride(0);
  p.z = reinterpret_cast<const __nv_bfloat16*>(z.data_ptr());
  p.a = reinterpret_cast<const __nv_bfloat16*>(a.data_ptr());
  p.b = reinterpret_cast<const __nv_bfloat16*>(b.data_ptr());
  p.ld_zab = z.stride(0);
  p.A_log = A_log.data_ptr<float>();
  p.dt_bias = dt_bias.data_ptr<float>();
  p.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w.data_ptr());
  p.eps = (float)eps;
  p.state = state.data_ptr<float>();
  p.state_slot_stride = state.stride(0);
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ld_out = out.stride(0);
  p.Hk = (int)Hk;
  p.Hv = (int)Hv;
  p.dk = (int)state.size(2);
  p.dv = (int)state.size(3);
  p.T = (int)out.size(0);
  at::Tensor gb = at::empty({std::max<int64_t>(p.T, 1), Hv, 4}, qkv.options().dtype(at::kFloat));
  p.gb = reinterpret_cast<float4*>(gb.data_ptr<float>());
  const int64_t B = seq_lens.size(0);
  // mode 0: chunked for prefill-sized steps (at least 128 tokens, 2 per sequence on average),
  // recurrent otherwise; 1: recurrent; 2: chunked
  const bool chunked = mode == 2 || (mode == 0 && p.T >= 128 && p.T >= 2 * B);
  if (chunked && B > 0 && p.T > 0) {
    const int64_t max_chunks = p.T / 64 + B;
    const auto f32 = qkv.options().dtype(at::kFloat);
    at::Tensor W = at::empty({p.T, Hv, 128}, f32), U = at::empty({p.T, Hv, 128}, f32);
    at::Tensor QKm = at::empty({max_chunks, Hv, 64, 64}, f32), lg = at::empty({p.T, Hv}, f32);
    at::Tensor chunks = at::empty({max_chunks, 4}, qkv.options().dtype(at::kInt));
    at::Tensor seq0 = at::empty({B + 1}, qkv.options().dtype(at::kInt));
    b200::GdnChunkScratch cs{W.data_ptr<float>(), U.data_ptr<float>(), QKm.data_ptr<float>(),
                             lg.data_ptr<float>(), reinterpret_cast<int4*>(chunks.data_ptr<int>()),
                             seq0.data_ptr<int>(), (int)max_chunks};
    b200::gated_delta_rule_chunked_launch(p, linear_batch(q_start, seq_lens, slots), cs, cur_stream());
    // norms / gates, chunk table, per-chunk solve, state pass, gated RMSNorm
    check_launch("gated_delta_rule", 5);
    return;
  }
  b200::gated_delta_rule_launch(p, linear_batch(q_start, seq_lens, slots), cur_stream());
  // normalisation / gates pass, recurrence, gated RMSNorm
  check_launch("gated_delta_rule", B > 0 ? (p.T > 0 ? 3 : 1) : 0);
}

void sigmoid_gate_mul(at::Tensor& x, const at::Tensor& gate) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(gate);
  TORCH_CHECK(x.stride(1) == 1 && gate.stride(1) == 1 && x.sizes() == gate.sizes(), "sigmoid_gate_mul: layouts");
  const c10::cuda::CUDAGuard guard(x.device());
  b200::sigmoid_gate_mul_launch(reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), x.stride(0),
                                reinterpret_cast<const __nv_bfloat16*>(gate.data_ptr()), gate.stride(0),
                                (int)x.size(0), (int)x.size(1), cur_stream());
  check_launch("sigmoid_gate_mul", x.size(0) > 0 ? 1 : 0);
}

void apply_token_bitmask(at::Tensor& logits, const at::Tensor& mask) {
  CHECK_CUDA(logits);
  CHECK_BF16(logits);
  TORCH_CHECK(mask.scalar_type() == at::kInt && mask.is_contiguous() && mask.size(0) == logits.size(0),
              "bitmask must be int32 [rows, ceil(V / 32)]");
  TORCH_CHECK(logits.stride(1) == 1 && mask.size(1) * 32 >= logits.size(1), "apply_token_bitmask: shapes");
  const c10::cuda::CUDAGuard guard(logits.device());
  b200::apply_token_bitmask_launch(reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
                                   (int)logits.size(0), (int)logits.size(1), mask.data_ptr<int32_t>(),
                                   (int)mask.size(1), cur_stream());
  check_launch("apply_token_bitmask", logits.size(0) > 0 ? 1 : 0);
}

// wt: MXFP4 weight tiles [E, ceil(N / 256), K / 64, tile_bytes] uint8 (ops.moe.pack_mxfp4);
// N = out.size(1).
void moe_mxfp4_gemm(const at::Tensor& x, const at::Tensor& wt, at::Tensor& out,
                    const at::Tensor& gtiles, const at::Tensor& gcount) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(out);
  TORCH_CHECK(wt.scalar_type() == at::kByte && wt.dim() == 4 && wt.is_contiguous() &&
                  wt.size(3) == b200::moe_mxfp4_tile_bytes(),
              "moe_mxfp4_gemm: wt must be uint8 [E, N/256, K/64, tile_bytes]");
  const int K = (int)wt.size(2) * 64;
  const int N = (int)out.size(1);
  TORCH_CHECK(x.size(1) == K && wt.size(1) * b200::moe_mxfp4_tile_cols() >= N, "moe_mxfp4_gemm: shapes");
  TORCH_CHECK(x.stride(1) == 1 && out.stride(1) == 1, "moe_mxfp4_gemm: layouts");
  const c10::cuda::CUDAGuard guard(x.device());
  b200::moe_mxfp4_gemm_launch(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
                              wt.data_ptr<uint8_t>(), gtiles.data_ptr<int>(), gcount.data_ptr<int>(),
                              (int)gtiles.size(0), N, K, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                              out.stride(0), status_word(), cur_stream());
  check_launch("moe_mxfp4_gemm");
}

// Bounded wait on flag[0] >= target for timeout_ms (failure-detection test of the peer waits).
void flag_wait_probe(const at::Tensor& flag, int64_t target, double timeout_ms, at::Tensor& result) {
  CHECK_CUDA(flag);
  TORCH_CHECK(flag.scalar_type() == at::kInt && result.scalar_type() == at::kInt, "int32 tensors");
  const c10::cuda::CUDAGuard guard(flag.device());
  b200::flag_wait_probe_launch(reinterpret_cast<const unsigned int*>(flag.data_ptr<int>()), (unsigned)target,
                               (unsigned long long)(timeout_ms * 1e6), status_word(), result.data_ptr<int>(),
                               cur_stream());
  check_launch("flag_wait_probe");
}

int64_t num_sms() { return b200::num_sms_cached(); }
int64_t launch_count() { return g_launches.load(); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of vllm_neuron_b200";
  m.def("gemm", &gemm);
  m.def("gemm_2sm_set", [](bool on) { b200::gemm2sm_set(on); });
  m.def("gemm_2sm_enabled", []() { return b200::gemm2sm_enabled(); });
  m.def("gemm_2sm_pairs", []() { return b200::gemm2sm_pairs(); });
  m.def("gemm_sp", &gemm_sp);
  m.def("gemm_fp8", &gemm_fp8);
  m.def("gemm_fp8_block", &gemm_fp8_block);
  m.def("gemm_fp8_block_prefill", &gemm_fp8_block_prefill);
  m.def("quant_fp8_block", &quant_fp8_block);
  m.def("quant_mx8", &quant_mx8);
  m.def("gemm_mx8", &gemm_mx8);
  m.def("quant_mx8_tiles", &quant_mx8_tiles);
  m.def("gemm_mx8_grouped", &gemm_mx8_grouped);
  m.def("quant_fp8", &quant_fp8);
  m.def("rmsnorm_quant", &rmsnorm_quant);
  m.def("sp_norm_push", &sp_norm_push);
  m.def("sp_wait", &sp_wait);
  m.def("paged_attention", &paged_attention);
  m.def("attn_combine", &attn_combine);
  m.def("add_rmsnorm", &add_rmsnorm);
  m.def("rope_kv_write", &rope_kv_write);
  m.def("silu_mul", &silu_mul);
  m.def("embedding", &embedding);
  m.def("sample", &sample);
  m.def("argmax", &argmax);
  m.def("read_status", &read_status);
  m.def("flag_wait_probe", &flag_wait_probe);
  m.def("reset_status", &reset_status);
  m.def("status_copy_async", &status_copy_async);
  m.def("num_sms", &num_sms);
  m.def("launch_count", &launch_count);
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_free", &symm_free);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("tp_allreduce_norm", &tp_allreduce_norm);
  m.def("gemm_w8", &gemm_w8);
  m.def("ep_exchange", &ep_exchange);
  m.def("gemm_grouped", &gemm_grouped);
  m.def("moe_route", &moe_route);
  m.def("moe_align", &moe_align);
  m.def("moe_router_topk", &moe_router_topk);
  m.def("moe_gather", &moe_gather);
  m.def("moe_act", &moe_act);
  m.def("moe_combine", &moe_combine);
  m.def("moe_mxfp4_gemm", &moe_mxfp4_gemm);
  m.def("causal_conv1d", &causal_conv1d);
  m.def("gated_delta_rule", &gated_delta_rule);
  m.def("sigmoid_gate_mul", &sigmoid_gate_mul);
  m.def("apply_token_bitmask", &apply_token_bitmask);
}
