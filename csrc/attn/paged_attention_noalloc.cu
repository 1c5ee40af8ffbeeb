// Allocation-free C entry point for paged attention (declared in paged_attention_noalloc.h,
// which explains who needs it, the scratch limit and the sharing rules).  No counterpart in
// the reference.
//
// The split-KV partials live in a file-scope device array instead of caller- or
// torch-allocated memory.  Host code cannot use the array's name as a device address (on
// the host it names a shadow variable), so set-up asks the runtime for the device address
// once per device and the launch passes that address in PagedAttnParams, exactly as the
// allocating path passes its torch buffers.  The kernels are the ones of
// paged_attention.cu, unchanged.
#include <cuda_runtime.h>
#include <stdio.h>

#include <atomic>
#include <exception>
#include <mutex>

#include "attention.h"
#include "paged_attention_noalloc.h"

namespace {

constexpr size_t kScratchBytes = B200_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// The scratch: fp32 partial outputs [splits, T, Hq, D], then (256-byte aligned) the fp32
// log-sum-exps [splits, T, Hq].
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mu;
std::atomic<void*> g_scratch_addr[kMaxDevices];

int fail(char* err, size_t err_len, int code, const char* fmt, long long a = 0,
         long long b = 0) {
  if (err != nullptr && err_len > 0) snprintf(err, err_len, fmt, a, b);
  return code;
}

// Device address of the scratch array on the current device, looked up on first use.
int scratch_on_current_device(void** out, char* err, size_t err_len) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(err, err_len, B200_NOALLOC_ERR_CUDA, "cudaGetDevice failed (error %lld)",
                (long long)e);
  if (dev < 0 || dev >= kMaxDevices)
    return fail(err, err_len, B200_NOALLOC_ERR_INVALID, "device ordinal %lld out of range",
                dev);
  void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    p = g_scratch_addr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || p == nullptr)
        return fail(err, err_len, B200_NOALLOC_ERR_CUDA,
                    "cudaGetSymbolAddress of the scratch array failed on device %lld "
                    "(error %lld)",
                    dev, (long long)e);
      g_scratch_addr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return B200_NOALLOC_OK;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int b200_paged_attention_noalloc(
    const void* q, long long q_stride_t, const void* k_cache, const void* v_cache,
    long long kv_block_stride, const int* block_tables, int bt_stride, const int* seq_lens,
    const int* q_start, const int* work, int num_work, void* out, long long o_stride_t,
    const float* sinks, int total_tokens, int num_q_heads, int num_kv_heads, int head_dim,
    int block_size, int window, float scale, int decode, int num_splits, void* stream,
    char* err, size_t err_len) {
  if (err != nullptr && err_len > 0) err[0] = '\0';
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || block_tables == nullptr ||
      seq_lens == nullptr || q_start == nullptr || work == nullptr || out == nullptr)
    return fail(err, err_len, B200_NOALLOC_ERR_INVALID, "a required pointer is NULL");
  if (head_dim != 64 && head_dim != 128)
    return fail(err, err_len, B200_NOALLOC_ERR_INVALID,
                "head_dim %lld is not supported (64 or 128)", head_dim);
  if (num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0)
    return fail(err, err_len, B200_NOALLOC_ERR_INVALID,
                "num_q_heads %lld must be a positive multiple of num_kv_heads %lld",
                num_q_heads, num_kv_heads);
  if (num_splits < 1 || num_splits > 64)
    return fail(err, err_len, B200_NOALLOC_ERR_INVALID, "num_splits %lld not in [1, 64]",
                num_splits);
  if (total_tokens < 0 || num_work < 0 || block_size <= 0 || bt_stride <= 0 || window < 0)
    return fail(err, err_len, B200_NOALLOC_ERR_INVALID,
                "negative size (total_tokens %lld, num_work %lld) or bad block layout",
                total_tokens, num_work);
  if (q_stride_t < (long long)num_q_heads * head_dim ||
      o_stride_t < (long long)num_q_heads * head_dim)
    return fail(err, err_len, B200_NOALLOC_ERR_INVALID,
                "token strides (q %lld, out %lld) are smaller than num_q_heads * head_dim",
                q_stride_t, o_stride_t);
  if (num_work == 0 || total_tokens == 0) return B200_NOALLOC_OK;

  b200::PagedAttnParams p{};
  if (num_splits > 1) {
    const unsigned long long rows =
        (unsigned long long)num_splits * (unsigned long long)total_tokens * num_q_heads;
    const unsigned long long o_bytes = rows * head_dim * sizeof(float);
    const unsigned long long lse_off = (o_bytes + 255ull) & ~255ull;
    const unsigned long long need = lse_off + rows * sizeof(float);
    if (need > kScratchBytes)
      return fail(err, err_len, B200_NOALLOC_ERR_TOO_LARGE,
                  "split-KV partials need %lld bytes; the scratch array holds %lld "
                  "(lower num_splits or the batch size)",
                  (long long)need, (long long)kScratchBytes);
    void* base = nullptr;
    const int rc = scratch_on_current_device(&base, err, err_len);
    if (rc != B200_NOALLOC_OK) return rc;
    p.part_o = reinterpret_cast<float*>(base);
    p.part_lse = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(base) + lse_off);
  }
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.q_stride_t = q_stride_t;
  p.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache);
  p.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache);
  p.kv_block_stride = kv_block_stride;
  p.block_tables = block_tables;
  p.bt_stride = bt_stride;
  p.seq_lens = seq_lens;
  p.q_start = q_start;
  p.work = reinterpret_cast<const int2*>(work);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.o_stride_t = o_stride_t;
  p.sinks = sinks;
  p.num_splits = num_splits;
  p.Hq = num_q_heads;
  p.Hkv = num_kv_heads;
  p.G = num_q_heads / num_kv_heads;
  p.block_size = block_size;
  p.window = window;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.total_tokens = total_tokens;
  try {
    b200::paged_attention_launch(p, num_work, head_dim, decode != 0,
                                 reinterpret_cast<cudaStream_t>(stream));
  } catch (const std::exception& e) {
    if (err != nullptr && err_len > 0)
      snprintf(err, err_len, "launch rejected the arguments: %s", e.what());
    return B200_NOALLOC_ERR_INVALID;
  } catch (...) {
    return fail(err, err_len, B200_NOALLOC_ERR_INVALID, "launch rejected the arguments");
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(err, err_len, B200_NOALLOC_ERR_CUDA, "kernel launch failed (error %lld)",
                (long long)e);
  return B200_NOALLOC_OK;
}
