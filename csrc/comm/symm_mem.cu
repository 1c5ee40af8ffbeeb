// Symmetric peer memory for one node: every rank allocates a buffer of the same size,
// exports a CUDA IPC handle, and maps the buffers of its peers (NVLink P2P through
// NVSwitch).  Kernels then load/store/reduce into peer memory with ordinary global
// instructions through the mapped pointers.  No TMA load ever reads peer memory here.
#include <cuda_runtime.h>

#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "symm_mem.h"

namespace b200 {

static void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

void* symm_alloc(size_t bytes, std::string* handle_out) {
  void* p = nullptr;
  check(cudaMalloc(&p, bytes), "symm_alloc cudaMalloc");
  check(cudaMemset(p, 0, bytes), "symm_alloc cudaMemset");
  cudaIpcMemHandle_t h;
  check(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  handle_out->assign(reinterpret_cast<const char*>(&h), sizeof(h));
  return p;
}

void* symm_open(const std::string& handle) {
  if (handle.size() != sizeof(cudaIpcMemHandle_t)) throw std::invalid_argument("bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return p;
}

void symm_close(void* peer_ptr) { check(cudaIpcCloseMemHandle(peer_ptr), "cudaIpcCloseMemHandle"); }

void symm_free(void* p) { check(cudaFree(p), "symm_free"); }

}  // namespace b200
