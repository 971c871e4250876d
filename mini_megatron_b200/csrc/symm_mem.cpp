// Symmetric device memory across the ranks of one node (CUDA IPC).
//
// Every rank allocates a buffer of the same size with cudaMalloc (NOT the
// PyTorch caching allocator: an IPC handle names a whole allocation, so the
// buffer must be its own allocation), exports a cudaIpcMemHandle_t, and the
// handles are exchanged through torch.distributed (all_gather_object on the
// host).  Each rank then opens its peers' handles; the returned device
// pointers are valid in this process and address the peer GPU's memory over
// NVLink, so the kernels of this package can load from / store to any
// rank's buffer directly.
//
// The first bytes of every symmetric allocation made for the fused kernels
// hold a signal pad (flags written by peers); see fused_dp.cu.
#include "symm_mem.h"

#include <cstring>
#include <mutex>
#include <unordered_map>

namespace mmb {

int symm_alloc(size_t bytes, void** ptr) {
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return (int)e;
  e = cudaMemset(*ptr, 0, bytes);
  return (int)e;
}

int symm_free(void* ptr) { return (int)cudaFree(ptr); }

int symm_export(void* ptr, unsigned char out[64]) {
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return (int)e;
  static_assert(sizeof(h) == 64, "unexpected IPC handle size");
  std::memcpy(out, &h, 64);
  return 0;
}

int symm_open(const unsigned char in[64], void** ptr) {
  cudaIpcMemHandle_t h;
  std::memcpy(&h, in, 64);
  return (int)cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

int symm_close(void* ptr) { return (int)cudaIpcCloseMemHandle(ptr); }

}  // namespace mmb
