// Symmetric (peer-mapped) device memory: allocation, IPC export/open.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

namespace mmb {
int symm_alloc(size_t bytes, void** ptr);
int symm_free(void* ptr);
int symm_export(void* ptr, unsigned char out[64]);
int symm_open(const unsigned char in[64], void** ptr);
int symm_close(void* ptr);
}  // namespace mmb
