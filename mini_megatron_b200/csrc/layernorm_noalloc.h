// Allocation-free LayerNorm backward: C entry point.
//
// This entry point has no counterpart in the reference (mini-megatron has no
// native code at all); it is an addition of this library.
//
// Who it is for: code that must not allocate device memory while it runs --
// for example a host runtime that does all of its allocation up front and
// forbids cudaMalloc afterwards, a caller inside a custom memory pool or
// arena that cannot hand out extra blocks, or plain C/C++ code that links
// this library without PyTorch and therefore has no caching allocator to
// borrow temporary buffers from.  The regular binding
// (``mini_megatron_b200._C.layernorm_bwd``) takes its temporary buffer for
// the dgamma/dbeta partial sums from the PyTorch allocator; this one uses a
// fixed buffer that lives inside the library instead.
//
// Contract
//   * The caller passes inputs and outputs (all device pointers, row-major,
//     16-byte aligned):  dy [rows, H] bf16, x [rows, H] fp32, mean/rstd [rows]
//     fp32, gamma [H] fp32, optional dres [rows, H] fp32 (may be NULL),
//     dx [rows, H] fp32 (written), dgamma/dbeta [H] fp32 (ACCUMULATED: the
//     function adds to their current contents, like a gradient buffer).
//   * Scratch: a 8 MiB file-scope device array (MMB_LN_NOALLOC_SCRATCH_FLOATS
//     floats).  Every GPU that loads the library holds it until the process
//     exits.  H must be a multiple of 4 and at most 4096; larger or ragged
//     widths are rejected with MMB_LN_NOALLOC_EBADSHAPE before anything is
//     launched.
//   * No cudaMalloc, cudaFree or allocating library call is made.
//   * The first call on each device looks up the scratch array's device
//     address (cudaGetSymbolAddress) with that device current, and caches it.
//     Make that first call outside any CUDA stream capture.
//   * All calls share the one scratch array, whose previous contents are left
//     in place; every call fully rewrites the part it reads, so nothing needs
//     clearing.  Calls that overlap on the GPU (different streams or threads
//     without ordering between them) race on the scratch and give wrong
//     results: order them on one stream or synchronise between them.
//
// Return value: 0 on success, MMB_LN_NOALLOC_EBADSHAPE for a rejected shape,
// MMB_LN_NOALLOC_ESETUP if the scratch address could not be obtained, or a
// positive cudaError_t from the launch.
#pragma once
#include <cuda_runtime.h>

#define MMB_LN_NOALLOC_SCRATCH_FLOATS (2u * 1024u * 1024u) /* 8 MiB */
#define MMB_LN_NOALLOC_MAX_H 4096
#define MMB_LN_NOALLOC_EBADSHAPE (-1)
#define MMB_LN_NOALLOC_ESETUP (-2)

#ifdef __cplusplus
extern "C" {
#endif

int mmb_layernorm_bwd_noalloc(const void* dy_bf16, const float* x, const float* mean, const float* rstd,
                              const float* gamma, const float* dres, float* dx, float* dgamma, float* dbeta,
                              int rows, int H, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
