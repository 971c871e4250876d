// Allocation-free LayerNorm backward (see layernorm_noalloc.h for the contract).
//
// Same kernels as the regular backward (layernorm.cu); the only difference
// is where the dgamma/dbeta partial sums live: in the fixed device array
// below instead of a buffer from the caller's allocator.  The number of
// partial rows is capped so that they fit in that array.
#include <mutex>

#include "layernorm_noalloc.h"
#include "ops.h"

namespace {

// The scratch buffer.  In host code this name is only a host-side stand-in
// for the device array: its device address must be obtained with
// cudaGetSymbolAddress (done once per device below) before a kernel may use it.
static __device__ __align__(256) float g_ln_bwd_scratch[MMB_LN_NOALLOC_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;

struct DeviceSetup {
  std::once_flag once;
  float* scratch = nullptr;
  int num_sms = 0;
  cudaError_t status = cudaSuccess;
};

DeviceSetup g_setup[kMaxDevices];

// Per-device set-up with that device current: scratch address and SM count.
// Neither call allocates.
DeviceSetup* setup_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  DeviceSetup& s = g_setup[dev];
  std::call_once(s.once, [&s, dev] {
    void* p = nullptr;
    s.status = cudaGetSymbolAddress(&p, g_ln_bwd_scratch);
    if (s.status == cudaSuccess) {
      s.scratch = static_cast<float*>(p);
      s.status = cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev);
    }
  });
  if (s.status != cudaSuccess || s.scratch == nullptr || s.num_sms <= 0) return nullptr;
  return &s;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int mmb_layernorm_bwd_noalloc(
    const void* dy_bf16, const float* x, const float* mean, const float* rstd, const float* gamma, const float* dres,
    float* dx, float* dgamma, float* dbeta, int rows, int H, cudaStream_t stream) {
  if (rows <= 0 || H <= 0 || H % 4 != 0 || H > MMB_LN_NOALLOC_MAX_H) return MMB_LN_NOALLOC_EBADSHAPE;
  DeviceSetup* s = setup_for_current_device();
  if (s == nullptr) return MMB_LN_NOALLOC_ESETUP;
  // Partial rows the regular path would use, capped to what the scratch holds.
  const long cap = (long)MMB_LN_NOALLOC_SCRATCH_FLOATS / (2L * H);
  int nparts = mmb::layernorm_bwd_parts(rows, H, s->num_sms);
  if (nparts > cap) nparts = (int)cap;
  if (nparts < 1) return MMB_LN_NOALLOC_EBADSHAPE;
  const int rc = mmb::layernorm_bwd(static_cast<const __nv_bfloat16*>(dy_bf16), x, mean, rstd, gamma, dres, dx,
                                    s->scratch, dgamma, dbeta, rows, H, nparts, stream);
  return rc;
}
