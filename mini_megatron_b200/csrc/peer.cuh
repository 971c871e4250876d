// Cross-GPU signalling over NVLink peer memory (flags in symmetric buffers).
//
// Writers publish with a system-scope release after a system fence; readers
// spin with system-scope acquire loads.  Every wait is bounded: after
// kPeerTimeoutNs the waiter records kErrPeerWait in the device error word and
// gives up (the host raises), so a dead or diverged peer never hangs a GPU.
#pragma once
#include "common.cuh"

namespace mmb {

constexpr int kPeerMaxRanks = 8;
constexpr unsigned long long kPeerTimeoutNs = 10000000000ull;  // 10 s: ranks may drift between launches

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *flag >= epoch (single thread).
__device__ __forceinline__ bool wait_flag_ge(const int* flag, int epoch, int* err,
                                             unsigned long long timeout_ns = kPeerTimeoutNs) {
  if (ld_acquire_sys(flag) >= epoch) return true;
  const unsigned long long t0 = globaltimer();
  while (ld_acquire_sys(flag) < epoch) {
    if (globaltimer() - t0 > timeout_ns) {
      if (err) atomicExch(err, kErrPeerWait);
      return false;
    }
  }
  return true;
}

// CTA-wide: threads 0..n-1 each wait for flags[i] >= epoch; returns true if all arrived.
__device__ __forceinline__ bool cta_wait_flags(const int* flags, int n, int epoch, int* err,
                                               unsigned long long timeout_ns = kPeerTimeoutNs) {
  bool ok = true;
  if (threadIdx.x < n) ok = wait_flag_ge(flags + threadIdx.x, epoch, err, timeout_ns);
  return __syncthreads_and(ok) != 0;
}

// Called by every thread of every CTA at the end of a producer kernel: the
// last CTA to finish publishes `epoch` into slot [rank] of each peer's flag
// array `peer_flags[p]` (so a consumer learns that all of this rank's writes
// to it are complete).  `counter` is a zero-initialised local word, reset here.
__device__ __forceinline__ void grid_done_signal(int* const* peer_flags, int world, int rank, int epoch,
                                                 unsigned* counter) {
  __threadfence_system();
  __shared__ unsigned prev_done;
  __syncthreads();
  if (threadIdx.x == 0) prev_done = atomicAdd(counter, 1u);
  __syncthreads();
  if (prev_done != gridDim.x - 1) return;
  if (threadIdx.x == 0) *counter = 0;
  if (threadIdx.x < world) {
    __threadfence_system();
    st_release_sys(peer_flags[threadIdx.x] + rank, epoch);
  }
}

}  // namespace mmb
