// Fused data-parallel step for one gradient bucket, over NVLink peer memory:
//
//   reduce-scatter (peer loads) -> fp32 AdamW on the owned shard -> all-gather
//   of the updated fp32 master and bf16 shadow (peer stores)
//
// in ONE kernel per bucket.  The reference does a blocking per-parameter
// NCCL all-reduce followed by a full-model AdamW on every rank
// (parallel/data_parallel.py:5-15, main.py:144,177); its ZeRO-1 module
// (parallel/distributed_optimizer.py:7-48) broadcasts every parameter.  Here
// each rank owns a contiguous 1/dp slice of the bucket: it reads that slice of
// every peer's gradient buffer directly (P2P loads through NVSwitch), sums in
// fp32, applies AdamW with its local (sharded) moments, and writes the new
// fp32 parameter and its bf16 copy straight into every peer's parameter
// buffers.  Optimizer state is 1/dp per rank (ZeRO-1) and no gradient or
// parameter ever goes through an intermediate buffer.
//
// Cross-rank ordering uses flags in each rank's signal pad
// (int32 [kMaxBuckets][2][kMaxRanks], values = step epoch):
//   ready[bucket][r]  rank r's gradients of this bucket are final
//   done[bucket][r]   rank r has written its slice into every peer
// Writers publish with a system-scope release after a system fence; readers
// spin with system-scope acquire loads, bounded by a time limit after which
// the kernel records an error code and returns (the host raises).
#include "common.cuh"
#include "ops.h"

#include <algorithm>

namespace mmb {

constexpr int kDpMaxRanks = 8;
constexpr int kDpMaxBuckets = 256;
constexpr unsigned long long kPeerTimeoutNs = 10000000000ull;  // 10 s: ranks may drift between launches

struct DpPeers {
  float* param[kDpMaxRanks];
  float* grad[kDpMaxRanks];
  __nv_bfloat16* pbf16[kDpMaxRanks];
  int* sig[kDpMaxRanks];
};

struct DpArgs {
  int world, rank, bucket;
  int epoch;
  long lo, hi;          // owned range (flat elements, multiple of 4)
  float* exp_avg;       // moments of the owned range, index 0 == lo
  float* exp_avg_sq;
  float lr, b1, b2, eps, wd, step_size, bc2_sqrt, grad_scale;
  unsigned* counter;    // local CTA-completion counter for this bucket
  int* err;
  int defer_done;       // 1: publish "done" and return; dp_wait_done_kernel waits for all buckets at step end
  const int* epoch_ptr;   // non-null: the epoch is read from device memory (CUDA-graph replays)
  const float* hyper;     // non-null: {lr, lr / bc1, sqrt(bc2)} from device memory (see adamw_hyper_step)
};

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until every rank's flag `slot` reached `epoch` (threads 0..world-1 each poll one rank).
__device__ bool wait_flags(const int* pad, int slot, int world, int epoch, int* err) {
  bool ok = true;
  if (threadIdx.x < world) {
    const int* f = pad + slot * kDpMaxRanks + threadIdx.x;
    const unsigned long long t0 = globaltimer();
    while (ld_acquire_sys(f) < epoch) {
      if (globaltimer() - t0 > kPeerTimeoutNs) {
        atomicExch(err, kErrPeerWait);
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

__global__ void __launch_bounds__(256) dp_rs_adamw_ag_kernel(const DpPeers P, DpArgs a) {
  pdl_trigger();
  pdl_wait();
  if (a.epoch_ptr) a.epoch = *a.epoch_ptr;
  if (a.hyper) {
    a.lr = a.hyper[0];
    a.step_size = a.hyper[1];
    a.bc2_sqrt = a.hyper[2];
  }
  const int world = a.world;
  const int slot_ready = a.bucket * 2, slot_done = a.bucket * 2 + 1;
  // 1. publish "my gradients of this bucket are final" (written by earlier kernels on this stream)
  if (blockIdx.x == 0 && threadIdx.x < world) {
    __threadfence_system();
    st_release_sys(P.sig[threadIdx.x] + slot_ready * kDpMaxRanks + a.rank, a.epoch);
  }
  // 2. wait for every rank's gradients
  if (!wait_flags(P.sig[a.rank], slot_ready, world, a.epoch, a.err)) return;

  // 3. reduce-scatter + AdamW + all-gather of the owned range, 4 elements per thread-iteration
  const long n4 = (a.hi - a.lo) >> 2;
  const float decay = 1.f - a.lr * a.wd;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    const long e = a.lo + 4 * i;
    float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kDpMaxRanks; ++r) {
      if (r < world) {
        const float4 x = *reinterpret_cast<const float4*>(P.grad[r] + e);
        g.x += x.x; g.y += x.y; g.z += x.z; g.w += x.w;
      }
    }
    float4 p = *reinterpret_cast<const float4*>(P.param[a.rank] + e);
    float4 m = reinterpret_cast<float4*>(a.exp_avg)[i];
    float4 v = reinterpret_cast<float4*>(a.exp_avg_sq)[i];
    float* pp = &p.x;
    float* mm = &m.x;
    float* vv = &v.x;
    const float* gg = &g.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gr = gg[k] * a.grad_scale;
      const float pe = pp[k] * decay;
      mm[k] = mm[k] + (1.f - a.b1) * (gr - mm[k]);
      vv[k] = vv[k] * a.b2 + (1.f - a.b2) * gr * gr;
      pp[k] = pe - a.step_size * (mm[k] / (sqrtf(vv[k]) / a.bc2_sqrt + a.eps));
    }
    reinterpret_cast<float4*>(a.exp_avg)[i] = m;
    reinterpret_cast<float4*>(a.exp_avg_sq)[i] = v;
    uint2 pb;
    pb.x = pack_bf16x2(p.x, p.y);
    pb.y = pack_bf16x2(p.z, p.w);
#pragma unroll
    for (int r = 0; r < kDpMaxRanks; ++r) {
      if (r < world) {
        *reinterpret_cast<float4*>(P.param[r] + e) = p;
        *reinterpret_cast<uint2*>(P.pbf16[r] + e) = pb;
      }
    }
  }

  // 4. last CTA to finish publishes "done" to every rank, then waits for every rank's "done"
  __threadfence_system();
  __shared__ unsigned prev;
  __syncthreads();
  if (threadIdx.x == 0) prev = atomicAdd(a.counter, 1u);
  __syncthreads();
  if (prev != gridDim.x - 1) return;
  if (threadIdx.x == 0) *a.counter = 0;  // ready for the next use of this bucket
  if (threadIdx.x < world) {
    __threadfence_system();
    st_release_sys(P.sig[threadIdx.x] + slot_done * kDpMaxRanks + a.rank, a.epoch);
  }
  if (a.defer_done) return;
  wait_flags(P.sig[a.rank], slot_done, world, a.epoch, a.err);
}

// End of an optimizer step with deferred completion: wait (bounded, polling
// with a short sleep) until every rank has published "done" for every bucket,
// i.e. all peers finished reading this rank's gradients and writing its
// parameters.  One thread per (bucket, rank) flag, strided over the block.
__global__ void __launch_bounds__(256) dp_wait_done_kernel(const int* __restrict__ pad, int nbuckets, int world,
                                                           int epoch, const int* __restrict__ epoch_ptr,
                                                           unsigned long long timeout_ns, int* err) {
  pdl_trigger();
  pdl_wait();
  if (epoch_ptr) epoch = *epoch_ptr;
  const int n = nbuckets * world;
  const unsigned long long t0 = globaltimer();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int b = i / world, r = i % world;
    const int* f = pad + (b * 2 + 1) * kDpMaxRanks + r;
    while (ld_acquire_sys(f) < epoch) {
      if (globaltimer() - t0 > timeout_ns) {
        atomicExch(err, kErrPeerWait);
        return;
      }
      __nanosleep(200);
    }
  }
}

int dp_wait_done(const void* sig_local, int nbuckets, int world, int epoch, const int* epoch_ptr,
                 unsigned long long timeout_ns, int* err, cudaStream_t stream) {
  if (nbuckets < 1 || nbuckets > kDpMaxBuckets || world < 1 || world > kDpMaxRanks) return -1;
  launch_k(dp_wait_done_kernel, 1, 256, 0, stream, reinterpret_cast<const int*>(sig_local), nbuckets, world, epoch,
           epoch_ptr, timeout_ns, err);
  return (int)cudaGetLastError();
}

// One thread: advance the device epoch of the cross-rank flags by one step.
__global__ void dp_epoch_step_kernel(int* __restrict__ epoch) {
  pdl_trigger();
  pdl_wait();
  if (blockIdx.x == 0 && threadIdx.x == 0) *epoch += 1;
}

int dp_epoch_step(int* epoch, cudaStream_t stream) {
  launch_k(dp_epoch_step_kernel, 1, 32, 0, stream, epoch);
  return (int)cudaGetLastError();
}

int dp_rs_adamw_ag(const DpPeersHost& peers, const DpStepHost& s, cudaStream_t stream) {
  if (peers.world < 1 || peers.world > kDpMaxRanks || s.bucket < 0 || s.bucket >= kDpMaxBuckets) return -1;
  if ((s.lo & 3) || (s.hi & 3)) return -2;
  DpPeers P;
  for (int r = 0; r < kDpMaxRanks; ++r) {
    P.param[r] = r < peers.world ? reinterpret_cast<float*>(peers.param[r]) : nullptr;
    P.grad[r] = r < peers.world ? reinterpret_cast<float*>(peers.grad[r]) : nullptr;
    P.pbf16[r] = r < peers.world ? reinterpret_cast<__nv_bfloat16*>(peers.pbf16[r]) : nullptr;
    P.sig[r] = r < peers.world ? reinterpret_cast<int*>(peers.sig[r]) : nullptr;
  }
  DpArgs a;
  a.world = peers.world;
  a.rank = peers.rank;
  a.bucket = s.bucket;
  a.epoch = s.epoch;
  a.lo = s.lo;
  a.hi = s.hi;
  a.exp_avg = s.exp_avg;
  a.exp_avg_sq = s.exp_avg_sq;
  a.lr = s.lr;
  a.b1 = s.b1;
  a.b2 = s.b2;
  a.eps = s.eps;
  a.wd = s.wd;
  a.step_size = s.step_size;
  a.bc2_sqrt = s.bc2_sqrt;
  a.grad_scale = s.grad_scale;
  a.counter = s.counter;
  a.err = s.err;
  a.defer_done = s.defer_done;
  a.epoch_ptr = s.epoch_ptr;
  a.hyper = s.hyper;
  const long n4 = (s.hi - s.lo) / 4;
  const int blocks = (int)std::max<long>(1, std::min<long>((n4 + 255) / 256, s.max_ctas));
  launch_k(dp_rs_adamw_ag_kernel, blocks, 256, 0, stream, P, a);
  return (int)cudaGetLastError();
}

int dp_signal_pad_bytes() { return kDpMaxBuckets * 2 * kDpMaxRanks * (int)sizeof(int); }

}  // namespace mmb
