// Fused data-parallel step for one gradient bucket, over NVLink peer memory:
//
//   reduce-scatter (peer loads) -> fp32 AdamW on the owned shard -> all-gather
//   (peer stores) of only the copy of each parameter that the forward reads
//
// in ONE kernel per bucket.  The reference does a blocking per-parameter
// NCCL all-reduce followed by a full-model AdamW on every rank
// (parallel/data_parallel.py:5-15, main.py:144,177); its ZeRO-1 module
// (parallel/distributed_optimizer.py:7-48) broadcasts every parameter.  Here
// each rank owns a contiguous 1/dp slice of the bucket: it reads that slice of
// every peer's gradient buffer directly (P2P loads through NVSwitch), sums in
// fp32, applies AdamW with its local (sharded) moments and its fp32 master,
// and stores the result into every peer:
//
//   kind 0 (GEMM weights)            bf16 shadow to every rank, fp32 master stays on the owner
//   kind 1 (LayerNorm, embeddings)   fp32 master to every rank (their kernels read fp32)
//   kind 2 (no run table given)      both
//
// so a parameter crosses NVLink as 4 B of gradient plus 2 B (kind 0) or 4 B
// (kind 1) per element, and the fp32 master of a GEMM weight is current only
// on its owner (dp_gather_master copies the other shards back on demand, e.g.
// for a checkpoint).  No gradient or parameter goes through a staging buffer.
//
// Memory-level parallelism: NVLink loads take microseconds, so every thread
// issues the loads of U float4 groups from all ranks (and its local master /
// moments) before it uses any of them.
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

// One run of the owned range with the same replication kind, in float4 units relative to `lo`.
struct DpSeg {
  int begin4, end4, kind, pad;
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
  const DpSeg* segs;      // sorted runs covering [0, n4); nullptr = one run of kind 2
  int nseg;
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

constexpr int kDpU = 2;          // float4 groups per thread per iteration
constexpr int kDpMaxSegs = 64;   // replication runs per bucket (staged in shared memory, 1 KB)

__device__ __forceinline__ void adamw4(float4& p, float4& m, float4& v, const float4 g, const DpArgs& a,
                                       float decay) {
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
}

template <int W>
__global__ void __launch_bounds__(256) dp_rs_adamw_ag_kernel(const DpPeers P, DpArgs a) {
  pdl_trigger();
  pdl_wait();
  if (a.epoch_ptr) a.epoch = *a.epoch_ptr;
  if (a.hyper) {
    a.lr = a.hyper[0];
    a.step_size = a.hyper[1];
    a.bc2_sqrt = a.hyper[2];
  }
  __shared__ DpSeg seg_s[kDpMaxSegs];
  const int nseg = a.segs ? a.nseg : 1;
  for (int i = threadIdx.x; i < nseg; i += blockDim.x)
    seg_s[i] = a.segs ? a.segs[i] : DpSeg{0, 0x7fffffff, 2, 0};
  const int slot_ready = a.bucket * 2, slot_done = a.bucket * 2 + 1;
  // 1. publish "my gradients of this bucket are final" (written by earlier kernels on this stream)
  if (blockIdx.x == 0 && threadIdx.x < W) {
    __threadfence_system();
    st_release_sys(P.sig[threadIdx.x] + slot_ready * kDpMaxRanks + a.rank, a.epoch);
  }
  // 2. wait for every rank's gradients (the wait ends with a block barrier, which also covers seg_s).
  //    A CTA whose wait ran out (error recorded) skips the data movement but still takes part in the
  //    completion count below, so the bucket's counter returns to zero and a later launch of this
  //    bucket is not left waiting for a CTA that already left.
  const bool ready = wait_flags(P.sig[a.rank], slot_ready, W, a.epoch, a.err);

  // 3. reduce-scatter + AdamW + all-gather of the owned range
  const long n4 = ready ? (a.hi - a.lo) >> 2 : 0;
  const long stride = (long)gridDim.x * blockDim.x;
  const float decay = 1.f - a.lr * a.wd;
  const float* gsrc[W];
#pragma unroll
  for (int r = 0; r < W; ++r) gsrc[r] = P.grad[r] + a.lo;
  float* master = P.param[a.rank] + a.lo;
  int cur = 0;
  for (long i0 = blockIdx.x * (long)blockDim.x + threadIdx.x; i0 < n4; i0 += kDpU * stride) {
    float4 x[W][kDpU], p[kDpU], m[kDpU], v[kDpU];
    // issue every load of this iteration before using any of them
#pragma unroll
    for (int u = 0; u < kDpU; ++u) {
      const long i = i0 + u * stride;
      if (i < n4) {
#pragma unroll
        for (int r = 0; r < W; ++r) x[r][u] = reinterpret_cast<const float4*>(gsrc[r])[i];
        p[u] = reinterpret_cast<const float4*>(master)[i];
        m[u] = reinterpret_cast<const float4*>(a.exp_avg)[i];
        v[u] = reinterpret_cast<const float4*>(a.exp_avg_sq)[i];
      }
    }
#pragma unroll
    for (int u = 0; u < kDpU; ++u) {
      const long i = i0 + u * stride;
      if (i >= n4) break;
      float4 g = x[0][u];
#pragma unroll
      for (int r = 1; r < W; ++r) {
        g.x += x[r][u].x; g.y += x[r][u].y; g.z += x[r][u].z; g.w += x[r][u].w;
      }
      adamw4(p[u], m[u], v[u], g, a, decay);
      reinterpret_cast<float4*>(a.exp_avg)[i] = m[u];
      reinterpret_cast<float4*>(a.exp_avg_sq)[i] = v[u];
      reinterpret_cast<float4*>(master)[i] = p[u];
      while (cur + 1 < nseg && i >= seg_s[cur].end4) ++cur;  // runs are sorted and i only grows
      uint2 pb;
      pb.x = pack_bf16x2(p[u].x, p[u].y);
      pb.y = pack_bf16x2(p[u].z, p[u].w);
      const long e = a.lo + 4 * i;
      const int kind = seg_s[cur].kind;
      if (kind != 0) {  // fp32 master to the other ranks
#pragma unroll
        for (int r = 0; r < W; ++r)
          if (r != a.rank) *reinterpret_cast<float4*>(P.param[r] + e) = p[u];
      }
      if (kind != 1) {  // bf16 shadow to every rank
#pragma unroll
        for (int r = 0; r < W; ++r) *reinterpret_cast<uint2*>(P.pbf16[r] + e) = pb;
      } else {          // bf16 shadow kept current locally only
        *reinterpret_cast<uint2*>(P.pbf16[a.rank] + e) = pb;
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
  if (!ready) return;                    // the error word holds the time-out; "done" is not published
  if (threadIdx.x < W) {
    __threadfence_system();
    st_release_sys(P.sig[threadIdx.x] + slot_done * kDpMaxRanks + a.rank, a.epoch);
  }
  if (a.defer_done) return;
  wait_flags(P.sig[a.rank], slot_done, W, a.epoch, a.err);
}

// Copy every other rank's shard of the fp32 master of one bucket into this
// rank's buffer (peer loads).  Only kind-0 runs are stale off their owner, but
// the copy covers the whole bucket: it runs outside the step (checkpoints,
// state_dict), never on the training path.  Ordered after this rank's last
// optimizer step on its stream, and each owner cannot start its next update
// before this rank publishes "ready" again, so the owners' values are stable.
__global__ void __launch_bounds__(256) dp_gather_master_kernel(const DpPeers P, int world, int rank, long start,
                                                               long shard) {
  const long n4 = shard * world / 4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    const long e = start + 4 * i;
    const int owner = (int)((4 * i) / shard);
    if (owner == rank) continue;
    *reinterpret_cast<float4*>(P.param[rank] + e) = *reinterpret_cast<const float4*>(P.param[owner] + e);
  }
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

static DpPeers make_peers(const DpPeersHost& peers) {
  DpPeers P;
  for (int r = 0; r < kDpMaxRanks; ++r) {
    P.param[r] = r < peers.world ? reinterpret_cast<float*>(peers.param[r]) : nullptr;
    P.grad[r] = r < peers.world ? reinterpret_cast<float*>(peers.grad[r]) : nullptr;
    P.pbf16[r] = r < peers.world ? reinterpret_cast<__nv_bfloat16*>(peers.pbf16[r]) : nullptr;
    P.sig[r] = r < peers.world ? reinterpret_cast<int*>(peers.sig[r]) : nullptr;
  }
  return P;
}

int dp_rs_adamw_ag(const DpPeersHost& peers, const DpStepHost& s, cudaStream_t stream) {
  if (peers.world < 1 || peers.world > kDpMaxRanks || s.bucket < 0 || s.bucket >= kDpMaxBuckets) return -1;
  if ((s.lo & 3) || (s.hi & 3)) return -2;
  if (s.nseg < 0 || s.nseg > kDpMaxSegs || (s.nseg > 0 && s.segs == nullptr)) return -3;
  const DpPeers P = make_peers(peers);
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
  a.segs = s.nseg > 0 ? reinterpret_cast<const DpSeg*>(s.segs) : nullptr;
  a.nseg = s.nseg;
  const long n4 = (s.hi - s.lo) / 4;
  const long per_cta = 256L * kDpU;
  long want = std::max<long>(1, std::min<long>((n4 + per_cta - 1) / per_cta, s.max_ctas));
  auto launch = [&](auto kernel) {
    // no more CTAs than fit at once: the grid-stride loop spreads the work evenly, so a second
    // wave would only run after the first one had finished its share
    static int resident[kDpMaxRanks + 1] = {};  // per world size (one kernel instance each)
    int& res = resident[peers.world];
    if (res == 0) {
      int per_sm = 1, dev = 0, sms = 1;
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, 0);
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      res = std::max(1, per_sm) * sms;
    }
    launch_k(kernel, (int)std::min<long>(want, res), 256, 0, stream, P, a);
  };
  switch (peers.world) {
    case 1: launch(dp_rs_adamw_ag_kernel<1>); break;
    case 2: launch(dp_rs_adamw_ag_kernel<2>); break;
    case 3: launch(dp_rs_adamw_ag_kernel<3>); break;
    case 4: launch(dp_rs_adamw_ag_kernel<4>); break;
    case 5: launch(dp_rs_adamw_ag_kernel<5>); break;
    case 6: launch(dp_rs_adamw_ag_kernel<6>); break;
    case 7: launch(dp_rs_adamw_ag_kernel<7>); break;
    default: launch(dp_rs_adamw_ag_kernel<8>); break;
  }
  return (int)cudaGetLastError();
}

int dp_gather_master(const DpPeersHost& peers, long start, long end, int num_sms, cudaStream_t stream) {
  if (peers.world < 1 || peers.world > kDpMaxRanks || ((end - start) % (4L * peers.world)) || (start & 3)) return -1;
  const long shard = (end - start) / peers.world;
  if (shard % 4) return -1;
  const DpPeers P = make_peers(peers);
  const long n4 = (end - start) / 4;
  const int blocks = (int)std::max<long>(1, std::min<long>((n4 + 255) / 256, 4L * num_sms));
  dp_gather_master_kernel<<<blocks, 256, 0, stream>>>(P, peers.world, peers.rank, start, shard);
  return (int)cudaGetLastError();
}

int dp_max_segments() { return kDpMaxSegs; }

int dp_signal_pad_bytes() { return kDpMaxBuckets * 2 * kDpMaxRanks * (int)sizeof(int); }

}  // namespace mmb
