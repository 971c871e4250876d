// Tensor-parallel collectives fused with the kernels around them (sequence-
// parallel dataflow over NVLink peer memory).
//
// The reference all-reduces Row-parallel outputs and Column-parallel input
// gradients with NCCL (comm/all_reduce.py:5-43) and keeps a sequence-parallel
// module that is not wired (comm/sequence_parallel.py).  Here, with
// sequence parallelism, every activation between TP GEMMs is sharded along
// the sequence, and the two collectives are folded into the kernels that
// produce / consume the data:
//
//   all-gather      the producer of a sequence shard (LayerNorm forward, or
//                   LayerNorm backward for gradients; layernorm.cu) writes
//                   each bf16 row straight into every TP rank's gathered
//                   buffer; the next Column GEMM's TMA producer waits per
//                   source rank for that rank's flag before loading its rows
//                   (gemm_sm100.cu), so local rows start immediately;
//   reduce-scatter  the Row GEMM's epilogue pushes each bf16 partial output
//                   tile into the owning rank's per-source slot
//                   (gemm_sm100.cu, EPI_PUSH_BF16); `tp_rs_reduce` below waits
//                   for every source and sums the slots (plus the residual).
//
// Flags hold monotonically increasing epochs (one counter per collective kind,
// advanced identically on every rank); every wait is bounded (peer.cuh).
#include "common.cuh"
#include "ops.h"
#include "peer.cuh"

#include <algorithm>

namespace mmb {

// out[r] = (resid ? resid[r] : 0) + sum_src slot[src][r]   over rows_l x H,
// after every source rank's flag reached `epoch`.  Outputs fp32 and/or bf16.
__global__ void __launch_bounds__(256) tp_rs_reduce_kernel(const __nv_bfloat16* __restrict__ slots, long slot_stride,
                                                           int world, const int* __restrict__ flags, int epoch,
                                                           const float* __restrict__ resid, float* __restrict__ out,
                                                           __nv_bfloat16* __restrict__ out_bf16, long n, int* err,
                                                           unsigned long long timeout_ns) {
  pdl_trigger();
  pdl_wait();
  if (!cta_wait_flags(flags, world, epoch, err, timeout_ns)) return;
  const long n8 = n >> 3;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    float acc[8];
    if (resid) {
      const float4 a = reinterpret_cast<const float4*>(resid)[2 * i];
      const float4 b = reinterpret_cast<const float4*>(resid)[2 * i + 1];
      acc[0] = a.x; acc[1] = a.y; acc[2] = a.z; acc[3] = a.w; acc[4] = b.x; acc[5] = b.y; acc[6] = b.z; acc[7] = b.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    }
    for (int src = 0; src < world; ++src) {
      const uint4 u = reinterpret_cast<const uint4*>(slots + src * slot_stride)[i];
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(w[e]);
        acc[2 * e] += f.x;
        acc[2 * e + 1] += f.y;
      }
    }
    if (out) {
      reinterpret_cast<float4*>(out)[2 * i] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      reinterpret_cast<float4*>(out)[2 * i + 1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
    if (out_bf16)
      reinterpret_cast<uint4*>(out_bf16)[i] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                                         pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
  }
}

// Stand-alone all-gather push of a local bf16 shard (used where the producer
// kernel is not one of ours, e.g. a gradient handed in by autograd).
__global__ void __launch_bounds__(256) tp_ag_push_kernel(const __nv_bfloat16* __restrict__ src, int rows, int H,
                                                         const AgPush P) {
  pdl_trigger();
  pdl_wait();
  const int units = H / 8;
  const long n = (long)rows * units;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int r = (int)(i / units), u = (int)(i % units);
    const uint4 v = reinterpret_cast<const uint4*>(src + (size_t)r * H)[u];
    const long grow = (long)(r / P.Sl) * P.S + (long)P.rank * P.Sl + r % P.Sl;
    for (int p = 0; p < P.world; ++p)
      reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(P.dst[p]) + grow * P.ld)[u] = v;
  }
  grid_done_signal(P.flags, P.world, P.rank, P.epoch, P.counter);
}

// Vocabulary-parallel cross-entropy statistics across the TP group: every rank
// holds (row max, sum of exp(logit - max), target logit or 0) of its vocabulary
// shard for every token row.  Push: each rank writes its triplets into slot
// [rank] of every peer (16 B per row) and the last CTA raises the flags.
// Reduce: once every source has signalled, lse = M + log(sum_r se_r exp(mx_r - M))
// with M = max_r mx_r, and the target logit is the sum over ranks (only the
// owner of the label's vocabulary row contributes a non-zero value).
__global__ void __launch_bounds__(256) tp_ce_push_kernel(const float* __restrict__ mx, const float* __restrict__ se,
                                                         const float* __restrict__ tg, int rows, const AgPush P) {
  pdl_trigger();
  pdl_wait();
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const float4 v = make_float4(mx[r], se[r], tg[r], 0.f);
    for (int p = 0; p < P.world; ++p)
      reinterpret_cast<float4*>(P.dst[p])[(long)P.rank * rows + r] = v;
  }
  grid_done_signal(P.flags, P.world, P.rank, P.epoch, P.counter);
}

__global__ void __launch_bounds__(256) tp_ce_reduce_kernel(const float4* __restrict__ slots, int rows, int world,
                                                           const int* __restrict__ flags, int epoch,
                                                           float* __restrict__ lse, float* __restrict__ tg,
                                                           int* err, unsigned long long timeout_ns) {
  pdl_trigger();
  pdl_wait();
  if (!cta_wait_flags(flags, world, epoch, err, timeout_ns)) return;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    float m = -INFINITY;
    for (int s = 0; s < world; ++s) m = fmaxf(m, slots[(long)s * rows + r].x);
    float sum = 0.f, t = 0.f;
    for (int s = 0; s < world; ++s) {
      const float4 v = slots[(long)s * rows + r];
      sum += v.y * __expf(v.x - m);
      t += v.z;
    }
    lse[r] = m + logf(sum);
    tg[r] = t;
  }
}

int tp_ce_allreduce(const float* mx, const float* se, const float* tg_in, int rows, const AgPush& push,
                    const void* slots_local, const int* flags_local, float* lse, float* tg_out, int* err, int num_sms,
                    cudaStream_t s, unsigned long long timeout_ns) {
  if (push.world < 1 || push.world > 8 || rows < 1) return -1;
  const int blocks = std::max(1, std::min((rows + 255) / 256, num_sms));
  launch_k(tp_ce_push_kernel, blocks, 256, 0, s, mx, se, tg_in, rows, push);
  launch_k(tp_ce_reduce_kernel, blocks, 256, 0, s, reinterpret_cast<const float4*>(slots_local), rows, push.world,
           flags_local, push.epoch, lse, tg_out, err, timeout_ns);
  return (int)cudaGetLastError();
}

// ---------------------------------------------------------------- embedding under fused TP
// The token table is vocabulary-sharded, the activations sequence-sharded.  Every token row
// has exactly one vocabulary owner, so no reduction is needed: the owner of id[p] writes
// tok[id] + pos[p % S] (fp32) straight into row p's slot in its sequence owner's output
// buffer, and the last CTA raises the flags.  One warp per row.
__global__ void __launch_bounds__(256) tp_emb_fwd_push_kernel(const long* __restrict__ ids,
                                                              const float* __restrict__ tok,
                                                              const float* __restrict__ pos, int rows, int H,
                                                              long vstart, long vend, const AgPush P) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const long nw = ((long)gridDim.x * blockDim.x) >> 5;
  for (long p = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < rows; p += nw) {
    const long id = ids[p];
    if (id < vstart || id >= vend) continue;
    const int s = (int)(p % P.S), owner = s / P.Sl;
    const long local = (p / P.S) * P.Sl + (s - owner * P.Sl);
    const float4* t = reinterpret_cast<const float4*>(tok + (size_t)(id - vstart) * H);
    const float4* q = reinterpret_cast<const float4*>(pos + (size_t)s * H);
    float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(P.dst[owner]) + (size_t)local * H);
    for (int c = lane; c < H / 4; c += 32) {
      float4 v = t[c];
      const float4 w = q[c];
      v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
      o[c] = v;
    }
  }
  grid_done_signal(P.flags, P.world, P.rank, P.epoch, P.counter);
}

// dst[i] = src[i] (add == 0) or dst[i] += src[i] (add == 1), after every source rank's flag
// reached `epoch` (each CTA waits).  n is a multiple of 4.
__global__ void __launch_bounds__(256) tp_wait_copy_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                           long n, int add, const int* __restrict__ flags,
                                                           int world, int epoch, int* err,
                                                           unsigned long long timeout_ns) {
  pdl_trigger();
  pdl_wait();
  if (!cta_wait_flags(flags, world, epoch, err, timeout_ns)) return;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n / 4; i += (long)gridDim.x * blockDim.x) {
    float4 v = reinterpret_cast<const float4*>(src)[i];
    if (add) {
      const float4 d = reinterpret_cast<const float4*>(dst)[i];
      v.x += d.x; v.y += d.y; v.z += d.z; v.w += d.w;
    }
    reinterpret_cast<float4*>(dst)[i] = v;
  }
}

// Copy this rank's fp32 rows into its own peer-readable slot (P.dst[P.rank]) and tell every
// rank that they are there.
__global__ void __launch_bounds__(256) tp_publish_kernel(const float* __restrict__ src, long n, const AgPush P) {
  pdl_trigger();
  pdl_wait();
  float4* dst = reinterpret_cast<float4*>(P.dst[P.rank]);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n / 4; i += (long)gridDim.x * blockDim.x)
    dst[i] = reinterpret_cast<const float4*>(src)[i];
  grid_done_signal(P.flags, P.world, P.rank, P.epoch, P.counter);
}

// Position-table gradient of this rank's sequence shard: row s of the shard gets
// sum_b dout[b, s] (local rows [B, Sl, H]) and is pushed to row rank*Sl + s of every rank's
// [S, H] slot; each rank later adds the full slot to its (replicated) table's main grad.
__global__ void __launch_bounds__(256) tp_pos_grad_push_kernel(const float* __restrict__ dout, int B, int H,
                                                               const AgPush P) {
  pdl_trigger();
  pdl_wait();
  const long n = (long)P.Sl * (H / 4);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int s = (int)(i / (H / 4)), c = (int)(i % (H / 4));
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int b = 0; b < B; ++b) {
      const float4 v = reinterpret_cast<const float4*>(dout + ((size_t)b * P.Sl + s) * H)[c];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    const size_t row = (size_t)P.rank * P.Sl + s;
    for (int p = 0; p < P.world; ++p) reinterpret_cast<float4*>(reinterpret_cast<float*>(P.dst[p]) + row * H)[c] = acc;
  }
  grid_done_signal(P.flags, P.world, P.rank, P.epoch, P.counter);
}

// Sum of a small fp32 vector over the TP group: push into slot [rank] of every peer, then
// (second kernel) sum the world slots once every source has signalled.
__global__ void __launch_bounds__(256) tp_vec_push_kernel(const float* __restrict__ v, long n, const AgPush P) {
  pdl_trigger();
  pdl_wait();
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float x = v[i];
    for (int p = 0; p < P.world; ++p) reinterpret_cast<float*>(P.dst[p])[(long)P.rank * n + i] = x;
  }
  grid_done_signal(P.flags, P.world, P.rank, P.epoch, P.counter);
}

__global__ void __launch_bounds__(256) tp_vec_reduce_kernel(const float* __restrict__ slots, long n, int world,
                                                            float* __restrict__ out, const int* __restrict__ flags,
                                                            int epoch, int* err, unsigned long long timeout_ns) {
  pdl_trigger();
  pdl_wait();
  if (!cta_wait_flags(flags, world, epoch, err, timeout_ns)) return;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < world; ++s) acc += slots[(long)s * n + i];
    out[i] = acc;
  }
}

static int tp_grid(long work, int num_sms) {
  return (int)std::max<long>(1, std::min<long>((work + 255) / 256, (long)num_sms * 4));
}

int tp_emb_fwd_push(const long* ids, const float* tok, const float* pos, int rows, int H, long vstart, long vend,
                    const AgPush& push, int num_sms, cudaStream_t s) {
  if (H % 4 || push.world < 1 || push.world > 8 || push.Sl <= 0) return -1;
  launch_k(tp_emb_fwd_push_kernel, tp_grid((long)rows * 32, num_sms), 256, 0, s, ids, tok, pos, rows, H, vstart,
           vend, push);
  return (int)cudaGetLastError();
}

int tp_wait_copy(const float* src, float* dst, long n, int add, const int* flags, int world, int epoch, int* err,
                 int num_sms, cudaStream_t s, unsigned long long timeout_ns) {
  if (n % 4 || world < 1 || world > 8) return -1;
  launch_k(tp_wait_copy_kernel, tp_grid(n / 4, num_sms), 256, 0, s, src, dst, n, add, flags, world, epoch, err,
           timeout_ns);
  return (int)cudaGetLastError();
}

int tp_publish(const float* src, long n, const AgPush& push, int num_sms, cudaStream_t s) {
  if (n % 4 || push.world < 1 || push.world > 8) return -1;
  launch_k(tp_publish_kernel, tp_grid(n / 4, num_sms), 256, 0, s, src, n, push);
  return (int)cudaGetLastError();
}

int tp_pos_grad_push(const float* dout, int B, int H, const AgPush& push, int num_sms, cudaStream_t s) {
  if (H % 4 || push.world < 1 || push.world > 8 || push.Sl <= 0) return -1;
  launch_k(tp_pos_grad_push_kernel, tp_grid((long)push.Sl * (H / 4), num_sms), 256, 0, s, dout, B, H, push);
  return (int)cudaGetLastError();
}

int tp_vec_allreduce(const float* v, float* out, long n, const AgPush& push, const float* slots_local,
                     const int* flags_local, int* err, int num_sms, cudaStream_t s, unsigned long long timeout_ns) {
  if (n < 1 || push.world < 1 || push.world > 8) return -1;
  const int g = tp_grid(n, num_sms);
  launch_k(tp_vec_push_kernel, g, 256, 0, s, v, n, push);
  launch_k(tp_vec_reduce_kernel, g, 256, 0, s, slots_local, n, push.world, out, flags_local, push.epoch, err,
           timeout_ns);
  return (int)cudaGetLastError();
}

int tp_rs_reduce(const __nv_bfloat16* slots, long slot_stride, int world, const int* flags, int epoch,
                 const float* resid, float* out, __nv_bfloat16* out_bf16, long n, int* err, int num_sms,
                 cudaStream_t s, unsigned long long timeout_ns) {
  if (n % 8 != 0 || world < 1 || world > 8 || slot_stride % 8 != 0) return -1;
  const int blocks = (int)std::max<long>(1, std::min<long>((n / 8 + 255) / 256, (long)num_sms * 4));
  launch_k(tp_rs_reduce_kernel, blocks, 256, 0, s, slots, slot_stride, world, flags, epoch, resid, out, out_bf16, n, err,
                                             timeout_ns);
  return (int)cudaGetLastError();
}

int tp_ag_push(const __nv_bfloat16* src, int rows, int H, const AgPush& push, int num_sms, cudaStream_t s) {
  if (H % 8 != 0 || push.world < 1 || push.world > 8) return -1;
  const long n = (long)rows * (H / 8);
  const int blocks = (int)std::max<long>(1, std::min<long>((n + 255) / 256, (long)num_sms * 4));
  launch_k(tp_ag_push_kernel, blocks, 256, 0, s, src, rows, H, push);
  return (int)cudaGetLastError();
}

}  // namespace mmb
