// Vocab-parallel softmax cross-entropy for sm_100a.
//
// The reference all-gathers full-vocabulary logits across TP ranks and runs
// F.cross_entropy on them in fp32 (main.py:131-133, model/loss.py:4-16).
// Here each rank only touches its local vocabulary shard of bf16 logits:
//
//   forward : per row, (max, sum exp(x - max), target logit if the label is
//             in this shard) -> three fp32 scalars per token.  The TP
//             combine is three tiny all-reduces of [tokens] vectors.
//   backward: d logits = (softmax - onehot) * scale_row, written as bf16 in
//             place over the logits (they are dead after this), padded
//             vocabulary columns get zero gradient.
//
// One CTA per row; the row is streamed with 16-byte loads and an online
// (max, sumexp) update per 8 elements.
#include "common.cuh"
#include "ops.h"

namespace mmb {

constexpr int kCeThreads = 256;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;          // the other side saw no element
  if (m == -INFINITY) {
    m = m2;
    s = s2;
    return;
  }
  if (m2 > m) {
    s = s * __expf(m - m2) + s2;
    m = m2;
  } else {
    s += s2 * __expf(m2 - m);
  }
}

__global__ void __launch_bounds__(kCeThreads) ce_fwd_kernel(const __nv_bfloat16* __restrict__ logits, long ld,
                                                            const long* __restrict__ labels, long vocab_start,
                                                            int n_valid, float* __restrict__ out_max,
                                                            float* __restrict__ out_sum, float* __restrict__ out_tgt) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + (size_t)row * ld;
  float m = -INFINITY, s = 0.f;
  const int nvec = n_valid >> 3;  // full 8-wide chunks
  const uint4* x8 = reinterpret_cast<const uint4*>(x);
  for (int i = threadIdx.x; i < nvec; i += kCeThreads) {
    const uint4 u = x8[i];
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&u);
    float v[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16x2(w[e]);
      v[2 * e] = f.x;
      v[2 * e + 1] = f.y;
    }
    float cm = v[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) cm = fmaxf(cm, v[e]);
    if (cm > m) {
      s *= __expf(m - cm);
      m = cm;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) s += __expf(v[e] - m);
  }
  for (int i = (nvec << 3) + threadIdx.x; i < n_valid; i += kCeThreads) {
    const float v = __bfloat162float(x[i]);
    online_merge(m, s, v, 1.f);
  }
  // block reduce (m, s)
  __shared__ float sm[kCeThreads / 32], ss[kCeThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[wid] = m;
    ss[wid] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm[0], S = ss[0];
    for (int w = 1; w < kCeThreads / 32; ++w) online_merge(M, S, sm[w], ss[w]);
    out_max[row] = M;
    out_sum[row] = S;
    const long lab = labels[row] - vocab_start;
    out_tgt[row] = (lab >= 0 && lab < n_valid) ? __bfloat162float(x[lab]) : 0.f;
  }
}

// dlogits = (exp(x - lse) - onehot(label)) * scale[row]; padded columns -> 0.
__global__ void __launch_bounds__(kCeThreads) ce_bwd_kernel(__nv_bfloat16* __restrict__ logits, long ld, int n_cols,
                                                            const long* __restrict__ labels, long vocab_start,
                                                            int n_valid, const float* __restrict__ lse,
                                                            const float* __restrict__ scale) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  __nv_bfloat16* x = logits + (size_t)row * ld;
  const float l = lse[row];
  const float sc = scale[row];
  long lab = labels[row] - vocab_start;
  if (lab < 0 || lab >= n_valid) lab = -1;  // label owned by another shard (or padding): no one-hot here
  const int nvec = n_cols >> 3;
  uint4* x8 = reinterpret_cast<uint4*>(x);
  for (int i = threadIdx.x; i < nvec; i += kCeThreads) {
    uint4 u = x8[i];
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16x2(w[e]);
      const int c0 = 8 * i + 2 * e, c1 = c0 + 1;
      float g0 = (c0 < n_valid) ? __expf(f.x - l) : 0.f;
      float g1 = (c1 < n_valid) ? __expf(f.y - l) : 0.f;
      if (c0 == lab) g0 -= 1.f;
      if (c1 == lab) g1 -= 1.f;
      w[e] = pack_bf16x2(g0 * sc, g1 * sc);
    }
    x8[i] = u;
  }
  for (int c = (nvec << 3) + threadIdx.x; c < n_cols; c += kCeThreads) {
    float g = (c < n_valid) ? __expf(__bfloat162float(x[c]) - l) : 0.f;
    if (c == lab) g -= 1.f;
    x[c] = __float2bfloat16(g * sc);
  }
}

// Merges the per-tile (max, sumexp) partials that the lm_head GEMM epilogue
// (EPI_CE_STATS) wrote, one warp per row, and gathers the target logit: the
// forward statistics without re-reading the [rows, vocab] logits.
__global__ void __launch_bounds__(256) ce_merge_kernel(const float2* __restrict__ part, long ld_part, int nparts,
                                                       const __nv_bfloat16* __restrict__ logits, long ld,
                                                       const long* __restrict__ labels, long vocab_start, int n_valid,
                                                       int rows, float* __restrict__ out_max,
                                                       float* __restrict__ out_sum, float* __restrict__ out_tgt) {
  pdl_trigger();
  pdl_wait();
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float m = -INFINITY, s = 0.f;
  const float2* pr = part + (size_t)row * ld_part;
  for (int i = lane; i < nparts; i += 32) {
    const float2 q = pr[i];
    online_merge(m, s, q.x, q.y);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  if (lane == 0) {
    out_max[row] = m;
    out_sum[row] = s;
    const long lab = labels[row] - vocab_start;
    out_tgt[row] = (lab >= 0 && lab < n_valid) ? __bfloat162float(logits[(size_t)row * ld + lab]) : 0.f;
  }
}

int ce_merge_stats(const float2* part, long ld_part, int nparts, const __nv_bfloat16* logits, long ld,
                   const long* labels, long vocab_start, int n_valid, int rows, float* out_max, float* out_sum,
                   float* out_tgt, cudaStream_t s) {
  if (nparts < 1 || ld_part < nparts) return -1;
  const int blocks = (rows * 32 + 255) / 256;
  launch_k(ce_merge_kernel, blocks, 256, 0, s, part, ld_part, nparts, logits, ld, labels, vocab_start, n_valid, rows,
                                         out_max, out_sum, out_tgt);
  return (int)cudaGetLastError();
}

int ce_fwd_stats(const __nv_bfloat16* logits, long ld, const long* labels, long vocab_start, int n_valid, int rows,
                 float* out_max, float* out_sum, float* out_tgt, cudaStream_t s) {
  if ((ld % 8) != 0 || (reinterpret_cast<uintptr_t>(logits) & 15)) return -1;
  launch_k(ce_fwd_kernel, rows, kCeThreads, 0, s, logits, ld, labels, vocab_start, n_valid, out_max, out_sum, out_tgt);
  return (int)cudaGetLastError();
}

int ce_bwd(__nv_bfloat16* logits, long ld, int n_cols, const long* labels, long vocab_start, int n_valid, int rows,
           const float* lse, const float* scale, cudaStream_t s) {
  if ((ld % 8) != 0 || (reinterpret_cast<uintptr_t>(logits) & 15)) return -1;
  launch_k(ce_bwd_kernel, rows, kCeThreads, 0, s, logits, ld, n_cols, labels, vocab_start, n_valid, lse, scale);
  return (int)cudaGetLastError();
}

}  // namespace mmb
