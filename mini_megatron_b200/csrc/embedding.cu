// Vocab-parallel token + learned-position embedding for sm_100a.
//
// Forward : out[r] = (vocab_start <= id < vocab_end ? wte[id - vocab_start] : 0)
//                    + (add_pos ? wpe[r % S] : 0)          (fp32, one warp per row)
//           Under TP the caller all-reduces `out`; only TP rank 0 adds the
//           position term so the sum is the reference's tok + pos
//           (model/embedding.py:11-16, parallel/tensor_parallel.py:99-105).
// Backward: dwte[v] += sum of dout[r] over the rows r whose id is v, in
//           increasing r (deterministic: no atomics, see emb_bwd_tok_kernel);
//           dwpe[s] += sum_b dout[b*S+s] (a column kernel).  Both accumulate into
//           the main grads.
#include "common.cuh"
#include "ops.h"

#include <algorithm>

namespace mmb {

__global__ void emb_fwd_kernel(const long* __restrict__ ids, const float* __restrict__ wte,
                               const float* __restrict__ wpe, float* __restrict__ out, int rows, int H, int S,
                               long vstart, long vend) {
  pdl_trigger();
  pdl_wait();
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const long id = ids[row];
  const bool inside = id >= vstart && id < vend;
  const float4* t = reinterpret_cast<const float4*>(wte + (size_t)(inside ? id - vstart : 0) * H);
  const float4* p = wpe ? reinterpret_cast<const float4*>(wpe + (size_t)(row % S) * H) : nullptr;
  float4* o = reinterpret_cast<float4*>(out + (size_t)row * H);
  for (int c = lane; c < H / 4; c += 32) {
    float4 v = inside ? t[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    if (p) {
      const float4 q = p[c];
      v.x += q.x; v.y += q.y; v.z += q.z; v.w += q.w;
    }
    o[c] = v;
  }
}

// Token-table gradient with per-row ownership (deterministic, no atomics).
//
// Warp w of the grid owns the table rows [w * R, (w + 1) * R).  Each CTA streams
// the token ids through shared memory in chunks of 256 positions (stored as
// the row in this vocabulary shard, or -1); every warp scans the chunk 32
// positions at a time and, for each distinct owned row among them, adds the
// sum of those positions' gradient rows (in position order) to its row of the
// main grad.  Every element is therefore summed in one fixed order, run after
// run, unlike a scatter with atomics.
constexpr int kEmbChunk = 256;

__global__ void __launch_bounds__(256) emb_bwd_tok_kernel(const long* __restrict__ ids,
                                                          const float* __restrict__ dout, float* __restrict__ dwte,
                                                          int rows, int H, long vstart, long vend, int rows_per_warp) {
  pdl_trigger();
  pdl_wait();
  __shared__ int rel[kEmbChunk];
  const int lane = threadIdx.x & 31;
  const long gw = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long lo = gw * rows_per_warp;
  const long hi = min(lo + rows_per_warp, vend - vstart);
  const int h4 = H / 4;
  for (int base = 0; base < rows; base += kEmbChunk) {
    __syncthreads();
    for (int i = threadIdx.x; i < kEmbChunk; i += blockDim.x) {
      const int r = base + i;
      const long id = r < rows ? ids[r] : -1;
      rel[i] = (id >= vstart && id < vend) ? (int)(id - vstart) : -1;
    }
    __syncthreads();
    if (lo >= hi) continue;
    for (int sub = 0; sub < kEmbChunk; sub += 32) {
      const int v = rel[sub + lane];
      unsigned mask = __ballot_sync(0xffffffffu, v >= lo && v < hi);
      while (mask) {
        const int src = __ffs(mask) - 1;
        const int row = __shfl_sync(0xffffffffu, v, src);
        const unsigned same = __ballot_sync(0xffffffffu, v == row) & mask;
        mask &= ~same;
        float4* w = reinterpret_cast<float4*>(dwte + (size_t)row * H);
        for (int c = lane; c < h4; c += 32) {
          float4 acc = w[c];
          unsigned m2 = same;
          while (m2) {  // positions in increasing order
            const int k = __ffs(m2) - 1;
            m2 &= m2 - 1;
            const float4 d = reinterpret_cast<const float4*>(dout + (size_t)(base + sub + k) * H)[c];
            acc.x += d.x; acc.y += d.y; acc.z += d.z; acc.w += d.w;
          }
          w[c] = acc;
        }
      }
    }
  }
}

__global__ void emb_bwd_pos_kernel(const float* __restrict__ dout, float* __restrict__ dwpe, int B, int S, int H) {
  pdl_trigger();
  pdl_wait();
  const int s = blockIdx.x;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float acc = 0.f;
    for (int b = 0; b < B; ++b) acc += dout[((size_t)b * S + s) * H + c];
    dwpe[(size_t)s * H + c] += acc;
  }
}

int embedding_fwd(const long* ids, const float* wte, const float* wpe, float* out, int rows, int H, int S,
                  long vstart, long vend, cudaStream_t s) {
  if (H % 4) return -1;
  launch_k(emb_fwd_kernel, (rows * 32 + 255) / 256, 256, 0, s, ids, wte, wpe, out, rows, H, S, vstart, vend);
  return (int)cudaGetLastError();
}

int embedding_bwd(const long* ids, const float* dout, float* dwte, float* dwpe, int B, int S, int H, long vstart,
                  long vend, cudaStream_t s) {
  if (H % 4) return -1;
  const int rows = B * S;
  int dev = 0, sms = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long vrows = vend - vstart;
  const int grid = (int)std::max<long>(1, std::min<long>(4L * sms, (vrows + 7) / 8));
  const int rows_per_warp = (int)((vrows + 8L * grid - 1) / (8L * grid));
  launch_k(emb_bwd_tok_kernel, grid, 256, 0, s, ids, dout, dwte, rows, H, vstart, vend, rows_per_warp);
  if (dwpe) launch_k(emb_bwd_pos_kernel, S, 256, 0, s, dout, dwpe, B, S, H);
  return (int)cudaGetLastError();
}

}  // namespace mmb
