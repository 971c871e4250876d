// Vocab-parallel token + learned-position embedding for sm_100a.
//
// Forward : out[r] = (vocab_start <= id < vocab_end ? wte[id - vocab_start] : 0)
//                    + (add_pos ? wpe[r % S] : 0)          (fp32, one warp per row)
//           Under TP the caller all-reduces `out`; only TP rank 0 adds the
//           position term so the sum is the reference's tok + pos
//           (model/embedding.py:11-16, parallel/tensor_parallel.py:99-105).
// Backward: dwte[id - vocab_start] += dout[r] (vector fp32 atomics, rows whose
//           id is outside the shard are skipped); dwpe[s] += sum_b dout[b*S+s]
//           (a column kernel, no atomics).  Both accumulate into main grads.
#include "common.cuh"
#include "ops.h"

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

__global__ void emb_bwd_tok_kernel(const long* __restrict__ ids, const float* __restrict__ dout,
                                   float* __restrict__ dwte, int rows, int H, long vstart, long vend) {
  pdl_trigger();
  pdl_wait();
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const long id = ids[row];
  if (id < vstart || id >= vend) return;
  const float4* d = reinterpret_cast<const float4*>(dout + (size_t)row * H);
  float4* w = reinterpret_cast<float4*>(dwte + (size_t)(id - vstart) * H);
  for (int c = lane; c < H / 4; c += 32) atomicAdd(w + c, d[c]);
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
  launch_k(emb_bwd_tok_kernel, (rows * 32 + 255) / 256, 256, 0, s, ids, dout, dwte, rows, H, vstart, vend);
  if (dwpe) launch_k(emb_bwd_pos_kernel, S, 256, 0, s, dout, dwpe, B, S, H);
  return (int)cudaGetLastError();
}

}  // namespace mmb
