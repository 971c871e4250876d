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
#include "peer.cuh"

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
// CTA c owns the table rows [c * R, (c + 1) * R) of this vocabulary shard.  It
// reads every token id once (thread t takes a contiguous run of positions, so
// a block-wide exclusive scan of the per-thread match counts lays the matching
// positions out in shared memory in increasing position order), then warp w
// walks that list and handles the rows with row % 8 == w: for each distinct row
// among 32 consecutive entries it adds the sum of those positions' gradient
// rows, in position order, to the row of the main grad.  Every element is thus
// summed in one fixed order, run after run.  The list holds kEmbList entries;
// a CTA with more matches (a very skewed batch) handles its positions in
// several windows, still in order.
constexpr int kEmbList = 4096;
constexpr int kEmbThreads = 256;

// PEERS: the gradient rows are spread over the TP ranks by sequence shard (row p of the full
// [B*S, H] gradient is local row (p / S) * Sl + p % S - o * Sl of rank o = (p % S) / Sl) and
// read from there over NVLink once every rank has published its rows.
template <bool PEERS>
__global__ void __launch_bounds__(kEmbThreads) emb_bwd_tok_kernel(const long* __restrict__ ids,
                                                                  const float* __restrict__ dout,
                                                                  float* __restrict__ dwte, int rows, int H,
                                                                  long vstart, long vend, int rows_per_cta,
                                                                  const EmbPeers peers, int* err) {
  pdl_trigger();
  pdl_wait();
  if constexpr (PEERS) {
    if (!cta_wait_flags(peers.flags, peers.world, peers.epoch, err)) return;
  }
  auto grad_row = [&](int p) -> const float* {
    if constexpr (PEERS) {
      const int s = p % peers.S, o = s / peers.Sl;
      return peers.src[o] + ((size_t)(p / peers.S) * peers.Sl + (s - o * peers.Sl)) * H;
    } else {
      return dout + (size_t)p * H;
    }
  };
  __shared__ int list_pos[kEmbList];
  __shared__ int list_row[kEmbList];
  __shared__ int warp_tot[kEmbThreads / 32];
  __shared__ int total_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long lo = (long)blockIdx.x * rows_per_cta;
  const long hi = min(lo + rows_per_cta, vend - vstart);
  if (lo >= hi) return;
  const int h4 = H / 4;
  // positions per window: each thread scans `per` consecutive positions of the window
  const int per = (kEmbList + kEmbThreads - 1) / kEmbThreads;  // at most kEmbList matches per window
  const int win = per * kEmbThreads;
  for (int w0 = 0; w0 < rows; w0 += win) {
    const int p0 = w0 + tid * per;
    int cnt = 0;
    for (int k = 0; k < per; ++k) {
      const int p = p0 + k;
      if (p < rows) {
        const long v = ids[p] - vstart;
        cnt += (v >= lo && v < hi) ? 1 : 0;
      }
    }
    // block-wide exclusive scan of the counts (warp shuffles, then the 8 warp totals)
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int off = incl - cnt;
    for (int w = 0; w < warp; ++w) off += warp_tot[w];
    if (tid == kEmbThreads - 1) total_s = off + cnt;
    for (int k = 0; k < per && cnt > 0; ++k) {
      const int p = p0 + k;
      if (p < rows) {
        const long v = ids[p] - vstart;
        if (v >= lo && v < hi) {
          list_pos[off] = p;
          list_row[off] = (int)v;
          ++off;
        }
      }
    }
    __syncthreads();
    const int total = total_s;
    // warp `warp` owns the rows with row % 8 == warp; entries are in increasing position order
    for (int b = 0; b < total; b += 32) {
      const int e = b + lane;
      const int row = e < total ? list_row[e] : -1;
      unsigned mask = __ballot_sync(0xffffffffu, row >= 0 && (row & 7) == warp);
      while (mask) {
        const int src = __ffs(mask) - 1;
        const int r = __shfl_sync(0xffffffffu, row, src);
        const unsigned same = __ballot_sync(0xffffffffu, row == r) & mask;
        mask &= ~same;
        float4* wrow = reinterpret_cast<float4*>(dwte + (size_t)r * H);
        for (int c = lane; c < h4; c += 32) {
          float4 acc = wrow[c];
          unsigned m2 = same;
          while (m2) {
            const int k = __ffs(m2) - 1;
            m2 &= m2 - 1;
            const float4 d = reinterpret_cast<const float4*>(grad_row(list_pos[b + k]))[c];
            acc.x += d.x; acc.y += d.y; acc.z += d.z; acc.w += d.w;
          }
          wrow[c] = acc;
        }
      }
    }
    __syncthreads();  // the list is rebuilt for the next window
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
  const int grid = (int)std::max<long>(1, std::min<long>(2L * sms, (vrows + 63) / 64));
  const int rows_per_cta = (int)((vrows + grid - 1) / grid);
  launch_k(emb_bwd_tok_kernel<false>, grid, kEmbThreads, 0, s, ids, dout, dwte, rows, H, vstart, vend, rows_per_cta,
           EmbPeers{}, (int*)nullptr);
  if (dwpe) launch_k(emb_bwd_pos_kernel, S, 256, 0, s, dout, dwpe, B, S, H);
  return (int)cudaGetLastError();
}

int embedding_bwd_peers(const long* ids, const EmbPeers& peers, float* dwte, int rows, int H, long vstart, long vend,
                        int* err, cudaStream_t s) {
  if (H % 4 || peers.world < 1 || peers.world > 8 || peers.Sl <= 0 || peers.S % peers.Sl) return -1;
  int dev = 0, sms = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long vrows = vend - vstart;
  const int grid = (int)std::max<long>(1, std::min<long>(2L * sms, (vrows + 63) / 64));
  const int rows_per_cta = (int)((vrows + grid - 1) / grid);
  launch_k(emb_bwd_tok_kernel<true>, grid, kEmbThreads, 0, s, ids, (const float*)nullptr, dwte, rows, H, vstart, vend,
           rows_per_cta, peers, err);
  return (int)cudaGetLastError();
}

}  // namespace mmb
