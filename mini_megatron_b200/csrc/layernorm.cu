// LayerNorm forward / backward for sm_100a.
//
// Forward : y(bf16) = (x - mean) * rstd * gamma + beta, x fp32 (the fp32
//           residual stream), statistics in fp32; mean/rstd saved for backward.
//           The bf16 output feeds the next GEMM directly (the reference
//           runs nn.LayerNorm in fp32 under autocast and then casts to bf16
//           at every F.linear: model/transformer.py:54-61).
// Backward: dx(fp32) = rstd * (g*dy - mean(g*dy) - xhat*mean(g*dy*xhat))
//           [+ dres: the residual-stream gradient is added in the same pass]
//           dgamma/dbeta: per-warp partial sums (fused into the row pass for
//           H <= 1024, a separate column pass above that), folded by a last
//           kernel that accumulates into the fp32 main-grad buffers.
//
// One warp per row; a row is held in registers as float4 (H/128 per lane) so
// x is read exactly once per pass.
#include <algorithm>

#include "common.cuh"
#include "ops.h"
#include "peer.cuh"

namespace mmb {

template <int NV>  // float4 per lane
__global__ void __launch_bounds__(256) ln_fwd_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                     const float* __restrict__ beta, __nv_bfloat16* __restrict__ y,
                                                     float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                     int rows, int H, float eps) {
  pdl_trigger();
  pdl_wait();
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nvec = H >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * H);
  float4 v[NV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    v[i] = (c < nvec) ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    s += v[i].x + v[i].y + v[i].z + v[i].w;
  }
  const float mean = warp_sum(s) / H;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      const float a = v[i].x - mean, b = v[i].y - mean, cc = v[i].z - mean, d = v[i].w - mean;
      ss += a * a + b * b + cc * cc + d * d;
    }
  }
  const float rstd = rsqrtf(warp_sum(ss) / H + eps);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  uint2* yr = reinterpret_cast<uint2*>(y + (size_t)row * H);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      const float4 g = g4[c], b = b4[c];
      uint2 o;
      o.x = pack_bf16x2((v[i].x - mean) * rstd * g.x + b.x, (v[i].y - mean) * rstd * g.y + b.y);
      o.y = pack_bf16x2((v[i].z - mean) * rstd * g.z + b.z, (v[i].w - mean) * rstd * g.w + b.w);
      yr[c] = o;
    }
  }
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// Forward with the tensor-parallel all-gather fused in: each warp normalises
// rows of this rank's sequence shard and writes the bf16 row into EVERY TP
// rank's gathered buffer (NVLink stores for the peers), then the last CTA
// signals the peers that this rank's shard is complete.
template <int NV>
__global__ void __launch_bounds__(256) ln_fwd_push_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                          const float* __restrict__ beta, float* __restrict__ mean_out,
                                                          float* __restrict__ rstd_out, int rows, int H, float eps,
                                                          const AgPush P) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const int nvec = H >> 2;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows; row += nwarps) {
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * H);
    float4 v[NV];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = lane + 32 * i;
      v[i] = (c < nvec) ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      s += v[i].x + v[i].y + v[i].z + v[i].w;
    }
    const float mean = warp_sum(s) / H;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        const float a = v[i].x - mean, b = v[i].y - mean, cc = v[i].z - mean, d = v[i].w - mean;
        ss += a * a + b * b + cc * cc + d * d;
      }
    }
    const float rstd = rsqrtf(warp_sum(ss) / H + eps);
    const long grow = (long)(row / P.Sl) * P.S + (long)P.rank * P.Sl + row % P.Sl;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        const float4 g = g4[c], b = b4[c];
        uint2 o;
        o.x = pack_bf16x2((v[i].x - mean) * rstd * g.x + b.x, (v[i].y - mean) * rstd * g.y + b.y);
        o.y = pack_bf16x2((v[i].z - mean) * rstd * g.z + b.z, (v[i].w - mean) * rstd * g.w + b.w);
        for (int p = 0; p < P.world; ++p)
          reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(P.dst[p]) + grow * P.ld)[c] = o;
      }
    }
    if (lane == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
  grid_done_signal(P.flags, P.world, P.rank, P.epoch, P.counter);
}

// Row pass.  Every load of a row (x, dy and the residual gradient) is issued
// before the two row reductions, so a warp keeps all of its row's bytes in
// flight at once.  With FUSE_PARAM, each warp also accumulates dgamma/dbeta of
// the rows it visits in its own slice of shared memory (each lane owns its
// columns, so no atomics), and the CTA folds its 8 warps into one partial row
// part[blockIdx.x][0:2H]; keeping these sums out of registers leaves room for
// more resident warps.
template <int NV, bool FUSE_PARAM, bool PUSH = false>
__global__ void __launch_bounds__(256, NV <= 6 ? 3 : 1) ln_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const float* __restrict__ x,
                                                     const float* __restrict__ mean, const float* __restrict__ rstd,
                                                     const float* __restrict__ gamma, const float* __restrict__ dres,
                                                     float* __restrict__ dx, __nv_bfloat16* __restrict__ dx_bf16,
                                                     float* __restrict__ part, int rows, int H, const AgPush P = AgPush{}) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const int nvec = H >> 2;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  extern __shared__ float4 red[];  // FUSE_PARAM: [8 warps][2 * nvec] = (dgamma | dbeta) partial sums
  float4* my_dg = red + wid * 2 * nvec;
  float4* my_db = my_dg + nvec;
  if constexpr (FUSE_PARAM) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) my_dg[c] = my_db[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  for (int r = gw; r < rows; r += nwarps) {
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)r * H);
    const uint2* dyr = reinterpret_cast<const uint2*>(dy + (size_t)r * H);
    const float4* drr = dres ? reinterpret_cast<const float4*>(dres + (size_t)r * H) : nullptr;
    // rows of up to 1024 columns also prefetch the residual gradient; wider rows
    // load it after the reductions to stay within the register file
    constexpr bool kPrefetchRes = NV <= 8;
    float4 xv[NV], dv[kPrefetchRes ? NV : 1];
    uint2 du[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        xv[i] = xr[c];
        du[i] = dyr[c];
        if constexpr (kPrefetchRes) dv[i] = drr ? drr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    const float mu = mean[r], rs = rstd[r];
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        const float4 g = g4[c];
        const float2 d01 = unpack_bf16x2(du[i].x), d23 = unpack_bf16x2(du[i].y);
        xv[i] = make_float4((xv[i].x - mu) * rs, (xv[i].y - mu) * rs, (xv[i].z - mu) * rs, (xv[i].w - mu) * rs);
        const float4 gd = make_float4(d01.x * g.x, d01.y * g.y, d23.x * g.z, d23.y * g.w);
        a += gd.x + gd.y + gd.z + gd.w;
        b += gd.x * xv[i].x + gd.y * xv[i].y + gd.z * xv[i].z + gd.w * xv[i].w;
        if constexpr (FUSE_PARAM) {
          float4 t = my_dg[c];
          t.x += d01.x * xv[i].x; t.y += d01.y * xv[i].y; t.z += d23.x * xv[i].z; t.w += d23.y * xv[i].w;
          my_dg[c] = t;
          float4 u = my_db[c];
          u.x += d01.x; u.y += d01.y; u.z += d23.x; u.w += d23.y;
          my_db[c] = u;
        }
      }
    }
    a = warp_sum(a) / H;
    b = warp_sum(b) / H;
    float4* dxr = reinterpret_cast<float4*>(dx + (size_t)r * H);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        const float4 g = g4[c];
        const float2 d01 = unpack_bf16x2(du[i].x), d23 = unpack_bf16x2(du[i].y);
        float4 res;
        if constexpr (kPrefetchRes) res = dv[i];
        else res = drr ? drr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 o = make_float4(rs * (d01.x * g.x - a - xv[i].x * b) + res.x,
                               rs * (d01.y * g.y - a - xv[i].y * b) + res.y,
                               rs * (d23.x * g.z - a - xv[i].z * b) + res.z,
                               rs * (d23.y * g.w - a - xv[i].w * b) + res.w);
        dxr[c] = o;
        if (dx_bf16 || PUSH) {
          uint2 ob;
          ob.x = pack_bf16x2(o.x, o.y);
          ob.y = pack_bf16x2(o.z, o.w);
          if (dx_bf16) reinterpret_cast<uint2*>(dx_bf16 + (size_t)r * H)[c] = ob;
          if constexpr (PUSH) {
            // all-gather fused in: the bf16 gradient row goes to every TP rank's gathered buffer
            const long grow = (long)(r / P.Sl) * P.S + (long)P.rank * P.Sl + r % P.Sl;
            for (int p = 0; p < P.world; ++p)
              reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(P.dst[p]) + grow * P.ld)[c] = ob;
          }
        }
      }
    }
  }
  if constexpr (FUSE_PARAM) {
    // fold the 8 warps' partial sums: one partial row per CTA
    __syncthreads();
    float4* pg = reinterpret_cast<float4*>(part + (size_t)blockIdx.x * 2 * H);
    for (int c = threadIdx.x; c < 2 * nvec; c += blockDim.x) {
      float4 acc = red[c];
#pragma unroll
      for (int w = 1; w < 8; ++w) {
        const float4 t = red[w * 2 * nvec + c];
        acc.x += t.x; acc.y += t.y; acc.z += t.z; acc.w += t.w;
      }
      pg[c] = acc;
    }
  }
  if constexpr (PUSH) grid_done_signal(P.flags, P.world, P.rank, P.epoch, P.counter);
}

// Column pass for wide rows: CTA (band, column block of 256 columns); each
// thread owns one column and walks the band's rows.
__global__ void __launch_bounds__(256) ln_param_part_kernel(const __nv_bfloat16* __restrict__ dy,
                                                            const float* __restrict__ x, const float* __restrict__ mean,
                                                            const float* __restrict__ rstd, float* __restrict__ part,
                                                            int rows, int H, int rows_per_band) {
  pdl_trigger();
  pdl_wait();
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= H) return;
  const int r0 = blockIdx.x * rows_per_band, r1 = min(rows, r0 + rows_per_band);
  float g = 0.f, b = 0.f;
  for (int r = r0; r < r1; ++r) {
    const float d = __bfloat162float(dy[(size_t)r * H + c]);
    g += d * (x[(size_t)r * H + c] - mean[r]) * rstd[r];
    b += d;
  }
  part[(size_t)blockIdx.x * 2 * H + c] = g;
  part[(size_t)blockIdx.x * 2 * H + H + c] = b;
}

// main_grad[gamma] += sum_p part[p][0:H]; main_grad[beta] += sum_p part[p][H:2H]
// Grid (column blocks, row groups): each CTA folds a slice of the partial rows
// for 256 columns and adds it to the main grads with one atomic per column.
constexpr int kLnFoldGroups = 32;
__global__ void ln_param_grad_kernel(const float* __restrict__ part, int nparts, int H, float* __restrict__ dgamma,
                                     float* __restrict__ dbeta) {
  pdl_trigger();
  pdl_wait();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= 2 * H) return;
  const int per = (nparts + gridDim.y - 1) / gridDim.y;
  const int p0 = blockIdx.y * per, p1 = min(nparts, p0 + per);
  if (p0 >= p1) return;
  float acc = 0.f;
  for (int p = p0; p < p1; ++p) acc += part[(size_t)p * 2 * H + c];
  atomicAdd(c < H ? &dgamma[c] : &dbeta[c - H], acc);
}

int layernorm_fwd(const float* x, const float* gamma, const float* beta, __nv_bfloat16* y, float* mean, float* rstd,
                  int rows, int H, float eps, cudaStream_t s) {
  if (H % 4 != 0 || H > 4096) return -1;
  const int threads = 256;
  const int blocks = (rows * 32 + threads - 1) / threads;
  const int nv = (H / 4 + 31) / 32;
#define LN_FWD(NVV) launch_k(ln_fwd_kernel<NVV>, blocks, threads, 0, s, x, gamma, beta, y, mean, rstd, rows, H, eps)
  if (nv <= 2) LN_FWD(2);
  else if (nv <= 6) LN_FWD(6);
  else if (nv <= 8) LN_FWD(8);
  else if (nv <= 16) LN_FWD(16);
  else LN_FWD(32);
#undef LN_FWD
  return (int)cudaGetLastError();
}

// Number of fp32 [2H] partial rows the backward needs as scratch.
// Static shared memory a row-pass kernel may add on top of its dynamic
// partial-sum buffer (the completion word of the all-gather push variant);
// above 48 KB in total the dynamic size must be opted in explicitly.
constexpr int kLnStaticSmem = 256;

// CTAs of the fused row pass that are resident at once: the row pass uses exactly that many
// (one wave; a partial second wave of CTAs, each walking its rows in sequence, would leave
// most SMs idle for its whole length).
template <int NV>
static int ln_bwd_resident(int H, int num_sms) {
  static int cached_h = -1, n = 0;  // the occupancy depends on H through the shared-memory size
  const int smem = 8 * 2 * (H / 4) * 16;
  if (cached_h != H) {
    cached_h = H;
    if (smem + kLnStaticSmem > 48 * 1024)
      cudaFuncSetAttribute(ln_bwd_kernel<NV, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, ln_bwd_kernel<NV, true>, 256, smem) != cudaSuccess || b < 1)
      b = 1;
    n = b;
  }
  return n * num_sms;
}

int layernorm_bwd_parts(int rows, int H, int num_sms) {
  const int nv = (H / 4 + 31) / 32;
  if (nv <= 8) {  // one partial row per CTA of 8 warps
    const int resident = nv <= 2 ? ln_bwd_resident<2>(H, num_sms)
                                 : (nv <= 6 ? ln_bwd_resident<6>(H, num_sms) : ln_bwd_resident<8>(H, num_sms));
    return std::min(resident, std::max(1, (rows + 7) / 8));
  }
  return std::min(4 * num_sms, std::max(1, rows / 16));  // one per band
}

int layernorm_bwd(const __nv_bfloat16* dy, const float* x, const float* mean, const float* rstd, const float* gamma,
                  const float* dres, float* dx, float* part, float* dgamma, float* dbeta, int rows, int H,
                  int nparts, cudaStream_t s) {
  return layernorm_bwd2(dy, x, mean, rstd, gamma, dres, dx, nullptr, part, dgamma, dbeta, rows, H, nparts, s);
}

int layernorm_bwd2(const __nv_bfloat16* dy, const float* x, const float* mean, const float* rstd, const float* gamma,
                   const float* dres, float* dx, __nv_bfloat16* dx_bf16, float* part, float* dgamma, float* dbeta,
                   int rows, int H, int nparts, cudaStream_t s) {
  if (H % 4 != 0 || H > 4096) return -1;
  const int nv = (H / 4 + 31) / 32;
  if (nv <= 8) {
    const int blocks = nparts;  // one partial row per CTA
    const int smem = 8 * 2 * (H / 4) * 16;
#define LN_BWD(NVV)                                                                                      \
  do {                                                                                                   \
    if (smem + kLnStaticSmem > 48 * 1024)                                                                \
      cudaFuncSetAttribute(ln_bwd_kernel<NVV, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); \
    launch_k(ln_bwd_kernel<NVV, true>, blocks, 256, smem, s, dy, x, mean, rstd, gamma, dres, dx, dx_bf16, part, rows, H, AgPush{}); \
  } while (0)
    if (nv <= 2) LN_BWD(2);
    else if (nv <= 6) LN_BWD(6);
    else LN_BWD(8);
#undef LN_BWD
  } else {
    const int blocks = std::max(1, (rows * 32 + 255) / 256);
    if (nv <= 16)
      launch_k(ln_bwd_kernel<16, false>, std::min(blocks, 1184), 256, 0, s, dy, x, mean, rstd, gamma, dres, dx, dx_bf16,
                                                                         nullptr, rows, H, AgPush{});
    else
      launch_k(ln_bwd_kernel<32, false>, std::min(blocks, 1184), 256, 0, s, dy, x, mean, rstd, gamma, dres, dx, dx_bf16,
                                                                         nullptr, rows, H, AgPush{});
    const int rows_per_band = (rows + nparts - 1) / nparts;
    dim3 grid(nparts, (H + 255) / 256);
    launch_k(ln_param_part_kernel, grid, 256, 0, s, dy, x, mean, rstd, part, rows, H, rows_per_band);
  }
  dim3 fold((2 * H + 255) / 256, std::min(kLnFoldGroups, nparts));
  launch_k(ln_param_grad_kernel, fold, 256, 0, s, part, nparts, H, dgamma, dbeta);
  return (int)cudaGetLastError();
}

int layernorm_fwd_push(const float* x, const float* gamma, const float* beta, float* mean, float* rstd, int rows,
                       int H, float eps, const AgPush& push, int num_sms, cudaStream_t s) {
  if (H % 4 != 0 || H > 4096 || push.world < 1 || push.world > 8 || push.Sl <= 0) return -1;
  const int blocks = std::max(1, std::min((rows + 7) / 8, 4 * num_sms));
  const int nv = (H / 4 + 31) / 32;
#define LN_FWDP(NVV) launch_k(ln_fwd_push_kernel<NVV>, blocks, 256, 0, s, x, gamma, beta, mean, rstd, rows, H, eps, push)
  if (nv <= 2) LN_FWDP(2);
  else if (nv <= 6) LN_FWDP(6);
  else if (nv <= 8) LN_FWDP(8);
  else if (nv <= 16) LN_FWDP(16);
  else LN_FWDP(32);
#undef LN_FWDP
  return (int)cudaGetLastError();
}

int layernorm_bwd_push(const __nv_bfloat16* dy, const float* x, const float* mean, const float* rstd,
                       const float* gamma, const float* dres, float* dx, float* part, float* dgamma, float* dbeta,
                       int rows, int H, int nparts, const AgPush& push, cudaStream_t s) {
  if (H % 4 != 0 || H > 4096 || push.world < 1 || push.world > 8 || push.Sl <= 0) return -1;
  const int nv = (H / 4 + 31) / 32;
  if (nv <= 8) {
    const int smem = 8 * 2 * (H / 4) * 16;
#define LN_BWDP(NVV)                                                                                               \
  do {                                                                                                             \
    if (smem + kLnStaticSmem > 48 * 1024)                                                                          \
      cudaFuncSetAttribute(ln_bwd_kernel<NVV, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);     \
    launch_k(ln_bwd_kernel<NVV, true, true>, nparts, 256, smem, s, dy, x, mean, rstd, gamma, dres, dx, nullptr, part, rows, \
                                                             H, push);                                              \
  } while (0)
    if (nv <= 2) LN_BWDP(2);
    else if (nv <= 6) LN_BWDP(6);
    else LN_BWDP(8);
#undef LN_BWDP
  } else {
    const int blocks = std::min(std::max(1, (rows * 32 + 255) / 256), 1184);
    if (nv <= 16)
      launch_k(ln_bwd_kernel<16, false, true>, blocks, 256, 0, s, dy, x, mean, rstd, gamma, dres, dx, nullptr, nullptr, rows,
                                                             H, push);
    else
      launch_k(ln_bwd_kernel<32, false, true>, blocks, 256, 0, s, dy, x, mean, rstd, gamma, dres, dx, nullptr, nullptr, rows,
                                                             H, push);
    const int rows_per_band = (rows + nparts - 1) / nparts;
    dim3 grid(nparts, (H + 255) / 256);
    launch_k(ln_param_part_kernel, grid, 256, 0, s, dy, x, mean, rstd, part, rows, H, rows_per_band);
  }
  dim3 fold((2 * H + 255) / 256, std::min(kLnFoldGroups, nparts));
  launch_k(ln_param_grad_kernel, fold, 256, 0, s, part, nparts, H, dgamma, dbeta);
  return (int)cudaGetLastError();
}

}  // namespace mmb
