// Single-pass AdamW over a flat fp32 parameter buffer (sm_100a).
//
// All parameters of a model chunk live in one contiguous fp32 buffer (with
// matching flat grad / exp_avg / exp_avg_sq buffers), so the whole optimizer
// step is ONE launch: read p, g, m, v; write p, m, v and the bf16 shadow
// copy that the GEMMs consume.  That removes both the foreach kernel chain
// of torch.optim.AdamW and the per-GEMM fp32->bf16 weight casts of autocast.
//
// Update (same order of operations as torch.optim.AdamW, decoupled decay):
//   g  = g * grad_scale
//   p  = p * (1 - lr*wd)
//   m  = m + (1-b1) * (g - m)
//   v  = b2*v + (1-b2)*g*g
//   p  = p - (lr/bc1) * m / (sqrt(v)/sqrt(bc2) + eps)
#include "common.cuh"
#include "ops.h"
#include <algorithm>

namespace mmb {

__global__ void __launch_bounds__(256) adamw_kernel(float* __restrict__ p, const float* __restrict__ g,
                                                    float* __restrict__ m, float* __restrict__ v,
                                                    __nv_bfloat16* __restrict__ pb, long n, float lr, float b1,
                                                    float b2, float eps, float wd, float step_size,
                                                    float bc2_sqrt, float grad_scale,
                                                    const float* __restrict__ hyper) {
  pdl_trigger();
  pdl_wait();
  if (hyper) {  // step-dependent scalars from device memory (CUDA-graph replays)
    lr = hyper[0];
    step_size = hyper[1];
    bc2_sqrt = hyper[2];
  }
  const long n4 = n >> 2;
  const float decay = 1.f - lr * wd;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    const float4 gg = reinterpret_cast<const float4*>(g)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* P = &pp.x;
    const float* G = &gg.x;
    float* Mv = &mm.x;
    float* V = &vv.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float gr = G[e] * grad_scale;
      float pe = P[e] * decay;
      Mv[e] = Mv[e] + (1.f - b1) * (gr - Mv[e]);
      V[e] = V[e] * b2 + (1.f - b2) * gr * gr;
      const float denom = sqrtf(V[e]) / bc2_sqrt + eps;
      P[e] = pe - step_size * (Mv[e] / denom);
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (pb) {
      uint2 o;
      o.x = pack_bf16x2(pp.x, pp.y);
      o.y = pack_bf16x2(pp.z, pp.w);
      reinterpret_cast<uint2*>(pb)[i] = o;
    }
  }
  // scalar tail
  for (long i = (n4 << 2) + blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float gr = g[i] * grad_scale;
    float pe = p[i] * decay;
    m[i] = m[i] + (1.f - b1) * (gr - m[i]);
    v[i] = v[i] * b2 + (1.f - b2) * gr * gr;
    pe = pe - step_size * (m[i] / (sqrtf(v[i]) / bc2_sqrt + eps));
    p[i] = pe;
    if (pb) pb[i] = __float2bfloat16(pe);
  }
}

// Advances the device step counter and derives this step's scalars, so that a
// captured optimizer step replays correctly: lr = lr_table[step - 1] (the
// schedule's value for this step, clamped to the table's end), then
// hyper = {lr, lr / (1 - b1^step), sqrt(1 - b2^step)}.
__global__ void adamw_hyper_kernel(int* __restrict__ step, const float* __restrict__ lr_table, int n_table, double b1,
                                   double b2, float* __restrict__ hyper) {
  pdl_trigger();
  pdl_wait();
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  const int s = *step + 1;
  *step = s;
  const float lr = lr_table[min(s - 1, n_table - 1)];
  hyper[0] = lr;
  hyper[1] = (float)((double)lr / (1.0 - pow(b1, (double)s)));
  hyper[2] = (float)sqrt(1.0 - pow(b2, (double)s));
}

int adamw_hyper_step(int* step, const float* lr_table, int n_table, double b1, double b2, float* hyper,
                     cudaStream_t s) {
  if (n_table < 1) return -1;
  launch_k(adamw_hyper_kernel, 1, 32, 0, s, step, lr_table, n_table, b1, b2, hyper);
  return (int)cudaGetLastError();
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, long n) {
  pdl_trigger();
  pdl_wait();
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16(x[i]);
}

int adamw_flat(float* p, const float* g, float* m, float* v, __nv_bfloat16* pb, long n, float lr, float b1, float b2,
               float eps, float wd, float step_size, float bc2_sqrt, float grad_scale, int num_sms, cudaStream_t s,
               const float* hyper) {
  if ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(m) |
       reinterpret_cast<uintptr_t>(v)) & 15)
    return -1;
  if (pb && (reinterpret_cast<uintptr_t>(pb) & 7)) return -2;
  const long n4 = (n + 3) / 4;
  const int blocks = (int)std::min<long>((n4 + 255) / 256, (long)num_sms * 8);
  launch_k(adamw_kernel, std::max(blocks, 1), 256, 0, s, p, g, m, v, pb, n, lr, b1, b2, eps, wd, step_size, bc2_sqrt,
                                                   grad_scale, hyper);
  return (int)cudaGetLastError();
}

int cast_f32_bf16(const float* x, __nv_bfloat16* y, long n, int num_sms, cudaStream_t s) {
  const int blocks = (int)std::min<long>((n + 255) / 256, (long)num_sms * 8);
  launch_k(f32_to_bf16_kernel, std::max(blocks, 1), 256, 0, s, x, y, n);
  return (int)cudaGetLastError();
}

}  // namespace mmb

namespace mmb {

// y = gelu(x), g = gelu'(x) in fp32 (the epilogue math, exposed for accuracy checks)
__global__ void gelu_fwd_bwd_kernel(const float* __restrict__ x, float* __restrict__ y, float* __restrict__ g, long n) {
  pdl_trigger();
  pdl_wait();
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    y[i] = gelu_f(x[i]);
    g[i] = gelu_grad_f(x[i]);
  }
}

int gelu_fwd_bwd_f32(const float* x, float* y, float* g, long n, int num_sms, cudaStream_t s) {
  const int blocks = (int)std::min<long>((n + 255) / 256, (long)num_sms * 8);
  launch_k(gelu_fwd_bwd_kernel, std::max(blocks, 1), 256, 0, s, x, y, g, n);
  return (int)cudaGetLastError();
}

}  // namespace mmb
