// Declarations of every kernel launcher exported by the extension.  Launchers
// return 0 on success, a negative code for a host-side validation failure, or
// a positive cudaError_t.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "gemm_sm100.h"
#include "symm_mem.h"

namespace mmb {

// All-gather push target for the fused tensor-parallel path: the producer of a
// sequence-sharded bf16 activation writes each of its rows straight into every
// TP rank's gathered buffer ([B*S, ld] bf16, peer pointers), then the last CTA
// publishes `epoch` in slot [rank] of every rank's AG flag array.
struct AgPush {
  int world, rank;
  void* dst[8];
  long ld;
  int S, Sl;           // local row r = b*Sl + s  ->  gathered row b*S + rank*Sl + s
  int* flags[8];
  int epoch;
  unsigned* counter;   // local, zero-initialised completion counter
};

int layernorm_fwd(const float* x, const float* gamma, const float* beta, __nv_bfloat16* y, float* mean, float* rstd,
                  int rows, int H, float eps, cudaStream_t s);
int layernorm_bwd_parts(int rows, int H, int num_sms);
int layernorm_bwd(const __nv_bfloat16* dy, const float* x, const float* mean, const float* rstd, const float* gamma,
                  const float* dres, float* dx, float* part, float* dgamma, float* dbeta, int rows, int H,
                  int nparts, cudaStream_t s);

int layernorm_bwd2(const __nv_bfloat16* dy, const float* x, const float* mean, const float* rstd, const float* gamma,
                   const float* dres, float* dx, __nv_bfloat16* dx_bf16, float* part, float* dgamma, float* dbeta,
                   int rows, int H, int nparts, cudaStream_t s);

int layernorm_fwd_push(const float* x, const float* gamma, const float* beta, float* mean, float* rstd, int rows,
                       int H, float eps, const AgPush& push, int num_sms, cudaStream_t s);
int layernorm_bwd_push(const __nv_bfloat16* dy, const float* x, const float* mean, const float* rstd,
                       const float* gamma, const float* dres, float* dx, float* part, float* dgamma, float* dbeta,
                       int rows, int H, int nparts, const AgPush& push, cudaStream_t s);

int tp_ce_allreduce(const float* mx, const float* se, const float* tg_in, int rows, const AgPush& push,
                    const void* slots_local, const int* flags_local, float* lse, float* tg_out, int* err, int num_sms,
                    cudaStream_t s, unsigned long long timeout_ns);
int tp_emb_fwd_push(const long* ids, const float* tok, const float* pos, int rows, int H, long vstart, long vend,
                    const AgPush& push, int num_sms, cudaStream_t s);
int tp_wait_copy(const float* src, float* dst, long n, int add, const int* flags, int world, int epoch, int* err,
                 int num_sms, cudaStream_t s, unsigned long long timeout_ns);
int tp_publish(const float* src, long n, const AgPush& push, int num_sms, cudaStream_t s);
int tp_pos_grad_push(const float* dout, int B, int H, const AgPush& push, int num_sms, cudaStream_t s);
int tp_vec_allreduce(const float* v, float* out, long n, const AgPush& push, const float* slots_local,
                     const int* flags_local, int* err, int num_sms, cudaStream_t s, unsigned long long timeout_ns);
// token-table gradient reading the gradient rows of other ranks' sequence shards (fused TP)
struct EmbPeers {
  const float* src[8];   // each rank's published [B*Sl, H] gradient rows
  const int* flags;      // this rank's flags, one per source rank
  int world, epoch, S, Sl;
};
int embedding_bwd_peers(const long* ids, const EmbPeers& peers, float* dwte, int rows, int H, long vstart, long vend,
                        int* err, cudaStream_t s);
int tp_rs_reduce(const __nv_bfloat16* slots, long slot_stride, int world, const int* flags, int epoch,
                 const float* resid, float* out, __nv_bfloat16* out_bf16, long n, int* err, int num_sms,
                 cudaStream_t s,
                 unsigned long long timeout_ns = 10000000000ull);
int tp_ag_push(const __nv_bfloat16* src, int rows, int H, const AgPush& push, int num_sms, cudaStream_t s);

int ce_merge_stats(const float2* part, long ld_part, int nparts, const __nv_bfloat16* logits, long ld,
                   const long* labels, long vocab_start, int n_valid, int rows, float* out_max, float* out_sum,
                   float* out_tgt, cudaStream_t s);
int ce_fwd_stats(const __nv_bfloat16* logits, long ld, const long* labels, long vocab_start, int n_valid, int rows,
                 float* out_max, float* out_sum, float* out_tgt, cudaStream_t s);
int ce_bwd(__nv_bfloat16* logits, long ld, int n_cols, const long* labels, long vocab_start, int n_valid, int rows,
           const float* lse, const float* scale, cudaStream_t s);

int embedding_fwd(const long* ids, const float* wte, const float* wpe, float* out, int rows, int H, int S,
                  long vstart, long vend, cudaStream_t s);
int embedding_bwd(const long* ids, const float* dout, float* dwte, float* dwpe, int B, int S, int H, long vstart,
                  long vend, cudaStream_t s);

int adamw_flat(float* p, const float* g, float* m, float* v, __nv_bfloat16* pb, long n, float lr, float b1, float b2,
               float eps, float wd, float step_size, float bc2_sqrt, float grad_scale, int num_sms, cudaStream_t s,
               const float* hyper = nullptr);
int adamw_hyper_step(int* step, const float* lr_table, int n_table, double b1, double b2, float* hyper,
                     cudaStream_t s);
int gelu_fwd_bwd_f32(const float* x, float* y, float* g, long n, int num_sms, cudaStream_t s);
int cast_f32_bf16(const float* x, __nv_bfloat16* y, long n, int num_sms, cudaStream_t s);

int flash_attn_fwd(const __nv_bfloat16* qkv, long ld_qkv, int B, int S, int nh, int d, __nv_bfloat16* out,
                   long ld_out, float* lse, float softmax_scale, int* err, cudaStream_t stream);
int flash_attn_fwd_sm100(const __nv_bfloat16* qkv, long ld_qkv, int B, int S, int nh, int d, __nv_bfloat16* out,
                         long ld_out, float* lse, float softmax_scale, int* err, int num_sms, cudaStream_t stream);
int flash_attn_bwd(const __nv_bfloat16* dout, long ld_do, const __nv_bfloat16* qkv, long ld_qkv,
                   const __nv_bfloat16* out, const float* lse, float* delta, float* dq_acc, __nv_bfloat16* dqkv,
                   long ld_dqkv, int B, int S, int nh, int d, float softmax_scale, int* err, int num_sms,
                   cudaStream_t stream, bool one_tile_per_cta = false);
int flash_attn_bwd_sm100_d64(const __nv_bfloat16* dout, long ld_do, const __nv_bfloat16* qkv, long ld_qkv,
                             const float* lse, const float* delta, float* dq_acc, __nv_bfloat16* dqkv, long ld_dqkv,
                             int B, int S, int nh, float softmax_scale, int* err, int num_sms, cudaStream_t stream);

// Fused DP step (fused_dp.cu)
struct DpPeersHost {
  int world, rank;
  void* param[8];
  void* grad[8];
  void* pbf16[8];
  void* sig[8];
};
struct DpStepHost {
  int bucket, epoch;
  long lo, hi;
  float* exp_avg;
  float* exp_avg_sq;
  float lr, b1, b2, eps, wd, step_size, bc2_sqrt, grad_scale;
  unsigned* counter;
  int* err;
  int max_ctas;
  int defer_done;
  const int* epoch_ptr;
  const float* hyper;
  const void* segs;  // int32 [nseg][4]: {begin4, end4, kind, 0} runs of the owned range (nullptr: all kind 2)
  int nseg;
};
int dp_rs_adamw_ag(const DpPeersHost& peers, const DpStepHost& s, cudaStream_t stream);
int dp_gather_master(const DpPeersHost& peers, long start, long end, int num_sms, cudaStream_t stream);
int dp_max_segments();
int dp_wait_done(const void* sig_local, int nbuckets, int world, int epoch, const int* epoch_ptr,
                 unsigned long long timeout_ns, int* err, cudaStream_t stream);
int dp_epoch_step(int* epoch, cudaStream_t stream);
int dp_signal_pad_bytes();

}  // namespace mmb
