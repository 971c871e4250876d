// Python bindings for the sm_100a kernels.  Only this translation unit
// includes the torch headers; kernels live in plain .cu files.
#include <execinfo.h>
#include <signal.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <cstdio>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>
#include <vector>

#include "ops.h"

namespace {

using at::Tensor;

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

int num_sms() {
  static int n = 0;
  if (n == 0) n = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  return n;
}

// One device error word per device; kernels record bounded-wait timeouts here.
int* error_word() {
  static std::vector<Tensor> words;
  const int dev = at::cuda::current_device();
  if ((int)words.size() <= dev) words.resize(dev + 1);
  if (!words[dev].defined())
    words[dev] = at::zeros({4}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, dev));
  return words[dev].data_ptr<int>();
}

int64_t get_error() {
  int h = 0;
  C10_CUDA_CHECK(cudaMemcpy(&h, error_word(), sizeof(int), cudaMemcpyDeviceToHost));
  return h;
}

void clear_error() { C10_CUDA_CHECK(cudaMemset(error_word(), 0, sizeof(int))); }

// Host-side write of the error word: lets tests check that the host notices a
// recorded kernel error without making any kernel time out.
void set_error(int64_t code) {
  const int h = (int)code;
  C10_CUDA_CHECK(cudaMemcpy(error_word(), &h, sizeof(int), cudaMemcpyHostToDevice));
}

// ----------------------------------------------------------------- GEMM
void gemm(const Tensor& A, bool a_mn, const Tensor& B, bool b_mn, Tensor& D, int64_t epi,
          const c10::optional<Tensor>& aux, const c10::optional<Tensor>& resid, double alpha, int64_t bn,
          int64_t cg) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  check_cuda(D, "D");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && D.dim() == 2, "gemm expects 2-D operands");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm operands must be bf16");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && D.stride(1) == 1, "gemm operands must be row-major");
  const int64_t M = a_mn ? A.size(1) : A.size(0);
  const int64_t K = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0);
  const int64_t Kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(K == Kb, "gemm: K mismatch ", K, " vs ", Kb);
  TORCH_CHECK(D.size(0) == M && D.size(1) == N, "gemm: D shape mismatch");
  const bool out_bf16 = (epi == mmb::EPI_BF16 || epi == mmb::EPI_GELU || epi == mmb::EPI_DGELU);
  TORCH_CHECK(D.scalar_type() == (out_bf16 ? at::kBFloat16 : at::kFloat), "gemm: wrong output dtype for epilogue");
  TORCH_CHECK(N % 8 == 0, "gemm: N must be a multiple of 8");
  const at::cuda::CUDAGuard guard(A.device());

  mmb::GemmProblem p{};
  p.A = A.data_ptr();
  p.lda = A.stride(0);
  p.a_mn = a_mn;
  p.B = B.data_ptr();
  p.ldb = B.stride(0);
  p.b_mn = b_mn;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.bn = (int)bn;
  p.cg = (int)cg;
  p.num_sms = num_sms();
  p.allow_split = true;
  p.args.epi = (int)epi;
  p.args.D = D.data_ptr();
  p.args.ldd = D.stride(0);
  p.args.alpha = (float)alpha;
  p.args.err = error_word();
  p.args.aux = nullptr;
  p.args.resid = nullptr;
  if (epi == mmb::EPI_GELU || epi == mmb::EPI_DGELU) {
    TORCH_CHECK(aux.has_value(), "gemm: epilogue needs aux");
    const Tensor& x = *aux;
    TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.size(0) == M && x.size(1) == N &&
                    x.stride(1) == 1 && x.stride(0) % 8 == 0,
                "gemm: bad aux");
    p.args.aux = x.data_ptr();
    p.args.ld_aux = x.stride(0);
  }
  if (epi == mmb::EPI_RESID) {
    TORCH_CHECK(resid.has_value(), "gemm: epilogue needs resid");
    const Tensor& r = *resid;
    TORCH_CHECK(r.scalar_type() == at::kFloat && r.dim() == 2 && r.size(0) == M && r.size(1) == N &&
                    r.stride(1) == 1 && r.stride(0) % 4 == 0,
                "gemm: bad resid");
    p.args.resid = r.data_ptr<float>();
    p.args.ld_resid = r.stride(0);
  }
  TORCH_CHECK(D.stride(0) % (out_bf16 ? 8 : 4) == 0, "gemm: D leading dim must be 16-byte aligned");
  const int rc = mmb::gemm_bf16_launch(p, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "gemm launch failed, code ", rc);
}

#define MMB_CHECK_RC(rc, what) TORCH_CHECK((rc) == 0, what " failed, code ", (rc))

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

void check_f32(const Tensor& t, const char* n) {
  check_cuda(t, n);
  TORCH_CHECK(t.scalar_type() == at::kFloat && t.is_contiguous(), n, " must be contiguous fp32");
}
void check_bf16(const Tensor& t, const char* n) {
  check_cuda(t, n);
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 && t.is_contiguous(), n, " must be contiguous bf16");
}

// ----------------------------------------------------------------- LayerNorm
// x [rows, H] fp32 -> y bf16, mean/rstd fp32 [rows]
void layernorm_fwd(const Tensor& x, const Tensor& gamma, const Tensor& beta, Tensor& y, Tensor& mean, Tensor& rstd,
                   double eps) {
  check_f32(x, "x");
  check_f32(gamma, "gamma");
  check_f32(beta, "beta");
  check_bf16(y, "y");
  const int H = (int)x.size(-1);
  const int rows = (int)(x.numel() / H);
  const int rc = mmb::layernorm_fwd(x.data_ptr<float>(), gamma.data_ptr<float>(), beta.data_ptr<float>(),
                                    reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), mean.data_ptr<float>(),
                                    rstd.data_ptr<float>(), rows, H, (float)eps, cur_stream());
  MMB_CHECK_RC(rc, "layernorm_fwd");
}

// dx = LN_bwd(dy) (+ dres); dgamma/dbeta accumulated (+=) into the given fp32 buffers.
void layernorm_bwd(const Tensor& dy, const Tensor& x, const Tensor& mean, const Tensor& rstd, const Tensor& gamma,
                   const c10::optional<Tensor>& dres, Tensor& dx, Tensor& dgamma, Tensor& dbeta,
                   const c10::optional<Tensor>& dx_bf16) {
  check_bf16(dy, "dy");
  check_f32(x, "x");
  check_f32(dx, "dx");
  const int H = (int)x.size(-1);
  const int rows = (int)(x.numel() / H);
  const int nparts = mmb::layernorm_bwd_parts(rows, H, num_sms());
  Tensor part = at::empty({nparts, 2 * H}, x.options());
  const float* dr = nullptr;
  if (dres.has_value()) {
    check_f32(*dres, "dres");
    dr = dres->data_ptr<float>();
  }
  __nv_bfloat16* xb = nullptr;
  if (dx_bf16.has_value()) {
    check_bf16(*dx_bf16, "dx_bf16");
    TORCH_CHECK(dx_bf16->numel() == dx.numel(), "dx_bf16 size mismatch");
    xb = reinterpret_cast<__nv_bfloat16*>(dx_bf16->data_ptr());
  }
  const int rc = mmb::layernorm_bwd2(reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), x.data_ptr<float>(),
                                     mean.data_ptr<float>(), rstd.data_ptr<float>(), gamma.data_ptr<float>(), dr,
                                     dx.data_ptr<float>(), xb, part.data_ptr<float>(), dgamma.data_ptr<float>(),
                                     dbeta.data_ptr<float>(), rows, H, nparts, cur_stream());
  MMB_CHECK_RC(rc, "layernorm_bwd");
}

// ----------------------------------------------------------------- cross-entropy
std::vector<Tensor> ce_fwd_stats(const Tensor& logits, const Tensor& labels, int64_t vocab_start, int64_t n_valid) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1 && logits.scalar_type() == at::kBFloat16, "bad logits");
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous(), "labels must be int64");
  const int rows = (int)logits.size(0);
  auto opt = logits.options().dtype(at::kFloat);
  Tensor mx = at::empty({rows}, opt), sm = at::empty({rows}, opt), tg = at::empty({rows}, opt);
  const int rc = mmb::ce_fwd_stats(reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
                                   labels.data_ptr<int64_t>(), vocab_start, (int)n_valid, rows, mx.data_ptr<float>(),
                                   sm.data_ptr<float>(), tg.data_ptr<float>(), cur_stream());
  MMB_CHECK_RC(rc, "ce_fwd_stats");
  return {mx, sm, tg};
}

void ce_bwd(Tensor& logits, const Tensor& labels, int64_t vocab_start, int64_t n_valid, const Tensor& lse,
            const Tensor& scale) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1 && logits.scalar_type() == at::kBFloat16, "bad logits");
  check_f32(lse, "lse");
  check_f32(scale, "scale");
  const int rc = mmb::ce_bwd(reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
                             (int)logits.size(1), labels.data_ptr<int64_t>(), vocab_start, (int)n_valid,
                             (int)logits.size(0), lse.data_ptr<float>(), scale.data_ptr<float>(), cur_stream());
  MMB_CHECK_RC(rc, "ce_bwd");
}

// ----------------------------------------------------------------- embedding
void embedding_fwd(const Tensor& ids, const Tensor& wte, const c10::optional<Tensor>& wpe, Tensor& out, int64_t S,
                   int64_t vstart, int64_t vend) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "ids must be int64");
  check_f32(wte, "wte");
  check_f32(out, "out");
  const int H = (int)wte.size(1);
  const float* p = nullptr;
  if (wpe.has_value()) {
    check_f32(*wpe, "wpe");
    p = wpe->data_ptr<float>();
  }
  const int rc = mmb::embedding_fwd(ids.data_ptr<int64_t>(), wte.data_ptr<float>(), p, out.data_ptr<float>(),
                                    (int)ids.numel(), H, (int)S, vstart, vend, cur_stream());
  MMB_CHECK_RC(rc, "embedding_fwd");
}

void embedding_bwd(const Tensor& ids, const Tensor& dout, Tensor& dwte, const c10::optional<Tensor>& dwpe,
                   int64_t B, int64_t S, int64_t vstart, int64_t vend) {
  check_f32(dout, "dout");
  check_f32(dwte, "dwte");
  float* p = nullptr;
  if (dwpe.has_value()) {
    check_f32(*dwpe, "dwpe");
    p = dwpe->data_ptr<float>();
  }
  const int rc = mmb::embedding_bwd(ids.data_ptr<int64_t>(), dout.data_ptr<float>(), dwte.data_ptr<float>(), p,
                                    (int)B, (int)S, (int)dwte.size(1), vstart, vend, cur_stream());
  MMB_CHECK_RC(rc, "embedding_bwd");
}

// ----------------------------------------------------------------- AdamW
void adamw_flat(Tensor& p, const Tensor& g, Tensor& m, Tensor& v, const c10::optional<Tensor>& pb, double lr,
                double b1, double b2, double eps, double wd, int64_t step, double grad_scale) {
  check_f32(p, "p");
  check_f32(g, "g");
  check_f32(m, "m");
  check_f32(v, "v");
  TORCH_CHECK(p.numel() == g.numel() && p.numel() == m.numel() && p.numel() == v.numel(), "adamw size mismatch");
  __nv_bfloat16* pbp = nullptr;
  if (pb.has_value()) {
    check_bf16(*pb, "pb");
    TORCH_CHECK(pb->numel() == p.numel(), "adamw bf16 shadow size mismatch");
    pbp = reinterpret_cast<__nv_bfloat16*>(pb->data_ptr());
  }
  const double bc1 = 1.0 - std::pow(b1, (double)step);
  const double bc2 = 1.0 - std::pow(b2, (double)step);
  const int rc = mmb::adamw_flat(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                                 pbp, p.numel(), (float)lr, (float)b1, (float)b2, (float)eps, (float)wd,
                                 (float)(lr / bc1), (float)std::sqrt(bc2), (float)grad_scale, num_sms(),
                                 cur_stream());
  MMB_CHECK_RC(rc, "adamw_flat");
}

// AdamW whose lr / bias corrections come from `hyper` (device float[3]) -- the
// form a CUDA graph can replay; `adamw_hyper_step` advances the device step.
void adamw_flat_dev(Tensor& p, const Tensor& g, Tensor& m, Tensor& v, const c10::optional<Tensor>& pb,
                    const Tensor& hyper, double b1, double b2, double eps, double wd, double grad_scale) {
  check_f32(p, "p");
  check_f32(g, "g");
  check_f32(m, "m");
  check_f32(v, "v");
  check_f32(hyper, "hyper");
  TORCH_CHECK(hyper.numel() >= 3, "hyper needs 3 floats");
  TORCH_CHECK(p.numel() == g.numel() && p.numel() == m.numel() && p.numel() == v.numel(), "adamw size mismatch");
  __nv_bfloat16* pbp = nullptr;
  if (pb.has_value()) {
    check_bf16(*pb, "pb");
    TORCH_CHECK(pb->numel() == p.numel(), "adamw bf16 shadow size mismatch");
    pbp = reinterpret_cast<__nv_bfloat16*>(pb->data_ptr());
  }
  const int rc = mmb::adamw_flat(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                                 pbp, p.numel(), 0.f, (float)b1, (float)b2, (float)eps, (float)wd, 0.f, 1.f,
                                 (float)grad_scale, num_sms(), cur_stream(), hyper.data_ptr<float>());
  MMB_CHECK_RC(rc, "adamw_flat_dev");
}

void adamw_hyper_step(Tensor& step, const Tensor& lr_table, double b1, double b2, Tensor& hyper) {
  check_cuda(step, "step");
  TORCH_CHECK(step.scalar_type() == at::kInt && step.numel() == 1, "step must be one int32");
  check_f32(lr_table, "lr_table");
  check_f32(hyper, "hyper");
  MMB_CHECK_RC(mmb::adamw_hyper_step(step.data_ptr<int>(), lr_table.data_ptr<float>(), (int)lr_table.numel(), b1, b2,
                                     hyper.data_ptr<float>(), cur_stream()),
               "adamw_hyper_step");
}

std::vector<Tensor> gelu_fwd_bwd_f32(const Tensor& x) {
  check_f32(x, "x");
  Tensor y = at::empty_like(x), g = at::empty_like(x);
  MMB_CHECK_RC(mmb::gelu_fwd_bwd_f32(x.data_ptr<float>(), y.data_ptr<float>(), g.data_ptr<float>(), x.numel(),
                                     num_sms(), cur_stream()),
               "gelu_fwd_bwd_f32");
  return {y, g};
}

void cast_f32_bf16(const Tensor& x, Tensor& y) {
  check_f32(x, "x");
  check_bf16(y, "y");
  TORCH_CHECK(x.numel() == y.numel(), "cast size mismatch");
  MMB_CHECK_RC(mmb::cast_f32_bf16(x.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), x.numel(),
                                  num_sms(), cur_stream()),
               "cast_f32_bf16");
}

// ----------------------------------------------------------------- attention
// qkv [B*S, 3*nh*d] bf16 (columns [Q heads | K heads | V heads]) -> (out [B*S, nh*d] bf16, lse [B, nh, S] fp32)
std::vector<Tensor> flash_attn_fwd_impl(const Tensor& qkv, int64_t B, int64_t S, int64_t nh, int64_t d, bool v1) {
  check_cuda(qkv, "qkv");
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 2 && qkv.stride(1) == 1, "qkv must be 2-D bf16");
  TORCH_CHECK(qkv.size(0) == B * S && qkv.size(1) == 3 * nh * d, "qkv shape mismatch");
  TORCH_CHECK(S % 128 == 0, "flash attention needs S % 128 == 0");
  TORCH_CHECK(d == 64 || d == 128, "flash attention supports head_dim 64 and 128");
  Tensor out = at::empty({B * S, nh * d}, qkv.options());
  Tensor lse = at::empty({B, nh, S}, qkv.options().dtype(at::kFloat));
  const auto* q = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  const float scale = (float)(1.0 / std::sqrt((double)d));
  const int rc = v1 ? mmb::flash_attn_fwd(q, qkv.stride(0), (int)B, (int)S, (int)nh, (int)d, o, out.stride(0),
                                          lse.data_ptr<float>(), scale, error_word(), cur_stream())
                    : mmb::flash_attn_fwd_sm100(q, qkv.stride(0), (int)B, (int)S, (int)nh, (int)d, o, out.stride(0),
                                                lse.data_ptr<float>(), scale, error_word(), num_sms(), cur_stream());
  MMB_CHECK_RC(rc, "flash_attn_fwd");
  return {out, lse};
}

std::vector<Tensor> flash_attn_fwd(const Tensor& qkv, int64_t B, int64_t S, int64_t nh, int64_t d) {
  return flash_attn_fwd_impl(qkv, B, S, nh, d, false);
}
std::vector<Tensor> flash_attn_fwd_v1(const Tensor& qkv, int64_t B, int64_t S, int64_t nh, int64_t d) {
  return flash_attn_fwd_impl(qkv, B, S, nh, d, true);
}

Tensor flash_attn_bwd_impl(const Tensor& dout, const Tensor& qkv, const Tensor& out, const Tensor& lse, int64_t B,
                           int64_t S, int64_t nh, int64_t d, bool v1) {
  check_bf16(dout, "dout");
  check_bf16(out, "out");
  check_f32(lse, "lse");
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 2 && qkv.stride(1) == 1, "qkv must be 2-D bf16");
  TORCH_CHECK(dout.numel() == B * S * nh * d && out.numel() == B * S * nh * d, "attention bwd shape mismatch");
  TORCH_CHECK(S % 128 == 0 && (d == 64 || d == 128), "unsupported attention shape");
  Tensor dqkv = at::empty({B * S, 3 * nh * d}, qkv.options());
  Tensor delta = at::empty({B, nh, S}, lse.options());
  Tensor dq_acc = at::empty({B * S, nh * d}, lse.options());
  const int rc = mmb::flash_attn_bwd(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), nh * d,
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), lse.data_ptr<float>(), delta.data_ptr<float>(),
      dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), dqkv.stride(0), (int)B, (int)S,
      (int)nh, (int)d, (float)(1.0 / std::sqrt((double)d)), error_word(), num_sms(), cur_stream(), v1);
  MMB_CHECK_RC(rc, "flash_attn_bwd");
  return dqkv;
}

Tensor flash_attn_bwd(const Tensor& dout, const Tensor& qkv, const Tensor& out, const Tensor& lse, int64_t B,
                      int64_t S, int64_t nh, int64_t d) {
  return flash_attn_bwd_impl(dout, qkv, out, lse, B, S, nh, d, false);
}
Tensor flash_attn_bwd_v1(const Tensor& dout, const Tensor& qkv, const Tensor& out, const Tensor& lse, int64_t B,
                         int64_t S, int64_t nh, int64_t d) {
  return flash_attn_bwd_impl(dout, qkv, out, lse, B, S, nh, d, true);
}

// ----------------------------------------------------------------- symmetric memory
int64_t symm_alloc(int64_t bytes) {
  void* p = nullptr;
  MMB_CHECK_RC(mmb::symm_alloc((size_t)bytes, &p), "symm_alloc");
  return reinterpret_cast<int64_t>(p);
}
void symm_free(int64_t ptr) { MMB_CHECK_RC(mmb::symm_free(reinterpret_cast<void*>(ptr)), "symm_free"); }
py::bytes symm_export(int64_t ptr) {
  unsigned char h[64];
  MMB_CHECK_RC(mmb::symm_export(reinterpret_cast<void*>(ptr), h), "symm_export");
  return py::bytes(reinterpret_cast<const char*>(h), 64);
}
int64_t symm_open(py::bytes handle) {
  std::string s = handle;
  TORCH_CHECK(s.size() == 64, "IPC handle must be 64 bytes");
  void* p = nullptr;
  MMB_CHECK_RC(mmb::symm_open(reinterpret_cast<const unsigned char*>(s.data()), &p), "symm_open");
  return reinterpret_cast<int64_t>(p);
}
void symm_close(int64_t ptr) { MMB_CHECK_RC(mmb::symm_close(reinterpret_cast<void*>(ptr)), "symm_close"); }

// A tensor view of device memory owned elsewhere (the caller keeps it alive).
Tensor tensor_from_ptr(int64_t ptr, int64_t numel, at::ScalarType dtype, int64_t device) {
  return torch::from_blob(reinterpret_cast<void*>(ptr), {numel}, [](void*) {},
                          at::TensorOptions().dtype(dtype).device(at::kCUDA, device));
}

// ----------------------------------------------------------------- fused DP step
void dp_rs_adamw_ag(const std::vector<int64_t>& param, const std::vector<int64_t>& grad,
                    const std::vector<int64_t>& pbf16, const std::vector<int64_t>& sig, int64_t rank, int64_t bucket,
                    int64_t epoch, int64_t lo, int64_t hi, Tensor& exp_avg, Tensor& exp_avg_sq, Tensor& counter,
                    double lr, double b1, double b2, double eps, double wd, int64_t step, double grad_scale,
                    int64_t max_ctas, int64_t defer_done, const c10::optional<Tensor>& epoch_dev,
                    const c10::optional<Tensor>& hyper, const c10::optional<Tensor>& segs) {
  const int world = (int)param.size();
  TORCH_CHECK(world >= 1 && world <= 8 && grad.size() == param.size() && pbf16.size() == param.size() &&
                  sig.size() == param.size(),
              "fused DP needs 1..8 ranks");
  check_f32(exp_avg, "exp_avg");
  check_f32(exp_avg_sq, "exp_avg_sq");
  TORCH_CHECK(exp_avg.numel() >= hi - lo && exp_avg_sq.numel() >= hi - lo, "moment buffers too small");
  mmb::DpPeersHost P{};
  P.world = world;
  P.rank = (int)rank;
  for (int r = 0; r < world; ++r) {
    P.param[r] = reinterpret_cast<void*>(param[r]);
    P.grad[r] = reinterpret_cast<void*>(grad[r]);
    P.pbf16[r] = reinterpret_cast<void*>(pbf16[r]);
    P.sig[r] = reinterpret_cast<void*>(sig[r]);
  }
  const double bc1 = 1.0 - std::pow(b1, (double)step), bc2 = 1.0 - std::pow(b2, (double)step);
  mmb::DpStepHost s{};
  s.bucket = (int)bucket;
  s.epoch = (int)epoch;
  s.lo = lo;
  s.hi = hi;
  s.exp_avg = exp_avg.data_ptr<float>();
  s.exp_avg_sq = exp_avg_sq.data_ptr<float>();
  s.lr = (float)lr;
  s.b1 = (float)b1;
  s.b2 = (float)b2;
  s.eps = (float)eps;
  s.wd = (float)wd;
  s.step_size = (float)(lr / bc1);
  s.bc2_sqrt = (float)std::sqrt(bc2);
  s.grad_scale = (float)grad_scale;
  s.counter = reinterpret_cast<unsigned*>(counter.data_ptr<int>());
  s.err = error_word();
  s.max_ctas = (int)max_ctas;
  s.defer_done = defer_done ? 1 : 0;
  if (epoch_dev.has_value()) {
    TORCH_CHECK(epoch_dev->scalar_type() == at::kInt && epoch_dev->is_cuda(), "epoch_dev must be a CUDA int32");
    s.epoch_ptr = epoch_dev->data_ptr<int>();
  }
  if (hyper.has_value()) {
    check_f32(*hyper, "hyper");
    s.hyper = hyper->data_ptr<float>();
  }
  if (segs.has_value()) {
    TORCH_CHECK(segs->is_cuda() && segs->scalar_type() == at::kInt && segs->dim() == 2 && segs->size(1) == 4 &&
                    segs->is_contiguous(),
                "segs: contiguous CUDA int32 [nseg, 4]");
    s.segs = segs->data_ptr<int>();
    s.nseg = (int)segs->size(0);
  }
  MMB_CHECK_RC(mmb::dp_rs_adamw_ag(P, s, cur_stream()), "dp_rs_adamw_ag");
}

void dp_gather_master(const std::vector<int64_t>& param, int64_t rank, int64_t start, int64_t end) {
  const int world = (int)param.size();
  TORCH_CHECK(world >= 1 && world <= 8 && rank >= 0 && rank < world, "fused DP needs 1..8 ranks");
  mmb::DpPeersHost P{};
  P.world = world;
  P.rank = (int)rank;
  for (int r = 0; r < world; ++r) P.param[r] = reinterpret_cast<void*>(param[r]);
  MMB_CHECK_RC(mmb::dp_gather_master(P, start, end, num_sms(), cur_stream()), "dp_gather_master");
}

// ----------------------------------------------------------------- fused tensor parallel
// push = (dst_ptrs[world], flag_ptrs[world], rank, epoch, S, Sl, ld, counter tensor)
mmb::AgPush make_push(const std::vector<int64_t>& dst, const std::vector<int64_t>& flags, int64_t rank,
                      int64_t epoch, int64_t S, int64_t Sl, int64_t ld, Tensor& counter) {
  TORCH_CHECK(dst.size() == flags.size() && dst.size() >= 1 && dst.size() <= 8, "push: 1..8 ranks");
  mmb::AgPush P{};
  P.world = (int)dst.size();
  P.rank = (int)rank;
  for (size_t i = 0; i < dst.size(); ++i) {
    P.dst[i] = reinterpret_cast<void*>(dst[i]);
    P.flags[i] = reinterpret_cast<int*>(flags[i]);
  }
  P.ld = ld;
  P.S = (int)S;
  P.Sl = (int)Sl;
  P.epoch = (int)epoch;
  P.counter = reinterpret_cast<unsigned*>(counter.data_ptr<int>());
  return P;
}

void layernorm_fwd_push(const Tensor& x, const Tensor& gamma, const Tensor& beta, Tensor& mean, Tensor& rstd,
                        double eps, const std::vector<int64_t>& dst, const std::vector<int64_t>& flags, int64_t rank,
                        int64_t epoch, int64_t S, int64_t Sl, Tensor& counter) {
  check_f32(x, "x");
  const int H = (int)x.size(-1);
  const int rows = (int)(x.numel() / H);
  mmb::AgPush P = make_push(dst, flags, rank, epoch, S, Sl, H, counter);
  MMB_CHECK_RC(mmb::layernorm_fwd_push(x.data_ptr<float>(), gamma.data_ptr<float>(), beta.data_ptr<float>(),
                                       mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, H, (float)eps, P,
                                       num_sms(), cur_stream()),
               "layernorm_fwd_push");
}

void layernorm_bwd_push(const Tensor& dy, const Tensor& x, const Tensor& mean, const Tensor& rstd,
                        const Tensor& gamma, const c10::optional<Tensor>& dres, Tensor& dx, Tensor& dgamma,
                        Tensor& dbeta, const std::vector<int64_t>& dst, const std::vector<int64_t>& flags,
                        int64_t rank, int64_t epoch, int64_t S, int64_t Sl, Tensor& counter) {
  check_bf16(dy, "dy");
  check_f32(x, "x");
  check_f32(dx, "dx");
  const int H = (int)x.size(-1);
  const int rows = (int)(x.numel() / H);
  const int nparts = mmb::layernorm_bwd_parts(rows, H, num_sms());
  Tensor part = at::empty({nparts, 2 * H}, x.options());
  const float* dr = dres.has_value() ? dres->data_ptr<float>() : nullptr;
  mmb::AgPush P = make_push(dst, flags, rank, epoch, S, Sl, H, counter);
  MMB_CHECK_RC(mmb::layernorm_bwd_push(reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), x.data_ptr<float>(),
                                       mean.data_ptr<float>(), rstd.data_ptr<float>(), gamma.data_ptr<float>(), dr,
                                       dx.data_ptr<float>(), part.data_ptr<float>(), dgamma.data_ptr<float>(),
                                       dbeta.data_ptr<float>(), rows, H, nparts, P, cur_stream()),
               "layernorm_bwd_push");
}

void tp_ag_push(const Tensor& src, const std::vector<int64_t>& dst, const std::vector<int64_t>& flags, int64_t rank,
                int64_t epoch, int64_t S, int64_t Sl, Tensor& counter) {
  check_bf16(src, "src");
  const int H = (int)src.size(-1);
  const int rows = (int)(src.numel() / H);
  mmb::AgPush P = make_push(dst, flags, rank, epoch, S, Sl, H, counter);
  MMB_CHECK_RC(mmb::tp_ag_push(reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), rows, H, P, num_sms(),
                               cur_stream()),
               "tp_ag_push");
}

// out = resid + sum of `world` bf16 slots [rows_l, H] (slot s at slots_ptr + s*slot_stride elements)
void tp_rs_reduce(int64_t slots_ptr, int64_t slot_stride, int64_t world, int64_t flags_ptr, int64_t epoch,
                  const c10::optional<Tensor>& resid, const c10::optional<Tensor>& out,
                  const c10::optional<Tensor>& out_bf16, int64_t n, int64_t timeout_ms) {
  TORCH_CHECK(timeout_ms > 0, "tp_rs_reduce: timeout_ms must be positive");
  const float* r = resid.has_value() ? resid->data_ptr<float>() : nullptr;
  float* o = out.has_value() ? out->data_ptr<float>() : nullptr;
  __nv_bfloat16* ob = out_bf16.has_value() ? reinterpret_cast<__nv_bfloat16*>(out_bf16->data_ptr()) : nullptr;
  MMB_CHECK_RC(mmb::tp_rs_reduce(reinterpret_cast<const __nv_bfloat16*>(slots_ptr), slot_stride, (int)world,
                                 reinterpret_cast<const int*>(flags_ptr), (int)epoch, r, o, ob, n, error_word(),
                                 num_sms(), cur_stream(), (unsigned long long)timeout_ms * 1000000ull),
               "tp_rs_reduce");
}

// Cross-entropy statistics across the TP group over NVLink: push this rank's (max, sumexp,
// target) triplets into every peer's slots, then reduce all sources into (lse, target logit).
std::vector<Tensor> tp_ce_allreduce(const Tensor& mx, const Tensor& se, const Tensor& tg,
                                    const std::vector<int64_t>& dst, const std::vector<int64_t>& flags, int64_t rank,
                                    int64_t epoch, Tensor& counter, int64_t slots_local, int64_t flags_local,
                                    int64_t timeout_ms) {
  check_f32(mx, "mx");
  check_f32(se, "se");
  check_f32(tg, "tg");
  const int rows = (int)mx.numel();
  TORCH_CHECK(se.numel() == rows && tg.numel() == rows, "tp_ce_allreduce: shapes");
  mmb::AgPush P = make_push(dst, flags, rank, epoch, 1, 1, 4, counter);
  Tensor lse = at::empty_like(mx), tgo = at::empty_like(mx);
  MMB_CHECK_RC(mmb::tp_ce_allreduce(mx.data_ptr<float>(), se.data_ptr<float>(), tg.data_ptr<float>(), rows, P,
                                    reinterpret_cast<const void*>(slots_local),
                                    reinterpret_cast<const int*>(flags_local), lse.data_ptr<float>(),
                                    tgo.data_ptr<float>(), error_word(), num_sms(), cur_stream(),
                                    (unsigned long long)timeout_ms * 1000000ull),
               "tp_ce_allreduce");
  return {lse, tgo};
}

// ---- embedding and sequence-parallel gradients under fused TP (NVLink, no NCCL)
void tp_emb_fwd_push(const Tensor& ids, const Tensor& tok, const Tensor& pos, const std::vector<int64_t>& dst,
                     const std::vector<int64_t>& flags, int64_t rank, int64_t epoch, int64_t S, int64_t Sl,
                     Tensor& counter, int64_t vstart, int64_t vend) {
  check_f32(tok, "tok");
  check_f32(pos, "pos");
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous() && ids.is_cuda(), "ids: contiguous CUDA int64");
  const int H = (int)tok.size(1);
  mmb::AgPush P = make_push(dst, flags, rank, epoch, S, Sl, H, counter);
  MMB_CHECK_RC(mmb::tp_emb_fwd_push(ids.data_ptr<int64_t>(), tok.data_ptr<float>(), pos.data_ptr<float>(),
                                    (int)ids.numel(), H, vstart, vend, P, num_sms(), cur_stream()),
               "tp_emb_fwd_push");
}

void tp_wait_copy(int64_t src, Tensor& dst, int64_t add, int64_t flags, int64_t world, int64_t epoch,
                  int64_t timeout_ms) {
  check_f32(dst, "dst");
  MMB_CHECK_RC(mmb::tp_wait_copy(reinterpret_cast<const float*>(src), dst.data_ptr<float>(), dst.numel(), (int)add,
                                 reinterpret_cast<const int*>(flags), (int)world, (int)epoch, error_word(), num_sms(),
                                 cur_stream(), (unsigned long long)timeout_ms * 1000000ull),
               "tp_wait_copy");
}

void tp_publish(const Tensor& src, const std::vector<int64_t>& dst, const std::vector<int64_t>& flags, int64_t rank,
                int64_t epoch, Tensor& counter) {
  check_f32(src, "src");
  mmb::AgPush P = make_push(dst, flags, rank, epoch, 1, 1, 4, counter);
  MMB_CHECK_RC(mmb::tp_publish(src.data_ptr<float>(), src.numel(), P, num_sms(), cur_stream()), "tp_publish");
}

void tp_pos_grad_push(const Tensor& dout, int64_t B, const std::vector<int64_t>& dst,
                      const std::vector<int64_t>& flags, int64_t rank, int64_t epoch, int64_t S, int64_t Sl,
                      Tensor& counter) {
  check_f32(dout, "dout");
  const int H = (int)dout.size(-1);
  TORCH_CHECK(dout.numel() == B * Sl * H, "tp_pos_grad_push: dout must be [B*Sl, H]");
  mmb::AgPush P = make_push(dst, flags, rank, epoch, S, Sl, H, counter);
  MMB_CHECK_RC(mmb::tp_pos_grad_push(dout.data_ptr<float>(), (int)B, H, P, num_sms(), cur_stream()),
               "tp_pos_grad_push");
}

void tp_vec_allreduce(const Tensor& v, Tensor& out, const std::vector<int64_t>& dst,
                      const std::vector<int64_t>& flags, int64_t rank, int64_t epoch, Tensor& counter,
                      int64_t slots_local, int64_t flags_local, int64_t timeout_ms) {
  check_f32(v, "v");
  check_f32(out, "out");
  TORCH_CHECK(v.numel() == out.numel(), "tp_vec_allreduce: sizes");
  mmb::AgPush P = make_push(dst, flags, rank, epoch, 1, 1, 1, counter);
  MMB_CHECK_RC(mmb::tp_vec_allreduce(v.data_ptr<float>(), out.data_ptr<float>(), v.numel(), P,
                                     reinterpret_cast<const float*>(slots_local),
                                     reinterpret_cast<const int*>(flags_local), error_word(), num_sms(), cur_stream(),
                                     (unsigned long long)timeout_ms * 1000000ull),
               "tp_vec_allreduce");
}

void embedding_bwd_peers(const Tensor& ids, const std::vector<int64_t>& src, int64_t flags_local, int64_t epoch,
                         int64_t S, int64_t Sl, Tensor& dwte, int64_t vstart, int64_t vend) {
  check_f32(dwte, "dwte");
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous() && ids.is_cuda(), "ids: contiguous CUDA int64");
  TORCH_CHECK(src.size() >= 1 && src.size() <= 8, "embedding_bwd_peers: 1..8 ranks");
  mmb::EmbPeers P{};
  for (size_t i = 0; i < src.size(); ++i) P.src[i] = reinterpret_cast<const float*>(src[i]);
  P.flags = reinterpret_cast<const int*>(flags_local);
  P.world = (int)src.size();
  P.epoch = (int)epoch;
  P.S = (int)S;
  P.Sl = (int)Sl;
  MMB_CHECK_RC(mmb::embedding_bwd_peers(ids.data_ptr<int64_t>(), P, dwte.data_ptr<float>(), (int)ids.numel(),
                                        (int)dwte.size(1), vstart, vend, error_word(), cur_stream()),
               "embedding_bwd_peers");
}

// lm_head GEMM whose epilogue also writes per-tile cross-entropy partials, then the
// merge: returns (max, sumexp, target logit) per row like ce_fwd_stats.
// With ag_flags != 0 the rows of A are a sequence-parallel all-gather in progress: the GEMM's
// TMA producer waits per source rank (flags >= ag_epoch) before loading that rank's rows.
std::vector<Tensor> gemm_ce_stats(const Tensor& A, const Tensor& B, Tensor& D, const Tensor& labels,
                                  int64_t vocab_start, int64_t n_valid, int64_t ag_flags, int64_t ag_epoch,
                                  int64_t S, int64_t Sl, int64_t rank) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  check_bf16(D, "D");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && A.size(1) == B.size(1), "gemm_ce_stats operands");
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous(), "labels must be contiguous int64");
  const int64_t M = A.size(0), N = B.size(0), K = A.size(1);
  TORCH_CHECK(D.size(0) == M && D.size(1) == N, "D shape");
  const int64_t nparts = 2 * ((N + 255) / 256);
  Tensor part = at::empty({M, nparts, 2}, A.options().dtype(at::kFloat));
  mmb::GemmProblem p{};
  p.A = A.data_ptr();
  p.lda = A.stride(0);
  p.B = B.data_ptr();
  p.ldb = B.stride(0);
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.bn = 256;
  p.num_sms = num_sms();
  p.args.epi = mmb::EPI_CE_STATS;
  p.args.alpha = 1.f;
  p.args.err = error_word();
  p.args.D = D.data_ptr();
  p.args.ldd = D.stride(0);
  p.args.ce_part = reinterpret_cast<float2*>(part.data_ptr<float>());
  p.args.ce_ld = nparts;
  p.args.ce_n_valid = (int)n_valid;
  if (ag_flags != 0) {
    TORCH_CHECK(Sl % 128 == 0 && S % Sl == 0 && M % S == 0, "gemm_ce_stats: all-gather shards must be 128-row tiles");
    p.args.ag_flags = reinterpret_cast<const int*>(ag_flags);
    p.args.ag_epoch = (int)ag_epoch;
    p.args.ag_S = (int)S;
    p.args.ag_Sl = (int)Sl;
    p.args.ag_rank = (int)rank;
  }
  MMB_CHECK_RC(mmb::gemm_bf16_launch(p, cur_stream()), "gemm_ce_stats");
  Tensor mx = at::empty({M}, A.options().dtype(at::kFloat));
  Tensor se = at::empty_like(mx), tg = at::empty_like(mx);
  MMB_CHECK_RC(mmb::ce_merge_stats(reinterpret_cast<const float2*>(part.data_ptr<float>()), nparts, (int)nparts,
                                   reinterpret_cast<const __nv_bfloat16*>(D.data_ptr()), D.stride(0),
                                   labels.data_ptr<int64_t>(), vocab_start, (int)n_valid, (int)M, mx.data_ptr<float>(),
                                   se.data_ptr<float>(), tg.data_ptr<float>(), cur_stream()),
               "ce_merge_stats");
  return {mx, se, tg};
}

// GEMM with the TP collectives fused: optional all-gather wait on A rows and/or
// reduce-scatter push epilogue (epi == EPI_PUSH_BF16, D unused).
void gemm_tp(const Tensor& A, bool a_mn, const Tensor& B, bool b_mn, const c10::optional<Tensor>& D, int64_t epi,
             const c10::optional<Tensor>& aux, int64_t ag_flags, int64_t ag_epoch, int64_t S, int64_t Sl,
             const std::vector<int64_t>& push_dst, const std::vector<int64_t>& push_flags, int64_t rank,
             int64_t push_epoch, const c10::optional<Tensor>& push_counter, int64_t N_out) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "gemm_tp operands must be row-major");
  const int64_t M = a_mn ? A.size(1) : A.size(0);
  const int64_t K = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0);
  TORCH_CHECK((b_mn ? B.size(0) : B.size(1)) == K, "gemm_tp: K mismatch");
  TORCH_CHECK(N % 8 == 0 && N == N_out, "gemm_tp: N");
  mmb::GemmProblem p{};
  p.A = A.data_ptr();
  p.lda = A.stride(0);
  p.a_mn = a_mn;
  p.B = B.data_ptr();
  p.ldb = B.stride(0);
  p.b_mn = b_mn;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.num_sms = num_sms();
  p.allow_split = false;
  p.args.epi = (int)epi;
  p.args.alpha = 1.f;
  p.args.err = error_word();
  if (ag_flags != 0) {
    TORCH_CHECK(Sl % 128 == 0 && S % Sl == 0, "gemm_tp: all-gather shards must be multiples of 128 rows");
    p.args.ag_flags = reinterpret_cast<const int*>(ag_flags);
    p.args.ag_epoch = (int)ag_epoch;
    p.args.ag_S = (int)S;
    p.args.ag_Sl = (int)Sl;
    p.args.ag_rank = (int)rank;
  }
  if (epi == mmb::EPI_PUSH_BF16) {
    TORCH_CHECK(push_dst.size() == push_flags.size() && push_dst.size() >= 1 && push_dst.size() <= 8, "push ranks");
    TORCH_CHECK(push_counter.has_value(), "push needs a counter");
    p.args.ldd = N;
    p.args.push_world = (int)push_dst.size();
    p.args.push_rank = (int)rank;
    p.args.push_epoch = (int)push_epoch;
    p.args.push_S = (int)S;
    p.args.push_Sl = (int)Sl;
    for (size_t i = 0; i < push_dst.size(); ++i) {
      p.args.push_dst[i] = reinterpret_cast<void*>(push_dst[i]);
      p.args.push_flags[i] = reinterpret_cast<int*>(push_flags[i]);
    }
    p.args.push_counter = reinterpret_cast<unsigned*>(push_counter->data_ptr<int>());
    p.args.D = p.args.push_dst[rank];
  } else {
    TORCH_CHECK(D.has_value(), "gemm_tp: D required");
    p.args.D = D->data_ptr();
    p.args.ldd = D->stride(0);
    if (aux.has_value()) {
      p.args.aux = aux->data_ptr();
      p.args.ld_aux = aux->stride(0);
    }
  }
  const int rc = mmb::gemm_bf16_launch(p, cur_stream());
  TORCH_CHECK(rc == 0, "gemm_tp launch failed, code ", rc);
}

// ----------------------------------------------------------------- crash diagnostics
// Optional SIGSEGV/SIGBUS handler that prints the faulting address, the thread
// id and a native backtrace to stderr, then hands over to the previous handler
// (e.g. Python's faulthandler) so the process still dies with the signal.
struct sigaction g_prev_segv, g_prev_bus;

void crash_handler(int sig, siginfo_t* info, void* uctx) {
  char buf[160];
  const int n = snprintf(buf, sizeof buf, "mmb: signal %d at address %p in thread %ld; native backtrace:\n", sig,
                         info ? info->si_addr : nullptr, (long)syscall(SYS_gettid));
  if (n > 0) (void)!write(2, buf, (size_t)n);
  void* frames[64];
  const int k = backtrace(frames, 64);
  backtrace_symbols_fd(frames, k, 2);
  struct sigaction* prev = sig == SIGSEGV ? &g_prev_segv : &g_prev_bus;
  if (prev->sa_flags & SA_SIGINFO) {
    if (prev->sa_sigaction) prev->sa_sigaction(sig, info, uctx);
  } else if (prev->sa_handler != SIG_DFL && prev->sa_handler != SIG_IGN && prev->sa_handler) {
    prev->sa_handler(sig);
  }
  signal(sig, SIG_DFL);
  raise(sig);
}

void install_crash_handler() {
  struct sigaction sa {};
  sa.sa_sigaction = crash_handler;
  sa.sa_flags = SA_SIGINFO | SA_ONSTACK;
  sigemptyset(&sa.sa_mask);
  sigaction(SIGSEGV, &sa, &g_prev_segv);
  sigaction(SIGBUS, &sa, &g_prev_bus);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of mini_megatron_b200";
  m.def("get_error", &get_error, "read the device error word (0 = ok)");
  m.def("install_crash_handler", &install_crash_handler,
        "print a native backtrace on SIGSEGV/SIGBUS before the previous handler runs");
  m.def("clear_error", &clear_error);
  m.def("set_error", &set_error, "write the device error word from the host (tests of the host-side check)");
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM with fused epilogue", py::arg("A"), py::arg("a_mn"), py::arg("B"),
        py::arg("b_mn"), py::arg("D"), py::arg("epi"), py::arg("aux") = c10::nullopt,
        py::arg("resid") = c10::nullopt, py::arg("alpha") = 1.0, py::arg("bn") = 0, py::arg("cg") = 0);
  m.def("layernorm_fwd", &layernorm_fwd);
  m.def("layernorm_bwd", &layernorm_bwd, py::arg("dy"), py::arg("x"), py::arg("mean"), py::arg("rstd"),
        py::arg("gamma"), py::arg("dres"), py::arg("dx"), py::arg("dgamma"), py::arg("dbeta"),
        py::arg("dx_bf16") = c10::nullopt);
  m.def("ce_fwd_stats", &ce_fwd_stats);
  m.def("gemm_ce_stats", &gemm_ce_stats, "lm_head GEMM with cross-entropy statistics fused into its epilogue",
        py::arg("A"), py::arg("B"), py::arg("D"), py::arg("labels"), py::arg("vocab_start"), py::arg("n_valid"),
        py::arg("ag_flags") = 0, py::arg("ag_epoch") = 0, py::arg("S") = 0, py::arg("Sl") = 0, py::arg("rank") = 0);
  m.def("tp_emb_fwd_push", &tp_emb_fwd_push);
  m.def("tp_wait_copy", &tp_wait_copy, py::arg("src"), py::arg("dst"), py::arg("add"), py::arg("flags"),
        py::arg("world"), py::arg("epoch"), py::arg("timeout_ms") = 10000);
  m.def("tp_publish", &tp_publish);
  m.def("tp_pos_grad_push", &tp_pos_grad_push);
  m.def("tp_vec_allreduce", &tp_vec_allreduce, py::arg("v"), py::arg("out"), py::arg("dst"), py::arg("flags"),
        py::arg("rank"), py::arg("epoch"), py::arg("counter"), py::arg("slots_local"), py::arg("flags_local"),
        py::arg("timeout_ms") = 10000);
  m.def("embedding_bwd_peers", &embedding_bwd_peers);
  m.def("tp_ce_allreduce", &tp_ce_allreduce, py::arg("mx"), py::arg("se"), py::arg("tg"), py::arg("dst"),
        py::arg("flags"), py::arg("rank"), py::arg("epoch"), py::arg("counter"), py::arg("slots_local"),
        py::arg("flags_local"), py::arg("timeout_ms") = 10000);
  m.def("ce_bwd", &ce_bwd);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("adamw_flat", &adamw_flat);
  m.def("adamw_flat_dev", &adamw_flat_dev);
  m.def("adamw_hyper_step", &adamw_hyper_step);
  m.def("cast_f32_bf16", &cast_f32_bf16);
  m.def("gelu_fwd_bwd_f32", &gelu_fwd_bwd_f32);
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_free", &symm_free);
  m.def("symm_export", &symm_export);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("dp_rs_adamw_ag", &dp_rs_adamw_ag, py::arg("param"), py::arg("grad"), py::arg("pbf16"), py::arg("sig"),
        py::arg("rank"), py::arg("bucket"), py::arg("epoch"), py::arg("lo"), py::arg("hi"), py::arg("exp_avg"),
        py::arg("exp_avg_sq"), py::arg("counter"), py::arg("lr"), py::arg("b1"), py::arg("b2"), py::arg("eps"),
        py::arg("wd"), py::arg("step"), py::arg("grad_scale"), py::arg("max_ctas"), py::arg("defer_done") = 0,
        py::arg("epoch_dev") = c10::nullopt, py::arg("hyper") = c10::nullopt, py::arg("segs") = c10::nullopt);
  m.def("dp_gather_master", &dp_gather_master, "copy the other ranks' fp32 master shards of one bucket here",
        py::arg("param"), py::arg("rank"), py::arg("start"), py::arg("end"));
  m.def("dp_wait_done", [](int64_t sig_local, int64_t nbuckets, int64_t world, int64_t epoch,
                           const c10::optional<Tensor>& epoch_dev, int64_t timeout_ms) {
    const int* ep = epoch_dev.has_value() ? epoch_dev->data_ptr<int>() : nullptr;
    MMB_CHECK_RC(mmb::dp_wait_done(reinterpret_cast<const void*>(sig_local), (int)nbuckets, (int)world, (int)epoch,
                                   ep, (unsigned long long)timeout_ms * 1000000ull, error_word(), cur_stream()),
                 "dp_wait_done");
  }, py::arg("sig_local"), py::arg("nbuckets"), py::arg("world"), py::arg("epoch"),
        py::arg("epoch_dev") = c10::nullopt, py::arg("timeout_ms") = 10000);
  m.def("dp_epoch_step", [](Tensor& epoch) {
    TORCH_CHECK(epoch.scalar_type() == at::kInt && epoch.is_cuda() && epoch.numel() == 1, "epoch: one CUDA int32");
    MMB_CHECK_RC(mmb::dp_epoch_step(epoch.data_ptr<int>(), cur_stream()), "dp_epoch_step");
  });
  m.def("dp_signal_pad_bytes", &mmb::dp_signal_pad_bytes);
  m.def("dp_max_segments", &mmb::dp_max_segments);
  m.def("layernorm_fwd_push", &layernorm_fwd_push);
  m.def("layernorm_bwd_push", &layernorm_bwd_push);
  m.def("tp_ag_push", &tp_ag_push);
  m.def("tp_rs_reduce", &tp_rs_reduce, py::arg("slots_ptr"), py::arg("slot_stride"), py::arg("world"),
        py::arg("flags_ptr"), py::arg("epoch"), py::arg("resid"), py::arg("out"), py::arg("out_bf16"), py::arg("n"),
        py::arg("timeout_ms") = 10000);
  m.def("gemm_tp", &gemm_tp);
  m.attr("EPI_CE_STATS") = (int)mmb::EPI_CE_STATS;
  m.attr("EPI_PUSH_BF16") = (int)mmb::EPI_PUSH_BF16;
  m.def("num_sms", &num_sms);
  m.def("flash_attn_fwd", &flash_attn_fwd);
  m.def("flash_attn_fwd_v1", &flash_attn_fwd_v1, "previous one-tile-per-CTA forward (comparison only)");
  m.def("flash_attn_bwd", &flash_attn_bwd);
  m.def("flash_attn_bwd_v1", &flash_attn_bwd_v1, "one-key-tile-per-CTA backward (comparison only)");
  m.attr("EPI_F32_ATOMIC") = (int)mmb::EPI_F32_ATOMIC;
  m.attr("EPI_BF16") = (int)mmb::EPI_BF16;
  m.attr("EPI_F32") = (int)mmb::EPI_F32;
  m.attr("EPI_F32_ACC") = (int)mmb::EPI_F32_ACC;
  m.attr("EPI_GELU") = (int)mmb::EPI_GELU;
  m.attr("EPI_RESID") = (int)mmb::EPI_RESID;
  m.attr("EPI_DGELU") = (int)mmb::EPI_DGELU;
}
