// Python bindings for the sm_100a kernels.  Only this translation unit
// includes the torch headers; kernels live in plain .cu files.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

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

// ----------------------------------------------------------------- GEMM
void gemm(const Tensor& A, bool a_mn, const Tensor& B, bool b_mn, Tensor& D, int64_t epi,
          const c10::optional<Tensor>& aux, const c10::optional<Tensor>& resid, double alpha, int64_t bn) {
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
  p.num_sms = num_sms();
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

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of mini_megatron_b200";
  m.def("get_error", &get_error, "read the device error word (0 = ok)");
  m.def("clear_error", &clear_error);
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM with fused epilogue", py::arg("A"), py::arg("a_mn"), py::arg("B"),
        py::arg("b_mn"), py::arg("D"), py::arg("epi"), py::arg("aux") = c10::nullopt,
        py::arg("resid") = c10::nullopt, py::arg("alpha") = 1.0, py::arg("bn") = 0);
  m.attr("EPI_BF16") = (int)mmb::EPI_BF16;
  m.attr("EPI_F32") = (int)mmb::EPI_F32;
  m.attr("EPI_F32_ACC") = (int)mmb::EPI_F32_ACC;
  m.attr("EPI_GELU") = (int)mmb::EPI_GELU;
  m.attr("EPI_RESID") = (int)mmb::EPI_RESID;
  m.attr("EPI_DGELU") = (int)mmb::EPI_DGELU;
}
