// Python bindings of the sm_100a kernels. Every entry point validates devices, dtypes and extents before launching
// on the current torch CUDA stream, and raises on a launch error.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>

#include "gemm_tcgen05.cuh"
#include "kernels.cuh"

namespace {

void check_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

template <typename T>
T* ptr_or_null(const c10::optional<torch::Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

// Elements addressable from t's first element to the end of its storage (strided row views reach past numel()).
int64_t avail(const torch::Tensor& t) {
  return static_cast<int64_t>(t.storage().nbytes() / t.element_size()) - t.storage_offset();
}

void raise_on(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, " failed: ", cudaGetErrorString(e));
}

// out[M, N] = sum_k A(m, k) B(n, k); see gemm_tcgen05.cuh for operand layouts.
void gemm(const torch::Tensor& a, int64_t lda, bool a_mn, const torch::Tensor& b, int64_t ldb, bool b_mn, int64_t M,
          int64_t N, int64_t K, int64_t epilogue, const torch::Tensor& out, int64_t ldo, int64_t splits,
          int64_t split_stride, const c10::optional<torch::Tensor>& bias, const c10::optional<torch::Tensor>& aux,
          int64_t ld_aux, const c10::optional<torch::Tensor>& colsum, const c10::optional<torch::Tensor>& status,
          int64_t out_cols) {
  check_cuda(a, "a");
  check_cuda(b, "b");
  check_cuda(out, "out");
  TORCH_CHECK(a.scalar_type() == torch::kBFloat16 && b.scalar_type() == torch::kBFloat16, "gemm operands must be bf16");
  TORCH_CHECK(epilogue >= rlb::kEpiF32 && epilogue <= rlb::kEpiPartialF32,
              "gemm: unknown epilogue (the recurrent-cell epilogue is rnn_step_fused)");
  const bool out_f32 = epilogue == rlb::kEpiF32 || epilogue == rlb::kEpiPartialF32;
  TORCH_CHECK(out.scalar_type() == (out_f32 ? torch::kFloat32 : torch::kBFloat16), "gemm: wrong output dtype");
  // extent checks (elements reachable by the kernel)
  const int64_t a_need = a_mn ? (K - 1) * lda + M : (M - 1) * lda + K;
  const int64_t b_need = b_mn ? (K - 1) * ldb + N : (N - 1) * ldb + K;
  TORCH_CHECK(avail(a) >= a_need, "gemm: A too small");
  TORCH_CHECK(avail(b) >= b_need, "gemm: B too small");
  TORCH_CHECK(avail(out) >= (splits - 1) * split_stride + (M - 1) * ldo + std::max(N, out_cols), "gemm: out too small");
  TORCH_CHECK(out_cols == 0 || (epilogue == rlb::kEpiF32 && out_cols >= N && out_cols <= ldo),
              "gemm: out_cols (fp32 output only) must lie in [N, ldo]");
  if (bias.has_value() && bias->defined()) {
    TORCH_CHECK(bias->scalar_type() == torch::kFloat32 && bias->numel() >= N, "gemm: bad bias");
  }
  if (aux.has_value() && aux->defined()) {
    TORCH_CHECK(aux->scalar_type() == torch::kBFloat16 && avail(*aux) >= (M - 1) * ld_aux + N, "gemm: bad aux");
  }
  int64_t colsum_rows = 0;
  if (colsum.has_value() && colsum->defined()) {
    // one row of N column sums per CTA: [rows, N] with rows >= the launch's CTA count (checked by the launcher)
    TORCH_CHECK(colsum->scalar_type() == torch::kFloat32 && colsum->dim() == 2 && colsum->is_contiguous() &&
                    colsum->size(1) == N,
                "gemm: colsum must be a contiguous fp32 [rows, N] tensor");
    TORCH_CHECK(N <= rlb::kColsumMaxN, "gemm: column sums need N <= ", rlb::kColsumMaxN);
    colsum_rows = colsum->size(0);
  }
  const at::cuda::CUDAGuard guard(a.device());
  rlb::GemmParams p;
  p.a = a.data_ptr();
  p.lda = static_cast<int>(lda);
  p.a_mn_major = a_mn;
  p.b = b.data_ptr();
  p.ldb = static_cast<int>(ldb);
  p.b_mn_major = b_mn;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.splits = static_cast<int>(splits);
  p.epilogue = static_cast<int>(epilogue);
  p.out = out.data_ptr();
  p.ldo = static_cast<int>(ldo);
  p.split_stride = split_stride;
  p.bias = ptr_or_null<const float>(bias);
  p.aux = ptr_or_null<const void>(aux);
  p.ld_aux = static_cast<int>(ld_aux);
  p.colsum = ptr_or_null<float>(colsum);
  p.colsum_rows = static_cast<int>(colsum_rows);
  p.status = ptr_or_null<unsigned int>(status);
  p.out_cols = static_cast<int>(out_cols);
  raise_on(rlb::gemm_launch(p, at::cuda::getCurrentCUDAStream()), "gemm");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of tt_rsl_rl_b200";
  m.def("gemm", &gemm, "tcgen05 GEMM with fused MLP epilogues");
  m.def("gemm_colsum_rows", [](int64_t sms) { return static_cast<int64_t>(rlb::gemm_colsum_rows(static_cast<int>(sms))); });
  rlb_register_kernels(m);
  rlb_register_p2p(m);
  rlb_register_rnn(m);
}
