// PyTorch bindings for the sm_100a kernel library.  Validates tensors and
// forwards raw pointers to the torch-free launchers declared in kernels.h.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "kernels.h"

using oxi::Mat;

namespace {

Mat bf16_mat(const torch::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda(), what, " must be a CUDA tensor");
  TORCH_CHECK(t.dim() == 2, what, " must be 2-D");
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, what, " must be bf16");
  TORCH_CHECK(t.stride(1) == 1 || t.size(1) == 1, what, " must have unit inner stride");
  return Mat{t.data_ptr(), t.size(0), t.size(1), t.stride(0)};
}

int* status_ptr(const torch::Tensor& s) {
  TORCH_CHECK(s.is_cuda() && s.scalar_type() == torch::kInt32, "status must be a CUDA int32 tensor");
  return s.data_ptr<int>();
}

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

void check_out(const torch::Tensor& o, int64_t rows, int64_t cols, const char* what) {
  TORCH_CHECK(o.is_cuda() && o.dim() == 2 && o.size(0) == rows && o.size(1) == cols && o.stride(1) == 1, what,
              " must be a CUDA tensor of shape [", rows, ", ", cols, "] with unit inner stride");
}

// ------------------------------------------------------------------ GEMM
void gemm(torch::Tensor a, bool a_mn, torch::Tensor b, bool b_mn, torch::Tensor out,
          c10::optional<torch::Tensor> resid, double beta, double alpha, torch::Tensor status) {
  c10::cuda::CUDAGuard g(a.device());
  Mat ma = bf16_mat(a, "a"), mb = bf16_mat(b, "b");
  const int64_t M = a_mn ? ma.cols : ma.rows, K = a_mn ? ma.rows : ma.cols;
  const int64_t N = b_mn ? mb.cols : mb.rows, Kb = b_mn ? mb.rows : mb.cols;
  TORCH_CHECK(K == Kb, "GEMM K mismatch ", K, " vs ", Kb);
  check_out(out, M, N, "out");
  const bool f32 = out.scalar_type() == torch::kFloat32;
  TORCH_CHECK(f32 || out.scalar_type() == torch::kBFloat16, "out must be bf16 or f32");
  if (K == 0) {
    if (beta == 0.0 || !f32) out.zero_();
    return;
  }
  const void* rp = nullptr;
  int64_t ldr = 0;
  if (resid.has_value() && resid->defined()) {
    TORCH_CHECK(!f32, "residual add only for bf16 output");
    check_out(*resid, M, N, "resid");
    TORCH_CHECK(resid->scalar_type() == torch::kBFloat16, "resid must be bf16");
    rp = resid->data_ptr();
    ldr = resid->stride(0);
  }
  oxi::launch_gemm(ma, a_mn, mb, b_mn, out.data_ptr(), out.stride(0), f32, rp, ldr, (float)beta, (float)alpha,
                   status_ptr(status), stream());
}

void gemm_swiglu(torch::Tensor x, torch::Tensor w, torch::Tensor h, c10::optional<torch::Tensor> gu,
                 torch::Tensor status) {
  c10::cuda::CUDAGuard g(x.device());
  Mat mx = bf16_mat(x, "x"), mw = bf16_mat(w, "w");
  check_out(h, mx.rows, mw.rows / 2, "h");
  void* gp = nullptr;
  int64_t ldgu = 0;
  if (gu.has_value() && gu->defined()) {
    check_out(*gu, mx.rows, mw.rows, "gu");
    gp = gu->data_ptr();
    ldgu = gu->stride(0);
  }
  oxi::launch_gemm_swiglu(mx, mw, h.data_ptr(), h.stride(0), gp, ldgu, status_ptr(status), stream());
}

void gemm_swiglu_bwd(torch::Tensor dy, torch::Tensor w_down, torch::Tensor gu, torch::Tensor dgu,
                     torch::Tensor status) {
  c10::cuda::CUDAGuard g(dy.device());
  Mat md = bf16_mat(dy, "dy"), mw = bf16_mat(w_down, "w_down");
  check_out(gu, md.rows, 2 * mw.cols, "gu");
  check_out(dgu, md.rows, 2 * mw.cols, "dgu");
  oxi::launch_gemm_swiglu_bwd(md, mw, gu.data_ptr(), gu.stride(0), dgu.data_ptr(), dgu.stride(0),
                              status_ptr(status), stream());
}

void gemm_ce(torch::Tensor x, torch::Tensor w, torch::Tensor targets, torch::Tensor part_max,
             torch::Tensor part_sum, torch::Tensor tgt_logit, c10::optional<torch::Tensor> logits, double alpha,
             torch::Tensor status) {
  c10::cuda::CUDAGuard g(x.device());
  Mat mx = bf16_mat(x, "x"), mw = bf16_mat(w, "w");
  const int tn = oxi::gemm_ce_tiles_n(mw.rows);
  TORCH_CHECK(targets.scalar_type() == torch::kInt64 && targets.numel() == mx.rows && targets.is_contiguous(),
              "targets must be contiguous int64 [M]");
  TORCH_CHECK(part_max.scalar_type() == torch::kFloat32 && part_max.is_contiguous() && part_max.size(0) == mx.rows &&
                  part_max.size(1) == tn, "part_max must be f32 [M, ", tn, "]");
  TORCH_CHECK(part_sum.sizes() == part_max.sizes() && part_sum.is_contiguous(), "part_sum shape");
  TORCH_CHECK(tgt_logit.scalar_type() == torch::kFloat32 && tgt_logit.numel() == mx.rows, "tgt_logit f32 [M]");
  void* lp = nullptr;
  int64_t ldl = 0;
  if (logits.has_value() && logits->defined()) {
    TORCH_CHECK(logits->scalar_type() == torch::kBFloat16 && logits->size(0) == mx.rows &&
                    logits->size(1) >= mw.rows && logits->stride(1) == 1, "logits buffer");
    lp = logits->data_ptr();
    ldl = logits->stride(0);
  }
  oxi::launch_gemm_ce(mx, mw, targets.data_ptr<int64_t>(), part_max.data_ptr<float>(), part_sum.data_ptr<float>(),
                      tgt_logit.data_ptr<float>(), lp, ldl, (float)alpha, status_ptr(status), stream());
}

void gemm_rope(torch::Tensor x, torch::Tensor w, torch::Tensor out, torch::Tensor cos, torch::Tensor sin,
               int64_t hd, int64_t q_cols, int64_t k_cols, torch::Tensor status) {
  c10::cuda::CUDAGuard g(x.device());
  Mat mx = bf16_mat(x, "x"), mw = bf16_mat(w, "w");
  check_out(out, mx.rows, mw.rows, "out");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16, "out must be bf16");
  TORCH_CHECK(cos.scalar_type() == torch::kFloat32 && cos.is_contiguous() && sin.is_contiguous() &&
                  cos.size(1) == hd / 2 && sin.sizes() == cos.sizes(), "cos/sin must be contiguous f32 [S, hd/2]");
  oxi::launch_gemm_rope(mx, mw, out.data_ptr(), out.stride(0), cos.data_ptr<float>(), sin.data_ptr<float>(),
                        (int)cos.size(0), (int)hd, (int)q_cols, (int)k_cols, status_ptr(status), stream());
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "oxidizr_b200 sm_100a kernels";
  m.def("gemm", &gemm, "tcgen05 GEMM out = alpha * a @ b^T (+resid | + beta*out)");
  m.def("gemm_swiglu", &gemm_swiglu, "GEMM with fused SwiGLU epilogue");
  m.def("gemm_swiglu_bwd", &gemm_swiglu_bwd, "GEMM with fused SwiGLU backward epilogue");
  m.def("gemm_ce", &gemm_ce, "lm_head GEMM with fused cross-entropy partials");
  m.def("gemm_rope", &gemm_rope, "QKV GEMM with fused rotate-half RoPE epilogue");
}
