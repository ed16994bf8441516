// PyTorch bindings for the sm_100a kernel library.  Validates tensors and
// forwards raw pointers to the torch-free launchers declared in kernels.h.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "kernels.h"
#include "kernels_ew.h"
#include "kernels_attn.h"
#include "kernels_comm.h"
#include "kernels_mla.h"
#include "kernels_ssm.h"
#include "kernels_moe.h"
#include "kernels_ep.h"
#include "host_util.h"

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
          c10::optional<torch::Tensor> resid, double beta, double alpha, torch::Tensor status,
          c10::optional<torch::Tensor> bias) {
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
  const void* bp = nullptr;
  if (bias.has_value() && bias->defined()) {
    TORCH_CHECK(!f32 && bias->scalar_type() == torch::kBFloat16 && bias->is_contiguous() && bias->numel() == N,
                "bias: bf16 contiguous [N], bf16 output only");
    bp = bias->data_ptr();
  }
  oxi::launch_gemm(ma, a_mn, mb, b_mn, out.data_ptr(), out.stride(0), f32, rp, ldr, (float)beta, (float)alpha,
                   status_ptr(status), stream(), bp);
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

void swiglu_bwd(torch::Tensor dh, torch::Tensor gu, torch::Tensor dgu) {
  c10::cuda::CUDAGuard g(dh.device());
  TORCH_CHECK(dh.scalar_type() == torch::kBFloat16 && gu.scalar_type() == torch::kBFloat16 &&
                  dgu.scalar_type() == torch::kBFloat16 && dh.is_contiguous() && gu.is_contiguous() &&
                  dgu.is_contiguous() && dh.dim() == 2 && gu.sizes() == dgu.sizes() && gu.size(0) == dh.size(0) &&
                  gu.size(1) == 2 * dh.size(1),
              "swiglu_bwd: contiguous bf16 dH [rows, I], GU / dGU [rows, 2I]");
  oxi::launch_swiglu_bwd(dh.data_ptr(), gu.data_ptr(), dgu.data_ptr(), dh.size(0), (int)dh.size(1), stream());
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

// ------------------------------------------------------------ norms
void check_bf16_rows(const torch::Tensor& t, int64_t rows, int64_t H, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16 && t.is_contiguous() && t.numel() == rows * H, what,
              " must be a contiguous bf16 CUDA tensor with ", rows, "x", H, " elements");
}

void norm_fwd(int64_t mode, torch::Tensor x, c10::optional<torch::Tensor> gate, torch::Tensor w,
              c10::optional<torch::Tensor> b, torch::Tensor y, torch::Tensor rstd, c10::optional<torch::Tensor> mean,
              double eps) {
  c10::cuda::CUDAGuard g(x.device());
  const int64_t H = x.size(-1), rows = x.numel() / H;
  check_bf16_rows(x, rows, H, "x");
  check_bf16_rows(y, rows, H, "y");
  TORCH_CHECK(w.is_contiguous() && w.numel() == H, "weight shape");
  const bool wf32 = w.scalar_type() == torch::kFloat32;
  if (mode == 2) check_bf16_rows(*gate, rows, H, "gate");
  const void* bp = nullptr;
  if (mode == 1) {
    TORCH_CHECK(b.has_value() && b->scalar_type() == w.scalar_type() && b->numel() == H, "bias");
    bp = b->data_ptr();
  }
  oxi::launch_norm_fwd((int)mode, x.data_ptr(), mode == 2 ? gate->data_ptr() : nullptr, w.data_ptr(), wf32, bp,
                       y.data_ptr(), rstd.data_ptr<float>(), mode == 1 ? mean->data_ptr<float>() : nullptr, rows,
                       (int)H, (float)eps, stream());
}

void norm_bwd(int64_t mode, torch::Tensor dy, torch::Tensor x, c10::optional<torch::Tensor> gate, torch::Tensor w,
              torch::Tensor rstd, c10::optional<torch::Tensor> mean, c10::optional<torch::Tensor> dres,
              torch::Tensor dx, c10::optional<torch::Tensor> dgate, torch::Tensor dw, c10::optional<torch::Tensor> db) {
  c10::cuda::CUDAGuard g(x.device());
  const int64_t H = x.size(-1), rows = x.numel() / H;
  check_bf16_rows(dy, rows, H, "dy");
  check_bf16_rows(x, rows, H, "x");
  check_bf16_rows(dx, rows, H, "dx");
  TORCH_CHECK(dw.scalar_type() == torch::kFloat32 && dw.numel() == H && dw.is_contiguous(), "dw must be f32 [H]");
  const void* dr = nullptr;
  if (dres.has_value() && dres->defined()) {
    check_bf16_rows(*dres, rows, H, "dres");
    dr = dres->data_ptr();
  }
  const int prow = oxi::norm_bwd_partial_rows(rows, (int)H);
  torch::Tensor part;
  if (prow > 0) part = torch::empty({prow, 2 * H}, x.options().dtype(torch::kFloat32));
  oxi::launch_norm_bwd((int)mode, dy.data_ptr(), x.data_ptr(), mode == 2 ? gate->data_ptr() : nullptr, w.data_ptr(),
                       w.scalar_type() == torch::kFloat32, rstd.data_ptr<float>(),
                       mode == 1 ? mean->data_ptr<float>() : nullptr, dr, dx.data_ptr(),
                       mode == 2 ? dgate->data_ptr() : nullptr, dw.data_ptr<float>(),
                       mode == 1 ? db->data_ptr<float>() : nullptr, rows, (int)H, stream(),
                       prow > 0 ? part.data_ptr<float>() : nullptr, prow);
}

// ------------------------------------------------------------ CE
void ce_finish(torch::Tensor pmax, torch::Tensor psum, torch::Tensor tgt_logit, torch::Tensor targets,
               torch::Tensor lse, torch::Tensor loss) {
  c10::cuda::CUDAGuard g(pmax.device());
  oxi::launch_ce_finish(pmax.data_ptr<float>(), psum.data_ptr<float>(), (int)pmax.size(1), tgt_logit.data_ptr<float>(),
                        targets.data_ptr<int64_t>(), lse.data_ptr<float>(), loss.data_ptr<float>(), pmax.size(0),
                        stream());
}

void ce_bwd(torch::Tensor logits, int64_t V, torch::Tensor lse, torch::Tensor targets, torch::Tensor gscale,
            double inv_count, int64_t col0) {
  c10::cuda::CUDAGuard g(logits.device());
  TORCH_CHECK(logits.scalar_type() == torch::kBFloat16 && logits.stride(1) == 1, "logits");
  TORCH_CHECK(logits.size(1) >= V && lse.numel() == logits.size(0) && targets.numel() == logits.size(0),
              "ce_bwd: logits [M, >= V], lse / targets [M]");
  oxi::launch_ce_bwd(logits.data_ptr(), logits.stride(0), V, logits.size(0), lse.data_ptr<float>(),
                     targets.data_ptr<int64_t>(), gscale.data_ptr<float>(), (float)inv_count, stream(), col0);
}

// ------------------------------------------------------------ embedding / rope
void embed_fwd(torch::Tensor ids, torch::Tensor w, torch::Tensor out) {
  c10::cuda::CUDAGuard g(w.device());
  TORCH_CHECK(ids.scalar_type() == torch::kInt64 && ids.is_contiguous(), "ids must be contiguous int64");
  TORCH_CHECK(w.scalar_type() == torch::kBFloat16 && w.is_contiguous() && out.is_contiguous(), "embedding tensors");
  oxi::launch_embed_fwd(ids.data_ptr<int64_t>(), w.data_ptr(), out.data_ptr(), ids.numel(), (int)w.size(1), stream());
}

void embed_bwd(torch::Tensor ids, torch::Tensor dy, torch::Tensor dw) {
  c10::cuda::CUDAGuard g(dy.device());
  TORCH_CHECK(dw.scalar_type() == torch::kFloat32 && dw.is_contiguous() && dy.is_contiguous(), "embedding grad");
  oxi::launch_embed_bwd(ids.data_ptr<int64_t>(), dy.data_ptr(), dw.data_ptr<float>(), ids.numel(), (int)dw.size(1),
                        stream());
}

void rope_bwd(torch::Tensor x, int64_t ncols_rot, int64_t hd, torch::Tensor cos, torch::Tensor sin) {
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "rope_bwd x");
  oxi::launch_rope_bwd(x.data_ptr(), x.stride(0), x.size(0), (int)ncols_rot, (int)hd, cos.data_ptr<float>(),
                       sin.data_ptr<float>(), (int)cos.size(0), stream());
}

torch::Tensor rope_bwd_to(torch::Tensor x, int64_t ncols_rot, int64_t hd, torch::Tensor cos, torch::Tensor sin) {
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "rope_bwd_to x");
  auto out = torch::empty({x.size(0), x.size(1)}, x.options());
  oxi::launch_rope_bwd_to(x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0), x.size(0), (int)ncols_rot,
                          (int)x.size(1), (int)hd, cos.data_ptr<float>(), sin.data_ptr<float>(), (int)cos.size(0),
                          stream());
  return out;
}

// ------------------------------------------------------------ optimizer
void sqsum(torch::Tensor g, torch::Tensor out) {
  c10::cuda::CUDAGuard gd(g.device());
  TORCH_CHECK(g.scalar_type() == torch::kFloat32 && g.is_contiguous(), "sqsum input must be contiguous f32");
  oxi::launch_sqsum(g.data_ptr<float>(), g.numel(), out.data_ptr<float>(), stream());
}

void colsum_add(torch::Tensor x, torch::Tensor out) {
  c10::cuda::CUDAGuard gd(x.device());
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.scalar_type() == torch::kBFloat16 && x.stride(1) == 1,
              "colsum: bf16 [rows, N] with unit inner stride");
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.is_contiguous() && out.numel() == x.size(1),
              "colsum: out f32 [N]");
  oxi::launch_colsum_bf16(x.data_ptr(), x.size(0), (int)x.size(1), x.stride(0), out.data_ptr<float>(), stream());
}

void clip_coef(torch::Tensor sq, double max_norm, double pre_scale, torch::Tensor coef, torch::Tensor norm,
               c10::optional<torch::Tensor> step_state, double b1, double b2, c10::optional<torch::Tensor> skip) {
  c10::cuda::CUDAGuard gd(sq.device());
  float* ss = nullptr;
  if (step_state.has_value() && step_state->defined()) {
    TORCH_CHECK(step_state->scalar_type() == torch::kFloat32 && step_state->is_contiguous() &&
                    step_state->numel() == 3, "step_state: f32 [3]");
    ss = step_state->data_ptr<float>();
  }
  const int* sk = nullptr;
  if (skip.has_value() && skip->defined()) {
    TORCH_CHECK(skip->scalar_type() == torch::kInt32 && skip->is_cuda(), "skip: int32 CUDA word");
    sk = skip->data_ptr<int>();
  }
  oxi::launch_clip_coef(sq.data_ptr<float>(), (float)max_norm, (float)pre_scale, coef.data_ptr<float>(),
                        norm.data_ptr<float>(), stream(), ss, (float)b1, (float)b2, sk);
}

void adamw(torch::Tensor p, c10::optional<torch::Tensor> p16, torch::Tensor g, torch::Tensor m, torch::Tensor v,
           double lr, double b1, double b2, double eps, double wd, double bc1, double bc2,
           c10::optional<torch::Tensor> gscale, c10::optional<torch::Tensor> bc_dev) {
  c10::cuda::CUDAGuard gd(p.device());
  TORCH_CHECK(p.scalar_type() == torch::kFloat32 && g.scalar_type() == torch::kFloat32 && p.is_contiguous() &&
                  g.is_contiguous() && m.is_contiguous() && v.is_contiguous() && p.numel() == g.numel() &&
                  m.numel() == p.numel() && v.numel() == p.numel(), "adamw: flat f32 buffers of equal size");
  void* p16p = nullptr;
  if (p16.has_value() && p16->defined()) {
    TORCH_CHECK(p16->scalar_type() == torch::kBFloat16 && p16->numel() == p.numel() && p16->is_contiguous(), "p16");
    p16p = p16->data_ptr();
  }
  oxi::launch_adamw(p.data_ptr<float>(), p16p, g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                    p.numel(), (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, (float)bc1, (float)bc2,
                    gscale.has_value() && gscale->defined() ? gscale->data_ptr<float>() : nullptr, stream(),
                    bc_dev.has_value() && bc_dev->defined() ? bc_dev->data_ptr<float>() : nullptr);
}

// ------------------------------------------------------------ attention
// q, k, v: [B*S, H*D]-shaped row-major bf16 views (unit inner stride)
void flash_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor lse, int64_t B,
               int64_t S, int64_t Hq, int64_t Hk, int64_t Dqk, int64_t Dv, double scale, bool causal,
               torch::Tensor status) {
  c10::cuda::CUDAGuard g(q.device());
  for (auto* t : {&q, &k, &v, &o})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kBFloat16 && t->dim() == 2 && t->stride(1) == 1 &&
                    t->size(0) == B * S, "attention operands must be bf16 [B*S, H*D] with unit inner stride");
  TORCH_CHECK(q.size(1) == Hq * Dqk && k.size(1) == Hk * Dqk && v.size(1) == Hk * Dv && o.size(1) == Hq * Dv,
              "head dims");
  TORCH_CHECK(lse.scalar_type() == torch::kFloat32 && lse.numel() == B * Hq * S && lse.is_contiguous(), "lse");
  oxi::launch_fa_fwd(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), o.data_ptr(),
                     o.stride(0), lse.data_ptr<float>(), (int)B, (int)S, (int)Hq, (int)Hk, (int)Dqk, (int)Dv,
                     (float)scale, causal, status_ptr(status), stream());
}

void flash_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
               torch::Tensor lse, torch::Tensor delta, torch::Tensor dq_acc, torch::Tensor dq, torch::Tensor dk,
               torch::Tensor dv, int64_t B, int64_t S, int64_t Hq, int64_t Hk, int64_t Dqk, int64_t Dv, double scale,
               bool causal, torch::Tensor status, std::optional<torch::Tensor> rope_cos,
               std::optional<torch::Tensor> rope_sin) {
  c10::cuda::CUDAGuard g(q.device());
  for (auto* t : {&q, &k, &v, &o, &dout, &dq, &dk, &dv})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kBFloat16 && t->dim() == 2 && t->stride(1) == 1 &&
                    t->size(0) == B * S, "attention tensors must be bf16 [B*S, H*D] with unit inner stride");
  TORCH_CHECK(dq.size(1) == Hq * Dqk && dk.size(1) == Hk * Dqk && dv.size(1) == Hk * Dv, "gradient head dims");
  TORCH_CHECK(dq_acc.scalar_type() == torch::kFloat32 && dq_acc.is_contiguous() && dq_acc.numel() == B * S * Hq * Dqk,
              "dq_acc must be contiguous f32 [B*S, Hq*Dqk]");
  TORCH_CHECK(delta.scalar_type() == torch::kFloat32 && delta.numel() == B * Hq * S, "delta");
  const float* rc = nullptr;
  const float* rs = nullptr;
  if (rope_cos.has_value() && rope_cos->defined()) {
    TORCH_CHECK(rope_sin.has_value() && rope_sin->defined(), "rope_cos without rope_sin");
    for (auto* t : {&*rope_cos, &*rope_sin})
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat32 && t->is_contiguous() &&
                      t->numel() >= S * (Dqk / 2), "RoPE tables must be contiguous f32 [>= S, Dqk/2]");
    rc = rope_cos->data_ptr<float>();
    rs = rope_sin->data_ptr<float>();
  }
  oxi::launch_fa_bwd(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), o.data_ptr(),
                     o.stride(0), dout.data_ptr(), dout.stride(0), lse.data_ptr<float>(), delta.data_ptr<float>(),
                     dq_acc.data_ptr<float>(), dq.data_ptr(), dq.stride(0), dk.data_ptr(), dk.stride(0), dv.data_ptr(),
                     dv.stride(0), (int)B, (int)S, (int)Hq, (int)Hk, (int)Dqk, (int)Dv, (float)scale, causal,
                     status_ptr(status), stream(), rc, rs);
}

bool flash_supported(int64_t Dqk, int64_t Dv, bool backward) {
  return backward ? oxi::fa_bwd_supported((int)Dqk, (int)Dv) : oxi::fa_supported((int)Dqk, (int)Dv);
}

// ------------------------------------------------------------ NVLink DDP runtime
// Allocates nbytes of zeroed device memory exportable over CUDA IPC; returns
// (uint8 tensor owning it, IPC handle bytes).
std::tuple<torch::Tensor, py::bytes> ipc_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  std::string h;
  void* p = oxi::ipc_alloc((size_t)nbytes, &h);
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  torch::Tensor t = torch::from_blob(p, {nbytes}, [](void* q) { oxi::ipc_free(q); }, opts);
  return {t, py::bytes(h)};
}

int64_t ipc_open(py::bytes handle, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  return reinterpret_cast<int64_t>(oxi::ipc_open(std::string(handle)));
}

void ipc_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  oxi::ipc_close(reinterpret_cast<void*>(ptr));
}

int64_t pad_words() { return oxi::PAD_WORDS; }

void grad_to_bf16(torch::Tensor g, torch::Tensor out, bool zero) {
  c10::cuda::CUDAGuard gd(g.device());
  TORCH_CHECK(g.scalar_type() == torch::kFloat32 && out.scalar_type() == torch::kBFloat16 && g.numel() == out.numel()
              && g.is_contiguous() && out.is_contiguous(), "grad_to_bf16");
  oxi::launch_grad_to_bf16(g.data_ptr<float>(), out.data_ptr(), g.numel(), zero, stream());
}

void bf16_to_f32_sumsq(torch::Tensor src, torch::Tensor dst, torch::Tensor sumsq) {
  c10::cuda::CUDAGuard gd(src.device());
  TORCH_CHECK(src.scalar_type() == torch::kBFloat16 && dst.scalar_type() == torch::kFloat32 &&
                  src.numel() == dst.numel() && src.is_contiguous() && dst.is_contiguous() &&
                  sumsq.scalar_type() == torch::kFloat32,
              "bf16_to_f32_sumsq: bf16 src, f32 dst of the same size, f32 sumsq");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(src.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(dst.data_ptr()) & 15) == 0,
              "bf16_to_f32_sumsq: 16-byte aligned buffers");
  oxi::launch_bf16_to_f32_sumsq(src.data_ptr(), dst.data_ptr<float>(), src.numel(), sumsq.data_ptr<float>(),
                                stream());
}

void rs_bucket(int64_t mode, torch::Tensor grad, bool zero_grad, torch::Tensor peers_buf, torch::Tensor my_buf,
               int64_t mc_buf, torch::Tensor peer_pads, torch::Tensor my_pad, torch::Tensor done_ctr, int64_t rank,
               int64_t W, int64_t bucket, int64_t epoch, int64_t lo, int64_t len, torch::Tensor rgrad_shard,
               torch::Tensor sumsq, int64_t ctas, torch::Tensor status, int64_t wait_ns) {
  c10::cuda::CUDAGuard gd(my_pad.device());
  TORCH_CHECK(grad.scalar_type() == torch::kFloat32 && grad.is_contiguous(), "grad must be contiguous f32");
  TORCH_CHECK(done_ctr.scalar_type() == torch::kInt32 && done_ctr.numel() >= oxi::PAD_MAXB, "done_ctr");
  TORCH_CHECK(lo >= 0 && len >= 0 && lo + len <= grad.numel() && rgrad_shard.numel() >= len / std::max<int64_t>(W, 1),
              "bucket range outside the gradient buffer");
  oxi::launch_rs_bucket((int)mode, grad.data_ptr<float>(), zero_grad,
                        reinterpret_cast<const uint64_t*>(peers_buf.data_ptr<int64_t>()), my_buf.data_ptr(),
                        reinterpret_cast<void*>(mc_buf), reinterpret_cast<const uint64_t*>(peer_pads.data_ptr<int64_t>()),
                        my_pad.data_ptr<int>(), done_ctr.data_ptr<int>(), (int)rank, (int)W, (int)bucket, (int)epoch,
                        lo, len, rgrad_shard.data_ptr<float>(), sumsq.data_ptr<float>(), (int)ctas,
                        status_ptr(status), wait_ns, stream());
}

void norm_exchange(torch::Tensor peer_pads, torch::Tensor my_pad, int64_t rank, int64_t W, int64_t epoch,
                   torch::Tensor sumsq, double max_norm, torch::Tensor coef, torch::Tensor norm, torch::Tensor status,
                   int64_t wait_ns, c10::optional<torch::Tensor> skip) {
  c10::cuda::CUDAGuard gd(my_pad.device());
  const int* sk = nullptr;
  if (skip.has_value() && skip->defined()) {
    TORCH_CHECK(skip->scalar_type() == torch::kInt32 && skip->is_cuda(), "skip: int32 CUDA word");
    sk = skip->data_ptr<int>();
  }
  oxi::launch_norm_exchange(reinterpret_cast<const uint64_t*>(peer_pads.data_ptr<int64_t>()), my_pad.data_ptr<int>(),
                            (int)rank, (int)W, (int)epoch, sumsq.data_ptr<float>(), (float)max_norm,
                            coef.data_ptr<float>(), norm.data_ptr<float>(), status_ptr(status), wait_ns, sk,
                            stream());
}

void adamw_ag_bucket(int64_t mode, int64_t lo, int64_t len, int64_t so, int64_t W, int64_t rank, int64_t ndst,
                     torch::Tensor rgrad, torch::Tensor master, torch::Tensor m, torch::Tensor v,
                     torch::Tensor peers_param, int64_t mc_param, c10::optional<torch::Tensor> peer_pads,
                     int64_t bucket, int64_t epoch, double lr, double b1, double b2, double eps, double wd, double bc1,
                     double bc2, torch::Tensor coef, torch::Tensor done_ctr, torch::Tensor status, int64_t ctas) {
  c10::cuda::CUDAGuard gd(master.device());
  TORCH_CHECK(rgrad.scalar_type() == torch::kFloat32 && master.scalar_type() == torch::kFloat32 &&
                  m.scalar_type() == torch::kFloat32 && v.scalar_type() == torch::kFloat32,
              "adamw_ag_bucket: f32 shard state");
  TORCH_CHECK(W >= 1 && so >= 0 && so + len / W <= master.numel() && rgrad.numel() == master.numel() &&
                  m.numel() == master.numel() && v.numel() == master.numel(),
              "adamw_ag_bucket: shard range outside the optimizer state");
  const uint64_t* pads = nullptr;
  if (peer_pads.has_value() && peer_pads->defined())
    pads = reinterpret_cast<const uint64_t*>(peer_pads->data_ptr<int64_t>());
  oxi::launch_adamw_ag_bucket((int)mode, lo, len, so, (int)W, (int)rank, (int)ndst, rgrad.data_ptr<float>(),
                              master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                              reinterpret_cast<const uint64_t*>(peers_param.data_ptr<int64_t>()),
                              reinterpret_cast<void*>(mc_param), pads, (int)bucket, (int)epoch, (float)lr, (float)b1,
                              (float)b2, (float)eps, (float)wd, (float)bc1, (float)bc2, coef.data_ptr<float>(),
                              done_ctr.data_ptr<int>(), status_ptr(status), (int)ctas, stream());
}

void ag_wait(torch::Tensor my_pad, int64_t W, int64_t bucket, int64_t epoch, torch::Tensor status, int64_t wait_ns) {
  c10::cuda::CUDAGuard gd(my_pad.device());
  oxi::launch_ag_wait(my_pad.data_ptr<int>(), (int)W, (int)bucket, (int)epoch, status_ptr(status), wait_ns, stream());
}

// ------------------------------------------------------------ Mamba3 scan coefficients
namespace {
void m3c_check(const torch::Tensor& t, int64_t T, int64_t H, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16 && t.is_contiguous() && t.numel() == T * H, what,
              ": bf16 contiguous [T, H]");
}
const float* opt_f32(const c10::optional<torch::Tensor>& t, int64_t n) {
  if (!t.has_value() || !t->defined()) return nullptr;
  TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat32 && t->is_contiguous() && t->numel() == n,
              "coefficient gradient: f32 contiguous [T, H]");
  return t->data_ptr<float>();
}
}  // namespace

std::vector<torch::Tensor> m3_coef_fwd(torch::Tensor dt_raw, torch::Tensor bias, torch::Tensor lam_raw,
                                       torch::Tensor A, int64_t S, double lo, double hi) {
  c10::cuda::CUDAGuard g(dt_raw.device());
  const int64_t H = bias.numel(), T = dt_raw.numel() / std::max<int64_t>(H, 1);
  m3c_check(dt_raw, T, H, "dt_raw");
  m3c_check(lam_raw, T, H, "lam_raw");
  TORCH_CHECK(bias.scalar_type() == torch::kBFloat16 && bias.is_contiguous() && A.scalar_type() == torch::kFloat32 &&
                  A.is_contiguous() && A.numel() == H, "dt_bias bf16 [H], A f32 [H]");
  auto o = dt_raw.options().dtype(torch::kFloat32);
  auto dt = torch::empty({T, H}, o), loga = torch::empty({T, H}, o), gp = torch::empty({T, H}, o),
       c = torch::empty({T, H}, o);
  oxi::launch_m3_coef_fwd(dt_raw.data_ptr(), bias.data_ptr(), lam_raw.data_ptr(), A.data_ptr<float>(), T, (int)S,
                          (int)H, (float)lo, (float)hi, dt.data_ptr<float>(), loga.data_ptr<float>(),
                          gp.data_ptr<float>(), c.data_ptr<float>(), stream());
  return {dt, loga, gp, c};
}

std::vector<torch::Tensor> m3_coef_bwd(torch::Tensor dt_raw, torch::Tensor bias, torch::Tensor lam_raw,
                                       torch::Tensor A, int64_t S, double lo, double hi,
                                       c10::optional<torch::Tensor> d_dt, c10::optional<torch::Tensor> d_loga,
                                       c10::optional<torch::Tensor> d_gp, c10::optional<torch::Tensor> d_c) {
  c10::cuda::CUDAGuard g(dt_raw.device());
  const int64_t H = bias.numel(), T = dt_raw.numel() / std::max<int64_t>(H, 1);
  m3c_check(dt_raw, T, H, "dt_raw");
  m3c_check(lam_raw, T, H, "lam_raw");
  auto ddt_raw = torch::empty_like(dt_raw), dlam_raw = torch::empty_like(lam_raw);
  auto dbias = torch::zeros({H}, dt_raw.options().dtype(torch::kFloat32)), dA = torch::zeros_like(dbias);
  oxi::launch_m3_coef_bwd(dt_raw.data_ptr(), bias.data_ptr(), lam_raw.data_ptr(), A.data_ptr<float>(), T, (int)S,
                          (int)H, (float)lo, (float)hi, opt_f32(d_dt, T * H), opt_f32(d_loga, T * H),
                          opt_f32(d_gp, T * H), opt_f32(d_c, T * H), ddt_raw.data_ptr(), dlam_raw.data_ptr(),
                          dbias.data_ptr<float>(), dA.data_ptr<float>(), stream());
  return {ddt_raw, dlam_raw, dbias, dA};
}

// ------------------------------------------------------------ multi-head latent attention
namespace {
void mla_check(const torch::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16 && t.dim() == 2 && t.stride(1) == 1 &&
                  (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0,
              what, ": bf16 CUDA [rows, cols] with unit inner stride and a 16-byte aligned start");
}
}  // namespace

std::vector<torch::Tensor> mla_pack_fwd(torch::Tensor qc, torch::Tensor kv, torch::Tensor rp, torch::Tensor cos_t,
                                        torch::Tensor sin_t, int64_t S, int64_t nh, int64_t hd, int64_t dr) {
  c10::cuda::CUDAGuard g(qc.device());
  mla_check(qc, "q_c");
  mla_check(kv, "kv");
  TORCH_CHECK(rp.is_cuda() && rp.scalar_type() == torch::kBFloat16 && rp.dim() == 2 && rp.stride(1) == 1, "rope block");
  const int64_t T = qc.size(0);
  TORCH_CHECK(qc.size(1) == nh * hd && kv.size(0) == T && kv.size(1) == 2 * nh * hd && rp.size(0) == T &&
                  rp.size(1) == dr + nh * dr && T % S == 0,
              "MLA pack: q_c [T, nh*hd], kv [T, 2*nh*hd], rope block [T, dr + nh*dr], T a multiple of S");
  TORCH_CHECK(cos_t.scalar_type() == torch::kFloat32 && sin_t.scalar_type() == torch::kFloat32 &&
                  cos_t.is_contiguous() && sin_t.is_contiguous() && cos_t.size(0) >= S && cos_t.size(1) == dr / 2,
              "RoPE tables: f32 [>= S, dr/2]");
  auto o = qc.options();
  auto q = torch::empty({T, nh, hd + dr}, o), k = torch::empty({T, nh, hd + dr}, o), v = torch::empty({T, nh, hd}, o);
  oxi::launch_mla_pack_fwd(qc.data_ptr(), qc.stride(0), kv.data_ptr(), kv.stride(0), rp.data_ptr(), rp.stride(0),
                           cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), T, (int)S, (int)nh, (int)hd, (int)dr,
                           q.data_ptr(), k.data_ptr(), v.data_ptr(), stream());
  return {q, k, v};
}

std::vector<torch::Tensor> mla_pack_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor cos_t,
                                        torch::Tensor sin_t, int64_t S, int64_t nh, int64_t hd, int64_t dr) {
  c10::cuda::CUDAGuard g(dq.device());
  const int64_t T = dq.size(0);
  for (const torch::Tensor* t : {&dq, &dk, &dv})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kBFloat16 && t->is_contiguous() && t->size(0) == T &&
                    (reinterpret_cast<uintptr_t>(t->data_ptr()) & 15) == 0,
                "MLA pack backward: contiguous bf16 gradients with 16-byte aligned starts");
  TORCH_CHECK(dq.numel() == T * nh * (hd + dr) && dk.numel() == dq.numel() && dv.numel() == T * nh * hd && T % S == 0,
              "MLA pack backward: dq, dk [T, nh, hd + dr], dv [T, nh, hd]");
  auto o = dq.options();
  auto dqc = torch::empty({T, nh * hd}, o), dkv = torch::empty({T, 2 * nh * hd}, o),
       drp = torch::empty({T, dr + nh * dr}, o);
  oxi::launch_mla_pack_bwd(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), cos_t.data_ptr<float>(),
                           sin_t.data_ptr<float>(), T, (int)S, (int)nh, (int)hd, (int)dr, dqc.data_ptr(),
                           dkv.data_ptr(), drp.data_ptr(), stream());
  return {dqc, dkv, drp};
}

// ------------------------------------------------------------ expert parallelism (NVLink)
namespace {
const uint64_t* u64p(const torch::Tensor& t) {
  TORCH_CHECK(t.scalar_type() == torch::kInt64 && t.is_cuda() && t.is_contiguous(), "pointer tables: int64 CUDA");
  return reinterpret_cast<const uint64_t*>(t.data_ptr<int64_t>());
}
}  // namespace

int64_t ep_pad_words() { return oxi::EP_PAD_WORDS; }

std::vector<torch::Tensor> ep_counts(torch::Tensor local_counts, torch::Tensor peer_pads, torch::Tensor my_pad,
                                     int64_t rank, int64_t W, int64_t seq, int64_t cap, torch::Tensor overflow,
                                     torch::Tensor status, int64_t wait_ns) {
  c10::cuda::CUDAGuard g(my_pad.device());
  TORCH_CHECK(local_counts.scalar_type() == torch::kInt32 && local_counts.is_contiguous(), "counts int32");
  TORCH_CHECK(overflow.scalar_type() == torch::kInt32 && overflow.is_cuda() && overflow.numel() >= 2,
              "overflow: int32 CUDA [2] (flag, rows needed)");
  const int64_t E = local_counts.numel(), El = E / W;
  auto io = torch::TensorOptions().dtype(torch::kInt32).device(my_pad.device());
  auto all = torch::empty({W, E}, io), seg = torch::empty({El + 2}, io), rc = torch::empty({El}, io);
  int* ov = overflow.data_ptr<int>();
  oxi::launch_ep_counts(local_counts.data_ptr<int>(), u64p(peer_pads), my_pad.data_ptr<int>(), (int)rank, (int)W,
                        (int)E, (int)seq, all.data_ptr<int>(), seg.data_ptr<int>(), rc.data_ptr<int>(), (int)cap, ov,
                        ov + 1, status_ptr(status), wait_ns, stream());
  return {all, seg, rc};
}

torch::Tensor ep_dispatch(torch::Tensor x, torch::Tensor topi, torch::Tensor topw, torch::Tensor all_counts,
                          int64_t rank, int64_t W, torch::Tensor cursor, torch::Tensor peers_xrecv,
                          torch::Tensor peers_metaw, torch::Tensor peers_srcidx, torch::Tensor done_ctr,
                          torch::Tensor peer_pads, int64_t seq, torch::Tensor seg_off, torch::Tensor status) {
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x bf16 [T, H]");
  TORCH_CHECK(topi.scalar_type() == torch::kInt64 && topi.is_contiguous() && topw.is_contiguous() &&
                  topw.scalar_type() == torch::kFloat32, "topi int64 / topw f32 [T, k]");
  const int64_t T = topi.size(0), k = topi.size(1), E = all_counts.size(1);
  auto pos = torch::empty({T * k}, torch::TensorOptions().dtype(torch::kInt32).device(x.device()));
  oxi::launch_ep_dispatch(x.data_ptr(), x.stride(0), topi.data_ptr<int64_t>(), topw.data_ptr<float>(), T, (int)k,
                          (int)x.size(1), all_counts.data_ptr<int>(), (int)rank, (int)W, (int)E, cursor.data_ptr<int>(),
                          u64p(peers_xrecv), u64p(peers_metaw), u64p(peers_srcidx), pos.data_ptr<int>(),
                          done_ctr.data_ptr<int>(), u64p(peer_pads), (int)seq, seg_off.data_ptr<int>(),
                          status_ptr(status), stream());
  return pos;
}

void ep_mark_pad(torch::Tensor seg_off, torch::Tensor recv_counts, torch::Tensor srcidx) {
  c10::cuda::CUDAGuard g(srcidx.device());
  TORCH_CHECK(srcidx.scalar_type() == torch::kInt32 && srcidx.is_contiguous(), "srcidx int32");
  oxi::launch_ep_mark_pad(seg_off.data_ptr<int>(), recv_counts.data_ptr<int>(), (int)recv_counts.numel(),
                          srcidx.data_ptr<int>(), stream());
}

void ep_wait(torch::Tensor my_pad, int64_t kind, int64_t W, int64_t seq, torch::Tensor status, int64_t wait_ns) {
  c10::cuda::CUDAGuard g(my_pad.device());
  oxi::launch_ep_wait(my_pad.data_ptr<int>(), (int)kind, (int)W, (int)seq, status_ptr(status), wait_ns, stream());
}

void ep_signal(torch::Tensor peer_pads, int64_t kind, int64_t rank, int64_t W, int64_t seq) {
  c10::cuda::CUDAGuard g(peer_pads.device());
  oxi::launch_ep_signal(u64p(peer_pads), (int)kind, (int)rank, (int)W, (int)seq, stream());
}

// Grouped expert GEMM (group-M, bf16) whose epilogue stores row r into row
// srcidx[r] % rows_per_peer of peer srcidx[r] / rows_per_peer's buffer (P2P) and
// whose last CTA posts flag `kind` to every peer.
void ep_expert_gemm_scatter(torch::Tensor a, torch::Tensor b, bool b_mn, int64_t n_groups, torch::Tensor seg_off,
                            int64_t group_rows_b, torch::Tensor srcidx, torch::Tensor peers_out, int64_t rows_per_peer,
                            torch::Tensor post_ctr, torch::Tensor peer_pads, int64_t kind, int64_t rank, int64_t W,
                            int64_t seq, torch::Tensor status) {
  c10::cuda::CUDAGuard g(a.device());
  Mat ma = bf16_mat(a, "a"), mb = bf16_mat(b, "b");
  TORCH_CHECK(seg_off.scalar_type() == torch::kInt32 && seg_off.numel() >= n_groups + 1, "seg_off");
  TORCH_CHECK(srcidx.scalar_type() == torch::kInt32 && srcidx.numel() >= a.size(0), "srcidx int32 [rows]");
  const int64_t N = b_mn ? b.size(1) : group_rows_b;
  oxi::GroupedScatter sc;
  sc.idx = srcidx.data_ptr<int>();
  sc.ptrs = u64p(peers_out);
  sc.rows_per_peer = (int)rows_per_peer;
  sc.post_ctr = post_ctr.data_ptr<int>();
  sc.post_pads = u64p(peer_pads);
  sc.post_kind = (int)kind;
  sc.post_rank = (int)rank;
  sc.post_W = (int)W;
  sc.post_seq = (int)seq;
  // the destination rows are N wide and contiguous (row stride N)
  oxi::launch_gemm_grouped(1, 0, ma, false, mb, b_mn, (int)n_groups, seg_off.data_ptr<int>(), group_rows_b, nullptr,
                           N, nullptr, 0, nullptr, 0, status_ptr(status), stream(), &sc);
}

// wait for flag `wait_kind` from every owner, then out = (resid) + sum_j (w) * rows[t*k + j]
torch::Tensor ep_sum_pairs(torch::Tensor rows, c10::optional<torch::Tensor> w, int64_t T, int64_t k,
                           c10::optional<torch::Tensor> resid, torch::Tensor my_pad, int64_t wait_kind, int64_t W,
                           int64_t seq, torch::Tensor status, int64_t wait_ns) {
  c10::cuda::CUDAGuard g(rows.device());
  TORCH_CHECK(rows.scalar_type() == torch::kBFloat16 && rows.is_contiguous() && rows.dim() == 2 &&
                  rows.size(0) >= T * k, "rows bf16 [>= T*k, H]");
  const int64_t H = rows.size(1);
  auto out = torch::empty({T, H}, rows.options());
  const float* wp = nullptr;
  if (w.has_value() && w->defined()) {
    TORCH_CHECK(w->scalar_type() == torch::kFloat32 && w->is_contiguous() && w->numel() == T * k, "w f32 [T, k]");
    wp = w->data_ptr<float>();
  }
  const void* rp = nullptr;
  if (resid.has_value() && resid->defined()) {
    TORCH_CHECK(resid->is_contiguous() && resid->numel() == T * H && resid->scalar_type() == torch::kBFloat16,
                "resid bf16 [T, H] contiguous");
    rp = resid->data_ptr();
  }
  oxi::launch_ep_sum_pairs(rows.data_ptr(), wp, T, (int)k, (int)H, rp, out.data_ptr(), my_pad.data_ptr<int>(),
                           (int)wait_kind, (int)W, (int)seq, status_ptr(status), wait_ns, stream());
  return out;
}

torch::Tensor ep_push_dy(torch::Tensor dy, torch::Tensor topi, torch::Tensor pos, int64_t El,
                         torch::Tensor peers_dyrecv, torch::Tensor yret, torch::Tensor done_ctr,
                         torch::Tensor peer_pads, int64_t rank, int64_t W, int64_t seq, torch::Tensor seg_off,
                         torch::Tensor status) {
  c10::cuda::CUDAGuard g(dy.device());
  TORCH_CHECK(dy.scalar_type() == torch::kBFloat16 && dy.is_contiguous(), "dy bf16 contiguous");
  const int64_t T = topi.size(0), k = topi.size(1);
  TORCH_CHECK(yret.scalar_type() == torch::kBFloat16 && yret.is_contiguous() && yret.size(0) >= T * k &&
                  yret.size(1) == dy.size(-1), "yret bf16 [>= T*k, H]");
  auto dw = torch::empty({T, k}, torch::TensorOptions().dtype(torch::kFloat32).device(dy.device()));
  oxi::launch_ep_push_dy(dy.data_ptr(), topi.data_ptr<int64_t>(), pos.data_ptr<int>(), T, (int)k, (int)dy.size(-1),
                         (int)El, u64p(peers_dyrecv), yret.data_ptr(), dw.data_ptr<float>(), done_ctr.data_ptr<int>(),
                         u64p(peer_pads), (int)rank, (int)W, (int)seq, seg_off.data_ptr<int>(), status_ptr(status),
                         stream());
  return dw;
}

void ep_scale_rows(torch::Tensor dyrecv, torch::Tensor metaw, torch::Tensor seg_off, torch::Tensor recv_counts,
                   int64_t El) {
  c10::cuda::CUDAGuard g(dyrecv.device());
  oxi::launch_ep_scale_rows(dyrecv.data_ptr(), metaw.data_ptr<float>(), seg_off.data_ptr<int>(),
                            recv_counts.data_ptr<int>(), (int)El, (int)dyrecv.size(1), dyrecv.size(0), stream());
}

// ------------------------------------------------------------ NVLink microbenchmarks
bool enable_peer_access(int64_t device, int64_t peer) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  int can = 0;
  C10_CUDA_CHECK(cudaDeviceCanAccessPeer(&can, (int)device, (int)peer));
  if (!can) return false;
  cudaError_t e = cudaDeviceEnablePeerAccess((int)peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return true;
  }
  C10_CUDA_CHECK(e);
  return true;
}

// ------------------------------------------------------------ tensor-core SSD
namespace {
void ssd_check(const torch::Tensor& t, int64_t rows, int64_t cols, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16 && t.dim() == 2 && t.stride(1) == 1 &&
                  t.size(0) == rows && t.size(1) >= cols, what, ": bf16 [rows, >= cols] with unit inner stride");
}
}  // namespace

bool ssd_tc_supported(int64_t N, int64_t P, int64_t S) { return oxi::ssd_tc_supported((int)N, (int)P, (int)S); }

// Returns {y f32, hs bf16} and, when dskip is given, out = bf16(y + dskip x) third.
std::vector<torch::Tensor> ssd_tc_fwd(torch::Tensor x, torch::Tensor Bm, torch::Tensor Cm, torch::Tensor loga,
                                      torch::Tensor gamma, int64_t B, int64_t S, int64_t H, int64_t P, int64_t G,
                                      torch::Tensor status, c10::optional<torch::Tensor> dskip) {
  c10::cuda::CUDAGuard g(x.device());
  ssd_check(x, B * S, H * P, "x");
  ssd_check(Bm, B * S, G * 128, "B");
  ssd_check(Cm, B * S, G * 128, "C");
  TORCH_CHECK(loga.scalar_type() == torch::kFloat32 && loga.is_contiguous() && loga.numel() == B * S * H &&
                  gamma.scalar_type() == torch::kFloat32 && gamma.is_contiguous() && gamma.numel() == B * S * H,
              "loga / gamma: f32 contiguous [B, S, H]");
  const int64_t nc = S / 128;
  auto f32 = x.options().dtype(torch::kFloat32);
  auto y = torch::empty({B * S, H * P}, f32);
  auto hs = torch::empty({B * H * nc * 128, P}, x.options());
  auto hloc = torch::empty({B * H * nc * 128, P}, f32);
  auto lamend = torch::empty({B * H * nc}, f32);
  oxi::SsdTcIO io{};
  io.B = (int)B; io.S = (int)S; io.H = (int)H; io.P = (int)P; io.N = 128; io.G = (int)G;
  io.x = x.data_ptr(); io.ldx = x.stride(0);
  io.Bm = Bm.data_ptr(); io.ldb = Bm.stride(0);
  io.Cm = Cm.data_ptr(); io.ldc = Cm.stride(0);
  io.loga = loga.data_ptr<float>(); io.gamma = gamma.data_ptr<float>();
  io.y = y.data_ptr<float>(); io.hs = hs.data_ptr();
  io.hloc = hloc.data_ptr<float>(); io.lamend = lamend.data_ptr<float>();
  torch::Tensor out;
  if (dskip.has_value() && dskip->defined()) {
    TORCH_CHECK(dskip->scalar_type() == torch::kFloat32 && dskip->is_contiguous() &&
                    (dskip->numel() == B * S * H || dskip->numel() == H),
                "dskip: f32 contiguous [B, S, H] or [H]");
    out = torch::empty({B * S, H * P}, x.options());
    io.out = out.data_ptr();
    io.dskip = dskip->data_ptr<float>();
    io.dskip_per_row = dskip->numel() == B * S * H && B * S > 1 ? 1 : 0;
  }
  io.status = status_ptr(status);
  oxi::launch_ssd_fwd(io, stream());
  if (out.defined()) return {y, hs, out};
  return {y, hs};
}

std::vector<torch::Tensor> ssd_tc_bwd(torch::Tensor x, torch::Tensor Bm, torch::Tensor Cm, torch::Tensor loga,
                                      torch::Tensor gamma, torch::Tensor hs, torch::Tensor dy, int64_t B, int64_t S,
                                      int64_t H, int64_t P, int64_t G, torch::Tensor status) {
  c10::cuda::CUDAGuard g(x.device());
  ssd_check(x, B * S, H * P, "x");
  ssd_check(Bm, B * S, G * 128, "B");
  ssd_check(Cm, B * S, G * 128, "C");
  TORCH_CHECK(dy.scalar_type() == torch::kBFloat16 && dy.is_contiguous() && dy.numel() == B * S * H * P,
              "dy: bf16 contiguous [B*S, H*P]");
  TORCH_CHECK(hs.is_contiguous() && hs.scalar_type() == torch::kBFloat16, "hs");
  auto f32 = x.options().dtype(torch::kFloat32);
  auto dx = torch::empty({B * S, H * P}, f32);
  // every row written by the chunk pass; per-head B/C (G == H, bf16) get bf16 gradients
  const bool dbc_bf16 = G == H && Bm.scalar_type() == torch::kBFloat16;
  auto dB = torch::empty({B * S, H * 128}, dbc_bf16 ? x.options() : f32);
  auto dC = torch::empty({B * S, H * 128}, dbc_bf16 ? x.options() : f32);
  auto dg = torch::zeros({B, S, H}, f32);
  auto dhs = torch::empty_like(hs);
  oxi::SsdTcIO io{};
  io.B = (int)B; io.S = (int)S; io.H = (int)H; io.P = (int)P; io.N = 128; io.G = (int)G;
  io.x = x.data_ptr(); io.ldx = x.stride(0);
  io.Bm = Bm.data_ptr(); io.ldb = Bm.stride(0);
  io.Cm = Cm.data_ptr(); io.ldc = Cm.stride(0);
  io.loga = loga.data_ptr<float>(); io.gamma = gamma.data_ptr<float>();
  io.hs = hs.data_ptr(); io.dy = dy.data_ptr(); io.dhs = dhs.data_ptr();
  io.dx = dx.data_ptr<float>();
  io.dB = reinterpret_cast<float*>(dB.data_ptr()); io.dC = reinterpret_cast<float*>(dC.data_ptr());
  io.dbc_bf16 = dbc_bf16 ? 1 : 0;
  io.dgamma = dg.data_ptr<float>();
  const int64_t nc = S / 128;
  auto hloc = torch::empty({B * H * nc * 128, P}, f32);
  auto lamend = torch::empty({B * H * nc}, f32);
  io.hloc = hloc.data_ptr<float>(); io.lamend = lamend.data_ptr<float>();
  io.status = status_ptr(status);
  oxi::launch_ssd_bwd(io, stream());
  return {dx, dB, dC, dg};
}

// ------------------------------------------------------------ Mamba3 B/C prologue
std::vector<torch::Tensor> m3_bc_fwd(torch::Tensor braw, torch::Tensor craw, torch::Tensor w, torch::Tensor bbias,
                                     torch::Tensor cbias, torch::Tensor ang, int64_t B, int64_t S, int64_t H,
                                     int64_t G, double eps) {
  c10::cuda::CUDAGuard g(braw.device());
  TORCH_CHECK(braw.scalar_type() == torch::kBFloat16 && craw.scalar_type() == torch::kBFloat16 && braw.dim() == 2 &&
                  craw.dim() == 2 && braw.stride(1) == 1 && craw.stride(1) == 1 && braw.stride(0) == craw.stride(0),
              "B/C raw: bf16 [B*S, G*N] views sharing a row stride");
  TORCH_CHECK(ang.scalar_type() == torch::kFloat32 && ang.is_contiguous() && ang.numel() == B * S * H * 64, "ang");
  TORCH_CHECK(w.is_contiguous() && bbias.is_contiguous() && cbias.is_contiguous() &&
                  w.scalar_type() == torch::kBFloat16 && bbias.scalar_type() == torch::kBFloat16 &&
                  cbias.scalar_type() == torch::kBFloat16, "bc_norm weight / biases: bf16 contiguous");
  auto bo = torch::empty({B, S, H, 128}, braw.options());
  auto co = torch::empty({B, S, H, 128}, braw.options());
  auto dot = torch::empty({B, S, H}, braw.options().dtype(torch::kFloat32));
  oxi::launch_m3_bc_fwd(braw.data_ptr(), craw.data_ptr(), braw.stride(0), w.data_ptr(), bbias.data_ptr(),
                        cbias.data_ptr(), ang.data_ptr<float>(), (int)B, (int)S, (int)H, (int)G, 128, (float)eps,
                        bo.data_ptr(), co.data_ptr(), dot.data_ptr<float>(), stream());
  return {bo, co, dot};
}

std::vector<torch::Tensor> m3_bc_bwd(torch::Tensor braw, torch::Tensor craw, torch::Tensor w, torch::Tensor bbias,
                                     torch::Tensor cbias, torch::Tensor ang, torch::Tensor db, torch::Tensor dc,
                                     c10::optional<torch::Tensor> dbcdot, int64_t B, int64_t S, int64_t H, int64_t G,
                                     double eps) {
  c10::cuda::CUDAGuard g(braw.device());
  TORCH_CHECK(db.scalar_type() == dc.scalar_type() &&
                  (db.scalar_type() == torch::kFloat32 || db.scalar_type() == torch::kBFloat16) &&
                  db.is_contiguous() && dc.is_contiguous() && db.numel() == B * S * H * 128 && dc.numel() == db.numel(),
              "db / dc: f32 or bf16 contiguous [B, S, H, N]");
  const float* dd = nullptr;
  if (dbcdot.has_value() && dbcdot->defined()) {
    TORCH_CHECK(dbcdot->scalar_type() == torch::kFloat32 && dbcdot->is_contiguous() && dbcdot->numel() == B * S * H,
                "dbcdot: f32 contiguous [B, S, H]");
    dd = dbcdot->data_ptr<float>();
  }
  auto f32 = braw.options().dtype(torch::kFloat32);
  auto dbraw = torch::empty({B * S, G * 128}, f32);
  auto dcraw = torch::empty({B * S, G * 128}, f32);
  auto dw = torch::zeros({128}, f32);
  auto dbb = torch::zeros({H, 128}, f32);
  auto dcb = torch::zeros({H, 128}, f32);
  auto dang = torch::empty({B, S, H, 64}, f32);
  auto part = torch::empty({oxi::m3_bc_bwd_blocks(B * S), 2 * H * 128}, f32);
  oxi::launch_m3_bc_bwd(braw.data_ptr(), craw.data_ptr(), braw.stride(0), w.data_ptr(), bbias.data_ptr(),
                        cbias.data_ptr(), ang.data_ptr<float>(), db.data_ptr(), dc.data_ptr(),
                        db.scalar_type() == torch::kBFloat16, dd,
                        (int)B, (int)S, (int)H, (int)G, 128, (float)eps, dbraw.data_ptr<float>(),
                        dcraw.data_ptr<float>(), dbraw.stride(0), dw.data_ptr<float>(), dbb.data_ptr<float>(),
                        dcb.data_ptr<float>(), dang.data_ptr<float>(), stream(), part.data_ptr<float>());
  return {dbraw, dcraw, dw, dbb, dcb, dang};
}

torch::Tensor dskip_fwd(torch::Tensor y, torch::Tensor x, torch::Tensor d, int64_t H) {
  c10::cuda::CUDAGuard g(y.device());
  TORCH_CHECK(y.dim() == 2 && y.scalar_type() == torch::kFloat32 && y.is_contiguous(), "y: f32 contiguous [T, H*P]");
  TORCH_CHECK(x.sizes() == y.sizes() && x.scalar_type() == torch::kBFloat16 && x.is_contiguous(), "x: bf16 like y");
  const int64_t rows = y.size(0) * H, P = y.size(1) / H;
  TORCH_CHECK(d.scalar_type() == torch::kFloat32 && d.is_contiguous() && (d.numel() == rows || d.numel() == H),
              "d: f32 [T, H] or [H]");
  auto out = torch::empty(y.sizes(), x.options());
  oxi::launch_dskip_fwd(y.data_ptr<float>(), x.data_ptr(), d.data_ptr<float>(), rows, (int)H, (int)P,
                        d.numel() == rows && rows != H, out.data_ptr(), stream());
  return out;
}

std::vector<torch::Tensor> dskip_bwd(torch::Tensor gout, torch::Tensor x, torch::Tensor y, torch::Tensor d,
                                     torch::Tensor dx_scan, int64_t H) {
  c10::cuda::CUDAGuard g(y.device());
  TORCH_CHECK(y.dim() == 2 && y.scalar_type() == torch::kFloat32 && y.is_contiguous(), "y: f32 contiguous [T, H*P]");
  TORCH_CHECK(x.sizes() == y.sizes() && x.scalar_type() == torch::kBFloat16 && x.is_contiguous(), "x: bf16 like y");
  TORCH_CHECK(gout.sizes() == y.sizes() && gout.scalar_type() == torch::kBFloat16 && gout.is_contiguous(),
              "grad: bf16 like y");
  TORCH_CHECK(dx_scan.sizes() == y.sizes() && dx_scan.scalar_type() == torch::kFloat32 && dx_scan.is_contiguous(),
              "dx_scan: f32 like y");
  const int64_t rows = y.size(0) * H, P = y.size(1) / H;
  TORCH_CHECK(d.scalar_type() == torch::kFloat32 && d.is_contiguous() && (d.numel() == rows || d.numel() == H),
              "d: f32 [T, H] or [H]");
  auto dx = torch::empty(y.sizes(), x.options());
  auto dd = torch::empty({y.size(0), H}, y.options());
  auto e = torch::empty({y.size(0), H}, y.options());
  oxi::launch_dskip_bwd(gout.data_ptr(), x.data_ptr(), y.data_ptr<float>(), d.data_ptr<float>(),
                        dx_scan.data_ptr<float>(), rows, (int)H, (int)P, d.numel() == rows && rows != H, dx.data_ptr(),
                        dd.data_ptr<float>(), e.data_ptr<float>(), stream());
  return {dx, dd, e};
}

torch::Tensor ssd_dloga(torch::Tensor e, torch::Tensor ga, torch::Tensor dg) {
  c10::cuda::CUDAGuard g(e.device());
  TORCH_CHECK(e.dim() == 3 && e.scalar_type() == torch::kFloat32 && e.is_contiguous() && ga.sizes() == e.sizes() &&
                  dg.sizes() == e.sizes() && ga.scalar_type() == torch::kFloat32 &&
                  dg.scalar_type() == torch::kFloat32 && ga.is_contiguous() && dg.is_contiguous(),
              "e / gamma / dgamma: f32 contiguous [B, S, H]");
  const int64_t B = e.size(0), S = e.size(1), H = e.size(2);
  auto dla = torch::empty_like(e);
  auto sums = torch::empty({B * ((S + 127) / 128) * H}, e.options());
  oxi::launch_ssd_dloga(e.data_ptr<float>(), ga.data_ptr<float>(), dg.data_ptr<float>(), (int)B, (int)S, (int)H,
                        sums.data_ptr<float>(), dla.data_ptr<float>(), stream());
  return dla;
}

// ------------------------------------------------------------ Mamba3 angles
torch::Tensor angle_cumsum(torch::Tensor theta, torch::Tensor dt) {
  c10::cuda::CUDAGuard g(theta.device());
  TORCH_CHECK(theta.scalar_type() == torch::kFloat32 && theta.is_contiguous() && theta.dim() == 4 &&
                  dt.scalar_type() == torch::kFloat32 && dt.is_contiguous(), "theta f32 [B,S,H,J], dt f32 [B,S,H]");
  const int64_t B = theta.size(0), S = theta.size(1), H = theta.size(2), J = theta.size(3);
  auto ang = torch::empty_like(theta);
  auto sums = torch::empty({B * ((S + 127) / 128) * H * J}, theta.options());
  oxi::launch_angle_cumsum(theta.data_ptr<float>(), dt.data_ptr<float>(), (int)B, (int)S, (int)H, (int)J,
                           sums.data_ptr<float>(), ang.data_ptr<float>(), stream());
  return ang;
}

std::vector<torch::Tensor> angle_cumsum_bwd(torch::Tensor theta, torch::Tensor dt, torch::Tensor dang) {
  c10::cuda::CUDAGuard g(theta.device());
  TORCH_CHECK(dang.scalar_type() == torch::kFloat32 && dang.is_contiguous() && dang.sizes() == theta.sizes(), "dang");
  const int64_t B = theta.size(0), S = theta.size(1), H = theta.size(2), J = theta.size(3);
  auto dtheta = torch::empty_like(theta);
  auto ddt = torch::zeros_like(dt);
  auto sums = torch::empty({B * ((S + 127) / 128) * H * J}, theta.options());
  oxi::launch_angle_cumsum_bwd(theta.data_ptr<float>(), dt.data_ptr<float>(), dang.data_ptr<float>(), (int)B, (int)S,
                               (int)H, (int)J, sums.data_ptr<float>(), dtheta.data_ptr<float>(), ddt.data_ptr<float>(),
                               stream());
  return {dtheta, ddt};
}

// ------------------------------------------------------------ SSM
void conv1d_fwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias, torch::Tensor y, int64_t B,
                int64_t S, bool act) {
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1 && x.size(0) == B * S,
              "conv1d x must be bf16 [B*S, C] with unit inner stride");
  const int64_t C = x.size(1);
  TORCH_CHECK(w.scalar_type() == torch::kBFloat16 && w.is_contiguous() && w.numel() % C == 0, "conv1d weight");
  TORCH_CHECK(y.sizes() == x.sizes() && y.stride(1) == 1, "conv1d y");
  const void* bp = nullptr;
  if (bias.has_value() && bias->defined()) {
    TORCH_CHECK(bias->scalar_type() == torch::kBFloat16 && bias->numel() == C, "conv1d bias");
    bp = bias->data_ptr();
  }
  oxi::launch_conv1d_fwd(x.data_ptr(), x.stride(0), w.data_ptr(), bp, y.data_ptr(), y.stride(0), (int)B, (int)S,
                         (int)C, (int)(w.numel() / C), act, stream());
}

void conv1d_bwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias, torch::Tensor dy,
                torch::Tensor dx, torch::Tensor dw, c10::optional<torch::Tensor> db, int64_t B, int64_t S, bool act) {
  c10::cuda::CUDAGuard g(x.device());
  const int64_t C = x.size(1);
  TORCH_CHECK(dy.stride(1) == 1 && dx.stride(1) == 1 && dy.size(1) == C && dx.size(1) == C, "conv1d grads");
  TORCH_CHECK(dw.scalar_type() == torch::kFloat32 && dw.numel() == w.numel() && dw.is_contiguous(), "dw f32");
  const void* bp = nullptr;
  float* dbp = nullptr;
  if (bias.has_value() && bias->defined()) {
    bp = bias->data_ptr();
    TORCH_CHECK(db.has_value() && db->scalar_type() == torch::kFloat32 && db->numel() == C, "db f32");
    dbp = db->data_ptr<float>();
  }
  oxi::launch_conv1d_bwd(x.data_ptr(), x.stride(0), w.data_ptr(), bp, dy.data_ptr(), dy.stride(0), dx.data_ptr(),
                         dx.stride(0), dw.data_ptr<float>(), dbp, (int)B, (int)S, (int)C, (int)(w.numel() / C), act,
                         stream());
}

// x [B, S, H, P], Bm/Cm [B, S, H, N] (any strides), loga/gamma/beta [B, S, H]
static oxi::SsmScanIO scan_io(torch::Tensor x, torch::Tensor Bm, torch::Tensor Cm, torch::Tensor loga,
                              torch::Tensor gamma, c10::optional<torch::Tensor> beta) {
  for (auto* t : {&x, &Bm, &Cm, &loga, &gamma})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat32, "scan tensors must be f32 CUDA");
  TORCH_CHECK(x.dim() == 4 && Bm.dim() == 4 && Cm.dim() == 4 && loga.dim() == 3, "scan ranks");
  TORCH_CHECK(x.stride(3) == 1 && Bm.stride(3) == 1 && Cm.stride(3) == 1, "scan inner dims must be contiguous");
  TORCH_CHECK(Bm.strides() == Cm.strides(), "B and C must share strides");
  TORCH_CHECK(gamma.strides() == loga.strides(), "gamma/loga strides");
  oxi::SsmScanIO io{};
  io.x = x.data_ptr<float>(); io.Bm = Bm.data_ptr<float>(); io.Cm = Cm.data_ptr<float>();
  io.loga = loga.data_ptr<float>(); io.gamma = gamma.data_ptr<float>();
  if (beta.has_value() && beta->defined()) {
    TORCH_CHECK(beta->strides() == loga.strides(), "beta strides");
    io.beta = beta->data_ptr<float>();
  }
  for (int i = 0; i < 3; ++i) {
    io.xs[i] = x.stride(i);
    io.bs[i] = Bm.stride(i);
    io.ss[i] = loga.stride(i);
  }
  return io;
}

torch::Tensor ssm_scan_fwd(torch::Tensor x, torch::Tensor Bm, torch::Tensor Cm, torch::Tensor loga,
                           torch::Tensor gamma, c10::optional<torch::Tensor> beta) {
  c10::cuda::CUDAGuard g(x.device());
  auto io = scan_io(x, Bm, Cm, loga, gamma, beta);
  auto y = torch::empty_strided(x.sizes(), x.strides(), x.options());
  io.y = y.data_ptr<float>();
  oxi::launch_ssm_scan(io, x.size(0), x.size(1), x.size(2), Bm.size(3), x.size(3), io.beta != nullptr, 0, stream());
  return y;
}

// returns (dx, dB, dC, dgamma, dbeta); dB/dC have B's strides (a zero head stride sums over heads)
std::vector<torch::Tensor> ssm_scan_bwd(torch::Tensor x, torch::Tensor Bm, torch::Tensor Cm, torch::Tensor loga,
                                        torch::Tensor gamma, c10::optional<torch::Tensor> beta, torch::Tensor dy) {
  c10::cuda::CUDAGuard g(x.device());
  auto io = scan_io(x, Bm, Cm, loga, gamma, beta);
  TORCH_CHECK(dy.strides() == x.strides() && dy.scalar_type() == torch::kFloat32, "dy must match x");
  io.dy = dy.data_ptr<float>();
  auto dx = torch::empty_strided(x.sizes(), x.strides(), x.options());
  // gradient buffers with B's (possibly zero) strides: allocate the storage B spans
  auto make_like = [&](const torch::Tensor& t) {
    auto base = torch::zeros({t.size(0), t.size(1), t.stride(2) == 0 ? 1 : t.size(2), t.size(3)}, t.options());
    return base.expand(t.sizes());
  };
  auto dB = make_like(Bm), dC = make_like(Cm);
  TORCH_CHECK(dB.strides() == Bm.strides(), "B must be contiguous or a head-broadcast of a contiguous tensor");
  auto dgam = torch::zeros_like(gamma);
  torch::Tensor dbet;
  io.dx = dx.data_ptr<float>(); io.dB = dB.data_ptr<float>(); io.dC = dC.data_ptr<float>();
  io.dgamma = dgam.data_ptr<float>();
  if (io.beta) {
    dbet = torch::zeros_like(gamma);
    io.dbeta = dbet.data_ptr<float>();
  }
  const bool two = io.beta != nullptr;
  oxi::launch_ssm_scan(io, x.size(0), x.size(1), x.size(2), Bm.size(3), x.size(3), two, 1, stream());
  oxi::launch_ssm_scan(io, x.size(0), x.size(1), x.size(2), Bm.size(3), x.size(3), two, 2, stream());
  return {dx, dB, dC, dgam, dbet.defined() ? dbet : torch::Tensor()};
}

std::vector<torch::Tensor> mamba1_scan_fwd(torch::Tensor u, torch::Tensor delta, torch::Tensor A, torch::Tensor Bm,
                                           torch::Tensor Cm, double clamp) {
  c10::cuda::CUDAGuard g(u.device());
  for (auto* t : {&u, &delta, &A, &Bm, &Cm})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat32 && t->is_contiguous(), "mamba1 scan: f32 contiguous");
  const int64_t B = u.size(0), S = u.size(1), D = u.size(2);
  TORCH_CHECK(A.size(1) == 16 && Bm.size(2) == 16, "Mamba1 state size is 16");
  auto y = torch::empty_like(u);
  auto hs = torch::empty({B, S, D, 16}, u.options());
  oxi::launch_mamba1_fwd(u.data_ptr<float>(), delta.data_ptr<float>(), A.data_ptr<float>(), Bm.data_ptr<float>(),
                         Cm.data_ptr<float>(), y.data_ptr<float>(), hs.data_ptr<float>(), (int)B, (int)S, (int)D,
                         (float)clamp, stream());
  return {y, hs};
}

std::vector<torch::Tensor> mamba1_scan_bwd(torch::Tensor u, torch::Tensor delta, torch::Tensor A, torch::Tensor Bm,
                                           torch::Tensor Cm, torch::Tensor hs, torch::Tensor dy, double clamp) {
  c10::cuda::CUDAGuard g(u.device());
  const int64_t B = u.size(0), S = u.size(1), D = u.size(2);
  auto dyc = dy.contiguous();
  auto du = torch::empty_like(u), ddelta = torch::empty_like(u);
  auto dA = torch::zeros_like(A), dB = torch::zeros_like(Bm), dC = torch::zeros_like(Cm);
  oxi::launch_mamba1_bwd(u.data_ptr<float>(), delta.data_ptr<float>(), A.data_ptr<float>(), Bm.data_ptr<float>(),
                         Cm.data_ptr<float>(), hs.data_ptr<float>(), dyc.data_ptr<float>(), du.data_ptr<float>(),
                         ddelta.data_ptr<float>(), dA.data_ptr<float>(), dB.data_ptr<float>(), dC.data_ptr<float>(),
                         (int)B, (int)S, (int)D, (float)clamp, stream());
  return {du, ddelta, dA, dB, dC};
}

// ------------------------------------------------------------ MoE
// returns (counts [E] i32, seg_off [E+1] i32, pos [T*k] i32, xp [rows_cap, H] bf16)
std::vector<torch::Tensor> moe_permute(torch::Tensor x, torch::Tensor topi, int64_t E, int64_t rows_cap) {
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "moe x");
  TORCH_CHECK(topi.scalar_type() == torch::kInt64 && topi.is_contiguous() && topi.dim() == 2, "topi int64 [T,k]");
  const int64_t T = topi.size(0), k = topi.size(1), H = x.size(1);
  auto io = torch::TensorOptions().dtype(torch::kInt32).device(x.device());
  auto counts = torch::empty({E}, io), seg = torch::empty({E + 1}, io), cursor = torch::empty({E}, io);
  auto pos = torch::empty({T * k}, io);
  auto xp = torch::empty({rows_cap, H}, x.options());
  oxi::launch_moe_permute(x.data_ptr(), x.stride(0), topi.data_ptr<int64_t>(), T, (int)k, (int)E, (int)H,
                          counts.data_ptr<int>(), seg.data_ptr<int>(), cursor.data_ptr<int>(), pos.data_ptr<int>(),
                          xp.data_ptr(), stream());
  return {counts, seg, pos, xp};
}

std::vector<torch::Tensor> router_fwd(torch::Tensor logits, int64_t k) {
  c10::cuda::CUDAGuard g(logits.device());
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1 &&
                  (logits.scalar_type() == torch::kBFloat16 || logits.scalar_type() == torch::kFloat32),
              "router logits must be bf16/f32 [T, E] with unit inner stride");
  const int64_t T = logits.size(0), E = logits.size(1);
  auto dev = logits.device();
  auto topi = torch::empty({T, k}, torch::TensorOptions().dtype(torch::kInt64).device(dev));
  auto topw = torch::empty({T, k}, torch::TensorOptions().dtype(torch::kFloat32).device(dev));
  auto usage = torch::empty({E}, torch::TensorOptions().dtype(torch::kFloat32).device(dev));
  auto counts = torch::empty({E}, torch::TensorOptions().dtype(torch::kInt32).device(dev));
  oxi::launch_router_fwd(logits.data_ptr(), logits.scalar_type() == torch::kBFloat16, logits.stride(0), T, (int)E,
                         (int)k, topi.data_ptr<int64_t>(), topw.data_ptr<float>(), usage.data_ptr<float>(),
                         counts.data_ptr<int>(), stream());
  return {topi, topw, usage, counts};
}

torch::Tensor router_bwd(torch::Tensor logits, torch::Tensor topi, torch::Tensor topw, torch::Tensor dtopw,
                         c10::optional<torch::Tensor> dusage) {
  c10::cuda::CUDAGuard g(logits.device());
  TORCH_CHECK(topi.is_contiguous() && topw.is_contiguous() && dtopw.is_contiguous() &&
                  dtopw.scalar_type() == torch::kFloat32 && dtopw.numel() == topw.numel(), "router bwd operands");
  const int64_t T = logits.size(0), E = logits.size(1), k = topi.size(1);
  auto dl = torch::empty({T, E}, logits.options());
  const float* du = nullptr;
  if (dusage.has_value() && dusage->defined()) {
    TORCH_CHECK(dusage->scalar_type() == torch::kFloat32 && dusage->is_contiguous() && dusage->numel() == E, "dusage");
    du = dusage->data_ptr<float>();
  }
  oxi::launch_router_bwd(logits.data_ptr(), logits.scalar_type() == torch::kBFloat16, logits.stride(0), T, (int)E,
                         (int)k, topi.data_ptr<int64_t>(), topw.data_ptr<float>(), dtopw.data_ptr<float>(), du,
                         dl.data_ptr(), dl.stride(0), stream());
  return dl;
}

void moe_zero_pad(torch::Tensor seg, torch::Tensor counts, torch::Tensor m) {
  c10::cuda::CUDAGuard g(m.device());
  oxi::launch_moe_zero_pad(seg.data_ptr<int>(), counts.data_ptr<int>(), (int)counts.numel(), m.data_ptr(),
                           (int)m.size(1), stream());
}

torch::Tensor moe_combine(torch::Tensor yp, torch::Tensor pos, torch::Tensor w, int64_t T, int64_t k,
                          c10::optional<torch::Tensor> resid) {
  c10::cuda::CUDAGuard g(yp.device());
  const int64_t H = yp.size(1);
  auto y = torch::empty({T, H}, yp.options());
  const void* rp = nullptr;
  if (resid.has_value() && resid->defined()) {
    TORCH_CHECK(resid->is_contiguous() && resid->numel() == T * H, "resid");
    rp = resid->data_ptr();
  }
  oxi::launch_moe_combine(yp.data_ptr(), pos.data_ptr<int>(), w.data_ptr<float>(), T, (int)k, (int)H, rp,
                          y.data_ptr(), stream());
  return y;
}

std::vector<torch::Tensor> moe_combine_bwd(torch::Tensor dy, torch::Tensor yp, torch::Tensor pos, torch::Tensor w,
                                           int64_t k) {
  c10::cuda::CUDAGuard g(dy.device());
  const int64_t T = dy.size(0), H = dy.size(1);
  auto dyp = torch::empty_like(yp);
  auto dw = torch::empty({T, k}, w.options());
  oxi::launch_moe_combine_bwd(dy.data_ptr(), yp.data_ptr(), pos.data_ptr<int>(), w.data_ptr<float>(), T, (int)k,
                              (int)H, dyp.data_ptr(), dw.data_ptr<float>(), stream());
  return {dyp, dw};
}

torch::Tensor moe_gather_sum(torch::Tensor dxp, torch::Tensor pos, int64_t T, int64_t k) {
  c10::cuda::CUDAGuard g(dxp.device());
  const int64_t H = dxp.size(1);
  auto dx = torch::empty({T, H}, dxp.options());
  oxi::launch_moe_gather_sum(dxp.data_ptr(), pos.data_ptr<int>(), T, (int)k, (int)H, dx.data_ptr(), stream());
  return dx;
}

void gemm_grouped(int64_t mode, int64_t epi, torch::Tensor a, bool a_mn, torch::Tensor b, bool b_mn, int64_t n_groups,
                  torch::Tensor seg_off, int64_t group_rows_b, torch::Tensor out, c10::optional<torch::Tensor> out2,
                  c10::optional<torch::Tensor> aux, torch::Tensor status) {
  c10::cuda::CUDAGuard g(a.device());
  Mat ma = bf16_mat(a, "a"), mb = bf16_mat(b, "b");
  TORCH_CHECK(seg_off.scalar_type() == torch::kInt32 && seg_off.numel() >= n_groups + 1, "seg_off");
  TORCH_CHECK(out.stride(-1) == 1, "out inner stride");
  void* o2 = nullptr;
  int64_t ld2 = 0;
  if (out2.has_value() && out2->defined()) { o2 = out2->data_ptr(); ld2 = out2->stride(0); }
  const void* ax = nullptr;
  int64_t ldax = 0;
  if (aux.has_value() && aux->defined()) { ax = aux->data_ptr(); ldax = aux->stride(0); }
  const int64_t ldo = out.stride(out.dim() - 2);
  oxi::launch_gemm_grouped((int)mode, (int)epi, ma, a_mn, mb, b_mn, (int)n_groups, seg_off.data_ptr<int>(),
                           group_rows_b, out.data_ptr(), ldo, o2, ld2, ax, ldax, status_ptr(status), stream());
}

}  // namespace

// Raises through the launchers' own error path (no CUDA involved), so a test
// can check that a failed host-side check reaches Python as an exception.
void host_check_selftest(int64_t v) { OXI_CHECK(v == 0, "value ", v, " of ", 2.5, " ", true); }

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("host_check_selftest", &host_check_selftest, "raise via the launcher error path unless v == 0");
  m.doc() = "oxidizr_b200 sm_100a kernels";
  m.def("gemm", &gemm, "tcgen05 GEMM out = alpha * a @ b^T (+bias) (+resid | + beta*out)", py::arg("a"),
        py::arg("a_mn"), py::arg("b"), py::arg("b_mn"), py::arg("out"), py::arg("resid"), py::arg("beta"),
        py::arg("alpha"), py::arg("status"), py::arg("bias") = py::none());
  m.def("gemm_swiglu", &gemm_swiglu, "GEMM with fused SwiGLU epilogue");
  m.def("gemm_swiglu_bwd", &gemm_swiglu_bwd, "GEMM with fused SwiGLU backward epilogue");
  m.def("gemm_ce", &gemm_ce, "lm_head GEMM with fused cross-entropy partials");
  m.def("gemm_rope", &gemm_rope, "QKV GEMM with fused rotate-half RoPE epilogue");
  m.def("norm_fwd", &norm_fwd, "RMSNorm / LayerNorm / gated RMSNorm forward");
  m.def("norm_bwd", &norm_bwd, "RMSNorm / LayerNorm / gated RMSNorm backward");
  m.def("ce_finish", &ce_finish, "combine CE partials into lse and per-row loss");
  m.def("swiglu_bwd", &swiglu_bwd, "SwiGLU backward, element-wise: dH and the saved gate / up -> dGU");
  m.def("ce_bwd", &ce_bwd, "in-place softmax-minus-onehot gradient of the logits (of a column chunk from col0)",
        py::arg("logits"), py::arg("V"), py::arg("lse"), py::arg("targets"), py::arg("gscale"), py::arg("inv_count"),
        py::arg("col0") = 0);
  m.def("embed_fwd", &embed_fwd, "embedding gather");
  m.def("embed_bwd", &embed_bwd, "embedding scatter-add into f32 grad");
  m.def("rope_bwd_to", &rope_bwd_to, "out-of-place RoPE backward (+ copy of the unrotated columns)");
  m.def("rope_bwd", &rope_bwd, "in-place inverse rotate-half RoPE");
  m.def("sqsum", &sqsum, "sum of squares (atomically added into out)");
  m.def("colsum_add", &colsum_add, "out += column sums of a bf16 matrix (bias gradients)");
  m.def("clip_coef", &clip_coef, "global-norm clip coefficient (and device step state) on device", py::arg("sq"),
        py::arg("max_norm"), py::arg("pre_scale"), py::arg("coef"), py::arg("norm"),
        py::arg("step_state") = py::none(), py::arg("b1") = 0.9, py::arg("b2") = 0.999,
        py::arg("skip") = py::none());
  m.def("adamw", &adamw, "flat multi-tensor AdamW (f32 master, bf16 copy)", py::arg("p"), py::arg("p16"),
        py::arg("g"), py::arg("m"), py::arg("v"), py::arg("lr"), py::arg("b1"), py::arg("b2"), py::arg("eps"),
        py::arg("wd"), py::arg("bc1"), py::arg("bc2"), py::arg("gscale") = py::none(),
        py::arg("bc_dev") = py::none());
  m.def("flash_fwd", &flash_fwd, "causal flash attention forward (tcgen05)");
  m.def("flash_bwd", &flash_bwd, "causal flash attention backward (tcgen05)");
  m.def("flash_supported", &flash_supported, "whether a flash kernel exists for head dims (qk, v)");
  m.def("conv1d_fwd", &conv1d_fwd, "depthwise causal conv1d (+bias, +SiLU) forward");
  m.def("conv1d_bwd", &conv1d_bwd, "depthwise causal conv1d backward");
  m.def("ssd_tc_supported", &ssd_tc_supported, "whether the tensor-core SSD handles (N, P, S)");
  m.def("ssd_tc_fwd", &ssd_tc_fwd, "tensor-core chunked SSD forward (chunk-parallel, optional fused D skip)",
        py::arg("x"), py::arg("Bm"), py::arg("Cm"), py::arg("loga"), py::arg("gamma"), py::arg("B"), py::arg("S"),
        py::arg("H"), py::arg("P"), py::arg("G"), py::arg("status"), py::arg("dskip") = py::none());
  m.def("ssd_tc_bwd", &ssd_tc_bwd, "tensor-core chunked SSD backward");
  m.def("angle_cumsum", &angle_cumsum, "Mamba3 rotation angles: cumsum over time of theta * dt");
  m.def("angle_cumsum_bwd", &angle_cumsum_bwd, "backward of angle_cumsum");
  m.def("m3_bc_fwd", &m3_bc_fwd, "Mamba3 B/C norm + bias + complex RoPE (+ <B, C> per head)");
  m.def("ssd_dloga", &ssd_dloga, "SSD d loga reverse scan");
  m.def("dskip_fwd", &dskip_fwd, "SSD D-skip epilogue: bf16(y + d x)");
  m.def("dskip_bwd", &dskip_bwd, "backward of dskip_fwd (+ <g, y> for d loga)");
  m.def("m3_bc_bwd", &m3_bc_bwd, "backward of m3_bc_fwd");
  m.def("ssm_scan_fwd", &ssm_scan_fwd, "Mamba2/3 selective scan forward");
  m.def("ssm_scan_bwd", &ssm_scan_bwd, "Mamba2/3 selective scan backward");
  m.def("mamba1_scan_fwd", &mamba1_scan_fwd, "Mamba1 selective scan forward (saves states)");
  m.def("mamba1_scan_bwd", &mamba1_scan_bwd, "Mamba1 selective scan backward");
  m.def("router_fwd", &router_fwd, "MoE router softmax + top-k + usage");
  m.def("router_bwd", &router_bwd, "MoE router backward");
  m.def("moe_permute", &moe_permute, "MoE counting-sort permutation into aligned expert segments");
  m.def("moe_zero_pad", &moe_zero_pad, "zero the padding rows of expert segments");
  m.def("moe_combine", &moe_combine, "weighted combine of expert outputs (+ residual)");
  m.def("moe_combine_bwd", &moe_combine_bwd, "backward of the combine");
  m.def("moe_gather_sum", &moe_gather_sum, "sum permuted rows back per token");
  m.def("gemm_grouped", &gemm_grouped, "grouped (per-expert) tcgen05 GEMM");
  m.def("ep_pad_words", &ep_pad_words, "int32 words of one expert-parallel signal pad");
  m.def("m3_coef_fwd", &m3_coef_fwd, "Mamba3 scan coefficients (dt, log alpha, gamma', c) in one pass");
  m.def("m3_coef_bwd", &m3_coef_bwd, "backward of the Mamba3 scan coefficients");
  m.def("mla_pack_fwd", &mla_pack_fwd, "MLA: q, k (shared k_rope, RoPE applied) and packed v from the projections");
  m.def("mla_pack_bwd", &mla_pack_bwd, "MLA: gradients of q_c, kv and the rope block from dq, dk, dv");
  m.def("ep_counts", &ep_counts, "expert-parallel count all-gather over NVLink");
  m.def("ep_dispatch", &ep_dispatch, "expert-parallel token dispatch (P2P stores)");
  m.def("ep_wait", &ep_wait, "bounded wait for an expert-parallel flag from every peer");
  m.def("ep_signal", &ep_signal, "post an expert-parallel flag to every peer");
  m.def("ep_mark_pad", &ep_mark_pad, "mark the padding rows of the expert segments (srcidx = -1)");
  m.def("ep_expert_gemm_scatter", &ep_expert_gemm_scatter,
        "grouped expert GEMM whose epilogue stores rows into the sources' buffers over NVLink, then posts a flag");
  m.def("ep_sum_pairs", &ep_sum_pairs, "wait for the owners, then the local weighted sum of each token's k rows");
  m.def("ep_push_dy", &ep_push_dy, "expert-parallel backward: push output gradients to the owners, routing-weight grads");
  m.def("ep_scale_rows", &ep_scale_rows, "owner side: scale received gradient rows by their routing weights");
  m.def("enable_peer_access", &enable_peer_access, "cudaDeviceEnablePeerAccess(device -> peer)");
  m.def("ipc_alloc", &ipc_alloc, "zeroed device buffer exportable over CUDA IPC");
  m.def("ipc_open", &ipc_open, "map a peer's IPC buffer");
  m.def("ipc_close", &ipc_close, "unmap a peer's IPC buffer");
  m.def("pad_words", &pad_words, "int32 words of one signal pad");
  m.def("grad_to_bf16", &grad_to_bf16, "f32 gradient -> bf16 NVLink payload (optionally clearing the source)");
  m.def("bf16_to_f32_sumsq", &bf16_to_f32_sumsq, "bf16 shard -> f32 copy + sum of squares");
  m.def("ag_wait", &ag_wait, "bounded wait for every rank's all-gather of one bucket");
  m.def("rs_bucket", &rs_bucket, "reduce-scatter of one gradient bucket (pull, push or NVLS)");
  m.def("norm_exchange", &norm_exchange, "cross-rank gradient norm and clip coefficient", py::arg("peer_pads"),
        py::arg("my_pad"), py::arg("rank"), py::arg("W"), py::arg("epoch"), py::arg("sumsq"), py::arg("max_norm"),
        py::arg("coef"), py::arg("norm"), py::arg("status"), py::arg("wait_ns"), py::arg("skip") = py::none());
  m.def("adamw_ag_bucket", &adamw_ag_bucket, "sharded AdamW + bf16 parameter all-gather of one bucket");
}
