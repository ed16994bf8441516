// Plain GEMM launcher (kernel in gemm_kernel.cuh): bf16 or f32 output.
// Upstream: the reference's Linear / matmul calls (Candle on cuBLAS), e.g. model.rs:238,248,367,377,
// mamba2.rs:563,611,673,732.
#include "gemm_kernel.cuh"
#include "kernels.h"

namespace oxi {

Operand to_operand(const Mat& m, bool mn) {
  Operand o;
  o.ptr = m.ptr;
  o.ld = m.ld;
  o.mn = mn;
  if (!mn) { o.rows = m.rows; o.k = m.cols; }
  else { o.rows = m.cols; o.k = m.rows; }
  return o;
}

void launch_gemm(const Mat& a, bool a_mn, const Mat& b, bool b_mn, void* out, int64_t ldo, bool out_f32,
                 const void* resid, int64_t ldr, float beta, float alpha, int* status, cudaStream_t st,
                 const void* bias) {
  Operand oa = to_operand(a, a_mn), ob = to_operand(b, b_mn);
  GemmParams p{};
  fill_common(p, oa, ob);
  use_pairs(p);
  p.alpha = alpha;
  p.D = out;
  p.ldd = ldo;
  p.status = status;
  if (p.M == 0 || p.N == 0) return;
  OXI_CHECK(p.K > 0, "GEMM with K == 0 must be handled by the caller");
  CUtensorMap ta = operand_tmap(oa, BM), tb = operand_tmap(ob, b_tile_rows(p));
  if (!out_f32) {
    p.vec_ok = aligned16(out, ldo, 2);
    p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
    if (resid) {
      p.R = reinterpret_cast<const __nv_bfloat16*>(resid);
      p.ldr = ldr;
      p.vec_ok = p.vec_ok && aligned16(resid, ldr, 2);
    }
    if (gemm_tma_epilogue() && aligned16(out, ldo, 2)) {
      const CUtensorMap td = make_tmap_out(out, p.M, p.N, ldo, false);
      p.tma_out = 1;
      launch_epi<EPI_BF16>(a_mn, b_mn, ta, tb, p, st, &td);
    } else {
      launch_epi<EPI_BF16>(a_mn, b_mn, ta, tb, p, st);
    }
  } else {
    OXI_CHECK(bias == nullptr, "bias epilogue only for bf16 output");
    p.vec_ok = aligned16(out, ldo, 4);
    p.beta = beta;
    if (beta == 1.0f) choose_splits(p);
    if (gemm_tma_epilogue() && aligned16(out, ldo, 4) && (beta == 0.0f || beta == 1.0f)) {
      // beta 1 (weight gradients, split-K partials): the epilogue's TMA adds in L2
      const CUtensorMap td = make_tmap_out(out, p.M, p.N, ldo, true);
      p.tma_out = beta == 1.0f ? 3 : 2;
      launch_epi<EPI_F32>(a_mn, b_mn, ta, tb, p, st, &td);
    } else {
      launch_epi<EPI_F32>(a_mn, b_mn, ta, tb, p, st);
    }
  }
}

}  // namespace oxi
