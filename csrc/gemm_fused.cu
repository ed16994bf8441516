// GEMM launchers with fused epilogues (kernel in gemm_kernel.cuh).
// Upstream: SwiGLU MLP model.rs:430-455; RoPE on q/k model.rs:68-117 (applied at
// model.rs:333-386); lm_head + cross-entropy model.rs:1002, trainer.rs:166-171.
#include "gemm_kernel.cuh"
#include "kernels.h"

namespace oxi {

Operand to_operand(const Mat& m, bool mn);

void launch_gemm_swiglu(const Mat& x, const Mat& w, void* h, int64_t ldh, void* gu, int64_t ldgu, int* status,
                        cudaStream_t st) {
  Operand oa = to_operand(x, false), ob = to_operand(w, false);
  GemmParams p{};
  fill_common(p, oa, ob);
  use_pairs(p);
  OXI_CHECK(p.N % 256 == 0, "SwiGLU GEMM needs 2*intermediate % 256 == 0");
  p.D = h;
  p.ldd = ldh;
  p.vec_ok = aligned16(h, ldh, 2);
  if (gu) {
    p.D2 = gu;
    p.ldd2 = ldgu;
    p.vec_ok = p.vec_ok && aligned16(gu, ldgu, 2);
  }
  p.status = status;
  if (p.M == 0) return;
  CUtensorMap ta = operand_tmap(oa, BM), tb = operand_tmap(ob, b_tile_rows(p));
  if (gemm_tma_swiglu() && aligned16(h, ldh, 2) && (!gu || aligned16(gu, ldgu, 2))) {
    const CUtensorMap th = make_tmap_out(h, p.M, p.N / 2, ldh, false);
    CUtensorMap tg;
    if (gu) tg = make_tmap_out(gu, p.M, p.N, ldgu, false);
    p.tma_out = 1;
    launch_t<false, false, EPI_SWIGLU>(ta, tb, p, st, &th, gu ? &tg : nullptr);
    return;
  }
  launch_t<false, false, EPI_SWIGLU>(ta, tb, p, st);
}

void launch_gemm_swiglu_bwd(const Mat& dy, const Mat& w_down, const void* gu, int64_t ldgu, void* dgu, int64_t lddgu,
                            int* status, cudaStream_t st) {
  Operand oa = to_operand(dy, false), ob = to_operand(w_down, true);
  GemmParams p{};
  fill_common(p, oa, ob);  // N = intermediate
  use_pairs(p);
  OXI_CHECK(p.N % 128 == 0, "intermediate must be a multiple of 128");
  p.D = dgu;
  p.ldd = lddgu;
  p.R = reinterpret_cast<const __nv_bfloat16*>(gu);
  p.ldr = ldgu;
  p.vec_ok = aligned16(dgu, lddgu, 2) && aligned16(gu, ldgu, 2);
  p.status = status;
  if (p.M == 0) return;
  CUtensorMap ta = operand_tmap(oa, BM), tb = operand_tmap(ob, b_tile_rows(p));
  launch_t<false, true, EPI_SWIGLU_BWD>(ta, tb, p, st);
}

int gemm_ce_tiles_n(int64_t V) { return (int)((V + BN - 1) / BN); }

void launch_gemm_ce(const Mat& x, const Mat& w, const int64_t* targets, float* part_max, float* part_sum,
                    float* tgt_logit, void* logits, int64_t ldl, float alpha, int* status, cudaStream_t st) {
  Operand oa = to_operand(x, false), ob = to_operand(w, false);
  GemmParams p{};
  fill_common(p, oa, ob);
  use_pairs(p);
  p.alpha = alpha;
  p.targets = targets;
  p.part_max = part_max;
  p.part_sum = part_sum;
  p.tgt_logit = tgt_logit;
  p.vec_ok = 1;
  if (logits) {
    p.D = logits;
    p.ldd = ldl;
    p.vec_ok = aligned16(logits, ldl, 2);
  }
  p.status = status;
  if (p.M == 0) return;
  CUtensorMap ta = operand_tmap(oa, BM), tb = operand_tmap(ob, b_tile_rows(p));
  if (logits && gemm_tma_ce() && aligned16(logits, ldl, 2)) {
    // the bf16 logits leave through TMA stores (the row statistics stay per thread)
    const CUtensorMap td = make_tmap_out(logits, p.M, p.N, ldl, false);
    p.tma_out = 1;
    launch_t<false, false, EPI_CE>(ta, tb, p, st, &td);
    return;
  }
  launch_t<false, false, EPI_CE>(ta, tb, p, st);
}

void launch_gemm_rope(const Mat& x, const Mat& w, void* out, int64_t ldo, const float* cos, const float* sin, int seq,
                      int hd, int q_cols, int k_cols, int* status, cudaStream_t st) {
  Operand oa = to_operand(x, false), ob = to_operand(w, false);
  GemmParams p{};
  fill_common(p, oa, ob);
  use_pairs(p);
  OXI_CHECK(hd == 64 || hd == 128, "RoPE epilogue supports head_dim 64 or 128");
  OXI_CHECK(q_cols % hd == 0 && k_cols % hd == 0 && p.N % hd == 0, "RoPE regions must be whole heads");
  OXI_CHECK((reinterpret_cast<uintptr_t>(cos) & 15) == 0 && (reinterpret_cast<uintptr_t>(sin) & 15) == 0,
            "RoPE cos/sin tables must be 16-byte aligned");
  p.D = out;
  p.ldd = ldo;
  p.vec_ok = aligned16(out, ldo, 2);
  p.rope_cos = cos;
  p.rope_sin = sin;
  p.rope_seq = seq;
  p.rope_hd = hd;
  p.rope_q_cols = q_cols;
  p.rope_k_cols = k_cols;
  p.status = status;
  if (p.M == 0) return;
  CUtensorMap ta = operand_tmap(oa, BM), tb = operand_tmap(ob, b_tile_rows(p));
  launch_t<false, false, EPI_ROPE>(ta, tb, p, st);
}

}  // namespace oxi
