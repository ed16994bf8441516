// Launchers of the MoE kernels (moe.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels.h"

namespace oxi {
// Expert segments of the permuted rows start on multiples of this many rows
// (the padding rows are zero), so a 256-row CTA-pair tile of the grouped
// expert GEMM never straddles two experts.
constexpr int MOE_SEG_ALIGN = 256;

void launch_moe_permute(const void* x, int64_t ldx, const int64_t* topi, int64_t T, int k, int E, int H, int* counts,
                        int* seg_off, int* cursor, int* pos, void* xp, cudaStream_t st);
void launch_moe_zero_pad(const int* seg_off, const int* counts, int E, void* m, int H, cudaStream_t st);
void launch_moe_combine(const void* yp, const int* pos, const float* w, int64_t T, int k, int H, const void* resid,
                        void* y, cudaStream_t st);
void launch_moe_combine_bwd(const void* dy, const void* yp, const int* pos, const float* w, int64_t T, int k, int H,
                            void* dyp, float* dw, cudaStream_t st);
void launch_moe_gather_sum(const void* dxp, const int* pos, int64_t T, int k, int H, void* dx, cudaStream_t st);
// Optional for the bf16 epilogue of group-M: scatter output rows into peers'
// buffers and post a flag when done (see GemmParams::scatter_idx / post_ctr).
struct GroupedScatter {
  const int* idx = nullptr;        // [rows] peer * rows_per_peer + row, or -1
  const uint64_t* ptrs = nullptr;  // [W] destination buffers
  int rows_per_peer = 0;
  int* post_ctr = nullptr;
  const uint64_t* post_pads = nullptr;
  int post_kind = 0, post_rank = 0, post_W = 0, post_seq = 0;
};
void launch_gemm_grouped(int mode, int epi, const Mat& a, bool a_mn, const Mat& b, bool b_mn, int n_groups,
                         const int* seg_off, int64_t group_rows_b, void* out, int64_t ldo, void* out2, int64_t ldo2,
                         const void* aux, int64_t ldaux, int* status, cudaStream_t st,
                         const GroupedScatter* scatter = nullptr);
// Router (router.cu): logits [T, E] (bf16 or f32, row stride ld) -> top-k
// indices / weights [T, k], mean routing probability usage [E] (f32), and
// optional per-expert selection counts [E].
void launch_router_fwd(const void* logits, bool bf16, int64_t ld, int64_t T, int E, int k, int64_t* topi, float* topw,
                       float* usage, int* counts, cudaStream_t st);
void launch_router_bwd(const void* logits, bool bf16, int64_t ld, int64_t T, int E, int k, const int64_t* topi,
                       const float* topw, const float* dtopw, const float* dusage, void* dlogits, int64_t ldd,
                       cudaStream_t st);
}  // namespace oxi
