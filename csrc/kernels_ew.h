// Launchers of the memory-bound kernels (norms.cu, train_ew.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace oxi {

// mode: 0 RMSNorm, 1 LayerNorm, 2 gated RMSNorm (rmsnorm(x * silu(gate)))
void launch_norm_fwd(int mode, const void* x, const void* gate, const void* w, bool wf32, const void* b, void* y,
                     float* rstd, float* mean, int64_t rows, int H, float eps, cudaStream_t st);
// part (nullable): f32 scratch [part_rows, 2H] for per-CTA weight-gradient partials
// (part_rows >= norm_bwd_partial_rows(rows, H)); without it the CTAs add with atomics.
void launch_norm_bwd(int mode, const void* dy, const void* x, const void* gate, const void* w, bool wf32,
                     const float* rstd, const float* mean, const void* dres, void* dx, void* dgate, float* dw,
                     float* db, int64_t rows, int H, cudaStream_t st, float* part = nullptr, int part_rows = 0);
int norm_bwd_partial_rows(int64_t rows, int H);

void launch_ce_finish(const float* pmax, const float* psum, int nt, const float* tgt_logit, const int64_t* targets,
                      float* lse, float* loss, int64_t rows, cudaStream_t st);
void launch_ce_bwd(void* logits, int64_t ld, int64_t V, int64_t rows, const float* lse, const int64_t* targets,
                   const float* gscale, float inv_count, cudaStream_t st,
                   int64_t col0 = 0);
void launch_embed_fwd(const int64_t* ids, const void* w, void* out, int64_t rows, int H, cudaStream_t st);
void launch_embed_bwd(const int64_t* ids, const void* dy, float* dw, int64_t rows, int H, cudaStream_t st);
void launch_rope_bwd(void* x, int64_t ld, int64_t rows, int ncols_rot, int hd, const float* cos, const float* sin,
                     int seq, cudaStream_t st);
// out of place: dst[:, :ncols_rot] = rope backward of src, dst[:, ncols_rot:ncols] = src
void launch_rope_bwd_to(const void* src, int64_t lds, void* dst, int64_t ldd, int64_t rows, int ncols_rot, int ncols,
                        int hd, const float* cos, const float* sin, int seq, cudaStream_t st);
void launch_sqsum(const float* g, int64_t n, float* out, cudaStream_t st);
// out[c] += sum over rows of a bf16 [rows, N] matrix with row stride ld (bias gradients)
void launch_colsum_bf16(const void* x, int64_t rows, int N, int64_t ld, float* out, cudaStream_t st);
// step_state (nullable): device [t, 1 - b1^t, 1 - b2^t], advanced by one here.
void launch_clip_coef(const float* sqsum, float max_norm, float pre_scale, float* coef, float* norm_out,
                      cudaStream_t st, float* step_state = nullptr, float b1 = 0.9f, float b2 = 0.999f,
                      const int* skip = nullptr);
// bc_dev (nullable): device [1 - b1^t, 1 - b2^t] used instead of bc1 / bc2.
void launch_adamw(float* p, void* p16, const float* g, float* m, float* v, int64_t n, float lr, float b1, float b2,
                  float eps, float wd, float bc1, float bc2, const float* gscale, cudaStream_t st,
                  const float* bc_dev = nullptr);

// SwiGLU backward from dH [rows, I] and the saved GU [rows, 2I] (gate / up interleaved in
// 128-column blocks) into dGU [rows, 2I] (same layout); all contiguous bf16.
void launch_swiglu_bwd(const void* dh, const void* gu, void* dgu, int64_t rows, int I, cudaStream_t st);
}  // namespace oxi
