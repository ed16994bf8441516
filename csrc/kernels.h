// Torch-free launcher API of the sm_100a kernel library.  Every launcher takes
// raw device pointers, sizes, a status word (device int, see ptx.cuh) and the
// stream to launch on.  ops.cpp binds these to PyTorch tensors.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace oxi {

// Row-major 2-D view with unit inner stride: element (r, c) at ptr[r * ld + c].
struct Mat {
  const void* ptr;
  int64_t rows, cols, ld;
};

// ------------------------------------------------------------------- GEMM
// out[M,N] = alpha * A @ B^T (+ bias[N]) (+ resid)  or  (+ beta * out) for f32 output.
// a_mn=false: A stored [M,K]; a_mn=true: A stored [K,M].  Same for B with N.
void launch_gemm(const Mat& a, bool a_mn, const Mat& b, bool b_mn, void* out, int64_t ldo, bool out_f32,
                 const void* resid, int64_t ldr, float beta, float alpha, int* status, cudaStream_t st,
                 const void* bias = nullptr);
// h[M, N/2] = silu(g) * u from x[M,K] @ w[N,K]^T, w rows interleaved [gate128|up128]...;
// gu (nullable) receives the pre-activation [M, N] in the same interleaved order.
void launch_gemm_swiglu(const Mat& x, const Mat& w, void* h, int64_t ldh, void* gu, int64_t ldgu, int* status,
                        cudaStream_t st);
// dgu[M, 2I] from dh = dy[M,H] @ w_down[H,I] and the saved pre-activation gu.
void launch_gemm_swiglu_bwd(const Mat& dy, const Mat& w_down, const void* gu, int64_t ldgu, void* dgu, int64_t lddgu,
                            int* status, cudaStream_t st);
// Cross-entropy partials of logits = x[M,K] @ w[V,K]^T; part_* are [M, ceil(V/256)].
void launch_gemm_ce(const Mat& x, const Mat& w, const int64_t* targets, float* part_max, float* part_sum,
                    float* tgt_logit, void* logits, int64_t ldl, float alpha, int* status, cudaStream_t st);
int gemm_ce_tiles_n(int64_t V);
// qkv[M,N] = x @ w^T with rotate-half RoPE on the first q_cols + k_cols columns.
void launch_gemm_rope(const Mat& x, const Mat& w, void* out, int64_t ldo, const float* cos, const float* sin, int seq,
                      int hd, int q_cols, int k_cols, int* status, cudaStream_t st);

}  // namespace oxi
