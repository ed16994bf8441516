// Launchers of the state-space-model kernels (conv1d.cu, ssd.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace oxi {
// x/y: [B*S, C] row-major views (row strides ldx/ldy), w [C, K], bias [C] (nullable).
void launch_conv1d_fwd(const void* x, int64_t ldx, const void* w, const void* bias, void* y, int64_t ldy, int B,
                       int S, int C, int K, bool act, cudaStream_t st);
void launch_conv1d_bwd(const void* x, int64_t ldx, const void* w, const void* bias, const void* dy, int64_t lddy,
                       void* dx, int64_t lddx, float* dw, float* db, int B, int S, int C, int K, bool act,
                       cudaStream_t st);
}  // namespace oxi

namespace oxi {
// Mamba2/3 selective scan I/O (f32).  x/dx/y/dy share element strides xs
// (batch, time, head), B/C/dB/dC share bs (a head stride of 0 shares B/C, and
// sums dB/dC, across heads), per-step scalars share ss.
struct SsmScanIO {
  const float *x, *Bm, *Cm, *loga, *gamma, *beta, *dy;
  float *y, *dx, *dB, *dC, *dgamma, *dbeta;
  int64_t xs[3], bs[3], ss[3];
};
// mode 0: y; 1: dC (recompute); 2: dx, dB, dgamma, dbeta (reverse adjoint).
void launch_ssm_scan(const SsmScanIO& io, int B, int S, int H, int N, int P, bool two, int mode, cudaStream_t st);
void launch_mamba1_fwd(const float* u, const float* delta, const float* A, const float* Bm, const float* Cm, float* y,
                       float* hs, int B, int S, int D, float clamp, cudaStream_t st);
void launch_mamba1_bwd(const float* u, const float* delta, const float* A, const float* Bm, const float* Cm,
                       const float* hs, const float* dy, float* du, float* ddelta, float* dA, float* dB, float* dC,
                       int B, int S, int D, float clamp, cudaStream_t st);
}  // namespace oxi
