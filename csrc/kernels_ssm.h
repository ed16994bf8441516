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

namespace oxi {
// Tensor-core chunked SSD (ssd.cu), single-term recurrence
//   H_t = exp(loga_t) H_{t-1} + gamma_t B_t x_t^T,  y_t = H_t^T C_t,
// N = 128, P % 64 == 0, S % 128 == 0.  x: bf16 [B*S, >= H*P] (row stride ldx);
// B/C: bf16 [B*S, >= G*N] (head h uses group h / (H/G)); loga/gamma f32
// [B, S, H].  fwd: y f32 [B*S, H*P], hs bf16 [B*H*(S/128)*N, P] chunk-start
// states.  bwd: dy bf16 [B*S, H*P], dhs bf16 (scratch like hs); dx f32 [B*S,
// H*P]; dB/dC f32 [B*S, H*N] and dgamma f32 [B, S, H] accumulated (zero them).
struct SsdTcIO {
  int B, S, H, P, N, G;
  const void* x;
  int64_t ldx;
  const void* Bm;
  int64_t ldb;
  const void* Cm;
  int64_t ldc;
  const float* loga;
  const float* gamma;
  float* y;
  void* hs;
  const void* dy;
  void* dhs;
  float* dx;
  float* dB;            // f32, or bf16 when dbc_bf16
  float* dC;
  int dbc_bf16;
  float* dgamma;
  float* hloc;          // forward scratch [B*H*nc*N, P] f32
  float* lamend;        // forward scratch [B*H*nc] f32
  void* out;            // optional bf16 [B*S, H*P] = y + d x (fused D skip)
  const float* dskip;   // d: [B*S*H] per token or [H] per head
  int dskip_per_row;
  int* status;
};
bool ssd_tc_supported(int N, int P, int S);
void launch_ssd_fwd(const SsdTcIO& io, cudaStream_t st);
void launch_ssd_bwd(const SsdTcIO& io, cudaStream_t st);
}  // namespace oxi

namespace oxi {
// Mamba3 B/C prologue (mamba3.cu): rmsnorm + bias + complex RoPE, written as
// per-head bf16 B_rot / C_rot [B, S, H, N] plus bcdot f32 [B, S, H] =
// <B_rot, C_rot>.  braw/craw bf16 rows of stride ldr (group g at column g*N);
// ang f32 [B, S, H, N/2].  Backward: db/dc [B, S, H, N] (f32, or bf16 when
// grads_bf16), dbcdot f32 [B, S, H] or null; dbraw/dcraw f32 rows of stride ldd; dw [N], dbb/dcb
// [H, N] accumulated (zero them); dang f32 [B, S, H, N/2].
void launch_m3_bc_fwd(const void* braw, const void* craw, int64_t ldr, const void* w, const void* bbias,
                      const void* cbias, const float* ang, int B, int S, int H, int G, int N, float eps, void* bout,
                      void* cout, float* bcdot, cudaStream_t st);
void launch_m3_bc_bwd(const void* braw, const void* craw, int64_t ldr, const void* w, const void* bbias,
                      const void* cbias, const float* ang, const void* db, const void* dc, bool grads_bf16,
                      const float* dbcdot, int B, int S, int H, int G, int N, float eps, float* dbraw, float* dcraw,
                      int64_t ldd, float* dw, float* dbb, float* dcb, float* dang, cudaStream_t st,
                      float* part = nullptr);
// blocks of the prologue backward = rows of its bias-gradient partials `part` [rows, 2 * H * N]
int m3_bc_bwd_blocks(int64_t tokens);
}  // namespace oxi

namespace oxi {
// Mamba3 angles ang[b,t,h,j] = sum_{u<=t} theta[b,u,h,j] dt[b,u,h] (cumsum.cu);
// sums: f32 scratch [B * ceil(S/128) * H * J].  Backward: dtheta [B,S,H,J],
// ddt [B,S,H] accumulated (zero it).
void launch_angle_cumsum(const float* theta, const float* dt, int B, int S, int H, int J, float* sums, float* ang,
                         cudaStream_t st);
void launch_angle_cumsum_bwd(const float* theta, const float* dt, const float* dang, int B, int S, int H, int J,
                             float* sums, float* dtheta, float* ddt, cudaStream_t st);
// SSD d loga from the identity q_t = e_t + q_{t+1} - v_{t+1}, dla_t = q_t - v_t
// with v = gamma * dgamma: e, ga, dg, dla f32 [B, S, H]; sums scratch
// [B * ceil(S/128) * H].
// D-skip epilogue of the SSD (ssm_glue.cu): out = bf16(y + d x) per row of P;
// backward dx = bf16(dx_scan + d g), dd = <g, x>, e = <g, y> per row.  d per row
// or per head (r % H).
void launch_dskip_fwd(const float* y, const void* x, const float* d, int64_t rows, int H, int P, bool per_row,
                      void* out, cudaStream_t st);
void launch_dskip_bwd(const void* g, const void* x, const float* y, const float* d, const float* dx_scan,
                      int64_t rows, int H, int P, bool per_row, void* dx, float* dd, float* e, cudaStream_t st);
void launch_ssd_dloga(const float* e, const float* ga, const float* dg, int B, int S, int H, float* sums, float* dla,
                      cudaStream_t st);
// Mamba3 per-(token, head) scan coefficients (m3_glue.cu).  dt_raw, lam_raw bf16 [T, H]
// contiguous, bias bf16 [H], A f32 [H]; out f32 [T, H]: dt (softplus + clamp), loga = A dt,
// gamma' = lam dt + c, c (shifted-state coefficient).  Backward takes the gradients of the
// four outputs (any may be null) and writes d dt_raw, d lam_raw (bf16) and adds d dt_bias,
// d A (f32 [H]).
void launch_m3_coef_fwd(const void* dt_raw, const void* bias, const void* lam_raw, const float* A, int64_t T, int S,
                        int H, float lo, float hi, float* dt_out, float* loga, float* gp, float* c_out,
                        cudaStream_t st);
void launch_m3_coef_bwd(const void* dt_raw, const void* bias, const void* lam_raw, const float* A, int64_t T, int S,
                        int H, float lo, float hi, const float* d_dt, const float* d_loga, const float* d_gp,
                        const float* d_c, void* d_dt_raw, void* d_lam_raw, float* d_bias, float* d_A,
                        cudaStream_t st);
}  // namespace oxi
