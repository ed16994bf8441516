// Mamba3 per-(token, head) coefficients of the shifted-state tensor-core scan,
// forward and backward, one pass each (mamba3.rs:412-546: dt = clamp(softplus(dt
// + dt_bias), 1e-3, 0.1), lambda = sigmoid(lambda_proj x); trapezoidal rule with
// alpha = exp(dt A), gamma = lambda dt, beta = (1 - lambda) dt alpha).
//
// The scan runs the single-term recurrence K_t = alpha_t K_{t-1} + gamma'_t u_t
// with gamma'_t = lambda_t dt_t + c_t and c_t = (1 - lambda_{t+1}) dt_{t+1}
// (c = 0 at the last position of a sequence); the D skip carries -c_t <B_t, C_t>.
// Forward, per (token t, head h):
//   dt = clamp(softplus(z), lo, hi), z = dt_raw + dt_bias;  lam = sigmoid(l_raw)
//   loga = A dt;  c = w_{t+1}, w = (1 - lam) dt;  gamma' = lam dt + c
// Backward (d_w_t = d_c_{t-1} + d_gamma'_{t-1}, since c_{t-1} = w_t is both an output and
// part of gamma'_{t-1}):
//   d_lam = (d_gamma' - d_w) dt
//   d_dt  = d_dt_in + d_loga A + d_gamma' lam + d_w (1 - lam)
//   d_z   = d_dt sigmoid(z) where lo <= softplus(z) <= hi, else 0
//   d_dt_raw = d_z, d_l_raw = d_lam lam (1 - lam), d_dt_bias = sum_t d_z, d_A = sum_t d_loga dt
// One thread per (token, head); the per-head sums go through shared memory and
// one atomic per head per CTA.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>

#include "host_util.h"
#include "kernels_ssm.h"
#include "ptx.cuh"

namespace oxi {
namespace {

constexpr int M3C_THREADS = 256;
constexpr int M3C_MAXH = 256;

__device__ __forceinline__ float softplus_f(float z) { return z > 20.f ? z : log1pf(expf(z)); }
__device__ __forceinline__ float sigmoid_f(float z) { return 1.f / (1.f + expf(-z)); }

struct Coef {
  float dt, lam, sp, z;
};

__device__ __forceinline__ Coef coef_at(const __nv_bfloat16* __restrict__ dt_raw,
                                        const __nv_bfloat16* __restrict__ bias,
                                        const __nv_bfloat16* __restrict__ lam_raw, int64_t i, int h, float lo,
                                        float hi) {
  Coef c;
  c.z = __bfloat162float(dt_raw[i]) + __bfloat162float(bias[h]);
  c.sp = softplus_f(c.z);
  c.dt = fminf(fmaxf(c.sp, lo), hi);
  c.lam = sigmoid_f(__bfloat162float(lam_raw[i]));
  return c;
}

__global__ void __launch_bounds__(M3C_THREADS) m3_coef_fwd_kernel(
    const __nv_bfloat16* __restrict__ dt_raw, const __nv_bfloat16* __restrict__ bias,
    const __nv_bfloat16* __restrict__ lam_raw, const float* __restrict__ A, int64_t T, int S, int H, float lo,
    float hi, float* __restrict__ dt_out, float* __restrict__ loga, float* __restrict__ gp, float* __restrict__ c_out) {
  const int64_t n = T * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / H;
    const int h = (int)(i - t * H);
    const Coef k = coef_at(dt_raw, bias, lam_raw, i, h, lo, hi);
    float c = 0.f;
    if ((int)(t % S) < S - 1) {
      const Coef k1 = coef_at(dt_raw, bias, lam_raw, i + H, h, lo, hi);
      c = (1.f - k1.lam) * k1.dt;
    }
    dt_out[i] = k.dt;
    loga[i] = A[h] * k.dt;
    gp[i] = k.lam * k.dt + c;
    c_out[i] = c;
  }
}

__global__ void __launch_bounds__(M3C_THREADS) m3_coef_bwd_kernel(
    const __nv_bfloat16* __restrict__ dt_raw, const __nv_bfloat16* __restrict__ bias,
    const __nv_bfloat16* __restrict__ lam_raw, const float* __restrict__ A, int64_t T, int S, int H, float lo,
    float hi, const float* __restrict__ d_dt, const float* __restrict__ d_loga, const float* __restrict__ d_gp,
    const float* __restrict__ d_c, __nv_bfloat16* __restrict__ d_dt_raw, __nv_bfloat16* __restrict__ d_lam_raw,
    float* __restrict__ d_bias, float* __restrict__ d_A) {
  __shared__ float s_bias[M3C_MAXH], s_A[M3C_MAXH];
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    s_bias[h] = 0.f;
    s_A[h] = 0.f;
  }
  __syncthreads();
  const int64_t n = T * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / H;
    const int h = (int)(i - t * H);
    const Coef k = coef_at(dt_raw, bias, lam_raw, i, h, lo, hi);
    const float gdt = d_dt ? d_dt[i] : 0.f, gla = d_loga ? d_loga[i] : 0.f, ggp = d_gp ? d_gp[i] : 0.f;
    // w_t = (1 - lam_t) dt_t is c_{t-1}, which gamma'_{t-1} also contains
    float gw = 0.f;
    if ((int)(t % S) > 0) gw = (d_c ? d_c[i - H] : 0.f) + (d_gp ? d_gp[i - H] : 0.f);
    const float dlam = (ggp - gw) * k.dt;
    const float ddt = gdt + gla * A[h] + ggp * k.lam + gw * (1.f - k.lam);
    const float dz = (k.sp >= lo && k.sp <= hi) ? ddt * sigmoid_f(k.z) : 0.f;
    d_dt_raw[i] = __float2bfloat16(dz);
    d_lam_raw[i] = __float2bfloat16(dlam * k.lam * (1.f - k.lam));
    atomicAdd(&s_bias[h], dz);
    atomicAdd(&s_A[h], gla * k.dt);
  }
  __syncthreads();
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    atomicAdd(&d_bias[h], s_bias[h]);
    atomicAdd(&d_A[h], s_A[h]);
  }
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int d;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
  }
  return n;
}

unsigned grid_for(int64_t n) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + M3C_THREADS - 1) / M3C_THREADS,
                                                          (int64_t)sm_count() * 8));
}

}  // namespace

void launch_m3_coef_fwd(const void* dt_raw, const void* bias, const void* lam_raw, const float* A, int64_t T, int S,
                        int H, float lo, float hi, float* dt_out, float* loga, float* gp, float* c_out,
                        cudaStream_t st) {
  OXI_CHECK(H >= 1 && H <= M3C_MAXH && S >= 1 && T % S == 0, "Mamba3 coefficients: 1 <= heads <= 256, T = B * S");
  if (!T) return;
  m3_coef_fwd_kernel<<<grid_for(T * H), M3C_THREADS, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(dt_raw), reinterpret_cast<const __nv_bfloat16*>(bias),
      reinterpret_cast<const __nv_bfloat16*>(lam_raw), A, T, S, H, lo, hi, dt_out, loga, gp, c_out);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_m3_coef_bwd(const void* dt_raw, const void* bias, const void* lam_raw, const float* A, int64_t T, int S,
                        int H, float lo, float hi, const float* d_dt, const float* d_loga, const float* d_gp,
                        const float* d_c, void* d_dt_raw, void* d_lam_raw, float* d_bias, float* d_A,
                        cudaStream_t st) {
  OXI_CHECK(H >= 1 && H <= M3C_MAXH && S >= 1 && T % S == 0, "Mamba3 coefficients: 1 <= heads <= 256, T = B * S");
  if (!T) return;
  m3_coef_bwd_kernel<<<grid_for(T * H), M3C_THREADS, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(dt_raw), reinterpret_cast<const __nv_bfloat16*>(bias),
      reinterpret_cast<const __nv_bfloat16*>(lam_raw), A, T, S, H, lo, hi, d_dt, d_loga, d_gp, d_c,
      reinterpret_cast<__nv_bfloat16*>(d_dt_raw), reinterpret_cast<__nv_bfloat16*>(d_lam_raw), d_bias, d_A);
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
