// Sequence scans of the Mamba3 / SSD glue.
// Mamba3 rotation angles: ang[b, t, c] = sum_{u <= t} theta[b, u, c] * dt[b, u, c / J]
// (mamba3.rs:490, cumsum over the whole sequence), and its backward
//   R[t] = sum_{u >= t} dang[u];  dtheta[t] = dt[t] R[t];  ddt[t] = sum_j theta[t, j] R[t, j].
// theta / ang: f32 [B, S, C] with C = H * J (J angles per head), dt f32 [B, S, H].
// Two passes over chunks of SEG steps so that B * C * S / SEG threads work in
// parallel: (1) chunk sums, (2) each thread scans its chunk starting from the
// sum of the chunks before it.
#include <cuda_runtime.h>
#include <cstdint>

#include "host_util.h"
#include "kernels_ssm.h"

namespace oxi {
namespace {

constexpr int SEG = 128;

// thread -> (b, chunk, c); consecutive threads take consecutive c (coalesced)
__global__ void ang_chunk_sums(const float* __restrict__ theta, const float* __restrict__ dt, int B, int S, int C,
                               int J, int nseg, bool reverse, float* __restrict__ sums) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)B * nseg * C;
  if (i >= total) return;
  const int c = (int)(i % C);
  const int64_t bs = i / C;
  const int seg = (int)(bs % nseg);
  const int b = (int)(bs / nseg);
  const int H = C / J;
  float acc = 0.f;
  const int t0 = seg * SEG, t1 = min(S, t0 + SEG);
  for (int t = t0; t < t1; ++t) {
    const int64_t row = (int64_t)b * S + t;
    const float v = theta[row * C + c];
    acc += reverse ? v : v * dt[row * H + c / J];
  }
  sums[i] = acc;
}

__global__ void ang_scan_fwd(const float* __restrict__ theta, const float* __restrict__ dt,
                             const float* __restrict__ sums, int B, int S, int C, int J, int nseg,
                             float* __restrict__ ang) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)B * nseg * C;
  if (i >= total) return;
  const int c = (int)(i % C);
  const int64_t bs = i / C;
  const int seg = (int)(bs % nseg);
  const int b = (int)(bs / nseg);
  const int H = C / J;
  float acc = 0.f;
  for (int k = 0; k < seg; ++k) acc += sums[((int64_t)b * nseg + k) * C + c];
  const int t0 = seg * SEG, t1 = min(S, t0 + SEG);
  for (int t = t0; t < t1; ++t) {
    const int64_t row = (int64_t)b * S + t;
    acc += theta[row * C + c] * dt[row * H + c / J];
    ang[row * C + c] = acc;
  }
}

// reverse scan of dang; sums hold the per-chunk sums of dang
__global__ void ang_scan_bwd(const float* __restrict__ theta, const float* __restrict__ dt,
                             const float* __restrict__ dang, const float* __restrict__ sums, int B, int S, int C, int J,
                             int nseg, float* __restrict__ dtheta, float* __restrict__ ddt) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)B * nseg * C;
  const bool live = i < total;
  const int c = live ? (int)(i % C) : 0;
  const int64_t bs = live ? i / C : 0;
  const int seg = (int)(bs % nseg);
  const int b = (int)(bs / nseg);
  const int H = C / J;
  float acc = 0.f;
  if (live)
    for (int k = seg + 1; k < nseg; ++k) acc += sums[((int64_t)b * nseg + k) * C + c];
  const int t0 = seg * SEG, t1 = min(S, t0 + SEG);
  // every lane of a warp walks the same steps (J is a multiple of 32: a warp
  // covers 32 angles of one head), so ddt can be reduced across the warp
  for (int t = t1 - 1; t >= t0; --t) {
    const int64_t row = (int64_t)b * S + t;
    float prod = 0.f;
    if (live) {
      acc += dang[row * C + c];
      const float d = dt[row * H + c / J];
      dtheta[row * C + c] = d * acc;
      prod = theta[row * C + c] * acc;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) prod += __shfl_xor_sync(0xffffffffu, prod, o);
    if (live && (threadIdx.x & 31) == 0) atomicAdd(ddt + row * H + c / J, prod);
  }
}

// w_t = e_t - ga_{t+1} dg_{t+1} (0 past the end); thread -> (b, chunk, h)
__device__ __forceinline__ float dloga_w(const float* e, const float* ga, const float* dg, int64_t row, int t, int S,
                                         int H, int h) {
  float w = e[row * H + h];
  if (t + 1 < S) w -= ga[(row + 1) * H + h] * dg[(row + 1) * H + h];
  return w;
}

__global__ void dloga_chunk_sums(const float* __restrict__ e, const float* __restrict__ ga,
                                 const float* __restrict__ dg, int B, int S, int H, int nseg,
                                 float* __restrict__ sums) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * nseg * H) return;
  const int h = (int)(i % H);
  const int64_t bs = i / H;
  const int seg = (int)(bs % nseg);
  const int b = (int)(bs / nseg);
  float acc = 0.f;
  const int t0 = seg * SEG, t1 = min(S, t0 + SEG);
  for (int t = t0; t < t1; ++t) acc += dloga_w(e, ga, dg, (int64_t)b * S + t, t, S, H, h);
  sums[i] = acc;
}

__global__ void dloga_scan(const float* __restrict__ e, const float* __restrict__ ga, const float* __restrict__ dg,
                           const float* __restrict__ sums, int B, int S, int H, int nseg, float* __restrict__ dla) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * nseg * H) return;
  const int h = (int)(i % H);
  const int64_t bs = i / H;
  const int seg = (int)(bs % nseg);
  const int b = (int)(bs / nseg);
  float acc = 0.f;
  for (int k = seg + 1; k < nseg; ++k) acc += sums[((int64_t)b * nseg + k) * H + h];
  const int t0 = seg * SEG, t1 = min(S, t0 + SEG);
  for (int t = t1 - 1; t >= t0; --t) {
    const int64_t row = (int64_t)b * S + t;
    acc += dloga_w(e, ga, dg, row, t, S, H, h);
    dla[row * H + h] = acc - ga[row * H + h] * dg[row * H + h];
  }
}

}  // namespace

void launch_ssd_dloga(const float* e, const float* ga, const float* dg, int B, int S, int H, float* sums, float* dla,
                      cudaStream_t st) {
  const int nseg = (S + SEG - 1) / SEG;
  const int64_t total = (int64_t)B * nseg * H;
  const unsigned grid = (unsigned)((total + 127) / 128);
  dloga_chunk_sums<<<grid, 128, 0, st>>>(e, ga, dg, B, S, H, nseg, sums);
  dloga_scan<<<grid, 128, 0, st>>>(e, ga, dg, sums, B, S, H, nseg, dla);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_angle_cumsum(const float* theta, const float* dt, int B, int S, int H, int J, float* sums, float* ang,
                         cudaStream_t st) {
  const int C = H * J;
  const int nseg = (S + SEG - 1) / SEG;
  const int64_t total = (int64_t)B * nseg * C;
  const unsigned grid = (unsigned)((total + 255) / 256);
  ang_chunk_sums<<<grid, 256, 0, st>>>(theta, dt, B, S, C, J, nseg, false, sums);
  ang_scan_fwd<<<grid, 256, 0, st>>>(theta, dt, sums, B, S, C, J, nseg, ang);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_angle_cumsum_bwd(const float* theta, const float* dt, const float* dang, int B, int S, int H, int J,
                             float* sums, float* dtheta, float* ddt, cudaStream_t st) {
  OXI_CHECK(J % 32 == 0, "angles per head must be a multiple of 32");
  const int C = H * J;
  const int nseg = (S + SEG - 1) / SEG;
  const int64_t total = (int64_t)B * nseg * C;
  const unsigned grid = (unsigned)((total + 255) / 256);
  ang_chunk_sums<<<grid, 256, 0, st>>>(dang, dt, B, S, C, J, nseg, true, sums);
  ang_scan_bwd<<<grid, 256, 0, st>>>(theta, dt, dang, sums, B, S, C, J, nseg, dtheta, ddt);
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
