// Depthwise causal conv1d with fused bias + SiLU (Mamba short convolution),
// forward and backward, channels-last bf16 activations.
//
//   pre[b,s,c] = bias[c] + sum_{i<K} w[c,i] * x[b, s-K+1+i, c]   (x = 0 for s < 0)
//   y = silu(pre)  (or pre when act == 0)
//
// One thread owns 8 consecutive channels (16-byte vectors) and a segment of
// SEG time steps, sliding a K-tap window through registers, so x is read once
// and y written once.  Backward recomputes pre from x, walks its segment
// backwards keeping the K-1 future values of dpre in registers, and reduces
// dw / dbias per thread before one f32 atomic per (channel, tap).
// Upstream: mamba2.rs:344-352 (candle conv1d with padding K-1, crop, SiLU).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "host_util.h"
#include "kernels_ssm.h"
#include "ptx.cuh"

namespace oxi {
namespace {

constexpr int SEG = 64;
constexpr int MAXK = 8;

__device__ __forceinline__ void ld8f(const __nv_bfloat16* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void st8f(__nv_bfloat16* p, const float* f) {
  *reinterpret_cast<uint4*>(p) =
      make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]), pack_bf16(f[6], f[7]));
}

template <int K>
__global__ void conv1d_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                  const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ y, int B, int S,
                                  int C, int64_t ldx, int64_t ldy, int act) {
  const int cg = C / 8;
  const int nseg = (S + SEG - 1) / SEG;
  const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= (int64_t)B * nseg * cg) return;
  const int c8 = (int)(id % cg);
  const int seg = (int)((id / cg) % nseg);
  const int b = (int)(id / ((int64_t)cg * nseg));
  const int c0 = c8 * 8;
  float wk[K][8], bs[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    bs[j] = bias ? __bfloat162float(bias[c0 + j]) : 0.f;
#pragma unroll
    for (int i = 0; i < K; ++i) wk[i][j] = __bfloat162float(w[(c0 + j) * K + i]);
  }
  float win[K][8];  // win[K-1] is the newest input
  const int s0 = seg * SEG;
#pragma unroll
  for (int i = 0; i < K - 1; ++i) {
    const int s = s0 - (K - 1) + i;
    if (s >= 0) ld8f(x + ((int64_t)b * S + s) * ldx + c0, win[i + 1]);
    else {
#pragma unroll
      for (int j = 0; j < 8; ++j) win[i + 1][j] = 0.f;
    }
  }
  const int s1 = min(S, s0 + SEG);
  for (int s = s0; s < s1; ++s) {
#pragma unroll
    for (int i = 0; i < K - 1; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) win[i][j] = win[i + 1][j];
    ld8f(x + ((int64_t)b * S + s) * ldx + c0, win[K - 1]);
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float a = bs[j];
#pragma unroll
      for (int i = 0; i < K; ++i) a += wk[i][j] * win[i][j];
      o[j] = act ? a / (1.f + __expf(-a)) : a;
    }
    st8f(y + ((int64_t)b * S + s) * ldy + c0, o);
  }
}

template <int K>
__global__ void conv1d_bwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                  const __nv_bfloat16* __restrict__ bias, const __nv_bfloat16* __restrict__ dy,
                                  __nv_bfloat16* __restrict__ dx, float* __restrict__ dw, float* __restrict__ db,
                                  int B, int S, int C, int64_t ldx, int64_t lddy, int64_t lddx, int act) {
  const int cg = C / 8;
  const int nseg = (S + SEG - 1) / SEG;
  const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= (int64_t)B * nseg * cg) return;
  const int c8 = (int)(id % cg);
  const int seg = (int)((id / cg) % nseg);
  const int b = (int)(id / ((int64_t)cg * nseg));
  const int c0 = c8 * 8;
  float wk[K][8], bs[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    bs[j] = bias ? __bfloat162float(bias[c0 + j]) : 0.f;
#pragma unroll
    for (int i = 0; i < K; ++i) wk[i][j] = __bfloat162float(w[(c0 + j) * K + i]);
  }
  const int s0 = seg * SEG;
  const int s1 = min(S, s0 + SEG);
  // dpre at time t (0 outside [0, S))
  auto dpre_at = [&](int t, float* out) {
    if (t < 0 || t >= S) {
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j] = 0.f;
      return;
    }
    float xs[K][8];
#pragma unroll
    for (int i = 0; i < K; ++i) {
      const int tt = t - (K - 1) + i;
      if (tt >= 0) ld8f(x + ((int64_t)b * S + tt) * ldx + c0, xs[i]);
      else {
#pragma unroll
        for (int j = 0; j < 8; ++j) xs[i][j] = 0.f;
      }
    }
    float g[8];
    ld8f(dy + ((int64_t)b * S + t) * lddy + c0, g);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float a = bs[j];
#pragma unroll
      for (int i = 0; i < K; ++i) a += wk[i][j] * xs[i][j];
      if (act) {
        const float sg = 1.f / (1.f + __expf(-a));
        out[j] = g[j] * sg * (1.f + a * (1.f - sg));
      } else {
        out[j] = g[j];
      }
    }
  };
  // fut[i] = dpre at t + 1 + i  (i < K-1)
  float fut[MAXK][8];
#pragma unroll
  for (int i = 0; i < K - 1; ++i) dpre_at(s1 + i, fut[i]);
  float pdw[K][8], pdb[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    pdb[j] = 0.f;
#pragma unroll
    for (int i = 0; i < K; ++i) pdw[i][j] = 0.f;
  }
  for (int t = s1 - 1; t >= s0; --t) {
    float d[8];
    dpre_at(t, d);
    // dx[t] = sum_i w[K-1-i] * dpre[t + i]
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float a = wk[K - 1][j] * d[j];
#pragma unroll
      for (int i = 1; i < K; ++i) a += wk[K - 1 - i][j] * fut[i - 1][j];
      o[j] = a;
    }
    st8f(dx + ((int64_t)b * S + t) * lddx + c0, o);
    // dw[i] += dpre[t] * x[t - K + 1 + i]; db += dpre[t]
#pragma unroll
    for (int i = 0; i < K; ++i) {
      const int tt = t - (K - 1) + i;
      if (tt >= 0) {
        float xv[8];
        ld8f(x + ((int64_t)b * S + tt) * ldx + c0, xv);
#pragma unroll
        for (int j = 0; j < 8; ++j) pdw[i][j] += d[j] * xv[j];
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) pdb[j] += d[j];
#pragma unroll
    for (int i = K - 2; i > 0; --i)
#pragma unroll
      for (int j = 0; j < 8; ++j) fut[i][j] = fut[i - 1][j];
    if (K > 1) {
#pragma unroll
      for (int j = 0; j < 8; ++j) fut[0][j] = d[j];
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (db) atomicAdd(&db[c0 + j], pdb[j]);
#pragma unroll
    for (int i = 0; i < K; ++i) atomicAdd(&dw[(c0 + j) * K + i], pdw[i][j]);
  }
}

}  // namespace

void launch_conv1d_fwd(const void* x, int64_t ldx, const void* w, const void* bias, void* y, int64_t ldy, int B,
                       int S, int C, int K, bool act, cudaStream_t st) {
  OXI_CHECK(C % 8 == 0 && ldx % 8 == 0 && ldy % 8 == 0, "conv1d: channels and strides must be multiples of 8");
  if (!B || !S) return;
  const int64_t threads = (int64_t)B * ((S + SEG - 1) / SEG) * (C / 8);
  const unsigned grid = (unsigned)((threads + 127) / 128);
  auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto Wt = reinterpret_cast<const __nv_bfloat16*>(w);
  auto Bi = reinterpret_cast<const __nv_bfloat16*>(bias);
  auto Y = reinterpret_cast<__nv_bfloat16*>(y);
  switch (K) {
    case 2: conv1d_fwd_kernel<2><<<grid, 128, 0, st>>>(X, Wt, Bi, Y, B, S, C, ldx, ldy, act); break;
    case 3: conv1d_fwd_kernel<3><<<grid, 128, 0, st>>>(X, Wt, Bi, Y, B, S, C, ldx, ldy, act); break;
    case 4: conv1d_fwd_kernel<4><<<grid, 128, 0, st>>>(X, Wt, Bi, Y, B, S, C, ldx, ldy, act); break;
    default: OXI_CHECK(false, "conv1d kernel width must be 2, 3 or 4, got ", K);
  }
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_conv1d_bwd(const void* x, int64_t ldx, const void* w, const void* bias, const void* dy, int64_t lddy,
                       void* dx, int64_t lddx, float* dw, float* db, int B, int S, int C, int K, bool act,
                       cudaStream_t st) {
  OXI_CHECK(C % 8 == 0 && ldx % 8 == 0 && lddy % 8 == 0 && lddx % 8 == 0, "conv1d: alignment");
  if (!B || !S) return;
  const int64_t threads = (int64_t)B * ((S + SEG - 1) / SEG) * (C / 8);
  const unsigned grid = (unsigned)((threads + 127) / 128);
  auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto Wt = reinterpret_cast<const __nv_bfloat16*>(w);
  auto Bi = reinterpret_cast<const __nv_bfloat16*>(bias);
  auto DY = reinterpret_cast<const __nv_bfloat16*>(dy);
  auto DX = reinterpret_cast<__nv_bfloat16*>(dx);
  switch (K) {
    case 2: conv1d_bwd_kernel<2><<<grid, 128, 0, st>>>(X, Wt, Bi, DY, DX, dw, db, B, S, C, ldx, lddy, lddx, act); break;
    case 3: conv1d_bwd_kernel<3><<<grid, 128, 0, st>>>(X, Wt, Bi, DY, DX, dw, db, B, S, C, ldx, lddy, lddx, act); break;
    case 4: conv1d_bwd_kernel<4><<<grid, 128, 0, st>>>(X, Wt, Bi, DY, DX, dw, db, B, S, C, ldx, lddy, lddx, act); break;
    default: OXI_CHECK(false, "conv1d kernel width must be 2, 3 or 4, got ", K);
  }
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
