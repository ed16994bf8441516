// Row-wise normalisation kernels (bandwidth bound): RMSNorm, LayerNorm and the
// gated RMSNorm of the Mamba2/3 mixers, forward and backward.
//
// Forward: one warp per row, 16-byte vector loads, f32 math.  Backward kernels
// optionally add an incoming residual-stream gradient (dres) into dx, which
// removes the separate autograd add of the pre-norm residual.  Widths that are
// multiples of 256 (up to 4096) take the row kernel: one CTA per row (H/8
// threads, the row in registers), weight / bias gradients written as per-CTA
// partials that a sliced pass sums (no same-address atomics).  Other widths take
// the warp-per-row kernel, which reduces per CTA in shared memory and adds one
// f32 atomic per column per CTA.
// Upstream: RMSNorm model.rs:9-32 (eps 1e-5 at model.rs:796,971); gated RMSNorm
// mamba2.rs:185-217; the Mamba2/3 pre-LayerNorm mamba2.rs:768, mamba3.rs:959.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>

#include "host_util.h"
#include "kernels_ew.h"

namespace oxi {

namespace {

constexpr int NW = 8;  // warps per CTA
constexpr int MAXV = 16;  // max 8-element vectors per lane -> H <= 32*8*16 = 4096

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float* f) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void st8(__nv_bfloat16* p, const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
// 8 consecutive weights (or biases) from column c, a multiple of 8: one 16-byte
// load for bf16, two for f32
__device__ __forceinline__ void ldw8(const void* w, int wf32, int c, float* f) {
  if (wf32) {
    const float4 a = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(w) + c)[0];
    const float4 b = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(w) + c)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    ld8(reinterpret_cast<const __nv_bfloat16*>(w) + c, f);
  }
}
__device__ __forceinline__ float ldw(const void* w, int wf32, int i) {
  return wf32 ? reinterpret_cast<const float*>(w)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w)[i]);
}

// mode 0: RMSNorm, 1: LayerNorm, 2: gated RMSNorm (x * silu(gate) then RMSNorm)
template <int MODE, int VPL>
__global__ void norm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ gate,
                                const void* __restrict__ w, int wf32, const void* __restrict__ b,
                                __nv_bfloat16* __restrict__ y, float* __restrict__ stat_rstd,
                                float* __restrict__ stat_mean, int64_t rows, int H, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * NW + threadIdx.x / 32;
  if (row >= rows) return;
  const int nv = H / 8;
  float v[VPL][8];
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nv) {
      ld8(x + row * H + vi * 8, v[i]);
      if (MODE == 2) {
        float g[8];
        ld8(gate + row * H + vi * 8, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] *= g[j] / (1.f + __expf(-g[j]));
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) { s1 += v[i][j]; s2 += v[i][j] * v[i][j]; }
    }
  }
  s1 = warp_sum(s1);
  s2 = warp_sum(s2);
  float mean = 0.f, rstd;
  if (MODE == 1) {
    mean = s1 / H;
    const float var = fmaxf(s2 / H - mean * mean, 0.f);
    rstd = rsqrtf(var + eps);
  } else {
    rstd = rsqrtf(s2 / H + eps);
  }
  if (lane == 0) {
    stat_rstd[row] = rstd;
    if (MODE == 1) stat_mean[row] = mean;
  }
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nv) {
      float o[8], wv[8], bv[8];
      ldw8(w, wf32, vi * 8, wv);
      if (MODE == 1) ldw8(b, wf32, vi * 8, bv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float t = (v[i][j] - mean) * rstd * wv[j];
        if (MODE == 1) t += bv[j];
        o[j] = t;
      }
      st8(y + row * H + vi * 8, o);
    }
  }
}

template <int MODE, int VPL>
__global__ void norm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                const __nv_bfloat16* __restrict__ gate, const void* __restrict__ w, int wf32,
                                const float* __restrict__ stat_rstd, const float* __restrict__ stat_mean,
                                const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx,
                                __nv_bfloat16* __restrict__ dgate, float* __restrict__ dw, float* __restrict__ db,
                                int64_t rows, int H) {
  extern __shared__ float sm[];  // [2][H] partial dw/db
  float* sdw = sm;
  float* sdb = sm + H;
  for (int c = threadIdx.x; c < 2 * H; c += blockDim.x) sm[c] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x / 32;
  const int nv = H / 8;
  float pdw[VPL][8], pdb[VPL][8];
#pragma unroll
  for (int i = 0; i < VPL; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) { pdw[i][j] = 0.f; pdb[i][j] = 0.f; }

  for (int64_t row = (int64_t)blockIdx.x * NW + warp; row < rows; row += (int64_t)gridDim.x * NW) {
    const float rstd = stat_rstd[row];
    const float mean = MODE == 1 ? stat_mean[row] : 0.f;
    const __nv_bfloat16* xr = x + row * H;
    const __nv_bfloat16* dyr = dy + row * H;
    const __nv_bfloat16* gr = gate + (MODE == 2 ? row * H : 0);
    // pass 1: row reductions and weight-gradient partials
    float a1 = 0.f, a2 = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nv) {
        float xv[8], dv[8];
        ld8(xr + vi * 8, xv);
        ld8(dyr + vi * 8, dv);
        if (MODE == 2) {
          float g[8];
          ld8(gr + vi * 8, g);
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[j] *= g[j] / (1.f + __expf(-g[j]));
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = (xv[j] - mean) * rstd;
          const float wd = dv[j] * ldw(w, wf32, vi * 8 + j);
          pdw[i][j] += dv[j] * xh;
          if (MODE == 1) pdb[i][j] += dv[j];
          a1 += wd;
          a2 += wd * xh;
        }
      }
    }
    a1 = warp_sum(a1) / H;
    a2 = warp_sum(a2) / H;
    // pass 2: input gradient (row is L1-resident)
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nv) {
        float xv[8], dv[8], g[8], o[8];
        ld8(xr + vi * 8, xv);
        ld8(dyr + vi * 8, dv);
        if (MODE == 2) ld8(gr + vi * 8, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float xin = xv[j];
          if (MODE == 2) xin *= g[j] / (1.f + __expf(-g[j]));
          const float xh = (xin - mean) * rstd;
          const float wd = dv[j] * ldw(w, wf32, vi * 8 + j);
          o[j] = (MODE == 1) ? rstd * (wd - a1 - xh * a2) : rstd * (wd - xh * a2);
        }
        if (MODE == 2) {
          // h = y * silu(g): dh -> dy_in = dh * silu(g), dg = dh * y * silu'(g)
          float dg[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float s = 1.f / (1.f + __expf(-g[j]));
            const float dh = o[j];
            o[j] = dh * g[j] * s;
            dg[j] = dh * xv[j] * s * (1.f + g[j] * (1.f - s));
          }
          st8(dgate + row * H + vi * 8, dg);
        }
        if (dres) {
          float r[8];
          ld8(dres + row * H + vi * 8, r);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] += r[j];
        }
        st8(dx + row * H + vi * 8, o);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nv) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        atomicAdd(&sdw[vi * 8 + j], pdw[i][j]);
        if (MODE == 1) atomicAdd(&sdb[vi * 8 + j], pdb[i][j]);
      }
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    atomicAdd(&dw[c], sdw[c]);
    if (MODE == 1) atomicAdd(&db[c], sdb[c]);
  }
}

// Backward with a CTA per row (H / 8 threads, thread t owns columns 8t..8t+7):
// x, dy (and gate) are loaded once and kept in registers across the two
// reductions; the weight-gradient partials stay per thread (the same columns
// for every row of this CTA) and are added with one atomic per column at the end.
template <int MODE>
__global__ void __launch_bounds__(512) norm_bwd_row_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ gate,
    const void* __restrict__ w, int wf32, const float* __restrict__ stat_rstd, const float* __restrict__ stat_mean,
    const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx, __nv_bfloat16* __restrict__ dgate,
    float* __restrict__ dw, float* __restrict__ db, float* __restrict__ part, int64_t rows, int H) {
  __shared__ float red[2][2][16];  // [row parity][a1 | a2][warp]
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5, nw = blockDim.x >> 5;
  const int c0 = t * 8;
  float wv[8], pdw[8], pdb[8];
  ldw8(w, wf32, c0, wv);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    pdw[j] = 0.f;
    pdb[j] = 0.f;
  }
  const float inv_h = 1.f / (float)H;
  int it = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x, ++it) {
    const float rstd = stat_rstd[row];
    const float mean = MODE == 1 ? stat_mean[row] : 0.f;
    float xv[8], dv[8], g[8], xh[8], rv[8];
    ld8(x + row * H + c0, xv);
    ld8(dy + row * H + c0, dv);
    if (MODE == 2) ld8(gate + row * H + c0, g);
    if (dres) ld8(dres + row * H + c0, rv);
    float a1 = 0.f, a2 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float xin = MODE == 2 ? xv[j] * (g[j] / (1.f + __expf(-g[j]))) : xv[j];
      xh[j] = (xin - mean) * rstd;
      const float wd = dv[j] * wv[j];
      pdw[j] += dv[j] * xh[j];
      if (MODE == 1) pdb[j] += dv[j];
      a1 += wd;
      a2 += wd * xh[j];
    }
    a1 = warp_sum(a1);
    a2 = warp_sum(a2);
    float(*rb)[16] = red[it & 1];
    if (lane == 0) {
      rb[0][wid] = a1;
      rb[1][wid] = a2;
    }
    __syncthreads();
    a1 = 0.f;
    a2 = 0.f;
    for (int i = 0; i < nw; ++i) {
      a1 += rb[0][i];
      a2 += rb[1][i];
    }
    a1 *= inv_h;
    a2 *= inv_h;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float wd = dv[j] * wv[j];
      o[j] = (MODE == 1) ? rstd * (wd - a1 - xh[j] * a2) : rstd * (wd - xh[j] * a2);
    }
    if (MODE == 2) {
      float dg[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float sg = 1.f / (1.f + __expf(-g[j]));
        const float dh = o[j];
        o[j] = dh * g[j] * sg;
        dg[j] = dh * xv[j] * sg * (1.f + g[j] * (1.f - sg));
      }
      st8(dgate + row * H + c0, dg);
    }
    if (dres) {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] += rv[j];
    }
    st8(dx + row * H + c0, o);
  }
  if (part) {
    // per-CTA partials [gridDim.x][2H], summed over CTAs by norm_part_sum_kernel
    float* pw = part + (int64_t)blockIdx.x * 2 * H;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      pw[c0 + j] = pdw[j];
      if (MODE == 1) pw[H + c0 + j] = pdb[j];
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    atomicAdd(&dw[c0 + j], pdw[j]);
    if (MODE == 1) atomicAdd(&db[c0 + j], pdb[j]);
  }
}

// dw[c] += sum_g part[g][c] (and db from the second half).  A CTA sums a slice of
// the CTAs' partials for 256 columns and adds it with one atomic per column: a
// few dozen adds per address instead of one per row-CTA.
__global__ void norm_part_sum_kernel(const float* __restrict__ part, int G, int H, float* __restrict__ dw,
                                     float* __restrict__ db) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int width = db ? 2 * H : H;
  if (c >= width) return;
  const int per = (G + gridDim.y - 1) / gridDim.y;
  const int g0 = blockIdx.y * per, g1 = min(G, g0 + per);
  float s = 0.f;
  for (int g = g0; g < g1; ++g) s += part[(int64_t)g * 2 * H + c];
  if (g1 > g0) atomicAdd(c < H ? dw + c : db + (c - H), s);
}

int num_sms_norm() {
  static int sms = 0;
  if (!sms) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return sms;
}

}  // namespace

// CTAs of the row-per-CTA norm backward (rows of its weight-gradient partials)
int norm_bwd_partial_rows(int64_t rows, int H) {
  if (H % 256 != 0 || H > 4096) return 0;
  return (int)std::min<int64_t>(rows, (int64_t)num_sms_norm() * (2048 / (H / 8)));
}

namespace {

int norm_grid(int64_t rows) {
  int64_t need = (rows + NW - 1) / NW;
  return (int)std::min<int64_t>(need, (int64_t)num_sms_norm() * 4);
}

}  // namespace

void launch_norm_fwd(int mode, const void* x, const void* gate, const void* w, bool wf32, const void* b, void* y,
                     float* rstd, float* mean, int64_t rows, int H, float eps, cudaStream_t st) {
  OXI_CHECK(H % 8 == 0 && H <= 32 * 8 * MAXV, "norm: hidden must be a multiple of 8 and <= 4096, got ", H);
  OXI_CHECK((reinterpret_cast<uintptr_t>(w) & 15) == 0 && (reinterpret_cast<uintptr_t>(b) & 15) == 0,
            "norm: weight and bias must be 16-byte aligned (8-element vector loads)");
  if (rows == 0) return;
  dim3 grid((unsigned)((rows + NW - 1) / NW)), block(NW * 32);
  auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto G = reinterpret_cast<const __nv_bfloat16*>(gate);
  auto Y = reinterpret_cast<__nv_bfloat16*>(y);
  const int vpl = (H / 8 + 31) / 32;
#define OXI_NF(M, V) norm_fwd_kernel<M, V><<<grid, block, 0, st>>>(X, G, w, wf32, b, Y, rstd, mean, rows, H, eps)
#define OXI_NF_V(M) \
  if (vpl <= 1) OXI_NF(M, 1); else if (vpl <= 2) OXI_NF(M, 2); else if (vpl <= 4) OXI_NF(M, 4); \
  else if (vpl <= 8) OXI_NF(M, 8); else OXI_NF(M, 16);
  if (mode == 0) { OXI_NF_V(0) } else if (mode == 1) { OXI_NF_V(1) } else { OXI_NF_V(2) }
#undef OXI_NF_V
#undef OXI_NF
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_norm_bwd(int mode, const void* dy, const void* x, const void* gate, const void* w, bool wf32,
                     const float* rstd, const float* mean, const void* dres, void* dx, void* dgate, float* dw,
                     float* db, int64_t rows, int H, cudaStream_t st, float* part, int part_rows) {
  OXI_CHECK(H % 8 == 0 && H <= 32 * 8 * MAXV, "norm: hidden must be a multiple of 8 and <= 4096");
  OXI_CHECK((reinterpret_cast<uintptr_t>(w) & 15) == 0, "norm: weight must be 16-byte aligned (8-element vector loads)");
  if (rows == 0) return;
  if (H % 256 == 0 && H <= 4096) {
    // CTA per row: H / 8 threads; enough CTAs for every SM to hold 2048 threads
    const int threads = H / 8;
    const int grid = norm_bwd_partial_rows(rows, H);
    auto DY_ = reinterpret_cast<const __nv_bfloat16*>(dy);
    auto X_ = reinterpret_cast<const __nv_bfloat16*>(x);
    auto G_ = reinterpret_cast<const __nv_bfloat16*>(gate);
    auto DR_ = reinterpret_cast<const __nv_bfloat16*>(dres);
    auto DX_ = reinterpret_cast<__nv_bfloat16*>(dx);
    auto DG_ = reinterpret_cast<__nv_bfloat16*>(dgate);
    float* pp = part && grid <= part_rows ? part : nullptr;
    if (mode == 0)
      norm_bwd_row_kernel<0><<<grid, threads, 0, st>>>(DY_, X_, G_, w, wf32, rstd, mean, DR_, DX_, DG_, dw, db, pp, rows,
                                                       H);
    else if (mode == 1)
      norm_bwd_row_kernel<1><<<grid, threads, 0, st>>>(DY_, X_, G_, w, wf32, rstd, mean, DR_, DX_, DG_, dw, db, pp, rows,
                                                       H);
    else
      norm_bwd_row_kernel<2><<<grid, threads, 0, st>>>(DY_, X_, G_, w, wf32, rstd, mean, DR_, DX_, DG_, dw, db, pp, rows,
                                                       H);
    OXI_CUDA_CHECK(cudaGetLastError());
    if (pp) {
      const int width = mode == 1 ? 2 * H : H;
      const int slices = std::max(1, std::min(grid / 16, 64));
      norm_part_sum_kernel<<<dim3((width + 255) / 256, slices), 256, 0, st>>>(pp, grid, H, dw,
                                                                              mode == 1 ? db : nullptr);
      OXI_CUDA_CHECK(cudaGetLastError());
    }
    return;
  }
  const int grid = norm_grid(rows);
  const size_t smem = 2 * H * sizeof(float);
  auto DY = reinterpret_cast<const __nv_bfloat16*>(dy);
  auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto G = reinterpret_cast<const __nv_bfloat16*>(gate);
  auto DR = reinterpret_cast<const __nv_bfloat16*>(dres);
  auto DX = reinterpret_cast<__nv_bfloat16*>(dx);
  auto DG = reinterpret_cast<__nv_bfloat16*>(dgate);
  const int vpl = (H / 8 + 31) / 32;
#define OXI_NB(M, V) \
  norm_bwd_kernel<M, V><<<grid, NW * 32, smem, st>>>(DY, X, G, w, wf32, rstd, mean, DR, DX, DG, dw, db, rows, H)
#define OXI_NB_V(M) \
  if (vpl <= 1) OXI_NB(M, 1); else if (vpl <= 2) OXI_NB(M, 2); else if (vpl <= 4) OXI_NB(M, 4); \
  else if (vpl <= 8) OXI_NB(M, 8); else OXI_NB(M, 16);
  if (mode == 0) { OXI_NB_V(0) } else if (mode == 1) { OXI_NB_V(1) } else { OXI_NB_V(2) }
#undef OXI_NB_V
#undef OXI_NB
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
