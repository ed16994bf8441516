// Depthwise causal conv1d with fused bias + SiLU (Mamba short convolution),
// forward and backward, channels-last bf16 activations.
//
//   pre[b,s,c] = bias[c] + sum_{i<K} w[c,i] * x[b, s-K+1+i, c]   (x = 0 for s < 0)
//   y = silu(pre)  (or pre when act == 0)
//
// A warp owns 32 x 4 consecutive channels (8-byte vectors per lane, coalesced rows) and
// each of the block's 8 warps one time segment.  A thread loads its segment's rows (plus
// the K-1 halo) into registers before any arithmetic, so every load of a segment is in
// flight at once.  Backward recomputes pre from x, walks its segment backwards keeping
// the K-1 future values of dpre, and reduces dw / dbias over the block's warps in shared
// memory before one f32 atomic per (channel, tap) per block.
// Upstream: mamba2.rs:344-352 (candle conv1d with padding K-1, crop, SiLU).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "host_util.h"
#include "kernels_ssm.h"
#include "ptx.cuh"

namespace oxi {
namespace {

constexpr int FSEG = 16;  // forward steps per thread
constexpr int BSEG = 8;   // backward steps per thread
constexpr int WARPS = 8;  // segments per block (blockDim = 32 x WARPS)
constexpr int V = 4;      // channels per lane (8-byte vectors; a warp row is 256 contiguous bytes)

__device__ __forceinline__ void unpack4(const uint2& u, float* f) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}
__device__ __forceinline__ uint2 ld_row(const __nv_bfloat16* base, int b, int S, int s, int64_t ld, int c0) {
  if (s < 0 || s >= S) return make_uint2(0u, 0u);
  return __ldg(reinterpret_cast<const uint2*>(base + ((int64_t)b * S + s) * ld + c0));
}
__device__ __forceinline__ void st4f(__nv_bfloat16* p, const float* f) {
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]));
}
__device__ __forceinline__ float sigmoid_fast(float a) { return __fdividef(1.f, 1.f + __expf(-a)); }

// w [C, K] bf16: the lane's V channels are V*K contiguous values at c0*K (8-byte aligned)
template <int K>
__device__ __forceinline__ void load_w(const __nv_bfloat16* w, const __nv_bfloat16* bias, int c0, float (&wk)[K][V],
                                       float (&bs)[V]) {
  float t[V * K];
#pragma unroll
  for (int q = 0; q < K; ++q) unpack4(__ldg(reinterpret_cast<const uint2*>(w + (int64_t)c0 * K) + q), t + 4 * q);
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int i = 0; i < K; ++i) wk[i][j] = t[j * K + i];
  if (bias) {
    unpack4(__ldg(reinterpret_cast<const uint2*>(bias + c0)), bs);
  } else {
#pragma unroll
    for (int j = 0; j < V; ++j) bs[j] = 0.f;
  }
}

template <int K>
__global__ void __launch_bounds__(256) conv1d_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                         const __nv_bfloat16* __restrict__ w,
                                                         const __nv_bfloat16* __restrict__ bias,
                                                         __nv_bfloat16* __restrict__ y, int B, int S, int C,
                                                         int64_t ldx, int64_t ldy, int act) {
  const int cg = C / V;
  const int cv = blockIdx.x * 32 + threadIdx.x;
  const int nseg = (S + FSEG - 1) / FSEG;
  const int64_t bs_id = (int64_t)blockIdx.y * WARPS + threadIdx.y;
  if (cv >= cg || bs_id >= (int64_t)B * nseg) return;
  const int b = (int)(bs_id / nseg), s0 = (int)(bs_id % nseg) * FSEG;
  const int c0 = cv * V;
  constexpr int NX = FSEG + K - 1;
  uint2 xr[NX];  // xr[i] = x row s0 - K + 1 + i
#pragma unroll
  for (int i = 0; i < NX; ++i) xr[i] = ld_row(x, b, S, s0 - (K - 1) + i, ldx, c0);
  float wk[K][V], bs[V];
  load_w<K>(w, bias, c0, wk, bs);
#pragma unroll
  for (int u = 0; u < FSEG; ++u) {
    if (s0 + u >= S) break;
    float o[V];
#pragma unroll
    for (int j = 0; j < V; ++j) o[j] = bs[j];
#pragma unroll
    for (int i = 0; i < K; ++i) {
      float xv[V];
      unpack4(xr[u + i], xv);
#pragma unroll
      for (int j = 0; j < V; ++j) o[j] = fmaf(wk[i][j], xv[j], o[j]);
    }
    if (act) {
#pragma unroll
      for (int j = 0; j < V; ++j) o[j] *= sigmoid_fast(o[j]);
    }
    st4f(y + ((int64_t)b * S + s0 + u) * ldy + c0, o);
  }
}

template <int K>
__global__ void __launch_bounds__(256, 2) conv1d_bwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                            const __nv_bfloat16* __restrict__ w,
                                                            const __nv_bfloat16* __restrict__ bias,
                                                            const __nv_bfloat16* __restrict__ dy,
                                                            __nv_bfloat16* __restrict__ dx, float* __restrict__ dw,
                                                            float* __restrict__ db, int B, int S, int C, int64_t ldx,
                                                            int64_t lddy, int64_t lddx, int act) {
  __shared__ float red[WARPS][K + 1][V][32];
  const int cg = C / V;
  const int lane = threadIdx.x, wy = threadIdx.y;
  const int cv = blockIdx.x * 32 + lane;
  const int nseg = (S + BSEG - 1) / BSEG;
  const int64_t bs_id = (int64_t)blockIdx.y * WARPS + wy;
  const bool live = cv < cg && bs_id < (int64_t)B * nseg;
  float pdw[K][V], pdb[V];
#pragma unroll
  for (int j = 0; j < V; ++j) {
    pdb[j] = 0.f;
#pragma unroll
    for (int i = 0; i < K; ++i) pdw[i][j] = 0.f;
  }
  if (live) {
    const int b = (int)(bs_id / nseg), s0 = (int)(bs_id % nseg) * BSEG;
    const int c0 = cv * V;
    constexpr int ND = BSEG + K - 1;   // dpre at s0 .. s0 + BSEG + K - 2
    constexpr int NX = ND + K - 1;     // x rows s0 - K + 1 .. s0 + BSEG + K - 2
    uint2 xr[NX], gr[ND];
#pragma unroll
    for (int i = 0; i < NX; ++i) xr[i] = ld_row(x, b, S, s0 - (K - 1) + i, ldx, c0);
#pragma unroll
    for (int u = 0; u < ND; ++u) gr[u] = ld_row(dy, b, S, s0 + u, lddy, c0);
    float wk[K][V], bs[V];
    load_w<K>(w, bias, c0, wk, bs);
    float fut[K][V];  // fut[i] = dpre at step u + 1 + i
#pragma unroll
    for (int i = 0; i < K; ++i)
#pragma unroll
      for (int j = 0; j < V; ++j) fut[i][j] = 0.f;
#pragma unroll
    for (int u = ND - 1; u >= 0; --u) {
      // dpre_u = dy * d act(pre) / d pre, pre over x rows u .. u + K - 1 of xr (0 past S: dy = 0)
      float d[V], g[V];
      unpack4(gr[u], g);
      if (act) {
#pragma unroll
        for (int j = 0; j < V; ++j) d[j] = bs[j];
#pragma unroll
        for (int i = 0; i < K; ++i) {
          float xv[V];
          unpack4(xr[u + i], xv);
#pragma unroll
          for (int j = 0; j < V; ++j) d[j] = fmaf(wk[i][j], xv[j], d[j]);
        }
#pragma unroll
        for (int j = 0; j < V; ++j) {
          const float a = d[j];
          const float sg = sigmoid_fast(a);
          d[j] = g[j] * sg * (1.f + a * (1.f - sg));
        }
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j) d[j] = g[j];
      }
      if (u < BSEG && s0 + u < S) {
        // dx[t] = sum_i w[K-1-i] dpre[t+i];  dw[i] += dpre[t] x[t-K+1+i];  db += dpre[t]
        float o[V];
#pragma unroll
        for (int j = 0; j < V; ++j) {
          float a = wk[K - 1][j] * d[j];
#pragma unroll
          for (int i = 1; i < K; ++i) a = fmaf(wk[K - 1 - i][j], fut[i - 1][j], a);
          o[j] = a;
          pdb[j] += d[j];
        }
        st4f(dx + ((int64_t)b * S + s0 + u) * lddx + c0, o);
#pragma unroll
        for (int i = 0; i < K; ++i) {
          float xv[V];
          unpack4(xr[u + i], xv);
#pragma unroll
          for (int j = 0; j < V; ++j) pdw[i][j] = fmaf(d[j], xv[j], pdw[i][j]);
        }
      }
#pragma unroll
      for (int i = K - 1; i > 0; --i)
#pragma unroll
        for (int j = 0; j < V; ++j) fut[i][j] = fut[i - 1][j];
#pragma unroll
      for (int j = 0; j < V; ++j) fut[0][j] = d[j];
    }
  }
#pragma unroll
  for (int j = 0; j < V; ++j) {
    red[wy][K][j][lane] = pdb[j];
#pragma unroll
    for (int i = 0; i < K; ++i) red[wy][i][j][lane] = pdw[i][j];
  }
  __syncthreads();
  const int tid = wy * 32 + lane;
  for (int e = tid; e < (K + 1) * V * 32; e += 32 * WARPS) {
    const int l = e & 31, j = (e >> 5) % V, i = (e >> 5) / V;
    if (blockIdx.x * 32 + l >= cg) continue;
    const int c = (blockIdx.x * 32 + l) * V + j;
    float sum = 0.f;
#pragma unroll
    for (int q = 0; q < WARPS; ++q) sum += red[q][i][j][l];
    if (i == K) {
      if (db) atomicAdd(&db[c], sum);
    } else {
      atomicAdd(&dw[c * K + i], sum);
    }
  }
}

inline bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }

}  // namespace

void launch_conv1d_fwd(const void* x, int64_t ldx, const void* w, const void* bias, void* y, int64_t ldy, int B,
                       int S, int C, int K, bool act, cudaStream_t st) {
  OXI_CHECK(C % 8 == 0 && ldx % 8 == 0 && ldy % 8 == 0 && K >= 2 && K <= 4,
            "conv1d: channels and strides must be multiples of 8, width 2..4");
  if (!B || !S) return;
  OXI_CHECK(aligned8(x) && aligned8(y) && aligned8(w) && aligned8(bias), "conv1d: pointers must be 8-byte aligned");
  const int64_t segs = (int64_t)B * ((S + FSEG - 1) / FSEG);
  OXI_CHECK((segs + WARPS - 1) / WARPS <= 65535, "conv1d: too many rows for one launch");
  const dim3 grid((unsigned)((C / V + 31) / 32), (unsigned)((segs + WARPS - 1) / WARPS)), block(32, WARPS);
  auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto Wt = reinterpret_cast<const __nv_bfloat16*>(w);
  auto Bi = reinterpret_cast<const __nv_bfloat16*>(bias);
  auto Y = reinterpret_cast<__nv_bfloat16*>(y);
  switch (K) {
    case 2: conv1d_fwd_kernel<2><<<grid, block, 0, st>>>(X, Wt, Bi, Y, B, S, C, ldx, ldy, act); break;
    case 3: conv1d_fwd_kernel<3><<<grid, block, 0, st>>>(X, Wt, Bi, Y, B, S, C, ldx, ldy, act); break;
    case 4: conv1d_fwd_kernel<4><<<grid, block, 0, st>>>(X, Wt, Bi, Y, B, S, C, ldx, ldy, act); break;
    default: OXI_CHECK(false, "conv1d kernel width must be 2, 3 or 4, got ", K);
  }
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_conv1d_bwd(const void* x, int64_t ldx, const void* w, const void* bias, const void* dy, int64_t lddy,
                       void* dx, int64_t lddx, float* dw, float* db, int B, int S, int C, int K, bool act,
                       cudaStream_t st) {
  OXI_CHECK(C % 8 == 0 && ldx % 8 == 0 && lddy % 8 == 0 && lddx % 8 == 0, "conv1d: alignment");
  if (!B || !S) return;
  OXI_CHECK(aligned8(x) && aligned8(dy) && aligned8(dx) && aligned8(w) && aligned8(bias),
            "conv1d: pointers must be 8-byte aligned");
  const int64_t segs = (int64_t)B * ((S + BSEG - 1) / BSEG);
  OXI_CHECK((segs + WARPS - 1) / WARPS <= 65535, "conv1d: too many rows for one launch");
  const dim3 grid((unsigned)((C / V + 31) / 32), (unsigned)((segs + WARPS - 1) / WARPS)), block(32, WARPS);
  auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto Wt = reinterpret_cast<const __nv_bfloat16*>(w);
  auto Bi = reinterpret_cast<const __nv_bfloat16*>(bias);
  auto DY = reinterpret_cast<const __nv_bfloat16*>(dy);
  auto DX = reinterpret_cast<__nv_bfloat16*>(dx);
  switch (K) {
    case 2: conv1d_bwd_kernel<2><<<grid, block, 0, st>>>(X, Wt, Bi, DY, DX, dw, db, B, S, C, ldx, lddy, lddx, act); break;
    case 3: conv1d_bwd_kernel<3><<<grid, block, 0, st>>>(X, Wt, Bi, DY, DX, dw, db, B, S, C, ldx, lddy, lddx, act); break;
    case 4: conv1d_bwd_kernel<4><<<grid, block, 0, st>>>(X, Wt, Bi, DY, DX, dw, db, B, S, C, ldx, lddy, lddx, act); break;
    default: OXI_CHECK(false, "conv1d kernel width must be 2, 3 or 4, got ", K);
  }
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
