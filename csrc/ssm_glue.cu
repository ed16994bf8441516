// D-skip epilogue of the tensor-core SSD (mamba2.rs:381-400 y + D x, and the
// Mamba3 form whose per-(token, head) coefficient also carries the diagonal
// correction of the shifted two-term scan):
//   out[r, :] = bf16(y[r, :] + d[r] x[r, :])            r = token * H + head
// and its backward for an upstream gradient g = d out:
//   dx[r, :]  = bf16(dx_scan[r, :] + d[r] g[r, :])      (dx_scan from the scan backward)
//   dd[r]     = <g[r, :], x[r, :]>
//   e[r]      = <g[r, :], y[r, :]>                      (feeds the d loga identity)
// d is per row (d_stride_rows = 1) or per head (index r % H).  One warp per row,
// each lane owns P / 32 consecutive elements (P in {64, 128, 256}).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "host_util.h"
#include "kernels_ssm.h"
#include "ptx.cuh"

namespace oxi {
namespace {

template <int V>
__device__ __forceinline__ void ld_bf16(const __nv_bfloat16* p, float* v) {
  if constexpr (V == 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y), c = unpack_bf16(u.z), d = unpack_bf16(u.w);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
  } else if constexpr (V == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  } else {
    const float2 a = unpack_bf16(*reinterpret_cast<const uint32_t*>(p));
    v[0] = a.x; v[1] = a.y;
  }
}

template <int V>
__device__ __forceinline__ void st_bf16(__nv_bfloat16* p, const float* v) {
  if constexpr (V == 8) {
    *reinterpret_cast<uint4*>(p) =
        make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
  } else if constexpr (V == 4) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]));
  } else {
    *reinterpret_cast<uint32_t*>(p) = pack_bf16(v[0], v[1]);
  }
}

template <int V>
__device__ __forceinline__ void ld_f32(const float* p, float* v) {
#pragma unroll
  for (int i = 0; i < V; i += 2) {
    const float2 a = reinterpret_cast<const float2*>(p)[i / 2];
    v[i] = a.x;
    v[i + 1] = a.y;
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int V>
__global__ void __launch_bounds__(256) dskip_fwd_kernel(const float* __restrict__ y, const __nv_bfloat16* __restrict__ x,
                                                        const float* __restrict__ d, int64_t rows, int H, bool per_row,
                                                        __nv_bfloat16* __restrict__ out) {
  constexpr int P = 32 * V;
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * 8 + threadIdx.x / 32; r < rows; r += (int64_t)gridDim.x * 8) {
    const float dv = d[per_row ? r : r % H];
    float a[V], b[V];
    ld_f32<V>(y + r * P + lane * V, a);
    ld_bf16<V>(x + r * P + lane * V, b);
#pragma unroll
    for (int i = 0; i < V; ++i) a[i] += dv * b[i];
    st_bf16<V>(out + r * P + lane * V, a);
  }
}

template <int V>
__global__ void __launch_bounds__(256) dskip_bwd_kernel(const __nv_bfloat16* __restrict__ g,
                                                        const __nv_bfloat16* __restrict__ x,
                                                        const float* __restrict__ y, const float* __restrict__ d,
                                                        const float* __restrict__ dx_scan, int64_t rows, int H,
                                                        bool per_row, __nv_bfloat16* __restrict__ dx,
                                                        float* __restrict__ dd, float* __restrict__ e) {
  constexpr int P = 32 * V;
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * 8 + threadIdx.x / 32; r < rows; r += (int64_t)gridDim.x * 8) {
    const float dv = d[per_row ? r : r % H];
    float gv[V], xv[V], yv[V], sv[V];
    ld_bf16<V>(g + r * P + lane * V, gv);
    ld_bf16<V>(x + r * P + lane * V, xv);
    ld_f32<V>(y + r * P + lane * V, yv);
    ld_f32<V>(dx_scan + r * P + lane * V, sv);
    float sx = 0.f, sy = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      sx += gv[i] * xv[i];
      sy += gv[i] * yv[i];
      sv[i] += dv * gv[i];
    }
    st_bf16<V>(dx + r * P + lane * V, sv);
    sx = warp_sum(sx);
    sy = warp_sum(sy);
    if (lane == 0) {
      dd[r] = sx;
      e[r] = sy;
    }
  }
}

unsigned grid_rows(int64_t rows) {
  const int64_t blocks = (rows + 7) / 8;
  return (unsigned)(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

}  // namespace

void launch_dskip_fwd(const float* y, const void* x, const float* d, int64_t rows, int H, int P, bool per_row,
                      void* out, cudaStream_t st) {
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  auto* ob = reinterpret_cast<__nv_bfloat16*>(out);
  const unsigned grid = grid_rows(rows);
  if (P == 256) dskip_fwd_kernel<8><<<grid, 256, 0, st>>>(y, xb, d, rows, H, per_row, ob);
  else if (P == 128) dskip_fwd_kernel<4><<<grid, 256, 0, st>>>(y, xb, d, rows, H, per_row, ob);
  else if (P == 64) dskip_fwd_kernel<2><<<grid, 256, 0, st>>>(y, xb, d, rows, H, per_row, ob);
  else OXI_CHECK(false, "D-skip epilogue supports head dims 64, 128, 256; got ", P);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_dskip_bwd(const void* g, const void* x, const float* y, const float* d, const float* dx_scan,
                      int64_t rows, int H, int P, bool per_row, void* dx, float* dd, float* e, cudaStream_t st) {
  const auto* gb = reinterpret_cast<const __nv_bfloat16*>(g);
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  auto* dxb = reinterpret_cast<__nv_bfloat16*>(dx);
  const unsigned grid = grid_rows(rows);
  if (P == 256) dskip_bwd_kernel<8><<<grid, 256, 0, st>>>(gb, xb, y, d, dx_scan, rows, H, per_row, dxb, dd, e);
  else if (P == 128) dskip_bwd_kernel<4><<<grid, 256, 0, st>>>(gb, xb, y, d, dx_scan, rows, H, per_row, dxb, dd, e);
  else if (P == 64) dskip_bwd_kernel<2><<<grid, 256, 0, st>>>(gb, xb, y, d, dx_scan, rows, H, per_row, dxb, dd, e);
  else OXI_CHECK(false, "D-skip epilogue supports head dims 64, 128, 256; got ", P);
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
