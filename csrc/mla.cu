// Multi-head latent attention: assembling the attention operands from the
// projections, forward and backward, in one pass each.
//
// Upstream (model.rs:196-256): q = [W_uq c_q, rope(q_rope)] per head and
// k = [W_uk c_kv, rope(k_rope)] with ONE k_rope row per token shared by all
// heads, rotate-half RoPE (model.rs:68-117) over the d_rope columns.  Here:
//   forward : q [T, nh, hd + dr], k [T, nh, hd + dr] and a packed
//             v [T, nh, hd] from q_c [T, nh*hd], kv [T, 2*nh*hd] (k | v) and
//             the rope block rp [T, dr + nh*dr] (k_rope | q_rope) of the
//             down-projection output; RoPE in f32 from the [S, dr/2] tables,
//             the shared k_rope rotated once per token and stored to every head.
//   backward: dq_c [T, nh*hd], dkv [T, 2*nh*hd] and drp [T, dr + nh*dr]: the
//             inverse rotation of dq_rope, and of the head sum of dk_rope.
// One warp per token, its lanes spread over every head: 16-byte loads / stores
// for the no-RoPE columns, (head, pair) items for the RoPE columns.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>

#include "host_util.h"
#include "ptx.cuh"

namespace oxi {
namespace {

__device__ __forceinline__ float ldf(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// The warp of token t spreads every column block of the token over its lanes:
// the no-RoPE parts as 16-byte vectors (nh * hd / 8 of them per tensor), the RoPE
// parts as (head, pair) items, nh * dr / 2 of them; lane l always owns pair
// index e = l % (dr / 2) when dr / 2 divides 32, so the head sum of dk_rope
// needs one shuffle at the end.
__global__ void __launch_bounds__(256) mla_pack_fwd_kernel(
    const __nv_bfloat16* __restrict__ qc, int64_t ldqc, const __nv_bfloat16* __restrict__ kv, int64_t ldkv,
    const __nv_bfloat16* __restrict__ rp, int64_t ldrp, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, int64_t T, int S, int nh, int hd, int dr, __nv_bfloat16* __restrict__ q,
    __nv_bfloat16* __restrict__ k, __nv_bfloat16* __restrict__ v) {
  const int lane = threadIdx.x & 31;
  const int dq = hd + dr, half = dr / 2, vph = hd / 8, nvec = nh * vph, npair = nh * half;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; t < T;
       t += (int64_t)gridDim.x * (blockDim.x / 32)) {
    const int pos = (int)(t % S);
    const uint4* qsrc = reinterpret_cast<const uint4*>(qc + t * ldqc);
    const uint4* ksrc = reinterpret_cast<const uint4*>(kv + t * ldkv);
    const uint4* vsrc = reinterpret_cast<const uint4*>(kv + t * ldkv + (int64_t)nh * hd);
    uint4* vdst = reinterpret_cast<uint4*>(v + t * (int64_t)nh * hd);
#pragma unroll 4
    for (int i = lane; i < nvec; i += 32) {
      const int h = i / vph, j = i - h * vph;
      const uint4 a = qsrc[i], b = ksrc[i], c = vsrc[i];
      reinterpret_cast<uint4*>(q + (t * nh + h) * dq)[j] = a;
      reinterpret_cast<uint4*>(k + (t * nh + h) * dq)[j] = b;
      vdst[i] = c;
    }
    const __nv_bfloat16* rrow = rp + t * ldrp;
    const float* ct = cos_t + (int64_t)pos * half;
    const float* st = sin_t + (int64_t)pos * half;
    for (int i = lane; i < npair; i += 32) {
      const int h = i / half, e = i - h * half;
      const float c = ct[e], s = st[e];
      const __nv_bfloat16* qr = rrow + dr + h * dr;
      const float x1 = ldf(qr + e), x2 = ldf(qr + e + half);
      const float y1 = ldf(rrow + e), y2 = ldf(rrow + e + half);  // the shared k_rope
      __nv_bfloat16* qo = q + (t * nh + h) * dq + hd;
      __nv_bfloat16* ko = k + (t * nh + h) * dq + hd;
      qo[e] = __float2bfloat16(x1 * c - x2 * s);
      qo[e + half] = __float2bfloat16(x2 * c + x1 * s);
      ko[e] = __float2bfloat16(y1 * c - y2 * s);
      ko[e + half] = __float2bfloat16(y2 * c + y1 * s);
    }
  }
}

__global__ void __launch_bounds__(256) mla_pack_bwd_kernel(
    const __nv_bfloat16* __restrict__ dq, const __nv_bfloat16* __restrict__ dk, const __nv_bfloat16* __restrict__ dv,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, int64_t T, int S, int nh, int hd, int dr,
    __nv_bfloat16* __restrict__ dqc, __nv_bfloat16* __restrict__ dkv, __nv_bfloat16* __restrict__ drp) {
  const int lane = threadIdx.x & 31;
  const int dqw = hd + dr, half = dr / 2, vph = hd / 8, nvec = nh * vph, npair = nh * half;
  const bool lane_pairs = (32 % half) == 0;  // lane l always owns pair e = l % half
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; t < T;
       t += (int64_t)gridDim.x * (blockDim.x / 32)) {
    const int pos = (int)(t % S);
    uint4* qdst = reinterpret_cast<uint4*>(dqc + t * (int64_t)nh * hd);
    uint4* kdst = reinterpret_cast<uint4*>(dkv + t * (int64_t)2 * nh * hd);
    uint4* vdst = reinterpret_cast<uint4*>(dkv + t * (int64_t)2 * nh * hd + (int64_t)nh * hd);
    const uint4* vsrc = reinterpret_cast<const uint4*>(dv + t * (int64_t)nh * hd);
#pragma unroll 4
    for (int i = lane; i < nvec; i += 32) {
      const int h = i / vph, j = i - h * vph;
      const uint4 a = reinterpret_cast<const uint4*>(dq + (t * nh + h) * dqw)[j];
      const uint4 b = reinterpret_cast<const uint4*>(dk + (t * nh + h) * dqw)[j];
      const uint4 c = vsrc[i];
      qdst[i] = a;
      kdst[i] = b;
      vdst[i] = c;
    }
    __nv_bfloat16* rrow = drp + t * (int64_t)(dr + nh * dr);
    const float* ct = cos_t + (int64_t)pos * half;
    const float* st = sin_t + (int64_t)pos * half;
    float ks1 = 0.f, ks2 = 0.f;  // this lane's part of the head sum of dk_rope (pair lane % half)
    for (int i = lane; i < npair; i += 32) {
      const int h = i / half, e = i - h * half;
      const float c = ct[e], s = st[e];
      const __nv_bfloat16* dqi = dq + (t * nh + h) * dqw + hd;
      const __nv_bfloat16* dki = dk + (t * nh + h) * dqw + hd;
      // inverse rotation: dx1 = dy1 c + dy2 s, dx2 = dy2 c - dy1 s
      const float y1 = ldf(dqi + e), y2 = ldf(dqi + e + half);
      rrow[dr + h * dr + e] = __float2bfloat16(y1 * c + y2 * s);
      rrow[dr + h * dr + e + half] = __float2bfloat16(y2 * c - y1 * s);
      if (lane_pairs) {
        ks1 += ldf(dki + e);
        ks2 += ldf(dki + e + half);
      }
    }
    if (lane_pairs) {
      // lanes with the same pair index: l, l + half, l + 2 half, ...
      for (int o = half; o < 32; o <<= 1) {
        ks1 += __shfl_xor_sync(0xffffffffu, ks1, o);
        ks2 += __shfl_xor_sync(0xffffffffu, ks2, o);
      }
      if (lane < half) {
        const float c = ct[lane], s = st[lane];
        rrow[lane] = __float2bfloat16(ks1 * c + ks2 * s);
        rrow[lane + half] = __float2bfloat16(ks2 * c - ks1 * s);
      }
    } else if (lane < half) {
      float a1 = 0.f, a2 = 0.f;
      for (int h = 0; h < nh; ++h) {
        const __nv_bfloat16* dki = dk + (t * nh + h) * dqw + hd;
        a1 += ldf(dki + lane);
        a2 += ldf(dki + lane + half);
      }
      const float c = ct[lane], s = st[lane];
      rrow[lane] = __float2bfloat16(a1 * c + a2 * s);
      rrow[lane + half] = __float2bfloat16(a2 * c - a1 * s);
    }
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

unsigned warp_grid(int64_t items) {
  const int64_t blocks = (items + 7) / 8;  // 8 warps per 256-thread CTA
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sm_count() * 16));
}

void check_dims(int nh, int hd, int dr) {
  OXI_CHECK(nh >= 1 && hd % 8 == 0 && hd > 0 && dr % 2 == 0 && dr > 0 && dr / 2 <= 32 && (hd + dr) % 8 == 0,
            "MLA pack: head dim a multiple of 8, rope dim even and at most 64, got hd=", hd, " dr=", dr);
}

}  // namespace

void launch_mla_pack_fwd(const void* qc, int64_t ldqc, const void* kv, int64_t ldkv, const void* rp, int64_t ldrp,
                         const float* cos_t, const float* sin_t, int64_t T, int S, int nh, int hd, int dr, void* q,
                         void* k, void* v, cudaStream_t st) {
  check_dims(nh, hd, dr);
  OXI_CHECK(ldqc % 8 == 0 && ldkv % 8 == 0, "MLA pack: q_c / kv row strides must be multiples of 8 elements");
  if (!T) return;
  mla_pack_fwd_kernel<<<warp_grid(T), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(qc), ldqc, reinterpret_cast<const __nv_bfloat16*>(kv), ldkv,
      reinterpret_cast<const __nv_bfloat16*>(rp), ldrp, cos_t, sin_t, T, S, nh, hd, dr,
      reinterpret_cast<__nv_bfloat16*>(q), reinterpret_cast<__nv_bfloat16*>(k), reinterpret_cast<__nv_bfloat16*>(v));
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_mla_pack_bwd(const void* dq, const void* dk, const void* dv, const float* cos_t, const float* sin_t,
                         int64_t T, int S, int nh, int hd, int dr, void* dqc, void* dkv, void* drp, cudaStream_t st) {
  check_dims(nh, hd, dr);
  if (!T) return;
  mla_pack_bwd_kernel<<<warp_grid(T), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(dq), reinterpret_cast<const __nv_bfloat16*>(dk),
      reinterpret_cast<const __nv_bfloat16*>(dv), cos_t, sin_t, T, S, nh, hd, dr,
      reinterpret_cast<__nv_bfloat16*>(dqc), reinterpret_cast<__nv_bfloat16*>(dkv),
      reinterpret_cast<__nv_bfloat16*>(drp));
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
