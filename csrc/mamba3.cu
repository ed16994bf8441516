// Mamba3 B/C prologue (mamba3.rs:167-211 bc_norm + bias, mamba3.rs:581-612
// complex RoPE), fused: for every token t and head h
//   Bn = rmsnorm(B_raw[group(h)]) * w + b_bias[h]      (over the state dim N)
//   B_rot = rotate(Bn, ang[t, h])   pairs (2j, 2j+1) turned by ang[..., j]
// and the same for C with c_bias.  The angles (a cumulative sum over time of
// theta * dt) come in precomputed.  Outputs: per-head B_rot, C_rot [B, S, H, N]
// bf16 (the operands of the tensor-core scan) and bcdot[t, h] = <B_rot, C_rot>
// of the bf16-rounded vectors, which the two-term scan needs for its diagonal
// correction.  One warp per (token, head); each lane owns 4 consecutive state
// entries (two rotation pairs) for N = 128.
//
// Backward (one warp per token, looping over the heads of each group):
//   dB_rot += dbcdot C_rot, dC_rot += dbcdot B_rot
//   d_rot -> d_n (inverse rotation), d ang = d_re * (-rot_im) + d_im * rot_re
//   d b_bias[h] += d_n ; d w += d_n * raw / rms ; d raw = rmsnorm-backward(sum_h w d_n)
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>

#include "host_util.h"
#include "kernels_ssm.h"
#include "ptx.cuh"

namespace oxi {
namespace {

constexpr int M3N = 128;

// sin / cos of a rotation angle that can be large (a cumulative sum over the
// sequence): Cody-Waite range reduction (Cody & Waite, "Software Manual for the
// Elementary Functions", 1980) by 2*pi split into a short head (few significant
// bits, so k * head is exact for |k| < 2^16) and the tail, then the hardware
// __sincosf on the reduced angle in [-pi, pi], where its absolute error is about
// 1e-6 (far below the bf16 rounding of the outputs).
__device__ __forceinline__ void rot_sincos(float a, float* s, float* c) {
  constexpr float kInv2Pi = 0.15915494309189535f;
  constexpr float kHead = 6.28125f;                   // 2*pi rounded to 8 significant bits
  constexpr float kTail = 1.9353071795864769e-3f;     // 2*pi - kHead
  const float k = rintf(a * kInv2Pi);
  float r = fmaf(-k, kHead, a);
  r = fmaf(-k, kTail, r);
  __sincosf(r, s, c);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load4(const __nv_bfloat16* p, float* v) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void store4(__nv_bfloat16* p, const float* v) {
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]));
}
__device__ __forceinline__ void round4(float* v) {
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(__float2bfloat16(v[i]));
}

// raw [4] -> rotated [4] for one lane; returns nothing, fills out
__device__ __forceinline__ void norm_bias_rot(const float* raw, float rinv, const float* w, const float* bias,
                                              float c0, float s0, float c1, float s1, float* out) {
  float n[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) n[i] = raw[i] * rinv * w[i] + bias[i];
  out[0] = n[0] * c0 - n[1] * s0;
  out[1] = n[0] * s0 + n[1] * c0;
  out[2] = n[2] * c1 - n[3] * s1;
  out[3] = n[2] * s1 + n[3] * c1;
}

// one warp per token: the RMSNorm statistics of the token's raw B / C rows are
// computed once per group, then every head of the group is biased, rotated and
// stored (heads unrolled by four for independent loads and shuffles)
__global__ void __launch_bounds__(256) m3_bc_fwd_kernel(const __nv_bfloat16* __restrict__ braw,
                                                        const __nv_bfloat16* __restrict__ craw, int64_t ldr,
                                                        const __nv_bfloat16* __restrict__ w,
                                                        const __nv_bfloat16* __restrict__ bbias,
                                                        const __nv_bfloat16* __restrict__ cbias,
                                                        const float* __restrict__ ang, int Bsz, int S, int H, int G,
                                                        float eps, __nv_bfloat16* __restrict__ bout,
                                                        __nv_bfloat16* __restrict__ cout,
                                                        float* __restrict__ bcdot) {
  const int lane = threadIdx.x & 31;
  const int64_t tokens = (int64_t)Bsz * S;
  const int hpg = H / G;
  float wv[4];
  load4(w + lane * 4, wv);
  for (int64_t bt = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; bt < tokens;
       bt += (int64_t)gridDim.x * (blockDim.x / 32)) {
    for (int g = 0; g < G; ++g) {
      float rb[4], rc[4];
      load4(braw + bt * ldr + g * M3N + lane * 4, rb);
      load4(craw + bt * ldr + g * M3N + lane * 4, rc);
      const float sb = warp_sum(rb[0] * rb[0] + rb[1] * rb[1] + rb[2] * rb[2] + rb[3] * rb[3]);
      const float sc = warp_sum(rc[0] * rc[0] + rc[1] * rc[1] + rc[2] * rc[2] + rc[3] * rc[3]);
      const float rib = rsqrtf(sb / M3N + eps), ric = rsqrtf(sc / M3N + eps);
#pragma unroll 4
      for (int hh = 0; hh < hpg; ++hh) {
        const int h = g * hpg + hh;
        const int64_t it = bt * H + h;
        float bb[4], cb[4];
        load4(bbias + h * M3N + lane * 4, bb);
        load4(cbias + h * M3N + lane * 4, cb);
        const float2 a = *reinterpret_cast<const float2*>(ang + it * (M3N / 2) + lane * 2);
        float s0, c0, s1, c1;
        rot_sincos(a.x, &s0, &c0);
        rot_sincos(a.y, &s1, &c1);
        float ob[4], oc[4];
        norm_bias_rot(rb, rib, wv, bb, c0, s0, c1, s1, ob);
        norm_bias_rot(rc, ric, wv, cb, c0, s0, c1, s1, oc);
        round4(ob);
        round4(oc);
        store4(bout + it * M3N + lane * 4, ob);
        store4(cout + it * M3N + lane * 4, oc);
        const float d = warp_sum(ob[0] * oc[0] + ob[1] * oc[1] + ob[2] * oc[2] + ob[3] * oc[3]);
        if (lane == 0) bcdot[it] = d;
      }
    }
  }
}

__device__ __forceinline__ void load_grad4(const float* p, float* v) {
  const float4 d = *reinterpret_cast<const float4*>(p);
  v[0] = d.x; v[1] = d.y; v[2] = d.z; v[3] = d.w;
}
__device__ __forceinline__ void load_grad4(const __nv_bfloat16* p, float* v) { load4(p, v); }

// db/dc: gradients of B_rot / C_rot [B, S, H, N] (f32 or bf16); dbcdot [B, S, H] (may be null).
template <typename GT>
__global__ void __launch_bounds__(256) m3_bc_bwd_kernel(const __nv_bfloat16* __restrict__ braw,
                                                        const __nv_bfloat16* __restrict__ craw, int64_t ldr,
                                                        const __nv_bfloat16* __restrict__ w,
                                                        const __nv_bfloat16* __restrict__ bbias,
                                                        const __nv_bfloat16* __restrict__ cbias,
                                                        const float* __restrict__ ang, const GT* __restrict__ db2,
                                                        const GT* __restrict__ dc2,
                                                        const float* __restrict__ dbcdot, int Bsz, int S, int H, int G,
                                                        float eps, float* __restrict__ dbraw, float* __restrict__ dcraw,
                                                        int64_t ldd, float* __restrict__ dw, float* __restrict__ dbb,
                                                        float* __restrict__ dcb, float* __restrict__ dang,
                                                        float* __restrict__ part) {
  extern __shared__ float s_db[];  // [2][H][N] bias-gradient partials of this block
  float* s_dbb = s_db;
  float* s_dcb = s_db + H * M3N;
  for (int i = threadIdx.x; i < 2 * H * M3N; i += blockDim.x) s_db[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int hpg = H / G;
  const int64_t tokens = (int64_t)Bsz * S;
  float wv[4];
  load4(w + lane * 4, wv);
  float dw_acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t bt = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; bt < tokens;
       bt += (int64_t)gridDim.x * (blockDim.x / 32)) {
    for (int g = 0; g < G; ++g) {
      float rb[4], rc[4];
      load4(braw + bt * ldr + g * M3N + lane * 4, rb);
      load4(craw + bt * ldr + g * M3N + lane * 4, rc);
      const float sb = warp_sum(rb[0] * rb[0] + rb[1] * rb[1] + rb[2] * rb[2] + rb[3] * rb[3]);
      const float sc = warp_sum(rc[0] * rc[0] + rc[1] * rc[1] + rc[2] * rc[2] + rc[3] * rc[3]);
      const float rib = rsqrtf(sb / M3N + eps), ric = rsqrtf(sc / M3N + eps);
      float gb[4] = {0.f, 0.f, 0.f, 0.f}, gc[4] = {0.f, 0.f, 0.f, 0.f};  // sum over heads of d_n
#pragma unroll 4
      for (int hh = 0; hh < hpg; ++hh) {
        const int h = g * hpg + hh;
        const int64_t it = bt * H + h;
        float dB[4], dC[4];
        load_grad4(db2 + it * M3N + lane * 4, dB);
        load_grad4(dc2 + it * M3N + lane * 4, dC);
        float bb[4], cb[4];
        load4(bbias + h * M3N + lane * 4, bb);
        load4(cbias + h * M3N + lane * 4, cb);
        const float2 a = *reinterpret_cast<const float2*>(ang + it * (M3N / 2) + lane * 2);
        float s0, c0, s1, c1;
        rot_sincos(a.x, &s0, &c0);
        rot_sincos(a.y, &s1, &c1);
        float ob[4], oc[4];
        norm_bias_rot(rb, rib, wv, bb, c0, s0, c1, s1, ob);
        norm_bias_rot(rc, ric, wv, cb, c0, s0, c1, s1, oc);
        if (dbcdot) {
          float rob[4] = {ob[0], ob[1], ob[2], ob[3]}, roc[4] = {oc[0], oc[1], oc[2], oc[3]};
          round4(rob);
          round4(roc);
          const float g = dbcdot[it];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            dB[i] += g * roc[i];
            dC[i] += g * rob[i];
          }
        }
        // d angle of both pairs (B and C share the angles)
        const float da0 = dB[0] * (-ob[1]) + dB[1] * ob[0] + dC[0] * (-oc[1]) + dC[1] * oc[0];
        const float da1 = dB[2] * (-ob[3]) + dB[3] * ob[2] + dC[2] * (-oc[3]) + dC[3] * oc[2];
        *reinterpret_cast<float2*>(dang + it * (M3N / 2) + lane * 2) = make_float2(da0, da1);
        // inverse rotation -> gradient of the normalised + biased vector
        float nb[4], nc[4];
        nb[0] = dB[0] * c0 + dB[1] * s0;  nb[1] = -dB[0] * s0 + dB[1] * c0;
        nb[2] = dB[2] * c1 + dB[3] * s1;  nb[3] = -dB[2] * s1 + dB[3] * c1;
        nc[0] = dC[0] * c0 + dC[1] * s0;  nc[1] = -dC[0] * s0 + dC[1] * c0;
        nc[2] = dC[2] * c1 + dC[3] * s1;  nc[3] = -dC[2] * s1 + dC[3] * c1;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          // element lane*4+i kept at i*32+lane: the 32 lanes of one add hit 32 banks
          atomicAdd(s_dbb + h * M3N + i * 32 + lane, nb[i]);
          atomicAdd(s_dcb + h * M3N + i * 32 + lane, nc[i]);
          gb[i] += nb[i];
          gc[i] += nc[i];
        }
      }
      // rmsnorm backward of the shared raw rows (x r w): u = w * g
      float ub[4], uc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ub[i] = wv[i] * gb[i];
        uc[i] = wv[i] * gc[i];
        dw_acc[i] += gb[i] * rb[i] * rib + gc[i] * rc[i] * ric;
      }
      const float pb = warp_sum(ub[0] * rb[0] + ub[1] * rb[1] + ub[2] * rb[2] + ub[3] * rb[3]) / M3N;
      const float pc = warp_sum(uc[0] * rc[0] + uc[1] * rc[1] + uc[2] * rc[2] + uc[3] * rc[3]) / M3N;
      float* ob_ = dbraw + bt * ldd + g * M3N + lane * 4;
      float* oc_ = dcraw + bt * ldd + g * M3N + lane * 4;
      *reinterpret_cast<float4*>(ob_) = make_float4(rib * ub[0] - rb[0] * rib * rib * rib * pb,
                                                    rib * ub[1] - rb[1] * rib * rib * rib * pb,
                                                    rib * ub[2] - rb[2] * rib * rib * rib * pb,
                                                    rib * ub[3] - rb[3] * rib * rib * rib * pb);
      *reinterpret_cast<float4*>(oc_) = make_float4(ric * uc[0] - rc[0] * ric * ric * ric * pc,
                                                    ric * uc[1] - rc[1] * ric * ric * ric * pc,
                                                    ric * uc[2] - rc[2] * ric * ric * ric * pc,
                                                    ric * uc[3] - rc[3] * ric * ric * ric * pc);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) atomicAdd(dw + lane * 4 + i, dw_acc[i]);
  __syncthreads();
  // position i*32+lane of a head's slot holds element lane*4+i
  auto slot = [](int e) { return (e / M3N) * M3N + (e % 4) * 32 + (e % M3N) / 4; };
  if (part) {  // block partials, summed by m3_part_sum_kernel (no same-address atomics)
    for (int e = threadIdx.x; e < 2 * H * M3N; e += blockDim.x)
      part[(int64_t)blockIdx.x * 2 * H * M3N + e] = s_db[slot(e)];
    return;
  }
  for (int e = threadIdx.x; e < H * M3N; e += blockDim.x) {
    atomicAdd(dbb + e, s_dbb[slot(e)]);
    atomicAdd(dcb + e, s_dcb[slot(e)]);
  }
}

// out[c] += sum over a slice of the blocks' partials [G][2 * HN] (c < HN -> dbb, else dcb)
__global__ void m3_part_sum_kernel(const float* __restrict__ part, int G, int HN, float* __restrict__ dbb,
                                   float* __restrict__ dcb) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= 2 * HN) return;
  const int per = (G + gridDim.y - 1) / gridDim.y;
  const int g0 = blockIdx.y * per, g1 = min(G, g0 + per);
  float sum = 0.f;
  for (int g = g0; g < g1; ++g) sum += part[(int64_t)g * 2 * HN + c];
  if (g1 > g0) atomicAdd(c < HN ? dbb + c : dcb + (c - HN), sum);
}

unsigned grid_of(int64_t warps_needed) {
  const int64_t blocks = (warps_needed + 7) / 8;
  return (unsigned)(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

}  // namespace

void launch_m3_bc_fwd(const void* braw, const void* craw, int64_t ldr, const void* w, const void* bbias,
                      const void* cbias, const float* ang, int B, int S, int H, int G, int N, float eps, void* bout,
                      void* cout, float* bcdot, cudaStream_t st) {
  OXI_CHECK(N == M3N && H % G == 0 && ldr % 4 == 0, "Mamba3 B/C prologue supports state size 128");
  m3_bc_fwd_kernel<<<grid_of((int64_t)B * S), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(braw), reinterpret_cast<const __nv_bfloat16*>(craw), ldr,
      reinterpret_cast<const __nv_bfloat16*>(w), reinterpret_cast<const __nv_bfloat16*>(bbias),
      reinterpret_cast<const __nv_bfloat16*>(cbias), ang, B, S, H, G, eps, reinterpret_cast<__nv_bfloat16*>(bout),
      reinterpret_cast<__nv_bfloat16*>(cout), bcdot);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_m3_bc_bwd(const void* braw, const void* craw, int64_t ldr, const void* w, const void* bbias,
                      const void* cbias, const float* ang, const void* db, const void* dc, bool grads_bf16,
                      const float* dbcdot, int B, int S, int H, int G, int N, float eps, float* dbraw, float* dcraw,
                      int64_t ldd, float* dw, float* dbb, float* dcb, float* dang, cudaStream_t st,
                      float* part) {
  OXI_CHECK(N == M3N && H % G == 0 && H <= 64, "Mamba3 B/C prologue supports state size 128, <= 64 heads");
  const int64_t blocks = m3_bc_bwd_blocks((int64_t)B * S);
  const int smem = 2 * H * M3N * (int)sizeof(float);
  const auto* br = reinterpret_cast<const __nv_bfloat16*>(braw);
  const auto* cr = reinterpret_cast<const __nv_bfloat16*>(craw);
  const auto* wb = reinterpret_cast<const __nv_bfloat16*>(w);
  const auto* bb = reinterpret_cast<const __nv_bfloat16*>(bbias);
  const auto* cb = reinterpret_cast<const __nv_bfloat16*>(cbias);
  const unsigned grid = (unsigned)std::max<int64_t>(blocks, 1);
  if (grads_bf16) {
    auto kern = m3_bc_bwd_kernel<__nv_bfloat16>;
    if (smem > 48 * 1024) OXI_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<grid, 256, smem, st>>>(br, cr, ldr, wb, bb, cb, ang, reinterpret_cast<const __nv_bfloat16*>(db),
                                  reinterpret_cast<const __nv_bfloat16*>(dc), dbcdot, B, S, H, G, eps, dbraw, dcraw,
                                  ldd, dw, dbb, dcb, dang, part);
  } else {
    auto kern = m3_bc_bwd_kernel<float>;
    if (smem > 48 * 1024) OXI_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<grid, 256, smem, st>>>(br, cr, ldr, wb, bb, cb, ang, reinterpret_cast<const float*>(db),
                                  reinterpret_cast<const float*>(dc), dbcdot, B, S, H, G, eps, dbraw, dcraw, ldd, dw,
                                  dbb, dcb, dang, part);
  }
  OXI_CUDA_CHECK(cudaGetLastError());
  if (part) {
    const int HN = H * M3N;
    const int slices = std::max(1, std::min((int)grid / 16, 64));
    m3_part_sum_kernel<<<dim3((2 * HN + 255) / 256, slices), 256, 0, st>>>(part, (int)grid, HN, dbb, dcb);
    OXI_CUDA_CHECK(cudaGetLastError());
  }
}

int m3_bc_bwd_blocks(int64_t tokens) { return (int)std::max<int64_t>(1, std::min<int64_t>((tokens + 7) / 8, 148 * 4)); }

}  // namespace oxi
