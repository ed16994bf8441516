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

// (already normalised) n [4] + bias -> rotated [4] for one lane
__device__ __forceinline__ void bias_rot(const float* nrm, const float* bias, float c0, float s0, float c1, float s1,
                                         float* out) {
  float n[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) n[i] = nrm[i] + bias[i];
  out[0] = n[0] * c0 - n[1] * s0;
  out[1] = n[0] * s0 + n[1] * c0;
  out[2] = n[2] * c1 - n[3] * s1;
  out[3] = n[2] * s1 + n[3] * c1;
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

// Heads-per-warp variant for one B/C group (G == 1) and H == 8 * HPW: a block takes tiles of
// 8 tokens; warp w owns heads w, w + 8, ... for the whole kernel, so their bias gradients stay in
// registers (no shared-memory atomics).  Per tile: (A) warp w normalises token w's raw rows into
// shared memory; (B) every warp runs its heads over the 8 tokens and leaves, per token, the sum
// over its heads of the normalised-row gradient in its own shared slot; (C) warp w adds the 8
// slots of token w and runs the RMSNorm backward.
// (four or more heads per warp keep every head's loads in flight at once: one block per SM
// with the whole register file instead of spilling at 128 registers)
template <typename GT, int HPW>
__global__ void __launch_bounds__(256, HPW >= 4 ? 1 : 2) m3_bc_bwd_hw_kernel(
    const __nv_bfloat16* __restrict__ braw, const __nv_bfloat16* __restrict__ craw, int64_t ldr,
    const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ bbias, const __nv_bfloat16* __restrict__ cbias,
    const float* __restrict__ ang, const GT* __restrict__ db2, const GT* __restrict__ dc2,
    const float* __restrict__ dbcdot, int64_t tokens, float eps, float* __restrict__ dbraw, float* __restrict__ dcraw,
    int64_t ldd, float* __restrict__ dw, float* __restrict__ dbb, float* __restrict__ dcb, float* __restrict__ dang,
    float* __restrict__ part) {
  constexpr int TT = 8, H = 8 * HPW;
  extern __shared__ float4 smem4[];
  float4* s_nb = smem4;                 // [TT][32]   normalised x r w rows (4 elements per lane)
  float4* s_nc = s_nb + TT * 32;
  float4* s_gb = s_nc + TT * 32;        // [8 warps][TT][32] per-warp head sums of the gradient
  float4* s_gc = s_gb + 8 * TT * 32;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float wv[4];
  load4(w + lane * 4, wv);
  float accb[HPW][4], accc[HPW][4];
#pragma unroll
  for (int hi = 0; hi < HPW; ++hi)
#pragma unroll
    for (int i = 0; i < 4; ++i) accb[hi][i] = accc[hi][i] = 0.f;
  float dw_acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t t0 = (int64_t)blockIdx.x * TT; t0 < tokens; t0 += (int64_t)gridDim.x * TT) {
    // (A) token t0 + wid
    const int64_t tw = t0 + wid;
    float rb[4] = {0.f, 0.f, 0.f, 0.f}, rc[4] = {0.f, 0.f, 0.f, 0.f}, rib = 0.f, ric = 0.f;
    if (tw < tokens) {
      load4(braw + tw * ldr + lane * 4, rb);
      load4(craw + tw * ldr + lane * 4, rc);
      const float sb = warp_sum(rb[0] * rb[0] + rb[1] * rb[1] + rb[2] * rb[2] + rb[3] * rb[3]);
      const float sc = warp_sum(rc[0] * rc[0] + rc[1] * rc[1] + rc[2] * rc[2] + rc[3] * rc[3]);
      rib = rsqrtf(sb / M3N + eps);
      ric = rsqrtf(sc / M3N + eps);
    }
    s_nb[wid * 32 + lane] = make_float4(rb[0] * rib * wv[0], rb[1] * rib * wv[1], rb[2] * rib * wv[2], rb[3] * rib * wv[3]);
    s_nc[wid * 32 + lane] = make_float4(rc[0] * ric * wv[0], rc[1] * ric * wv[1], rc[2] * ric * wv[2], rc[3] * ric * wv[3]);
    __syncthreads();
    // (B) this warp's heads over the tile's tokens
    const int nt = tokens - t0 < TT ? (int)(tokens - t0) : TT;
    for (int t = 0; t < nt; ++t) {
      const int64_t tok = t0 + t;
      const float4 nb4 = s_nb[t * 32 + lane], nc4 = s_nc[t * 32 + lane];
      float gsb[4] = {0.f, 0.f, 0.f, 0.f}, gsc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int hi = 0; hi < HPW; ++hi) {
        const int64_t it = tok * H + wid + 8 * hi;
        float dB[4], dC[4];
        load_grad4(db2 + it * M3N + lane * 4, dB);
        load_grad4(dc2 + it * M3N + lane * 4, dC);
        const float2 a = *reinterpret_cast<const float2*>(ang + it * (M3N / 2) + lane * 2);
        const float gdot = dbcdot ? dbcdot[it] : 0.f;
        float s0, c0, s1, c1;
        rot_sincos(a.x, &s0, &c0);
        rot_sincos(a.y, &s1, &c1);
        const float nbv[4] = {nb4.x, nb4.y, nb4.z, nb4.w}, ncv[4] = {nc4.x, nc4.y, nc4.z, nc4.w};
        float bb[4], cb[4], ob[4], oc[4];  // per-head biases: L1-resident
        load4(bbias + (wid + 8 * hi) * M3N + lane * 4, bb);
        load4(cbias + (wid + 8 * hi) * M3N + lane * 4, cb);
        bias_rot(nbv, bb, c0, s0, c1, s1, ob);
        bias_rot(ncv, cb, c0, s0, c1, s1, oc);
        if (dbcdot) {
          float rob[4] = {ob[0], ob[1], ob[2], ob[3]}, roc[4] = {oc[0], oc[1], oc[2], oc[3]};
          round4(rob);
          round4(roc);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            dB[i] += gdot * roc[i];
            dC[i] += gdot * rob[i];
          }
        }
        const float da0 = dB[0] * (-ob[1]) + dB[1] * ob[0] + dC[0] * (-oc[1]) + dC[1] * oc[0];
        const float da1 = dB[2] * (-ob[3]) + dB[3] * ob[2] + dC[2] * (-oc[3]) + dC[3] * oc[2];
        *reinterpret_cast<float2*>(dang + it * (M3N / 2) + lane * 2) = make_float2(da0, da1);
        float nb[4], nc[4];
        nb[0] = dB[0] * c0 + dB[1] * s0;  nb[1] = -dB[0] * s0 + dB[1] * c0;
        nb[2] = dB[2] * c1 + dB[3] * s1;  nb[3] = -dB[2] * s1 + dB[3] * c1;
        nc[0] = dC[0] * c0 + dC[1] * s0;  nc[1] = -dC[0] * s0 + dC[1] * c0;
        nc[2] = dC[2] * c1 + dC[3] * s1;  nc[3] = -dC[2] * s1 + dC[3] * c1;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          accb[hi][i] += nb[i];
          accc[hi][i] += nc[i];
          gsb[i] += nb[i];
          gsc[i] += nc[i];
        }
      }
      s_gb[(wid * TT + t) * 32 + lane] = make_float4(gsb[0], gsb[1], gsb[2], gsb[3]);
      s_gc[(wid * TT + t) * 32 + lane] = make_float4(gsc[0], gsc[1], gsc[2], gsc[3]);
    }
    __syncthreads();
    // (C) RMSNorm backward of token t0 + wid: u = w * g
    if (tw < tokens) {
      float gb[4] = {0.f, 0.f, 0.f, 0.f}, gc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 x = s_gb[(q * TT + wid) * 32 + lane], y = s_gc[(q * TT + wid) * 32 + lane];
        gb[0] += x.x; gb[1] += x.y; gb[2] += x.z; gb[3] += x.w;
        gc[0] += y.x; gc[1] += y.y; gc[2] += y.z; gc[3] += y.w;
      }
      float ub[4], uc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ub[i] = wv[i] * gb[i];
        uc[i] = wv[i] * gc[i];
        dw_acc[i] += gb[i] * rb[i] * rib + gc[i] * rc[i] * ric;
      }
      const float pb = warp_sum(ub[0] * rb[0] + ub[1] * rb[1] + ub[2] * rb[2] + ub[3] * rb[3]) / M3N;
      const float pc = warp_sum(uc[0] * rc[0] + uc[1] * rc[1] + uc[2] * rc[2] + uc[3] * rc[3]) / M3N;
      const float rb3 = rib * rib * rib * pb, rc3 = ric * ric * ric * pc;
      *reinterpret_cast<float4*>(dbraw + tw * ldd + lane * 4) =
          make_float4(rib * ub[0] - rb[0] * rb3, rib * ub[1] - rb[1] * rb3, rib * ub[2] - rb[2] * rb3,
                      rib * ub[3] - rb[3] * rb3);
      *reinterpret_cast<float4*>(dcraw + tw * ldd + lane * 4) =
          make_float4(ric * uc[0] - rc[0] * rc3, ric * uc[1] - rc[1] * rc3, ric * uc[2] - rc[2] * rc3,
                      ric * uc[3] - rc[3] * rc3);
    }
    __syncthreads();  // the next tile rewrites s_nb / s_gb
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) atomicAdd(dw + lane * 4 + i, dw_acc[i]);
#pragma unroll
  for (int hi = 0; hi < HPW; ++hi) {
    const int e = (wid + 8 * hi) * M3N + lane * 4;
    if (part) {
      float* pb = part + (int64_t)blockIdx.x * 2 * H * M3N;
      *reinterpret_cast<float4*>(pb + e) = make_float4(accb[hi][0], accb[hi][1], accb[hi][2], accb[hi][3]);
      *reinterpret_cast<float4*>(pb + H * M3N + e) =
          make_float4(accc[hi][0], accc[hi][1], accc[hi][2], accc[hi][3]);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        atomicAdd(dbb + e + i, accb[hi][i]);
        atomicAdd(dcb + e + i, accc[hi][i]);
      }
    }
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

namespace {
// the shared-memory opt-in once per instantiation (outside any CUDA-graph capture: the
// trainer runs eager steps before it captures one)
template <typename GT, int HPW>
void launch_bc_bwd_hw(unsigned grid, cudaStream_t st, const __nv_bfloat16* br, const __nv_bfloat16* cr, int64_t ldr,
                      const __nv_bfloat16* wb, const __nv_bfloat16* bb, const __nv_bfloat16* cb, const float* ang,
                      const GT* db, const GT* dc, const float* dbcdot, int64_t tokens, float eps, float* dbraw,
                      float* dcraw, int64_t ldd, float* dw, float* dbb, float* dcb, float* dang, float* part) {
  constexpr int kSmem = (2 * 8 + 2 * 8 * 8) * 32 * (int)sizeof(float4);  // 72 KB
  auto kern = m3_bc_bwd_hw_kernel<GT, HPW>;
  static bool attr = false;
  if (!attr) {
    OXI_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    attr = true;
  }
  kern<<<grid, 256, kSmem, st>>>(br, cr, ldr, wb, bb, cb, ang, db, dc, dbcdot, tokens, eps, dbraw, dcraw, ldd, dw, dbb,
                                 dcb, dang, part);
}
}  // namespace

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
  const int64_t tokens = (int64_t)B * S;
  if (G == 1 && (H == 8 || H == 16 || H == 32 || H == 64)) {
    const auto* dbh = reinterpret_cast<const __nv_bfloat16*>(db);
    const auto* dch = reinterpret_cast<const __nv_bfloat16*>(dc);
    const auto* dbf = reinterpret_cast<const float*>(db);
    const auto* dcf = reinterpret_cast<const float*>(dc);
#define OXI_M3_HW(hpw)                                                                                            \
  if (grads_bf16)                                                                                                 \
    launch_bc_bwd_hw<__nv_bfloat16, hpw>(grid, st, br, cr, ldr, wb, bb, cb, ang, dbh, dch, dbcdot, tokens, eps, dbraw, \
                                         dcraw, ldd, dw, dbb, dcb, dang, part);                                   \
  else                                                                                                            \
    launch_bc_bwd_hw<float, hpw>(grid, st, br, cr, ldr, wb, bb, cb, ang, dbf, dcf, dbcdot, tokens, eps, dbraw, dcraw, \
                                 ldd, dw, dbb, dcb, dang, part);
    switch (H) {
      case 8: OXI_M3_HW(1) break;
      case 16: OXI_M3_HW(2) break;
      case 32: OXI_M3_HW(4) break;
      default: OXI_M3_HW(8) break;
    }
#undef OXI_M3_HW
  } else if (grads_bf16) {
    auto kern = m3_bc_bwd_kernel<__nv_bfloat16>;
    static bool attr = false;  // once, for the largest block (64 heads)
    if (!attr) {
      OXI_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 64 * M3N * 4));
      attr = true;
    }
    kern<<<grid, 256, smem, st>>>(br, cr, ldr, wb, bb, cb, ang, reinterpret_cast<const __nv_bfloat16*>(db),
                                  reinterpret_cast<const __nv_bfloat16*>(dc), dbcdot, B, S, H, G, eps, dbraw, dcraw,
                                  ldd, dw, dbb, dcb, dang, part);
  } else {
    auto kern = m3_bc_bwd_kernel<float>;
    static bool attr = false;
    if (!attr) {
      OXI_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 64 * M3N * 4));
      attr = true;
    }
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
