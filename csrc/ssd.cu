// Chunked state-space scan (Mamba2 SSD form) on the tensor cores, sm_100a.
//
// Per batch b and head h the recurrence (state H is N x P, N = 128):
//   H_t = exp(a_t) H_{t-1} + g_t B_t x_t^T ,   y_t = H_t^T C_t
// (mamba2.rs:381-482; Mamba3's two-term update runs as this recurrence on a
// shifted state, see ops/ssd_tc.py).  With chunks of
// L = 128 steps and Lam_t = sum_{u<=t} a_u inside a chunk:
//   M[t,s]  = (C_t . B_s) exp(Lam_t - Lam_s) g_s   (s <= t)
//   Y       = M X + diag(exp Lam) C H_prev
//   H_end   = exp(Lam_L) H_prev + B^T diag(w) X,   w_s = exp(Lam_L - Lam_s) g_s
// Every product is a tcgen05.mma (bf16 in, f32 accumulate in TMEM); operands
// come from 128B-swizzled shared memory tiles that TMA loads (x, B, C, dy,
// stored states) or that the math warps write (M, scaled x / dy / C).
// Forward: chunk-parallel in three phases (chunk-local end states, an
// element-wise scan over chunks, then the outputs; see below).
//
// Backward, chunk-parallel like the forward, dH = adjoint of a chunk's end state:
//   dH_prev = exp(Lam_L) dH + C^T diag(exp Lam) dY  (chunk-local part per chunk,
//            then an element-wise reverse scan storing every chunk's dH, bf16)
//   dX = M^T dY + diag(w) B dH ; dg_s += exp(Lam_L - Lam_s) <x_s, (B dH)_s>  (ssd_dx_kernel)
// Backward, pass 2 (one CTA per chunk, all p-blocks): dM = dY X^T, dS = dM o D o g,
//          dC = dS B + diag(exp Lam) dY H_prev^T ,  dB = dS^T C + diag(w) X dH^T
//          dg_s += sum_t dM[t,s] S[t,s] D[t,s]
// (dg collects the two passes' parts with f32 atomics).  d(a_t) follows
// outside from <dy, y> and dg (see ops/ssd_tc.py).
//
// Warps: 0 TMA, 1 MMA + TMEM owner, 2..5 math (thread m <-> TMEM lane m).
// Every TMA load fills this CTA's shared memory only; every wait is bounded.
#include <algorithm>
#include <cudaTypedefs.h>

#include "gemm_kernel.cuh"
#include "kernels_ssm.h"

namespace oxi {
namespace {

constexpr int SL = 128;         // chunk length
constexpr int SN = 128;         // state size
constexpr int SP = 64;          // P columns per CTA
constexpr int T_NN = SL * SN * 2;   // 32 KB: [128 rows][128] bf16 (two 64-col blocks)
constexpr int T_NP = SL * SP * 2;   // 16 KB: [128 rows][64] bf16
constexpr int SSD_THREADS = 192;

__device__ __forceinline__ uint64_t kdesc(uint32_t base, int kk) {  // K-major, 64-col blocks of 16 KB
  return umma_desc_sw128(base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t mdesc(uint32_t base, int kk) {  // MN-major, K rows of 128 B
  return umma_desc_sw128(base + kk * 2048, 16384, 1024);
}

struct SsdParams {
  int B, S, H, P, G;          // G: groups of B/C (head h uses group h / (H / G))
  int nc;                     // chunks per sequence
  const float* loga;          // [B, S, H]
  const float* gamma;         // [B, S, H]
  float* y;                   // [B*S, H*P] f32 (fwd)
  __nv_bfloat16* hs;          // [B*H*nc*N, P] chunk-start states (fwd writes, bwd reads via TMA)
  __nv_bfloat16* dhs;         // [B*H*nc*N, P] chunk-end adjoints (bwd pass 1 writes)
  float* dx;                  // [B*S, H*P] f32
  float* dB;                  // [B*S, H*N] f32 (bf16 when dbc_bf16)
  float* dC;                  // [B*S, H*N] f32 (bf16 when dbc_bf16)
  int dbc_bf16;
  float* dgamma;              // [B, S, H] f32 (atomics)
  float* hloc;                // [B*H*nc*N, P] f32 chunk-local end states (chunk-parallel forward)
  float* lamend;              // [B*H*nc] f32 sum of loga over each chunk
  __nv_bfloat16* out;         // [B*S, H*P] bf16 y + d x (fused D skip; null: none)
  const float* dskip;         // [B*S*H] (per token) or [H] (per head)
  int dskip_per_row;
  int* status;
};

// 128 math threads: inclusive cumsum of a over the chunk (thread m holds a_m).
__device__ __forceinline__ float chunk_cumsum(float a, int m, float* s_part) {
  const int lane = m & 31, q = m >> 5;
  float v = a;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  if (lane == 31) s_part[q] = v;
  asm volatile("bar.sync 1, 128;" ::: "memory");
  float off = 0.f;
  for (int i = 0; i < q; ++i) off += s_part[i];
  asm volatile("bar.sync 1, 128;" ::: "memory");
  return v + off;
}
__device__ __forceinline__ void math_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// row m of a [128][64] bf16 SW128 tile -> 64 floats
__device__ __forceinline__ void load_row64(const uint8_t* tile, int m, float* out) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 u = *reinterpret_cast<const uint4*>(tile + m * 128 + (((c ^ (m & 7)) & 7) << 4));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16(w[i]);
      out[c * 8 + 2 * i] = f.x;
      out[c * 8 + 2 * i + 1] = f.y;
    }
  }
}
__device__ __forceinline__ void store_row64(uint8_t* tile, int m, const float* v) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    sw128_store16(tile, m, c,
                  make_uint4(pack_bf16(v[c * 8], v[c * 8 + 1]), pack_bf16(v[c * 8 + 2], v[c * 8 + 3]),
                             pack_bf16(v[c * 8 + 4], v[c * 8 + 5]), pack_bf16(v[c * 8 + 6], v[c * 8 + 7])));
}
// 64 consecutive outputs at element offset `off` of an f32 (or, when bf16, a
// bf16-typed) buffer
__device__ __forceinline__ void store_row_out(float* base, int64_t off, const float* v, int bf16) {
  if (bf16) {
    uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + off);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      d[q] = make_uint4(pack_bf16(v[q * 8], v[q * 8 + 1]), pack_bf16(v[q * 8 + 2], v[q * 8 + 3]),
                        pack_bf16(v[q * 8 + 4], v[q * 8 + 5]), pack_bf16(v[q * 8 + 6], v[q * 8 + 7]));
  } else {
    float4* d = reinterpret_cast<float4*>(base + off);
#pragma unroll
    for (int k = 0; k < 16; ++k) d[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
  }
}

// row m, columns [32 h, 32 h + 32) of a [128][64] bf16 SW128 tile -> 32 floats
__device__ __forceinline__ void load_row32(const uint8_t* tile, int m, int h, float* out) {
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const int c = h * 4 + cc;
    const uint4 u = *reinterpret_cast<const uint4*>(tile + m * 128 + (((c ^ (m & 7)) & 7) << 4));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16(w[i]);
      out[cc * 8 + 2 * i] = f.x;
      out[cc * 8 + 2 * i + 1] = f.y;
    }
  }
}
// 32 TMEM columns -> 32 floats
__device__ __forceinline__ void tmem_row32(uint32_t addr, float* out) {
  uint32_t r0[32];
  tmem_ld32(addr, r0);
  tc_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) out[i] = __uint_as_float(r0[i]);
}
// SSD kernels with eight math warps: warps w and w + 4 share TMEM lane quarter
// (w & 3) and split the columns.  The 128 threads of the first four run the
// chunk cumsum (named barrier 1), then all 256 meet at named barrier 2.
constexpr int SSD_THREADS8 = 320;
__device__ __forceinline__ void math8_bar() { asm volatile("bar.sync 2, 256;" ::: "memory"); }

// TMEM row (lane base + 64 columns from col0) -> 64 floats
__device__ __forceinline__ void tmem_row64(uint32_t addr, float* out) {
  uint32_t r0[32], r1[32];
  tmem_ld32(addr, r0);
  tmem_ld32(addr + 32, r1);
  tc_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    out[i] = __uint_as_float(r0[i]);
    out[32 + i] = __uint_as_float(r1[i]);
  }
}

// ============================================ chunk-parallel forward
// Phase A (ssd_state_kernel, one CTA per (b, h, chunk)): the chunk's own
// contribution to its end state, Hloc = B^T diag(w) X (w_s = exp(Lam_L - Lam_s) g_s),
// f32, and Lam_L.  Phase B (ssd_state_scan_kernel): H_c = exp(Lam_L,c) H_{c-1} +
// Hloc_c over the chunks of each (b, h), storing every chunk-start state (bf16,
// the backward's copy too).  Phase C (ssd_out_kernel, one CTA per (b, h, chunk)):
// Y = M X + diag(exp Lam) C H_prev, accumulated in one TMEM tile by scaling C's
// rows in shared memory, with the optional D-skip epilogue.  Chunks of a
// sequence run in parallel; only the element-wise phase B walks the chunks.
struct StateSmem {
  static constexpr int OFF_B = 0;
  static constexpr int OFF_X = OFF_B + T_NN;
  static constexpr int OFF_VEC = OFF_X + T_NP;   // lam[128], gam[128], part[8]
  static constexpr int OFF_BAR = OFF_VEC + 2 * 128 * 4 + 64;
  static constexpr int TOTAL = OFF_BAR + 256 + 1024;
};

// REVERSE = false: Hloc = B^T diag(w) X (forward).  REVERSE = true: the chunk's
// own part of the adjoint carried to the previous chunk, C^T diag(exp Lam) dY
// (tmB then maps C and tmX maps dY).
template <bool REVERSE>
__global__ void __launch_bounds__(SSD_THREADS)
    ssd_state_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmB, SsdParams p) {
  using L = StateSmem;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sB = smem + L::OFF_B, *sX = smem + L::OFF_X;
  float* s_lam = reinterpret_cast<float*>(smem + L::OFF_VEC);
  float* s_gam = s_lam + 128;
  float* s_part = s_gam + 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t *ld_b = bars + 0, *ld_x = bars + 1, *w_ready = bars + 2, *x_free = bars + 3, *h_full = bars + 4,
           *h_free = bars + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.x, c = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int g = h / (p.H / p.G);
  const int r = b * p.S + c * SL;
  const int npb = p.P / SP;
  if (threadIdx.x == 0) {
    mbar_init(ld_b, 1);
    mbar_init(ld_x, 1);
    mbar_init(w_ready, 4);
    mbar_init(x_free, 1);
    mbar_init(h_full, 1);
    mbar_init(h_free, 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t TM_H = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(ld_b, T_NN);
      tma_load_2d(sB, &tmB, ld_b, g * SN, r);
      tma_load_2d(sB + 16384, &tmB, ld_b, g * SN + 64, r);
      int issued = 0;
      for (int pb = 0; pb < npb; ++pb) {
        if (pb > 0 && !mbar_wait(x_free, (pb - 1) & 1, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(ld_x, T_NP);
        tma_load_2d(sX, &tmX, ld_x, h * p.P + pb * SP, r);
        ++issued;
      }
      mbar_wait(ld_b, 0, nullptr, p.status);  // no copy in flight at exit
      if (issued > 0) mbar_wait(ld_x, (issued - 1) & 1, nullptr, p.status);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_H = umma_idesc_bf16(128, 64, true, true);
      const uint32_t aB = smem_u32(sB), aX = smem_u32(sX);
      bool ok = mbar_wait(ld_b, 0, abort_flag, p.status);
      for (int pb = 0; pb < npb && ok; ++pb) {
        if (!mbar_wait(w_ready, pb & 1, abort_flag, p.status)) break;
        if (pb > 0 && !mbar_wait(h_free, (pb - 1) & 1, abort_flag, p.status)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) tc_mma_f16(TM_H, mdesc(aB, kk), mdesc(aX, kk), ID_H, kk > 0);
        tc_commit(x_free);
        tc_commit(h_full);
      }
    }
    __syncwarp();
  } else {
    const int m = (warp & 3) * 32 + lane;  // chunk step s (W rows) / state row n (Hloc rows)
    const uint32_t lb = (uint32_t)((warp & 3) * 32) << 16;
    const int64_t si = ((int64_t)b * p.S + c * SL + m) * p.H + h;
    const float lam = chunk_cumsum(p.loga[si], m, s_part);
    s_lam[m] = lam;
    math_bar();
    const float lam_end = s_lam[SL - 1];
    if (m == 0) p.lamend[(int64_t)bh * p.nc + c] = lam_end;
    const float w = REVERSE ? __expf(lam) : __expf(lam_end - lam) * p.gamma[si];
    for (int pb = 0; pb < npb; ++pb) {
      if (!mbar_wait(ld_x, pb & 1, abort_flag, p.status)) break;
      float xv[64];
      load_row64(sX, m, xv);
#pragma unroll
      for (int i = 0; i < 64; ++i) xv[i] *= w;
      store_row64(sX, m, xv);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(w_ready);
      if (!mbar_wait(h_full, pb & 1, abort_flag, p.status)) break;
      tc_fence_after();
      float hv[64];
      tmem_row64(TM_H + lb, hv);
      float* dst = p.hloc + (((int64_t)bh * p.nc + c) * SN + m) * p.P + pb * SP;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        reinterpret_cast<float4*>(dst)[i] = make_float4(hv[4 * i], hv[4 * i + 1], hv[4 * i + 2], hv[4 * i + 3]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(h_free);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(TM_H, 64);
  }
}

// Forward: out[bh, c] = state at the start of chunk c, over c = 0, 1, ...
// Reverse: out[bh, c] = adjoint of chunk c's end state, over c = nc-1, nc-2, ...
// Both: H <- exp(Lam_L,c) H + loc[c] after storing out[c] (bf16).
template <bool REVERSE>
__global__ void __launch_bounds__(256) ssd_state_scan_kernel(const float* __restrict__ loc,
                                                             const float* __restrict__ lamend_all,
                                                             __nv_bfloat16* __restrict__ out, int nc, int P) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // n * P + p within one state
  const int64_t per = (int64_t)SN * P;
  if (e >= per) return;
  const int bh = blockIdx.y;
  float hcur = 0.f;
  const float* lamend = lamend_all + (int64_t)bh * nc;
#pragma unroll 4
  for (int i = 0; i < nc; ++i) {
    const int c = REVERSE ? nc - 1 - i : i;
    const int64_t idx = ((int64_t)bh * nc + c) * per + e;
    const float l = loc[idx];
    out[idx] = __float2bfloat16(hcur);
    hcur = __expf(__ldg(lamend + c)) * hcur + l;
  }
}

struct OutSmem {
  static constexpr int OFF_C = 0;
  static constexpr int OFF_B = OFF_C + T_NN;  // B, then M (bf16, K-major over s)
  static constexpr int OFF_X = OFF_B + T_NN;
  static constexpr int OFF_H = OFF_X + T_NP;
  static constexpr int OFF_VEC = OFF_H + T_NP;  // lam[128], gam[128], part[8]
  static constexpr int OFF_BAR = OFF_VEC + 2 * 128 * 4 + 64;
  static constexpr int TOTAL = OFF_BAR + 256 + 1024;
};

__global__ void __launch_bounds__(SSD_THREADS8, 2)
    ssd_out_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmH, SsdParams p) {
  using L = OutSmem;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sC = smem + L::OFF_C, *sB = smem + L::OFF_B, *sX = smem + L::OFF_X, *sH = smem + L::OFF_H;
  float* s_lam = reinterpret_cast<float*>(smem + L::OFF_VEC);
  float* s_gam = s_lam + 128;
  float* s_part = s_gam + 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t *ld_cb = bars + 0, *s_full = bars + 1, *m_ready = bars + 2, *ld_xh = bars + 3, *y_full = bars + 4,
           *y_free = bars + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.x, c = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int g = h / (p.H / p.G);
  const int r = b * p.S + c * SL;
  const int npb = p.P / SP;
  const int hrow = (bh * p.nc + c) * SN;
  if (threadIdx.x == 0) {
    mbar_init(ld_cb, 1);
    mbar_init(s_full, 1);
    mbar_init(m_ready, 8);
    mbar_init(ld_xh, 1);
    mbar_init(y_full, 1);
    mbar_init(y_free, 8);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t TM_S = tmem, TM_Y = tmem + 128;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(ld_cb, 2 * T_NN);
      tma_load_2d(sC, &tmC, ld_cb, g * SN, r);
      tma_load_2d(sC + 16384, &tmC, ld_cb, g * SN + 64, r);
      tma_load_2d(sB, &tmB, ld_cb, g * SN, r);
      tma_load_2d(sB + 16384, &tmB, ld_cb, g * SN + 64, r);
      int issued = 0;
      for (int pb = 0; pb < npb; ++pb) {
        // the previous p-block's X (D skip) and TMEM tile are done with
        if (pb > 0 && !mbar_wait(y_free, (pb - 1) & 1, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(ld_xh, 2 * T_NP);
        tma_load_2d(sX, &tmX, ld_xh, h * p.P + pb * SP, r);
        tma_load_2d(sH, &tmH, ld_xh, pb * SP, hrow);
        ++issued;
      }
      mbar_wait(ld_cb, 0, nullptr, p.status);  // no copy in flight at exit
      if (issued > 0) mbar_wait(ld_xh, (issued - 1) & 1, nullptr, p.status);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = umma_idesc_bf16(128, 128, false, false);
      constexpr uint32_t ID_Y = umma_idesc_bf16(128, 64, false, true);
      const uint32_t aC = smem_u32(sC), aM = smem_u32(sB), aX = smem_u32(sX), aH = smem_u32(sH);
      bool ok = mbar_wait(ld_cb, 0, abort_flag, p.status);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) tc_mma_f16(TM_S, kdesc(aC, kk), kdesc(aM, kk), ID_S, kk != 0);
        tc_commit(s_full);
        ok = mbar_wait(m_ready, 0, abort_flag, p.status);
      }
      for (int pb = 0; pb < npb && ok; ++pb) {
        if (!mbar_wait(ld_xh, pb & 1, abort_flag, p.status)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) tc_mma_f16(TM_Y, kdesc(aM, kk), mdesc(aX, kk), ID_Y, kk != 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) tc_mma_f16(TM_Y, kdesc(aC, kk), mdesc(aH, kk), ID_Y, 1);
        tc_commit(y_full);
      }
    }
    __syncwarp();
  } else {
    const int m = (warp & 3) * 32 + lane;  // chunk step t
    const int colhalf = (warp - 2) >> 2;
    const uint32_t lb = (uint32_t)((warp & 3) * 32) << 16;
    const int64_t si = ((int64_t)b * p.S + c * SL + m) * p.H + h;
    if (colhalf == 0) {
      s_lam[m] = chunk_cumsum(p.loga[si], m, s_part);
      s_gam[m] = p.gamma[si];
    }
    math8_bar();
    const float lam = s_lam[m];
    const float dsk = p.out ? p.dskip[p.dskip_per_row ? si : h] : 0.f;
    bool ok = mbar_wait(s_full, 0, abort_flag, p.status);
    if (ok) {
      tc_fence_after();
      // M = (C B^T) o decay o g -> over B's tile (B was only needed for S)
#pragma unroll 1
      for (int q = 2 * colhalf; q < 2 * colhalf + 2; ++q) {
        uint32_t sr[32];
        tmem_ld32(TM_S + lb + q * 32, sr);
        tc_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          float v[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int s2 = q * 32 + t + e;
            v[e] = (s2 <= m) ? __uint_as_float(sr[t + e]) * __expf(lam - s_lam[s2]) * s_gam[s2] : 0.f;
          }
          pk[t / 2] = pack_bf16(v[0], v[1]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int ch = q * 4 + j;
          sw128_store16(sB + (ch >> 3) * 16384, m, ch & 7,
                        make_uint4(pk[j * 4], pk[j * 4 + 1], pk[j * 4 + 2], pk[j * 4 + 3]));
        }
      }
      // C row t scaled by exp(Lam_t): the inter-chunk term joins the same accumulator
      const float el = __expf(lam);
      {
        const int half = colhalf;
        float cv[64];
        load_row64(sC + half * 16384, m, cv);
#pragma unroll
        for (int i = 0; i < 64; ++i) cv[i] *= el;
        store_row64(sC + half * 16384, m, cv);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(m_ready);
    }
    for (int pb = 0; pb < npb && ok; ++pb) {
      if (!mbar_wait(y_full, pb & 1, abort_flag, p.status)) break;
      tc_fence_after();
      float yv[32];
      tmem_row32(TM_Y + lb + colhalf * 32, yv);
      const int64_t orow = (int64_t)(r + m) * ((int64_t)p.H * p.P) + h * p.P + pb * SP + colhalf * 32;
      float* yr = p.y + orow;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        reinterpret_cast<float4*>(yr)[i] = make_float4(yv[4 * i], yv[4 * i + 1], yv[4 * i + 2], yv[4 * i + 3]);
      if (p.out) {
        float xv[32];
        load_row32(sX, m, colhalf, xv);
#pragma unroll
        for (int i = 0; i < 32; ++i) yv[i] += dsk * xv[i];
        uint4* orp = reinterpret_cast<uint4*>(p.out + orow);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          orp[q] = make_uint4(pack_bf16(yv[q * 8], yv[q * 8 + 1]), pack_bf16(yv[q * 8 + 2], yv[q * 8 + 3]),
                              pack_bf16(yv[q * 8 + 4], yv[q * 8 + 5]), pack_bf16(yv[q * 8 + 6], yv[q * 8 + 7]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(y_free);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ============================================ chunk-parallel dx
// One CTA per (b, h, chunk), all p-blocks: dX = M^T dY + diag(w) B dH (dH = the
// chunk-end adjoint from the reverse scan) and dg_s += exp(Lam_L - Lam_s) <x_s, (B dH)_s>.
// M is written over C's tile once S = C B^T has been read; x rows come from global.
struct DxSmem {
  static constexpr int OFF_C = 0;  // C, then M
  static constexpr int OFF_B = OFF_C + T_NN;
  static constexpr int OFF_DY = OFF_B + T_NN;
  static constexpr int OFF_DH = OFF_DY + T_NP;
  static constexpr int OFF_VEC = OFF_DH + T_NP;  // lam[128], gam[128], part[8]
  static constexpr int OFF_BAR = OFF_VEC + 2 * 128 * 4 + 64;
  static constexpr int TOTAL = OFF_BAR + 256 + 1024;
};

__global__ void __launch_bounds__(SSD_THREADS8, 2)
    ssd_dx_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmC,
                  const __grid_constant__ CUtensorMap tmDY, const __grid_constant__ CUtensorMap tmDH,
                  const __nv_bfloat16* __restrict__ x, int64_t ldx, SsdParams p) {
  using L = DxSmem;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sC = smem + L::OFF_C, *sB = smem + L::OFF_B, *sDY = smem + L::OFF_DY, *sDH = smem + L::OFF_DH;
  float* s_lam = reinterpret_cast<float*>(smem + L::OFF_VEC);
  float* s_gam = s_lam + 128;
  float* s_part = s_gam + 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t *ld_cb = bars + 0, *s_full = bars + 1, *m_ready = bars + 2, *ld_t = bars + 3, *d_full = bars + 4,
           *d_free = bars + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.x, c = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int g = h / (p.H / p.G);
  const int r = b * p.S + c * SL;
  const int npb = p.P / SP;
  const int hrow = (bh * p.nc + c) * SN;
  if (threadIdx.x == 0) {
    mbar_init(ld_cb, 1);
    mbar_init(s_full, 1);
    mbar_init(m_ready, 8);
    mbar_init(ld_t, 1);
    mbar_init(d_full, 1);
    mbar_init(d_free, 8);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t TM_S = tmem, TM_DX = tmem + 128, TM_BDH = tmem + 192;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(ld_cb, 2 * T_NN);
      tma_load_2d(sC, &tmC, ld_cb, g * SN, r);
      tma_load_2d(sC + 16384, &tmC, ld_cb, g * SN + 64, r);
      tma_load_2d(sB, &tmB, ld_cb, g * SN, r);
      tma_load_2d(sB + 16384, &tmB, ld_cb, g * SN + 64, r);
      int issued = 0;
      for (int pb = 0; pb < npb; ++pb) {
        if (pb > 0 && !mbar_wait(d_free, (pb - 1) & 1, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(ld_t, 2 * T_NP);
        tma_load_2d(sDY, &tmDY, ld_t, h * p.P + pb * SP, r);
        tma_load_2d(sDH, &tmDH, ld_t, pb * SP, hrow);
        ++issued;
      }
      mbar_wait(ld_cb, 0, nullptr, p.status);  // no copy in flight at exit
      if (issued > 0) mbar_wait(ld_t, (issued - 1) & 1, nullptr, p.status);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = umma_idesc_bf16(128, 128, false, false);
      constexpr uint32_t ID_DX = umma_idesc_bf16(128, 64, true, true);
      constexpr uint32_t ID_BDH = umma_idesc_bf16(128, 64, false, true);
      const uint32_t aM = smem_u32(sC), aB = smem_u32(sB), aDY = smem_u32(sDY), aDH = smem_u32(sDH);
      bool ok = mbar_wait(ld_cb, 0, abort_flag, p.status);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) tc_mma_f16(TM_S, kdesc(aM, kk), kdesc(aB, kk), ID_S, kk != 0);
        tc_commit(s_full);
        ok = mbar_wait(m_ready, 0, abort_flag, p.status);
      }
      for (int pb = 0; pb < npb && ok; ++pb) {
        if (!mbar_wait(ld_t, pb & 1, abort_flag, p.status)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) tc_mma_f16(TM_DX, mdesc(aM, kk), mdesc(aDY, kk), ID_DX, kk != 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) tc_mma_f16(TM_BDH, kdesc(aB, kk), mdesc(aDH, kk), ID_BDH, kk != 0);
        tc_commit(d_full);
      }
    }
    __syncwarp();
  } else {
    const int m = (warp & 3) * 32 + lane;  // chunk step (t for M rows, s for dx rows)
    const int colhalf = (warp - 2) >> 2;
    const uint32_t lb = (uint32_t)((warp & 3) * 32) << 16;
    const int64_t si = ((int64_t)b * p.S + c * SL + m) * p.H + h;
    if (colhalf == 0) {
      s_lam[m] = chunk_cumsum(p.loga[si], m, s_part);
      s_gam[m] = p.gamma[si];
    }
    math8_bar();
    const float lam = s_lam[m];
    const float gm = s_gam[m];
    const float lam_end = s_lam[SL - 1];
    bool ok = mbar_wait(s_full, 0, abort_flag, p.status);
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int q = 2 * colhalf; q < 2 * colhalf + 2; ++q) {
        uint32_t sr[32];
        tmem_ld32(TM_S + lb + q * 32, sr);
        tc_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          float v[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int s2 = q * 32 + t + e;
            v[e] = (s2 <= m) ? __uint_as_float(sr[t + e]) * __expf(lam - s_lam[s2]) * s_gam[s2] : 0.f;
          }
          pk[t / 2] = pack_bf16(v[0], v[1]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int ch = q * 4 + j;
          sw128_store16(sC + (ch >> 3) * 16384, m, ch & 7,
                        make_uint4(pk[j * 4], pk[j * 4 + 1], pk[j * 4 + 2], pk[j * 4 + 3]));
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(m_ready);
    }
    const float dec = __expf(lam_end - lam);
    const float w = dec * gm;
    float dot = 0.f;
    const bool last = c == p.nc - 1;  // the last chunk's end adjoint is zero
    for (int pb = 0; pb < npb && ok; ++pb) {
      if (!mbar_wait(d_full, pb & 1, abort_flag, p.status)) { ok = false; break; }
      tc_fence_after();
      float dxv[32];
      tmem_row32(TM_DX + lb + colhalf * 32, dxv);
      if (!last) {
        float bd[32];
        tmem_row32(TM_BDH + lb + colhalf * 32, bd);
        const uint4* xr =
            reinterpret_cast<const uint4*>(x + (int64_t)(r + m) * ldx + h * p.P + pb * SP + colhalf * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 u = __ldg(xr + q);
          const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = unpack_bf16(wv[i]);
            dot += f.x * bd[q * 8 + 2 * i] + f.y * bd[q * 8 + 2 * i + 1];
          }
        }
#pragma unroll
        for (int k = 0; k < 32; ++k) dxv[k] += w * bd[k];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(d_free);
      float* dr = p.dx + (int64_t)(r + m) * ((int64_t)p.H * p.P) + h * p.P + pb * SP + colhalf * 32;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        reinterpret_cast<float4*>(dr)[k] = make_float4(dxv[4 * k], dxv[4 * k + 1], dxv[4 * k + 2], dxv[4 * k + 3]);
    }
    if (ok && !last) atomicAdd(p.dgamma + si, dec * dot);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ====================================================== backward, pass 2
// One CTA per (b, h, chunk) covering every P column, so dB / dC rows are
// written once (no atomics).  Per p-block, straight from the loaded tiles
// (double-buffered, no math in between):
//   dM += dY X^T ;  dCp += dY H^T ;  dBp += X dH^T          (four TMEM tiles with S)
// then dS = dM o D o g (smem bf16), dg_s += sum_t dM o S o D, and
//   dC = dS B + diag(exp lam) dCp ,  dB = dS^T C + diag(w) dBp
// with the diagonal scalings applied while reading TMEM out.
struct Bwd2Smem {
  static constexpr int OFF_C = 0;
  static constexpr int OFF_B = OFF_C + T_NN;
  static constexpr int OFF_DS = OFF_B + T_NN;
  static constexpr int OFF_T = OFF_DS + T_NN;            // 2 buffers x (X, dY, H, dH)
  static constexpr int T_SET = 4 * T_NP;
  static constexpr int OFF_VEC = OFF_T + 2 * T_SET;      // lam, gam, colsum, part
  static constexpr int OFF_BAR = OFF_VEC + 3 * 128 * 4 + 64;
  static constexpr int TOTAL = OFF_BAR + 128 + 1024;
};

constexpr int BWD2_THREADS = SSD_THREADS8;

__global__ void __launch_bounds__(BWD2_THREADS, 1)
    ssd_bwd2_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmDY,
                    const __grid_constant__ CUtensorMap tmHS, const __grid_constant__ CUtensorMap tmDHS, SsdParams p) {
  using L = Bwd2Smem;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sC = smem + L::OFF_C, *sB = smem + L::OFF_B, *sDS = smem + L::OFF_DS, *sT = smem + L::OFF_T;
  float* s_lam = reinterpret_cast<float*>(smem + L::OFF_VEC);
  float* s_gam = s_lam + 128;
  float* s_col = s_gam + 128;
  float* s_part = s_col + 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t *cb_full = bars + 0, *t_full = bars + 1 /* [2] */, *t_free = bars + 3 /* [2] */, *sdm_full = bars + 5,
           *ds_ready = bars + 6, *out_full = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.x, c = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int g = h / (p.H / p.G);
  const int row0 = b * p.S;
  const int r = row0 + c * SL;
  const int hrow = (bh * p.nc + c) * SN;
  const int npb = p.P / SP;
  if (threadIdx.x == 0) {
    mbar_init(cb_full, 1);
    mbar_init(&t_full[0], 1);
    mbar_init(&t_full[1], 1);
    mbar_init(&t_free[0], 1);
    mbar_init(&t_free[1], 1);
    mbar_init(sdm_full, 1);
    mbar_init(ds_ready, 8);
    mbar_init(out_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // S, then dC = dS B;  dM, then dB = dS^T C;  dY H^T;  X dH^T
  const uint32_t TM_S = tmem, TM_DM = tmem + 128, TM_CP = tmem + 256, TM_BP = tmem + 384;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(cb_full, 2 * T_NN);
      tma_load_2d(sC, &tmC, cb_full, g * SN, r);
      tma_load_2d(sC + 16384, &tmC, cb_full, g * SN + 64, r);
      tma_load_2d(sB, &tmB, cb_full, g * SN, r);
      tma_load_2d(sB + 16384, &tmB, cb_full, g * SN + 64, r);
      int pb = 0;
      for (; pb < npb; ++pb) {
        const int buf = pb & 1;
        if (pb >= 2 && !mbar_wait(&t_free[buf], ((pb >> 1) - 1) & 1, abort_flag, p.status)) break;
        uint8_t* t = sT + buf * L::T_SET;
        mbar_arrive_expect_tx(&t_full[buf], 4 * T_NP);
        tma_load_2d(t, &tmX, &t_full[buf], h * p.P + pb * SP, r);
        tma_load_2d(t + T_NP, &tmDY, &t_full[buf], h * p.P + pb * SP, r);
        tma_load_2d(t + 2 * T_NP, &tmHS, &t_full[buf], pb * SP, hrow);
        tma_load_2d(t + 3 * T_NP, &tmDHS, &t_full[buf], pb * SP, hrow);
      }
      // no copy in flight at exit: the last load into each buffer has landed
      for (int q = std::max(0, pb - 2); q < pb; ++q) mbar_wait(&t_full[q & 1], (q >> 1) & 1, nullptr, p.status);
      mbar_wait(cb_full, 0, nullptr, p.status);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_SS = umma_idesc_bf16(128, 128, false, false);
      constexpr uint32_t ID_DC1 = umma_idesc_bf16(128, 128, false, true);
      constexpr uint32_t ID_DB1 = umma_idesc_bf16(128, 128, true, true);
      const uint32_t aC = smem_u32(sC), aB = smem_u32(sB), aDS = smem_u32(sDS);
      bool ok = mbar_wait(cb_full, 0, abort_flag, p.status);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) tc_mma_f16(TM_S, kdesc(aC, kk), kdesc(aB, kk), ID_SS, kk != 0);
      }
      for (int pb = 0; pb < npb && ok; ++pb) {
        const int buf = pb & 1;
        if (!mbar_wait(&t_full[buf], (pb >> 1) & 1, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t aX = smem_u32(sT + buf * L::T_SET), aDY = aX + T_NP, aH = aX + 2 * T_NP, aDH = aX + 3 * T_NP;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t acc = (pb > 0 || kk > 0) ? 1u : 0u;
          tc_mma_f16(TM_DM, kdesc(aDY, kk), kdesc(aX, kk), ID_SS, acc);
          tc_mma_f16(TM_CP, kdesc(aDY, kk), kdesc(aH, kk), ID_SS, acc);
          tc_mma_f16(TM_BP, kdesc(aX, kk), kdesc(aDH, kk), ID_SS, acc);
        }
        tc_commit(&t_free[buf]);
      }
      if (ok) {
        tc_commit(sdm_full);
        ok = mbar_wait(ds_ready, 0, abort_flag, p.status);
      }
      if (ok) {
        tc_fence_after();
        // dC = dS B (into the S columns), dB = dS^T C (into the dM columns)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) tc_mma_f16(TM_S, kdesc(aDS, kk), mdesc(aB, kk), ID_DC1, kk != 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) tc_mma_f16(TM_DM, mdesc(aDS, kk), mdesc(aC, kk), ID_DB1, kk != 0);
        tc_commit(out_full);
      }
    }
    __syncwarp();
  } else {
    // row m (TMEM lane) of the chunk; the two warps of a lane quarter split the columns
    const int m = (warp & 3) * 32 + lane;
    const int colhalf = (warp - 2) >> 2;
    const uint32_t lb = (uint32_t)((warp & 3) * 32) << 16;
    const int64_t si = ((int64_t)b * p.S + c * SL + m) * p.H + h;
    if (colhalf == 0) {
      const float lam0 = chunk_cumsum(p.loga[si], m, s_part);  // named barrier over these 128 threads
      s_lam[m] = lam0;
      s_gam[m] = p.gamma[si];
      s_col[m] = 0.f;
    }
    asm volatile("bar.sync 2, 256;" ::: "memory");
    const float lam = s_lam[m];
    const float gm = s_gam[m];
    const float lam_end = s_lam[SL - 1];
    bool ok = mbar_wait(sdm_full, 0, abort_flag, p.status);
    if (ok) {
      tc_fence_after();
      // dS = dM o decay o g (row t = m);  column sums of dM o S o decay -> dg
#pragma unroll 1
      for (int q = 2 * colhalf; q < 2 * colhalf + 2; ++q) {
        uint32_t sr[32], dr[32];
        tmem_ld32(TM_S + lb + q * 32, sr);
        tmem_ld32(TM_DM + lb + q * 32, dr);
        tc_wait_ld();
        uint32_t pk[16];
        float cs[32];  // this row's dM o S o D over the 32 columns of chunk q
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          float v[2];
#pragma unroll
          for (int e2 = 0; e2 < 2; ++e2) {
            const int s2 = q * 32 + t + e2;
            const float d = (s2 <= m) ? __expf(lam - s_lam[s2]) : 0.f;
            const float dm = __uint_as_float(dr[t + e2]) * d;
            v[e2] = dm * s_gam[s2];
            cs[t + e2] = dm * __uint_as_float(sr[t + e2]);
          }
          pk[t / 2] = pack_bf16(v[0], v[1]);
        }
        // column sums over the warp's 32 rows by recursive halving: after the
        // exchanges at distances 16, 8, 4, 2, 1 lane L holds column q*32 + L
        // (31 shuffles instead of 5 per column)
#pragma unroll
        for (int o = 16, w = 32; o > 0; o >>= 1, w >>= 1) {
          const bool up = (lane & o) != 0;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (i < w / 2) {
              const float send = up ? cs[i] : cs[i + w / 2];
              const float keep = up ? cs[i + w / 2] : cs[i];
              cs[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
          }
        }
        atomicAdd(&s_col[q * 32 + lane], cs[0]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int ch = q * 4 + j;
          sw128_store16(sDS + (ch >> 3) * 16384, m, ch & 7, make_uint4(pk[j * 4], pk[j * 4 + 1], pk[j * 4 + 2], pk[j * 4 + 3]));
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_ready);
      asm volatile("bar.sync 2, 256;" ::: "memory");
      if (colhalf == 0) atomicAdd(p.dgamma + si, s_col[m]);
    }
    if (ok && mbar_wait(out_full, 0, abort_flag, p.status)) {
      tc_fence_after();
      // row m: dC_t (t = m) and dB_s (s = m), 128 values each, written once
      const float e = __expf(lam);
      const float w = __expf(lam_end - lam) * gm;
      const int64_t orow = ((int64_t)row0 + c * SL + m) * ((int64_t)p.H * SN) + h * SN + colhalf * 64;
      {
        float v[64], u[64];
        tmem_row64(TM_S + lb + colhalf * 64, v);
        tmem_row64(TM_CP + lb + colhalf * 64, u);
#pragma unroll
        for (int k = 0; k < 64; ++k) v[k] += e * u[k];
        store_row_out(p.dC, orow, v, p.dbc_bf16);
        tmem_row64(TM_DM + lb + colhalf * 64, v);
        tmem_row64(TM_BP + lb + colhalf * 64, u);
#pragma unroll
        for (int k = 0; k < 64; ++k) v[k] += w * u[k];
        store_row_out(p.dB, orow, v, p.dbc_bf16);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <typename K>
void set_smem(K kern, int bytes) {
  OXI_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

}  // namespace

bool ssd_tc_supported(int N, int P, int S) { return N == SN && P % SP == 0 && S % SL == 0 && S > 0; }

void launch_ssd_fwd(const SsdTcIO& io, cudaStream_t st) {
  OXI_CHECK(ssd_tc_supported(io.N, io.P, io.S), "tensor-core SSD needs N == 128, P % 64 == 0, S % 128 == 0");
  OXI_CHECK(io.H % io.G == 0, "heads must be a multiple of the B/C groups");
  OXI_CHECK(io.hloc && io.lamend, "forward scratch missing");
  const int64_t T = (int64_t)io.B * io.S;
  const int nc = io.S / SL;
  CUtensorMap tx = make_tmap_bf16(io.x, T, (int64_t)io.H * io.P, io.ldx, 64, SL);
  CUtensorMap tb = make_tmap_bf16(io.Bm, T, (int64_t)io.G * SN, io.ldb, 64, SL);
  CUtensorMap tc = make_tmap_bf16(io.Cm, T, (int64_t)io.G * SN, io.ldc, 64, SL);
  const int64_t hrows = (int64_t)io.B * io.H * nc * SN;
  CUtensorMap ths = make_tmap_bf16(io.hs, hrows, io.P, io.P, 64, SN);
  SsdParams p{};
  p.B = io.B; p.S = io.S; p.H = io.H; p.P = io.P; p.G = io.G; p.nc = nc;
  p.loga = io.loga; p.gamma = io.gamma; p.y = io.y;
  p.hs = reinterpret_cast<__nv_bfloat16*>(io.hs);
  p.hloc = io.hloc; p.lamend = io.lamend;
  p.out = reinterpret_cast<__nv_bfloat16*>(io.out);
  p.dskip = io.dskip; p.dskip_per_row = io.dskip_per_row;
  p.status = io.status;
  static bool attr = false;
  if (!attr) {
    set_smem(ssd_state_kernel<false>, StateSmem::TOTAL);
    set_smem(ssd_out_kernel, OutSmem::TOTAL);
    attr = true;
  }
  const dim3 grid(io.B * io.H, nc);
  ssd_state_kernel<false><<<grid, SSD_THREADS, StateSmem::TOTAL, st>>>(tx, tb, p);
  OXI_CUDA_CHECK(cudaGetLastError());
  const int64_t per = (int64_t)SN * io.P;
  ssd_state_scan_kernel<false><<<dim3((unsigned)((per + 255) / 256), io.B * io.H), 256, 0, st>>>(
      p.hloc, p.lamend, p.hs, nc, io.P);
  OXI_CUDA_CHECK(cudaGetLastError());
  ssd_out_kernel<<<grid, SSD_THREADS8, OutSmem::TOTAL, st>>>(tx, tb, tc, ths, p);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_ssd_bwd(const SsdTcIO& io, cudaStream_t st) {
  OXI_CHECK(ssd_tc_supported(io.N, io.P, io.S), "tensor-core SSD needs N == 128, P % 64 == 0, S % 128 == 0");
  const int64_t T = (int64_t)io.B * io.S;
  const int nc = io.S / SL;
  CUtensorMap tx = make_tmap_bf16(io.x, T, (int64_t)io.H * io.P, io.ldx, 64, SL);
  CUtensorMap tb = make_tmap_bf16(io.Bm, T, (int64_t)io.G * SN, io.ldb, 64, SL);
  CUtensorMap tc = make_tmap_bf16(io.Cm, T, (int64_t)io.G * SN, io.ldc, 64, SL);
  CUtensorMap tdy = make_tmap_bf16(io.dy, T, (int64_t)io.H * io.P, (int64_t)io.H * io.P, 64, SL);
  const int64_t hrows = (int64_t)io.B * io.H * nc * SN;
  CUtensorMap ths = make_tmap_bf16(io.hs, hrows, io.P, io.P, 64, SN);
  CUtensorMap tdhs = make_tmap_bf16(io.dhs, hrows, io.P, io.P, 64, SN);
  SsdParams p{};
  p.B = io.B; p.S = io.S; p.H = io.H; p.P = io.P; p.G = io.G; p.nc = nc;
  p.loga = io.loga; p.gamma = io.gamma;
  p.hs = reinterpret_cast<__nv_bfloat16*>(io.hs);
  p.dhs = reinterpret_cast<__nv_bfloat16*>(io.dhs);
  p.dx = io.dx; p.dB = io.dB; p.dC = io.dC; p.dgamma = io.dgamma; p.dbc_bf16 = io.dbc_bf16;
  p.hloc = io.hloc; p.lamend = io.lamend;
  p.status = io.status;
  OXI_CHECK(io.hloc && io.lamend, "backward scratch missing");
  static bool attr = false;
  if (!attr) {
    set_smem(ssd_state_kernel<true>, StateSmem::TOTAL);
    set_smem(ssd_dx_kernel, DxSmem::TOTAL);
    set_smem(ssd_bwd2_kernel, Bwd2Smem::TOTAL);
    attr = true;
  }
  const dim3 grid(io.B * io.H, nc);
  // chunk-local adjoints C^T diag(exp Lam) dY, then the reverse scan -> chunk-end adjoints
  ssd_state_kernel<true><<<grid, SSD_THREADS, StateSmem::TOTAL, st>>>(tdy, tc, p);
  OXI_CUDA_CHECK(cudaGetLastError());
  const int64_t per = (int64_t)SN * io.P;
  ssd_state_scan_kernel<true><<<dim3((unsigned)((per + 255) / 256), io.B * io.H), 256, 0, st>>>(
      p.hloc, p.lamend, p.dhs, nc, io.P);
  OXI_CUDA_CHECK(cudaGetLastError());
  ssd_dx_kernel<<<grid, SSD_THREADS8, DxSmem::TOTAL, st>>>(tb, tc, tdy, tdhs, reinterpret_cast<const __nv_bfloat16*>(io.x),
                                                          io.ldx, p);
  OXI_CUDA_CHECK(cudaGetLastError());
  ssd_bwd2_kernel<<<grid, BWD2_THREADS, Bwd2Smem::TOTAL, st>>>(tx, tb, tc, tdy, ths, tdhs, p);
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
