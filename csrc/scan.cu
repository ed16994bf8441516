// Selective state-space scans on CUDA cores: the Mamba2 SSD recurrence, the
// Mamba3 trapezoidal two-term recurrence, and the Mamba1 diagonal scan.
//
// Mamba2/3 (per batch b, head h; state H_t is N x P):
//   H_t = alpha_t H_{t-1} + gamma_t B_t x_t^T + beta_t B_{t-1} x_{t-1}^T
//   y_t = H_t^T C_t
// Mamba2: alpha = exp(A dt), gamma = dt, beta = 0 (mamba2.rs:381-482).
// Mamba3: alpha = exp(A dt), gamma = lambda dt, beta = (1 - lambda) dt alpha
//         (mamba3.rs:638-752; B, C already normed/biased/rotated).
// This is the exact recurrence the chunked SSD evaluates, so results do not
// depend on the chunk size.
//
// One CTA of 8 warps per (b, h).  Warp w owns P/8 columns p of the state, lane
// l owns rows n = l + 32 k (k < N/32): every thread holds (N/32) x (P/8)
// state values in registers.  y_t[p] reduces over n with warp shuffles, so a
// time step needs no block-level synchronisation.  Inputs of step t+1 are
// loaded while step t computes.
//
// Backward (two kernels; no per-step state is stored):
//   dC_t = H_t dy_t                                    (forward recompute)
//   G_t = C_t dy_t^T + alpha_{t+1} G_{t+1}             (reverse adjoint scan)
//   dx_t = gamma_t G_t^T B_t + beta_{t+1} G_{t+1}^T B_t
//   dB_t = gamma_t G_t x_t + beta_{t+1} G_{t+1} x_t
//   dgamma_t = <G_t, B_t x_t^T>,  dbeta_t = <G_t, B_{t-1} x_{t-1}^T>
// d(log alpha_t) = <G_t, alpha_t H_{t-1}> is recovered outside the kernel
// from q_t = <G_t, H_t> = <dy_t, y_t> + q_{t+1} - v_{t+1}, v = gamma dgamma +
// beta dbeta, since <G_t, alpha_t H_{t-1}> = q_t - v_t.
//
// Mamba1 (mamba.rs:212-291): per channel d, state h (N = 16):
//   h_t = exp(delta_t A_d) h_{t-1} + delta_t x_t B_t ;  y_t = C_t . h_t
// The compatibility clamp of every state to +-clamp makes the recurrence nonlinear,
// so the kernel stays sequential in t (for both modes); the parallelism is (b, d, n): a half-warp per channel,
// one lane per state, y / du / d delta as 16-lane shuffle sums.  The backward reads
// the per-step states the forward saved; both kernels load the operands of their
// next few steps while computing the current ones.  The dB / dC terms (sums over channels)
// are staged per 32-step chunk in shared memory, summed over the block's warps and
// added with one atomic per (step, n) per block.
#include <cuda_runtime.h>
#include <cstdint>

#include "host_util.h"
#include "kernels_ssm.h"

namespace oxi {
namespace {

constexpr int SCAN_WARPS = 8;

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

struct ScanArgs {
  const float *x, *Bm, *Cm, *loga, *gamma, *beta, *dy;
  float *y, *dx, *dB, *dC, *dgamma, *dbeta;
  int Bsz, S, H;
  // element strides (batch, time, head) of x/dx/y/dy [.., P] and B/C/dB/dC [.., N]
  int64_t xs_b, xs_t, xs_h;
  int64_t bs_b, bs_t, bs_h;
  int64_t ss_b, ss_t, ss_h;  // scalars loga/gamma/beta/dgamma/dbeta [B, S, H]
};

// ---------------------------------------------------------------- forward
template <int NL, int PW, bool TWO, bool DC>
__global__ void __launch_bounds__(SCAN_WARPS * 32) ssm_scan_fwd_kernel(ScanArgs a) {
  const int bh = blockIdx.x;
  const int b = bh / a.H, h = bh % a.H;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int p0 = warp * PW;
  const float* xb = a.x + b * a.xs_b + h * a.xs_h + p0;
  const float* Bb = a.Bm + b * a.bs_b + h * a.bs_h + lane;
  const float* Cb = a.Cm + b * a.bs_b + h * a.bs_h + lane;
  const int64_t so = b * a.ss_b + h * a.ss_h;
  float st[NL][PW];
#pragma unroll
  for (int i = 0; i < NL; ++i)
#pragma unroll
    for (int j = 0; j < PW; ++j) st[i][j] = 0.f;
  float bprev[NL], xprev[PW];
#pragma unroll
  for (int i = 0; i < NL; ++i) bprev[i] = 0.f;
#pragma unroll
  for (int j = 0; j < PW; ++j) xprev[j] = 0.f;
  // prefetched inputs of the current step
  float bn[NL], cn[NL], xv[PW], la, ga, be;
  auto load = [&](int t) {
#pragma unroll
    for (int i = 0; i < NL; ++i) {
      bn[i] = Bb[t * a.bs_t + 32 * i];
      cn[i] = Cb[t * a.bs_t + 32 * i];
    }
#pragma unroll
    for (int j = 0; j < PW; ++j) xv[j] = xb[t * a.xs_t + j];
    la = a.loga[so + t * a.ss_t];
    ga = a.gamma[so + t * a.ss_t];
    be = TWO ? a.beta[so + t * a.ss_t] : 0.f;
  };
  if (a.S > 0) load(0);
  for (int t = 0; t < a.S; ++t) {
    float cbn[NL], ccn[NL], cx[PW];
#pragma unroll
    for (int i = 0; i < NL; ++i) { cbn[i] = bn[i]; ccn[i] = cn[i]; }
#pragma unroll
    for (int j = 0; j < PW; ++j) cx[j] = xv[j];
    const float al = __expf(la), g = ga, bt = be;
    if (t + 1 < a.S) load(t + 1);
    float ypart[PW];
#pragma unroll
    for (int j = 0; j < PW; ++j) ypart[j] = 0.f;
#pragma unroll
    for (int i = 0; i < NL; ++i) {
      const float gb = g * cbn[i];
      const float bb = TWO ? bt * bprev[i] : 0.f;
#pragma unroll
      for (int j = 0; j < PW; ++j) {
        float v = al * st[i][j] + gb * cx[j];
        if (TWO) v += bb * xprev[j];
        st[i][j] = v;
        ypart[j] += ccn[i] * v;
      }
    }
    if (DC) {
      // dC_t[n] = sum_p H_t[n, p] dy_t[p]: this warp's partial over its p columns
      const float* dyb = a.dy + b * a.xs_b + h * a.xs_h + p0 + t * a.xs_t;
      float dyv[PW];
#pragma unroll
      for (int j = 0; j < PW; ++j) dyv[j] = dyb[j];
#pragma unroll
      for (int i = 0; i < NL; ++i) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < PW; ++j) s += st[i][j] * dyv[j];
        atomicAdd(a.dC + b * a.bs_b + h * a.bs_h + t * a.bs_t + lane + 32 * i, s);
      }
    } else {
#pragma unroll
      for (int j = 0; j < PW; ++j) {
        const float yv = warp_allsum(ypart[j]);
        if (lane == j % 32) a.y[b * a.xs_b + h * a.xs_h + t * a.xs_t + p0 + j] = yv;
      }
    }
    if (TWO) {
#pragma unroll
      for (int i = 0; i < NL; ++i) bprev[i] = cbn[i];
#pragma unroll
      for (int j = 0; j < PW; ++j) xprev[j] = cx[j];
    }
  }
}

// ------------------------------------------------------- reverse adjoint
template <int NL, int PW, bool TWO>
__global__ void __launch_bounds__(SCAN_WARPS * 32) ssm_scan_bwd_kernel(ScanArgs a) {
  const int bh = blockIdx.x;
  const int b = bh / a.H, h = bh % a.H;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int p0 = warp * PW;
  const int64_t xo = b * a.xs_b + h * a.xs_h + p0;
  const int64_t bo = b * a.bs_b + h * a.bs_h + lane;
  const int64_t so = b * a.ss_b + h * a.ss_h;
  float G[NL][PW];  // adjoint G_{t+1} on entry to step t
#pragma unroll
  for (int i = 0; i < NL; ++i)
#pragma unroll
    for (int j = 0; j < PW; ++j) G[i][j] = 0.f;
  float al_next = 0.f, be_next = 0.f;  // alpha_{t+1}, beta_{t+1}
  for (int t = a.S - 1; t >= 0; --t) {
    float bn[NL], cn[NL], bp[NL], xv[PW], xp[PW], dyv[PW];
#pragma unroll
    for (int i = 0; i < NL; ++i) {
      bn[i] = a.Bm[bo + t * a.bs_t + 32 * i];
      cn[i] = a.Cm[bo + t * a.bs_t + 32 * i];
      bp[i] = (TWO && t > 0) ? a.Bm[bo + (t - 1) * a.bs_t + 32 * i] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < PW; ++j) {
      xv[j] = a.x[xo + t * a.xs_t + j];
      xp[j] = (TWO && t > 0) ? a.x[xo + (t - 1) * a.xs_t + j] : 0.f;
      dyv[j] = a.dy[xo + t * a.xs_t + j];
    }
    const float g = a.gamma[so + t * a.ss_t];
    const float be = TWO ? a.beta[so + t * a.ss_t] : 0.f;
    // terms with G_{t+1} (beta_{t+1}): contributions of x_t, B_t to u_{t+1}
    float dxp[PW], dbn[NL];
#pragma unroll
    for (int j = 0; j < PW; ++j) dxp[j] = 0.f;
#pragma unroll
    for (int i = 0; i < NL; ++i) dbn[i] = 0.f;
    if (TWO) {
#pragma unroll
      for (int i = 0; i < NL; ++i)
#pragma unroll
        for (int j = 0; j < PW; ++j) {
          dxp[j] += be_next * G[i][j] * bn[i];
          dbn[i] += be_next * G[i][j] * xv[j];
        }
    }
    // G_t = C_t dy_t^T + alpha_{t+1} G_{t+1}
#pragma unroll
    for (int i = 0; i < NL; ++i)
#pragma unroll
      for (int j = 0; j < PW; ++j) G[i][j] = cn[i] * dyv[j] + al_next * G[i][j];
    float dg = 0.f, dbt = 0.f;
#pragma unroll
    for (int i = 0; i < NL; ++i) {
      float sx = 0.f, sxp = 0.f;
#pragma unroll
      for (int j = 0; j < PW; ++j) {
        sx += G[i][j] * xv[j];
        if (TWO) sxp += G[i][j] * xp[j];
        dxp[j] += g * G[i][j] * bn[i];
      }
      dbn[i] += g * sx;
      dg += bn[i] * sx;
      if (TWO) dbt += bp[i] * sxp;
    }
    // dx_t[p]: reduce over n (lanes); dB_t[n]: partial over this warp's p -> atomics
#pragma unroll
    for (int j = 0; j < PW; ++j) {
      const float v = warp_allsum(dxp[j]);
      if (lane == j % 32) a.dx[xo + t * a.xs_t + j] = v;
    }
#pragma unroll
    for (int i = 0; i < NL; ++i) atomicAdd(a.dB + bo + t * a.bs_t + 32 * i, dbn[i]);
    dg = warp_allsum(dg);
    if (TWO) dbt = warp_allsum(dbt);
    if (lane == 0) {
      atomicAdd(a.dgamma + so + t * a.ss_t, dg);
      if (TWO) atomicAdd(a.dbeta + so + t * a.ss_t, dbt);
    }
    al_next = __expf(a.loga[so + t * a.ss_t]);
    be_next = be;
  }
}

// ---------------------------------------------------------------- Mamba1
constexpr int M1N = 16;

constexpr int M1_CH = 32;  // backward chunk (steps) for the dB / dC staging
constexpr int M1_PFF = 8;  // forward steps whose operands are loaded one group ahead
constexpr int M1_PFB = 4;  // backward steps per prefetch group (M1_CH is a multiple)

// block = 8 warps x 2 channels x 16 states: 16 channels of one batch row; grid (ceil(D / 16), B).
// Each thread loads the operands of its next M1_PFF steps while it computes the current ones.
__global__ void __launch_bounds__(256) mamba1_fwd_kernel(const float* __restrict__ u, const float* __restrict__ delta,
                                                         const float* __restrict__ A, const float* __restrict__ Bm,
                                                         const float* __restrict__ Cm, float* __restrict__ y,
                                                         float* __restrict__ hs, int S, int Dch, float clamp) {
  const int lane = threadIdx.x & 31, n = lane & 15;
  const int d = blockIdx.x * 16 + (threadIdx.x >> 5) * 2 + (lane >> 4);
  const int b = blockIdx.y;
  const bool live = d < Dch;
  const float a = live ? A[d * M1N + n] : 0.f;
  const int64_t base = (int64_t)b * S;
  auto load = [&](int tg, float* dl, float* xv, float* bv, float* cv) {
#pragma unroll
    for (int i = 0; i < M1_PFF; ++i) {
      const int t = tg + i;
      const bool ok = t < S;
      const int64_t r = base + (ok ? t : 0);
      dl[i] = (live && ok) ? delta[r * Dch + d] : 0.f;
      xv[i] = (live && ok) ? u[r * Dch + d] : 0.f;
      bv[i] = ok ? Bm[r * M1N + n] : 0.f;
      cv[i] = ok ? Cm[r * M1N + n] : 0.f;
    }
  };
  float dl[M1_PFF], xv[M1_PFF], bv[M1_PFF], cv[M1_PFF];
  load(0, dl, xv, bv, cv);
  float h = 0.f;
  for (int tg = 0; tg < S; tg += M1_PFF) {
    float ndl[M1_PFF], nxv[M1_PFF], nbv[M1_PFF], ncv[M1_PFF];
    if (tg + M1_PFF < S) load(tg + M1_PFF, ndl, nxv, nbv, ncv);
    // decays and inputs of the group do not depend on h: computed together
    float e[M1_PFF], wb[M1_PFF], p[M1_PFF];
#pragma unroll
    for (int i = 0; i < M1_PFF; ++i) {
      e[i] = __expf(dl[i] * a);
      wb[i] = dl[i] * xv[i] * bv[i];
    }
    // the sequential part: one FMA (and the clamp) per step
#pragma unroll
    for (int i = 0; i < M1_PFF; ++i) {
      float v = e[i] * h + wb[i];
      if (clamp > 0.f) v = fminf(fmaxf(v, -clamp), clamp);
      h = v;
      p[i] = v * cv[i];
      if (live && tg + i < S) hs[((base + tg + i) * Dch + d) * M1N + n] = v;
    }
    // the group's 16-lane sums, shuffles of all steps interleaved per level
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < M1_PFF; ++i) p[i] += __shfl_xor_sync(0xffffffffu, p[i], o);
    if (live && n < M1_PFF && tg + n < S) {
      float yv = p[0];
#pragma unroll
      for (int i = 1; i < M1_PFF; ++i) yv = n == i ? p[i] : yv;
      y[(base + tg + n) * Dch + d] = yv;
    }
#pragma unroll
    for (int i = 0; i < M1_PFF; ++i) {
      dl[i] = ndl[i];
      xv[i] = nxv[i];
      bv[i] = nbv[i];
      cv[i] = ncv[i];
    }
  }
}

__global__ void __launch_bounds__(256) mamba1_bwd_kernel(const float* __restrict__ u, const float* __restrict__ delta,
                                                         const float* __restrict__ A, const float* __restrict__ Bm,
                                                         const float* __restrict__ Cm, const float* __restrict__ hs,
                                                         const float* __restrict__ dy, float* __restrict__ du,
                                                         float* __restrict__ ddelta, float* __restrict__ dA,
                                                         float* __restrict__ dB, float* __restrict__ dC, int S,
                                                         int Dch, float clamp) {
  __shared__ float s_db[8][M1_CH][M1N], s_dc[8][M1_CH][M1N];
  const int lane = threadIdx.x & 31, n = lane & 15, wid = threadIdx.x >> 5;
  const int d = blockIdx.x * 16 + wid * 2 + (lane >> 4);
  const int b = blockIdx.y;
  const bool live = d < Dch;
  const float a = live ? A[d * M1N + n] : 0.f;
  const int64_t base = (int64_t)b * S;
  // group k holds steps S-1-k*PF .. S-PF-k*PF (descending); q: 0 h_{t-1}, 1 delta, 2 x, 3 dy, 4 C, 5 B
  auto load = [&](int k, float (*q)[M1_PFB]) {
#pragma unroll
    for (int i = 0; i < M1_PFB; ++i) {
      const int t = S - 1 - k * M1_PFB - i;
      const bool ok = t >= 0;
      const int64_t r = base + (ok ? t : 0);
      q[0][i] = (live && t > 0) ? hs[((r - 1) * Dch + d) * M1N + n] : 0.f;
      q[1][i] = (live && ok) ? delta[r * Dch + d] : 0.f;
      q[2][i] = (live && ok) ? u[r * Dch + d] : 0.f;
      q[3][i] = (live && ok) ? dy[r * Dch + d] : 0.f;
      q[4][i] = ok ? Cm[r * M1N + n] : 0.f;
      q[5][i] = ok ? Bm[r * M1N + n] : 0.f;
    }
  };
  const int ngroups = (S + M1_PFB - 1) / M1_PFB;
  constexpr int GPC = M1_CH / M1_PFB;  // groups per chunk (chunks are aligned from the top step)
  float cur[6][M1_PFB];
  load(0, cur);
  float hn = live ? hs[((base + S - 1) * Dch + d) * M1N + n] : 0.f;
  float g = 0.f, dAacc = 0.f;
  for (int k = 0; k < ngroups; ++k) {
    float nxt[6][M1_PFB];
    if (k + 1 < ngroups) load(k + 1, nxt);
    const int t1 = S - M1_CH * (k / GPC), t0 = t1 > M1_CH ? t1 - M1_CH : 0;
    // decays of the group first (independent of the adjoint); then the sequential adjoint chain;
    // then the group's reductions with the shuffles of all steps interleaved per level
    float e[M1_PFB], ddl[M1_PFB], dxv[M1_PFB], cdb[M1_PFB], cdc[M1_PFB];
#pragma unroll
    for (int i = 0; i < M1_PFB; ++i) e[i] = __expf(cur[1][i] * a);
#pragma unroll
    for (int i = 0; i < M1_PFB; ++i) {
      const float hp = cur[0][i], dl = cur[1][i], xv = cur[2][i], gy = cur[3][i], cv = cur[4][i], bv = cur[5][i];
      // steps past the start (t < 0) have zero inputs: their terms vanish
      g += gy * cv;
      cdc[i] = gy * hn;
      // clamp: the gradient passes only where the state was not clipped
      if (clamp > 0.f && (hn >= clamp || hn <= -clamp)) g = 0.f;
      ddl[i] = g * (a * e[i] * hp + xv * bv);
      dAacc += g * dl * e[i] * hp;
      dxv[i] = g * dl * bv;
      cdb[i] = g * dl * xv;
      g *= e[i];  // to h_{t-1}
      hn = hp;
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < M1_PFB; ++i) {
        ddl[i] += __shfl_xor_sync(0xffffffffu, ddl[i], o);
        dxv[i] += __shfl_xor_sync(0xffffffffu, dxv[i], o);
      }
#pragma unroll
    for (int i = 0; i < M1_PFB; ++i) {
      cdc[i] += __shfl_xor_sync(0xffffffffu, cdc[i], 16);  // the warp's two channels
      cdb[i] += __shfl_xor_sync(0xffffffffu, cdb[i], 16);
    }
#pragma unroll
    for (int i = 0; i < M1_PFB; ++i) {
      const int t = S - 1 - k * M1_PFB - i;
      if (t < 0) break;
      if (lane < 16) {
        s_dc[wid][t - t0][n] = cdc[i];
        s_db[wid][t - t0][n] = cdb[i];
      }
      if (live && n == 0) {
        du[(base + t) * Dch + d] = dxv[i];
        ddelta[(base + t) * Dch + d] = ddl[i];
      }
    }
    if (k % GPC == GPC - 1 || k == ngroups - 1) {
      __syncthreads();
      for (int e = threadIdx.x; e < (t1 - t0) * M1N; e += blockDim.x) {
        const int j = e / M1N, c = e % M1N;
        float sb = 0.f, sc = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          sb += s_db[w][j][c];
          sc += s_dc[w][j][c];
        }
        atomicAdd(&dB[(base + t0 + j) * M1N + c], sb);
        atomicAdd(&dC[(base + t0 + j) * M1N + c], sc);
      }
      __syncthreads();
    }
#pragma unroll
    for (int q = 0; q < 6; ++q)
#pragma unroll
      for (int i = 0; i < M1_PFB; ++i) cur[q][i] = nxt[q][i];
  }
  if (live) atomicAdd(&dA[d * M1N + n], dAacc);
}

template <int NL, int PW>
void dispatch_two(const ScanArgs& a, bool two, bool dc, cudaStream_t st) {
  const dim3 grid(a.Bsz * a.H), block(SCAN_WARPS * 32);
  if (dc) {
    if (two) ssm_scan_fwd_kernel<NL, PW, true, true><<<grid, block, 0, st>>>(a);
    else ssm_scan_fwd_kernel<NL, PW, false, true><<<grid, block, 0, st>>>(a);
  } else {
    if (two) ssm_scan_fwd_kernel<NL, PW, true, false><<<grid, block, 0, st>>>(a);
    else ssm_scan_fwd_kernel<NL, PW, false, false><<<grid, block, 0, st>>>(a);
  }
}

template <int NL, int PW>
void dispatch_bwd(const ScanArgs& a, bool two, cudaStream_t st) {
  const dim3 grid(a.Bsz * a.H), block(SCAN_WARPS * 32);
  if (two) ssm_scan_bwd_kernel<NL, PW, true><<<grid, block, 0, st>>>(a);
  else ssm_scan_bwd_kernel<NL, PW, false><<<grid, block, 0, st>>>(a);
}

#define OXI_SCAN_SHAPES(X) \
  X(1, 2) X(2, 2) X(4, 2) X(1, 8) X(2, 8) X(4, 8) X(1, 16) X(2, 16) X(4, 16) X(1, 32) X(2, 32) X(4, 32) X(1, 4) X(2, 4) X(4, 4)

bool run_fwd(int N, int P, const ScanArgs& a, bool two, bool dc, cudaStream_t st) {
  const int NL = N / 32, PW = P / SCAN_WARPS;
#define X(nl, pw) \
  if (NL == nl && PW == pw) { dispatch_two<nl, pw>(a, two, dc, st); return true; }
  OXI_SCAN_SHAPES(X)
#undef X
  return false;
}

bool run_bwd(int N, int P, const ScanArgs& a, bool two, cudaStream_t st) {
  const int NL = N / 32, PW = P / SCAN_WARPS;
#define X(nl, pw) \
  if (NL == nl && PW == pw) { dispatch_bwd<nl, pw>(a, two, st); return true; }
  OXI_SCAN_SHAPES(X)
#undef X
  return false;
}

}  // namespace

void launch_ssm_scan(const SsmScanIO& io, int Bsz, int S, int H, int N, int P, bool two, int mode,
                     cudaStream_t st) {
  OXI_CHECK(N % 32 == 0 && P % SCAN_WARPS == 0, "scan: state size must be a multiple of 32 and head dim of 8");
  if (!Bsz || !S || !H) return;
  ScanArgs a;
  a.x = io.x; a.Bm = io.Bm; a.Cm = io.Cm; a.loga = io.loga; a.gamma = io.gamma; a.beta = io.beta; a.dy = io.dy;
  a.y = io.y; a.dx = io.dx; a.dB = io.dB; a.dC = io.dC; a.dgamma = io.dgamma; a.dbeta = io.dbeta;
  a.Bsz = Bsz; a.S = S; a.H = H;
  a.xs_b = io.xs[0]; a.xs_t = io.xs[1]; a.xs_h = io.xs[2];
  a.bs_b = io.bs[0]; a.bs_t = io.bs[1]; a.bs_h = io.bs[2];
  a.ss_b = io.ss[0]; a.ss_t = io.ss[1]; a.ss_h = io.ss[2];
  bool ok;
  if (mode == 0) ok = run_fwd(N, P, a, two, false, st);        // y
  else if (mode == 1) ok = run_fwd(N, P, a, two, true, st);    // dC
  else ok = run_bwd(N, P, a, two, st);                         // dx, dB, dgamma, dbeta
  OXI_CHECK(ok, "scan: unsupported (state, head_dim) = (", N, ", ", P, ")");
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_mamba1_fwd(const float* u, const float* delta, const float* A, const float* Bm, const float* Cm, float* y,
                       float* hs, int Bsz, int S, int Dch, float clamp, cudaStream_t st) {
  const int64_t n = (int64_t)Bsz * Dch;
  if (!n || !S) return;
  OXI_CHECK(Bsz <= 65535, "mamba1 scan: batch too large for one launch");
  mamba1_fwd_kernel<<<dim3((unsigned)((Dch + 15) / 16), (unsigned)Bsz), 256, 0, st>>>(u, delta, A, Bm, Cm, y, hs, S,
                                                                                     Dch, clamp);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_mamba1_bwd(const float* u, const float* delta, const float* A, const float* Bm, const float* Cm,
                       const float* hs, const float* dy, float* du, float* ddelta, float* dA, float* dB, float* dC,
                       int Bsz, int S, int Dch, float clamp, cudaStream_t st) {
  const int64_t n = (int64_t)Bsz * Dch;
  if (!n || !S) return;
  OXI_CHECK(Bsz <= 65535, "mamba1 scan: batch too large for one launch");
  mamba1_bwd_kernel<<<dim3((unsigned)((Dch + 15) / 16), (unsigned)Bsz), 256, 0, st>>>(u, delta, A, Bm, Cm, hs, dy, du,
                                                                                     ddelta, dA, dB, dC, S, Dch, clamp);
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
