// Memory-bound training kernels: cross-entropy finish/backward, embedding
// gather/scatter, RoPE backward, gradient-norm, clip coefficient and the flat
// multi-tensor AdamW update.  All are single-pass over their data with 16-byte
// vector accesses; none synchronises with the host.
// Upstream: cross-entropy trainer.rs:166-171 and model.rs:1002; embedding model.rs:964;
// RoPE model.rs:68-117; gradient norm trainer.rs:560-574; AdamW trainer.rs:60-64,245 and
// distributed/optimizer.rs:126-192.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "host_util.h"
#include "kernels_ew.h"
#include "ptx.cuh"

namespace oxi {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// --------------------------------------------------------------- CE finish
// One warp per row: lse = logsumexp over the per-tile (max, sum) partials;
// loss = lse - target_logit (0 for ignored rows, target < 0).
__global__ void ce_finish_kernel(const float* __restrict__ pmax, const float* __restrict__ psum, int nt,
                                 const float* __restrict__ tgt_logit, const int64_t* __restrict__ targets,
                                 float* __restrict__ lse, float* __restrict__ loss, int64_t rows) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= rows) return;
  float m = -INFINITY;
  for (int i = lane; i < nt; i += 32) m = fmaxf(m, pmax[row * nt + i]);
  m = warp_max(m);
  float s = 0.f;
  for (int i = lane; i < nt; i += 32) {
    const float mi = pmax[row * nt + i];
    if (mi > -INFINITY) s += psum[row * nt + i] * __expf(mi - m);
  }
  s = warp_sum(s);
  if (lane == 0) {
    const float l = m + logf(s);
    lse[row] = l;
    loss[row] = targets[row] >= 0 ? (l - tgt_logit[row]) : 0.f;
  }
}

// ------------------------------------------------------------------ CE bwd
// In place: logits[r, v] <- (exp(logits - lse[r]) - [v == t_r]) * scale, where
// scale = (*gscale) * inv_count.  Rows with target < 0 get zero gradient.
// col0: vocabulary index of the buffer's first column (a column chunk of the
// logits recomputed in the logit-free backward); a target outside the chunk adds
// no one-hot term, an ignored row (target < 0) is zero.
// In place: logits[row, c] <- (softmax - onehot) * scale for the columns c of a
// vocabulary slice starting at col0.  Each thread handles CE_BWD_VEC 16-byte vectors
// per pass (all loads issued before the math), so a row needs few CTAs and every
// thread keeps several loads in flight.
constexpr int CE_BWD_VEC = 4;

__global__ void __launch_bounds__(256) ce_bwd_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld, int64_t V,
                                                     const float* __restrict__ lse,
                                                     const int64_t* __restrict__ targets,
                                                     const float* __restrict__ gscale, float inv_count, int64_t col0) {
  const int64_t row = blockIdx.y;
  const float l = lse[row];
  const int64_t t0 = targets[row];
  const float sc = (t0 >= 0) ? (*gscale) * inv_count : 0.f;
  const int64_t t = t0 - col0;
  __nv_bfloat16* rp = logits + row * ld;
  uint4* rv = reinterpret_cast<uint4*>(rp);
  const int64_t nvec = V / 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < nvec; base += stride * CE_BWD_VEC) {
    uint4 u[CE_BWD_VEC];
#pragma unroll
    for (int q = 0; q < CE_BWD_VEC; ++q) {
      const int64_t i = base + q * stride;
      if (i < nvec) u[q] = rv[i];
    }
#pragma unroll
    for (int q = 0; q < CE_BWD_VEC; ++q) {
      const int64_t i = base + q * stride;
      if (i >= nvec) continue;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u[q]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float2 f = __bfloat1622float2(h[k]);
        const int64_t c = i * 8 + 2 * k;
        f.x = (__expf(f.x - l) - (c == t ? 1.f : 0.f)) * sc;
        f.y = (__expf(f.y - l) - (c + 1 == t ? 1.f : 0.f)) * sc;
        h[k] = __floats2bfloat162_rn(f.x, f.y);
      }
      rv[i] = u[q];
    }
  }
  if (blockIdx.x == 0) {
    for (int64_t c = nvec * 8 + threadIdx.x; c < V; c += blockDim.x) {
      const float f = __bfloat162float(rp[c]);
      rp[c] = __float2bfloat16((__expf(f - l) - (c == t ? 1.f : 0.f)) * sc);
    }
  }
}

// --------------------------------------------------------------- embedding
__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ w,
                                 __nv_bfloat16* __restrict__ out, int64_t rows, int H) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const uint4* src = reinterpret_cast<const uint4*>(w + ids[row] * (int64_t)H);
  uint4* dst = reinterpret_cast<uint4*>(out + row * (int64_t)H);
  for (int i = lane; i < H / 8; i += 32) dst[i] = src[i];
}

__global__ void embed_bwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ dy,
                                 float* __restrict__ dw, int64_t rows, int H) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const __nv_bfloat162* src = reinterpret_cast<const __nv_bfloat162*>(dy + row * (int64_t)H);
  float* dst = dw + ids[row] * (int64_t)H;
  for (int i = lane; i < H / 4; i += 32) {
    const float2 a = __bfloat1622float2(src[2 * i]);
    const float2 b = __bfloat1622float2(src[2 * i + 1]);
    atomicAdd(reinterpret_cast<float4*>(dst) + i, make_float4(a.x, a.y, b.x, b.y));
  }
}

// ---------------------------------------------------------------- RoPE bwd
// In place on the first `ncols_rot` columns of x [rows, ld] (heads of width hd):
// inverse rotate-half rotation (rotation by -angle).
__global__ void rope_bwd_kernel(__nv_bfloat16* __restrict__ x, int64_t ld, int64_t rows, int ncols_rot, int hd,
                                const float* __restrict__ cos, const float* __restrict__ sin, int seq) {
  const int half = hd / 2;
  const int pairs_per_row = ncols_rot / 2;
  const int64_t total = rows * pairs_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / pairs_per_row;
    const int p = (int)(i % pairs_per_row);
    const int head = p / half, j = p % half;
    const int pos = (int)(row % seq);
    __nv_bfloat16* base = x + row * ld + head * hd;
    const float c = cos[pos * half + j], s = sin[pos * half + j];
    const float d1 = __bfloat162float(base[j]), d2 = __bfloat162float(base[j + half]);
    base[j] = __float2bfloat16(d1 * c + d2 * s);
    base[j + half] = __float2bfloat16(d2 * c - d1 * s);
  }
}

// Same, 8 rotation pairs per thread with 16-byte loads and stores: one CTA per
// row (grid-stride), threads over (head, 8-pair group).  Needs half % 8 == 0 and
// 16-byte aligned rows.
// src may differ from x (out of place; then the columns past ncols_rot, up to
// ncols, are copied as they are).
__global__ void __launch_bounds__(256) rope_bwd_vec_kernel(const __nv_bfloat16* src, int64_t lds, __nv_bfloat16* x,
                                                           int64_t ld, int64_t rows, int ncols_rot, int ncols, int hd,
                                                           const float* __restrict__ cos,
                                                           const float* __restrict__ sin, int seq) {
  const int half = hd / 2;
  const int groups = half / 8;
  const int items = (ncols_rot / hd) * groups;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int pos = (int)(row % seq);
    const float* cr = cos + (int64_t)pos * half;
    const float* sr = sin + (int64_t)pos * half;
    for (int it = threadIdx.x; it < items; it += blockDim.x) {
      const int head = it / groups, j = (it % groups) * 8;
      __nv_bfloat16* base = x + row * ld + head * hd;
      const __nv_bfloat16* sbase = src + row * lds + head * hd;
      uint4 ua = *reinterpret_cast<const uint4*>(sbase + j);
      uint4 ub = *reinterpret_cast<const uint4*>(sbase + j + half);
      const float4 c0 = __ldg(reinterpret_cast<const float4*>(cr + j)), c1 = __ldg(reinterpret_cast<const float4*>(cr + j + 4));
      const float4 s0 = __ldg(reinterpret_cast<const float4*>(sr + j)), s1 = __ldg(reinterpret_cast<const float4*>(sr + j + 4));
      const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      __nv_bfloat162* ha = reinterpret_cast<__nv_bfloat162*>(&ua);
      __nv_bfloat162* hb = reinterpret_cast<__nv_bfloat162*>(&ub);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 a = __bfloat1622float2(ha[q]), b = __bfloat1622float2(hb[q]);
        const float c_0 = cc[2 * q], c_1 = cc[2 * q + 1], s_0 = ss[2 * q], s_1 = ss[2 * q + 1];
        ha[q] = __floats2bfloat162_rn(a.x * c_0 + b.x * s_0, a.y * c_1 + b.y * s_1);
        hb[q] = __floats2bfloat162_rn(b.x * c_0 - a.x * s_0, b.y * c_1 - a.y * s_1);
      }
      *reinterpret_cast<uint4*>(base + j) = ua;
      *reinterpret_cast<uint4*>(base + j + half) = ub;
    }
    if (src != x)
      for (int c = ncols_rot + threadIdx.x * 8; c < ncols; c += blockDim.x * 8)
        *reinterpret_cast<uint4*>(x + row * ld + c) = *reinterpret_cast<const uint4*>(src + row * lds + c);
  }
}

// --------------------------------------------------------- grad norm / clip
__global__ void sqsum_kernel(const float* __restrict__ g, int64_t n, float* __restrict__ out) {
  float s = 0.f;
  const int64_t nv = n / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(g)[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  if (blockIdx.x == 0)
    for (int64_t i = nv * 4 + threadIdx.x; i < n; i += blockDim.x) s += g[i] * g[i];
  s = warp_sum(s);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) atomicAdd(out, t);
  }
}

// coef = min(1, max_norm / (sqrt(sqsum) + 1e-6)) * pre_scale; also writes the norm.
// step_state (nullable) = [t, 1 - b1^t, 1 - b2^t] kept on the device so that a
// captured step (CUDA graph) advances the bias correction on every replay.
// skip (nullable): a non-zero word also skips the update (an expert-parallel layer
// that ran over its receive capacity this step) while the norm stays as measured.
__global__ void clip_coef_kernel(const float* __restrict__ sqsum, float max_norm, float pre_scale,
                                 float* __restrict__ coef, float* __restrict__ norm_out,
                                 float* __restrict__ step_state, float b1, float b2, const int* __restrict__ skip) {
  const float nrm = sqrtf(*sqsum) * pre_scale;
  *norm_out = nrm;
  float c = pre_scale;
  if (max_norm > 0.f && nrm > max_norm) c *= max_norm / (nrm + 1e-6f);
  // a non-finite gradient norm skips this update: the coefficient is NaN, which every
  // AdamW launch reading it takes as "leave p, m, v as they are"; the step count stays
  const bool finite = isfinite(nrm) && !(skip && *skip);
  *coef = finite ? c : __int_as_float(0x7fc00000);
  if (step_state && finite) {
    const float t = step_state[0] + 1.f;
    step_state[0] = t;
    step_state[1] = 1.f - powf(b1, t);
    step_state[2] = 1.f - powf(b2, t);
  }
}

// ----------------------------------------------------- column sums (bias grads)
// out[c] += sum_r x[r, c] for a bf16 [rows, N] matrix of row stride ld.  A block is
// 32 column lanes (8 consecutive columns each, one 16-byte load) x 8 row lanes;
// blockIdx.y splits the rows; one f32 atomic per column per block.
__global__ void __launch_bounds__(256) colsum_bf16_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int N,
                                                          int64_t ld, bool vec, float* __restrict__ out) {
  __shared__ float part[8][257];
  const int cl = threadIdx.x & 31, rl = threadIdx.x >> 5;
  const int c0 = (blockIdx.x * 32 + cl) * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (c0 < N) {
    const bool full = vec && c0 + 8 <= N;
    for (int64_t r = (int64_t)blockIdx.y * 8 + rl; r < rows; r += (int64_t)gridDim.y * 8) {
      const __nv_bfloat16* row = x + r * ld + c0;
      if (full) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(row));
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h2[i]);
          acc[2 * i] += f.x;
          acc[2 * i + 1] += f.y;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (c0 + j < N) acc[j] += __bfloat162float(row[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) part[rl][cl * 8 + j] = acc[j];
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    const int c = blockIdx.x * 256 + i;
    if (c < N) {
      float sum = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) sum += part[q][i];
      atomicAdd(out + c, sum);
    }
  }
}

// ------------------------------------------------------------------- AdamW
// Decoupled AdamW on flat f32 master weights, f32 moments; writes the bf16
// model copy.  g is scaled by *gscale (clip coefficient and 1/world).
__global__ void adamw_kernel(float* __restrict__ p, __nv_bfloat16* __restrict__ p16, const float* __restrict__ g,
                             float* __restrict__ m, float* __restrict__ v, int64_t n, float lr, float b1, float b2,
                             float eps, float wd, float bc1, float bc2, const float* __restrict__ gscale,
                             const float* __restrict__ bc_dev) {
  const float gs = gscale ? *gscale : 1.f;
  if (gs != gs) return;  // NaN coefficient: non-finite gradient norm, the step is skipped
  // bias corrections from the device step state when given (graph-capturable step)
  const float rb1 = 1.f / (bc_dev ? bc_dev[0] : bc1), rb2 = 1.f / (bc_dev ? bc_dev[1] : bc2);
  const int64_t nv = n / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    float4 pv = reinterpret_cast<float4*>(p)[i];
    const float4 gv = reinterpret_cast<const float4*>(g)[i];
    float4 mv = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pp = &pv.x;
    const float* gg = &gv.x;
    float* mm = &mv.x;
    float* vvv = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gk = gg[k] * gs;
      mm[k] = b1 * mm[k] + (1.f - b1) * gk;
      vvv[k] = b2 * vvv[k] + (1.f - b2) * gk * gk;
      const float upd = (mm[k] * rb1) / (sqrtf(vvv[k] * rb2) + eps);
      pp[k] = pp[k] - lr * upd - lr * wd * pp[k];
    }
    reinterpret_cast<float4*>(p)[i] = pv;
    reinterpret_cast<float4*>(m)[i] = mv;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (p16) {
      uint2 o;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
      h[0] = __floats2bfloat162_rn(pv.x, pv.y);
      h[1] = __floats2bfloat162_rn(pv.z, pv.w);
      reinterpret_cast<uint2*>(p16)[i] = o;
    }
  }
  if (blockIdx.x == 0) {
    for (int64_t i = nv * 4 + threadIdx.x; i < n; i += blockDim.x) {
      const float gk = g[i] * gs;
      m[i] = b1 * m[i] + (1.f - b1) * gk;
      v[i] = b2 * v[i] + (1.f - b2) * gk * gk;
      const float upd = (m[i] * rb1) / (sqrtf(v[i] * rb2) + eps);
      p[i] = p[i] - lr * upd - lr * wd * p[i];
      if (p16) p16[i] = __float2bfloat16(p[i]);
    }
  }
}

}  // namespace

void launch_ce_finish(const float* pmax, const float* psum, int nt, const float* tgt_logit, const int64_t* targets,
                      float* lse, float* loss, int64_t rows, cudaStream_t st) {
  if (!rows) return;
  ce_finish_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(pmax, psum, nt, tgt_logit, targets, lse, loss, rows);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_ce_bwd(void* logits, int64_t ld, int64_t V, int64_t rows, const float* lse, const int64_t* targets,
                   const float* gscale, float inv_count, cudaStream_t st, int64_t col0) {
  if (!rows) return;
  OXI_CHECK(ld % 8 == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0, "logits rows must be 16-byte aligned");
  OXI_CHECK(rows < 65536 * 32768LL, "too many rows");
  const int64_t nvec = V / 8;
  // CTAs per row: enough for one pass of CE_BWD_VEC vectors per thread, at most 16
  unsigned gx = (unsigned)std::max<int64_t>(1, std::min<int64_t>((nvec + 256 * CE_BWD_VEC - 1) / (256 * CE_BWD_VEC), 16));
  dim3 grid(gx, (unsigned)rows);
  ce_bwd_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(logits), ld, V, lse, targets, gscale,
                                      inv_count, col0);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_embed_fwd(const int64_t* ids, const void* w, void* out, int64_t rows, int H, cudaStream_t st) {
  if (!rows) return;
  OXI_CHECK(H % 8 == 0, "embedding width must be a multiple of 8");
  embed_fwd_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(ids, reinterpret_cast<const __nv_bfloat16*>(w),
                                                                 reinterpret_cast<__nv_bfloat16*>(out), rows, H);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_embed_bwd(const int64_t* ids, const void* dy, float* dw, int64_t rows, int H, cudaStream_t st) {
  if (!rows) return;
  OXI_CHECK(H % 8 == 0, "embedding width must be a multiple of 8");
  embed_bwd_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(ids, reinterpret_cast<const __nv_bfloat16*>(dy), dw,
                                                                 rows, H);
  OXI_CUDA_CHECK(cudaGetLastError());
}

bool rope_bwd_vec_ok(const void* p, int64_t ld, int ncols_rot, int hd) {
  return (hd / 2) % 8 == 0 && ncols_rot % hd == 0 && ld % 8 == 0 && (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

void launch_rope_bwd_to(const void* src, int64_t lds, void* dst, int64_t ldd, int64_t rows, int ncols_rot, int ncols,
                        int hd, const float* cos, const float* sin, int seq, cudaStream_t st) {
  OXI_CHECK(rope_bwd_vec_ok(src, lds, ncols_rot, hd) && rope_bwd_vec_ok(dst, ldd, ncols_rot, hd) && ncols % 8 == 0 &&
                (reinterpret_cast<uintptr_t>(cos) & 15) == 0 && (reinterpret_cast<uintptr_t>(sin) & 15) == 0,
            "rope_bwd_to: 16-byte aligned rows, half head a multiple of 8");
  if (!rows) return;
  const unsigned grid = (unsigned)std::min<int64_t>(rows, (int64_t)sm_count() * 8);
  rope_bwd_vec_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(src), lds,
                                            reinterpret_cast<__nv_bfloat16*>(dst), ldd, rows, ncols_rot, ncols, hd,
                                            cos, sin, seq);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_rope_bwd(void* x, int64_t ld, int64_t rows, int ncols_rot, int hd, const float* cos, const float* sin,
                     int seq, cudaStream_t st) {
  if (!rows || !ncols_rot) return;
  if (rope_bwd_vec_ok(x, ld, ncols_rot, hd) && (reinterpret_cast<uintptr_t>(cos) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(sin) & 15) == 0) {
    launch_rope_bwd_to(x, ld, x, ld, rows, ncols_rot, ncols_rot, hd, cos, sin, seq, st);
    return;
  }
  const int64_t total = rows * (ncols_rot / 2);
  const unsigned grid = (unsigned)std::min<int64_t>((total + 255) / 256, (int64_t)sm_count() * 16);
  rope_bwd_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(x), ld, rows, ncols_rot, hd, cos, sin, seq);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_sqsum(const float* g, int64_t n, float* out, cudaStream_t st) {
  if (!n) return;
  const unsigned grid = (unsigned)std::min<int64_t>((n / 4 + 255) / 256 + 1, (int64_t)sm_count() * 4);
  sqsum_kernel<<<grid, 256, 0, st>>>(g, n, out);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_colsum_bf16(const void* x, int64_t rows, int N, int64_t ld, float* out, cudaStream_t st) {
  if (rows <= 0 || N <= 0) return;
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && ld % 8 == 0;
  const int gx = (N + 255) / 256;
  const int64_t want = std::max<int64_t>(1, (int64_t)sm_count() * 8 / gx);
  const int gy = (int)std::min<int64_t>(want, std::max<int64_t>(1, rows / 64));
  colsum_bf16_kernel<<<dim3(gx, gy), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x), rows, N, ld, vec, out);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_clip_coef(const float* sqsum, float max_norm, float pre_scale, float* coef, float* norm_out,
                      cudaStream_t st, float* step_state, float b1, float b2, const int* skip) {
  clip_coef_kernel<<<1, 1, 0, st>>>(sqsum, max_norm, pre_scale, coef, norm_out, step_state, b1, b2, skip);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_adamw(float* p, void* p16, const float* g, float* m, float* v, int64_t n, float lr, float b1, float b2,
                  float eps, float wd, float bc1, float bc2, const float* gscale, cudaStream_t st,
                  const float* bc_dev) {
  if (!n) return;
  OXI_CHECK((reinterpret_cast<uintptr_t>(p) & 15) == 0 && (reinterpret_cast<uintptr_t>(g) & 15) == 0 &&
                (reinterpret_cast<uintptr_t>(m) & 15) == 0 && (reinterpret_cast<uintptr_t>(v) & 15) == 0 &&
                (reinterpret_cast<uintptr_t>(p16) & 7) == 0,
            "AdamW buffers must be 16-byte aligned");
  const unsigned grid = (unsigned)std::min<int64_t>((n / 4 + 255) / 256 + 1, (int64_t)sm_count() * 8);
  adamw_kernel<<<grid, 256, 0, st>>>(p, reinterpret_cast<__nv_bfloat16*>(p16), g, m, v, n, lr, b1, b2, eps, wd, bc1,
                                     bc2, gscale, bc_dev);
  OXI_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------ SwiGLU backward (element-wise)
// From dH [rows, I] (the down projection's input gradient) and the saved
// pre-activations GU [rows, 2I] (gate / up interleaved in blocks of 128 columns):
//   dG = dH * u * s * (1 + g (1 - s)),  dU = dH * g * s,  s = sigmoid(g)
// written to dGU in GU's layout.  8 columns (16 bytes) per thread.
namespace {
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh,
                                                         const __nv_bfloat16* __restrict__ gu,
                                                         __nv_bfloat16* __restrict__ dgu, int64_t rows, int I) {
  const int vpr = I / 8;  // 8-column vectors per row of dH
  const int64_t n = rows * vpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vpr;
    const int c = (int)(i - r * vpr) * 8;
    const int64_t gcol = (int64_t)(c / 128) * 256 + c % 128;
    const uint4 hv = *reinterpret_cast<const uint4*>(dh + r * I + c);
    const uint4 gv = *reinterpret_cast<const uint4*>(gu + r * 2 * I + gcol);
    const uint4 uv = *reinterpret_cast<const uint4*>(gu + r * 2 * I + gcol + 128);
    const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t dg[4], du[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 h = unpack_bf16(hw[k]), g = unpack_bf16(gw[k]), u = unpack_bf16(uw[k]);
      const float s0 = 1.f / (1.f + __expf(-g.x)), s1 = 1.f / (1.f + __expf(-g.y));
      dg[k] = pack_bf16(h.x * u.x * s0 * (1.f + g.x * (1.f - s0)), h.y * u.y * s1 * (1.f + g.y * (1.f - s1)));
      du[k] = pack_bf16(h.x * g.x * s0, h.y * g.y * s1);
    }
    *reinterpret_cast<uint4*>(dgu + r * 2 * I + gcol) = make_uint4(dg[0], dg[1], dg[2], dg[3]);
    *reinterpret_cast<uint4*>(dgu + r * 2 * I + gcol + 128) = make_uint4(du[0], du[1], du[2], du[3]);
  }
}
}  // namespace

void launch_swiglu_bwd(const void* dh, const void* gu, void* dgu, int64_t rows, int I, cudaStream_t st) {
  OXI_CHECK(I % 128 == 0, "SwiGLU backward: intermediate size must be a multiple of 128");
  OXI_CHECK(((reinterpret_cast<uintptr_t>(dh) | reinterpret_cast<uintptr_t>(gu) | reinterpret_cast<uintptr_t>(dgu)) &
             15) == 0, "SwiGLU backward: 16-byte aligned buffers");
  if (!rows) return;
  const int64_t n = rows * (I / 8);
  const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 16);
  swiglu_bwd_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(dh),
                                          reinterpret_cast<const __nv_bfloat16*>(gu),
                                          reinterpret_cast<__nv_bfloat16*>(dgu), rows, I);
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
